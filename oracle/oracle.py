"""CPU oracle for the Block-GTQ hot path - TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm may use
this module, and only as the checker or the timed CPU baseline; the product
(libbgtq.so and the bgtq package) never imports it.

Contents
  * ctypes wrapper of bgtq_oracle.c (the C restatement of encode / reconstruct /
    attention, see that file's header for the reference lines it follows and the
    canonical FP32 operation order it shares with the CUDA encoder);
  * NumPy restatements of the integer parts:
      allocate_bits  src/reference/allocator.py:4-17
      pack / unpack  src/reference/mixed_layout.py:21-37
      grouping_ok    the PackedKeys group-range rule, src/runtime/packed-keys.ts:15-23

Pinning: tests/test_oracle.py checks this oracle against every golden vector the
reference commits for this path (fixtures/mixed/*, fixtures/attention/*,
fixtures/allocator.json, re-saved under tests/golden/ by tests/golden/make_golden.py)
and against reference encoder outputs on the config-1 / config-4 synthetic workloads.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "libbgtq_oracle.so"


def build(force: bool = False) -> Path:
    """Compile bgtq_oracle.c with gcc (see oracle/Makefile for the same recipe)."""
    src = HERE / "bgtq_oracle.c"
    if LIB.exists() and not force and LIB.stat().st_mtime >= src.stat().st_mtime:
        return LIB
    LIB.parent.mkdir(parents=True, exist_ok=True)
    cmd = ["gcc", "-O2", "-mavx2", "-mfma", "-ffp-contract=off", "-fopenmp", "-fPIC", "-shared",
           str(src), "-o", str(LIB), "-lm"]
    subprocess.run(cmd, check=True)
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        h = C.CDLL(str(LIB))
        P, L, I = C.c_void_p, C.c_long, C.c_int
        h.orc_half_bits.restype = C.c_uint16
        h.orc_half_bits.argtypes = [C.c_float]
        h.orc_half_value.restype = C.c_float
        h.orc_half_value.argtypes = [C.c_uint16]
        h.orc_encode_f16.restype = None
        h.orc_encode_f16.argtypes = [P, P, P, L, L, P, L, P, L, P, P, P, I]
        h.orc_encode_f32.restype = None
        h.orc_encode_f32.argtypes = [P, P, P, L, L, L, P, L, P, L, I]
        h.orc_reconstruct.restype = None
        h.orc_reconstruct.argtypes = [P, P, P, L, P, L, L, P, I]
        h.orc_attention.restype = None
        h.orc_attention.argtypes = [P, L, P, L, P, L, L, I, P, I, P, P, P, I]
        _lib = h
    return _lib


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def half_bits(x) -> np.ndarray:
    x = np.asarray(x, np.float32).reshape(-1)
    return np.array([lib().orc_half_bits(float(v)) for v in x], dtype=np.uint16)


def encode(config, table, k_bits, threads: int = 1, row_stride: int | None = None, scale_stride: int | None = None):
    """Encode FP16 keys [n, d] (uint16 bits).  Returns dict(packed, scales, codes, rotated, corrected)."""
    config, table = _c(config, np.uint32), _c(table, np.float32)
    d, ng = int(config[0]), int(config[1])
    rs = int(config[2]) if row_stride is None else row_stride
    ss = int(config[3]) if scale_stride is None else scale_stride
    k = _c(k_bits, np.uint16).reshape(-1, d)
    n = k.shape[0]
    packed = np.zeros((n, rs), np.uint8)
    scales = np.zeros((n, ss), np.uint16)
    codes = np.zeros((n, d), np.uint8)
    y = np.zeros((n, d), np.float32)
    corr = np.zeros((n, ng), np.float32)
    lib().orc_encode_f16(config.ctypes.data, table.ctypes.data, k.ctypes.data, n, d, packed.ctypes.data, rs,
                         scales.ctypes.data, ss, codes.ctypes.data, y.ctypes.data, corr.ctypes.data, threads)
    return dict(packed=packed, scales=scales, codes=codes, rotated=y, corrected=corr)


def encode_f32(config, table, act, row_elems: int, head_offset: int, n: int, threads: int = 1):
    """Model-path encode from FP32 activations (rounded to FP16 first)."""
    config, table = _c(config, np.uint32), _c(table, np.float32)
    a = _c(act, np.float32)
    rs, ss = int(config[2]), int(config[3])
    packed = np.zeros((n, rs), np.uint8)
    scales = np.zeros((n, ss), np.uint16)
    lib().orc_encode_f32(config.ctypes.data, table.ctypes.data, a.ctypes.data, n, row_elems, head_offset,
                         packed.ctypes.data, rs, scales.ctypes.data, ss, threads)
    return packed, scales


def reconstruct(config, table, packed, scales, threads: int = 1) -> np.ndarray:
    config, table = _c(config, np.uint32), _c(table, np.float32)
    packed, scales = _c(packed, np.uint8), _c(scales, np.uint16)
    n, d = packed.shape[0], int(config[0])
    out = np.zeros((n, d), np.float32)
    lib().orc_reconstruct(config.ctypes.data, table.ctypes.data, packed.ctypes.data, packed.shape[1],
                          scales.ctypes.data, scales.shape[1], n, out.ctypes.data, threads)
    return out


def attention(q, k, v, positions=None, causal: bool = False, threads: int = 1):
    """(logits, probabilities, output) in double precision, rounded to float32."""
    q, k, v = _c(q, np.float32), _c(k, np.float32), _c(v, np.float32)
    nq, d = q.shape
    T = k.shape[0]
    pos = _c(np.full(nq, T - 1) if positions is None else positions, np.uint32)
    logits = np.zeros((nq, T), np.float32)
    probs = np.zeros((nq, T), np.float32)
    out = np.zeros((nq, d), np.float32)
    lib().orc_attention(q.ctypes.data, nq, k.ctypes.data, k.shape[1], v.ctypes.data, v.shape[1], T, d,
                        pos.ctypes.data, int(bool(causal)), logits.ctypes.data, probs.ctypes.data, out.ctypes.data,
                        threads)
    return logits, probs, out


def allocate_bits(scores, budget: int, min_bits: int = 1, max_bits: int = 8) -> np.ndarray:
    """Greedy widths minimising sum s_i 4^-b_i (src/reference/allocator.py:4-17)."""
    scores = np.asarray(scores, dtype=np.float32)
    widths = np.full(len(scores), min_bits, dtype=np.int64)
    remaining = budget - int(widths.sum())
    while remaining > 0:
        priorities = scores * np.power(4.0, -widths.astype(np.float64))
        priorities[widths >= max_bits] = -1.0
        index = int(np.argmax(priorities))
        if priorities[index] <= 0:
            break
        widths[index] += 1
        remaining -= 1
    return widths


def pack(codes, nopack_start: int, row_bytes: int) -> np.ndarray:
    """Nibble region (dims < ns, even dim in the low nibble) then raw bytes (mixed_layout.py:21-27)."""
    c = np.asarray(codes, dtype=np.uint8)
    out = np.zeros((*c.shape[:-1], row_bytes), dtype=np.uint8)
    ns = nopack_start
    out[..., :ns // 2] = (c[..., :ns:2] & 15) | ((c[..., 1:ns:2] & 15) << 4)
    out[..., ns // 2:ns // 2 + c.shape[-1] - ns] = c[..., ns:]
    return out


def unpack(data, dim: int, nopack_start: int) -> np.ndarray:
    """Inverse of pack (mixed_layout.py:30-37)."""
    p = np.asarray(data, dtype=np.uint8)
    c = np.zeros((*p.shape[:-1], dim), dtype=np.uint8)
    ns = nopack_start
    c[..., :ns:2] = p[..., :ns // 2] & 15
    c[..., 1:ns:2] = p[..., :ns // 2] >> 4
    c[..., ns:] = p[..., ns // 2:ns // 2 + dim - ns]
    return c


def group_ranges(group_of, rotation, d: int) -> np.ndarray:
    """[start, end) of each dimension's group; raises on the cases PackedKeys rejects."""
    g = np.asarray(group_of)
    rot = np.asarray(rotation, np.float32).reshape(d, d)
    ranges = np.zeros(2 * d, np.uint32)
    for j in range(d):
        members = np.nonzero(g == g[j])[0]
        start, end = int(members[0]), int(members[-1]) + 1
        if end - start != len(members):
            raise ValueError("Non-contiguous transform group")
        outside = np.r_[0:start, end:d]
        if np.any(rot[outside, j] != 0):
            raise ValueError("Off-group transform is nonzero")
        ranges[2 * j], ranges[2 * j + 1] = start, end
    return ranges


def code_edge_distance(config, table, k_bits, mismatches) -> np.ndarray:
    """For each (row, dim) in `mismatches`, |t - round(t)| in bin units of the quantiser
    input t = (y - off) * inv computed in float64: the distance of y from the LUT bin
    edge the two encoders disagree about.  Codes may legitimately differ only where
    this is within a few float32 ulps of the edge."""
    config, table = _c(config, np.uint32), _c(table, np.float32)
    d, maxc = int(config[0]), int(config[5])
    perm = config[config[6]:config[6] + d]
    grp = config[config[7]:config[7] + d]
    rot = table[:d * d].reshape(d, d).astype(np.float64)
    off = table[d * d + d * maxc:d * d + d * maxc + d].astype(np.float64)
    inv = table[d * d + d * maxc + d:].astype(np.float64)
    k = np.asarray(k_bits, np.uint16).view(np.float16).astype(np.float64)
    out = []
    for r, j in mismatches:
        x = k[r][perm]
        n = np.array([np.sqrt((x[grp == g] ** 2).sum() + 1e-30) for g in range(int(config[1]))])
        xn = x / np.where(n[grp] > 1e-10, n[grp], 1.0)
        y = float(rot[j] @ xn)
        t = (y - off[j]) * inv[j]
        out.append(abs(t - round(t)))
    return np.asarray(out)
