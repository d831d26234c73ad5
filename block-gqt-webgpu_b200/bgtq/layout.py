"""Calibration tables: the reference's BlockGTQParameters and its flattened form.

Mirrors src/webgpu/layout.ts:2-31.  ``tables(p)`` produces the exact interchange format
the C ABI consumes (and that the reference's WGSL shaders and the SmolLM2 calibration
fixture use):

    config u32: [dim, groups, rowBytes, normStride, nibbleDims, maxCentroids,
                 off_perm, off_groupOf, off_posToCb, off_codeLut,
                 permutation..., groupOf..., positionToCodebook..., codeLut...]
    table  f32: [rotation (dim*dim), centroids (dim*maxCentroids), offsets (dim),
                 inverseScales (dim)]

Validation (``validate_layout``) runs in the native library on host memory, so the same
checks guard both this Python surface and direct C callers.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib


@dataclass
class BlockGTQParameters:
    dim: int
    groups: int
    row_bytes: int
    norm_stride: int
    nibble_dims: int
    max_centroids: int
    permutation: np.ndarray          # u32 [dim] head permutation (pairs sorted by width)
    group_of: np.ndarray             # u32 [dim] group of each permuted dimension
    position_to_codebook: np.ndarray  # u32 [dim]
    code_lut: np.ndarray             # u8 [codebooks*256]
    rotation: np.ndarray             # f32 [dim*dim] block-diagonal, row j = output j
    centroids: np.ndarray            # f32 [dim*max_centroids]
    offsets: np.ndarray              # f32 [dim]
    inverse_scales: np.ndarray       # f32 [dim]

    @classmethod
    def from_arrays(cls, z) -> "BlockGTQParameters":
        """Build from a mapping with the field names above (e.g. a golden .npz)."""
        return cls(dim=int(z["dim"]), groups=int(z["groups"]), row_bytes=int(z["row_bytes"]),
                   norm_stride=int(z["norm_stride"]), nibble_dims=int(z["nibble_dims"]),
                   max_centroids=int(z["max_centroids"]),
                   permutation=np.asarray(z["permutation"], np.uint32), group_of=np.asarray(z["group_of"], np.uint32),
                   position_to_codebook=np.asarray(z["position_to_codebook"], np.uint32),
                   code_lut=np.asarray(z["code_lut"], np.uint8).reshape(-1),
                   rotation=np.asarray(z["rotation"], np.float32).reshape(-1),
                   centroids=np.asarray(z["centroids"], np.float32).reshape(-1),
                   offsets=np.asarray(z["offsets"], np.float32), inverse_scales=np.asarray(z["inverse_scales"], np.float32))

    @classmethod
    def from_tables(cls, config, table) -> "BlockGTQParameters":
        """Inverse of ``tables()``: parse the flattened interchange format."""
        c = np.asarray(config, np.uint32)
        t = np.asarray(table, np.float32)
        d, maxc = int(c[0]), int(c[5])
        return cls(dim=d, groups=int(c[1]), row_bytes=int(c[2]), norm_stride=int(c[3]), nibble_dims=int(c[4]),
                   max_centroids=maxc, permutation=c[c[6]:c[6] + d].copy(), group_of=c[c[7]:c[7] + d].copy(),
                   position_to_codebook=c[c[8]:c[8] + d].copy(), code_lut=c[c[9]:].astype(np.uint8),
                   rotation=t[:d * d].copy(), centroids=t[d * d:d * d + d * maxc].copy(),
                   offsets=t[d * d + d * maxc:d * d + d * maxc + d].copy(), inverse_scales=t[d * d + d * maxc + d:].copy())


def tables(p: BlockGTQParameters) -> tuple[np.ndarray, np.ndarray]:
    """Flatten to (config u32, table f32) exactly as layout.ts:24-31 does."""
    config = [p.dim, p.groups, p.row_bytes, p.norm_stride, p.nibble_dims, p.max_centroids, 0, 0, 0, 0]
    for slot, values in ((6, p.permutation), (7, p.group_of), (8, p.position_to_codebook), (9, p.code_lut)):
        config[slot] = len(config)
        config.extend(int(v) for v in np.asarray(values).reshape(-1))
    floating = np.concatenate([np.asarray(a, np.float32).reshape(-1)
                               for a in (p.rotation, p.centroids, p.offsets, p.inverse_scales)])
    return np.asarray(config, dtype=np.uint32), floating.astype(np.float32)


def validate_layout(config: np.ndarray, table: np.ndarray) -> tuple[_lib.LayoutInfo, np.ndarray]:
    """validateLayout + the PackedKeys group check; returns (info, ranges[2*dim]).

    Raises LayoutError with the reference's messages ("Invalid Block-GTQ layout",
    "Invalid calibration table shape", "Code LUT incompatible with packing",
    "Non-contiguous transform group", "Off-group transform is nonzero", ...).
    """
    config = np.ascontiguousarray(config, dtype=np.uint32)
    table = np.ascontiguousarray(table, dtype=np.float32)
    dim = int(config[0]) if len(config) else 0
    ranges = np.zeros(max(2 * dim, 2), dtype=np.uint32)
    info = _lib.LayoutInfo()
    _lib.call("bgtq_layout_validate", config.ctypes.data, config.size, table.ctypes.data, table.size,
              ranges.ctypes.data, C.byref(info))
    return info, ranges[:2 * dim]


def build_tables(widths, rotation_threshold: int = 3, row_pad: int = 0, norm_stride: int = 0,
                 pair_order=None) -> tuple[np.ndarray, np.ndarray]:
    """Flattened (config u32, table f32) of one head from per-pair widths, built natively
    the way the reference's calibration builds them (block_gtq_pipeline.py:151-246,
    quant_kernels.py:276-364, quantizer.py:34-106; see bgtq_tables_build).  pair_order: an
    optional width-ascending permutation of the pairs to use instead of the argsort order."""
    w = np.ascontiguousarray(widths, dtype=np.int64)
    dim = 2 * len(w)
    po = None if pair_order is None else np.ascontiguousarray(pair_order, dtype=np.int64)
    pp = None if po is None else po.ctypes.data
    nc, nt = C.c_size_t(0), C.c_size_t(0)
    _lib.call("bgtq_tables_build", dim, w.ctypes.data, pp, rotation_threshold, row_pad, norm_stride, None, 0,
              C.byref(nc), None, 0, C.byref(nt))
    config = np.zeros(nc.value, np.uint32)
    table = np.zeros(nt.value, np.float32)
    _lib.call("bgtq_tables_build", dim, w.ctypes.data, pp, rotation_threshold, row_pad, norm_stride,
              config.ctypes.data, config.size, C.byref(nc), table.ctypes.data, table.size, C.byref(nt))
    return config, table


def haar_rotation(n: int, seed: int) -> np.ndarray:
    """NumPy default_rng(seed) Haar rotation of size n in FP32 (block_gtq_pipeline.py:81-92)."""
    out = np.zeros((n, n), np.float32)
    _lib.call("bgtq_haar_rotation", n, seed, out.ctypes.data)
    return out


def optimal_centroids(bits: int, n: int) -> np.ndarray:
    """Lloyd-Max centroids for N(0, 1/n) in FP32 (block_gtq_pipeline.py:24-78)."""
    out = np.zeros(1 << bits, np.float32)
    _lib.call("bgtq_optimal_centroids", bits, n, out.ctypes.data)
    return out


def allocate_bits(scores, budget: int, min_bits: int = 1, max_bits: int = 8) -> np.ndarray:
    """Greedy per-pair widths (src/reference/allocator.py:4-17), computed natively."""
    s = np.ascontiguousarray(scores, dtype=np.float32)
    out = np.zeros(len(s), dtype=np.int64)
    _lib.call("bgtq_allocate_bits", s.ctypes.data, len(s), int(budget), int(min_bits), int(max_bits), out.ctypes.data)
    return out
