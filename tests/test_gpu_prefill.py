"""Causal prefill over packed keys on the tensor cores (bgtq_attend_prefill) against the
oracle on the GPU's own codes, at the north-star tolerance (1e-5 abs + 1e-4 rel).

Follows the model path's chunked prefill (src/model/decoder.ts:30-81): all query heads of
every KV head (SmolLM2 GQA 3, Qwen GQA 7), whole-prefix and mid-sequence chunks, ragged
sequence lengths, different calibrations per KV head; and config 5's own size (8192
positions, 128 key tiles, the Qwen calibration's tables) on both tensor-core kernels.
"""
import os

import numpy as np
import pytest

import oracle
from bgtq import FP16Keys, GroupedAttention, PackedKeys, Values, _lib, device_status, synthetic
from conftest import GOLDEN

pytestmark = pytest.mark.gpu
ATOL, RTOL = 1e-5, 1e-4


def _stores(rng, heads, S, lengths, cap):
    zh = np.load(GOLDEN / "smollm2_heads.npz")
    keys, vals, kv = [], [], []
    for h in range(heads):
        cfg, tab = zh[f"h{h % 6}_config"], zh[f"h{h % 6}_table"]
        k = PackedKeys((cfg, tab), cap, sequences=S)
        v = Values(64, cap, "f16", sequences=S)
        per = []
        for s, L in enumerate(lengths):
            kb = synthetic.profiled(rng, L, 64).astype(np.float16)
            vb = rng.standard_normal((L, 64)).astype(np.float16)
            k.append(kb.view(np.uint16), seq_first=s)
            v.append(vb.view(np.uint16), seq_first=s)
            per.append(vb.astype(np.float32))
        keys.append(k)
        vals.append(v)
        kv.append((cfg, tab, per))
    return keys, vals, kv


def _check(att, keys, kv, q, pos_first, heads, G):
    out = att.prefill(q, pos_first)
    S, n = q.shape[0], q.shape[1]
    for s in range(S):
        for h in range(heads):
            cfg, tab, per = kv[h]
            kh = oracle.reconstruct(cfg, tab, *keys[h].read(s), threads=8)
            rows = q[s, :, h * G:(h + 1) * G, :].reshape(n * G, 64)
            pos = np.repeat(np.arange(pos_first, pos_first + n, dtype=np.uint32), G)
            _, _, ref = oracle.attention(rows, kh, per[s], pos, True, threads=8)
            got = out[s, :, h * G:(h + 1) * G, :].reshape(n * G, 64)
            np.testing.assert_allclose(got, ref, atol=ATOL, rtol=RTOL)
    return out


@pytest.mark.parametrize("kernel", ["umma", "mma"])
@pytest.mark.parametrize("heads,G", [(3, 3), (2, 7), (1, 1), (2, 4)])
def test_prefill_matches_oracle(cuda, heads, G, kernel):
    rng = np.random.default_rng(100 + G)
    S, lengths = 2, [700, 1203]
    keys, vals, kv = _stores(rng, heads, S, lengths, 1280)
    att = GroupedAttention(keys, vals, min(G, 8))
    att.set_prefill_kernel(kernel)
    # whole prefix of the shorter sequence, then a chunk in the middle
    q = synthetic.profiled(rng, S * 700 * heads * G, 64).reshape(S, 700, heads * G, 64)
    _check(att, keys, kv, q, 0, heads, G)
    q2 = synthetic.profiled(rng, S * 97 * heads * G, 64).reshape(S, 97, heads * G, 64)
    _check(att, keys, kv, q2, 333, heads, G)
    assert device_status(0) == 0


@pytest.mark.parametrize("kernel", ["umma", "mma"])
def test_prefill_at_config5_size_matches_oracle(cuda, kernel):
    """One sequence and one layer of config 5 at its benchmarked length: 8192 positions
    (128 key tiles of accumulation) over 2 KV heads x 7 query heads with the Qwen
    calibration's tables (a one-group and a three-group head).  Sampled query rows - the
    first tiles, the middle, and the last 64 positions - against the oracle."""
    import torch
    zq = np.load(GOLDEN / "qwen_calibration.npz")
    from bgtq import build_tables
    picks = [0, int(np.argmax(zq["norm_stride"]))]
    rng = np.random.default_rng(55)
    T, H, G = 8192, 2, 7
    keys, vals, kv = [], [], []
    for h, j in enumerate(picks):
        cfg, tab = build_tables(zq["widths"][j].astype(np.int64), rotation_threshold=2,
                                norm_stride=int(zq["norm_stride"][j]))
        k = PackedKeys((cfg, tab), T)
        v = Values(64, T, "f16")
        kb = (rng.standard_normal((T, 64)) * 1.5).astype(np.float16)
        vb = (rng.standard_normal((T, 64)) * 1.5).astype(np.float16)
        k.append(kb.view(np.uint16))
        v.append(vb.view(np.uint16))
        keys.append(k)
        vals.append(v)
        kv.append((cfg, tab, vb.astype(np.float32)))
    att = GroupedAttention(keys, vals, G)
    att.set_prefill_kernel(kernel)
    q = (rng.standard_normal((1, T, H * G, 64)) * 1.5).astype(np.float32)
    out = att.prefill(torch.from_numpy(q).to(cuda)).cpu().numpy()
    sample = np.unique(np.concatenate([[0, 1, 63, 64, 65, 127, 128, 2047, 4095, 4096, 6000],
                                       np.arange(T - 64, T)])).astype(np.uint32)
    threads = os.cpu_count() or 8
    for h in range(H):
        cfg, tab, vf = kv[h]
        kh = oracle.reconstruct(cfg, tab, *keys[h].read(0), threads=threads)
        rows = q[0, sample][:, h * G:(h + 1) * G].reshape(-1, 64)
        pos = np.repeat(sample, G)
        _, _, ref = oracle.attention(rows, kh, vf, pos, True, threads=threads)
        got = out[0, sample][:, h * G:(h + 1) * G].reshape(-1, 64)
        np.testing.assert_allclose(got, ref, atol=ATOL, rtol=RTOL)
    assert device_status(0) == 0


def test_prefill_device_io_and_chunks_agree(cuda):
    """Device tensors give the host path's bytes; two chunks give the one-call result."""
    import torch
    rng = np.random.default_rng(5)
    S, heads, G, L = 3, 3, 3, 640
    keys, vals, kv = _stores(rng, heads, S, [L] * S, 640)
    att = GroupedAttention(keys, vals, G)
    q = synthetic.profiled(rng, S * L * heads * G, 64).reshape(S, L, heads * G, 64)
    host = att.prefill(q)
    dev = att.prefill(torch.from_numpy(q).to(cuda))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(dev.cpu().numpy(), host)
    a = att.prefill(np.ascontiguousarray(q[:, :200]), 0)
    b = att.prefill(np.ascontiguousarray(q[:, 200:]), 200)
    np.testing.assert_array_equal(np.concatenate([a, b], 1), host)


def test_prefill_rejections(cuda):
    rng = np.random.default_rng(6)
    keys, vals, kv = _stores(rng, 1, 1, [100], 128)
    att = GroupedAttention(keys, vals, 3)
    q = np.zeros((1, 101, 3, 64), np.float32)
    with pytest.raises(_lib.RangeError):
        att.prefill(q)                       # positions beyond the appended keys
    q = np.zeros((1, 10, 9, 64), np.float32)
    with pytest.raises(_lib.RangeError):
        att.prefill(q)                       # 9 query heads per KV head
    bad = np.zeros((1, 10, 3, 64), np.float32)
    bad[0, 3, 1, 5] = np.nan
    with pytest.raises(_lib.RangeError, match="inite"):
        att.prefill(bad)
    fk = FP16Keys(64, 128)
    fk.append(np.zeros((100, 64), np.float16).view(np.uint16))
    att2 = GroupedAttention([fk], vals, 3)
    with pytest.raises(_lib.RangeError):
        att2.prefill(np.zeros((1, 10, 3, 64), np.float32))
