"""K encode on the GPU through the C ABI versus the CPU oracle (bit-exact) and the
reference's golden vectors.

Contracts follow the reference's GPU codec tests: codes and packed bytes exact, FP16
scales within one half-ulp of the reference encoder (tests/webgpu/phase2/phase2-test.ts:
53-59), appends split at an odd row boundary (tests/webgpu/attention-test.ts:33-39),
rejections leave state unchanged (tests/webgpu/runtime-contracts.ts:24-25), and the
model-path encoder fed from FP32 RoPE output equals the FP16 path
(tests/webgpu/model-codec-test.ts:7-26).
"""
import numpy as np
import pytest

import oracle
from bgtq import PackedKeys, _lib, device_status, synthetic
from conftest import GOLDEN, load_config, load_mixed, mixed_cases, params_tables

pytestmark = pytest.mark.gpu


def encode_gpu(cfg, tab, k_bits, capacity=None, chunks=None):
    n = k_bits.shape[0]
    keys = PackedKeys((cfg, tab), capacity or n)
    if chunks:
        start = 0
        for c in chunks:
            keys.append(k_bits[start:start + c])
            start += c
    else:
        keys.append(k_bits)
    packed, norms = keys.read()
    return keys, packed, norms


@pytest.mark.parametrize("name", mixed_cases())
def test_reference_fixtures_bit_exact(cuda, name):
    z = load_mixed(name)
    p, cfg, tab = params_tables(z)
    kb = z["original"].astype(np.float16).view(np.uint16)
    keys, packed, norms = encode_gpu(cfg, tab, kb, capacity=int(z["capacity"]), chunks=[3, 2])
    np.testing.assert_array_equal(packed, z["packed"])
    np.testing.assert_array_equal(oracle.unpack(packed, p.dim, p.nibble_dims), z["codes"])
    np.testing.assert_array_equal(norms, z["norm_bits"])
    # reserved capacity stays zero (test_mixed.py:81-90 / phase2 cache_packed)
    full, fnorms = keys.read(0, 0, int(z["capacity"]))
    np.testing.assert_array_equal(full, z["cache_packed"])
    np.testing.assert_array_equal(fnorms, z["cache_norm_bits"])
    assert device_status(0) == 0


@pytest.mark.parametrize("name,seed", [("config1", 0), ("config4", 4)])
def test_config_workloads_bit_exact_vs_oracle_and_reference(cuda, name, seed):
    z = load_config(name)
    p, cfg, tab = params_tables(z)
    k, q, v = synthetic.decode_workload(seed, int(z["tokens"]), p.dim)
    kb = k.view(np.uint16)
    _, packed, norms = encode_gpu(cfg, tab, kb)
    ref = oracle.encode(cfg, tab, kb, threads=4)
    np.testing.assert_array_equal(packed, ref["packed"])
    np.testing.assert_array_equal(norms, ref["scales"])
    n = int(z["sample"])
    np.testing.assert_array_equal(oracle.unpack(packed[:n], p.dim, p.nibble_dims), z["codes"])
    assert np.abs(norms[:n, :p.groups].astype(int) - z["norm_bits"][:, :p.groups].astype(int)).max() <= 1


def _edge_keys(rng, n, d):
    k = (rng.standard_normal((n, d)) * np.exp(rng.uniform(-6, 6, (n, 1)))).astype(np.float32)
    k[0] = 0.0                       # all-zero key: norm below 1e-10, scale rounds to 0
    k[1] = 65504.0                   # largest finite FP16
    k[2, ::3] = -1e-7                # subnormal FP16 inputs
    k[3] = np.where(np.arange(d) % 2, 1.0, -1.0)
    return np.clip(k, -65504, 65504).astype(np.float16).view(np.uint16)


def test_calibrated_heads_random_and_edge_keys(cuda):
    z = np.load(GOLDEN / "smollm2_heads.npz")
    rng = np.random.default_rng(7)
    for i in range(int(z["heads"])):
        cfg, tab = z[f"h{i}_config"], z[f"h{i}_table"]
        kb = _edge_keys(rng, 777, 64)
        _, packed, norms = encode_gpu(cfg, tab, kb, chunks=[1, 128, 300, 348])
        ref = oracle.encode(cfg, tab, kb)
        np.testing.assert_array_equal(packed, ref["packed"])
        np.testing.assert_array_equal(norms, ref["scales"])


def test_append_validation_leaves_state_unchanged(cuda):
    z = load_mixed("mixed_d64")
    p, cfg, tab = params_tables(z)
    kb = z["original"].astype(np.float16).view(np.uint16)
    keys = PackedKeys((cfg, tab), 6)
    keys.append(kb[:5])
    before = keys.read(0, 0, 6)
    with pytest.raises(_lib.RangeError, match="capacity"):
        keys.append(kb[:2])
    bad = kb[:1].copy()
    bad[0, 5] = 0x7c00  # +inf
    with pytest.raises(_lib.RangeError, match="Finite"):
        keys.append(bad)
    with pytest.raises(_lib.RangeError):
        keys.append(np.zeros(p.dim + 1, np.uint16))
    with pytest.raises(_lib.RangeError):
        keys.append(np.zeros(0, np.uint16))
    assert keys.length == 5
    after = keys.read(0, 0, 6)
    np.testing.assert_array_equal(before[0], after[0])
    np.testing.assert_array_equal(before[1], after[1])
    keys.append(kb[:1])
    assert keys.length == 6


def test_device_fp16_and_fp32_model_path_sources(cuda):
    import torch
    z = load_config("config4")
    p, cfg, tab = params_tables(z)
    rng = np.random.default_rng(11)
    rows, kvh = 333, 3
    act = synthetic.profiled(rng, rows * kvh, 64).reshape(rows, kvh, 64)
    dev = torch.from_numpy(act).to(cuda)
    for head in range(kvh):
        keys = PackedKeys((cfg, tab), rows + 7)
        keys.append(dev[:, head, :])            # FP32 strided source (codec.wgsl:14)
        packed, norms = keys.read()
        rp, rs = oracle.encode_f32(cfg, tab, act.reshape(-1), kvh * 64, head * 64, rows)
        np.testing.assert_array_equal(packed, rp)
        np.testing.assert_array_equal(norms, rs)
        # FP16 device source gives the same bytes as the FP16 host source
        k16 = torch.from_numpy(act[:, head, :].astype(np.float16)).to(cuda)
        keys2 = PackedKeys((cfg, tab), rows)
        keys2.append(k16)
        np.testing.assert_array_equal(keys2.read()[0], packed)


def test_bulk_fp32_strided_and_ragged_multi_sequence(cuda):
    """The tiled bulk encoder (launches of more than 4096 keys) on the sources the prefill
    path gives it - FP32 rows of a strided activation (rounded to FP16 first) - and on
    several sequences whose appends start at different rows; bytes equal the oracle's."""
    import torch
    z = load_config("config4")
    p, cfg, tab = params_tables(z)
    rng = np.random.default_rng(23)
    rows, kvh = 5000, 2
    act = (synthetic.profiled(rng, rows * kvh, 64) * 3).reshape(rows, kvh, 64)
    dev = torch.from_numpy(act).to(cuda)
    for head in range(kvh):
        keys = PackedKeys((cfg, tab), rows)
        keys.append(dev[:, head, :])                       # one 5000-key FP32 strided launch
        packed, norms = keys.read()
        rp, rs = oracle.encode_f32(cfg, tab, act.reshape(-1), kvh * 64, head * 64, rows)
        np.testing.assert_array_equal(packed, rp)
        np.testing.assert_array_equal(norms, rs)
    S = 3
    keys = PackedKeys((cfg, tab), 3000, sequences=S)
    lead = _edge_keys(rng, 7, 64)
    keys.append(lead, seq_first=1)                         # sequence 1 starts 7 rows further on
    batch = _edge_keys(rng, S * 2000, 64).reshape(S, 2000, 64)
    keys.append(torch.from_numpy(batch.view(np.float16)).to(cuda), seq_first=0)   # 6000 keys, one launch
    for s in range(S):
        rows_s = batch[s] if s != 1 else np.concatenate([lead, batch[1]])
        ref = oracle.encode(cfg, tab, rows_s, threads=4)
        packed, norms = keys.read(s)
        np.testing.assert_array_equal(packed, ref["packed"])
        np.testing.assert_array_equal(norms, ref["scales"])
    assert device_status(0) == 0


def test_multi_sequence_ragged_appends(cuda):
    z = load_config("config4")
    p, cfg, tab = params_tables(z)
    rng = np.random.default_rng(5)
    S = 4
    keys = PackedKeys((cfg, tab), 64, sequences=S)
    first = _edge_keys(rng, 5, 64)
    keys.append(first, seq_first=1)                       # only sequence 1
    batch = _edge_keys(rng, S * 3, 64).reshape(S, 3, 64)  # then 3 rows to every sequence
    keys.append(batch, seq_first=0)
    assert [keys.lengths(s) for s in range(S)] == [3, 8, 3, 3]
    for s in range(S):
        rows = batch[s] if s != 1 else np.concatenate([first, batch[1]])
        ref = oracle.encode(cfg, tab, rows)
        packed, norms = keys.read(s)
        np.testing.assert_array_equal(packed, ref["packed"])
        np.testing.assert_array_equal(norms, ref["scales"])


def test_large_batch_sampled_bit_exact_and_deterministic(cuda):
    """Two million keys encoded on the GPU; random rows checked against the oracle,
    and a second encode of the same input gives identical bytes."""
    import torch
    z = load_config("config4")
    p, cfg, tab = params_tables(z)
    n = 1 << 21
    g = torch.Generator(device=cuda).manual_seed(3)
    sig = torch.from_numpy(synthetic.pair_sigma(32).astype(np.float32)).to(cuda)
    blocks = torch.randn((n, 32, 2), device=cuda, generator=g) * sig[None, :, None]
    k = torch.cat([blocks[..., 0], blocks[..., 1]], dim=-1).half()
    a = PackedKeys((cfg, tab), n)
    b = PackedKeys((cfg, tab), n)
    a.append(k)
    b.append(k)
    pa, na = a.read()
    pb, nb = b.read()
    np.testing.assert_array_equal(pa, pb)
    np.testing.assert_array_equal(na, nb)
    rows = np.sort(np.random.default_rng(0).choice(n, 4096, replace=False))
    kh = k[torch.from_numpy(rows).to(cuda)].cpu().numpy().view(np.uint16)
    ref = oracle.encode(cfg, tab, kh, threads=4)
    np.testing.assert_array_equal(pa[rows], ref["packed"])
    np.testing.assert_array_equal(na[rows], ref["scales"])


@pytest.mark.parametrize("name", mixed_cases() + ["config4"])
def test_warp_and_bulk_encoders_agree(cuda, name):
    """Appends of up to 4096 keys per head run one warp per key, larger ones one thread
    per key; both give the oracle's bytes for every table shape (head dims 16 to 128,
    nibble-only, byte-only and mixed rows)."""
    z = load_config(name) if name.startswith("config") else load_mixed(name)
    p, cfg, tab = params_tables(z)
    kb = _edge_keys(np.random.default_rng(17), 5000, p.dim)
    _, bulk_p, bulk_n = encode_gpu(cfg, tab, kb)                              # one 5000-key launch
    _, warp_p, warp_n = encode_gpu(cfg, tab, kb, chunks=[1, 999, 4000])      # three small launches
    ref = oracle.encode(cfg, tab, kb, threads=4)
    np.testing.assert_array_equal(bulk_p, ref["packed"])
    np.testing.assert_array_equal(bulk_n, ref["scales"])
    np.testing.assert_array_equal(warp_p, ref["packed"])
    np.testing.assert_array_equal(warp_n, ref["scales"])
    assert device_status(0) == 0


def test_reset_starts_every_sequence_over(cuda):
    """bgtq_keys_reset / bgtq_values_reset: lengths back to 0, the next appends write from
    row 0 and attention sees only them."""
    from bgtq import GroupedAttention, Values
    z = load_config("config4")
    p, cfg, tab = params_tables(z)
    rng = np.random.default_rng(21)
    a, b = _edge_keys(rng, 300, 64), _edge_keys(rng, 120, 64)
    keys, vals = PackedKeys((cfg, tab), 320, sequences=2), Values(64, 320, "f16", sequences=2)
    keys.append(np.stack([a, a])), vals.append(np.zeros((2, 300, 64), np.float16).view(np.uint16))
    keys.reset(), vals.reset()
    assert keys.lengths(0) == keys.lengths(1) == vals.lengths(1) == 0
    vb = rng.standard_normal((2, 120, 64)).astype(np.float16)
    keys.append(np.stack([b, b])), vals.append(vb.view(np.uint16))
    fresh = PackedKeys((cfg, tab), 320, sequences=2)
    fresh.append(np.stack([b, b]))
    for s in range(2):
        np.testing.assert_array_equal(keys.read(s)[0], fresh.read(s)[0])
        np.testing.assert_array_equal(keys.read(s)[1], fresh.read(s)[1])
    q = rng.standard_normal((2, 1, 3, 64)).astype(np.float32)
    att = GroupedAttention([keys], [vals], 3)
    kh = oracle.reconstruct(cfg, tab, *keys.read(0))
    _, _, ref = oracle.attention(q[0, 0], kh, vb[0].astype(np.float32))
    np.testing.assert_allclose(att.attend(q)[0, 0], ref, atol=1e-5, rtol=1e-4)


@pytest.mark.parametrize("dtype", ["float16", "float32"])
def test_append_kv_equals_per_head_appends(cuda, dtype):
    """bgtq_append_kv (every KV head's K encode + V append in one launch) writes the bytes
    of per-head PackedKeys.append / Values.append, and attention over the stores agrees
    exactly, across appends of 4, 1, 1 and 3 tokens on 5 sequences (one of them offset)."""
    import torch
    from bgtq import GroupedAttention, Values, append_kv
    zh = np.load(GOLDEN / "smollm2_heads.npz")
    H, B, d = 3, 5, 64
    tabs = [(zh[f"h{h}_config"], zh[f"h{h}_table"]) for h in range(H)]
    fk = [PackedKeys(t, 64, sequences=B + 1) for t in tabs]
    fv = [Values(d, 64, "f16", sequences=B + 1) for _ in range(H)]
    rk = [PackedKeys(t, 64, sequences=B + 1) for t in tabs]
    rv = [Values(d, 64, "f16", sequences=B + 1) for _ in range(H)]
    gen = torch.Generator(device=cuda).manual_seed(5)
    dt = getattr(torch, dtype)
    for n in (4, 1, 1, 3):
        k = (torch.randn((B, n, H, d), device=cuda, generator=gen) * 2).to(dt)
        v = torch.randn((B, n, H, d), device=cuda, generator=gen).to(dt)
        append_kv(fk, fv, k, v, seq_first=1)
        for h in range(H):
            rk[h].append(k[:, :, h, :].contiguous(), seq_first=1)
            rv[h].append(v[:, :, h, :].contiguous(), seq_first=1)
    torch.cuda.synchronize()
    for h in range(H):
        assert fk[h].lengths(0) == 0 and fv[h].lengths(0) == 0
        for s in range(1, B + 1):
            assert fk[h].lengths(s) == rk[h].lengths(s) == 9 == fv[h].lengths(s)
            np.testing.assert_array_equal(fk[h].read(s)[0], rk[h].read(s)[0])
            np.testing.assert_array_equal(fk[h].read(s)[1], rk[h].read(s)[1])
    q = torch.randn((B, H, 3, d), device=cuda, generator=gen)
    o1 = GroupedAttention(fk, fv, 3).attend(q, seq_first=1)
    o2 = GroupedAttention(rk, rv, 3).attend(q, seq_first=1)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(o1.cpu().numpy(), o2.cpu().numpy())
    with pytest.raises(ValueError):
        append_kv(fk, fv, k, v[:, :, :2])
    assert device_status(0) == 0


def test_append_kv_host_sources(cuda):
    """bgtq_append_kv from host NumPy buffers (FP16 bits / float32, uploaded in stream order)
    writes what the device-source call writes; a non-finite host value is refused with the
    stores unchanged."""
    import torch
    from bgtq import RangeError, Values, append_kv
    zh = np.load(GOLDEN / "smollm2_heads.npz")
    H, B, d = 2, 4, 64
    tabs = [(zh[f"h{h}_config"], zh[f"h{h}_table"]) for h in range(H)]
    hk = [PackedKeys(t, 32, sequences=B) for t in tabs]
    hv = [Values(d, 32, "f16", sequences=B) for _ in range(H)]
    dk = [PackedKeys(t, 32, sequences=B) for t in tabs]
    dv = [Values(d, 32, "f16", sequences=B) for _ in range(H)]
    rng = np.random.default_rng(9)
    for n in (3, 1):
        k = (rng.standard_normal((B, n, H, d)) * 2).astype(np.float16)
        v = rng.standard_normal((B, n, H, d)).astype(np.float32)
        append_kv(hk, hv, k.view(np.uint16), v)
        append_kv(dk, dv, torch.from_numpy(k).to(cuda), torch.from_numpy(v).to(cuda))
    torch.cuda.synchronize()
    for h in range(H):
        for s in range(B):
            assert hk[h].lengths(s) == dk[h].lengths(s) == 4 == hv[h].lengths(s)
            np.testing.assert_array_equal(hk[h].read(s)[0], dk[h].read(s)[0])
            np.testing.assert_array_equal(hk[h].read(s)[1], dk[h].read(s)[1])
    bad = np.zeros((B, 1, H, d), np.float32)
    bad[1, 0, 1, 5] = np.inf
    with pytest.raises(RangeError):
        append_kv(hk, hv, np.zeros((B, 1, H, d), np.float16), bad)
    assert hk[0].lengths(0) == 4 and hv[1].lengths(3) == 4
    assert device_status(0) == 0


@pytest.mark.parametrize("dtype,dim", [("f16", 64), ("f16", 128), ("f16", 48), ("f32", 64)])
def test_values_read_round_trip(cuda, dtype, dim):
    """bgtq_values_read returns the rows as appended (FP16 rows of 64 / 128 halves are stored
    chunk-swizzled on the device; the read undoes it)."""
    from bgtq import Values
    rng = np.random.default_rng(dim)
    S, n = 3, 77
    v = Values(dim, 200, dtype, sequences=S)
    rows = rng.standard_normal((S, n, dim)).astype(np.float16 if dtype == "f16" else np.float32)
    v.append(rows)
    v.append(rows[:, :5], seq_first=0)
    for s in range(S):
        got = v.read(s)
        assert got.shape == (n + 5, dim)
        np.testing.assert_array_equal(got[:n], rows[s])
        np.testing.assert_array_equal(got[n:], rows[s, :5])
    np.testing.assert_array_equal(v.read(1, 10, 3), rows[1, 10:13])
