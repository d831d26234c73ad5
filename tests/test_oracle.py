"""Pin the CPU oracle against the reference's own golden vectors (CPU only).

The vectors under tests/golden/ were produced from the reference implementation by
tests/golden/make_golden.py: its committed fixtures (fixtures/mixed, fixtures/attention,
fixtures/allocator.json) and its Python encoder/attention on the config-1 / config-4
synthetic workloads.  Mirrors tests/test_mixed.py, tests/test_attention.py and
tests/test_allocator.py of the reference.
"""
import hashlib
import itertools

import numpy as np
import pytest

import oracle
from bgtq import synthetic
from conftest import (allocator_cases, attention_cases, load_attention, load_config, load_mixed, mixed_cases,
                      params_tables)


@pytest.mark.parametrize("name", mixed_cases())
def test_encoder_matches_reference_fixture(name):
    z = load_mixed(name)
    p, cfg, tab = params_tables(z)
    r = oracle.encode(cfg, tab, z["original"].astype(np.float16).view(np.uint16))
    np.testing.assert_array_equal(r["codes"], z["codes"])
    np.testing.assert_array_equal(r["packed"], z["packed"])
    # FP16 scale bits equal; FP32 corrected scales within the reference's own tolerance
    np.testing.assert_array_equal(r["scales"][:, :p.norm_stride], z["norm_bits"])
    np.testing.assert_allclose(r["corrected"], z["corrected_f32"][:, :p.groups], rtol=2e-5, atol=5e-4)


@pytest.mark.parametrize("name", mixed_cases())
def test_pack_unpack_and_reconstruct(name):
    z = load_mixed(name)
    p, cfg, tab = params_tables(z)
    np.testing.assert_array_equal(oracle.pack(z["codes"], p.nibble_dims, p.row_bytes), z["packed"])
    np.testing.assert_array_equal(oracle.unpack(z["packed"], p.dim, p.nibble_dims), z["codes"])
    assert np.all(z["packed"][:, int(z["logical_row_bytes"]):] == 0)
    rec = oracle.reconstruct(cfg, tab, z["packed"], z["norm_bits"])
    np.testing.assert_allclose(rec, z["reconstructed_f16"], atol=1e-3, rtol=2e-5)
    ranges = oracle.group_ranges(p.group_of, p.rotation, p.dim)
    assert np.all(ranges[1::2] > ranges[0::2])


def test_half_conversion_edges():
    values = [0, -0.0, 2 ** -24, 2 ** -25, 3 * 2 ** -25, 1 + 2 ** -11, 65504, 65520]
    np.testing.assert_array_equal(oracle.half_bits(values), [0, 32768, 1, 0, 2, 15360, 31743, 31744])
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(4000) * np.exp(rng.uniform(-20, 12, 4000))).astype(np.float32)
    with np.errstate(over="ignore"):
        np.testing.assert_array_equal(oracle.half_bits(x), x.astype(np.float16).view(np.uint16))


@pytest.mark.parametrize("name", attention_cases())
def test_attention_matches_reference_fixture(name):
    z = load_attention(name)
    p, cfg, tab = params_tables(load_mixed(str(z["layout"])))
    r = oracle.encode(cfg, tab, z["k_bits"])
    np.testing.assert_array_equal(r["packed"], z["packed_k"])
    np.testing.assert_array_equal(r["scales"], z["norm_bits"])
    k16 = z["k_bits"].view(np.float16).astype(np.float32)
    for causal in (False, True):
        pre = "causal_" if causal else ""
        for label, keys in (("baseline", k16), ("compressed", z["reconstructed_k"]), ("fp32_source", z["k_source"])):
            lg, pr, out = oracle.attention(z["q"], keys, z["v"], z["positions"], causal)
            for stage, val in (("logits", lg), ("probabilities", pr), ("output", out)):
                atol, rtol = z[f"tol_baseline_{stage}"]
                ref = z[pre + label + "_" + stage]
                fin = np.isfinite(ref)
                np.testing.assert_array_equal(np.isfinite(val), fin)
                np.testing.assert_allclose(val[fin], ref[fin], atol=atol, rtol=rtol)
            np.testing.assert_allclose(pr.sum(1), 1.0, atol=1e-6)
            if causal:
                assert np.all(pr[0, 1:] == 0)
                np.testing.assert_array_equal(out[0], z["v"][0])


def test_allocator_golden_cases_and_grid():
    for case in allocator_cases():
        got = oracle.allocate_bits(case["scores"], case["budget"], case["min_bits"], case["max_bits"])
        np.testing.assert_array_equal(got, case["expected"])


@pytest.mark.parametrize("name,dim,seed", [("config1", 128, 0), ("config4", 64, 4)])
def test_synthetic_workload_matches_reference_encoder(name, dim, seed):
    z = load_config(name)
    p, cfg, tab = params_tables(z)
    k, q, v = synthetic.decode_workload(seed, int(z["tokens"]), dim)
    h = hashlib.sha256()
    for a in (k, q, v):
        h.update(np.ascontiguousarray(a).tobytes())
    assert h.hexdigest() == str(z["input_sha256"]), "synthetic generator drifted"
    n = int(z["sample"])
    r = oracle.encode(cfg, tab, k[:n].view(np.uint16))
    mism = np.argwhere(r["codes"] != z["codes"])
    if len(mism):  # allowed only within float32 rounding of a LUT bin edge
        assert np.all(oracle.code_edge_distance(cfg, tab, k[:n].view(np.uint16), mism) < 1e-4)
    np.testing.assert_array_equal(r["packed"][np.all(r["codes"] == z["codes"], axis=1)],
                                  z["packed"][np.all(r["codes"] == z["codes"], axis=1)])
    diff = np.abs(r["scales"][:, :p.groups].astype(np.int64) - z["norm_bits"][:, :p.groups].astype(np.int64))
    assert diff.max() <= 1
    widths = oracle.allocate_bits(z["scores"], dim * 2, 1, 8)
    np.testing.assert_array_equal(widths, z["widths"])
    if "output" in z.files:
        full = oracle.encode(cfg, tab, k.view(np.uint16), threads=4)
        kh = oracle.reconstruct(cfg, tab, full["packed"], full["scales"], threads=4)
        lg, pr, out = oracle.attention(q, kh, v.astype(np.float32), [k.shape[0] - 1])
        np.testing.assert_allclose(out, z["output"], atol=1e-5, rtol=1e-4)
        np.testing.assert_allclose(lg, z["logits"], atol=1e-4, rtol=2e-5)


def test_group_ranges_rejections():
    z = load_mixed("mixed_d16")
    p, cfg, tab = params_tables(z)
    rot = p.rotation.reshape(p.dim, p.dim).copy()
    other = int(np.nonzero(p.group_of != p.group_of[0])[0][0])
    rot[other, 0] = 0.01
    with pytest.raises(ValueError, match="Off-group"):
        oracle.group_ranges(p.group_of, rot, p.dim)
    g = p.group_of.copy()
    g[0], g[-1] = g[-1], g[0]
    with pytest.raises(ValueError, match="Non-contiguous"):
        oracle.group_ranges(g, p.rotation, p.dim)


def test_pack_roundtrip_random():
    rng = np.random.default_rng(3)
    for d, ns in itertools.product((16, 64, 128), (0, 2, 40, 64)):
        if ns > d:
            continue
        codes = np.concatenate([rng.integers(0, 16, (9, ns)), rng.integers(0, 256, (9, d - ns))], axis=1).astype(np.uint8)
        rb = ns // 2 + d - ns + 5
        np.testing.assert_array_equal(oracle.unpack(oracle.pack(codes, ns, rb), d, ns), codes)


@pytest.mark.parametrize("name", ["config1", "config4"])
def test_torch_port_agrees_with_c_oracle(name):
    """The vectorised PyTorch restatement of the reference's CPU path (oracle/torch_port.py,
    the timed CPU baseline on the GPU box) against the C oracle: codes equal except at LUT
    bin edges, FP16 scales within one unit, and attention over the same packed keys within
    the attention tolerance."""
    import torch_port
    from bgtq import synthetic
    z = load_config(name)
    p, cfg, tab = params_tables(z)
    tb = torch_port.Tables(cfg, tab)
    k, q, v = synthetic.decode_workload(7, 2048, p.dim, queries=3)
    kb = k.view(np.uint16)
    codes, scales = torch_port.encode(tb, kb)
    ref = oracle.encode(cfg, tab, kb, threads=4)
    ref_codes = oracle.unpack(ref["packed"][:, :p.row_bytes], p.dim, p.nibble_dims)
    assert (codes.numpy() == ref_codes).mean() > 0.999
    d16 = np.abs(scales.numpy().view(np.uint16).astype(int)[:, :p.groups] -
                 ref["scales"][:, :p.groups].astype(int))
    assert d16.max() <= 1
    kh = torch_port.reconstruct(tb, ref["packed"][:, :p.row_bytes], ref["scales"])
    np.testing.assert_allclose(kh.numpy(), oracle.reconstruct(cfg, tab, ref["packed"], ref["scales"]),
                               atol=1e-5, rtol=1e-5)
    pos = np.array([0, 1000, 2047])
    _, _, out = torch_port.attention(q, kh, v.astype(np.float32), pos, True)
    _, _, out_c = oracle.attention(q, oracle.reconstruct(cfg, tab, ref["packed"], ref["scales"]),
                                   v.astype(np.float32), pos.astype(np.uint32), True)
    np.testing.assert_allclose(out.numpy(), out_c, atol=1e-5, rtol=1e-4)
    assert np.array_equal(torch_port.pack(tb, codes.numpy()), oracle.pack(codes.numpy(), p.nibble_dims, p.row_bytes))
