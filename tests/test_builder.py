"""The native table builder (bgtq_tables_build) against the reference's own tables (CPU only).

Pins, all bit-exact:
* config 1 / config 4 (tests/golden/config{1,4}.npz): built by the reference's table code
  (production_oracle.setup -> BlockGTQPipeline._post_allocation_setup, build_code_lut,
  build_pack_meta) from allocator widths; the builder reproduces config and table from the
  widths alone, permutation included.
* the ten encoder fixtures of fixtures/mixed (rotation threshold 2, rows padded by 3 bytes,
  norm stride = groups + 1, as export_mixed.py writes them) and the six SmolLM2 calibration
  heads: tables exact from the widths; configs exact given the fixtures' pair order (they were
  made by torch builds whose unstable argsort orders equal widths differently).
* all 90 heads of the SmolLM2 calibration (tests/golden/smollm2_calibration.npz: widths,
  pair order, row padding, scale stride and the SHA-256 of the reference's config / table):
  tables exact from the widths alone, configs exact given the pair order.
* all 48 heads of the Qwen2.5-0.5B-geometry calibration (tests/golden/qwen_calibration.npz,
  made by tests/golden/make_qwen_calibration.py with the reference's calibration procedure
  and table code on the seeded random-init model): config and table exact from the widths
  alone (the builder's own pair order).
* the Haar rotation against NumPy's own generator + QR (the reference's
  _random_rotation_dense_torch, vendor/blockgtq/block_gtq_pipeline.py:81-92), and the
  builder's pair order against torch.argsort.
"""
import numpy as np
import pytest

import bgtq
from bgtq import BGTQError
from conftest import GOLDEN, load_config, load_mixed, mixed_cases, params_tables


def _numpy_haar(n, seed):
    """block_gtq_pipeline.py:81-92 (NumPy part), FP32 like the torch tensor it returns."""
    g = np.random.default_rng(seed).standard_normal((n, n))
    q, r = np.linalg.qr(g)
    s = np.sign(np.diag(r))
    s[s == 0] = 1.0
    q = q * s[None, :]
    if np.linalg.slogdet(q)[0] < 0:
        q[:, 0] = -q[:, 0]
    return q.astype(np.float32)


@pytest.mark.parametrize("n,seed", [(2, 45), (18, 47), (22, 45), (64, 46), (100, 7), (128, 50)])
def test_haar_rotation_matches_numpy(n, seed):
    np.testing.assert_array_equal(bgtq.haar_rotation(n, seed), _numpy_haar(n, seed))


@pytest.mark.parametrize("name", ["config1", "config4"])
def test_tables_from_widths_match_reference(name):
    z = load_config(name)
    cfg, tab = bgtq.build_tables(z["widths"].astype(np.int64))
    _, rcfg, rtab = params_tables(z)
    np.testing.assert_array_equal(cfg, rcfg)
    np.testing.assert_array_equal(tab, rtab)


@pytest.mark.parametrize("name", mixed_cases())
def test_tables_match_mixed_fixture(name):
    z = load_mixed(name)
    w = z["allocation"].astype(np.int64)
    kw = dict(rotation_threshold=2, row_pad=int(z["row_bytes"]) - int(z["logical_row_bytes"]),
              norm_stride=int(z["norm_stride"]))
    _, rcfg, rtab = params_tables(z)
    cfg, tab = bgtq.build_tables(w, **kw)
    np.testing.assert_array_equal(tab, rtab)          # rotation, centroids, offsets, inverse scales
    cfg, tab = bgtq.build_tables(w, pair_order=z["permutation"][0::2], **kw)
    np.testing.assert_array_equal(cfg, rcfg)          # permutation, groups, codebooks, code LUT
    np.testing.assert_array_equal(tab, rtab)


@pytest.mark.parametrize("head", range(6))
def test_tables_match_smollm2_calibration(head):
    z = np.load(GOLDEN / "smollm2_heads.npz")
    rcfg, rtab, w = z[f"h{head}_config"], z[f"h{head}_table"], z[f"h{head}_widths"].astype(np.int64)
    d, ns = int(rcfg[0]), int(rcfg[4])
    kw = dict(row_pad=int(rcfg[2]) - (ns // 2 + d - ns), norm_stride=int(rcfg[3]))
    _, tab = bgtq.build_tables(w, **kw)
    np.testing.assert_array_equal(tab, rtab)
    perm = rcfg[rcfg[6]:rcfg[6] + d]
    cfg, tab = bgtq.build_tables(w, pair_order=perm[0::2], **kw)
    np.testing.assert_array_equal(cfg, rcfg)
    np.testing.assert_array_equal(tab, rtab)


def _sha(a):
    import hashlib
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_tables_match_full_smollm2_calibration():
    z = np.load(GOLDEN / "smollm2_calibration.npz")
    assert z["widths"].shape == (90, 32) and int(z["rotation_threshold"]) == 2
    for i in range(90):
        w = z["widths"][i].astype(np.int64)
        kw = dict(rotation_threshold=int(z["rotation_threshold"]), row_pad=int(z["row_pad"][i]),
                  norm_stride=int(z["norm_stride"][i]))
        _, tab = bgtq.build_tables(w, **kw)
        assert _sha(tab.astype(np.float32)) == z["table_sha256"][i], i
        cfg, tab = bgtq.build_tables(w, pair_order=z["pair_order"][i].astype(np.int64), **kw)
        assert _sha(cfg.astype(np.uint32)) == z["config_sha256"][i], i
        assert _sha(tab.astype(np.float32)) == z["table_sha256"][i], i


def test_tables_match_qwen_calibration():
    z = np.load(GOLDEN / "qwen_calibration.npz")
    assert z["widths"].shape == (48, 32) and int(z["rotation_threshold"]) == 2
    for i in range(48):
        cfg, tab = bgtq.build_tables(z["widths"][i].astype(np.int64), rotation_threshold=2,
                                     norm_stride=int(z["norm_stride"][i]))
        assert _sha(cfg.astype(np.uint32)) == z["config_sha256"][i], i
        assert _sha(tab.astype(np.float32)) == z["table_sha256"][i], i
        assert np.array_equal(cfg[cfg[6]:cfg[6] + 64:2], z["pair_order"][i]), i


def test_pair_order_is_torch_argsort():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(3)
    for n in (8, 16, 32, 64):
        for _ in range(20):
            w = rng.integers(1, 9, n).astype(np.int64)
            cfg, _ = bgtq.build_tables(w)
            perm = cfg[cfg[6]:cfg[6] + 2 * n]
            np.testing.assert_array_equal(perm[0::2], torch.from_numpy(w).argsort().numpy())
            np.testing.assert_array_equal(perm[1::2], perm[0::2] + n)


def test_built_tables_validate_and_encode():
    """Tables from random widths pass the layout checks and drive the oracle encoder."""
    import oracle
    rng = np.random.default_rng(11)
    for d in (16, 64, 128):
        w = rng.integers(1, 9, d // 2).astype(np.int64)
        cfg, tab = bgtq.build_tables(w)
        info, _ = bgtq.validate_layout(cfg, tab)
        assert info.dim == d and info.groups == len(np.unique(w))
        k = (rng.standard_normal((4, d)) * 0.3).astype(np.float16).view(np.uint16)
        r = oracle.encode(cfg, tab, k)
        assert r["packed"].shape[0] == 4


def test_builder_rejects_bad_requests():
    with pytest.raises(BGTQError):
        bgtq.build_tables(np.array([0, 3], np.int64))
    with pytest.raises(BGTQError):
        bgtq.build_tables(np.array([9, 3], np.int64))
    with pytest.raises(BGTQError, match="pair_order"):
        bgtq.build_tables(np.array([3, 4, 5], np.int64), pair_order=np.array([1, 0, 2]))   # not width-ascending
    with pytest.raises(BGTQError, match="pair_order"):
        bgtq.build_tables(np.array([3, 3, 5], np.int64), pair_order=np.array([0, 0, 2]))   # not a permutation
    with pytest.raises(BGTQError):
        bgtq.build_tables(np.array([3, 4], np.int64), norm_stride=1)                      # below the group count
