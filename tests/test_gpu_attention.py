"""Compressed-K (and FP16-K / materialised) attention on the GPU through the C ABI.

Parity bar: outputs within 1e-5 abs + 1e-4 rel of the oracle run on the GPU's own
codes (identical effective K, as tests/oracles/verify_attention.py does), logits and
probabilities within the reference's baseline tolerances; the reference's own goldens
within its "port" tolerances (fixtures/attention/*.json).  Contracts mirror
tests/webgpu/attention-test.ts, optimized-test.ts and runtime-contracts.ts.
"""
import numpy as np
import pytest

import oracle
from bgtq import (AttentionEngine, CompressedKeys, FP16Keys, GroupedAttention, OptimizedAttention, PackedKeys, Values,
                  _lib, device_status, synthetic)
from conftest import GOLDEN, attention_cases, load_attention, load_config, load_mixed, params_tables

pytestmark = pytest.mark.gpu
ATOL, RTOL = 1e-5, 1e-4   # north-star attention tolerance


def fixture_stores(z, kind="packed", vdtype="f32"):
    p, cfg, tab = params_tables(load_mixed(str(z["layout"])))
    T = z["k_bits"].shape[0]
    if kind == "packed":
        keys = PackedKeys((cfg, tab), T)
    elif kind == "compressed":
        keys = CompressedKeys((cfg, tab), T)
    else:
        keys = FP16Keys(p.dim, T)
    values = Values(p.dim, T, vdtype)
    kb = z["k_bits"]
    keys.append(kb[:3])          # odd boundary: shared packed words across appends
    keys.append(kb[3:])
    values.append(z["v"][:3])
    values.append(z["v"][3:])
    return p, cfg, tab, keys, values


def check_stage(actual, ref, tol, extra=None):
    fin = np.isfinite(ref)
    np.testing.assert_array_equal(np.isfinite(actual), fin)
    atol, rtol = tol
    bound = atol + rtol * np.abs(ref[fin]) + (0 if extra is None else extra[fin])
    err = np.abs(actual[fin] - ref[fin])
    assert np.all(err <= bound), f"max err {err.max()} (bound {bound.min()})"


@pytest.mark.parametrize("name", attention_cases())
def test_fused_attention_matches_oracle_and_reference(cuda, name):
    z = load_attention(name)
    p, cfg, tab, keys, values = fixture_stores(z)
    packed, norms = keys.read()
    np.testing.assert_array_equal(packed, z["packed_k"])
    np.testing.assert_array_equal(norms, z["norm_bits"])
    kh = oracle.reconstruct(cfg, tab, packed, norms)   # the GPU's own effective K
    att = OptimizedAttention.create(keys, values, 3)
    for causal in (False, True):
        pre = "causal_" if causal else ""
        att.set_queries(z["q"], z["positions"], causal)
        att.record()
        got = att.inspect()
        lg, pr, out = oracle.attention(z["q"], kh, z["v"], z["positions"], causal)
        check_stage(got["logits"], lg, z["tol_baseline_logits"])
        check_stage(got["probabilities"], pr, z["tol_baseline_probabilities"])
        np.testing.assert_allclose(got["output"], out, atol=ATOL, rtol=RTOL)
        for stage in ("probabilities", "output"):
            check_stage(got[stage], z[pre + "compressed_" + stage], z[f"tol_port_{stage}"])
        fused = att.attend(z["q"], z["positions"], causal)      # fused path, no capture
        np.testing.assert_allclose(fused, out, atol=ATOL, rtol=RTOL)
        # attention-test.ts:74-80 contracts
        assert np.all(got["probabilities"] >= 0)
        np.testing.assert_allclose(got["probabilities"].sum(1), 1.0, atol=1e-4)
        if causal:
            T = z["k_bits"].shape[0]
            for r, pos in enumerate(z["positions"]):
                assert np.all(got["probabilities"][r, pos + 1:] == 0)
                assert np.all(np.isneginf(got["logits"][r, pos + 1:]))
            np.testing.assert_array_equal(got["output"][0], z["v"][0])
        again = att.attend(z["q"], z["positions"], causal)
        np.testing.assert_array_equal(again, fused)            # deterministic repeats
    assert device_status(0) == 0


@pytest.mark.parametrize("name", attention_cases())
@pytest.mark.parametrize("kind", ["fp16", "compressed"])
def test_baseline_sessions_match_reference(cuda, name, kind):
    z = load_attention(name)
    p, cfg, tab, keys, values = fixture_stores(z, kind)
    label = "baseline" if kind == "fp16" else "compressed"
    session = AttentionEngine.create().session(keys, values, 3)
    for causal in (False, True):
        pre = "causal_" if causal else ""
        session.set_queries(z["q"], z["positions"], causal)
        session.record()
        got = session.inspect()
        for stage in ("logits", "probabilities", "output"):
            tol = z[f"tol_baseline_{stage}"] if kind == "fp16" else z[f"tol_port_{stage}"]
            if kind == "compressed" and stage == "logits":
                continue
            check_stage(got[stage], z[pre + label + "_" + stage], tol)
        if kind == "compressed":
            kh = oracle.reconstruct(cfg, tab, *keys.read())
            lg, pr, out = oracle.attention(z["q"], kh, z["v"], z["positions"], causal)
            np.testing.assert_allclose(got["output"], out, atol=ATOL, rtol=RTOL)
            check_stage(got["logits"], lg, z["tol_baseline_logits"])


def test_runtime_contracts(cuda):
    """runtime-contracts.ts + optimized-test.ts appendContracts."""
    z = load_attention("t128_d64")
    p, cfg, tab = params_tables(load_mixed(str(z["layout"])))
    kb, v = z["k_bits"], z["v"]
    for make in (lambda: PackedKeys((cfg, tab), 3), lambda: FP16Keys(p.dim, 3), lambda: CompressedKeys((cfg, tab), 3)):
        keys, values = make(), Values(p.dim, 3)
        att = OptimizedAttention(keys, values, 1)
        with pytest.raises(_lib.StateError):
            att.set_queries(np.zeros(p.dim, np.float32), [0])
        keys.append(kb[:1])
        values.append(v[:1])
        out = att.attend(np.zeros(p.dim, np.float32), [0], True)
        np.testing.assert_array_equal(out[0], v[0])             # single key returns V0 exactly
        keys.append(kb[1:3])
        with pytest.raises(_lib.RangeError):                      # K/V lengths differ
            att.set_queries(np.zeros(p.dim, np.float32), [0])
        values.append(v[1:3])
        out = att.attend(np.zeros(p.dim, np.float32), [2], True)  # zero query averages V
        np.testing.assert_allclose(out[0], v[:3].mean(0), atol=1e-6, rtol=1e-6)
        for bad in (lambda: keys.append(kb[:1]), lambda: values.append(v[:1]),
                    lambda: att.set_queries(np.zeros(p.dim, np.float32), [3]),
                    lambda: att.set_queries(np.zeros(p.dim - 1, np.float32), [0]),
                    lambda: att.set_queries(np.full(p.dim, np.nan, np.float32), [0])):
            with pytest.raises(_lib.RangeError):
                bad()
        assert keys.length == 3 and values.length == 3           # overflow did not mutate


def _grouped_case(rng, layouts, S, lengths, rows, vdtype, capacity):
    stores = []
    for cfg, tab in layouts:
        keys = PackedKeys((cfg, tab), capacity, sequences=S)
        values = Values(64, capacity, vdtype, sequences=S)
        ks, vs = [], []
        for s in range(S):
            k = synthetic.profiled(rng, lengths[s], 64).astype(np.float16)
            vv = rng.standard_normal((lengths[s], 64)).astype(np.float16 if vdtype == "f16" else np.float32)
            keys.append(k.view(np.uint16), seq_first=s)
            values.append(vv, seq_first=s)
            ks.append(k)
            vs.append(vv.astype(np.float32))
        stores.append((keys, values, ks, vs, cfg, tab))
    return stores


@pytest.mark.parametrize("vdtype", ["f16", "f32"])
@pytest.mark.parametrize("rows", [1, 3, 7])
def test_grouped_decode_ragged_batch(cuda, vdtype, rows):
    """GQA decode: 3 KV heads with different calibrations, ragged sequence lengths."""
    zh = np.load(GOLDEN / "smollm2_heads.npz")
    layouts = [(zh[f"h{i}_config"], zh[f"h{i}_table"]) for i in range(3)]
    rng = np.random.default_rng(rows)
    S, lengths = 5, [1, 77, 640, 1500, 3001]
    stores = _grouped_case(rng, layouts, S, lengths, rows, vdtype, 3072)
    att = GroupedAttention([s[0] for s in stores], [s[1] for s in stores], rows)
    q = synthetic.profiled(rng, S * 3 * rows, 64).reshape(S, 3, rows, 64)
    positions = np.array([[max(0, L - 1 - r * 5) for r in range(rows)] for L in lengths], np.uint32)
    for causal in (False, True):
        outs = []
        for splits in (0, 1, 5):
            att.set_splits(splits)
            outs.append(att.attend(q, positions, causal))
        for s in range(S):
            for h, (keys, values, ks, vs, cfg, tab) in enumerate(stores):
                kh = oracle.reconstruct(cfg, tab, *keys.read(s))
                _, _, ref = oracle.attention(q[s, h], kh, vs[s], positions[s], causal)
                for o in outs:
                    np.testing.assert_allclose(o[s, h], ref, atol=ATOL, rtol=RTOL)
    assert device_status(0) == 0


@pytest.mark.parametrize("vdtype", ["f16", "f32"])
@pytest.mark.parametrize("rows", [1, 3])
def test_stream_k_decode_matches_oracle(cuda, vdtype, rows):
    """Stream-K schedule (key tiles dealt to one wave of CTAs in equal ranges, ranges crossing
    pairs; segments merged like splits): ragged lengths, one calibration for every head
    (one kernel body), against the oracle and the split-KV schedule."""
    zh = np.load(GOLDEN / "smollm2_heads.npz")
    layouts = [(zh["h0_config"], zh["h0_table"])] * 3
    rng = np.random.default_rng(40 + rows)
    S, lengths = 6, [1, 77, 640, 1500, 3001, 4096]
    stores = _grouped_case(rng, layouts, S, lengths, rows, vdtype, 4096)
    att = GroupedAttention([s[0] for s in stores], [s[1] for s in stores], rows)
    q = synthetic.profiled(rng, S * 3 * rows, 64).reshape(S, 3, rows, 64)
    positions = np.array([[max(0, L - 1 - r * 5) for r in range(rows)] for L in lengths], np.uint32)
    for causal in (False, True):
        att.set_schedule("stream_k")
        sk = att.attend(q, positions, causal)
        assert att.last_stream_k > 0
        att.set_schedule("split")
        kv = att.attend(q, positions, causal)
        assert att.last_stream_k == 0
        for s in range(S):
            for h, (keys, values, ks, vs, cfg, tab) in enumerate(stores):
                kh = oracle.reconstruct(cfg, tab, *keys.read(s))
                _, _, ref = oracle.attention(q[s, h], kh, vs[s], positions[s], causal)
                np.testing.assert_allclose(sk[s, h], ref, atol=ATOL, rtol=RTOL)
                np.testing.assert_allclose(kv[s, h], ref, atol=ATOL, rtol=RTOL)
    # back to back: the per-pair tickets are reset by each launch's last segment
    att.set_schedule("stream_k")
    np.testing.assert_array_equal(att.attend(q), att.attend(q))
    assert device_status(0) == 0


def test_stream_k_fp16_keys_logits_and_sequence_window(cuda):
    """Stream-K with dense FP16 keys: ragged lengths over every sequence, then raw logits
    captured over every key of a window of equal-length sequences (seq_first > 0)."""
    rng = np.random.default_rng(7)
    S, lengths, rows = 5, [300, 1500, 1500, 1500, 77], 2
    keys = [FP16Keys(64, 2048, sequences=S) for _ in range(2)]
    values = [Values(64, 2048, "f16", sequences=S) for _ in range(2)]
    kv = []
    for k, v in zip(keys, values):
        ks, vs = [], []
        for s in range(S):
            kk = (rng.standard_normal((lengths[s], 64)) * 0.5).astype(np.float16)
            vv = rng.standard_normal((lengths[s], 64)).astype(np.float16)
            k.append(kk.view(np.uint16), seq_first=s)
            v.append(vv, seq_first=s)
            ks.append(kk.astype(np.float32))
            vs.append(vv.astype(np.float32))
        kv.append((ks, vs))
    att = GroupedAttention(keys, values, rows)
    att.set_schedule("stream_k")
    q = rng.standard_normal((S, 2, rows, 64)).astype(np.float32)
    out = att.attend(q)
    assert att.last_stream_k > 0
    for s in range(S):
        for h in range(2):
            ks, vs = kv[h]
            _, _, ref = oracle.attention(q[s, h], ks[s], vs[s])
            np.testing.assert_allclose(out[s, h], ref, atol=ATOL, rtol=RTOL)
    logits = np.zeros((3, 2, rows, 1500), np.float32)
    out = att.attend(q[1:4], seq_first=1, seq_count=3, logits=logits)
    assert att.last_stream_k > 0
    for i, s in enumerate(range(1, 4)):
        for h in range(2):
            ks, vs = kv[h]
            lg, _, ref = oracle.attention(q[s, h], ks[s], vs[s])
            np.testing.assert_allclose(out[i, h], ref, atol=ATOL, rtol=RTOL)
            np.testing.assert_allclose(logits[i, h], lg, atol=1e-4, rtol=1e-4)
    assert device_status(0) == 0


def test_stream_k_full_length_batch_and_schedule_switches(cuda):
    """A 32-sequence batch of 8192-token sequences over three KV heads of one calibration (the
    per-GPU share of config 4 at eight GPUs): stream-K, split-KV and the automatic schedule
    agree; a forced split count implies split-KV."""
    zh = np.load(GOLDEN / "smollm2_heads.npz")
    cfg, tab = zh["h0_config"], zh["h0_table"]
    rng = np.random.default_rng(3)
    S, T = 32, 8192
    keys = [PackedKeys((cfg, tab), T, sequences=S) for _ in range(3)]
    values = [Values(64, T, "f16", sequences=S) for _ in range(3)]
    k = synthetic.profiled(rng, T, 64).astype(np.float16).view(np.uint16)
    v = rng.standard_normal((T, 64)).astype(np.float16)
    for kk, vv in zip(keys, values):
        for s in range(S):
            kk.append(k, seq_first=s)
            vv.append(v, seq_first=s)
    att = GroupedAttention(keys, values, 3)
    q = synthetic.profiled(rng, S * 9, 64).reshape(S, 3, 3, 64)
    auto = att.attend(q)
    att.set_schedule("stream_k")
    sk = att.attend(q)
    assert att.last_stream_k > 0
    att.set_splits(4)
    forced = att.attend(q)
    assert att.last_stream_k == 0 and att.last_splits == 4
    np.testing.assert_allclose(sk, auto, atol=ATOL, rtol=RTOL)
    np.testing.assert_allclose(forced, auto, atol=ATOL, rtol=RTOL)
    kh = oracle.reconstruct(cfg, tab, *keys[1].read(5))
    _, _, ref = oracle.attention(q[5, 1], kh, v.astype(np.float32))
    np.testing.assert_allclose(sk[5, 1], ref, atol=ATOL, rtol=RTOL)
    assert device_status(0) == 0


def test_device_io_matches_host_io(cuda):
    import torch
    zh = np.load(GOLDEN / "smollm2_heads.npz")
    layouts = [(zh[f"h{i}_config"], zh[f"h{i}_table"]) for i in range(3)]
    rng = np.random.default_rng(9)
    S, lengths = 3, [4096, 4096, 4096]
    stores = _grouped_case(rng, layouts, S, lengths, 3, "f16", 4096)
    att = GroupedAttention([s[0] for s in stores], [s[1] for s in stores], 3)
    q = synthetic.profiled(rng, S * 9, 64).reshape(S, 3, 3, 64)
    host = att.attend(q)
    assert att.last_launches == 1   # one partial wave: every CTA rotates its own queries
    dev = att.attend(torch.from_numpy(q).to(cuda))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(dev.cpu().numpy(), host)
    # host buffers without the per-call wait: two calls queued, one synchronisation
    outs = [torch.empty((S, 3, 3, 64), pin_memory=True).numpy() for _ in range(2)]
    q2 = synthetic.profiled(rng, S * 9, 64).reshape(S, 3, 3, 64)
    att.attend(q, out=outs[0], wait=False)
    att.attend(q2, out=outs[1], wait=False)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(outs[0], host)
    np.testing.assert_array_equal(outs[1], att.attend(q2))


def test_config1_full_decode_matches_reference(cuda):
    """Config 1: 4096 keys, head_dim 128, one FP32 query at the last position."""
    z = load_config("config1")
    p, cfg, tab = params_tables(z)
    k, q, v = synthetic.decode_workload(0, 4096, 128)
    keys = PackedKeys((cfg, tab), 4096)
    values = Values(128, 4096, "f16")
    keys.append(k.view(np.uint16))
    values.append(v.view(np.uint16))
    att = OptimizedAttention(keys, values, 1)
    out = att.attend(q, [4095])
    np.testing.assert_allclose(out, z["output"], atol=ATOL, rtol=RTOL)
    att.record()
    np.testing.assert_allclose(att.inspect()["logits"], z["logits"], atol=1e-4, rtol=2e-5)
