"""Layout-specialised decode attention (bgtq_set_layout_jit): the kernel compiled at run
time for one group structure gives the generic kernel's outputs bit for bit - rows 1-4 and
7, FP16 and FP32 values, head dims 64 and 128, one and several splits, causal positions,
logit / log-sum-exp capture - and is what runs by default when the heads share a layout.
Heads with different structures (the SmolLM2 calibration) get a kernel compiled in the
background: every launch before and after it is ready gives the generic outputs."""
import time

import numpy as np
import pytest

import bgtq
from bgtq import GroupedAttention, PackedKeys, Values, device_status
from conftest import GOLDEN, load_config

pytestmark = pytest.mark.gpu


def _stores(cuda, name, S, T, H, vdtype, seed):
    import torch
    z = load_config(name)
    cfg, tab = bgtq.tables(bgtq.BlockGTQParameters.from_arrays(z))
    d = int(z["dim"])
    gen = torch.Generator(device=cuda).manual_seed(seed)
    keys = [PackedKeys((cfg, tab), T, sequences=S) for _ in range(H)]
    vals = [Values(d, T, vdtype, sequences=S) for _ in range(H)]
    for h in range(H):
        keys[h].append((torch.randn((S, T, d), device=cuda, generator=gen) * 0.4).half())
        v = torch.randn((S, T, d), device=cuda, generator=gen)
        vals[h].append(v.half() if vdtype == "f16" else v)
    return keys, vals, d, gen


@pytest.mark.parametrize("name,vdtype", [("config4", "f16"), ("config4", "f32"), ("config1", "f16")])
@pytest.mark.parametrize("rows", [1, 2, 3, 4, 7])
def test_specialised_equals_generic(cuda, name, vdtype, rows):
    import torch
    S, T, H = 3, 700, 2
    keys, vals, d, gen = _stores(cuda, name, S, T, H, vdtype, seed=rows)
    att = GroupedAttention(keys, vals, rows)
    q = torch.randn((S, H, rows, d), device=cuda, generator=gen)
    pos = torch.from_numpy(np.random.default_rng(rows).integers(0, T, (S, rows)).astype(np.uint32)).to(cuda)
    for splits in (1, 0):
        att.set_splits(splits)
        outs = []
        for on in (False, True):
            bgtq.set_layout_jit(on)
            o1 = att.attend(q).clone()
            o2 = att.attend(q, positions=pos, causal=True).clone()
            torch.cuda.synchronize()
            outs.append((o1.cpu().numpy(), o2.cpu().numpy()))
        np.testing.assert_array_equal(outs[0][0], outs[1][0])
        np.testing.assert_array_equal(outs[0][1], outs[1][1])
    bgtq.set_layout_jit(True)
    built, failed = bgtq.layout_jit_stats()
    assert built >= 1 and failed == 0
    assert device_status(0) == 0


def test_specialised_logits_and_lse(cuda):
    import torch
    S, T, H, R = 2, 300, 3, 3
    keys, vals, d, gen = _stores(cuda, "config4", S, T, H, "f16", seed=11)
    att = GroupedAttention(keys, vals, R)
    q = torch.randn((S, H, R, d), device=cuda, generator=gen)
    res = []
    for on in (False, True):
        bgtq.set_layout_jit(on)
        lg = torch.empty((S, H, R, T), device=cuda)
        pr = torch.empty((S, H, R, T), device=cuda)
        o = att.attend(q, logits=lg, probs=pr).clone()
        torch.cuda.synchronize()
        res.append([t.cpu().numpy() for t in (o, lg, pr)])
    bgtq.set_layout_jit(True)
    for a, b in zip(*res):
        np.testing.assert_array_equal(a, b)
    assert device_status(0) == 0


@pytest.mark.parametrize("rows", [2, 7])
def test_mixed_layouts_compile_in_background(cuda, rows):
    import torch
    z = np.load(GOLDEN / "smollm2_heads.npz")
    S, T, H, d = 2, 900, 6, 64
    gen = torch.Generator(device=cuda).manual_seed(40 + rows)
    keys = [PackedKeys((z[f"h{h}_config"], z[f"h{h}_table"]), T, sequences=S) for h in range(H)]
    vals = [Values(d, T, "f16", sequences=S) for _ in range(H)]
    for h in range(H):
        keys[h].append((torch.randn((S, T, d), device=cuda, generator=gen) * 0.4).half())
        vals[h].append(torch.randn((S, T, d), device=cuda, generator=gen).half())
    att = GroupedAttention(keys, vals, rows)
    q = torch.randn((S, H, rows, d), device=cuda, generator=gen)
    pos = torch.from_numpy(np.random.default_rng(rows).integers(0, T, (S, rows)).astype(np.uint32)).to(cuda)

    def run():
        o1 = att.attend(q).clone()
        o2 = att.attend(q, positions=pos, causal=True).clone()
        torch.cuda.synchronize()
        return o1.cpu().numpy(), o2.cpu().numpy()

    bgtq.set_layout_jit(False)
    ref = run()
    bgtq.set_layout_jit(True)
    built0, failed0 = bgtq.layout_jit_stats()
    deadline = time.monotonic() + 240
    while True:
        got = run()                      # generic until the specialised kernel is loaded
        np.testing.assert_array_equal(got[0], ref[0])
        np.testing.assert_array_equal(got[1], ref[1])
        built, failed = bgtq.layout_jit_stats()
        assert failed == failed0
        if built > built0:
            break
        assert time.monotonic() < deadline, "background compile did not finish"
        time.sleep(0.25)
    got = run()                          # the specialised kernel
    np.testing.assert_array_equal(got[0], ref[0])
    np.testing.assert_array_equal(got[1], ref[1])
    assert device_status(0) == 0
