"""Layout-specialised decode attention (bgtq_set_layout_jit): the kernel compiled at run
time for one group structure gives the generic kernel's outputs bit for bit - rows 1-4 and
7, FP16 and FP32 values, head dims 64 and 128, one and several splits, causal positions,
logit / log-sum-exp capture - and is what runs by default when the heads share a layout.
Heads with different structures (the SmolLM2 calibration) get a kernel compiled in the
background: every launch before and after it is ready gives the generic outputs, and a
launch inside a CUDA graph capture never loads it (the graph records the generic kernel)."""
import time

import numpy as np
import pytest

import bgtq
from bgtq import GroupedAttention, PackedKeys, Values, device_status
from conftest import GOLDEN, load_config

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _default_jit_mode():
    """Every test switches the specialised kernels on for every launch (its sizes are one wave
    of CTAs, which the automatic mode leaves on the generic kernel); the default comes back
    afterwards."""
    yield
    bgtq.set_layout_jit("auto")


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


def test_no_kernel_load_inside_graph_capture(cuda):
    import torch
    from bgtq import _lib
    z = np.load(GOLDEN / "smollm2_heads.npz")
    S, T, d, rows, heads = 2, 500, 64, 1, (0, 3, 1)   # three structures: a key no other test uses
    gen = torch.Generator(device=cuda).manual_seed(77)
    keys = [PackedKeys((z[f"h{h}_config"], z[f"h{h}_table"]), T, sequences=S) for h in heads]
    vals = [Values(d, T, "f16", sequences=S) for _ in heads]
    for k, v in zip(keys, vals):
        k.append((torch.randn((S, T, d), device=cuda, generator=gen) * 0.4).half())
        v.append(torch.randn((S, T, d), device=cuda, generator=gen).half())
    att = GroupedAttention(keys, vals, rows)
    _lib.call("bgtq_attention_plan_for_capacity", att._handle, 1)
    q = torch.randn((S, len(heads), rows, d), device=cuda, generator=gen)
    bgtq.set_layout_jit(False)
    ref = att.attend(q).clone()
    torch.cuda.synchronize()
    bgtq.set_layout_jit(True)
    assert bgtq.layout_jit_wait(240.0)                # no compile of an earlier test still pending
    c0 = bgtq.layout_jit_counts()
    att.attend(q)                                     # starts the background compile
    torch.cuda.synchronize()
    deadline = time.monotonic() + 240
    while bgtq.layout_jit_counts()["compiled"] == c0["compiled"]:   # no launches meanwhile
        assert bgtq.layout_jit_counts()["failed"] == c0["failed"]
        assert time.monotonic() < deadline, "background compile did not finish"
        time.sleep(0.25)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = att.attend(q)
    assert bgtq.layout_jit_counts()["loaded"] == c0["loaded"]        # not loaded while capturing
    graph.replay()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), ref.cpu().numpy())
    got = att.attend(q).clone()                       # outside a capture: loads and runs it
    torch.cuda.synchronize()
    assert bgtq.layout_jit_counts()["loaded"] == c0["loaded"] + 1
    np.testing.assert_array_equal(got.cpu().numpy(), ref.cpu().numpy())
    graph.replay()                                    # the recorded generic kernel still replays
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), ref.cpu().numpy())
    del graph
    assert device_status(0) == 0


def test_wait_loads_and_graph_records_specialised_kernel(cuda):
    import torch
    from bgtq import _lib
    z = np.load(GOLDEN / "smollm2_heads.npz")
    S, T, d, rows, heads = 3, 400, 64, 4, (2, 4, 5, 3)   # four structures: a key no other test uses
    gen = torch.Generator(device=cuda).manual_seed(78)
    keys = [PackedKeys((z[f"h{h}_config"], z[f"h{h}_table"]), T, sequences=S) for h in heads]
    vals = [Values(d, T, "f16", sequences=S) for _ in heads]
    for k, v in zip(keys, vals):
        k.append((torch.randn((S, T, d), device=cuda, generator=gen) * 0.4).half())
        v.append(torch.randn((S, T, d), device=cuda, generator=gen).half())
    att = GroupedAttention(keys, vals, rows)
    _lib.call("bgtq_attention_plan_for_capacity", att._handle, 1)
    q = torch.randn((S, len(heads), rows, d), device=cuda, generator=gen)
    bgtq.set_layout_jit(False)
    ref = att.attend(q).clone()
    torch.cuda.synchronize()
    bgtq.set_layout_jit(True)
    assert bgtq.layout_jit_wait(240.0)                # loads what earlier tests left compiled
    c0 = bgtq.layout_jit_counts()
    att.attend(q)                                     # queues the compile
    torch.cuda.synchronize()
    assert bgtq.layout_jit_wait(240.0)
    c1 = bgtq.layout_jit_counts()
    assert c1["loaded"] == c0["loaded"] + 1 and c1["failed"] == c0["failed"]   # loaded without a launch
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = att.attend(q)                           # records the specialised kernel
    for _ in range(2):
        graph.replay()
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy(), ref.cpu().numpy())
    assert bgtq.layout_jit_counts() == c1
    assert bgtq.layout_jit_wait(0.0)                  # nothing queued: returns at once
    del graph
    assert device_status(0) == 0


def test_prebuilt_kernel_serves_the_config4_heads(cuda):
    """The build compiles the specialised kernel of the benchmarked heads ahead of time
    (bgtq/aot/): a launch over three config-4 heads with three query rows takes it from
    there - no compiler needed at run time - and gives the generic kernel's bytes."""
    import ctypes as C
    import torch
    from bgtq import _lib
    aot = _lib.LIB_PATH.parent / "aot"
    assert aot.is_dir() and any(aot.glob("*.cubin")), "build() writes the prebuilt kernels"
    S, T, H, R = 4, 900, 3, 3
    keys, vals, d, gen = _stores(cuda, "config4", S, T, H, "f16", seed=31)
    att = GroupedAttention(keys, vals, R)
    q = torch.randn((S, H, R, d), device=cuda, generator=gen)
    bgtq.set_layout_jit(True)
    spec = att.attend(q).clone()
    n = C.c_uint32()
    _lib.call("bgtq_layout_jit_prebuilt", C.byref(n))
    assert n.value >= 1
    bgtq.set_layout_jit(False)
    generic = att.attend(q).clone()
    bgtq.set_layout_jit(True)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(spec.cpu().numpy(), generic.cpu().numpy())
    assert device_status(0) == 0
