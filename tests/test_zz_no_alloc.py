"""bgtq_attend_static: attention for callers that cannot allocate device memory.

Some callers may not call cudaMalloc when they run attention - a serving process whose
memory pool already holds all free device memory, or a plugin inside a framework that
owns every device allocation.  For them the library offers bgtq_attend_static, which
attends the key/value stores directly and takes all of its scratch from one fixed array
compiled into the library.  These tests call it through the C ABI and check it against
the regular entry point (bgtq_attend via GroupedAttention) and against the CPU oracle on
sampled rows, at the attention tolerance of the other GPU tests, on consecutive calls;
that the device's free memory does not change across calls after the first (set-up)
call; and that a request larger than the fixed scratch is refused.
"""
import ctypes as C

import numpy as np
import pytest

import oracle
from bgtq import GroupedAttention, PackedKeys, Values, _lib, device_status, synthetic
from conftest import GOLDEN

pytestmark = pytest.mark.gpu
ATOL, RTOL = 1e-5, 1e-4


def attend_static(keys, values, q, out, rows, positions=None, causal=False, seq_first=0, seq_count=None):
    import torch
    karr = (C.c_void_p * len(keys))(*[k._handle for k in keys])
    varr = (C.c_void_p * len(values))(*[v._handle for v in values])
    seq_count = q.shape[0] if seq_count is None else seq_count
    stream = torch.cuda.current_stream(q.device).cuda_stream
    _lib.call("bgtq_attend_static", len(keys), karr, varr, C.c_void_p(q.data_ptr()),
              None if positions is None else C.c_void_p(positions.data_ptr()), int(causal), rows, seq_first, seq_count,
              C.c_void_p(out.data_ptr()), C.c_void_p(int(stream)))


def build_stores(rng, S, lengths, capacity):
    z = np.load(GOLDEN / "smollm2_heads.npz")
    keys, values, vdata = [], [], []
    for i in range(3):
        k = PackedKeys((z[f"h{i}_config"], z[f"h{i}_table"]), capacity, sequences=S)
        v = Values(64, capacity, "f16", sequences=S)
        vd = []
        for s, n in enumerate(lengths):
            k.append(synthetic.profiled(rng, n, 64).astype(np.float16).view(np.uint16), seq_first=s)
            vv = rng.standard_normal((n, 64)).astype(np.float16)
            v.append(vv, seq_first=s)
            vd.append(vv)
        keys.append(k)
        values.append(v)
        vdata.append(vd)
    return keys, values, vdata


def check_oracle(keys, vdata, q, out, seqs, positions=None, causal=False, seq_first=0):
    """Rows of `out` for the sampled local sequences `seqs` against the oracle on the
    GPU's own codes (double-precision attention over the reconstructed keys)."""
    z = np.load(GOLDEN / "smollm2_heads.npz")
    qn, on = q.cpu().numpy(), out.cpu().numpy()
    for s in seqs:
        for h in range(len(keys)):
            packed, scales = keys[h].read(seq_first + s)
            kh = oracle.reconstruct(z[f"h{h}_config"], z[f"h{h}_table"], packed, scales)
            pos = None if positions is None else positions[s].cpu().numpy().astype(np.uint32)
            _, _, o = oracle.attention(qn[s, h], kh, vdata[h][seq_first + s].astype(np.float32), pos, causal)
            np.testing.assert_allclose(on[s, h], o, atol=ATOL, rtol=RTOL)


def test_static_scratch_matches_regular_entry_point(cuda):
    import torch
    rng = np.random.default_rng(21)
    lengths = [5, 300, 2048, 4096, 4096, 1]
    S, rows = len(lengths), 3
    keys, values, vdata = build_stores(rng, S, lengths, 4096)
    regular = GroupedAttention(keys, values, rows)
    q = torch.from_numpy(synthetic.profiled(rng, S * 3 * rows, 64).reshape(S, 3, rows, 64)).to(cuda)
    expected = regular.attend(q)
    out = torch.full_like(q, float("nan"))
    attend_static(keys, values, q, out, rows)            # the first call on the device does the set-up
    torch.cuda.synchronize()
    for _ in range(2):                                   # two calls in a row share the scratch
        out = torch.full_like(q, float("nan"))
        attend_static(keys, values, q, out, rows)
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.cpu().numpy(), expected.cpu().numpy(), atol=ATOL, rtol=RTOL)
    check_oracle(keys, vdata, q, out, [0, 3, 5])
    # a different sub-batch with causal positions, again twice
    pos = torch.tensor([[0, 1, 2], [2047, 1000, 5], [4095, 3000, 17]], dtype=torch.int32, device=cuda)
    sub = q[2:5].contiguous()
    expected = regular.attend(sub, positions=pos, causal=True, seq_first=2, seq_count=3)
    outs = [torch.full_like(sub, float("nan")) for _ in range(2)]
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info(cuda)[0]
    for o in outs:
        attend_static(keys, values, sub, o, rows, positions=pos, causal=True, seq_first=2, seq_count=3)
        torch.cuda.synchronize()
        np.testing.assert_allclose(o.cpu().numpy(), expected.cpu().numpy(), atol=ATOL, rtol=RTOL)
    assert torch.cuda.mem_get_info(cuda)[0] == free1      # the calls took no device memory
    check_oracle(keys, vdata, sub, outs[1], [0, 1, 2], positions=pos, causal=True, seq_first=2)
    assert device_status(0) == 0


def test_static_scratch_refuses_requests_beyond_its_size(cuda):
    import torch
    rng = np.random.default_rng(3)
    S = 400                                             # 400 x 3 heads x 64 x 4 floats > 262,144
    keys, values, _ = build_stores(rng, S, [2] * S, 8)
    q = torch.zeros((S, 3, 3, 64), device=cuda)
    out = torch.zeros_like(q)
    with pytest.raises(_lib.RangeError, match="static scratch"):
        attend_static(keys, values, q, out, 3)
    attend_static(keys, values, q[:100].contiguous(), out[:100], 3, seq_count=100)   # within the limit
    torch.cuda.synchronize()
    assert torch.isfinite(out[:100]).all()
