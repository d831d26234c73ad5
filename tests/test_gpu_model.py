"""Model-path decoder (bgtq.model.Decoder) against a plain PyTorch FP32 decoder whose
attention is the oracle on the library's own codes.

The reference decoder below restates src/model/decoder.ts:31-81 in torch (embedding,
RMSNorm, projections, split-half RoPE, SiLU-gated MLP, tied lm_head); its keys are the
oracle's reconstruction of the packed cache the Decoder wrote, its values the FP16-rounded
projections, and its attention is oracle.attention in double precision.  Both run the same
torch GEMMs on the same device, so the only difference is the attention kernels: logits
must agree to 1e-4 abs + 1e-3 rel through a prefill chunk and decode steps, for a
SmolLM2-like (GQA 3, no bias) and a Qwen-like (GQA 3 x 2 KV heads, QKV bias) geometry;
and, at the benchmarked context, through a 4096-token prefix prefilled in 1024-token chunks
followed by decode steps replayed from the recorded CUDA graph.
"""
import os

import numpy as np
import pytest

import oracle
from bgtq import device_status
from bgtq.model import Decoder, ModelGeometry, random_weights
from conftest import GOLDEN

pytestmark = pytest.mark.gpu
THREADS = os.cpu_count() or 8
GEOMS = {
    "smollm2-like": ModelGeometry("smollm2", 2, 192, 256, 3, 1, 1e5, 1e-5, 500, False),
    "qwen-like": ModelGeometry("qwen2", 2, 384, 512, 6, 2, 1e6, 1e-6, 700, True),
}


def _tables(g):
    zh = np.load(GOLDEN / "smollm2_heads.npz")
    return [(zh[f"h{i % 6}_config"], zh[f"h{i % 6}_table"]) for i in range(g.layers * g.kv_heads)]


def _reference_forward(dec, w, g, tokens, start, tables):
    """One forward of the restated decoder; K from the Decoder's packed cache."""
    import torch
    B, n = tokens.shape
    h = w["model.embed_tokens.weight"][tokens].float()

    def norm(x, wt):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + g.rms_eps) * wt.float()

    pairs = g.head_dim // 2
    inv = torch.pow(torch.tensor(float(g.rope_theta), device=h.device),
                    -torch.arange(pairs, device=h.device, dtype=torch.float32) / pairs)
    pos = torch.arange(start, start + n, device=h.device, dtype=torch.float32)
    ang = pos[:, None] * inv[None, :]
    c, s = torch.cos(ang)[None, :, None, :], torch.sin(ang)[None, :, None, :]

    def rope(x):
        a, b = x[..., :pairs], x[..., pairs:]
        return torch.cat([a * c - b * s, b * c + a * s], -1)

    for layer in range(g.layers):
        p = f"model.layers.{layer}."
        x = norm(h, w[p + "input_layernorm.weight"])
        lin = lambda t, nm, b=None: t @ w[nm].float().t() + (w[b].float() if b else 0)
        bias = (lambda nm: p + f"self_attn.{nm}.bias") if g.qkv_bias else (lambda nm: None)
        q = rope(lin(x, p + "self_attn.q_proj.weight", bias("q_proj")).view(B, n, g.q_heads, 64))
        v = lin(x, p + "self_attn.v_proj.weight", bias("v_proj")).view(B, n, g.kv_heads, 64)
        out = np.zeros((B, n, g.q_heads, 64), np.float32)
        qn = q.cpu().numpy()
        for b in range(B):
            for hd in range(g.kv_heads):
                # the Decoder's own FP16 V rows (as its own K codes below): the restated
                # projection agrees with them to FP32 rounding, but one FP16 rounding step
                # apart in a few elements, which the comparison is not about
                vh = dec.values[layer][hd].read(b, 0, start + n).astype(np.float32)
                mine = v[b, :, hd].half().float().cpu().numpy()
                assert np.abs(vh[start:] - mine).max() <= 2.0 ** -10 * max(1.0, float(np.abs(mine).max()))
                cfg, tab = tables[layer * g.kv_heads + hd]
                packed, scales = dec.keys[layer][hd].read(b, 0, start + n)
                kh = oracle.reconstruct(cfg, tab, packed, scales, threads=THREADS)
                rows = qn[b, :, hd * g.gqa:(hd + 1) * g.gqa].reshape(n * g.gqa, 64)
                ps = np.repeat(np.arange(start, start + n, dtype=np.uint32), g.gqa)
                _, _, o = oracle.attention(rows, kh, vh, ps, True, threads=THREADS)
                out[b, :, hd * g.gqa:(hd + 1) * g.gqa] = o.reshape(n, g.gqa, 64)
        att = torch.from_numpy(out).to(h.device).reshape(B, n, g.hidden)
        h = h + lin(att, p + "self_attn.o_proj.weight")
        x = norm(h, w[p + "post_attention_layernorm.weight"])
        up = lin(x, p + "mlp.up_proj.weight")
        h = h + lin(torch.nn.functional.silu(lin(x, p + "mlp.gate_proj.weight")) * up, p + "mlp.down_proj.weight")
    last = norm(h[:, -1], w["model.norm.weight"])
    return last @ w["model.embed_tokens.weight"].float().t()


@pytest.mark.parametrize("name", sorted(GEOMS))
def test_decoder_matches_reference_decoder(cuda, name):
    import torch
    g = GEOMS[name]
    tables = _tables(g)
    w = random_weights(g, seed=3, device=cuda, std=0.08)
    B, prompt, steps = 2, 150, 3
    dec = Decoder(w, g, 256, tables, batch=B)
    rng = np.random.default_rng(1)
    toks = torch.from_numpy(rng.integers(0, g.vocab, (B, prompt))).to(cuda)
    got = dec.prefill(toks, chunk=100)       # two chunks: 100 + 50 positions
    # the reference consumes the same chunks (its V cache grows with them)
    _reference_forward(dec, w, g, toks[:, :100], 0, tables)
    ref = _reference_forward(dec, w, g, toks[:, 100:], 100, tables)
    np.testing.assert_allclose(got.cpu().numpy(), ref.cpu().numpy(), atol=1e-4, rtol=1e-3)
    start = prompt
    for _ in range(steps):
        nxt = torch.from_numpy(rng.integers(0, g.vocab, (B, 1))).to(cuda)
        got = dec.decode(nxt)
        ref = _reference_forward(dec, w, g, nxt, start, tables)
        np.testing.assert_allclose(got.cpu().numpy(), ref.cpu().numpy(), atol=1e-4, rtol=1e-3)
        start += 1
    assert dec.length == prompt + steps
    assert device_status(0) == 0
    dec.destroy()


@pytest.mark.parametrize("name", sorted(GEOMS))
def test_graph_decode_after_4096_prefix_matches_reference(cuda, name):
    """The benchmarked decode path at its context: a 4096-token prefix prefilled in four
    1024-token chunks (tensor-core prefill), one eager decode step that records the CUDA
    graph, then two replayed steps - each step's logits against the restated decoder with
    oracle attention over the same 4096+ positions."""
    import torch
    g = GEOMS[name]
    tables = _tables(g)
    w = random_weights(g, seed=9, device=cuda, std=0.08)
    prefix, chunk = 4096, 1024
    dec = Decoder(w, g, prefix + 8, tables, batch=1)
    rng = np.random.default_rng(12)
    toks = torch.from_numpy(rng.integers(0, g.vocab, (1, prefix))).to(cuda)
    got = dec.prefill(toks, chunk=chunk)
    for a in range(0, prefix, chunk):
        ref = _reference_forward(dec, w, g, toks[:, a:a + chunk], a, tables)
    np.testing.assert_allclose(got.cpu().numpy(), ref.cpu().numpy(), atol=1e-4, rtol=1e-3)
    steps = [torch.from_numpy(rng.integers(0, g.vocab, (1, 1))).to(cuda) for _ in range(3)]
    got = dec.capture_decode(steps[0])                       # eager step, then the graph is recorded
    ref = _reference_forward(dec, w, g, steps[0], prefix, tables)
    np.testing.assert_allclose(got.cpu().numpy(), ref.cpu().numpy(), atol=1e-4, rtol=1e-3)
    for i, t in enumerate(steps[1:], start=1):
        got = dec.decode_graph(t).clone()
        dec._sync_lengths()                                  # the reference reads the replayed cache rows
        ref = _reference_forward(dec, w, g, t, prefix + i, tables)
        np.testing.assert_allclose(got.cpu().numpy(), ref.cpu().numpy(), atol=1e-4, rtol=1e-3)
    assert dec.length == prefix + 3
    assert device_status(0) == 0
    dec.destroy()


def test_decoder_rejects_bad_requests(cuda):
    g = GEOMS["smollm2-like"]
    with pytest.raises(ValueError, match="geometry"):
        ModelGeometry("smollm2", 2, 200, 256, 3, 1, 1e5, 1e-5, 500, False)
    with pytest.raises(ValueError, match="Calibration"):
        Decoder(random_weights(g, device=cuda), g, 64, _tables(g)[:1] * 0, batch=1)
    dec = Decoder(random_weights(g, device=cuda), g, 8, _tables(g), batch=1)
    with pytest.raises(ValueError, match="tokens"):
        dec.prefill(np.zeros((1, 9), np.int64))
    with pytest.raises(ValueError, match="tokens"):
        dec.decode(np.array([[g.vocab]]))
    dec.destroy()


def test_fused_rope_append_equals_separate_steps(cuda):
    """bgtq_append_kv_rope (one launch: RoPE on K, encode, FP16 V append for every KV head)
    writes the bytes that torch RoPE followed by PackedKeys / Values appends write."""
    import ctypes as C
    import torch
    from bgtq import GroupedAttention, PackedKeys, Values, _lib
    zh = np.load(GOLDEN / "smollm2_heads.npz")
    H, G, B, d = 2, 3, 3, 64
    pairs = d // 2
    inv = torch.pow(torch.tensor(1e5, dtype=torch.float32), -torch.arange(pairs, dtype=torch.float32) / pairs)
    rng = np.random.default_rng(8)
    tabs = [(zh[f"h{h}_config"], zh[f"h{h}_table"]) for h in range(H)]
    fused_k = [PackedKeys(t, 64, sequences=B) for t in tabs]
    fused_v = [Values(d, 64, "f16", sequences=B) for _ in range(H)]
    ref_k = [PackedKeys(t, 64, sequences=B) for t in tabs]
    ref_v = [Values(d, 64, "f16", sequences=B) for _ in range(H)]
    row = (H * G + 2 * H) * d
    kp = (C.c_void_p * H)(*[k._handle for k in fused_k])
    vp = (C.c_void_p * H)(*[v._handle for v in fused_v])
    start = 0
    for n in (5, 1, 1, 7):
        qkv = torch.from_numpy(rng.standard_normal((B, n, row)).astype(np.float32) * 3).to(cuda)
        _lib.call("bgtq_append_kv_rope", H, kp, vp, C.c_void_p(qkv.data_ptr()), row, n * row, H * G * d,
                  H * G * d + H * d, n, 0, B, inv.numpy().ctypes.data, None)
        pos = torch.arange(start, start + n, device=cuda, dtype=torch.float32)
        ang = pos[:, None] * inv.to(cuda)[None, :]
        c, s = torch.cos(ang), torch.sin(ang)
        for h in range(H):
            k = qkv[:, :, H * G * d + h * d:H * G * d + (h + 1) * d]
            a, b = k[..., :pairs], k[..., pairs:]
            kr = torch.cat([a * c - b * s, b * c + a * s], -1).contiguous()
            ref_k[h].append(kr)
            ref_v[h].append(qkv[:, :, H * G * d + H * d + h * d:H * G * d + H * d + (h + 1) * d].contiguous())
        start += n
    torch.cuda.synchronize()
    for h in range(H):
        for s_ in range(B):
            assert fused_k[h].lengths(s_) == ref_k[h].lengths(s_) == start
            np.testing.assert_array_equal(fused_k[h].read(s_)[0], ref_k[h].read(s_)[0])
            np.testing.assert_array_equal(fused_k[h].read(s_)[1], ref_k[h].read(s_)[1])
    # values: attention with the same keys sees the same V rows
    q = torch.from_numpy(rng.standard_normal((B, H, G, d)).astype(np.float32)).to(cuda)
    o1 = GroupedAttention(fused_k, fused_v, G).attend(q)
    o2 = GroupedAttention(fused_k, ref_v, G).attend(q)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(o1.cpu().numpy(), o2.cpu().numpy())
    assert device_status(0) == 0


def test_graph_replayed_decode_matches_eager(cuda):
    """A CUDA graph of the decode step (capture_decode / decode_graph) gives the eager
    decoder's logits while the caches grow across replays."""
    import torch
    g = GEOMS["qwen-like"]
    w = random_weights(g, seed=5, device=cuda, std=0.08)
    B = 2
    eager = Decoder(w, g, 200, _tables(g), batch=B)
    graph = Decoder(w, g, 200, _tables(g), batch=B)
    rng = np.random.default_rng(4)
    prompt = torch.from_numpy(rng.integers(0, g.vocab, (B, 60))).to(cuda)
    eager.prefill(prompt)
    graph.prefill(prompt)
    toks = [torch.from_numpy(rng.integers(0, g.vocab, (B, 1))).to(cuda) for _ in range(6)]
    np.testing.assert_allclose(graph.capture_decode(toks[0]).cpu().numpy(), eager.decode(toks[0]).cpu().numpy(),
                               atol=1e-5, rtol=1e-4)
    for t in toks[1:]:
        got = graph.decode_graph(t).clone()
        ref = eager.decode(t)
        np.testing.assert_allclose(got.cpu().numpy(), ref.cpu().numpy(), atol=1e-5, rtol=1e-4)
    assert graph.length == eager.length == 66
    graph._sync_lengths()
    assert graph.keys[0][0].lengths(1) == 66
    # an eager step after replays continues from the device lengths
    t = torch.from_numpy(rng.integers(0, g.vocab, (B, 1))).to(cuda)
    np.testing.assert_allclose(graph.decode(t).cpu().numpy(), eager.decode(t).cpu().numpy(), atol=1e-5, rtol=1e-4)
    assert device_status(0) == 0
    eager.destroy()
    graph.destroy()


@pytest.mark.parametrize("name,batch", [("smollm2-like", 1), ("qwen-like", 3), ("gqa7", 1), ("gqa7", 4)])
def test_persistent_step_matches_launch_path(cuda, name, batch):
    """The persistent decode step (one cooperative launch for the whole model) against the
    seven-launch fused path on the same weights and prompt: logits within 1e-5 abs + 1e-4
    rel; layer 0's new keys and values (inputs: the token embeddings, normalised and
    projected in the same order by both paths) bit for bit equal, so the step's K encode is
    the append kernel's; deeper layers' inputs differ by float rounding (the attention and
    query rotation compile apart), so their codes agree but for rare bin-edge flips."""
    import torch
    g = GEOMS.get(name) or ModelGeometry("qwen2", 2, 448, 384, 7, 1, 1e6, 1e-6, 300, True)
    tables = _tables(g)
    w = random_weights(g, seed=21, device=cuda, std=0.08)
    step = Decoder(w, g, 400, tables, batch=batch)
    ref = Decoder(w, g, 400, tables, batch=batch, step=False)
    assert step.step_kernel and not ref.step_kernel
    rng = np.random.default_rng(30 + batch)
    prompt = torch.from_numpy(rng.integers(0, g.vocab, (batch, 257))).to(cuda)
    step.prefill(prompt, chunk=200)
    ref.prefill(prompt, chunk=200)
    for _ in range(5):
        t = torch.from_numpy(rng.integers(0, g.vocab, (batch, 1))).to(cuda)
        a, b = step.decode(t), ref.decode(t)
        np.testing.assert_allclose(a.cpu().numpy(), b.cpu().numpy(), atol=1e-5, rtol=1e-4)
    ctas, smem, _ = step.step_info()
    assert ctas >= 148 and smem > 0
    for layer in range(g.layers):
        for hd in range(g.kv_heads):
            for s in range(batch):
                assert step.keys[layer][hd].lengths(s) == ref.keys[layer][hd].lengths(s) == 262
                pk, sk = step.keys[layer][hd].read(s)
                pr, sr = ref.keys[layer][hd].read(s)
                vk, vr = step.values[layer][hd].read(s, 0, 262), ref.values[layer][hd].read(s, 0, 262)
                np.testing.assert_array_equal(pk[:257], pr[:257])      # the shared prefill
                if layer == 0:
                    np.testing.assert_array_equal(pk, pr)
                    np.testing.assert_array_equal(sk, sr)
                    np.testing.assert_array_equal(vk, vr)
                else:
                    assert np.mean(pk != pr) < 1e-2
                    np.testing.assert_allclose(vk.astype(np.float32), vr.astype(np.float32), atol=2e-3, rtol=2e-3)
    assert device_status(0) == 0
    step.destroy()
    ref.destroy()


def test_persistent_step_rejects_bad_requests(cuda):
    """bgtq_decoder_create refuses geometries the step kernel does not serve (head dim other
    than 64, more than 4 sequences), and bgtq_decoder_step refuses stores whose lengths
    differ between layers; a refused step changes no length."""
    import ctypes as C
    import torch
    from bgtq import _lib
    g = GEOMS["smollm2-like"]
    dec = Decoder(random_weights(g, seed=2, device=cuda), g, 64, _tables(g), batch=1)
    handle = dec._step_handle()
    assert handle is not None
    base = C.c_void_p()
    desc = _lib.DecoderDesc(g.layers, 1, g.hidden, g.q_heads, g.kv_heads, 32, g.intermediate, g.vocab, g.rms_eps,
                            dec.inv_freq.ctypes.data, None, None, None, None, None, None, None, None, None, None, None,
                            0)
    with pytest.raises(_lib.RangeError):
        _lib.call("bgtq_decoder_create", C.byref(desc), C.byref(base))
    desc.head_dim, desc.batch = 64, 5
    with pytest.raises(_lib.RangeError):
        _lib.call("bgtq_decoder_create", C.byref(desc), C.byref(base))
    # layer 1's stores one row ahead of layer 0's: the step refuses before launching
    k = torch.zeros((1, 64), dtype=torch.float16, device=cuda)
    for ks, vs in zip(dec.keys[1:], dec.values[1:]):
        for kk, vv in zip(ks, vs):
            kk.append(k)
            vv.append(k)
    t = torch.zeros((1, 1), dtype=torch.int64, device=cuda)
    with pytest.raises(_lib.StateError):
        dec.forward(t, _check=False)
    assert dec.keys[0][0].lengths(0) == 0 and dec.keys[1][0].lengths(0) == 1
    assert device_status(0) == 0
    dec.destroy()
