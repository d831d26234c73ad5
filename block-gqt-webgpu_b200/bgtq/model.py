"""SmolLM2 / Qwen2 decoder over the Block-GTQ key cache (the reference's model path).

Mirrors src/model/decoder.ts:15-83 (Decoder.create / forward / prefill / decode),
src/model/adapter.ts:17-42 (the two supported families) and src/model/kernels.wgsl:11-54
(embedding, RMSNorm, matmul with optional bias, split-half RoPE, SiLU-gated MLP, tied
lm_head).  The projections and MLP are plain weight-bound GEMMs (cuBLAS through torch);
the key path is this library's kernels: every new post-RoPE key is encoded straight from
the FP32 projection into the packed cache (the model-path encode of
src/model/codec.wgsl:11-33), values are appended as FP16, decode steps attend with the
grouped decode kernel and multi-token chunks with the tensor-core prefill kernel.

One Decoder holds `batch` sequences that advance together (equal lengths).  Random-init
weights (`random_weights`) stand in for checkpoints, which this package does not fetch.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .attention import GroupedAttention
from .runtime import PackedKeys, Values


@dataclass(frozen=True)
class ModelGeometry:
    """adapter.ts:1-42 fields (head_dim fixed at 64, tied embeddings, as the adapter requires)."""
    family: str
    layers: int
    hidden: int
    intermediate: int
    q_heads: int
    kv_heads: int
    rope_theta: float
    rms_eps: float
    vocab: int
    qkv_bias: bool
    head_dim: int = 64

    def __post_init__(self):
        if self.head_dim != 64 or self.hidden != self.q_heads * self.head_dim or self.q_heads % self.kv_heads:
            raise ValueError("Unsupported attention geometry")  # adapter.ts:21
        if self.rms_eps not in (1e-5, 1e-6):
            raise ValueError("Unsupported RoPE or RMSNorm configuration")  # adapter.ts:24

    @property
    def gqa(self) -> int:
        return self.q_heads // self.kv_heads


SMOLLM2_135M = ModelGeometry("smollm2", 30, 576, 1536, 9, 3, 1e5, 1e-5, 49152, False)
QWEN25_05B = ModelGeometry("qwen2", 24, 896, 4864, 14, 2, 1e6, 1e-6, 151936, True)


def weight_names(g: ModelGeometry):
    """HF tensor names and shapes the reference loads (weights.ts:31-39)."""
    names = {"model.embed_tokens.weight": (g.vocab, g.hidden), "model.norm.weight": (g.hidden,)}
    kv = g.kv_heads * g.head_dim
    for layer in range(g.layers):
        p = f"model.layers.{layer}."
        names[p + "input_layernorm.weight"] = (g.hidden,)
        names[p + "post_attention_layernorm.weight"] = (g.hidden,)
        names[p + "self_attn.q_proj.weight"] = (g.hidden, g.hidden)
        names[p + "self_attn.k_proj.weight"] = (kv, g.hidden)
        names[p + "self_attn.v_proj.weight"] = (kv, g.hidden)
        names[p + "self_attn.o_proj.weight"] = (g.hidden, g.hidden)
        names[p + "mlp.gate_proj.weight"] = (g.intermediate, g.hidden)
        names[p + "mlp.up_proj.weight"] = (g.intermediate, g.hidden)
        names[p + "mlp.down_proj.weight"] = (g.hidden, g.intermediate)
        if g.qkv_bias:
            names[p + "self_attn.q_proj.bias"] = (g.hidden,)
            names[p + "self_attn.k_proj.bias"] = (kv,)
            names[p + "self_attn.v_proj.bias"] = (kv,)
    return names


def random_weights(g: ModelGeometry, seed: int = 0, device="cuda", std: float = 0.02):
    """FP16 weights drawn N(0, std) (norm weights 1), seeded on the device."""
    import torch
    gen = torch.Generator(device=device).manual_seed(seed)
    out = {}
    for name, shape in weight_names(g).items():
        if name.endswith("norm.weight"):
            out[name] = torch.ones(shape, dtype=torch.float16, device=device)
        else:
            out[name] = (torch.randn(shape, device=device, generator=gen) * std).half()
    return out


class Decoder:
    """Decoder.create(weights, capacity, chunk, calibration) of decoder.ts:15-30 for a batch.

    tables: per (layer, KV head) Block-GTQ tables, layer-major (calibration.ts heads order),
    each a (config u32, table f32) pair in the reference's flattened format.
    compute: torch dtype of the activations and GEMMs (float32 mirrors the reference's FP32
    shaders; float16 runs the GEMMs on FP16 tensor cores with FP32 accumulation).
    fused: decode steps (one token per sequence, batch <= 8, FP16 weights, FP32 compute) run
    the library's fused weight-streaming kernels on the FP16 weights (bgtq_model_gemv):
    seven launches per layer instead of about a dozen torch / cuBLAS ones.
    step: eager fused decode steps of up to 4 sequences run the whole model as one persistent
    cooperative launch (bgtq_decoder_step) with grid barriers between the phases; a step
    recorded into a CUDA graph (capture_decode) takes the seven-launch path.

    Per layer: RMSNorm, one fused Q/K/V GEMM, one library call that applies RoPE to the new
    keys, encodes them into the packed stores and appends the FP16 values
    (bgtq_append_kv_rope), attention on the raw query projection with RoPE applied inside
    the query rotation (bgtq_attention_set_rope), the output projection fused with the
    residual add, RMSNorm, one fused gate/up GEMM, SiLU gating and the down projection fused
    with the residual add.
    """

    def __init__(self, weights, geometry: ModelGeometry, capacity: int, tables, batch: int = 1,
                 compute=None, device: int = 0, fused: bool = True, step: bool = True, step_ctas_per_sm: int = 0):
        import torch
        from . import _lib
        g = geometry
        if capacity < 1 or batch < 1:
            raise ValueError("Unsupported capacity/batch")
        if len(tables) != g.layers * g.kv_heads:
            raise ValueError("Calibration does not match model geometry")  # decoder.ts:17
        self.g, self.capacity, self.batch, self.length = g, int(capacity), int(batch), 0
        self.compute = compute or torch.float32
        self.dev = torch.device("cuda", device)
        # decode steps of a few sequences run the fused weight-streaming kernels on the FP16
        # weights (bgtq_model_gemv); they need FP16 checkpoints and FP32 compute
        self.fused = bool(fused) and self.compute == torch.float32 and batch <= 8 and all(
            v.dtype == torch.float16 for v in weights.values())
        if self.fused:
            w16 = {k: v.to(self.dev, torch.float16) for k, v in weights.items()}
        w = {k: v.to(self.dev, self.compute) for k, v in weights.items()}
        self.emb, self.final_norm = w["model.embed_tokens.weight"], w["model.norm.weight"]
        self.layers = []
        for layer in range(g.layers):
            p = f"model.layers.{layer}."
            qkv = torch.cat([w[p + f"self_attn.{n}.weight"] for n in ("q_proj", "k_proj", "v_proj")]).contiguous()
            bias = (torch.cat([w[p + f"self_attn.{n}.bias"] for n in ("q_proj", "k_proj", "v_proj")]).contiguous()
                    if g.qkv_bias else None)
            gate_up = torch.cat([w[p + "mlp.gate_proj.weight"], w[p + "mlp.up_proj.weight"]]).contiguous()
            self.layers.append(dict(ln1=w[p + "input_layernorm.weight"], ln2=w[p + "post_attention_layernorm.weight"],
                                    qkv=qkv, qkv_b=bias, o=w[p + "self_attn.o_proj.weight"], gate_up=gate_up,
                                    down=w[p + "mlp.down_proj.weight"]))
        self.layers16 = []
        if self.fused:
            for layer in range(g.layers):
                p = f"model.layers.{layer}."
                self.layers16.append(dict(
                    qkv=torch.cat([w16[p + f"self_attn.{n}.weight"] for n in ("q_proj", "k_proj", "v_proj")]).contiguous(),
                    o=w16[p + "self_attn.o_proj.weight"].contiguous(),
                    gate_up=torch.cat([w16[p + "mlp.gate_proj.weight"], w16[p + "mlp.up_proj.weight"]]).contiguous(),
                    down=w16[p + "mlp.down_proj.weight"].contiguous()))
            self.emb16 = w16["model.embed_tokens.weight"].contiguous()
            del w16
        del w
        pairs = g.head_dim // 2
        # inv_freq as the reference's rope kernel raises theta (kernels.wgsl:52), FP32
        self.inv_freq = torch.pow(torch.tensor(float(g.rope_theta), dtype=torch.float32),
                                  -torch.arange(pairs, dtype=torch.float32) / pairs).numpy()
        self.keys, self.values, self.attn = [], [], []
        for layer in range(g.layers):
            ks = [PackedKeys(tables[layer * g.kv_heads + h], capacity, sequences=batch, device=device)
                  for h in range(g.kv_heads)]
            vs = [Values(g.head_dim, capacity, "f16", sequences=batch, device=device) for _ in range(g.kv_heads)]
            att = GroupedAttention(ks, vs, g.gqa)
            _lib.call("bgtq_attention_set_rope", att._handle, self.inv_freq.ctypes.data, pairs)
            self.keys.append(ks)
            self.values.append(vs)
            self.attn.append(att)
        # eager decode steps of up to 4 sequences run as one persistent launch (bgtq_decoder_step)
        self.step_kernel = bool(step) and self.fused and batch <= 4
        self._step = None
        self._step_ctas_per_sm = int(step_ctas_per_sm)
        self._kv_ptrs = []
        import ctypes as C
        for layer in range(g.layers):
            kp = (C.c_void_p * g.kv_heads)(*[k._handle for k in self.keys[layer]])
            vp = (C.c_void_p * g.kv_heads)(*[v._handle for v in self.values[layer]])
            self._kv_ptrs.append((kp, vp))

    def _norm(self, x, w):
        import torch
        return torch.nn.functional.rms_norm(x, (self.g.hidden,), w, self.g.rms_eps)

    def forward(self, tokens, _check: bool = True):
        """decoder.ts:31-81 for a [batch, n] chunk: returns the last position's logits
        [batch, vocab] (FP32)."""
        import ctypes as C
        import torch
        import torch.nn.functional as F
        from . import _lib
        g = self.g
        tokens = torch.as_tensor(tokens, device=self.dev).reshape(self.batch, -1).long()
        B, n = tokens.shape
        if _check:
            self._sync_lengths()
            if n < 1 or self.length + n > self.capacity or int(tokens.max()) >= g.vocab or int(tokens.min()) < 0:
                raise ValueError("Invalid tokens/capacity")  # decoder.ts:33
        start = self.length
        st = torch.cuda.current_stream(self.dev).cuda_stream
        # the persistent step is one cooperative launch; a stream being recorded into a CUDA
        # graph takes the seven-launch path
        if n == 1 and self.step_kernel and not torch.cuda.is_current_stream_capturing():
            return self._decode_step(tokens, st)
        if n == 1 and self.fused:
            return self._decode_fused(tokens, st)
        qw, kvw = g.q_heads * g.head_dim, g.kv_heads * g.head_dim
        row = qw + 2 * kvw
        h = self.emb[tokens]                                             # [B, n, hidden]
        for layer, lw in enumerate(self.layers):
            x = self._norm(h, lw["ln1"])
            qkv = F.linear(x, lw["qkv"], lw["qkv_b"]).float().contiguous()   # [B, n, row]
            kp, vp = self._kv_ptrs[layer]
            _lib.call("bgtq_append_kv_rope", g.kv_heads, kp, vp, C.c_void_p(qkv.data_ptr()), row, n * row, qw,
                      qw + kvw, n, 0, B, self.inv_freq.ctypes.data, C.c_void_p(st))
            if n == 1:
                q = qkv[:, 0, :qw].reshape(B, g.kv_heads, g.gqa, g.head_dim).contiguous()
                att = self.attn[layer].attend(q)
            else:
                q = qkv[:, :, :qw].reshape(B, n, g.q_heads, g.head_dim).contiguous()
                att = self.attn[layer].prefill(q, start)
            att = att.reshape(B * n, g.hidden).to(self.compute)
            h = torch.addmm(h.reshape(B * n, g.hidden), att, lw["o"].t()).view(B, n, g.hidden)
            x = self._norm(h, lw["ln2"])
            gate, up = F.linear(x, lw["gate_up"]).chunk(2, dim=-1)
            act = (F.silu(gate) * up).reshape(B * n, -1)
            h = torch.addmm(h.reshape(B * n, g.hidden), act, lw["down"].t()).view(B, n, g.hidden)
        last = self._norm(h[:, -1], self.final_norm)
        self.length += n
        return (last @ self.emb.t()).float()

    def _step_handle(self):
        """The persistent decode step (bgtq_decoder_create) over this decoder's FP16 weights,
        FP32 norms / bias / embedding and per-layer stores, created on first use."""
        if self._step is None:
            import ctypes as C
            from . import _lib
            g, L = self.g, self.g.layers

            def arr(ts):
                return (C.c_void_p * L)(*[None if t is None else t.data_ptr() for t in ts])

            keep = dict(ln1=arr([lw["ln1"] for lw in self.layers]), ln2=arr([lw["ln2"] for lw in self.layers]),
                        bias=arr([lw["qkv_b"] for lw in self.layers]) if g.qkv_bias else None,
                        qkv=arr([l16["qkv"] for l16 in self.layers16]), o=arr([l16["o"] for l16 in self.layers16]),
                        gu=arr([l16["gate_up"] for l16 in self.layers16]),
                        down=arr([l16["down"] for l16 in self.layers16]),
                        att=(C.c_void_p * L)(*[a._handle.value for a in self.attn]))
            ad = {k: (None if v is None else C.addressof(v)) for k, v in keep.items()}
            desc = _lib.DecoderDesc(L, self.batch, g.hidden, g.q_heads, g.kv_heads, g.head_dim, g.intermediate,
                                    g.vocab, g.rms_eps, self.inv_freq.ctypes.data, ad["ln1"], ad["bias"], ad["ln2"],
                                    ad["qkv"], ad["o"], ad["gu"], ad["down"], self.final_norm.data_ptr(),
                                    self.emb16.data_ptr(), self.emb.data_ptr(), ad["att"], self._step_ctas_per_sm)
            h = C.c_void_p()
            _lib.call("bgtq_decoder_create", C.byref(desc), C.byref(h))
            self._step = h
            import torch
            self._step_h = torch.empty((self.batch, g.hidden), device=self.dev, dtype=torch.float32)
        return self._step

    def step_info(self):
        """(CTAs, dynamic shared memory bytes, staged encode-table bytes) of the persistent
        decode step."""
        import ctypes as C
        from . import _lib
        n, smem, tab = C.c_uint32(), C.c_uint32(), C.c_uint32()
        _lib.call("bgtq_decoder_info", self._step_handle(), C.byref(n), C.byref(smem), C.byref(tab))
        return n.value, smem.value, tab.value

    def step_trace(self, on: bool = True):
        """Phase timing of the persistent step (bgtq_decoder_trace): switches recording on or
        off and returns the last traced step's stamps (ns, CTA 0's global timer: start, the
        end of each layer's five phases, the end of the lm_head) as a uint64 array."""
        import ctypes as C
        from . import _lib
        n = C.c_uint32()
        out = np.zeros(2 + 5 * self.g.layers, np.uint64)
        _lib.call("bgtq_decoder_trace", self._step_handle(), int(bool(on)), out.ctypes.data, len(out), C.byref(n))
        return out

    def _decode_step(self, tokens, st):
        """One token per sequence as one persistent launch (bgtq_decoder_step): the embedding
        rows, every layer and the lm_head; the same arithmetic as _decode_fused."""
        import ctypes as C
        import torch
        from . import _lib
        handle = self._step_handle()
        tok = tokens[:, 0].contiguous()
        logits = torch.empty((self.batch, self.g.vocab), device=self.dev, dtype=torch.float32)
        _lib.call("bgtq_decoder_step", handle, C.c_void_p(tok.data_ptr()), C.c_void_p(self._step_h.data_ptr()),
                  C.c_void_p(logits.data_ptr()), C.c_void_p(st))
        self.length += 1
        return logits

    def close(self):
        """Releases the persistent step (the stores and weights go with the object)."""
        from . import _lib
        if getattr(self, "_step", None) is not None:
            _lib.lib().bgtq_decoder_destroy(self._step)
            self._step = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _decode_fused(self, tokens, st):
        """One token per sequence through the fused decode kernels: per layer RMSNorm + Q/K/V
        (+ bias) in one GEMV, the RoPE + encode + V append launch, attention, o_proj with the
        residual add, RMSNorm + gate/up + SiLU gating in one GEMV, down_proj with the residual
        add; then the final RMSNorm + tied lm_head in one GEMV (decoder.ts:31-81,
        kernels.wgsl:11-54)."""
        import ctypes as C
        import torch
        from . import _lib
        g = self.g
        B = tokens.shape[0]
        qw, kvw = g.q_heads * g.head_dim, g.kv_heads * g.head_dim
        row = qw + 2 * kvw
        h = self.emb[tokens[:, 0]].contiguous()                         # [B, hidden] residual stream
        qkv = torch.empty((B, row), device=self.dev, dtype=torch.float32)
        act = torch.empty((B, g.intermediate), device=self.dev, dtype=torch.float32)
        sp = C.c_void_p(st)

        def gemv(mode, x, in_dim, norm, w16, bias, out_dim, y):
            _lib.call("bgtq_model_gemv", mode, C.c_void_p(x.data_ptr()), B, x.stride(0), in_dim,
                      None if norm is None else C.c_void_p(norm.data_ptr()), C.c_float(g.rms_eps),
                      C.c_void_p(w16.data_ptr()), None if bias is None else C.c_void_p(bias.data_ptr()), out_dim,
                      C.c_void_p(y.data_ptr()), y.stride(0), sp)

        for layer, (lw, l16) in enumerate(zip(self.layers, self.layers16)):
            gemv(0, h, g.hidden, lw["ln1"], l16["qkv"], lw["qkv_b"], row, qkv)
            kp, vp = self._kv_ptrs[layer]
            _lib.call("bgtq_append_kv_rope", g.kv_heads, kp, vp, C.c_void_p(qkv.data_ptr()), row, row, qw,
                      qw + kvw, 1, 0, B, self.inv_freq.ctypes.data, sp)
            q = qkv[:, :qw].reshape(B, g.kv_heads, g.gqa, g.head_dim).contiguous()
            att = self.attn[layer].attend(q).reshape(B, g.hidden)
            gemv(1, att, g.hidden, None, l16["o"], None, g.hidden, h)
            gemv(2, h, g.hidden, lw["ln2"], l16["gate_up"], None, g.intermediate, act)
            gemv(1, act, g.intermediate, None, l16["down"], None, g.hidden, h)
        logits = torch.empty((B, g.vocab), device=self.dev, dtype=torch.float32)
        gemv(0, h, g.hidden, self.final_norm, self.emb16, None, g.vocab, logits)
        self.length += 1
        return logits

    def prefill(self, tokens, chunk: int | None = None):
        """decoder.ts:82: the prompt in chunks; returns the last chunk's logits."""
        import torch
        tokens = torch.as_tensor(tokens, device=self.dev).reshape(self.batch, -1)
        n = tokens.shape[1]
        chunk = n if chunk is None else int(chunk)
        if n < 1:
            raise ValueError("Empty prompt")
        out = None
        for i in range(0, n, chunk):
            out = self.forward(tokens[:, i:i + chunk])
        return out

    def decode(self, token):
        """decoder.ts:83: one token per sequence."""
        return self.forward(token)

    # ---- CUDA graph of one decode step ----
    def capture_decode(self, token, jit_wait_s=300.0):
        """Decode `token` eagerly, then record the whole decode step (every layer's GEMMs,
        norms, K/V append and attention) as one CUDA graph; decode_graph() replays it.
        Attention plans its split-KV factor for the capacity, so replays stay exact while
        the sequences grow; appends inside replays move the device lengths only.  The
        layout-specialised attention kernels the eager step queued are waited for (up to
        `jit_wait_s`) and loaded first, so the graph records them."""
        import torch
        from . import _lib, layout_jit_wait
        for a in self.attn:
            _lib.call("bgtq_attention_plan_for_capacity", a._handle, 1)
        # the eager step runs the launches the graph will record (not the persistent step), so
        # every kernel they use - the layout-specialised attention kernels above all - is
        # loaded before the capture
        step, self.step_kernel = self.step_kernel, False
        try:
            out = self.forward(token)                  # eager step: warms every kernel up
        finally:
            self.step_kernel = step
        torch.cuda.synchronize(self.dev)
        layout_jit_wait(jit_wait_s)
        self._tok = torch.as_tensor(token, device=self.dev).reshape(self.batch, 1).long().clone()
        self._graph = torch.cuda.CUDAGraph()
        length = self.length
        with torch.cuda.graph(self._graph):
            self._logits = self.forward(self._tok, _check=False)
        self.length = length                           # recording appended nothing
        self._host_stale = True
        self._sync_lengths()
        return out

    def decode_graph(self, token):
        """Replay the recorded decode step for `token` [batch, 1]; returns the graph's
        logits buffer (overwritten by the next replay)."""
        if self.length + 1 > self.capacity:
            raise ValueError("Invalid tokens/capacity")
        self._tok.copy_(token.reshape(self.batch, 1))
        self._graph.replay()
        self.length += 1
        self._host_stale = True
        return self._logits

    def _sync_lengths(self):
        from . import _lib
        if getattr(self, "_host_stale", False):
            for ks, vs in zip(self.keys, self.values):
                for k in ks:
                    _lib.call("bgtq_keys_sync_lengths", k._handle)
                for v in vs:
                    _lib.call("bgtq_values_sync_lengths", v._handle)
            self._host_stale = False

    def destroy(self):
        self.close()
        self._graph = None
        for a in self.attn:
            a.destroy()
        for layer in self.keys + self.values:
            for o in layer:
                o.destroy()
