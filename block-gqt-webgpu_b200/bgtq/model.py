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
    """

    def __init__(self, weights, geometry: ModelGeometry, capacity: int, tables, batch: int = 1,
                 compute=None, device: int = 0):
        import torch
        g = geometry
        if capacity < 1 or batch < 1:
            raise ValueError("Unsupported capacity/batch")
        if len(tables) != g.layers * g.kv_heads:
            raise ValueError("Calibration does not match model geometry")  # decoder.ts:17
        self.g, self.capacity, self.batch, self.length = g, int(capacity), int(batch), 0
        self.compute = compute or torch.float32
        self.dev = torch.device("cuda", device)
        self.w = {k: v.to(self.dev, self.compute) for k, v in weights.items()}
        self.keys, self.values, self.attn = [], [], []
        for layer in range(g.layers):
            ks = [PackedKeys(tables[layer * g.kv_heads + h], capacity, sequences=batch, device=device)
                  for h in range(g.kv_heads)]
            vs = [Values(g.head_dim, capacity, "f16", sequences=batch, device=device) for _ in range(g.kv_heads)]
            self.keys.append(ks)
            self.values.append(vs)
            self.attn.append(GroupedAttention(ks, vs, g.gqa))
        pairs = g.head_dim // 2
        self.inv_freq = torch.pow(torch.tensor(float(g.rope_theta), device=self.dev),
                                  -torch.arange(pairs, device=self.dev, dtype=torch.float32) / pairs)

    # ---- kernels.wgsl equivalents ----
    def _norm(self, x, w):
        import torch
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.g.rms_eps)
        return (y * w.float()).to(self.compute)

    def _lin(self, x, name, bias=None):
        import torch
        y = x @ self.w[name].t()
        if bias is not None:
            y = y + self.w[bias]
        return y

    def _rope(self, x, start):
        """Split-half RoPE (kernels.wgsl:49-54): pair p of head h rotates dims p and p + d/2
        by (start + row) * theta^(-p / (d/2))."""
        import torch
        n = x.shape[1]
        pos = torch.arange(start, start + n, device=self.dev, dtype=torch.float32)
        ang = pos[:, None] * self.inv_freq[None, :]                     # [n, d/2]
        c, s = torch.cos(ang)[None, :, None, :], torch.sin(ang)[None, :, None, :]
        xf = x.float()
        a, b = xf[..., : self.g.head_dim // 2], xf[..., self.g.head_dim // 2:]
        return torch.cat([a * c - b * s, b * c + a * s], dim=-1)

    def forward(self, tokens):
        """decoder.ts:31-81 for a [batch, n] chunk: returns the last position's logits
        [batch, vocab] (FP32)."""
        import torch
        g = self.g
        tokens = torch.as_tensor(tokens, device=self.dev).reshape(self.batch, -1).long()
        B, n = tokens.shape
        if n < 1 or self.length + n > self.capacity or int(tokens.max()) >= g.vocab or int(tokens.min()) < 0:
            raise ValueError("Invalid tokens/capacity")  # decoder.ts:33
        start = self.length
        h = self.w["model.embed_tokens.weight"][tokens]                  # [B, n, hidden]
        for layer in range(g.layers):
            p = f"model.layers.{layer}."
            x = self._norm(h, self.w[p + "input_layernorm.weight"])
            bias = (lambda name: p + f"self_attn.{name}.bias") if g.qkv_bias else (lambda name: None)
            q = self._lin(x, p + "self_attn.q_proj.weight", bias("q_proj")).view(B, n, g.q_heads, g.head_dim)
            k = self._lin(x, p + "self_attn.k_proj.weight", bias("k_proj")).view(B, n, g.kv_heads, g.head_dim)
            v = self._lin(x, p + "self_attn.v_proj.weight", bias("v_proj")).view(B, n, g.kv_heads, g.head_dim)
            qr = self._rope(q, start)                                    # FP32 [B, n, Hq, d]
            kr = self._rope(k, start)
            vf = v.float()
            for hd in range(g.kv_heads):
                self.keys[layer][hd].append(kr[:, :, hd, :], seq_first=0)     # encode from FP32
                self.values[layer][hd].append(vf[:, :, hd, :], seq_first=0)   # FP32 -> FP16
            if n == 1:
                att = self.attn[layer].attend(qr.view(B, g.kv_heads, g.gqa, g.head_dim).contiguous())
            else:
                att = self.attn[layer].prefill(qr.contiguous(), start)
            att = att.reshape(B, n, g.hidden).to(self.compute)
            h = h + self._lin(att, p + "self_attn.o_proj.weight")
            x = self._norm(h, self.w[p + "post_attention_layernorm.weight"])
            gate = self._lin(x, p + "mlp.gate_proj.weight")
            up = self._lin(x, p + "mlp.up_proj.weight")
            h = h + self._lin(torch.nn.functional.silu(gate) * up, p + "mlp.down_proj.weight")
        last = self._norm(h[:, -1], self.w["model.norm.weight"])
        self.length += n
        return (last @ self.w["model.embed_tokens.weight"].t()).float()

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

    def destroy(self):
        for objs in (self.attn,):
            for a in objs:
                a.destroy()
        for layer in self.keys + self.values:
            for o in layer:
                o.destroy()
