"""Vectorised PyTorch restatement of the reference's CPU path - TEST INFRASTRUCTURE ONLY.

The reference's own CPU implementation of this path is PyTorch code
(``src/reference/production_math.py:4-31``, ``src/reference/mixed_layout.py:21-37``,
``src/reference/attention.py:5-22``): whole-batch tensor operations (a permutation gather,
masked group norms, one ``normalized @ rotation.T`` GEMM, LUT gathers; reconstruction as
a centroid gather, scale and ``@ rotation`` GEMM; attention as ``q @ k.T``, softmax,
``@ v``).  That checkout does not exist on the GPU box, so ``bench.py``'s reference arm and
CPU baseline time this restatement of it - the same tensor operations on the same shapes,
written here from the reference's description - with every host thread.  Its encode
divides each group by its own norm (as the GPU encoder and the WGSL shader do) where the
reference's emulator averages repeated per-position norms; the work is the same.

Tables come in the reference's flattened ``tables()`` format (``src/webgpu/layout.ts:24-31``):
u32 config = [d, groups, row_bytes, norm_stride, nibble_dims, max_centroids, offsets of
perm / group_of / pos_to_cb / code LUT, ...], f32 table = rotation [d][d], centroids
[d][maxC], LUT offsets [d], LUT inverse scales [d].

``tests/test_oracle.py`` checks it against the C oracle (codes, scales, outputs).
"""
from __future__ import annotations

import math

import numpy as np


class Tables:
    def __init__(self, config, table):
        import torch
        c = np.asarray(config, np.uint32)
        t = np.asarray(table, np.float32)
        d, ng, self.row_bytes, self.norm_stride, self.ns, maxc = (int(x) for x in c[:6])
        self.d, self.ng = d, ng
        self.perm = torch.from_numpy(c[c[6]:c[6] + d].astype(np.int64))
        self.inv_perm = torch.argsort(self.perm)
        self.group_of = torch.from_numpy(c[c[7]:c[7] + d].astype(np.int64))
        self.pos_to_cb = torch.from_numpy(c[c[8]:c[8] + d].astype(np.int64))
        ncb = (len(c) - int(c[9])) // 256
        self.lut = torch.from_numpy(c[c[9]:c[9] + ncb * 256].astype(np.int64).reshape(ncb, 256))
        o = 0
        self.rotation = torch.from_numpy(t[o:o + d * d].reshape(d, d).copy()); o += d * d
        self.centroids = torch.from_numpy(t[o:o + d * maxc].reshape(d, maxc).copy()); o += d * maxc
        self.offsets = torch.from_numpy(t[o:o + d].copy()); o += d
        self.inv_scales = torch.from_numpy(t[o:o + d].copy())
        self.masks = [self.group_of == g for g in range(ng)]
        self.dims = torch.arange(d)


def encode(tb: Tables, k_fp16_bits):
    """codes [n, d] uint8 (pack order = dimension order), FP16 scales [n, groups]."""
    import torch
    x = torch.from_numpy(np.asarray(k_fp16_bits, np.uint16).view(np.float16).astype(np.float32))
    xp = x[:, tb.perm]
    norms = torch.zeros(len(x), tb.ng)
    normalized = torch.zeros_like(xp)
    for g, m in enumerate(tb.masks):
        n = ((xp * xp) * m).sum(1).add(1e-30).sqrt()
        norms[:, g] = n
        normalized[:, m] = xp[:, m] / torch.where(n > 1e-10, n, 1.0)[:, None]
    y = normalized @ tb.rotation.T.contiguous()
    bins = ((y - tb.offsets) * tb.inv_scales).clamp(0, 255).long()
    codes = tb.lut[tb.pos_to_cb[None, :], bins]
    cents = tb.centroids[tb.dims[None, :], codes]
    scales = norms.clone()
    for g, m in enumerate(tb.masks):
        scales[:, g] /= ((cents * cents) * m).sum(1).sqrt().clamp(min=1e-10)
    return codes.to(torch.uint8), scales.half()


def pack(tb: Tables, codes):
    c = np.asarray(codes, np.uint8)
    out = np.zeros((len(c), tb.row_bytes), np.uint8)
    ns = tb.ns
    out[:, :ns // 2] = (c[:, :ns:2] & 15) | ((c[:, 1:ns:2] & 15) << 4)
    out[:, ns // 2:ns // 2 + tb.d - ns] = c[:, ns:]
    return out


def unpack(tb: Tables, packed):
    p = np.asarray(packed, np.uint8)
    c = np.zeros((len(p), tb.d), np.uint8)
    ns = tb.ns
    c[:, :ns:2] = p[:, :ns // 2] & 15
    c[:, 1:ns:2] = p[:, :ns // 2] >> 4
    c[:, ns:] = p[:, ns // 2:ns // 2 + tb.d - ns]
    return c


def reconstruct(tb: Tables, packed, scale_bits):
    """FP32 keys [n, d] in the original dimension order from packed rows and FP16 scales."""
    import torch
    codes = torch.from_numpy(unpack(tb, packed)).long()
    s = torch.from_numpy(np.asarray(scale_bits, np.uint16)[:, :tb.ng].view(np.float16).astype(np.float32))
    y = tb.centroids[tb.dims[None, :], codes] * s[:, tb.group_of]
    return (y @ tb.rotation)[:, tb.inv_perm]


def attention(q, k, v, positions=None, causal=False):
    """(logits, probabilities, output) of softmax(q k^T / sqrt(d)) v, causal mask t > position."""
    import torch
    q = torch.as_tensor(np.asarray(q, np.float32))
    v = torch.as_tensor(np.asarray(v, np.float32))
    logits = (q @ k.T) / math.sqrt(k.shape[1])
    if causal:
        pos = torch.as_tensor(np.asarray(positions, np.int64))
        logits = logits.masked_fill(torch.arange(len(k))[None, :] > pos[:, None], -torch.inf)
    p = torch.softmax(logits, dim=-1)
    return logits, p, p @ v
