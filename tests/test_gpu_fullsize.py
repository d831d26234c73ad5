"""Config 4 at its full per-GPU size (256 sequences x 32768 cached tokens, 3 KV heads,
GQA 3, head_dim 64, FP16 V) through the C ABI, checked by properties that do not need an
oracle run over the whole batch:

- sampled (sequence, head) pairs equal the oracle on the GPU's own codes (1e-5 / 1e-4);
- the output does not depend on the split-KV partition;
- with every V row equal to one vector u, every output row is u (softmax weights sum to 1);
- causal rows at early positions ignore everything after them.
"""
import numpy as np
import pytest

import oracle
from bgtq import GroupedAttention, PackedKeys, Values, device_status, synthetic
from conftest import load_config, params_tables

pytestmark = pytest.mark.gpu
ATOL, RTOL = 1e-5, 1e-4
B, T, H, R, D = 256, 32768, 3, 3, 64
SAMPLED = (0, 7, 131, 255)


@pytest.fixture(scope="module")
def batch(cuda):
    import torch
    z = load_config("config4")
    p, cfg, tab = params_tables(z)
    g = torch.Generator(device=cuda).manual_seed(44)
    sig = torch.from_numpy(synthetic.pair_sigma(D // 2).astype(np.float32)).to(cuda)
    keys, vals, consts = [], [], []
    vhost = {}  # (sequence, head) -> FP16 V rows of the sampled sequences, kept on the host
    u = torch.randn(D, device=cuda, generator=g).half()
    for h in range(H):
        k = PackedKeys((cfg, tab), T, sequences=B)
        v = Values(D, T, "f16", sequences=B)
        c = Values(D, T, "f16", sequences=B)
        for s0 in range(0, B, 32):
            blk = torch.randn((32, T, D // 2, 2), device=cuda, generator=g) * sig[None, None, :, None]
            k.append(torch.cat([blk[..., 0], blk[..., 1]], -1).half(), seq_first=s0)
            vb = torch.randn((32, T, D), device=cuda, generator=g).half()
            v.append(vb, seq_first=s0)
            for s in SAMPLED:
                if s0 <= s < s0 + 32:
                    vhost[(s, h)] = vb[s - s0].float().cpu().numpy()
            c.append(u.expand(32, T, D).contiguous(), seq_first=s0)
        keys.append(k)
        vals.append(v)
        consts.append(c)
    q = torch.randn((B, H, R, D), device=cuda, generator=g)
    yield dict(cfg=cfg, tab=tab, keys=keys, vals=vals, consts=consts, q=q, u=u, vhost=vhost)
    for objs in (keys, vals, consts):
        for o in objs:
            o.destroy()


def test_sampled_pairs_match_oracle_and_splits_agree(batch):
    att = GroupedAttention(batch["keys"], batch["vals"], R)
    q = batch["q"]
    outs = {}
    for splits in (0, 1, 7):
        att.set_splits(splits)
        outs[splits] = att.attend(q).cpu().numpy()
    qh = q.cpu().numpy()
    for s in SAMPLED:
        for h in range(H):
            kh = oracle.reconstruct(batch["cfg"], batch["tab"], *batch["keys"][h].read(s), threads=8)
            _, _, ref = oracle.attention(qh[s, h], kh, batch["vhost"][(s, h)], None, False, threads=8)
            np.testing.assert_allclose(outs[0][s, h], ref, atol=ATOL, rtol=RTOL)
    for splits in (1, 7):
        np.testing.assert_allclose(outs[splits], outs[0], atol=ATOL, rtol=RTOL)
    assert device_status(0) == 0


def test_constant_values_give_their_vector(batch):
    att = GroupedAttention(batch["keys"], batch["consts"], R)
    out = att.attend(batch["q"]).cpu().numpy()
    u = batch["u"].float().cpu().numpy()
    # FP32 sums over 32768 tokens (P split into FP16 halves for the MMA): ~2e-5 relative
    np.testing.assert_allclose(out, np.broadcast_to(u, out.shape), atol=ATOL, rtol=RTOL)


def test_causal_rows_ignore_later_tokens(batch):
    import torch
    att = GroupedAttention(batch["keys"], batch["vals"], R)
    pos = np.tile(np.array([0, 4095, T - 1], np.uint32), (B, 1))
    pos_dev = torch.from_numpy(pos).to(batch["q"].device)
    full = att.attend(batch["q"], pos_dev, True).cpu().numpy()
    # row 0 sees only token 0: its output is that token's value row
    for h in range(H):
        v0 = batch["vhost"][(7, h)][0]
        np.testing.assert_allclose(full[7, h, 0], v0, atol=ATOL, rtol=RTOL)
    # row 2 at the last position equals the non-causal result
    nc = att.attend(batch["q"]).cpu().numpy()
    np.testing.assert_allclose(full[:, :, 2], nc[:, :, 2], atol=ATOL, rtol=RTOL)
    torch.cuda.synchronize()
