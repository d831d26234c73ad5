"""Frozen Block-GTQ tables for the Qwen2.5-0.5B geometry (benchmark configs 3 and 5).

The reference's Qwen calibration is not part of its checkout (``models/qwen2.5-0.5b/`` is
git-ignored there), so this script runs the reference's calibration procedure
(``tests/oracles/calibrate_model.py:29-38``) on the random-init model of that geometry and
freezes the result:

1. the model: HuggingFace ``Qwen2ForCausalLM`` built from the geometry (24 layers, hidden
   896, 14 / 2 heads, head_dim 64, MLP 4864, RoPE theta 1e6, RMSNorm eps 1e-6, vocab
   151936, QKV bias, tied embeddings) with the seeded random-init weights of
   ``bgtq.model.random_weights(QWEN25_05B, seed=0)`` (FP16 N(0, 0.02), norms 1), run in FP32
   on the CPU;
2. the calibration input: 128 token ids drawn uniformly with NumPy ``default_rng(0)`` (no
   tokenizer or text corpus ships here; the reference feeds its calibration paragraph);
3. forward hooks on every layer's ``q_proj`` / ``k_proj`` (pre-RoPE, bias included), as
   ``calibrate_model.py:22-26`` does;
4. per (layer, KV head): the pair energies of the head's grouped Q rows and its K rows
   (the reference's vendored ``compute_freq_importance_energy``,
   ``vendor/blockgtq-calibration/freq_analysis.py:18-35``, over ``decompose_freq_blocks``),
   widths = ``greedy_bit_allocation(scores, 128, 1, 8)`` (``vendor/blockgtq/allocator.py``),
   tables = the reference's ``production_oracle`` setup / pack_meta / code_lut with rotation
   threshold 2 (``calibrate_model.py:33-41``).

Written: ``qwen_calibration.npz`` with, per head (layer-major, 48 heads): the widths, the
pair order the reference's setup chose, the scores, the scale stride (= groups) and row
padding (0), and the SHA-256 of the reference-built ``config`` (u32) and ``table`` (f32) in
the flattened format of ``src/webgpu/layout.ts:24-31``.  The library's native builder
(``bgtq_tables_build``) must reproduce those bytes from the widths and pair order
(``tests/test_builder.py``); the benches and tests build the tables that way.

    python tests/golden/make_qwen_calibration.py --reference <path to block-gqt-webgpu>
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO / "block-gqt-webgpu_b200"))

TOKENS, SEED, BUDGET, ROTATION_THRESHOLD = 128, 0, 128, 2


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def vendor(ref_root: Path, name: str):
    path = ref_root / "vendor" / "blockgtq-calibration" / f"{name}.py"
    spec = importlib.util.spec_from_file_location(name, path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def hf_model(g, weights, torch):
    from transformers import Qwen2Config, Qwen2ForCausalLM
    cfg = Qwen2Config(vocab_size=g.vocab, hidden_size=g.hidden, intermediate_size=g.intermediate,
                      num_hidden_layers=g.layers, num_attention_heads=g.q_heads, num_key_value_heads=g.kv_heads,
                      rms_norm_eps=g.rms_eps, rope_theta=g.rope_theta, tie_word_embeddings=True,
                      max_position_embeddings=4096, hidden_act="silu", attention_dropout=0.0)
    cfg._attn_implementation = "eager"
    model = Qwen2ForCausalLM(cfg).float().eval()
    state = {k: v.float() for k, v in weights.items()}
    state["lm_head.weight"] = state["model.embed_tokens.weight"]
    missing, unexpected = model.load_state_dict(state, strict=False)
    assert not unexpected and all("rotary" in m for m in missing), (missing, unexpected)
    return model


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    args = ap.parse_args()
    ref_root = args.reference.resolve()
    os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
    sys.dont_write_bytecode = True
    sys.path[:0] = [str(ref_root / "src"), str(ref_root)]
    import torch
    torch.set_num_threads(8)
    from tests.oracles import production_oracle as oracle
    from tests.oracles.oracle import load
    from bgtq.model import QWEN25_05B, random_weights

    g = QWEN25_05B
    model = hf_model(g, random_weights(g, seed=0, device="cpu"), torch)
    ids = np.random.default_rng(SEED).integers(0, g.vocab, TOKENS)
    qs, ks, hooks = {}, {}, []
    for i, layer in enumerate(model.model.layers):
        hooks.append(layer.self_attn.q_proj.register_forward_hook(lambda m, a, o, i=i: qs.__setitem__(i, o.detach())))
        hooks.append(layer.self_attn.k_proj.register_forward_hook(lambda m, a, o, i=i: ks.__setitem__(i, o.detach())))
    with torch.no_grad():
        model(torch.from_numpy(ids)[None], use_cache=False)
    for h in hooks:
        h.remove()

    freq, rope = vendor(ref_root, "freq_analysis"), vendor(ref_root, "rope_utils")
    gqa = g.q_heads // g.kv_heads
    rows = {k: [] for k in ("widths", "pair_order", "scores", "norm_stride", "row_pad", "layer", "kv_head",
                            "config_sha256", "table_sha256")}
    for layer in range(g.layers):
        for head in range(g.kv_heads):
            q = qs[layer].reshape(-1, g.q_heads, 64)[:, head * gqa:(head + 1) * gqa].reshape(-1, 64)
            k = ks[layer].reshape(-1, g.kv_heads, 64)[:, head]
            scores = freq.compute_freq_importance_energy(rope.decompose_freq_blocks(q, 64),
                                                         rope.decompose_freq_blocks(k, 64))
            widths = load("allocator").greedy_bit_allocation(scores, BUDGET, 1, 8)
            p = oracle.setup(widths)
            pm = oracle.pack_meta(widths, p._head_perm)
            assert torch.equal(pm["pack_perm"], torch.arange(64))
            lut, cb, offsets, inv = oracle.code_lut(p)
            ng = p._n_groups
            row = pm["nopack_start"] // 2 + pm["nopack_len"]
            config = [64, ng, row, ng, pm["nopack_start"], p._pos_centroids.shape[1], 0, 0, 0, 0]
            for slot, values in [(6, p._head_perm), (7, p._group_of), (8, cb), (9, lut.flatten())]:
                config[slot] = len(config)
                config.extend(values.tolist())
            table = torch.cat([p._block_rot_T.T.contiguous().flatten(), p._pos_centroids.flatten(), offsets, inv])
            perm = p._head_perm.numpy()
            rows["widths"].append(widths.numpy().astype(np.int8))
            rows["pair_order"].append(perm[0::2].astype(np.int16))
            rows["scores"].append(scores.numpy().astype(np.float32))
            rows["norm_stride"].append(ng)
            rows["row_pad"].append(0)
            rows["layer"].append(layer)
            rows["kv_head"].append(head)
            rows["config_sha256"].append(sha(np.asarray(config, np.uint32)))
            rows["table_sha256"].append(sha(table.numpy().astype(np.float32)))
    out = {k: np.asarray(v) for k, v in rows.items()}
    out["rotation_threshold"] = np.int32(ROTATION_THRESHOLD)
    out["calibration_ids"] = ids.astype(np.int64)
    out["weights_seed"] = np.int64(0)
    out["norm_stride"] = out["norm_stride"].astype(np.int32)
    out["row_pad"] = out["row_pad"].astype(np.int32)
    out["layer"] = out["layer"].astype(np.int32)
    out["kv_head"] = out["kv_head"].astype(np.int32)
    np.savez_compressed(HERE / "qwen_calibration.npz", **out)
    print(f"{len(rows['widths'])} Qwen heads written to {HERE / 'qwen_calibration.npz'}; "
          f"mean groups {np.mean(out['norm_stride']):.2f}")


if __name__ == "__main__":
    main()
