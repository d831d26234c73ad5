"""Generate the golden vectors under tests/golden/ from the reference implementation.

Run in a container that has the reference checkout (it is not needed afterwards):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --reference <path to block-gqt-webgpu>

What it writes, all derived from the reference's own Python CPU code and fixtures:

* ``mixed/<case>.npz`` - the ten encoder fixtures of ``fixtures/mixed`` (tables as
  ``BlockGTQParameters`` fields plus inputs, codes, raw/corrected scales, FP16 scale bits,
  packed rows and reconstructions), re-saved from ``tests/oracles/export_mixed.py`` output.
* ``attention/t<T>_d<d>.npz`` - the six attention fixtures of ``fixtures/attention``
  (``tests/oracles/export_attention.py``): Q, FP16 K, FP32 V, positions, packed K, FP16
  scales, reconstructed K and the logits / probabilities / outputs for the FP16-K,
  compressed-K and FP32-source paths, causal and not.
* ``allocator.json`` - the allocator golden cases of ``fixtures/allocator.json``.
* ``config1.npz`` / ``config4.npz`` - tables built by the reference's table code
  (``tests/oracles/production_oracle.py`` over the hash-pinned upstream
  ``BlockGTQPipeline._post_allocation_setup`` / ``build_code_lut`` / ``build_pack_meta``)
  from allocator widths for the synthetic pair-energy profile, plus the reference
  encoder's codes / scales for a key sample and, for config 1, reference attention
  outputs over all 4096 keys.  Inputs come from NumPy PCG64 (``bgtq.synthetic``), so the
  tests regenerate them bit-identically; their SHA-256 is stored beside the outputs.
* ``smollm2_heads.npz`` - the flattened ``config`` / ``table`` / ``ranges`` of the first
  six SmolLM2 calibration heads from ``fixtures/model/calibration.json`` (format check).
* ``smollm2_calibration.npz`` - all 90 heads of that calibration (30 layers x 3 KV heads) as
  table-builder inputs - widths, pair order, row padding, scale stride - with the SHA-256 of
  each head's reference ``config`` and ``table`` (``--only calibration`` writes just this).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO / "block-gqt-webgpu_b200"))

from bgtq import synthetic  # noqa: E402

PARAM_KEYS = ("head_perm", "group_of", "pos_to_cb", "code_lut", "rotation", "centroids",
              "lut_offsets", "lut_inv_scales")


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def save(path: Path, **arrays):
    path.parent.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(path, **arrays)


def params_from_fixture(meta, a):
    return dict(dim=np.int64(meta["dim"]), groups=np.int64(meta["n_groups"]),
                row_bytes=np.int64(meta["row_bytes"]), norm_stride=np.int64(meta["norm_stride"]),
                nibble_dims=np.int64(meta["nopack_start"]), max_centroids=np.int64(meta["max_centroids"]),
                logical_row_bytes=np.int64(meta["logical_row_bytes"]),
                permutation=a["head_perm"].astype(np.uint32), group_of=a["group_of"].astype(np.uint32),
                position_to_codebook=a["pos_to_cb"].astype(np.uint32), code_lut=a["code_lut"].astype(np.uint8).reshape(-1),
                rotation=a["rotation"].astype(np.float32).reshape(-1), centroids=a["centroids"].astype(np.float32).reshape(-1),
                offsets=a["lut_offsets"].astype(np.float32), inverse_scales=a["lut_inv_scales"].astype(np.float32))


def export_mixed(ref_root, read_fixture):
    index = json.loads((ref_root / "fixtures/mixed/index.json").read_text())
    for case in index["cases"]:
        meta, a = read_fixture(ref_root / f"fixtures/mixed/{case['name']}.json")
        p = params_from_fixture(meta, a)
        save(HERE / "mixed" / f"{case['name']}.npz", **p,
             allocation=a["allocation"].astype(np.uint32), pack_perm=a["pack_perm"].astype(np.uint32),
             rows=np.int64(meta["rows"]), capacity=np.int64(meta["capacity"]),
             original=a["original"], codes=a["codes"], raw_norms=a["raw_norms"], corrected_f32=a["corrected_f32"],
             norm_bits=a["norm_bits"], packed=a["packed"], rotated=a["rotated"],
             reconstructed_f32=a["reconstructed_f32"], reconstructed_f16=a["reconstructed_f16"],
             cache_packed=a["cache_packed"], cache_norm_bits=a["cache_norms"].view(np.uint16))


def export_attention(ref_root, read_fixture):
    index = json.loads((ref_root / "fixtures/attention/index.json").read_text())
    for case in index["cases"]:
        meta, a = read_fixture(ref_root / f"fixtures/attention/{case['name']}.json")
        out = {k: v for k, v in a.items() if k not in ("k", "norms", "k_source")}
        out["k_bits"] = a["k"].view(np.uint16)
        out["norm_bits"] = a["norms"].view(np.uint16)
        out["k_source"] = a["k_source"]
        out["layout"] = np.array(meta["layout"])
        for path, tol in meta["tolerances"].items():
            for stage, (atol, rtol) in tol.items():
                out[f"tol_{path}_{stage}"] = np.array([atol, rtol], dtype=np.float64)
        save(HERE / "attention" / f"{case['name']}.npz", **out)


def build_tables(widths, oracle, torch):
    """Reference table construction for one head from allocator widths."""
    p = oracle.setup(widths)
    pm = oracle.pack_meta(widths, p._head_perm)
    assert bool((pm["pack_perm"] == torch.arange(p.head_dim)).all())
    lut, cb, off, inv = oracle.code_lut(p)
    ns, nl = pm["nopack_start"], pm["nopack_len"]
    ng = p._n_groups
    arrays = dict(head_perm=p._head_perm, inv_head_perm=p._head_perm_inv, pack_perm=pm["pack_perm"],
                  inv_pack_perm=pm["inv_pack_perm"], group_of=p._group_of, group_bits=torch.unique(widths, sorted=True),
                  rotation=p._block_rot_T.T.contiguous(), centroids=p._pos_centroids, code_lut=lut, pos_to_cb=cb,
                  lut_offsets=off, lut_inv_scales=inv)
    params = dict(dim=np.int64(p.head_dim), groups=np.int64(ng), row_bytes=np.int64(ns // 2 + nl),
                  norm_stride=np.int64(ng), nibble_dims=np.int64(ns), max_centroids=np.int64(p._pos_centroids.shape[1]),
                  logical_row_bytes=np.int64(ns // 2 + nl),
                  permutation=p._head_perm.numpy().astype(np.uint32), group_of=p._group_of.numpy().astype(np.uint32),
                  position_to_codebook=cb.numpy().astype(np.uint32), code_lut=lut.numpy().astype(np.uint8).reshape(-1),
                  rotation=arrays["rotation"].numpy().astype(np.float32).reshape(-1),
                  centroids=p._pos_centroids.numpy().astype(np.float32).reshape(-1),
                  offsets=off.numpy().astype(np.float32), inverse_scales=inv.numpy().astype(np.float32),
                  widths=widths.numpy().astype(np.uint32))
    return arrays, params


def export_config(name, dim, tokens, budget, seed, sample, attention, ref):
    torch, oracle, load, encode, reconstruct, pack, attn_fn = ref
    calib_rng = np.random.default_rng(seed + 1000)
    q_cal = synthetic.profiled(calib_rng, 4096, dim)
    k_cal = synthetic.profiled(calib_rng, 4096, dim).astype(np.float16).astype(np.float32)
    scores = synthetic.pair_energy_scores(q_cal, k_cal)
    widths = load("allocator").greedy_bit_allocation(torch.from_numpy(scores), budget, 1, 8)
    arrays, params = build_tables(widths, oracle, torch)
    k, q, v = synthetic.decode_workload(seed, tokens, dim, queries=1)
    n = tokens if attention else sample
    codes, raw, corrected, _ = encode(torch.from_numpy(k[:n].astype(np.float32)), arrays)
    scales16 = corrected.half()
    out = dict(params, scores=scores, seed=np.int64(seed), tokens=np.int64(tokens),
               input_sha256=np.array(sha(k, q, v)), sample=np.int64(sample),
               codes=codes[:sample].numpy(), corrected_f32=corrected[:sample].numpy(),
               norm_bits=scales16[:sample].view(torch.uint16).numpy(),
               packed=pack(codes[:sample].numpy(), int(params["nibble_dims"]), int(params["row_bytes"])))
    if attention:
        khat = reconstruct(codes, scales16, arrays)
        positions = torch.tensor([tokens - 1])
        logits, probs, output = attn_fn(torch.from_numpy(q), khat, torch.from_numpy(v.astype(np.float32)), positions, False)
        out.update(logits=logits.numpy(), probabilities=probs.numpy(), output=output.numpy(),
                   all_codes_sha256=np.array(sha(codes.numpy())))
    save(HERE / f"{name}.npz", **out)


def export_smollm2(ref_root, read_fixture, count=6):
    meta, a = read_fixture(ref_root / "fixtures/model/calibration.json")
    out = {}
    for i in range(count):
        for part in ("config", "table", "ranges", "widths", "scores"):
            out[f"h{i}_{part}"] = a[f"h{i}_{part}"]
    out["heads"] = np.int64(count)
    save(HERE / "smollm2_heads.npz", **out)


def export_calibration(ref_root, read_fixture):
    meta, a = read_fixture(ref_root / "fixtures/model/calibration.json")
    n = len(meta["heads"])
    widths, order, pad, stride, cfg_sha, tab_sha = [], [], [], [], [], []
    for i in range(n):
        cfg, tab = a[f"h{i}_config"], a[f"h{i}_table"]
        d, ns = int(cfg[0]), int(cfg[4])
        perm = cfg[int(cfg[6]):int(cfg[6]) + d]
        widths.append(a[f"h{i}_widths"].astype(np.int8))
        order.append(perm[0::2].astype(np.int16))
        pad.append(int(cfg[2]) - (ns // 2 + d - ns))
        stride.append(int(cfg[3]))
        cfg_sha.append(sha(cfg.astype(np.uint32)))
        tab_sha.append(sha(tab.astype(np.float32)))
    save(HERE / "smollm2_calibration.npz", widths=np.stack(widths), pair_order=np.stack(order),
         row_pad=np.array(pad, np.int32), norm_stride=np.array(stride, np.int32),
         layer=np.array([h["layer"] for h in meta["heads"]], np.int32),
         kv_head=np.array([h["kv_head"] for h in meta["heads"]], np.int32),
         rotation_threshold=np.int32(meta["rotation_threshold"]),
         config_sha256=np.array(cfg_sha), table_sha256=np.array(tab_sha))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    ap.add_argument("--only", choices=["calibration"], default=None)
    args = ap.parse_args()
    ref_root = args.reference.resolve()
    os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
    sys.dont_write_bytecode = True
    sys.path[:0] = [str(ref_root / "src"), str(ref_root)]
    import torch
    torch.set_num_threads(1)
    from tests.oracles.fixture import read_fixture
    if args.only == "calibration":
        export_calibration(ref_root, read_fixture)
        return
    from tests.oracles import production_oracle as oracle
    from tests.oracles.oracle import load
    from reference.production_math import encode, reconstruct
    from reference.mixed_layout import pack
    from reference.attention import attention

    export_mixed(ref_root, read_fixture)
    export_attention(ref_root, read_fixture)
    alloc = json.loads((ref_root / "fixtures/allocator.json").read_text())
    (HERE / "allocator.json").write_text(json.dumps({"cases": alloc["cases"]}, indent=1) + "\n")
    ref = (torch, oracle, load, encode, reconstruct, pack, attention)
    export_config("config1", dim=128, tokens=4096, budget=256, seed=0, sample=512, attention=True, ref=ref)
    export_config("config4", dim=64, tokens=4096, budget=128, seed=4, sample=512, attention=False, ref=ref)
    export_smollm2(ref_root, read_fixture)
    export_calibration(ref_root, read_fixture)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
