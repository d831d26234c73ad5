"""Time the reference's own Python CPU path beside the oracle port, on config 1.

Test infrastructure (the CPU baselines), not the product.  Needs the reference checkout,
which exists only in the build container, so it runs there and writes its result to
``oracle/reference_cpu_timing.json``; ``bench.py`` quotes that file next to the port it
times live on the GPU box.

Workload: config 1 - 4096 FP16-rounded synthetic keys at head_dim 128 (``bgtq.synthetic.
decode_workload(0, 4096, 128)``, the golden fixture's inputs), the config-1 tables, one FP32
query at position 4095, non-causal.  Stages, as the reference times them
(``tests/oracles/benchmark.py:18-31``: ``perf_counter_ns`` around each call, 10 warm-up and
30 timed repetitions, median reported):
  encode   ``reference.production_math.encode`` + ``reference.mixed_layout.pack``
           (``src/reference/production_math.py:4-24``, ``src/reference/mixed_layout.py:21-27``)
  attend   ``reference.production_math.reconstruct`` + ``reference.attention.attention``
           (``production_math.py:27-31``, ``src/reference/attention.py:5-22``)
each with ``torch.set_num_threads(1)`` (the reference's convention) and with every host
core; the oracle port (``oracle/bgtq_oracle.c``) on the same stages and thread counts.

    python oracle/time_reference_cpu.py --reference <path to block-gqt-webgpu>
"""
from __future__ import annotations

import argparse
import json
import os
import platform
import statistics
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
sys.path[:0] = [str(REPO / "block-gqt-webgpu_b200"), str(HERE)]


def measure(fn, warmup=10, reps=30):
    samples = []
    for rep in range(-warmup, reps):
        t0 = time.perf_counter_ns()
        fn()
        if rep >= 0:
            samples.append((time.perf_counter_ns() - t0) / 1000.0)
    return {"median_us": statistics.median(samples), "min_us": min(samples), "mean_us": statistics.mean(samples)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    args = ap.parse_args()
    ref = args.reference.resolve()
    os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
    sys.dont_write_bytecode = True
    sys.path[:0] = [str(ref / "src"), str(ref)]
    import torch
    from reference.attention import attention
    from reference.mixed_layout import pack
    from reference.production_math import encode, reconstruct

    import bgtq
    import oracle
    from bgtq import synthetic
    z = np.load(REPO / "tests" / "golden" / "config1.npz")
    d, ng, ns, rb = int(z["dim"]), int(z["groups"]), int(z["nibble_dims"]), int(z["row_bytes"])
    perm = torch.from_numpy(z["permutation"].astype(np.int64))
    a = {"rotation": torch.from_numpy(z["rotation"].reshape(d, d)),
         "group_bits": torch.arange(ng), "head_perm": perm, "inv_head_perm": torch.argsort(perm),
         "group_of": torch.from_numpy(z["group_of"].astype(np.int64)),
         "lut_offsets": torch.from_numpy(z["offsets"]), "lut_inv_scales": torch.from_numpy(z["inverse_scales"]),
         "code_lut": torch.from_numpy(z["code_lut"].astype(np.int64).reshape(-1, 256)),
         "pos_to_cb": torch.from_numpy(z["position_to_codebook"].astype(np.int64)),
         "pack_perm": torch.arange(d), "inv_pack_perm": torch.arange(d),
         "centroids": torch.from_numpy(z["centroids"].reshape(d, -1))}
    k, q, v = synthetic.decode_workload(0, 4096, d)
    x = torch.from_numpy(k.astype(np.float32))
    qt, vt = torch.from_numpy(q), torch.from_numpy(v.astype(np.float32))
    pos = torch.tensor([4095])
    p = bgtq.BlockGTQParameters.from_arrays(z)
    cfg, tab = bgtq.tables(p)

    codes, _, corrected, _ = encode(x, a)
    scales = corrected.half()
    out_ref = attention(qt, reconstruct(codes, scales, a), vt, pos, False)[2].numpy()
    assert np.allclose(out_ref, z["output"], atol=1e-5, rtol=1e-4), "reference path reproduces the golden output"
    enc = oracle.encode(cfg, tab, k.view(np.uint16))
    assert np.array_equal(oracle.unpack(enc["packed"][:, :rb], d, ns), codes.numpy()), "port codes == reference codes"

    cores = os.cpu_count() or 1
    result = {"workload": "config 1: 4096 keys at head_dim 128 (FP16-rounded synthetic, seed 0), config-1 tables, "
                          "one FP32 query at position 4095, non-causal",
              "protocol": "perf_counter_ns around each call, 10 warm-up + 30 timed repetitions, median "
                          "(tests/oracles/benchmark.py:18-31)",
              "host": {"cores": cores, "machine": platform.machine(), "python": platform.python_version(),
                       "torch": torch.__version__, "note": "the build container, not the GPU box"},
              "reference_python": {}, "port_c": {}}
    for threads in sorted({1, cores}):
        torch.set_num_threads(threads)
        result["reference_python"][str(threads)] = {
            "encode": measure(lambda: (pack(encode(x, a)[0].numpy(), ns, rb))),
            "attend": measure(lambda: attention(qt, reconstruct(codes, scales, a), vt, pos, False))}
        result["port_c"][str(threads)] = {
            "encode": measure(lambda: oracle.encode(cfg, tab, k.view(np.uint16), threads=threads)),
            "attend": measure(lambda: oracle.attention(q, oracle.reconstruct(cfg, tab, enc["packed"], enc["scales"],
                                                                           threads=threads), v, threads=threads))}
    for impl in ("reference_python", "port_c"):
        for t, st in result[impl].items():
            st["step_us"] = st["encode"]["median_us"] + st["attend"]["median_us"]
    (HERE / "reference_cpu_timing.json").write_text(json.dumps(result, indent=1) + "\n")
    print(json.dumps({impl: {t: round(st["step_us"]) for t, st in result[impl].items()}
                      for impl in ("reference_python", "port_c")}))


if __name__ == "__main__":
    main()
