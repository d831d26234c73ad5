"""Benchmark: batched compressed-K GQA decode on B200 (the headline configuration, config 4).

Workload: SmolLM2-135M attention geometry - 30 layers, 3 KV heads, 9 query heads (GQA 3),
head_dim 64 - one batch of 256 sequences x 32768 cached tokens, Block-GTQ packed K
(config-4 tables: allocator widths for the synthetic pair-energy profile at budget 128,
built by the reference's table code) + FP16 V, synthetic data drawn on the device.
The batch is split by sequence over the N ranks (256/N each, one process per GPU, no
collective on the data path); after the timed region every rank's outputs are gathered
to rank 0 over NCCL and proven by exact per-rank checksums.
One step = one decode step of the whole batch through all 30 layers' attention: per
layer, append the new token's K (encode) and V for every sequence and KV head in one
launch (bgtq_append_kv), then compressed-K GQA attention over the cache (the kernel
specialised for the config-4 group structure, compiled on the first warm-up step).
Metric: decoded tokens/s (whole job).

  value  inputs resident in HBM, device-timed with CUDA events (max over ranks)
  e2e    the same step through the C ABI with host buffers: Q / new K / new V copied
         from pinned host memory (one host bgtq_append_kv and one host bgtq_attend per
         layer) and attention outputs copied back, inside the timed region
  roofline  attention launch (query rotation + attention kernel) timed with CUDA events
         inside the timed region, algorithmic bytes = tokens x KV heads x (row bytes +
         2 x groups + 2 x head_dim) at logical row size, against MEASURED_PEAKS.json HBM
  k_encode  bulk encode of the 32768-token prefix per (layer, head), Mkeys/s
  weak_scaling  (N > 1) every rank runs its own 256 sequences (the per-GPU workload fixed)
  fp16k_attention / prefill_config5_layer / config1  (N = 1) the FP16-K baseline attention
         at config-4 geometry, one config-5 prefill layer on the tensor cores, and the
         config-1 parity case's latency
  cpu_baseline  (N = 1, rank 0, after all GPU work) the reference's CPU path restated
         (vectorised PyTorch, oracle/torch_port.py, or the C oracle, the faster) on sampled
         (layer, sequence, KV head) pairs of the real cache, which the C oracle also checks:
         the prefix encode bit-exact and the GPU's attention outputs within 1e-5 / 1e-4

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  torchrun --nproc-per-node N bench.py --gpus N ...

Other workloads (--workload): model-smollm2 / model-qwen (configs 2-3, full decode step),
prefill (config 5, tensor-core causal prefill, 16 sequences split over the ranks) and
config1 (the parity case: latency of encoding 4096 keys at head_dim 128 plus one
attention output, beside the CPU oracle).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT / "block-gqt-webgpu_b200")]

LAYERS, KV_HEADS, Q_HEADS, HEAD_DIM = 30, 3, 9, 64
GQA = Q_HEADS // KV_HEADS
FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
ATOL, RTOL = 1e-5, 1e-4
METRIC = "compressed-K decode attention tokens/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=256, help="sequences in the batch (split over the ranks)")
    ap.add_argument("--context", type=int, default=32768)
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="budget of the CPU baseline sample")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-weak", action="store_true", help="N > 1: skip the per-GPU-256 weak-scaling run")
    ap.add_argument("--no-extras", action="store_true", help="N = 1: skip the FP16-K / prefill / config-1 keys")
    ap.add_argument("--clocks-dir", type=Path, default=None, help="keep the nvidia-smi samples here")
    ap.add_argument("--splits", type=int, default=0, help="decode: force the split-KV factor (0: the planner's)")
    ap.add_argument("--model-path", choices=["best", "step", "graph", "eager"], default="best",
                    help="model decode: both the persistent step kernel and the CUDA graph of per-layer launches, "
                         "headline the faster (default), or only one of them")
    ap.add_argument("--schedule", choices=["auto", "split", "stream_k"], default="auto",
                    help="decode attention schedule (auto: stream-K when estimated faster than split-KV)")
    ap.add_argument("--tables", choices=["config4", "calibration"], default="config4",
                    help="decode: config-4 tables for every head (the headline), or the 90 heads of the "
                         "reference's SmolLM2 calibration (30 layers x 3 KV heads)")
    ap.add_argument("--workload", choices=["decode", "model-smollm2", "model-qwen", "prefill", "config1"], default="decode",
                    help="decode: config 4 (the headline); model-*: configs 2/3; prefill: config 5")
    return ap.parse_args()


def tables():
    import bgtq
    z = np.load(ROOT / "tests" / "golden" / "config4.npz")
    p = bgtq.BlockGTQParameters.from_arrays(z)
    return p, *bgtq.tables(p)


def peaks():
    """Roofline denominators: MEASURED_PEAKS.json (driver-measured on this pool), else the
    pool's earlier measurement."""
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        m = json.loads(f.read_text())
        return {k: float(m.get(k, FALLBACK[k])) for k in FALLBACK}, "measured"
    return dict(FALLBACK), "fallback"


def bytes_per_token_head(p):
    logical = p.nibble_dims // 2 + p.dim - p.nibble_dims
    return logical + 2 * p.groups + 2 * p.dim


def encode_flops_per_key(p):
    sizes = np.bincount(np.asarray(p.group_of, np.int64))
    return int(2 * (sizes ** 2).sum())


def calibration_tables(family, n):
    """Tables of the first n heads (layer-major) of a frozen calibration, built by the native
    table builder from the calibrated bit widths and pair order (the reference's bytes):
    "smollm2" - the reference's own SmolLM2 calibration (30 layers x 3 KV heads);
    "qwen" - the reference's calibration procedure run on the random-init Qwen2.5-0.5B
    geometry (24 layers x 2 KV heads, tests/golden/make_qwen_calibration.py)."""
    import bgtq
    z = np.load(ROOT / "tests" / "golden" / f"{'smollm2' if family == 'smollm2' else 'qwen'}_calibration.npz")
    out = []
    for i in range(n):
        j = i % len(z["widths"])
        out.append(bgtq.build_tables(z["widths"][j].astype(np.int64), pair_order=z["pair_order"][j].astype(np.int64),
                                     rotation_threshold=int(z["rotation_threshold"]), row_pad=int(z["row_pad"][j]),
                                     norm_stride=int(z["norm_stride"][j])))
    return out


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during a timed region."""
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int, keep_dir: Path | None = None, tag: str = "main"):
        self.index, self.proc, self.path, self.keep_dir, self.tag = index, None, None, keep_dir, tag

    def start(self):
        try:
            if self.keep_dir:
                self.keep_dir.mkdir(parents=True, exist_ok=True)
                self.path = self.keep_dir / f"clocks_{self.tag}_gpu{self.index}.csv"
            else:
                fd, name = tempfile.mkstemp(prefix=f"bgtq_clocks_{self.tag}_", suffix=".csv")
                os.close(fd)
                self.path = Path(name)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 8:
                try:
                    rows.append((float(parts[0]), float(parts[1]), parts[4:8]))
                except ValueError:
                    pass
        if not self.keep_dir:
            self.path.unlink(missing_ok=True)
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, flags in rows for i, f in enumerate(flags) if f.lower() == "active"})
        loaded = [r[0] for r in rows if r[0] > 0.5 * r[1]] or [r[0] for r in rows]
        return {"sm_mhz": float(np.median(loaded)), "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                "samples": len(rows)}


def decode_config(args, world, calib):
    """The `config` of the decode line; the reference arm prints the same one."""
    return {"workload": "config4: SmolLM2 attention geometry, 30 layers x 3 KV / 9 Q heads (GQA 3), head_dim 64, "
                        f"one batch of {args.batch} sequences x context {args.context} split by sequence over the "
                        "GPUs, Block-GTQ K (" + ("the 90 SmolLM2 calibration heads" if calib else "config-4 tables")
                        + ") + FP16 V; step = append new K/V + attention for every layer",
            "tables": args.tables, "layers": args.layers, "kv_heads": KV_HEADS, "q_heads": Q_HEADS,
            "head_dim": HEAD_DIM, "global_batch": args.batch, "seq_len": args.context,
            "parallelism": f"sequence-sharded x{world} ({args.batch}/{world} sequences per GPU, no collective on "
                           "the data path; outputs gathered to rank 0 after the timed region)",
            "l2": "inputs larger than L2: the ~136 GB (N=1) cache is streamed every step, no flush needed"}


# ---------------------------------------------------------------------------------------
# CPU legs (the oracle port: the tests' checker, timed here as the CPU baseline)
# ---------------------------------------------------------------------------------------

def _oracle():
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    return oracle


def pair_runner(kind, threads):
    """The reference's per-decode-step CPU work for one (sequence, KV head) pair - encode the
    new key, reconstruct the pair's whole cache from its packed rows, attention for its GQA
    query rows - in one of the two CPU restatements of the reference's path: "torch" (the
    vectorised PyTorch form the reference's own CPU code has, oracle/torch_port.py) or "c"
    (the C oracle, oracle/bgtq_oracle.c)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    if kind == "torch":
        import torch
        import torch_port
        torch.set_num_threads(threads)
        tbs = {}

        def run(pr):
            key = id(pr["cfg"])
            if key not in tbs:
                tbs[key] = torch_port.Tables(pr["cfg"], pr["tab"])
            tb = tbs[key]
            torch_port.encode(tb, pr["knew"])
            kh = torch_port.reconstruct(tb, pr["packed"], pr["scales"])
            torch_port.attention(pr["q"], kh, pr["v"])
        return run
    import oracle

    def run(pr):
        oracle.encode(pr["cfg"], pr["tab"], pr["knew"], threads=1)
        kh = oracle.reconstruct(pr["cfg"], pr["tab"], pr["packed"], pr["scales"], threads=threads)
        oracle.attention(pr["q"], kh, pr["v"], threads=threads)
    return run


def cpu_pair_rate(run, pairs, budget_s, min_passes=1):
    """Run `run` over the sampled pairs until the budget is spent (at least min_passes
    passes); returns (seconds per pair, pairs run)."""
    done, t0 = 0, time.perf_counter()
    while True:
        for pr in pairs:
            run(pr)
            done += 1
        if done >= min_passes * len(pairs) and time.perf_counter() - t0 > budget_s:
            break
    return (time.perf_counter() - t0) / done, done


def fastest_port(pairs, threads, budget_s):
    """Both CPU restatements timed on the same pairs; the faster is the baseline."""
    times = {}
    for kind in ("torch", "c"):
        run = pair_runner(kind, threads)
        run(pairs[0])                                   # warm-up (tables, thread pools)
        times[kind] = cpu_pair_rate(run, pairs, budget_s)
    kind = min(times, key=lambda k: times[k][0])
    return kind, times


def synthetic_pairs(oracle, cfg, tab, context, n, seed=123):
    """n synthetic (sequence, KV head) pairs at the full context: profiled FP16 keys encoded
    by the oracle, N(0,1) values, GQA query rows."""
    from bgtq import synthetic
    rng = np.random.default_rng(seed)
    out = []
    k = synthetic.profiled(rng, context, HEAD_DIM).astype(np.float16).view(np.uint16)
    enc = oracle.encode(cfg, tab, k, threads=os.cpu_count() or 1)
    for _ in range(n):
        out.append({"cfg": cfg, "tab": tab, "knew": k[:1], "packed": enc["packed"], "scales": enc["scales"],
                    "q": synthetic.profiled(rng, GQA, HEAD_DIM),
                    "v": rng.standard_normal((context, HEAD_DIM)).astype(np.float32)})
    return out


def reference_timing_here():
    """The reference's own Python path against the C port on config 1, measured in the build
    container by oracle/time_reference_cpu.py (the reference checkout is not on this host)."""
    f = ROOT / "oracle" / "reference_cpu_timing.json"
    if not f.exists():
        return None
    r = json.loads(f.read_text())
    return {"workload": r["workload"], "host": r["host"],
            "reference_python_step_us": {t: round(v["step_us"]) for t, v in r["reference_python"].items()},
            "port_c_step_us": {t: round(v["step_us"]) for t, v in r["port_c"].items()}}


def cpu_baseline_and_check(samples, layers, budget_s):
    """The cpu_baseline leg of the decode bench (N = 1, rank 0, after all GPU work) on
    sampled pairs of the real cache.  Checks first (untimed, the C oracle): its encode of
    each pair's 32768-token prefix equals the packed rows and FP16 scales read back from the
    GPU bit for bit, and the GPU's attention outputs of the last timed step are within 1e-5
    abs + 1e-4 rel of the oracle's on the GPU's own codes.  Then times the per-decode-step
    CPU work on those pairs with all host threads in both CPU restatements (the faster is
    the baseline) and with one thread."""
    oracle = _oracle()
    threads = os.cpu_count() or 1
    enc_ok, worst = True, 0.0
    for pr in samples:
        enc = oracle.encode(pr["cfg"], pr["tab"], pr["prefix"], threads=threads)
        n = len(pr["prefix"])
        enc_ok &= bool(np.array_equal(enc["packed"], pr["packed"][:n]) and np.array_equal(enc["scales"], pr["scales"][:n]))
        kh = oracle.reconstruct(pr["cfg"], pr["tab"], pr["packed"], pr["scales"], threads=threads)
        _, _, o = oracle.attention(pr["q"], kh, pr["v"], threads=threads)
        err = np.abs(pr["out"] - o) / (ATOL + RTOL * np.abs(o))
        worst = max(worst, float(err.max()))
    kind, times = fastest_port(samples, threads, budget_s / 2)
    per_pair = times[kind][0]
    per_pair_1, _ = cpu_pair_rate(pair_runner(kind, 1), samples[:4], min(4.0, budget_s / 4))
    if kind == "torch":
        import torch
        torch.set_num_threads(threads)
    ctx = len(samples[0]["v"])
    return ({"value": 1.0 / (per_pair * layers * KV_HEADS), "unit": "tokens/s", "cores": threads, "kind": "port",
             "single_thread_value": 1.0 / (per_pair_1 * layers * KV_HEADS), "port": kind,
             "ms_per_pair": {k: v[0] * 1e3 for k, v in times.items()},
             "sample": f"{len(samples)} (layer, sequence, KV head) pairs of the real cache at context {ctx}: encode "
                       f"the new key + reconstruct the pair's keys + attention for its {GQA} query rows, in the "
                       f"vectorised PyTorch restatement of the reference's CPU path and in the C oracle on {threads} "
                       f"threads (the faster, {kind}: {per_pair * 1e3:.2f} ms per pair; 1 thread: "
                       f"{per_pair_1 * 1e3:.1f} ms); tokens/s = 1 / (time per pair x {layers} layers x {KV_HEADS} KV "
                       "heads), the same rate for any batch",
             "run_after_gpu_work": True, "reference_python_config1": reference_timing_here()},
            {"pairs": len(samples), "prefix_encode_bit_exact": enc_ok,
             "attention_worst_fraction_of_tolerance": worst, "attention_within_tolerance": worst <= 1.0})


def run_reference(args, rank, world):
    """The reference arm: the CPU implementation of this path on the decode workload's config,
    with all host threads - the vectorised PyTorch restatement of the reference's CPU code or
    the C oracle, whichever is faster here.  A step is a bounded sample: the per-decode-step
    CPU work (encode the new key, reconstruct, attention) of `pairs` synthetic (sequence, KV
    head) pairs at the full context; ms_per_step is that sample's measured time and value the
    tokens/s it implies (1 / (time per pair x layers x KV heads))."""
    if rank != 0:
        return
    import bgtq  # noqa: F401  (tables only)
    oracle = _oracle()
    p, cfg, tab = tables()
    threads = os.cpu_count() or 1
    pairs = synthetic_pairs(oracle, cfg, tab, args.context, 8)
    kind, times = fastest_port(pairs, threads, 0.0)
    run = pair_runner(kind, threads)
    per_pair = times[kind][0]
    per_step_pairs = max(8, int(1.0 / per_pair) // 8 * 8)            # about one second per step
    step_pairs = (pairs * (per_step_pairs // len(pairs) + 1))[:per_step_pairs]
    for _ in range(args.warmup):
        cpu_pair_rate(run, step_pairs, 0.0)
    times_s = []
    for _ in range(max(1, args.steps)):
        t0 = time.perf_counter()
        cpu_pair_rate(run, step_pairs, 0.0)
        times_s.append(time.perf_counter() - t0)
    step_s = float(np.sum(times_s)) / len(times_s)
    value = per_step_pairs / step_s / (args.layers * KV_HEADS)
    cb = {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "port": kind,
          "ms_per_pair": {k: v[0] * 1e3 for k, v in times.items()},
          "sample": f"each step: {per_step_pairs} synthetic (sequence, KV head) pairs at context {args.context} "
                    f"(encode the new key + reconstruct + attention for {GQA} query rows) in the {kind} restatement "
                    f"of the reference's CPU path, {step_s * 1e3:.0f} ms; tokens/s = pairs / time / "
                    f"({args.layers} layers x {KV_HEADS} KV heads)",
          "reference_python_config1": reference_timing_here()}
    print(json.dumps({"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
                      "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3,
                      "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                      "data": "synthetic", "config": decode_config(args, world, args.tables == "calibration"),
                      "cpu_baseline": cb,
                      "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
          flush=True)


# ---------------------------------------------------------------------------------------
# decode (config 4)
# ---------------------------------------------------------------------------------------

def run_ours(args, rank, world, local_rank):
    import torch
    import bgtq
    from bgtq import sharding, synthetic
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = sharding.init_from_env("nccl", timeout_s=300.0, device=dev)
    p, cfg, tab = tables()
    total, T, L, H, R, d = args.batch, args.context, args.layers, KV_HEADS, GQA, HEAD_DIM
    counts = [len(sharding.split_range(total, world, r)) for r in range(world)]
    mine = sharding.split_range(total, world, rank)
    B = len(mine)
    weak = world > 1 and not args.no_weak
    BA = total if weak else B                   # sequences held on this GPU
    steps, warmup = args.steps, args.warmup
    calib = args.tables == "calibration"
    head_tables = calibration_tables("smollm2", L * H) if calib else [(cfg, tab)] * (L * H)
    head_params = [bgtq.BlockGTQParameters.from_tables(*t) for t in head_tables] if calib else [p] * (L * H)
    e2e_steps = 0 if args.no_e2e else max(2, steps // 2)
    capacity = T + warmup + steps + (e2e_steps + 1) + (2 + steps if weak else 0) + 8
    sig = torch.from_numpy(synthetic.pair_sigma(d // 2).astype(np.float32)).to(dev)
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    checking = world == 1 and rank == 0 and args.cpu_seconds > 0
    check_seqs = sorted({0, B // 3, (2 * B) // 3, B - 1})
    check_layers = sorted({0, L - 1})
    saved = {}

    def profiled_keys(n0, n1):
        out = torch.empty((n0, n1, d), dtype=torch.float16, device=dev)
        chunk = max(1, (1 << 26) // (n1 * d))
        for i in range(0, n0, chunk):
            blocks = torch.randn((min(chunk, n0 - i), n1, d // 2, 2), device=dev, generator=gen) * sig[None, None, :, None]
            out[i:i + chunk] = torch.cat([blocks[..., 0], blocks[..., 1]], -1).half()
        return out

    # ---- build the caches: T tokens for BA sequences in every (layer, KV head) ----
    keys, values, atts, enc_ms = [], [], [], []
    t_setup = time.perf_counter()
    for layer in range(L):
        lk, lv = [], []
        for h in range(H):
            k = bgtq.PackedKeys(head_tables[layer * H + h], capacity, sequences=BA, device=local_rank)
            v = bgtq.Values(d, capacity, "f16", sequences=BA, device=local_rank)
            kk = profiled_keys(BA, T)
            vv = torch.randn((BA, T, d), device=dev, generator=gen).half()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            k.append(kk)
            e1.record()
            v.append(vv)
            if checking and layer in check_layers:
                for s in check_seqs:
                    saved[(layer, h, s)] = (kk[s].cpu().numpy().view(np.uint16), vv[s].cpu().numpy())
            del kk, vv
            torch.cuda.synchronize()
            enc_ms.append(e0.elapsed_time(e1))
            lk.append(k)
            lv.append(v)
        keys.append(lk)
        values.append(lv)
        atts.append(bgtq.GroupedAttention(lk, lv, R))
        if args.splits:
            atts[-1].set_splits(args.splits)
        atts[-1].set_schedule(args.schedule)
    setup_s = time.perf_counter() - t_setup
    q = [torch.randn((BA, H, R, d), device=dev, generator=gen) for _ in range(L)]
    knew = [profiled_keys(BA, H) for _ in range(L)]                 # [BA, H, d] new token keys
    vnew = [torch.randn((BA, H, d), device=dev, generator=gen).half() for _ in range(L)]
    outs = [torch.empty((BA, H, R, d), device=dev) for _ in range(L)]
    stream = torch.cuda.current_stream(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(L)]

    def step(n, record=False):
        for layer in range(L):
            bgtq.append_kv(keys[layer], values[layer], knew[layer][:n], vnew[layer][:n])  # every KV head, one launch
            if record:
                ev[layer][0].record(stream)
            atts[layer].attend(q[layer][:n], out=outs[layer][:n], seq_count=n)
            if record:
                ev[layer][1].record(stream)

    def barrier():
        sharding.barrier(dist, torch.cuda.synchronize)

    # ---- the batch split over the ranks: B sequences here ----
    for i in range(warmup):
        step(B)
        if i == 0 and calib:
            # the first step queued each layer's layout-specialised kernel: wait for them
            torch.cuda.synchronize()
            bgtq.layout_jit_wait(600.0)
    barrier()
    clocks = Clocks(local_rank, args.clocks_dir)
    clocks.start()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    attn_ms = []
    t_start.record(stream)
    for _ in range(steps):
        step(B, record=True)
        # per-layer attention durations are read after the region (events are async)
        attn_ms.append(ev)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(L)]
    t_end.record(stream)
    barrier()
    clk = clocks.stop()
    elapsed = t_start.elapsed_time(t_end) / 1e3
    launch_ms = [a.elapsed_time(b) for evs in attn_ms for a, b in evs]
    # per layer: the fused K/V append (bumps the lengths too) + the attention's launches (the
    # query rotation, unless the attention CTAs rotate their own queries, and the attention)
    launches = steps * L * (1 + atts[0].last_launches)
    strong_out = torch.stack([o[:B] for o in outs])          # [L, B, H, R, d] of the last timed step
    rows_seen = T + warmup + steps
    splits = atts[0].last_splits
    sk_ctas = atts[0].last_stream_k

    # ---- e2e through the C ABI with host buffers ----
    e2e = None
    if e2e_steps:
        qh = [t[:B].cpu().pin_memory() for t in q]
        kh = [t[:B].cpu().pin_memory() for t in knew]
        vh = [t[:B].cpu().pin_memory() for t in vnew]
        oh = [torch.empty((B, H, R, d), pin_memory=True) for _ in range(L)]
        qn = [t.numpy() for t in qh]
        kn = [t.view(torch.int16).numpy().view(np.uint16) for t in kh]
        vn = [t.view(torch.int16).numpy().view(np.uint16) for t in vh]
        on = [t.numpy() for t in oh]

        def step_host():
            for layer in range(L):
                bgtq.append_kv(keys[layer], values[layer], kn[layer], vn[layer])  # host K/V, every KV head
                atts[layer].attend(qn[layer], out=on[layer], wait=False)         # download queued
            stream.synchronize()                                                  # the step's outputs are on the host

        step_host()
        barrier()
        h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        h0.record(stream)
        for _ in range(e2e_steps):
            step_host()
        h1.record(stream)
        barrier()
        e2e = (h0.elapsed_time(h1) / 1e3, e2e_steps)

    # ---- weak scaling: every rank runs its own full batch (the per-GPU work fixed) ----
    weak_s = 0.0
    if weak:
        for _ in range(2):
            step(BA)
        barrier()
        w0, w1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        w0.record(stream)
        for _ in range(steps):
            step(BA)
        w1.record(stream)
        barrier()
        weak_s = w0.elapsed_time(w1) / 1e3

    # ---- max over ranks; the outputs of the split batch gathered to rank 0 (NCCL) ----
    elapsed_max, e2e_max, weak_max = sharding.max_over_ranks([elapsed, e2e[0] if e2e else 0.0, weak_s], dist, dev)
    gathered = sharding.gather_to_root(strong_out, counts, dist, dev, dim=1)
    bits = sharding.gather_ints([sharding.bit_checksum(strong_out)], dist, dev)
    status = bgtq.device_status(local_rank)
    gather = None
    if rank == 0:
        offs = np.concatenate([[0], np.cumsum(counts)])
        proven = [sharding.bit_checksum(gathered[:, offs[r]:offs[r + 1]]) == bits[r][0] for r in range(world)]
        gather = {"shape": list(gathered.shape), "bytes": int(gathered.numel() * 4), "backend": "nccl" if dist else None,
                  "ranks_proven_by_checksum": int(sum(proven)), "all_proven": all(proven),
                  "outputs_finite": bool(torch.isfinite(gathered).all())}

    # ---- extra keys (one GPU): FP16-K baseline attention, config-5 layer, config-1 ----
    extras = {}
    if world == 1 and not args.no_extras:
        xclk = Clocks(local_rank, args.clocks_dir, "extras")
        xclk.start()
        extras["fp16k_attention"] = fp16k_attention(B, T, R, d, local_rank, gen, profiled_keys,
                                                    float(np.mean(launch_ms)), head_params[0])
        extras["prefill_config5_layer"] = prefill_layer(local_rank)
        extras["config1"] = config1_latency(local_rank, 20, 3)
        extras["clocks"] = xclk.stop()

    # ---- the CPU baseline (the oracle, after all GPU work) and its checks ----
    cpu, parity = None, None
    if checking:
        samples = []
        for (layer, h, s), (k16, v16) in saved.items():
            cfg_h, tab_h = head_tables[layer * H + h]
            packed, scales = keys[layer][h].read(s, 0, rows_seen)
            extra_v = np.repeat(vnew[layer][s, h].cpu().numpy()[None], rows_seen - T, axis=0)
            samples.append({"cfg": cfg_h, "tab": tab_h, "prefix": k16, "packed": packed, "scales": scales,
                            "knew": knew[layer][s, h].cpu().numpy().view(np.uint16)[None],
                            "q": q[layer][s, h].cpu().numpy(), "out": strong_out[layer, s, h].cpu().numpy(),
                            "v": np.concatenate([v16, extra_v]).astype(np.float32)})
        cpu, parity = cpu_baseline_and_check(samples, L, args.cpu_seconds)

    if rank == 0:
        pk, peak_kind = peaks()
        hbm = pk["hbm_gbs"]
        ctx_mean = T + (warmup + 1 + warmup + steps) / 2.0
        bpt = float(np.mean([bytes_per_token_head(ph) for ph in head_params]))
        alg_bytes = B * ctx_mean * H * bpt
        mean_launch_s = float(np.mean(launch_ms)) / 1e3
        achieved = alg_bytes / mean_launch_s / 1e9
        traffic = None
        tf = ROOT / "profiles" / "attention_traffic.json"
        if tf.exists() and not calib:   # captured on the config-4 tables
            per_token_head = json.loads(tf.read_text())["dram_bytes_per_token_head"]
            traffic = per_token_head * B * ctx_mean * H
        enc_keys = BA * T
        enc_ms_med = float(np.median(enc_ms))
        enc_rate = enc_keys / (enc_ms_med / 1e3)
        enc_bytes = float(np.mean([2 * d + (ph.nibble_dims // 2 + d - ph.nibble_dims) + 2 * ph.groups
                                   for ph in head_params]))
        enc_flops = float(np.mean([encode_flops_per_key(ph) for ph in head_params]))
        value = total * steps / elapsed_max
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": elapsed_max / steps * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (device-drawn K with the pair-energy profile, N(0,1) V and Q)",
            "config": decode_config(args, world, calib),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback 6650 GB/s", "traffic": traffic,
                         "kernel": "query rotation + " + ("bgtq_attn_jit" if bgtq.layout_jit_stats()[0]
                                                          else "attn_kernel<64,3,packed,f16>")
                                   + " per layer (CUDA events, rank 0)",
                         "algorithmic_bytes_per_launch": alg_bytes,
                         "bytes_per_token_head": bpt, "mean_launch_ms": mean_launch_s * 1e3,
                         "split_kv": None if sk_ctas else splits, "stream_k_ctas": sk_ctas or None},
            "k_encode": {"value": enc_rate / 1e6, "unit": "Mkeys/s", "keys_per_launch": enc_keys,
                         "ms_per_launch": enc_ms_med, "hbm_frac": enc_rate * enc_bytes / 1e9 / hbm,
                         "fp32_tflops": enc_rate * enc_flops / 1e12,
                         "bytes_per_key": enc_bytes, "flops_per_key": enc_flops},
            "cpu_baseline": cpu if cpu is not None else
            {"value": None, "unit": "tokens/s", "cores": None, "kind": "port",
             "sample": "not run: the CPU baseline runs on rank 0 at N = 1 only"},
            "gpu_launches": launches,
            "clocks": clk,
            "attention_kernel": (("layout-specialised (compiled at run time for each layer's heads' group "
                                  "structures)" if calib else
                                  "layout-specialised (compiled at run time for the config-4 group structure)")
                                 if bgtq.layout_jit_stats()[0] else "generic"),
            "layout_jit": bgtq.layout_jit_counts(),
            "gather": gather,
            "checks": {"device_status": status, "setup_s": setup_s, "sequences_per_rank": counts,
                       "oracle": parity},
        }
        if e2e:
            h2d = L * B * (H * R * d * 4 + H * d * 2 + H * d * 2)
            line["e2e"] = {"value": total * e2e[1] / e2e_max, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                           "d2h_bytes_per_step": L * B * H * R * d * 4,
                           "path": "bgtq C ABI (host bgtq_append_kv of every KV head + host bgtq_attend per layer, "
                                   "downloads queued on the stream, one wait per step) on pinned host NumPy buffers"}
        if weak:
            line["weak_scaling"] = {"value": total * world * steps / weak_max, "unit": "tokens/s",
                                    "ms_per_step": weak_max / steps * 1e3, "global_batch": total * world,
                                    "note": f"every rank runs its own {total} sequences (per-GPU work fixed)"}
        line.update(extras)
        print(json.dumps(line), flush=True)
    for a in atts:
        a.destroy()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def fp16k_attention(B, T, R, d, local_rank, gen, profiled_keys, packed_ms, p):
    """The reference's FP16-K baseline attention (src/attention/attention.ts:44-59,
    src/model/attention.wgsl:13-39: FP16 K and FP16 V) at config-4 geometry on one layer of
    the same batch, beside the packed kernel's launch time from the timed region."""
    import torch
    import bgtq
    H = KV_HEADS
    dev = torch.device("cuda", local_rank)
    ks = [bgtq.FP16Keys(d, T, sequences=B, device=local_rank) for _ in range(H)]
    vs = [bgtq.Values(d, T, "f16", sequences=B, device=local_rank) for _ in range(H)]
    for h in range(H):
        ks[h].append(profiled_keys(B, T))
        vs[h].append(torch.randn((B, T, d), device=dev, generator=gen).half())
    att = bgtq.GroupedAttention(ks, vs, R)
    qq = torch.randn((B, H, R, d), device=dev, generator=gen)
    out = torch.empty_like(qq)
    for _ in range(3):
        att.attend(qq, out=out)
    torch.cuda.synchronize()
    n = 10
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n):
        att.attend(qq, out=out)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / n
    pk, kind = peaks()
    fp16_bytes = B * T * H * (2 * d + 2 * d)
    packed_bytes = B * T * H * bytes_per_token_head(p)
    res = {"batch": B, "context": T, "kv_heads": H, "q_rows_per_head": R, "layers": 1,
           "ms_per_launch": ms, "achieved_gbs": fp16_bytes / ms / 1e6, "hbm_frac": fp16_bytes / ms / 1e6 / pk["hbm_gbs"],
           "bytes_per_token_head": 4 * d, "packed_bytes_per_token_head": bytes_per_token_head(p),
           "packed_ms_per_launch": packed_ms,
           "packed_speedup": ms / packed_ms,
           "kv_cache_gb_config4": {"fp16_k": 256 * 32768 * 90 * 4 * d / 1e9,
                                   "packed_k": 256 * 32768 * 90 * bytes_per_token_head(p) / 1e9},
           "note": f"FP16-K moves {fp16_bytes / packed_bytes:.2f}x the packed path's bytes per token-head; "
                   "one layer of the same batch, CUDA events over 10 launches (query rotation + attention)"}
    att.destroy()
    for o in ks + vs:
        o.destroy()
    return res


def prefill_layer(local_rank):
    """One layer of config 5 (Qwen2.5-0.5B attention geometry, 16 sequences x 8192 tokens,
    the Qwen calibration's layer-0 tables): projections, RoPE, bulk encode, V append and the
    causal prefill on the tensor cores; the attention (query rotation + tcgen05 kernel)
    timed with CUDA events against the sustained BF16 peak."""
    import torch
    from bgtq.model import QWEN25_05B
    g = QWEN25_05B
    S, T = 16, 8192
    stores = _prefill_stores(g, S, T, 1, local_rank, range(S))
    run = _prefill_runner(g, S, T, stores, local_rank, seed=11)
    for _ in range(2):
        run(False)
    torch.cuda.synchronize()
    ev = []
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(3):
        run(True, ev)
    t1.record()
    torch.cuda.synchronize()
    layer_ms = t0.elapsed_time(t1) / 3
    attn_ms = float(np.mean([a.elapsed_time(b) for a, b in ev]))
    flops = S * g.q_heads * 2 * (2 * 64 * T * (T + 1) / 2)
    pk, kind = peaks()
    for ks, vs, att in stores:
        att.destroy()
    return {"sequences": S, "tokens": T, "layer_ms": layer_ms, "attention_ms": attn_ms,
            "tokens_per_s_per_layer": S * T / (layer_ms / 1e3),
            "roofline": {"bound": "tensor", "achieved": flops / attn_ms / 1e9, "peak": pk["bf16_tflops_sustained"],
                         "unit": "TFLOP/s", "frac": flops / attn_ms / 1e9 / pk["bf16_tflops_sustained"],
                         "peak_source": f"{kind} (bf16_tflops_sustained: the kernel runs inside a long step)",
                         "flops_per_layer": flops}}


def config1_latency(local_rank, steps, warmup):
    """Config 1 (the parity case) on the GPU: encode 4096 keys at head_dim 128 into a fresh
    store, write the 4096 FP16 V rows, one attention output; device-resident inputs
    (CUDA events) and host NumPy buffers through the C ABI (wall clock)."""
    import torch
    import bgtq
    from bgtq import synthetic
    dev = torch.device("cuda", local_rank)
    z = np.load(ROOT / "tests" / "golden" / "config1.npz")
    p = bgtq.BlockGTQParameters.from_arrays(z)
    cfg, tab = bgtq.tables(p)
    T, d = 4096, 128
    k, q, v = synthetic.decode_workload(0, T, d)
    keys, values = bgtq.PackedKeys((cfg, tab), T, device=local_rank), bgtq.Values(d, T, "f16", device=local_rank)
    att = bgtq.GroupedAttention([keys], [values], 1)
    k_dev, v_dev = torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev)
    q_dev = torch.from_numpy(q.reshape(1, 1, 1, d)).to(dev)
    k_host, v_host, q_host = k.copy(), v.copy(), q.reshape(1, 1, 1, d).copy()

    def step_dev():
        keys.reset()
        values.reset()
        keys.append(k_dev)
        values.append(v_dev)
        return att.attend(q_dev)

    def step_host():
        keys.reset()
        values.reset()
        keys.append(k_host)
        values.append(v_host)
        return att.attend(q_host)

    for _ in range(warmup):
        step_dev()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        step_dev()
    t1.record()
    torch.cuda.synchronize()
    dev_ms = t0.elapsed_time(t1) / steps
    out_dev = step_dev().float().cpu().numpy().reshape(1, d)
    for _ in range(warmup):
        step_host()
    torch.cuda.synchronize()
    w0 = time.perf_counter()
    for _ in range(steps):
        out_host = step_host()
    e2e_ms = (time.perf_counter() - w0) * 1e3 / steps
    out_host = np.asarray(out_host).reshape(1, d)
    ok = bool(np.allclose(out_dev, z["output"], atol=ATOL, rtol=RTOL) and np.array_equal(out_host, out_dev))
    moved = T * (2 * d + p.row_bytes + 2 * p.groups) + T * (p.row_bytes + 2 * p.groups + 2 * d) + 2 * T * 2 * d
    att.destroy()
    keys.destroy()
    values.destroy()
    return {"device_us": dev_ms * 1e3, "e2e_us": e2e_ms * 1e3, "bytes_per_step": moved,
            "h2d_bytes_per_step": k_host.nbytes + v_host.nbytes + q_host.nbytes, "d2h_bytes_per_step": 4 * d,
            "output_within_1e-5_1e-4_of_golden": ok, "bound": "latency (about 1.4 MB per step stays in L2)"}


# ---------------------------------------------------------------------------------------
# configs 2 / 3: whole-model decode
# ---------------------------------------------------------------------------------------

def _event_ms(fn, steps, warmup):
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        fn()
    t1.record()
    torch.cuda.synchronize()
    return t0.elapsed_time(t1) / steps


def run_model(args, rank, world, local_rank):
    """Configs 2/3: whole-model decode, batch 1 per GPU (replicas), random-init FP16
    weights computed in FP32 like the reference's shaders, 4096-token random-id prefix,
    then timed decode steps through bgtq.model.Decoder."""
    import torch
    import bgtq
    from bgtq import sharding
    from bgtq.model import QWEN25_05B, SMOLLM2_135M, Decoder, random_weights
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = sharding.init_from_env("nccl", timeout_s=300.0, device=dev)
    g = SMOLLM2_135M if args.workload == "model-smollm2" else QWEN25_05B
    prefix, steps, warmup = 4096, args.steps, max(3, args.warmup)
    tables = calibration_tables(g.family, g.layers * g.kv_heads)
    dec = Decoder(random_weights(g, seed=7 + rank, device=dev), g, prefix + 2 * (warmup + steps) + 16, tables, batch=1)
    rng = np.random.default_rng(rank)
    t_pre = time.perf_counter()
    dec.prefill(torch.from_numpy(rng.integers(0, g.vocab, (1, prefix))).to(dev), chunk=1024)
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t_pre
    toks = [torch.from_numpy(rng.integers(0, g.vocab, (1, 1))).to(dev) for _ in range(2 * (warmup + steps) + 4)]
    it = iter(toks)
    logits = []

    def barrier():
        sharding.barrier(dist, torch.cuda.synchronize)

    def timed(step):
        """W untimed, then K timed steps (CUDA events on the launching stream, max over ranks)."""
        def timed_step():
            torch.cuda.nvtx.range_push("timed_step")   # marks the timed steps for profilers
            step()
            torch.cuda.nvtx.range_pop()
        for _ in range(warmup):
            step()
        barrier()
        clocks = Clocks(local_rank, args.clocks_dir)
        clocks.start()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(steps):
            timed_step()
        t1.record()
        barrier()
        clk = clocks.stop()
        (ms,) = sharding.max_over_ranks([t0.elapsed_time(t1) / steps], dist, dev)
        return ms, clk

    # the persistent step: the whole model per token as one cooperative launch
    step_ms = None
    if dec.step_kernel and args.model_path in ("step", "best"):
        step_ms, step_clk = timed(lambda: logits.append(dec.forward(next(it), _check=False)))
        ctas, smem, _ = dec.step_info()
        # phase breakdown of one more step (CTA 0's global-timer stamps at the end of each
        # phase): medians over the layers, outside the timed region
        dec.step_trace(True)
        logits.append(dec.forward(next(it), _check=False))
        torch.cuda.synchronize()
        st = dec.step_trace(False).astype(np.int64)
        d_us = np.diff(st) / 1e3
        phases = d_us[:-1].reshape(g.layers, 5)
        step_phases = {"qkv": float(np.median(phases[:, 0])), "append_and_attention": float(np.median(phases[:, 1])),
                       "merge_and_o_proj": float(np.median(phases[:, 2])), "gate_up": float(np.median(phases[:, 3])),
                       "down": float(np.median(phases[:, 4])), "lm_head": float(d_us[-1]),
                       "total": float((st[-1] - st[0]) / 1e3), "unit": "us (median over layers; one traced step)"}
    # the seven launches per layer issued eagerly, one step at a time (no graph): for launch
    # lists, whose profiler does not follow every kernel node of a recorded graph
    if args.model_path == "eager":
        step_flag, dec.step_kernel = dec.step_kernel, False
        eager_ms, eager_clk = timed(lambda: logits.append(dec.forward(next(it), _check=False)))
        dec.step_kernel = step_flag
    # the same step as a CUDA graph of seven launches per layer
    graph_ms = None
    if args.model_path in ("graph", "best") or (step_ms is None and args.model_path != "eager"):
        dec.capture_decode(next(it))
        graph_ms, graph_clk = timed(lambda: logits.append(dec.decode_graph(next(it)).clone()))
    # the headline is the faster of the two measured paths, named in decode_path
    use_step = step_ms is not None and (graph_ms is None or step_ms <= graph_ms)
    if args.model_path == "eager":
        ms, clk = eager_ms, eager_clk
    else:
        ms, clk = (step_ms, step_clk) if use_step else (graph_ms, graph_clk)
    finite = all(bool(torch.isfinite(x).all()) for x in logits)
    if rank == 0:
        path = ("seven launches per layer issued eagerly" if args.model_path == "eager" else
                f"one persistent cooperative launch per token ({ctas} CTAs, {smem} B shared memory each)"
                if use_step else "CUDA graph of seven launches per layer")
        print(json.dumps({
            "metric": f"{g.family} whole-model decode tokens/s (batch 1 per GPU, 4096-token prefix)",
            "decode_path": path, "persistent_step_ms_per_step": step_ms, "graph_ms_per_step": graph_ms,
            "persistent_step_phases": step_phases if step_ms is not None else None,
            "value": world * 1e3 / ms, "unit": "tokens/s", "n_gpus": world, "steps": steps, "warmup": warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (random-init FP16 weights N(0,0.02), uniform random token ids)",
            "config": {"workload": f"config {2 if g.family == 'smollm2' else 3}: {g.family} geometry, {g.layers} layers, "
                                   f"{g.q_heads}/{g.kv_heads} heads, head_dim 64, Block-GTQ K + FP16 V",
                       "model": g.family, "global_batch": world, "seq_len": prefix, "parallelism": f"replicas x{world}",
                       "tables": ("the reference's SmolLM2 calibration (90 heads)" if g.family == "smollm2" else
                                  "the reference's calibration procedure on the random-init Qwen geometry (48 heads, "
                                  "tests/golden/qwen_calibration.npz)")},
            "attention_kernels": bgtq.layout_jit_counts(), "clocks": clk,
            "prefill_s": prefill_s, "reference_webgpu_ms_per_token": 375.6 if g.family == "smollm2" else 348.4,
            "checks": {"logits_finite": finite, "device_status": bgtq.device_status(local_rank)}}), flush=True)
    dec.destroy()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------------------
# config 5: compressed prefill
# ---------------------------------------------------------------------------------------

def _prefill_stores(g, S, T, layers, local_rank, seqs):
    import bgtq
    H = g.kv_heads
    heads = calibration_tables("qwen", layers * H)
    stores = []
    for layer in range(layers):
        ks = [bgtq.PackedKeys(heads[layer * H + h], T, sequences=len(seqs), device=local_rank) for h in range(H)]
        vs = [bgtq.Values(64, T, "f16", sequences=len(seqs), device=local_rank) for _ in range(H)]
        stores.append((ks, vs, bgtq.GroupedAttention(ks, vs, g.gqa)))
    return stores


def _prefill_runner(g, S, T, stores, local_rank, seed):
    """One prefill pass over `stores` (one entry per layer) for S sequences: BF16 N(0,1)
    activations through random-init BF16 Q/K/V projections (FP32 out), split-half RoPE, bulk
    K encode into the packed cache, FP16 V append, causal prefill attention."""
    import torch
    dev = torch.device("cuda", local_rank)
    H, d = g.kv_heads, 64
    gen = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn((S * T, g.hidden), device=dev, generator=gen, dtype=torch.bfloat16)
    wqkv = [(torch.randn((g.hidden, (g.q_heads + 2 * H) * d), device=dev, generator=gen) * 0.05).bfloat16()
            for _ in stores]
    pairs = d // 2
    inv = torch.pow(torch.tensor(float(g.rope_theta), device=dev), -torch.arange(pairs, device=dev) / pairs)
    ang = torch.arange(T, device=dev, dtype=torch.float32)[:, None] * inv[None, :]
    cos, sin = torch.cos(ang)[None, :, None, :], torch.sin(ang)[None, :, None, :]
    outs = [None] * len(stores)

    def rope(t):
        a, b = t[..., :pairs], t[..., pairs:]
        return torch.cat([a * cos - b * sin, b * cos + a * sin], -1)

    def run(record, ev=None):
        for layer, (ks, vs, att) in enumerate(stores):
            for o in ks + vs:
                o.reset()
            qkv = (x @ wqkv[layer]).float().view(S, T, g.q_heads + 2 * H, d)
            q = rope(qkv[:, :, :g.q_heads]).contiguous()
            k = rope(qkv[:, :, g.q_heads:g.q_heads + H])
            for h in range(H):
                ks[h].append(k[:, :, h, :])
                vs[h].append(qkv[:, :, g.q_heads + H + h, :])
            if record:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
            outs[layer] = att.prefill(q)
            if record:
                e1.record()
                ev.append((e0, e1))
        return outs

    return run


def run_prefill(args, rank, world, local_rank):
    """Config 5: compressed prefill, Qwen2.5-0.5B attention geometry (24 layers, 14 / 2
    heads, head_dim 64), one batch of 16 sequences x 8192 tokens split by sequence over the
    ranks.  Per layer: Q/K/V projections of N(0,1) BF16 activations (random-init BF16
    weights, FP32 out), split-half RoPE, bulk K encode into the packed cache, FP16 V append,
    causal prefill attention on the tensor cores.  Tables: the Qwen calibration.  roofline:
    attention FLOPs / attention launch time against the sustained dense BF16 peak."""
    import torch
    import bgtq
    from bgtq import sharding
    from bgtq.model import QWEN25_05B
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = sharding.init_from_env("nccl", timeout_s=300.0, device=dev)
    g = QWEN25_05B
    total, T, L = 16, 8192, args.layers if args.layers != LAYERS else g.layers
    mine = sharding.split_range(total, world, rank)
    counts = [len(sharding.split_range(total, world, r)) for r in range(world)]
    S = len(mine)
    stores = _prefill_stores(g, S, T, L, local_rank, mine)
    run = _prefill_runner(g, S, T, stores, local_rank, seed=11 + rank)
    steps, warmup = args.steps, max(3, args.warmup)
    ev = []
    for _ in range(warmup):
        run(False)
    sharding.barrier(dist, torch.cuda.synchronize)
    clocks = Clocks(local_rank, args.clocks_dir)
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        outs = run(True, ev)
    t1.record()
    sharding.barrier(dist, torch.cuda.synchronize)
    clk = clocks.stop()
    (ms,) = sharding.max_over_ranks([t0.elapsed_time(t1) / steps], dist, dev)
    attn_ms = float(np.mean([a.elapsed_time(b) for a, b in ev]))
    last = outs[-1]                                           # [S, T, 14, 64] of the last layer
    bits = sharding.gather_ints([sharding.bit_checksum(o) for o in outs], dist, dev)
    gathered = sharding.gather_to_root(last[:, -1:].contiguous(), counts, dist, dev)   # last position, every head
    flops = S * g.q_heads * 2 * (2 * 64 * T * (T + 1) / 2)
    pk, kind = peaks()
    if rank == 0:
        achieved = flops / attn_ms / 1e9
        print(json.dumps({
            "metric": "compressed prefill tokens/s (config 5)", "value": total * T / (ms / 1e3), "unit": "tokens/s",
            "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16x2 split (FP32-accurate) on tensor cores",
            "data": "synthetic (N(0,1) BF16 activations, random-init BF16 projections)",
            "config": {"workload": f"config 5: Qwen2.5-0.5B attention geometry, {L} layers, 14/2 heads, head_dim 64, "
                                   f"one batch of {total} sequences x {T} tokens split over the GPUs, causal",
                       "global_batch": total, "seq_len": T,
                       "parallelism": f"sequence-sharded x{world} ({counts} sequences per GPU)",
                       "tables": "the reference's calibration procedure on the random-init Qwen geometry "
                                 "(tests/golden/qwen_calibration.npz)"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": pk["bf16_tflops_sustained"],
                         "unit": "TFLOP/s", "frac": achieved / pk["bf16_tflops_sustained"],
                         "peak_source": f"{kind} (bf16_tflops_sustained: the kernel runs inside a long step)",
                         "flops_per_layer_rank0": flops, "mean_attention_ms": attn_ms,
                         "note": "real attention FLOPs; the FP16 high/low split issues 3 QK and 2 PV tensor-core "
                                 "products per real one"},
            "clocks": clk,
            "gather": {"last_positions_gathered": list(gathered.shape), "per_rank_layer_checksums": bits},
            "checks": {"device_status": bgtq.device_status(local_rank),
                       "outputs_finite": bool(torch.isfinite(gathered).all())}}), flush=True)
    for ks, vs, att in stores:
        att.destroy()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------------------
# config 1: the parity case
# ---------------------------------------------------------------------------------------

def run_config1(args, rank, world, local_rank):
    """Config 1, the parity case: one head of 4096 keys at head_dim 128 (config-1 tables),
    FP16 V, one FP32 query at position 4095, non-causal.  A step encodes all 4096 keys into
    a fresh packed store, writes the 4096 V rows and computes the attention output.  It is
    latency-bound (about 1.4 MB moved), so the metric is the step's latency.  value: device
    inputs, CUDA-event timed; e2e: the same step from host NumPy buffers through the C ABI
    (uploads and the output download inside the timed region).  Batch 1: replicas only."""
    import torch
    import bgtq
    from bgtq import synthetic
    torch.cuda.set_device(local_rank)
    steps, warmup = max(args.steps, 20), max(args.warmup, 3)
    res = config1_latency(local_rank, steps, warmup)
    z = np.load(ROOT / "tests" / "golden" / "config1.npz")
    p = bgtq.BlockGTQParameters.from_arrays(z)
    cfg, tab = bgtq.tables(p)
    T, d = 4096, 128
    k, q, v = synthetic.decode_workload(0, T, d)
    pk, peak_src = peaks()
    # the CPU oracle on the same step: encode + pack, reconstruct + attention
    oracle = _oracle()
    cpu = {}
    for threads in (1, os.cpu_count() or 1):
        t0 = time.perf_counter()
        n = 0
        while n < 3 or time.perf_counter() - t0 < 2.0:
            enc = oracle.encode(cfg, tab, k.view(np.uint16), threads=threads)
            kh = oracle.reconstruct(cfg, tab, enc["packed"], enc["scales"], threads=threads)
            oracle.attention(q, kh, v, threads=threads)
            n += 1
        cpu[threads] = (time.perf_counter() - t0) * 1e3 / n
    cores = max(cpu)
    if rank == 0:
        dev_s = res["device_us"] / 1e6
        print(json.dumps({
            "metric": "config 1 step latency (encode 4096 keys + one attention output)", "value": res["device_us"],
            "unit": "us", "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": res["device_us"] / 1e3,
            "higher_is_better": False, "scaling": "replicas only", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seed 0 decode workload, the config-1 golden fixture's inputs)",
            "config": {"workload": "config 1: one head, 4096 keys, head_dim 128, FP16 V, one query at position 4095, "
                                   "non-causal", "global_batch": 1, "seq_len": T, "parallelism": "replicas only",
                       "l2": "inputs (1.4 MB) stay in L2: a latency measurement"},
            "roofline": {"bound": "latency", "achieved": res["bytes_per_step"] / dev_s / 1e9, "peak": pk["hbm_gbs"],
                         "unit": "GB/s", "frac": res["bytes_per_step"] / dev_s / 1e9 / pk["hbm_gbs"],
                         "peak_source": peak_src, "bytes_per_step": res["bytes_per_step"]},
            "cpu_baseline": {"value": cpu[cores] * 1e3, "unit": "us", "cores": cores, "kind": "port",
                             "single_thread_us": cpu[1] * 1e3,
                             "sample": "the whole step (oracle encode + pack, reconstruct, attention)"},
            "e2e": {"value": res["e2e_us"], "unit": "us", "h2d_bytes_per_step": res["h2d_bytes_per_step"],
                    "d2h_bytes_per_step": res["d2h_bytes_per_step"]},
            "gpu_launches": None,
            "checks": {"output_within_1e-5_1e-4_of_golden": res["output_within_1e-5_1e-4_of_golden"],
                       "device_status": bgtq.device_status(local_rank)}}),
            flush=True)


def main():
    args = parse()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.workload == "decode":
        run_ours(args, rank, world, local_rank)
    elif args.workload == "prefill":
        run_prefill(args, rank, world, local_rank)
    elif args.workload == "config1":
        run_config1(args, rank, world, local_rank)
    else:
        run_model(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
