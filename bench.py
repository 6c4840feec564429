"""Benchmark of the b200 Laya forward (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload: one short "noul" question, batch 1,
sequence 64, bf16 weights of the 28x1024 Laya network (seeded random weights,
synthetic token ids), warm CUDA-graph replay.  A step is one forward = one
decision.  With N GPUs (torchrun, one process per GPU) every rank serves its
own stream of requests on its own weight replica (request parallel, no
collective on the data path; weak scaling); NCCL is used only for the
barriers and the max-over-ranks of the timed region.

* value: decisions/s of K back-to-back graph replays per rank with inputs
  resident in HBM, device time from CUDA events on the engine's stream,
  max over ranks; p50_ms is the median per-replay device time.
* e2e: the same metric through the public API (B200Engine.run_prepared) with
  host inputs: pinned H2D of the packed inputs, the graph, D2H of the logits
  and actions, per step.
* roofline: the projection GEMM family (the dominant kernel), timed live as a
  graph of the forward's GEMM launches only; algorithmic bytes = weight bytes
  + activation bytes each launch must move.
* cpu_baseline: the reference's own forward (FastDecisionModel from the
  offline install in baseline/_ref, its Triton RoPE replaced by the torch
  restatement the CPU needs) timed on this host's cores on a bounded sample of
  the same request; when the reference cannot be imported, the CPU oracle port
  (its bf16 Linears through torch's bf16 GEMM), labelled "port".
* configs: the other BASELINE configs measured in the same run, bounded to a
  few seconds each: C2 (FP8, 16 x 96), C3 (NVFP4, 1 x 512) and C4 (FP8, 64
  questions of s ~ U[32, 512] bucketed by 32; under torchrun its questions are
  sharded over the ranks by LPT: strong scaling), each with its device value,
  end-to-end value and tensor roofline.
* reference_gpu: the reference's own bf16 path on the same GPU (FastDecisionModel
  with its Triton RoPE under a CUDA graph, as BlackwellEngine._slot captures
  it), on the C1 request, C3's shape in bf16 and, with the reference's
  FP8Linear encoder, C1 and C2 in FP8: the GPU figure to beat.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "laya-inference-engine_b200"))
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

METRIC = "decisions/s at 1/2/4/8 B200 and p50 warm latency, one short question"
UNIT = "decisions/s"
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--precision", default="bf16", choices=["bf16", "fp8"])
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--token-tables", action="store_true",
                    help="c1: start each forward from the token tables (515 MB per GPU)")
    ap.add_argument("--lanes", type=int, default=2,
                    help="c1 / c4: also time this many serving lanes working at once (1: skip)")
    ap.add_argument("--no-configs", action="store_true", help="c1: skip the C2 / C3 / C4 legs")
    ap.add_argument("--no-reference-gpu", action="store_true", help="c1: skip the reference-on-this-GPU leg")
    ap.add_argument("--config-steps", type=int, default=20,
                    help="c1: timed steps of the C2 / C3 legs (C4: at least 50)")
    ap.add_argument("--workload", default="c1", choices=["c1", "c2", "c3", "c4"],
                    help="c1 (default, the contract line): b=1 s=64 noul; c2: FP8 16x96; c3: NVFP4 1x512; "
                         "c4: FP8 64 questions s~U[32,512] bucketed by 32, sharded over ranks")
    return ap.parse_args()


def workload(cfg, seed=0):
    from laya_b200.workload import synthetic_items, pack
    items = synthetic_items([64], ["noul"], seed=seed, vocab=cfg.vocab)
    return items, pack(items, 1, 64, 2, cfg.pad_token_id)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def gemm_bytes(cfg, b, s, k, precision):
    """Algorithmic bytes of one forward's projection kernels: each weight read
    once (plus fp8 row scales), each activation operand read once, each output
    written once (a residual epilogue reads and writes fp32).  On the batch-1
    bf16 path (32 < s <= 64) the Wo kernel reads q, k, v (attention fused) and
    writes LayerNorm tile statistics, and the QKV (layers > 0) / Wi kernels read
    the fp32 rows, their statistics and the norm weight (LayerNorm on load)."""
    T, R, BK = b * s, b * (1 + k), b * k
    d, I, F = cfg.hidden, cfg.intermediate, cfg.head_ff
    wb = 1 if precision == "fp8" else 2
    short = precision == "bf16" and b == 1 and 32 < s <= 64
    stats = T * (d // 128) * 8
    total, launches = 0, 0

    def g(M, N, K, wbytes, xbytes, obytes, extra=0):
        nonlocal total, launches
        total += N * K * wbytes + M * K * xbytes + M * N * obytes + (N * 4 if wbytes == 1 else 0) + extra
        launches += 1

    for i in range(cfg.layers):
        if short:
            if i == 0:
                g(T, 3 * d, d, 2, 2, 2)
            else:
                g(T, 3 * d, d, 2, 4, 2, stats + 4 * d)          # LN(h) on load
            g(T, d, d, 2, 0, 8, T * 3 * d * 2 + stats)          # q, k, v in; statistics out
            g(T, 2 * I, d, 2, 4, 1, stats + 4 * d)              # LN(h) on load, GEGLU out
            g(T, d, I, 2, 2, 8, stats if i + 1 < cfg.layers else 0)
            continue
        g(T, 3 * d, d, wb, wb, 2)
        g(T, d, d, wb, wb, 8)
        g(T, 2 * I, d, wb, wb, 1)   # GEGLU writes I outputs for 2I rows
        g(T, d, I, wb, wb, 8)
    for j in range(cfg.head_layers):
        rows = R if j == cfg.head_layers - 1 else T
        g(T, 3 * d, d, 2, 2, 2)
        g(rows, d, d, 2, 2, 8)
        g(rows, F, d, 2, 2, 2)
        g(rows, d, F, 2, 2, 8)
    g(BK, d, d, 2, 2, 2)
    return total, launches


def forward_bytes(cfg, precision):
    """Whole-forward algorithmic bytes at batch 1: every matrix weight read
    once (the survey's bytes_alg: 739,251,200 B in bf16 for the Laya shape)."""
    d, I, F, A = cfg.hidden, cfg.intermediate, cfg.head_ff, cfg.act_hidden
    wb = 1 if precision == "fp8" else 2
    enc = cfg.layers * (3 * d * d + d * d + 2 * I * d + d * I) * wb
    head = cfg.head_layers * (3 * d * d + 3 * d + d * d + d + F * d + F + d * F + d) * 2
    tail = (d * d + d + d + 1) * 2 + (A * (d + 4) + A + 2 * A + 2) * 2
    return enc + head + tail


class ClockSampler:
    """nvidia-smi samples during the timed region (clocks, throttle reasons)."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu = gpu
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *_):
        if self.proc:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for name, val in zip(names, parts[4:8]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def _reference_cpu_model(cfg, weights):
    """The reference's FastDecisionModel on the CPU (RoPE shim), or None with
    the reason when the reference package cannot be imported."""
    try:
        from baseline import laya_net
        return laya_net.build(cfg, weights, "cpu", rope="shim"), None
    except Exception as exc:  # noqa: BLE001 - any import / build failure falls back to the port
        return None, f"{type(exc).__name__}: {exc}"


def cpu_baseline(cfg, seconds, precision="bf16", max_steps=None, warmup=1, weights=None):
    """Time the reference's own CPU forward on this host (`warmup` untimed
    forwards first, bounded to a quarter of `seconds`); the oracle port when
    the reference cannot be imported."""
    import torch
    from laya_b200.weights import seeded_weights
    torch.set_num_threads(os.cpu_count() or 1)
    w = weights if weights is not None else seeded_weights(cfg, seed=0)
    _, inp = workload(cfg)
    model, why = _reference_cpu_model(cfg, w)
    if model is not None:
        from baseline import laya_net
        kind = "reference"
        tin = {k: torch.from_numpy(v) for k, v in inp.items()}
        laya_net.use_rope("shim")

        def fwd():
            with torch.inference_mode():
                model(**tin, global_attention_unmasked=True)
        what = ("the reference's FastDecisionModel.forward (baseline/_ref, bf16 Linears, fp32 residuals; its "
                "Triton RoPE replaced by the torch restatement of tests/test_kernels.py:42-49)")
    else:
        from oracle.laya_oracle import Oracle
        kind = "port"
        orc = Oracle(w, cfg, precision, bf16_gemm=True)  # bf16 Linears as the reference runs them on a CPU

        def fwd():
            orc.forward(**inp)
        what = (f"oracle/laya_oracle.py port (reference not importable: {why}), bf16 Linears through torch's "
                "bf16 GEMM as the reference's nn.Linear runs on a CPU")
    warm, t_warm = 0, time.perf_counter() + seconds / 4
    while warm < max(1, warmup) and (warm == 0 or time.perf_counter() < t_warm):
        fwd()
        warm += 1
    times = []
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end and (max_steps is None or len(times) < max_steps):
        t0 = time.perf_counter()
        fwd()
        times.append(time.perf_counter() - t0)
    total = sum(times)
    return {"value": len(times) / total, "unit": UNIT, "cores": torch.get_num_threads(), "kind": kind,
            "sample": f"{len(times)} forwards of b=1 s=64 noul (one decision each), {total:.1f} s, {what}, "
                      f"on {os.cpu_count()} host cores",
            "ms_per_forward": 1000 * total / len(times), "steps": len(times), "warmup": warm}


def cpu_fp32_restatement(cfg, seconds, weights):
    """BASELINE config 0's "CPU fp32", labelled as a restatement: the oracle
    port (oracle/laya_oracle.py) with every Linear in fp32 (bf16-valued
    weights, fp32 accumulation) on all host cores, a bounded sample of the
    same C0 request."""
    import torch
    from oracle.laya_oracle import Oracle
    torch.set_num_threads(os.cpu_count() or 1)
    _, inp = workload(cfg)
    orc = Oracle(weights, cfg, "bf16")
    orc.forward(**inp)
    times = []
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end:
        t0 = time.perf_counter()
        orc.forward(**inp)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    return {"value": len(times) / total, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "ms_per_forward": 1000 * total / len(times),
            "sample": f"{len(times)} forwards of b=1 s=64 noul, {total:.1f} s, oracle/laya_oracle.py restatement "
                      "with fp32 Linears (fp32 accumulation of the bf16-valued weights), labelled as a "
                      f"restatement, on {os.cpu_count()} host cores"}


def dist_setup(n):
    if n <= 1 and "WORLD_SIZE" not in os.environ:
        return 0, 1, 0, None
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    return rank, world, local, dist


def run_reference(args):
    rank, world, local, dist = 0, 1, 0, None
    if "WORLD_SIZE" in os.environ and int(os.environ["WORLD_SIZE"]) > 1:
        if int(os.environ.get("RANK", "0")) != 0:
            return 0
    from laya_b200.config import LAYA
    budget = max(10.0, min(120.0, args.cpu_seconds * 4))
    base = cpu_baseline(LAYA, budget, max_steps=args.steps, warmup=args.warmup)
    if base["kind"] != "reference":
        print(f"reference arm: the reference could not be imported, timing the oracle port "
              f"({base['sample']})", file=sys.stderr)
    steps = base["steps"]
    line = {"metric": METRIC, "value": base["value"], "unit": UNIT, "n_gpus": args.gpus, "steps": steps,
            "requested_steps": args.steps, "warmup": base["warmup"], "ms_per_step": base["ms_per_forward"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": "C1: b=1, s=64, one noul question (k=2), bf16 weights",
                       "model": "Laya 28x1024 encoder + 2-layer head, seeded N(0,0.02) weights"},
            "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def encoder_flops(cfg, items):
    """Algorithmic FLOPs of one forward over the valid tokens of `items`:
    encoder projections 2*params*tokens, attention 4*d*sum(visible keys),
    head layers (last one on 1+k rows) and the scorer."""
    d, I, F, H = cfg.hidden, cfg.intermediate, cfg.head_ff, cfg.layers
    proj = 3 * d * d + d * d + 2 * I * d + d * I
    fl = 0
    for it in items:
        n, k = len(it["ids"]), len(it["markers"])
        fl += 2 * proj * n * H
        for layer in range(H):
            if cfg.is_global(layer):
                keys = n * n
            else:
                w = cfg.window
                keys = sum(min(n, i + w + 1) - max(0, i - w) for i in range(n))
            fl += 4 * d * keys
        fl += 2 * (3 * d * d + d * d + 2 * F * d) * n                     # head layer 0
        fl += 2 * (2 * d * d) * n + 2 * (d * d + d * d + 2 * F * d) * (1 + k) + 4 * d * n * (1 + k)  # last layer
        fl += 2 * d * d * k
    return fl


def batched_plan(w, cfg):
    """(precision, sequence buckets, list of steps' items) of workload c2 / c3 / c4."""
    from laya_b200.workload import synthetic_items, mixed_kinds
    from laya_b200.dispatcher import c4_step
    if w == "c2":
        return "fp8", (96,), [synthetic_items([96] * 16, mixed_kinds(16, s), seed=100 + s, vocab=cfg.vocab)
                              for s in range(2)]
    if w == "c3":
        return "nvfp4", (512,), [synthetic_items([512], ["choice"], seed=200 + s, vocab=cfg.vocab) for s in range(2)]
    return "fp8", tuple(range(32, 513, 32)), [c4_step(300 + s, cfg.vocab) for s in range(4)]


def _barrier(dist):
    import torch
    if dist:
        dist.barrier()
    torch.cuda.synchronize()


def _max_over_ranks(dist, x):
    if not dist:
        return x
    import torch
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def measure_batched(w, cfg, weights, local, rank, world, dist, steps, warmup, lanes=1):
    """C2 / C3 / C4 through the public engine API on this rank's share of each
    step (C4 shards its questions over the ranks by LPT; C2 / C3 run whole on
    every rank).  Returns the measurement dict (every rank computes it; the
    values are maxima over ranks)."""
    from laya_b200.engine import B200Engine, request_from_items
    from laya_b200.dispatcher import shard_groups, group_by_bucket
    precision, buckets, steps_items = batched_plan(w, cfg)
    lanes = max(1, lanes) if w == "c4" else 1   # C4 steps hold several bucket groups
    eng = B200Engine(config=cfg, weights=weights, device=local, precision=precision, max_questions=64,
                     max_options=4, max_graphs=512, sequence_buckets=buckets, lanes=lanes)
    try:
        plans = []
        shard = w == "c4" and world > 1
        for items in steps_items:
            # C4 under torchrun: this rank's LPT share of the step's bucket groups
            groups = shard_groups(items, world, buckets, 64)[rank] if shard else \
                group_by_bucket(items, list(range(len(items))), buckets, 64)
            plans.append([request_from_items([items[i] for i in idx]) for _, idx in groups])
        for plan in plans * max(1, warmup // len(plans)):     # captures every shape, then warm
            for req in plan:
                eng._run_on(req, eng)
        for lane in eng._lanes[1:]:                  # every lane holds every shape's graph
            for plan in plans:
                for req in plan:
                    eng._run_on(req, lane)
        # device time per step: the step's graphs replayed back to back with inputs resident
        dev_ms, launches = [], 0
        for plan in plans:
            t = 0.0
            for req in plan:
                eng._run_on(req, eng)                 # lane 0: its staging buffer now holds req
                slot = eng.graphs[eng._graph_key(req)]
                t += float(np.mean(eng.native.replay_device(slot, 5)))
                launches += 5 * eng.native.kernel_count(slot)
            dev_ms.append(t)
        with ClockSampler(local) as clocks:
            _barrier(dist)
            t0 = time.perf_counter()
            for k in range(steps):
                for req in plans[k % len(plans)]:
                    eng.run_prepared(req)
            wall = _max_over_ranks(dist, time.perf_counter() - t0)
            _barrier(dist)
        # serving lanes (C4): the step's bucket groups dispatched concurrently,
        # one caller thread per lane; host wall clock over the steps
        lanes_line = None
        if lanes > 1:
            from concurrent.futures import ThreadPoolExecutor
            with ThreadPoolExecutor(max_workers=lanes) as pool:
                for plan in plans:
                    list(pool.map(eng.run_prepared, plan))
                _barrier(dist)
                t0 = time.perf_counter()
                for k in range(steps):
                    list(pool.map(eng.run_prepared, plans[k % len(plans)]))
                lanes_wall = _max_over_ranks(dist, time.perf_counter() - t0)
                _barrier(dist)
            lanes_line = {"lanes": lanes,
                          "value": steps * sum(len(it) for it in steps_items) / len(steps_items) / lanes_wall,
                          "unit": UNIT, "ms_per_step": 1000 * lanes_wall / steps,
                          "timing": "host wall clock, bucket groups of a step on concurrent lanes (public API, "
                                    "host buffers)"}
    finally:
        eng.close()
    questions = sum(len(it) for it in steps_items) / len(steps_items)
    dev_step = _max_over_ranks(dist, float(np.mean(dev_ms)))
    # C4 is sharded: the whole step's questions in the slowest rank's time;
    # C2 / C3 run whole on every rank: world x questions
    served = questions if shard else questions * world
    value = served / (dev_step / 1000.0)
    e2e = steps * served / wall
    flops = float(np.mean([encoder_flops(cfg, items) for items in steps_items]))
    d = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    bf16_peak = float(d.get("bf16_tflops", 1590.0))
    mult = 2 if precision == "fp8" else 4 if precision == "nvfp4" else 1
    peak = mult * bf16_peak
    # per GPU: the step's FLOPs (C4: divided over the ranks) in the slowest rank's device time
    achieved = flops * (served / questions) / world / (dev_step / 1000.0) / 1e12
    return {"metric": "decisions/s", "value": value, "unit": UNIT, "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": dev_step, "higher_is_better": True,
            "scaling": "strong" if shard else "weak",
            "dtype": {"fp8": "e4m3", "nvfp4": "e2m1"}[precision],
            "config": {"workload": w, "precision": precision, "questions_per_step": questions,
                       "buckets": list(buckets) if len(buckets) < 5 else "multiples of 32 up to 512",
                       "parallelism": (f"LPT shards of each step's bucket groups over {world} ranks" if shard else
                                       f"request-parallel replicas x{world}")},
            "e2e": {"value": e2e, "unit": UNIT, "path": "B200Engine.run_prepared per bucket group"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "flops_per_step": flops,
                         "peak_source": f"{mult}x measured cuBLAS bf16 (MEASURED_PEAKS.json)"},
            **({"serving_lanes": lanes_line} if lanes_line else {}),
            "gpu_launches": launches, "clocks": clocks.summary()}


def run_batched(args):
    """--workload c2 / c3 / c4: one JSON line of that workload."""
    rank, world, local, dist = dist_setup(args.gpus)
    from laya_b200.config import LAYA
    from laya_b200.weights import seeded_weights
    weights = seeded_weights(LAYA, seed=0)
    line = measure_batched(args.workload, LAYA, weights, local, rank, world, dist, args.steps, args.warmup,
                           args.lanes)
    if rank == 0:
        line["vs_baseline"] = None
        line["data"] = "synthetic"
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def reference_gpu(cfg, weights, local, steps, warmup):
    """The reference's own path on this GPU: FastDecisionModel with its Triton
    RoPE, each shape captured in a CUDA graph after three eager warm-ups on a
    side stream, as BlackwellEngine._slot does (src/laya_blackwell/engine.py:
    161-187); device time of back-to-back replays with inputs resident (CUDA
    events), and end to end as BlackwellEngine.run_prepared runs it (pinned
    host inputs copied into the graph's inputs, replay, outputs copied back).
    FP8 uses the reference's replace_encoder_linears (FP8Linear)."""
    import torch
    from baseline import laya_net
    from laya_b200.workload import synthetic_items, pack, mixed_kinds
    dev = torch.device("cuda", local)
    out = {"path": "baseline/_ref laya_blackwell.model.FastDecisionModel, Triton rope_qkv, torch.cuda.graph"}
    cases = [("c1_bf16", "bf16", synthetic_items([64], ["noul"], seed=0, vocab=cfg.vocab), 1, 64, 2),
             ("c3_bf16", "bf16", synthetic_items([512], ["choice"], seed=200, vocab=cfg.vocab), 1, 512, 4),
             ("c1_fp8", "fp8", synthetic_items([64], ["noul"], seed=0, vocab=cfg.vocab), 1, 64, 2),
             ("c2_fp8", "fp8", synthetic_items([96] * 16, mixed_kinds(16, 0), seed=100, vocab=cfg.vocab), 16, 96, 4)]
    model = laya_net.build(cfg, weights, dev, rope="native")
    fp8 = False
    for name, precision, items, b, s, k in cases:
        if precision == "fp8" and not fp8:
            laya_net.import_reference("quantization").replace_encoder_linears(model)
            fp8 = True
        laya_net.use_rope("native")
        host = {kk: torch.from_numpy(v).pin_memory() for kk, v in pack(items, b, s, k, cfg.pad_token_id).items()}
        host["marker_mask"] = host["marker_mask"].bool()
        unmasked = len(items) == b and all(len(it["ids"]) == s for it in items)
        with torch.inference_mode():
            inputs = {kk: v.to(dev) for kk, v in host.items()}
            stream = torch.cuda.Stream(device=dev)
            stream.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(stream):
                for _ in range(3):
                    model(**inputs, global_attention_unmasked=unmasked)
            torch.cuda.current_stream(dev).wait_stream(stream)
            torch.cuda.synchronize(dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                outputs = model(**inputs, global_attention_unmasked=unmasked)
            for _ in range(warmup):
                graph.replay()
            torch.cuda.synchronize(dev)
            n = steps if s <= 96 else max(10, steps // 8)
            evs = [torch.cuda.Event(enable_timing=True) for _ in range(n + 1)]
            cur = torch.cuda.current_stream(dev)
            evs[0].record(cur)
            for i in range(n):
                graph.replay()
                evs[i + 1].record(cur)
            torch.cuda.synchronize(dev)
            ms = [evs[i].elapsed_time(evs[i + 1]) for i in range(n)]
            out_host = [torch.empty_like(o, device="cpu").pin_memory() for o in outputs]
            t0 = time.perf_counter()
            for _ in range(n):
                for kk, v in host.items():
                    inputs[kk].copy_(v, non_blocking=True)
                graph.replay()
                for o, h in zip(outputs, out_host):
                    h.copy_(o, non_blocking=True)
                torch.cuda.synchronize(dev)
            e2e_s = (time.perf_counter() - t0) / n
            del graph
        dev_ms = float(np.mean(ms))
        out[name] = {"precision": precision, "shape": [b, s, k], "questions": len(items), "ms_per_step": dev_ms,
                     "p50_ms": float(np.median(ms)), "value": len(items) / (dev_ms / 1000.0), "unit": UNIT,
                     "e2e": {"value": len(items) / e2e_s, "unit": UNIT, "ms_per_step": 1000 * e2e_s},
                     "steps": n}
    del model
    torch.cuda.empty_cache()
    return out


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload != "c1":
        return run_batched(args)
    if args.warmup < 3:
        raise SystemExit("--warmup must be at least 3")
    rank, world, local, dist = dist_setup(args.gpus)
    import torch
    from laya_b200.config import LAYA
    from laya_b200.engine import B200Engine, request_from_items
    from laya_b200.weights import seeded_weights
    cfg = LAYA
    weights = seeded_weights(cfg, seed=0)
    eng = B200Engine(config=cfg, weights=weights, device=local, precision=args.precision, max_questions=1,
                     max_options=2, max_graphs=2, lanes=max(1, args.lanes), token_tables=args.token_tables)
    items, inp = workload(cfg, seed=rank)
    prepared = request_from_items(items)
    logits, act, meta = eng._run_on(prepared, eng)  # lane 0: captures the graph, inputs now resident
    slot = eng.graphs[(1, 64, 2, True)]
    native = eng.native
    kernels = native.kernel_count(slot)
    native.replay_device(slot, args.warmup)

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if not dist:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident throughput and latency (the value)
    with ClockSampler(local) as clocks:
        barrier()
        ms = native.replay_device(slot, args.steps)
        barrier()
    total_ms = max_over_ranks(float(ms.sum()))
    value = world * args.steps / (total_ms / 1000.0)
    p50 = float(np.median(ms))

    # ---- end to end through the public API (host buffers, H2D + D2H per step)
    for _ in range(args.warmup):
        eng.run_prepared(prepared)
    e2e_steps = min(args.steps, 2000)
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        eng.run_prepared(prepared)
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    barrier()
    e2e_value = world * e2e_steps / e2e_s
    b, s, k = 1, 64, 2
    h2d = 4 * (2 * b * s + b + 2 * b * k + 2 * b * (1 + k))
    d2h = 4 * (b * k + 2 * b)

    # ---- serving lanes: the same request replayed on every lane at once
    # (one GPU serving several requests concurrently); supplementary to the
    # single-lane value, host wall clock around the concurrent device loops
    lanes_line = None
    if args.lanes > 1:
        key = (1, 64, 2, True)
        lane_slots = []
        for lane in eng._lanes:
            eng._run_on(prepared, lane)          # captures the lane's graph
            lane_slots.append((lane.native, lane.graphs[key]))
            lane.native.replay_device(lane.graphs[key], args.warmup)
        lane_ms = [None] * len(lane_slots)

        def replay(i):
            lane_ms[i] = lane_slots[i][0].replay_device(lane_slots[i][1], args.steps)

        threads = [threading.Thread(target=replay, args=(i,)) for i in range(len(lane_slots))]
        barrier()
        t0 = time.perf_counter()
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        lanes_s = max_over_ranks(time.perf_counter() - t0)
        barrier()
        lanes_line = {"lanes": len(lane_slots), "value": world * len(lane_slots) * args.steps / lanes_s,
                      "unit": UNIT, "p50_ms": float(np.median(np.concatenate(lane_ms))),
                      "timing": "host wall clock around concurrent device replay loops, one per lane"}

    # ---- roofline of the dominant kernel family (projection GEMMs)
    gms = native.replay_device(slot, max(20, min(args.steps, 500)), kernel_mask=1)
    gemm_ms = float(np.mean(gms))
    gbytes, glaunch = gemm_bytes(cfg, b, s, k, args.precision)
    peak, peak_kind = peaks()
    achieved = gbytes / (gemm_ms / 1000.0) / 1e9
    fwd_bytes = forward_bytes(cfg, args.precision)
    fwd_achieved = fwd_bytes / (float(np.mean(ms)) / 1000.0) / 1e9
    traffic = None
    tfile = ROOT / "profiles" / f"gemm_{args.precision}_c1_traffic.txt"
    if tfile.exists():
        for line in tfile.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                traffic = float(line.split(":", 1)[1])

    eng.close()

    # ---- the other BASELINE configs, bounded (every rank takes part)
    configs = {}
    if not args.no_configs:
        for w in ("c2", "c3", "c4"):
            n = args.config_steps if w != "c4" else max(50, args.config_steps)  # C4: >= 50 steps
            configs[w] = measure_batched(w, cfg, weights, local, rank, world, dist, n, 3, lanes=1)

    ref_gpu = None
    if rank == 0 and not args.no_reference_gpu:
        try:
            ref_gpu = reference_gpu(cfg, weights, local, min(args.steps, 200), 3)
        except Exception as exc:  # noqa: BLE001 - reported in the line, not fatal
            ref_gpu = {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}
    _barrier(dist)

    if rank == 0:
        base = cpu_baseline(cfg, args.cpu_seconds, args.precision, weights=weights)
        fp32 = cpu_fp32_restatement(cfg, min(5.0, args.cpu_seconds / 3), weights)
        cs = clocks.summary()
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "p50_ms": p50,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": args.precision,
            "data": "synthetic (seeded token ids, seeded N(0,0.02) random-init weights of the 28x1024 Laya shape)",
            "config": {"workload": "C1: one short noul question, b=1, s=64, k=2, warm CUDA-graph replay"
                                   + (", token tables" if args.token_tables else ""),
                       "model": "Laya: ModernBERT-large-shaped 28x1024 encoder + 2-layer head + scorer",
                       "global_batch": world, "seq_len": 64,
                       "parallelism": f"request-parallel replicas x{world} (no collective)",
                       "l2": f"inputs larger than L2: {fwd_bytes / 1e6:.0f} MB of weights streamed per step"},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "path": "B200Engine.run_prepared -> laya_b200_run (pinned pack, H2D, graph, D2H)"},
            "roofline": {"bound": "hbm",
                         "kernel": "projection kernels of one forward: gemm_kernel, gemm_attn_kernel (Wo with the "
                                   "attention fused), gemm_ln_kernel (QKV / Wi with LayerNorm on load)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": traffic, "peak_source": peak_kind,
                         "launches_per_forward": glaunch, "algorithmic_bytes_per_launch": gbytes / glaunch,
                         "avg_launch_us": 1000 * gemm_ms / glaunch},
            "forward_roofline": {"bytes_alg": fwd_bytes, "achieved_gbs": fwd_achieved,
                                 "frac": fwd_achieved / peak},
            "cpu_baseline": {**{k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
                             "fp32_restatement": fp32},
            **({"serving_lanes": lanes_line} if lanes_line else {}),
            "gpu_launches": kernels * args.steps,
            "kernels_per_forward": kernels,
            "clocks": cs,
            **({"configs": configs} if configs else {}),
            **({"reference_gpu": ref_gpu} if ref_gpu else {}),
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
