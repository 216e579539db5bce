"""Benchmark of the B200 verify path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload sweep]
    python bench.py --impl reference ...      # the reference's CPU kernels

Workload "sweep": one step = one verify dequant-GEMV at
N=5 columns (draft length 4 + 1) over each of the 16 seeded weights
(Q4_K/Q5_K/Q6_K/Q8_0 x 4096x4096, 12288x4096, 4096x12288, 151936x4096),
weights resident in HBM (2.3 GB per step, larger than the 126 MB L2, so
every step streams them from DRAM).  value = quantized weight bytes streamed
per second (all ranks); `roofline` is the largest launch (Q4_K 151936x4096).

Multi-GPU: every rank runs the same sweep on its own GPU (replicas, no
collective); value sums the ranks' bytes over the max-over-ranks time.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "spec-decode tokens/s/GPU (Qwen3.5-shape Q4_K); verify dequant-GEMV % HBM peak"
SHAPES = [(4096, 4096), (12288, 4096), (4096, 12288), (151936, 4096)]
FORMATS = [(12, "Q4_K"), (13, "Q5_K"), (14, "Q6_K"), (8, "Q8_0")]
NCOLS = 5
BPW = {12: 144 / 256, 13: 176 / 256, 14: 210 / 256, 8: 34 / 32}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region"""

    def __init__(self, index):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4)
                          if len(r) > 3 + i and r[3 + i].lower().startswith("active")})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def dist_init():
    import torch
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl" if torch.cuda.is_available() else "gloo",
                                timeout=datetime.timedelta(seconds=120))
    return ws, rank, local


def max_over_ranks(v, ws):
    if ws == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def make_weights(O, qt, M, K, rng):
    """seeded N(0, 0.02) weights in `qt`: a 2048-row encoded pool tiled to M rows"""
    rb = O.row_bytes(qt, K)
    pool_rows = min(M, 2048)
    pool = O.quantize(qt, rng.normal(0, 0.02, (pool_rows, K)).astype(np.float32)).reshape(pool_rows, rb)
    idx = np.arange(M) % pool_rows
    return pool[idx].ravel()


# ------------------------------------------------------------------ ours ----

def run_ours(args):
    import torch
    import __graft_entry__ as ge
    ws, rank, local = dist_init()
    torch.cuda.set_device(local)
    pkg = ge.load_package()
    pkg.load()
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O  # noqa: E402  (encoder for the synthetic weights only)
    ctx = pkg.Context(local)
    rng = np.random.default_rng(1234)
    Ws, Xs, Ys, byts = [], [], [], []
    for qt, name in FORMATS:
        for (M, K) in SHAPES:
            q = make_weights(O, qt, M, K, rng)
            W = ctx.upload(qt, q, M, K)
            Ws.append(W)
            Xs.append(torch.from_numpy(rng.normal(0, 1, (NCOLS, K)).astype(np.float32)).cuda())
            Ys.append(torch.empty(NCOLS, M, dtype=torch.float32, device="cuda"))
            byts.append(W.algorithmic_bytes())
    step_bytes = sum(byts)
    stream = torch.cuda.current_stream()
    big_i = FORMATS.index((12, "Q4_K")) * len(SHAPES) + SHAPES.index((151936, 4096))

    def step(events=None):
        for i, W in enumerate(Ws):
            if events is not None and i == big_i:
                events[0].record(stream)
            ctx.qgemm(W, Xs[i], Ys[i])
            if events is not None and i == big_i:
                events[1].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(ws)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t0.record(stream)
        for k in range(args.steps):
            step(ev[k])
        t1.record(stream)
        torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    barrier(ws)
    ms_max = max_over_ranks(ms, ws)
    big_ms = float(np.mean([a.elapsed_time(b) for a, b in ev]))

    # end to end through the C ABI with host buffers: pinned X in, Y out, every call
    hX = [x.cpu().pin_memory() for x in Xs]
    hY = [torch.empty(y.shape, dtype=torch.float32).pin_memory() for y in Ys]
    dX = [torch.empty_like(x) for x in Xs]

    def e2e_step():
        for i, W in enumerate(Ws):
            dX[i].copy_(hX[i], non_blocking=True)
            ctx.qgemm(W, dX[i], Ys[i])
            hY[i].copy_(Ys[i], non_blocking=True)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    barrier(ws)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), ws)
    h2d = sum(x.numel() * 4 for x in hX)
    d2h = sum(y.numel() * 4 for y in hY)

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(O, args)
    if rank == 0:
        peak, peak_kind = measured_peaks()
        big_bytes = byts[big_i]
        achieved = big_bytes / (big_ms * 1e-3) / 1e9
        value = step_bytes * args.steps * ws / (ms_max * 1e-3) / 1e9
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": ws,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_max / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "q4_k/q5_k/q6_k/q8_0 weights, f32 activations (fp16 hi+lo split), f32 accumulate",
            "data": "synthetic: seeded N(0,0.02) weights encoded by the repo's own K-quant encoder, N(0,1) activations",
            "config": {"workload": "verify GEMV sweep (BASELINE config 2)", "ncols": NCOLS,
                       "shapes": [f"{m}x{k}" for m, k in SHAPES], "formats": [n for _, n in FORMATS],
                       "weight_bytes_per_step": step_bytes,
                       "l2": "inputs larger than L2: %.2f GB of weights per step" % (step_bytes / 1e9),
                       "parallelism": f"replicas x{ws}"},
            "per_gpu_GBps": round(value / ws, 2),
            "hbm_frac_of_measured_peak": round(value / ws / peak, 4),
            "roofline": {"bound": "hbm", "kernel": "qgemv Q4_K 151936x4096 N=5",
                         "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": None, "algorithmic_bytes_per_launch": big_bytes,
                         "launch_ms": round(big_ms, 5)},
            "e2e": {"value": round(step_bytes * args.steps * ws / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": len(Ws) * args.steps,
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    barrier(ws)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# --------------------------------------------------------- CPU reference ----

def ref_sample(O, rng, seconds_budget):
    """Bounded sample of the sweep for the CPU: 4096x4096 and 12288x4096 of
    every format, N=5 columns each as 5 single-column calls (how the
    reference's forward_cpu! runs the verify tokens)."""
    items = []
    for qt, name in FORMATS:
        for (M, K) in SHAPES[:2]:
            items.append((qt, name, M, K, make_weights(O, qt, M, K, rng),
                          rng.normal(0, 1, (NCOLS, K)).astype(np.float32)))
    return items


def time_ref_sample(O, items):
    t = time.perf_counter()
    nbytes = 0
    for qt, name, M, K, q, X in items:
        for n in range(NCOLS):
            O.ref_gemv(qt, q, M, K, X[n])
        nbytes += M * O.row_bytes(qt, K)
    return nbytes, time.perf_counter() - t


def cpu_baseline(O, args):
    if not O.ref_available():
        return {"value": None, "unit": "GB/s", "cores": 0, "kind": "reference",
                "sample": "oracle/_ref/libquant_ref.so missing"}
    cores = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(cores))
    rng = np.random.default_rng(99)
    items = ref_sample(O, rng, 20)
    time_ref_sample(O, items)  # warm-up
    nb, dt = time_ref_sample(O, items)
    return {"value": round(nb / dt / 1e9, 3), "unit": "GB/s", "cores": int(os.environ["OMP_NUM_THREADS"]),
            "kind": "reference",
            "sample": "reference quant_kernels.c (AVX2+OpenMP, built from source) over 4096x4096 and "
                      "12288x4096 of Q4_K/Q5_K/Q6_K/Q8_0, N=5 as 5 single-column calls; q8_0_gemv is "
                      "single-threaded in the reference", "seconds": round(dt, 2)}


def run_reference(args):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    if not O.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libquant_ref.so not built"}))
        return
    cores = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(cores))
    rng = np.random.default_rng(99)
    items = ref_sample(O, rng, 20)
    for _ in range(args.warmup):
        time_ref_sample(O, items)
    tot_b, tot_t = 0, 0.0
    for _ in range(args.steps):
        b, t = time_ref_sample(O, items)
        tot_b += b
        tot_t += t
    value = tot_b / tot_t / 1e9
    sample = ("reference quant_kernels.c on host cores: 4096x4096 and 12288x4096 of all four formats, "
              "N=5 as 5 single-column calls per step")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(tot_t / args.steps * 1e3, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "q-weights, Q8_K activations (reference)", "data": "synthetic",
        "config": {"workload": "verify GEMV sweep (BASELINE config 2), CPU sample", "ncols": NCOLS},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": int(os.environ["OMP_NUM_THREADS"]),
                         "kind": "reference", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="sweep", choices=["sweep"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
