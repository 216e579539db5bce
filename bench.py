"""Benchmark of the B200 verify path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload spec|sweep]
    python bench.py --impl reference ...      # the reference's CPU path

Workload "spec" (default, BASELINE config 1 and its headline metric): greedy
speculative decoding of the seeded tiny Qwen3.5-shape hybrid (hidden 1024, 24
layers, Q4_K matmuls, Q6_K tied embedding/lm_head, one-layer MTP draft head)
after a 128-token seeded prompt; one step = MTP draft of 4 tokens + one
5-column verify forward + greedy acceptance + state rollback, replayed as a
CUDA graph.  value = emitted tokens per second (all ranks).  `roofline` is the
verify's 97 dequant-GEMV launches (all decoder-layer GEMVs + the lm_head of
one step) captured back to back in a CUDA graph and timed with CUDA events.
Every step reads ~964 MB of weights (verify 407 MB + 4 drafts), far above L2.

Workload "sweep": one step = one verify dequant-GEMV at
N=5 columns (draft length 4 + 1) over each of the 16 seeded weights
(Q4_K/Q5_K/Q6_K/Q8_0 x 4096x4096, 12288x4096, 4096x12288, 151936x4096),
weights resident in HBM (2.3 GB per step, larger than the 126 MB L2, so
every step streams them from DRAM).  value = quantized weight bytes streamed
per second (all ranks); `roofline` is the Q4_K 151936x4096 launch (the model's
matmul format), `per_launch` every launch's own time and fraction of peak.

Multi-GPU: every rank runs the same workload on its own GPU (replicas, no
collective); value sums the ranks' units over the max-over-ranks time.

Profiling cases (no JSON line; the launches of interest are bracketed by
cudaProfilerStart/Stop for `ncu --profile-from-start off`):
    python bench.py --profile spec        # 2 graph-replayed spec steps, config 1
    python bench.py --profile qgemv --qtype Q4_K --shape 65536x4096 --ncols 5 [--act 1]
    python bench.py --profile dense --qtype Q4_K --shape 4096x4096 --ncols 320
    python bench.py --profile batch       # 1 graph-replayed step of the batch workload

Workload "batch": the ~9B-shape hybrid, 64 requests with
2048-token seeded prompts (split over the ranks), one step = MTP drafts +
one verify of 64 x 5 columns + acceptance, as a CUDA graph.
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
# arithmetic of the K-quant GEMVs per activation mode (--act); Q8_0 is always exact
ACT_DTYPE = {
    0: "q4_k/q6_k weights x f32 activations, exact products (fp16 hi+lo split on the tensor cores), f32 accumulate",
    1: "q4_k/q6_k weights x Q8_K activations (the reference's quantize_row_q8_K), exact int32 sub-block sums on the integer tensor cores, f32 scaling",
}


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
    t = torch.tensor([v], dtype=torch.float64, device="cuda" if torch.cuda.is_available() else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def rank_requests(total, ws, rank):
    """the requests (seed offsets) rank owns when `total` independent requests
    are split evenly over ws ranks: a contiguous block of total / ws"""
    if total % ws:
        raise SystemExit(f"--batch {total} does not split over {ws} ranks")
    B = total // ws
    return list(range(rank * B, (rank + 1) * B))


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def make_weights(pkg, qt, M, K, rng):
    """seeded N(0, 0.02) weights in `qt` (the library's encoder): a 2048-row
    pool tiled to M rows"""
    rb = pkg.row_bytes(qt, K)
    pool_rows = min(M, 2048)
    pool = pkg.quantize(qt, rng.normal(0, 0.02, (pool_rows, K)).astype(np.float32)).reshape(pool_rows, rb)
    idx = np.arange(M) % pool_rows
    return pool[idx].ravel()


# ------------------------------------------------------------------ ours ----

def run_sweep(args):
    import torch
    import __graft_entry__ as ge
    ws, rank, local = dist_init()
    torch.cuda.set_device(local)
    pkg = ge.load_package()
    pkg.load()
    ctx = pkg.Context(local)
    # the sweep's default is the reference's own kernel arithmetic (q4_k_gemv ..
    # q6_k_gemv quantize the activations to Q8_K); --act 0 makes exact f32 the line's
    act = 1 if args.act is None else args.act
    ctx.set_activation(act)
    rng = np.random.default_rng(1234)
    Ws, Xs, Ys, byts = [], [], [], []
    for qt, name in FORMATS:
        for (M, K) in SHAPES:
            q = make_weights(pkg, qt, M, K, rng)
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

    def timed(act):
        """the K-step sweep in activation mode act: (max-over-ranks ms, mean ms of the big launch)"""
        ctx.set_activation(act)
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(ws)
        torch.cuda.synchronize()
        t0.record(stream)
        for k in range(args.steps):
            step(ev[k])
        t1.record(stream)
        torch.cuda.synchronize()
        ms = t0.elapsed_time(t1)
        barrier(ws)
        return max_over_ranks(ms, ws), float(np.mean([a.elapsed_time(b) for a, b in ev]))

    # the other activation mode first (reported beside the line), then the line's own
    other = 1 - act
    o_ms, o_big = timed(other)
    with ClockSampler(local) as clk:
        ms_max, big_ms = timed(act)
    # every launch's own time in the line's mode: CUDA events around each
    # launch, in a separate pass after the timed region (3 passes, mean)
    per_ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in Ws]
              for _ in range(3)]
    for r in range(3):
        for i, W in enumerate(Ws):
            per_ev[r][i][0].record(stream)
            ctx.qgemm(W, Xs[i], Ys[i])
            per_ev[r][i][1].record(stream)
    torch.cuda.synchronize()
    per_us = [float(np.mean([per_ev[r][i][0].elapsed_time(per_ev[r][i][1]) for r in range(3)])) * 1e3
              for i in range(len(Ws))]

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
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O  # the CPU baseline leg only
        cpu = cpu_baseline(O, pkg, args)
    if rank == 0:
        peak, peak_kind = measured_peaks()
        names = [f"{name} {M}x{K}" for _, name in FORMATS for (M, K) in SHAPES]
        per_launch = {nm: {"us": round(per_us[i], 2), "GBps": round(byts[i] / per_us[i] / 1e3, 1),
                           "frac": round(byts[i] / per_us[i] / 1e3 / peak, 3)} for i, nm in enumerate(names)}
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
            "dtype": ACT_DTYPE[act].replace("q4_k/q6_k", "q4_k/q5_k/q6_k/q8_0"),
            "data": "synthetic: seeded N(0,0.02) weights encoded by the repo's own K-quant encoder, N(0,1) activations",
            "config": {"workload": "verify GEMV sweep (BASELINE config 2)", "ncols": NCOLS, "activations": ["exact f32", "Q8_K"][act],
                       "shapes": [f"{m}x{k}" for m, k in SHAPES], "formats": [n for _, n in FORMATS],
                       "weight_bytes_per_step": step_bytes,
                       "l2": "inputs larger than L2: %.2f GB of weights per step" % (step_bytes / 1e9),
                       "parallelism": f"replicas x{ws}"},
            "per_gpu_GBps": round(value / ws, 2),
            "hbm_frac_of_measured_peak": round(value / ws / peak, 4),
            "per_launch": per_launch,
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
            "other_activation_mode": {
                "activations": ["exact f32", "Q8_K"][other],
                "value": round(step_bytes * args.steps * ws / (o_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "roofline_achieved": round(big_bytes / (o_big * 1e-3) / 1e9, 1),
                "roofline_frac": round(big_bytes / (o_big * 1e-3) / 1e9 / peak, 4)},
        }
        print(json.dumps(line), flush=True)
    barrier(ws)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# --------------------------------------------------------- CPU reference ----

def ref_sample(O, pkg, rng, seconds_budget):
    """Bounded sample of the sweep for the CPU: 4096x4096 and 12288x4096 of
    every format, N=5 columns each as 5 single-column calls (how the
    reference's forward_cpu! runs the verify tokens)."""
    items = []
    for qt, name in FORMATS:
        for (M, K) in SHAPES[:2]:
            items.append((qt, name, M, K, make_weights(pkg, qt, M, K, rng),
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


def cpu_baseline(O, pkg, args):
    if not O.ref_available():
        return {"value": None, "unit": "GB/s", "cores": 0, "kind": "reference",
                "sample": "oracle/_ref/libquant_ref.so missing"}
    cores = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(cores))
    rng = np.random.default_rng(99)
    items = ref_sample(O, pkg, rng, 20)
    time_ref_sample(O, items)  # warm-up
    nb, dt = time_ref_sample(O, items)
    return {"value": round(nb / dt / 1e9, 3), "unit": "GB/s", "cores": int(os.environ["OMP_NUM_THREADS"]),
            "kind": "reference",
            "sample": "reference quant_kernels.c (AVX2+OpenMP, built from source) over 4096x4096 and "
                      "12288x4096 of Q4_K/Q5_K/Q6_K/Q8_0, N=5 as 5 single-column calls; q8_0_gemv is "
                      "single-threaded in the reference", "seconds": round(dt, 2)}


def run_reference_sweep(args):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    import __graft_entry__ as ge
    pkg = ge.load_package()
    if not O.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libquant_ref.so not built"}))
        return
    cores = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(cores))
    rng = np.random.default_rng(99)
    items = ref_sample(O, pkg, rng, 20)
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

# ------------------------------------------------------- spec workload ----

SPEC_PRESET, SPEC_SEED, SPEC_PROMPT = "tiny", 0, 128
SPEC_GEN = 128  # config 1: 128 greedy tokens per request
# DRAM bytes (read + write) of the verify's 97 GEMV launches, from one ncu
# capture of `bench.py --profile spec` (profiles/spec_step_launches_config1.md)
SPEC_VERIFY_TRAFFIC = 418144512


def spec_bytes_per_step_gguf(gf, gamma):
    """spec_bytes_per_step from the GGUF's own tensors (no library loaded):
    quantized bytes of the decoder layers and the lm_head per verify, plus
    per draft the MTP fc, its layer and the lm_head"""
    layers = mtp = 0
    for name, t in gf.tensors.items():
        if t.type in (8, 12, 13, 14) and name != "token_embd.weight":
            nb = t.nbytes
            if name.startswith("mtp."):
                mtp += nb
            else:
                layers += nb
    lm = gf.tensors["token_embd.weight"]
    lm_b = lm.nbytes
    return layers + lm_b + gamma * (mtp + lm_b)


def spec_bytes_per_step(info, gamma):
    """algorithmic weight bytes one spec step reads: the verify (decoder layers
    + lm_head) and, per draft, the MTP fc + layer + lm_head"""
    # fc (hidden x 2 hidden) + one attention layer, same formats as the target
    d, hd = info.hidden, info.head_dim
    mtp_rows_k = [(d, 2 * d), ((2 * info.n_head + 2 * info.n_kv_head) * hd, d), (d, info.n_head * hd),
                  (2 * info.ffn, d), (d, info.ffn)]
    mtp = sum(r * k for r, k in mtp_rows_k) * 144 // 256
    lm = info.vocab * d * 210 // 256
    return info.weight_bytes + gamma * (mtp + lm)


def spec_config(G, step_bytes, ws):
    """the config-1 workload, identical on both arms"""
    return {"workload": "greedy spec-decode, BASELINE config 1 (tiny Qwen3.5-shape hybrid)",
            "model": "hidden 1024, 24 layers (18 GatedDeltaNet + 6 attention), 8q/2kv x 256, FFN 3584, vocab 151936, 1-layer MTP head",
            "gamma": G, "verify_columns": G + 1, "prompt": SPEC_PROMPT, "batch": 1,
            "weight_bytes_per_step": int(step_bytes),
            "l2": "inputs larger than L2: %.0f MB of weights read per step" % (step_bytes / 1e6),
            "parallelism": f"replicas x{ws}"}


def run_spec(args):
    import torch
    import __graft_entry__ as ge
    ws, rank, local = dist_init()
    torch.cuda.set_device(local)
    pkg = ge.load_package()
    pkg.load()
    from inferno_b200 import synth
    from inferno_b200.engine import Model, State
    G = args.gamma
    ctx = pkg.Context(local, torch_stream=False)  # own stream: capturable
    ctx.set_activation(args.act)
    ctx.set_fused_layers(bool(args.fused_layers))
    path = synth.cached(SPEC_PRESET, SPEC_SEED)
    model = Model(ctx, path)
    info = model.info
    prompt = synth.prompt(info.vocab, SPEC_PROMPT, SPEC_SEED)
    max_ctx = SPEC_PROMPT + (args.warmup + 2 * args.steps + 8) * (G + 1) + 16
    st = State(model, max_ctx)
    st.prefill(prompt)
    st.spec_step(G)  # eager step: every kernel initialised before capture
    st.capture(G, 1)
    import ctypes
    sp = ctypes.c_void_p()
    pkg.check(pkg.load().ifr_ctx_get_stream(ctx.handle, ctypes.byref(sp)))
    stream = torch.cuda.ExternalStream(sp.value)
    for _ in range(args.warmup):
        st.launch()
    ctx.sync()
    n0 = len(st.read()[0])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(ws)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            st.launch()
        e1.record(stream)
        e1.synchronize()
    ms = e0.elapsed_time(e1)
    toks, pos, acc, nsteps = st.read()
    emitted = len(toks) - n0
    barrier(ws)
    ms_max = max_over_ranks(ms, ws)
    # the verify's dequant-GEMV launches alone (24 layers x 4 + lm_head, N = G+1
    # columns), back to back in a captured graph, timed with CUDA events
    gs = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    st.gemv_pass(G + 1)  # warm
    ctx.sync()
    pkg.check(pkg.load().ifr_ctx_set_stream(ctx.handle, ctypes.c_void_p(gs.cuda_stream)))
    with torch.cuda.graph(g, stream=gs):
        st.gemv_pass(G + 1)
    pkg.check(pkg.load().ifr_ctx_set_stream(ctx.handle, sp))
    torch.cuda.synchronize()
    reps = max(3, args.steps // 4)
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    v0, v1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    v0.record()
    for _ in range(reps):
        g.replay()
    v1.record()
    v1.synchronize()
    v_ms = v0.elapsed_time(v1) / reps
    v_bytes = info.weight_bytes
    del g
    # kernel launches of one eager step
    nl0 = _launches(st)
    st.spec_step(G)
    launches_per_step = _launches(st) - nl0
    # end to end: one config-1 request through the public C ABI with host
    # buffers: the 128-token prompt H2D + ifr_prefill, then spec steps
    # (ifr_spec_graph_launch of the state's captured step) each followed by
    # ifr_state_read (sync + D2H of the emitted tokens and the scalars) until
    # SPEC_GEN tokens have been emitted.  The state and its graph are set up
    # before the timed region (capture runs no kernel).
    st2 = State(model, SPEC_PROMPT + (SPEC_GEN + 2) * (G + 1) + 16)
    st2.capture(G, 1)
    ee0, ee1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx.sync()
    barrier(ws)
    ee0.record(stream)
    st2.prefill(prompt)
    d2h, e2e_steps, t2 = 0, 0, st2.read()[0]
    while len(t2) < SPEC_GEN:
        st2.launch()
        t2 = st2.read()[0]
        d2h += t2.nbytes + 16
        e2e_steps += 1
    ee1.record(stream)
    ee1.synchronize()
    e2e_ms = max_over_ranks(ee0.elapsed_time(ee1), ws)
    e2e_tokens = len(t2)
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cpu = spec_cpu_baseline(path, prompt, G, steps=3)
    # the other single-GPU configs as extra keys of the same line (one GPU
    # only; at N > 1 the line is the replicas' throughput)
    extras = {}
    if ws == 1 and not args.no_extras:
        extras["prefill_2048"] = prefill_extra(model, prompt_len=2048)
        extras["config3_accept"] = accept_extra(pkg, local, reps=max(3, args.steps // 2))
        extras["config2_sweep"] = sweep_extra(pkg, local)
    # the configs that shard, at this N: config 4 (64 requests split over the
    # ranks) always, config 5 (tensor parallel) from 2 GPUs on; a few steps each
    if not args.no_extras and not args.no_shard_legs:
        extras["config4_batch"] = batch_leg(args, pkg, ws, rank, local, 5, 3)
        if ws > 1:
            extras["config5_tp"] = tp_leg(args, pkg, ws, rank, local, 5, 3)
    if rank == 0:
        peak, peak_kind = measured_peaks()
        step_bytes = spec_bytes_per_step(info, G)
        value = emitted * ws / (ms_max * 1e-3)
        achieved = v_bytes / (v_ms * 1e-3) / 1e9
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "tokens/s",
            "n_gpus": ws,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_max / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": ACT_DTYPE[args.act],
            "data": "synthetic: seeded random-init Qwen3.5-shape hybrid GGUF (N(0,0.02) weights, the library's encoder), seeded uniform 128-token prompt",
            "config": spec_config(G, step_bytes, ws),
            "activations": ["exact f32", "Q8_K"][args.act],
            "tokens_emitted_timed": emitted, "accept_rate": round((emitted / args.steps - 1) / G, 4),
            "graph": "one CUDA graph per spec step",
            "per_gpu_value": round(value / ws, 2),
            "value_is": "the aggregate over all GPUs (tokens/s of the whole job); per_gpu_value = value / n_gpus",
            "step_hbm_GBps": round(step_bytes / (ms_max / args.steps * 1e-3) / 1e9, 1),
            "roofline": {"bound": "hbm", "kernel": "qgemv: the 97 dequant-GEMV launches of one verify (24 layers x 4 + Q6_K lm_head), N=5, back to back",
                         "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": SPEC_VERIFY_TRAFFIC,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum over the same 97 launches (profiles/spec_step_launches_config1.md)",
                         "algorithmic_bytes_per_launch": int(v_bytes), "launch_ms": round(v_ms, 4)},
            "e2e": {"value": round(e2e_tokens * ws / (e2e_ms * 1e-3), 2), "unit": "tokens/s",
                    "h2d_bytes_per_step": int(prompt.nbytes / max(1, e2e_steps)),
                    "d2h_bytes_per_step": int(d2h / max(1, e2e_steps)),
                    "tokens": e2e_tokens, "steps": e2e_steps, "ms": round(e2e_ms, 3),
                    "note": "one config-1 request per rank, end to end through the C ABI: H2D of the 128-token prompt + "
                            "ifr_prefill, then ifr_spec_graph_launch + ifr_state_read (sync, D2H of the emitted tokens) "
                            "per step until 128 tokens are emitted; graph captured before the timed region"},
            "gpu_launches": int(launches_per_step * args.steps),
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
        }
        line.update(extras)
        print(json.dumps(line), flush=True)
    barrier(ws)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def prefill_extra(model, prompt_len=2048, reps=2):
    """one request of the config-1 model with a seeded prompt of prompt_len
    tokens through ifr_prefill (H2D of the prompt, chunks of 64 tokens: every
    projection over the chunk's columns, the SSM layers scanning a chunk in
    one launch, then the last token with logits; synchronous), wall clock per
    call after one warm-up call on a fresh state each time"""
    from inferno_b200 import synth
    from inferno_b200.engine import State
    prompt = synth.prompt(model.info.vocab, prompt_len, 77)

    def timed(dense):
        model.ctx.set_prefill_dense(dense)
        times = []
        for i in range(reps + 1):
            st = State(model, prompt_len + 64)
            model.ctx.sync()
            t0 = time.perf_counter()
            st.prefill(prompt)
            dt = time.perf_counter() - t0
            if i:
                times.append(dt)
            st.free()
        model.ctx.set_prefill_dense(False)
        return float(np.median(times)) * 1e3

    ms, ms_d = timed(False), timed(True)
    return {"workload": f"ifr_prefill of one config-1 request, {prompt_len}-token seeded prompt",
            "chunk_tokens": 64, "ms": round(ms, 2), "tokens_per_s": round(prompt_len / (ms * 1e-3), 1),
            "path": "default (exact): projections on the exact small-N kernel in passes of 8 columns over each 64-token chunk, GatedDeltaNet chunk scan, attention in 8-token sub-calls",
            "dense_ms": round(ms_d, 2), "dense_tokens_per_s": round(prompt_len / (ms_d * 1e-3), 1),
            "dense_path": "ifr_ctx_set_prefill_dense: the chunk's projections on the tcgen05 GEMM (fp16 operands)",
            "calls_timed": reps}


def accept_extra(pkg, device, reps=5):
    """BASELINE config 3 on this GPU: sampled acceptance (ifr_accept) of 64
    sequences x draft length 5 over vocab 151936 at T = 0.8, target ~N(0, 3),
    draft = target + N(0, 1), seeded uniforms; logits resident in HBM (428 MB,
    above L2).  CUDA events around each call on the context's stream; the
    roofline bytes are one read of all logits."""
    import torch
    B, G, V, T = 64, 5, 151936, 0.8
    ctx = pkg.Context(device)
    gen = torch.Generator(device="cuda").manual_seed(3)
    tgt = torch.randn(B, G + 1, V, generator=gen, device="cuda") * 3
    dft = (tgt[:, :G] + torch.randn(B, G, V, generator=gen, device="cuda")).contiguous()
    u = torch.rand(B, 2 * G + 1, generator=gen, device="cuda")
    for _ in range(3):
        ctx.accept(tgt, dft, u, T)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for a, b in ev:
        a.record(stream)
        acc, _, _ = ctx.accept(tgt, dft, u, T)
        b.record(stream)
    torch.cuda.synchronize()
    ms = float(np.mean([a.elapsed_time(b) for a, b in ev]))
    nbytes = B * (2 * G + 1) * V * 4
    peak, kind = measured_peaks()
    r = {"workload": "BASELINE config 3: 64 x gamma 5 x vocab 151936, T 0.8, supplied uniforms",
         "kernels": "chunk_stats + row_decide + resid_chunks + finish (4 launches per call)",
         "ms_per_call": round(ms, 4), "sequences_per_s": round(B / (ms * 1e-3), 1),
         "roofline": {"bound": "hbm", "achieved": round(nbytes / (ms * 1e-3) / 1e9, 1), "peak": peak,
                      "peak_kind": kind, "unit": "GB/s", "frac": round(nbytes / (ms * 1e-3) / 1e9 / peak, 4),
                      "algorithmic_bytes_per_call": nbytes},
         "mean_accept": round(float(acc.float().mean()), 3), "calls_timed": reps}
    del tgt, dft
    ctx.close()
    return r


def sweep_extra(pkg, device):
    """BASELINE config 2 on this GPU: every format x shape at N = 5 columns,
    one CUDA-event pair per launch (mean of 3 after 2 warm-up passes), in the
    reference's arithmetic (Q8_K activations, the default) and with exact f32
    activations; weights resident, 2.3 GB per pass (above L2)"""
    import torch
    ctx = pkg.Context(device)
    rng = np.random.default_rng(1234)
    Ws, Xs, Ys, byts, names = [], [], [], [], []
    for qt, name in FORMATS:
        for (M, K) in SHAPES:
            Ws.append(ctx.upload(qt, make_weights(pkg, qt, M, K, rng), M, K))
            Xs.append(torch.from_numpy(rng.normal(0, 1, (NCOLS, K)).astype(np.float32)).cuda())
            Ys.append(torch.empty(NCOLS, M, dtype=torch.float32, device="cuda"))
            byts.append(Ws[-1].algorithmic_bytes())
            names.append(f"{name} {M}x{K}")
    stream = torch.cuda.current_stream()
    peak, kind = measured_peaks()
    out = {"workload": "BASELINE config 2: Q4_K/Q5_K/Q6_K/Q8_0 x (4096x4096, 12288x4096, 4096x12288, 151936x4096), N = 5",
           "peak": peak, "peak_kind": kind}
    for act, label in ((1, "q8k_activations"), (0, "exact_activations")):
        ctx.set_activation(act)
        for _ in range(2):
            for i, W in enumerate(Ws):
                ctx.qgemm(W, Xs[i], Ys[i])
        ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in Ws]
              for _ in range(3)]
        for r in range(3):
            for i, W in enumerate(Ws):
                ev[r][i][0].record(stream)
                ctx.qgemm(W, Xs[i], Ys[i])
                ev[r][i][1].record(stream)
        torch.cuda.synchronize()
        d = {}
        for i, nm in enumerate(names):
            us = float(np.mean([ev[r][i][0].elapsed_time(ev[r][i][1]) for r in range(3)])) * 1e3
            d[nm] = {"us": round(us, 2), "GBps": round(byts[i] / us / 1e3, 1),
                     "frac": round(byts[i] / us / 1e3 / peak, 3)}
        out[label] = d
    for W in Ws:
        W.free()
    ctx.close()
    return out


BATCH_PRESET, BATCH_SEED = "9b", 0


def run_batch(args):
    """BASELINE config 4 as its own line (`--workload batch`)"""
    import torch
    import __graft_entry__ as ge
    ws, rank, local = dist_init()
    torch.cuda.set_device(local)
    pkg = ge.load_package()
    pkg.load()
    line = batch_leg(args, pkg, ws, rank, local, args.steps, args.warmup)
    if rank == 0:
        print(json.dumps(line), flush=True)
    barrier(ws)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def batch_leg(args, pkg, ws, rank, local, steps, warmup):
    """the ~9B-shape hybrid, `--batch` independent requests
    (64) split evenly over the ranks, each with a seeded prompt of `--prompt`
    tokens (2048); one step = MTP draft of gamma tokens for every request +
    one verify of batch x (gamma+1) columns (dense tcgen05 GEMMs) + greedy
    acceptance + rollback, replayed as a CUDA graph.  Every rank runs it (no
    collective on the data path); returns the line on rank 0."""
    import ctypes
    import torch
    from inferno_b200 import synth
    from inferno_b200.engine import Model, State
    G = args.gamma
    mine = rank_requests(args.batch, ws, rank)
    B = len(mine)
    ctx = pkg.Context(local, torch_stream=False)
    ctx.set_kv_bf16(bool(getattr(args, "kv_bf16", 0)))
    t_load = time.time()
    if rank == 0:
        synth.cached(BATCH_PRESET, BATCH_SEED)
    barrier(ws)
    path = synth.cached(BATCH_PRESET, BATCH_SEED)
    model = Model(ctx, path)
    info = model.info
    t_load = time.time() - t_load
    P = args.prompt
    prompts = np.stack([synth.prompt(info.vocab, P, BATCH_SEED + 1000 + r) for r in mine])
    max_ctx = P + (warmup + steps + 4) * (G + 1) + 16
    st = State(model, max_ctx, batch=B)
    ctx.sync()
    t0 = time.time()
    st.prefill(prompts)
    ctx.sync()
    prefill_s = time.time() - t0
    st.spec_step(G)  # eager step: every kernel initialised before capture
    st.capture(G, 1)
    sp = ctypes.c_void_p()
    pkg.check(pkg.load().ifr_ctx_get_stream(ctx.handle, ctypes.byref(sp)))
    stream = torch.cuda.ExternalStream(sp.value)
    for _ in range(warmup):
        st.launch()
    ctx.sync()
    n0 = sum(len(st.read(b)[0]) for b in range(B))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(ws)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(steps):
            st.launch()
        e1.record(stream)
        e1.synchronize()
    ms = e0.elapsed_time(e1)
    emitted = sum(len(st.read(b)[0]) for b in range(B)) - n0
    barrier(ws)
    ms_max = max_over_ranks(ms, ws)
    emitted_all = int(max_over_ranks(float(emitted), ws) * ws)  # equal work per rank (zero acceptance)
    nl0 = _launches(st)
    st.spec_step(G)
    launches_per_step = _launches(st) - nl0
    # end to end through the public API with host buffers: per step ifr_spec_step
    # + D2H of every request's emitted tokens
    ctx.sync()
    barrier(ws)
    ee0, ee1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ee0.record(stream)
    d2h = 0
    k2 = max(1, min(steps, 4))
    for _ in range(k2):
        st.spec_step(G)
        for b in range(B):
            d2h += st.read(b)[0].nbytes
    ee1.record(stream)
    ee1.synchronize()
    e2e_ms = max_over_ranks(ee0.elapsed_time(ee1), ws)
    line = None
    if rank == 0:
        hd = info.head_dim
        kv_bytes = 2 * info.n_attention_layers * info.n_kv_head * hd * (2 if getattr(args, "kv_bf16", 0) else 4) * \
            (P + G + 1) * args.batch // ws
        flops = 2.0 * verify_weight_count(info) * B * (G + 1)
        line = {
            "metric": METRIC,
            "value": round(emitted_all / (ms_max * 1e-3), 2),
            "unit": "tokens/s",
            "n_gpus": ws,
            "steps": steps,
            "warmup": warmup,
            "ms_per_step": round(ms_max / steps, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "q4_k/q6_k weights; verify and draft projections of >= 24 columns on tcgen05 (fp16 operands, f32 accumulate), others exact f32",
            "data": "synthetic: seeded random-init ~9B-shape Qwen3.5 hybrid GGUF (rows drawn from a 1024-row pool per matrix), seeded uniform prompts",
            "config": {"workload": "batched greedy spec-decode, BASELINE config 4 (~9B-shape hybrid)",
                       "model": "hidden 4096, 32 layers (24 GatedDeltaNet + 8 attention), 16q/4kv x 256, SSM 32 x 128, FFN 12288, vocab 151936, Q4_K matmuls, Q6_K ffn_down/lm_head, 1-layer MTP head",
                       "requests": args.batch, "requests_per_gpu": B, "gamma": G, "verify_columns_per_gpu": B * (G + 1),
                       "prompt": P, "kv": "bf16" if getattr(args, "kv_bf16", 0) else "f32",
                       "prefill_s": round(prefill_s, 2), "load_s": round(t_load, 1),
                       "tokens_emitted_timed": emitted_all,
                       "l2": "inputs larger than L2: %.1f GB of weights + %.1f GB of KV per step per GPU" % (info.weight_bytes / 1e9, kv_bytes / 1e9),
                       "parallelism": f"requests split over {ws} GPU(s), weights replicated, no collective",
                       "graph": "one CUDA graph per spec step"},
            "per_gpu_tokens_per_s": round(emitted_all / ws / (ms_max * 1e-3), 2),
            "roofline": {"bound": "tensor", "kernel": "whole verify step (dense GEMMs dominate)",
                         "achieved": round(flops / (ms_max / steps * 1e-3) / 1e12, 1),
                         "peak": measured_peaks_tensor(), "unit": "TFLOP/s", "traffic": None,
                         "note": "verify weights x columns x 2 flop per step, over the step time"},
            "e2e": {"value": round(k2 * B * ws / (e2e_ms * 1e-3), 2), "unit": "tokens/s (lower bound: 1 token per request per step)",
                    "h2d_bytes_per_step": 0, "d2h_bytes_per_step": int(d2h / k2)},
            "gpu_launches": int(launches_per_step * steps),
            "clocks": clk.summary(),
            "cpu_baseline": None,
        }
        line["roofline"]["frac"] = round(line["roofline"]["achieved"] / line["roofline"]["peak"], 4)
    barrier(ws)
    st.free()
    model.free()
    ctx.close()
    return line


def verify_weight_count(info):
    """quantized weights one verify forward multiplies (decoder layers + lm_head)"""
    d, hd, f = info.hidden, info.head_dim, info.ffn
    inner = info.ssm_heads * info.ssm_head_dim
    conv = 3 * inner
    mlp = 3 * f * d
    ssm = (conv + inner) * d + d * inner + mlp
    attn = (2 * info.n_head + 2 * info.n_kv_head) * hd * d + d * info.n_head * hd + mlp
    n_attn = info.n_attention_layers
    return (info.n_layers - n_attn) * ssm + n_attn * attn + info.vocab * d


TP_PRESET, TP_DRAFT, TP_SEED = "gemma", "gemma_draft", 0


def run_tp(args):
    """BASELINE config 5 as its own line (`--workload tp`)"""
    import torch
    import __graft_entry__ as ge
    ws, rank, local = dist_init()
    torch.cuda.set_device(local)
    pkg = ge.load_package()
    pkg.load()
    line = tp_leg(args, pkg, ws, rank, local, args.steps, args.warmup)
    if rank == 0:
        print(json.dumps(line), flush=True)
    barrier(ws)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def tp_leg(args, pkg, ws, rank, local, steps, warmup):
    """the Gemma4-shape target (hidden 5376, 62 layers,
    32 q / 16 kv x 128, FFN 21504, vocab 262144, Q4_K, Gemma4 blocks)
    tensor-parallel over all ranks (NCCL all-reduce of each sub-block's output
    after the row-parallel projections, vocab-parallel lm_head), the Q8_0
    draft model (hidden 1152, 26 layers) replicated on every rank; one request
    with a seeded prompt of 4096 tokens; one step = 5 draft tokens + one
    verify of 6 columns + greedy acceptance, as a CUDA graph.  Returns the
    line on rank 0."""
    import ctypes
    import torch
    from inferno_b200 import synth
    from inferno_b200.engine import Comm, Model, State
    G = args.gamma if args.gamma != 4 else 5  # config 5: draft length 5
    P = args.prompt if args.prompt != 2048 else 4096
    ctx = pkg.Context(local, torch_stream=False)
    t_load = time.time()
    if rank == 0:
        synth.cached(TP_PRESET, TP_SEED)
        synth.cached(TP_DRAFT, TP_SEED)
    barrier(ws)
    uid = None
    if ws > 1:
        import torch.distributed as dist
        t = torch.zeros(Comm.ID_BYTES, dtype=torch.uint8, device="cuda")
        if rank == 0:
            t.copy_(torch.frombuffer(bytearray(Comm.unique_id()), dtype=torch.uint8))
        dist.broadcast(t, 0)
        uid = bytes(t.cpu().numpy())
    comm = Comm(ctx, rank, ws, uid)
    target = Model(ctx, synth.cached(TP_PRESET, TP_SEED), comm)
    draft = Model(ctx, synth.cached(TP_DRAFT, TP_SEED))
    info = target.info
    t_load = time.time() - t_load
    prompt = synth.prompt(info.vocab, P, TP_SEED)
    max_ctx = P + (warmup + 2 * steps + 8) * (G + 1) + 16
    ts, ds = State(target, max_ctx), State(draft, max_ctx)
    ctx.sync()
    t0 = time.time()
    ts.prefill(prompt)
    ds.prefill(prompt)
    ctx.sync()
    prefill_s = time.time() - t0
    ts.spec_step_draft(ds, G)  # eager: every kernel initialised before capture
    ts.capture_draft(ds, G, 1)
    sp = ctypes.c_void_p()
    pkg.check(pkg.load().ifr_ctx_get_stream(ctx.handle, ctypes.byref(sp)))
    stream = torch.cuda.ExternalStream(sp.value)
    for _ in range(warmup):
        ts.launch()
    ctx.sync()
    n0 = len(ts.read()[0])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(ws)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(steps):
            ts.launch()
        e1.record(stream)
        e1.synchronize()
    ms = e0.elapsed_time(e1)
    emitted = len(ts.read()[0]) - n0
    barrier(ws)
    ms_max = max_over_ranks(ms, ws)
    # end to end through the public API: per step ifr_spec_step_draft + D2H of the emitted tokens
    ctx.sync()
    barrier(ws)
    ee0, ee1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ee0.record(stream)
    d2h, k2 = 0, max(1, min(steps, 8))
    for _ in range(k2):
        ts.spec_step_draft(ds, G)
        d2h += ts.read()[0].nbytes
    ee1.record(stream)
    ee1.synchronize()
    e2e_ms = max_over_ranks(ee0.elapsed_time(ee1), ws)
    # the all-reduce share: one eager step with the target's launches timed
    # per category (CUDA events on the context stream); the draft state's
    # launches are not categorised
    ts.profile(True)
    barrier(ws)
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    ts.spec_step_draft(ds, G)
    p1.record(stream)
    p1.synchronize()
    prof, _ = ts.profile_read()
    ts.profile(False)
    prof_step = p0.elapsed_time(p1)
    comm_ms = max_over_ranks(prof["allreduce"]["ms"], ws)
    barrier(ws)
    line = None
    if rank == 0:
        peak, peak_kind = measured_peaks()
        shard_bytes = info.weight_bytes  # this rank's target shard (decoder layers + lm_head rows)
        step_ms = ms_max / steps
        line = {
            "metric": METRIC,
            "value": round(emitted / (ms_max * 1e-3), 2),
            "unit": "tokens/s",
            "n_gpus": ws,
            "steps": steps,
            "warmup": warmup,
            "ms_per_step": round(step_ms, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": ACT_DTYPE[0].replace("q4_k/q6_k", "q4_k target, q8_0 draft"),
            "data": "synthetic: seeded random-init Gemma4-shape target and draft GGUFs (rows drawn from a 1024-row pool per matrix), seeded uniform prompt",
            "config": {"workload": "greedy spec-decode with a draft model, BASELINE config 5 (Gemma4-shape target, tensor parallel)",
                       "target": "hidden 5376, 62 Gemma4 attention layers (5 sliding-window : 1 full, window 1024, GELU-tanh MLP, softcaps), 32q/16kv x 128, FFN 21504, vocab 262144, Q4_K",
                       "draft": "hidden 1152, 26 Gemma4 attention layers, 4q/1kv x 256, FFN 6912, Q8_0, replicated",
                       "gamma": G, "prompt": P, "batch": 1, "tp": ws, "prefill_s": round(prefill_s, 2),
                       "load_s": round(t_load, 1), "tokens_emitted_timed": emitted,
                       "l2": "inputs larger than L2: %.2f GB of target weights per rank per verify" % (shard_bytes / 1e9),
                       "parallelism": f"tensor parallel x{ws}: NCCL sum all-reduce after attention-output and down projections, vocab-parallel lm_head",
                       "graph": "one CUDA graph per spec step"},
            "allreduce": {"ms_per_step": round(comm_ms, 4), "share_of_eager_step": round(comm_ms / prof_step, 4),
                          "eager_step_ms": round(prof_step, 3), "per_step": 2 * info.n_layers,
                          "note": "one eager step, CUDA events around each NCCL all-reduce of the target (max over ranks)"},
            "roofline": {"bound": "hbm", "kernel": "whole spec step per rank: the target shard's weights once per verify",
                         "achieved": round(shard_bytes / (step_ms * 1e-3) / 1e9, 1), "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(shard_bytes / (step_ms * 1e-3) / 1e9 / peak, 4), "traffic": None,
                         "note": "target shard bytes per step / step time (the draft's 26 small forwards and the all-reduces are inside the step)"},
            "e2e": {"value": round(k2 * (emitted / steps) / (e2e_ms * 1e-3), 2), "unit": "tokens/s",
                    "h2d_bytes_per_step": 0, "d2h_bytes_per_step": int(d2h / k2)},
            "gpu_launches": None,
            "clocks": clk.summary(),
            "cpu_baseline": None,
        }
    barrier(ws)
    ts.free()
    ds.free()
    target.free()
    draft.free()
    comm.free()
    ctx.close()
    return line


def measured_peaks_tensor():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("bf16_tflops_sustained", d.get("bf16_tflops", 1405.8))
    return 1400.0


def _launches(st):
    import ctypes
    from inferno_b200._lib import load
    nl = ctypes.c_int64()
    load().ifr_state_profile_read(st.handle, None, None, None, ctypes.byref(nl))
    return nl.value


def _oracle_spec(path, prompt, gamma, steps, warmup=0):
    """tokens/s of `steps` oracle spec steps after the prefill and `warmup` steps"""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O  # CPU baseline / reference arm only
    import __graft_entry__ as ge
    ge.load_package()
    from inferno_b200 import gguf
    om = O.OracleModel(gguf.GGUFFile(path), len(prompt) + (steps + warmup + 2) * (gamma + 1) + 8)
    _, rec = om.spec_decode(prompt, warmup + steps, gamma)
    timed = rec[warmup:]
    dt = sum(r["seconds"] for r in timed)
    tokens = sum(r["acc"] + 1 for r in timed)
    return tokens / dt, dt, None


def spec_cpu_baseline(path, prompt, gamma, steps=3):
    cores = os.cpu_count() or 1
    tps, dt, _ = _oracle_spec(path, prompt, gamma, steps)
    return {"value": round(tps, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"C restatement of forward_cpu! + MTP head + the fixed spec-decode loop (oracle/model.c, "
                      f"f32 dequantized weights, {cores} threads over matvec rows): {steps} spec steps "
                      f"(gamma {gamma}) after the 128-token prefill, {dt:.1f} s"}


def run_reference_spec(args):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import __graft_entry__ as ge
    O = ge.load_oracle()
    ge.load_package()  # python modules only: libinferno_b200.so is never loaded on this arm
    from inferno_b200 import synth
    # the model's bytes come from the oracle's encoder (identical to the
    # library's, tests/test_oracle.py), so this arm maps no library of ours
    path = synth.cached(SPEC_PRESET, SPEC_SEED, quantize=O.quantize)
    from inferno_b200 import gguf
    gf = gguf.GGUFFile(path)
    V = int(gf.tensors["token_embd.weight"].dims[1])
    prompt = synth.prompt(V, SPEC_PROMPT, SPEC_SEED)
    # every step is one whole spec step of the workload (draft, verify,
    # accept) on the host cores; the steps and warm-up match the GPU arm's
    steps = max(1, args.steps)
    tps, dt, _ = _oracle_spec(path, prompt, args.gamma, steps, warmup=args.warmup)
    cores = os.cpu_count() or 1
    sample = (f"reference CPU path restated in C (oracle/model.c: forward_cpu! + MTP head + fixed greedy spec-decode "
              f"loop, {cores} threads): {steps} spec steps after {args.warmup} warm-up steps, gamma {args.gamma}, "
              f"after a 128-token prefill")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(tps, 3), "unit": "tokens/s", "n_gpus": ws,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(dt / steps * 1e3, 1), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (dequantized weights)", "data": "synthetic",
        "config": spec_config(args.gamma, spec_bytes_per_step_gguf(gf, args.gamma), ws),
        "cpu_baseline": {"value": round(tps, 3), "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": round(tps, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)



def run_profile(args):
    """small cases for ncu: only the launches between profiler start/stop count"""
    import torch
    import __graft_entry__ as ge
    pkg = ge.load_package()
    pkg.load()
    torch.cuda.set_device(0)
    if args.profile == "accept":
        # config 3: one sampled acceptance call (64 x gamma 5 x 151936, T 0.8)
        # between profiler start / stop, after three warm-up calls
        B, G, V, T = 64, 5, 151936, 0.8
        ctx = pkg.Context(0)
        gen = torch.Generator(device="cuda").manual_seed(3)
        tgt = torch.randn(B, G + 1, V, generator=gen, device="cuda") * 3
        dft = (tgt[:, :G] + torch.randn(B, G, V, generator=gen, device="cuda")).contiguous()
        u = torch.rand(B, 2 * G + 1, generator=gen, device="cuda")
        for _ in range(3):
            ctx.accept(tgt, dft, u, T)
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        ctx.accept(tgt, dft, u, T)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        print(json.dumps({"profile": "accept", "batch": B, "gamma": G, "vocab": V}))
        return
    if args.profile == "fused":
        import ctypes
        # the config-1 verify's decoder layers as one persistent launch
        # (ifr_ctx_set_fused_layers): per-phase times from the kernel's own
        # global-timer trace over 10 eager spec steps, and the step time of
        # both paths as CUDA graphs
        from inferno_b200 import synth
        from inferno_b200.engine import Model, State
        ctx = pkg.Context(0, torch_stream=False)
        model = Model(ctx, synth.cached(SPEC_PRESET, SPEC_SEED))
        prompt = synth.prompt(model.info.vocab, SPEC_PROMPT, SPEC_SEED)
        ctx.set_fused_layers(True)
        st = State(model, SPEC_PROMPT + 160)
        st.prefill(prompt)
        for _ in range(3):
            st.spec_step(args.gamma)
        st.profile(True)
        traces, bars = [], []
        for _ in range(10):
            st.spec_step(args.gamma)
            traces.append(st.fused_trace())
            bars.append(st.fused_barriers)
        st.free()
        kinds = [t[0] for t in traces[0]]
        A = np.array([[t[1:] for t in tr] for tr in traces])
        Bm = np.array(bars)
        out = {"profile": "fused", "phases": len(kinds), "layer_stack_us": round(float(A[:, :, 0].sum(1).mean()), 1)}
        cols = ["us", "slowest_cta_fragments", "slowest_cta_tiles", "slowest_cta_rest", "slowest_cta_to_next",
                "slowest_cta_whole"]
        for k in sorted(set(kinds)):
            idx = [i for i, kk in enumerate(kinds) if kk == k]
            m = A[:, idx].mean((0, 1))
            out[k] = {"phases": len(idx), **{c: round(float(v), 2) for c, v in zip(cols, m)},
                      "barrier": {c: round(float(v), 2) for c, v in zip(
                          ["arrival_skew", "propagation", "acquire", "to_next_start"], Bm[:, idx].mean((0, 1)))}}
        step = {}
        for fused in (1, 0):
            ctx.set_fused_layers(bool(fused))
            st = State(model, SPEC_PROMPT + 160)
            st.prefill(prompt)
            st.spec_step(args.gamma)
            st.capture(args.gamma, 1)
            for _ in range(3):
                st.launch()
            ctx.sync()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            sp = ctypes.c_void_p()
            pkg.check(pkg.load().ifr_ctx_get_stream(ctx.handle, ctypes.byref(sp)))
            stream = torch.cuda.ExternalStream(sp.value)
            e0.record(stream)
            for _ in range(20):
                st.launch()
            e1.record(stream)
            e1.synchronize()
            step["fused" if fused else "separate"] = round(e0.elapsed_time(e1) / 20, 4)
            st.free()
        out["graph_step_ms"] = step
        print(json.dumps(out))
        return
    if args.profile == "spec":
        from inferno_b200 import synth
        from inferno_b200.engine import Model, State
        ctx = pkg.Context(0, torch_stream=False)
        model = Model(ctx, synth.cached(SPEC_PRESET, SPEC_SEED))
        prompt = synth.prompt(model.info.vocab, SPEC_PROMPT, SPEC_SEED)
        st = State(model, SPEC_PROMPT + 64)
        st.prefill(prompt)
        st.spec_step(args.gamma)
        st.capture(args.gamma, 1)
        for _ in range(3):
            st.launch()
        ctx.sync()
        torch.cuda.profiler.start()
        for _ in range(2):
            st.launch()
        ctx.sync()
        torch.cuda.profiler.stop()
        print(json.dumps({"profile": "spec", "launches_per_step": _launches(st)}))
        return
    if args.profile == "batch":
        from inferno_b200 import synth
        from inferno_b200.engine import Model, State
        ctx = pkg.Context(0, torch_stream=False)
        ctx.set_kv_bf16(bool(args.kv_bf16))
        # --preset 9b_narrow: config 4's widths with 4 layers (a small case for ncu)
        model = Model(ctx, synth.cached(args.preset or BATCH_PRESET, BATCH_SEED))
        B, P = args.batch, args.prompt
        prompts = np.stack([synth.prompt(model.info.vocab, P, BATCH_SEED + 1000 + b) for b in range(B)])
        st = State(model, P + 64, batch=B)
        st.prefill(prompts)
        st.spec_step(args.gamma)
        st.capture(args.gamma, 1)
        for _ in range(2):
            st.launch()
        ctx.sync()
        torch.cuda.profiler.start()
        st.launch()
        ctx.sync()
        torch.cuda.profiler.stop()
        print(json.dumps({"profile": "batch", "requests": B, "prompt": P}))
        return
    qt = {"Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "Q8_0": 8}[args.qtype]
    M, K = (int(v) for v in args.shape.split("x"))
    rng = np.random.default_rng(7)
    ctx = pkg.Context(0)
    t = ctx.upload(qt, make_weights(pkg, qt, M, K, rng), M, K)
    X = torch.from_numpy(rng.normal(0, 1, (args.ncols, K)).astype(np.float32)).cuda()
    Y = torch.empty(args.ncols, M, device="cuda")
    ctx.set_activation(args.act)
    run = ctx.qgemm_dense if args.profile == "dense" else ctx.qgemm
    for _ in range(3):
        run(t, X, Y)
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    for _ in range(3):
        run(t, X, Y)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print(json.dumps({"profile": args.profile, "qtype": args.qtype, "shape": [M, K], "ncols": args.ncols,
                      "weight_bytes": int(M * K * BPW[qt])}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="spec", choices=["spec", "sweep", "batch", "tp"])
    ap.add_argument("--batch", type=int, default=64, help="requests of the batch workload (all ranks)")
    ap.add_argument("--prompt", type=int, default=2048, help="prompt tokens per request (batch workload)")
    ap.add_argument("--gamma", type=int, default=4)
    ap.add_argument("--fused-layers", type=int, default=0, choices=[0, 1],
                    help="spec workload: the verify's decoder layers as one persistent launch")
    ap.add_argument("--kv-bf16", type=int, default=0, choices=[0, 1],
                    help="batch workload / --profile batch: bf16 attention caches (ifr_ctx_set_kv_bf16)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="spec workload: skip every extra key")
    ap.add_argument("--no-shard-legs", action="store_true", help="spec workload: skip the config-4/5 legs")
    ap.add_argument("--act", type=int, default=None, choices=[0, 1],
                    help="K-quant GEMV activations: 0 = exact f32 (default of the model workloads), "
                         "1 = Q8_K (the reference's kernels; default of the sweep)")
    ap.add_argument("--profile", choices=["spec", "qgemv", "dense", "batch", "fused", "accept"],
                    help="small case for ncu (no JSON line); fused: the fused layer stack's phase trace")
    ap.add_argument("--preset", default=None, help="--profile batch: model preset (default: the config-4 model)")
    ap.add_argument("--qtype", default="Q4_K")
    ap.add_argument("--shape", default="65536x4096")
    ap.add_argument("--ncols", type=int, default=5)
    args = ap.parse_args()
    if args.act is None and (args.profile or args.workload != "sweep"):
        args.act = 0
    if args.profile:
        run_profile(args)
        return
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.workload == "tp":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the tp workload (config 5) has no CPU reference run: a 27B-parameter Gemma4-shape target over a 4096-token prompt is beyond the CPU oracle"}))
            return
        run_tp(args)
    elif args.workload == "batch":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the batch workload (config 4) has no CPU reference run: a 9B-shape model over 64 requests x 2048 tokens is beyond the CPU oracle; see the spec and sweep workloads"}))
            return
        run_batch(args)
    elif args.workload == "spec":
        (run_reference_spec if args.impl == "reference" else run_spec)(args)
    elif args.impl == "reference":
        run_reference_sweep(args)
    else:
        run_sweep(args)


if __name__ == "__main__":
    main()
