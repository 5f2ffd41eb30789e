#!/usr/bin/env python
"""bench.py -- MoE-layer decode tokens/s and Q4_K expert GEMV HBM GB/s.

Workload (one "step" = one decode token through one MoE layer):
  Mixtral-8x7B-shaped MoE FFN layer: hidden 4096, 8 experts, top-2 softmax
  routing renormalised, SwiGLU experts 4096->14336->4096 stored Q4_K
  (793 MB of expert weights per layer), fp32 router 4096x8.  Input tokens are
  N(0,1), RMSNorm'd by the layer ingress; the layer adds the residual
  (DistributedPipelineCoordinator.ExecuteStep semantics).  Weights are the
  documented seeded synthetic generator (no checkpoints exist offline).

  ours       : the sm_100a decode-layer kernel (router, gate/up GEMV + SwiGLU,
               grid barrier, down GEMV + weighted combine + residual, all in
               one persistent launch), one launch per step through
               glc_moe_forward_dev on the step's resident token buffer;
               the timed steps are captured in CUDA graphs that the timed
               region replays (as a serving loop would): one graph of all
               the steps up to 512, else graphs of 16 steps + a remainder;
               16 input tokens rotate so consecutive steps route to different
               experts; the 793 MB expert working set is > L2.
  reference  : the CPU port of the reference's CPU path (CpuWarmExpertPoolWorker
               shape: per expert gate/up/down mat-vec + SwiGLU, k-ordered
               combine) with all host threads.  The reference itself is C#
               (.NET) with its mat-vec in an un-vendored package and cannot run.

Multi-GPU (torchrun): each rank runs its own decode stream on its own GPU
(weak scaling, replicas of the layer: the headline value); the line also
carries an expert-parallel leg (experts split over the ranks, dispatch and
return written into the peers' memory over NVLink -- or, for comparison and
where peer mapping is unavailable, exchanged with NCCL -- around the grouped
tensor-core experts).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

WORKLOAD = dict(name="mixtral8x7b_moe_layer_decode", D=4096, F=14336, E=8, k=2, T=1, seed=20241201,
                flags=3)  # GLC_FWD_RMSNORM | GLC_FWD_RESIDUAL
N_TOKENS = 16
MAX_ONE_GRAPH = 512  # timed steps captured as one graph up to this many
BATCH_TOKENS = 64  # the 64-token batch of the same layer (grouped tensor-core path)
METRIC = "MoE-layer decode tokens/s & Q4_K expert GEMV HBM GB/s vs 8 TB/s, 1/2/4/8 GPU"
UNIT = "tokens/s"
REF_BUDGET_S = 120.0
GLC_FWD_UNFUSED = 16  # decode path as three launches (router, gate/up, down)
GLC_FWD_BATCHED = 8  # grouped tensor-core experts


def q4k_row_bytes(k):
    return (k // 256) * 144


def algorithmic_bytes(w):
    """Bytes a step must move: k experts' Q4_K weights + router + activations."""
    D, F, E, k, T = w["D"], w["F"], w["E"], w["k"], w["T"]
    gateup = T * k * 2 * F * q4k_row_bytes(D) + T * D * 4 + T * k * F * 4
    down = T * k * D * q4k_row_bytes(F) + T * k * F * 4 + 2 * T * D * 4
    router = D * E * 4 + 2 * T * D * 4
    return {"gateup": gateup, "down": down, "router": router, "step": gateup + down + router}


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profile_traffic(kernel_tag):
    """dram bytes per launch from the committed ncu summary (profiles/), or None."""
    path = os.path.join(REPO, "profiles", f"{kernel_tag}.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(line.split(":")[1].strip())
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.samples = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.samples.append(parts)

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return self.summary()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for s in self.samples:
            for n, v in zip(names, s[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.samples)}


def host_result_bytes(T, D, k):
    """Bytes that cross from the device to the host per decode call of the
    host-buffer forward: the kernel writes the T x D output, the expert ids and
    the combine weights into mapped host memory, plus the 16-byte completion
    and error words."""
    return 4 * T * D + 8 * T * k + 16


def workload_config(w, world):
    """The config both arms print (same keys and values for the same run)."""
    return {"workload": w["name"], "hidden": w["D"], "ffn": w["F"], "experts": w["E"], "top_k": w["k"],
            "tokens_per_step": w["T"], "weights": "Q4_K",
            "parallelism": f"replica x{world}" if world > 1 else "single",
            "l2": "inputs larger than L2: 793 MB expert working set, 16 rotating tokens"}


def make_tokens(w, n):
    rng = np.random.default_rng(w["seed"])
    return rng.standard_normal((n, w["T"], w["D"])).astype(np.float32)


# --------------------------------------------------------------------- CPU legs
def cpu_layer(w):
    from oracle import oracle as o
    D, F, E = w["D"], w["F"], w["E"]
    L = {}
    for m, key, rows, K in ((0, "gate", F, D), (1, "up", F, D), (2, "down", D, F)):
        L[key] = np.concatenate([o.synth_q4k(w["seed"], o.expert_tag(e, m), rows, K) for e in range(E)])
    L["router"] = o.fill_normal(w["seed"], 2, 0.02, D * E)
    return o, L


def cpu_run(o, L, w, tokens, budget_s, nthreads, min_tokens=2):
    """Time the CPU port token by token until budget_s is spent; returns tokens/s."""
    D = w["D"]
    out = np.empty(D, np.float32)
    done, t0 = 0, time.perf_counter()
    while True:
        x = tokens[done % len(tokens)][0]
        o.lib().oc_cpu_moe_token_fast(L["gate"], L["up"], L["down"], L["router"], D, w["F"], w["E"],
                                      w["k"], 1, w["flags"], x, out, nthreads)
        done += 1
        el = time.perf_counter() - t0
        if (el >= budget_s and done >= min_tokens) or done >= 100000:
            return done / el, done, el


def run_reference(args, w):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    nthreads = os.cpu_count() or 1
    o, L = cpu_layer(w)
    tokens = make_tokens(w, N_TOKENS)
    out = np.empty(w["D"], np.float32)

    def one(i):
        o.lib().oc_cpu_moe_token_fast(L["gate"], L["up"], L["down"], L["router"], w["D"], w["F"],
                                      w["E"], w["k"], 1, w["flags"], tokens[i % N_TOKENS][0], out,
                                      nthreads)

    for i in range(min(args.warmup, 3)):
        one(i)
    # A step is one decode token through the layer, as in the GPU arm; the
    # run stops after REF_BUDGET_S so that any --steps finishes in minutes.
    done, t0 = 0, time.perf_counter()
    while done < args.steps and time.perf_counter() - t0 < REF_BUDGET_S:
        one(done)
        done += 1
    total_s = time.perf_counter() - t0
    value = done / total_s
    sample = (f"{done} of {args.steps} requested decode steps (time cap {REF_BUDGET_S:.0f} s), "
              f"same layer and inputs as the GPU arm")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": done, "steps_requested": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 / value,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "q4k-f32",
        "data": "synthetic (seeded generator; no checkpoint offline)",
        "config": workload_config(w, int(os.environ.get("WORLD_SIZE", "1"))),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": nthreads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "CPU port of the reference CPU path (CpuWarmExpertPoolWorker + k-ordered combine); "
                "the reference C#/.NET build and its Glacier.Inference package are not runnable here",
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------- GPU leg
def run_ours(args, w):
    import torch
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        # no NVLink multicast objects: a rank that dies must not leave memory
        # bound to one (the exchanges here are point-to-point all-to-alls)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    from glacier.inference import distributed_b200 as glc

    D, T = w["D"], w["T"]
    worker = glc.GpuExpertStageWorker(D, w["F"], w["E"], w["k"], renormalize=True, device=local,
                                      max_tokens=max(T, BATCH_TOKENS))
    worker.synth_layer(0, w["seed"])
    stream = torch.cuda.Stream()
    s = stream.cuda_stream
    # the step's inputs are resident in HBM: step i reads token buffer i % 16
    tokens = torch.from_numpy(make_tokens(w, N_TOKENS)).cuda()
    out = torch.empty(T, D, device="cuda")
    torch.cuda.synchronize()

    def step(i):
        worker.forward_dev(0, tokens[i % N_TOKENS].data_ptr(), T, w["flags"], out.data_ptr(), stream=s)

    # A serving loop replays captured launches.  Up to MAX_ONE_GRAPH steps are
    # one CUDA graph of exactly `steps` consecutive decode steps (one layer
    # launch each, token buffers i % 16); more steps replay a graph of 16
    # steps and one graph of the remainder.  Every timed step is a
    # graph-replayed launch and every graph is replayed once before timing.
    for i in range(2):  # first launches (function attributes, tensor maps) outside any capture
        with torch.cuda.stream(stream):
            step(i)
    torch.cuda.synchronize()

    def capture(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(n):
                step(i)
        return g

    if args.steps <= MAX_ONE_GRAPH:
        plan = [(capture(args.steps), 1)]
    else:
        plan = [(capture(N_TOKENS), args.steps // N_TOKENS)]
        if args.steps % N_TOKENS:
            plan.append((capture(args.steps % N_TOKENS), 1))
    warm_graph = capture(N_TOKENS)  # for the extra warm-up below
    with torch.cuda.stream(stream):
        for g, _ in plan:
            g.replay()
    torch.cuda.synchronize()
    worker.poll_error()

    def replay_steps():
        for g, reps in plan:
            for _ in range(reps):
                g.replay()

    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    # The W warm-up steps run right before the timed region (after the clock
    # sampler's start-up pause), then the same launches keep the GPU busy for
    # ~30 ms more (40 replays of 16 steps), so the timed steps do not start on
    # a GPU that idled.
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i)
        for _ in range(40):
            warm_graph.replay()
    torch.cuda.synchronize()
    worker.poll_error()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        # an untimed spin kernel (~100 us) ahead of the start event, so the
        # first timed launch is already queued when the event fires and the
        # host's launch latency stays out of the timed region
        torch.cuda._sleep(200000)
        ev0.record(stream)
        replay_steps()
        ev1.record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    ms_total = ev0.elapsed_time(ev1)
    clocks = sampler.stop() if sampler else None
    worker.poll_error()
    t = torch.tensor([ms_total], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total = float(t.item())
    value = world * args.steps * T / (ms_total / 1000.0)

    # Per-kernel device times (CUDA events on the launching stream, same step):
    # the fused layer launch the graph replays, and for comparison the same
    # step as three launches (router, gate/up+SwiGLU, down+combine).
    def kernel_times(flags):
        worker.set_profiling(True)
        kt = []
        nprof = min(max(args.steps, 20), 400)
        with torch.cuda.stream(stream):
            for i in range(nprof):
                worker.forward_dev(0, tokens[i % N_TOKENS].data_ptr(), T, flags, out.data_ptr(), stream=s)
                kt.append(worker.kernel_times_ms())
        worker.set_profiling(False)
        return np.array(kt)

    kf = kernel_times(w["flags"])
    if kf.shape[1] != 1:
        raise RuntimeError(f"expected the single fused decode launch, got {kf.shape[1]} launches")
    ku = kernel_times(w["flags"] | GLC_FWD_UNFUSED)  # [n, 3]
    fused_avg = float(kf[:, 0].mean())
    med = np.median(ku, axis=0)
    avg = ku.mean(axis=0)
    ab = algorithmic_bytes(w)
    peak, peak_kind = peaks()
    fused_gbs = ab["step"] / (fused_avg * 1e-3) / 1e9
    gu_gbs = ab["gateup"] / (avg[1] * 1e-3) / 1e9
    dn_gbs = ab["down"] / (avg[2] * 1e-3) / 1e9
    layer_gbs = ab["step"] / (ms_total / args.steps * 1e-3) / 1e9

    # End to end through the public host API: pinned host input -> H2D ->
    # layer -> D2H output + expert ids/weights, every step.
    e2e_steps = max(200, min(args.steps, 2000))  # at least 200 calls (~15 ms) for a stable host-clock figure
    hx = torch.from_numpy(make_tokens(w, N_TOKENS)).pin_memory().numpy()
    hout = torch.empty(T, D, pin_memory=True).numpy()
    hids = torch.empty(T, w["k"], dtype=torch.int32, pin_memory=True).numpy()
    hw = torch.empty(T, w["k"], pin_memory=True).numpy()
    import ctypes as C
    L = glc.lib()
    # the buffers' addresses are taken once, as a host holding pinned buffers
    # would; every timed call is the full C-ABI glc_moe_forward on host memory
    fwd = L.glc_moe_forward
    h = worker._handle()
    xp = [hx[i].ctypes.data for i in range(N_TOKENS)]
    op, ip, wp, fl = hout.ctypes.data, hids.ctypes.data, hw.ctypes.data, w["flags"]
    for i in range(min(args.warmup, 20)):
        glc._lib.check(fwd(h, 0, xp[i % N_TOKENS], T, fl, op, ip, wp))
    if dist:
        dist.barrier()
    bad = 0
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        bad |= fwd(h, 0, xp[i % N_TOKENS], T, fl, op, ip, wp)
    e2e_s = time.perf_counter() - t0
    glc._lib.check(bad)  # statuses are 0 or negative: any failure leaves a non-zero OR
    te = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = world * e2e_steps * T / float(te.item())
    del C

    batched = measure_batched(torch, worker, w, stream, args) if not args.skip_batched else None
    gemv = measure_gemv(torch, glc, worker, w, stream) if not args.skip_batched else None
    qwen = None
    if not args.skip_qwen:
        worker.dispose()  # the Qwen layer (1.1 GB) gets the device to itself
        worker = None
        qwen = measure_qwen(torch, glc, args, stream, rank == 0 and world == 1 and not args.skip_cpu_baseline, local)
    ep_leg = measure_ep(torch, dist, glc, w, stream, args, world, rank, local) if not args.skip_ep else None
    dense = measure_dense(torch, dist, glc, args, stream, world, rank, local) if not args.skip_dense else None
    # the Mixtral-8x22B model fits one GPU (~80 GB); measured at N = 1 only (the ranks of a
    # multi-GPU run would each synthesise their own copy on the same host)
    mix22 = measure_mixtral22b(torch, glc, args, stream, local) if (world == 1 and not args.skip_dense) else None
    paging = measure_residency(glc, w, local) if (world == 1 and not args.skip_batched) else None

    cpu_baseline = None
    if rank == 0 and world == 1 and not args.skip_cpu_baseline:
        o, Lc = cpu_layer(w)
        nthreads = os.cpu_count() or 1
        r, n, el = cpu_run(o, Lc, w, make_tokens(w, N_TOKENS), args.cpu_seconds, nthreads)
        cpu_baseline = {"value": r, "unit": UNIT, "cores": nthreads, "kind": "port",
                        "sample": f"{n} decode tokens in {el:.1f} s through the CPU port of the "
                                  f"reference CPU path, same layer and inputs"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_total / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "q4k-int16dp-f32",
            "data": "synthetic (seeded generator; no checkpoint offline)",
            "config": workload_config(w, world),
            "submission": "one fused layer launch per step (glc_moe_forward_dev) on the step's resident token "
                          "buffer; the timed steps are one replayed CUDA graph of all of them (up to 512 steps; "
                          "more: graphs of 16 steps plus one of the remainder), no direct launch is timed",
            "roofline": {"bound": "hbm", "kernel": "moe_decode_fused_kernel (router + gate/up+SwiGLU + "
                                                      "down+combine, one launch per step)",
                         "achieved": layer_gbs, "peak": peak, "unit": "GB/s", "frac": layer_gbs / peak,
                         "peak_kind": peak_kind,
                         "algorithmic_bytes_per_launch": ab["step"],
                         # one fused launch per step, nothing else on the stream: the
                         # timed region's CUDA events give its average duration
                         "avg_launch_ms": ms_total / args.steps,
                         "isolated_launch_ms": fused_avg,
                         "traffic": profile_traffic("moe_decode_fused_kernel_mixtral_t1")},
            "kernels": {"fused_layer_ms": fused_avg, "fused_layer_ms_median": float(np.median(kf[:, 0])),
                        "fused_layer_note": "event marks around each launch (adds the marks' own gaps)",
                        "isolated_launch_gbs": fused_gbs,
                        "layer_gbs": layer_gbs, "layer_frac": layer_gbs / peak,
                        "algorithmic_bytes_per_step": ab["step"],
                        "unfused": {"router_ms": float(avg[0]), "gateup_ms": float(avg[1]),
                                    "down_ms": float(avg[2]), "gateup_ms_median": float(med[1]),
                                    "down_ms_median": float(med[2]), "gateup_gbs": gu_gbs,
                                    "gateup_frac": gu_gbs / peak, "down_gbs": dn_gbs,
                                    "down_frac": dn_gbs / peak,
                                    "note": "same step as three launches (q4k_gemv_kernel x2 + router), "
                                            "event marks between launches"}},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": T * D * 4,
                    "d2h_bytes_per_step": host_result_bytes(T, D, w["k"]), "steps": e2e_steps,
                    "api": "glc_moe_forward (host buffers, synchronous)"},
            "gpu_launches": args.steps,
            "clocks": clocks,
        }
        if cpu_baseline:
            line["cpu_baseline"] = cpu_baseline
        if batched:
            line["batched_64"] = batched
        if gemv:
            line["gemv_isolated"] = gemv
        if qwen:
            line["qwen2_57b"] = qwen
        if dense is not None:
            line["dense_pp"] = dense
        if mix22 is not None:
            line["mixtral8x22b"] = mix22
        if paging is not None:
            line["expert_residency"] = paging
        if ep_leg is not None:
            line["ep"] = ep_leg
        print(json.dumps(line), flush=True)
    if worker is not None:
        worker.dispose()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def measure_gemv(torch, glc, worker, w, stream):
    """The Q4_K GEMV (the MatVecMul drop-in) in isolation: y = W x at K=4096,
    N=28672 (gate + up rows of one expert pair) and K=14336, N=8192 (down rows
    of two experts), each over 4 distinct 66 MB weight copies (the resident
    layer's experts: 264 MB rotating, more than L2) in turn.

    Headline: glc_gemv_q4k_chain_dev, 64 GEMVs in one launch, every GEMV after
    the first behind a grid-wide wait for the one before (as if it read its
    output), replayed from a CUDA graph; per-GEMV time = launch time / 64.
    Beside it: glc_gemv_q4k_dev as a CUDA graph of 64 programmatically
    serialised launches, and the event-timed single launch."""
    D, F = w["D"], w["F"]
    g, u, d, r = worker.layer_device_ptrs(0)
    gu_bytes, dn_bytes = F * q4k_row_bytes(D), D * q4k_row_bytes(F)  # one expert's matrix
    shapes = {"K4096_N28672": (D, 2 * F, [g + i * 2 * gu_bytes for i in range(4)]),
              "K14336_N8192": (F, 2 * D, [d + i * 2 * dn_bytes for i in range(4)])}
    peak, _ = peaks()
    s = stream.cuda_stream
    res = {}
    rng = np.random.default_rng(7)
    for name, (K, N, copies) in shapes.items():
        x = torch.from_numpy(rng.standard_normal(K).astype(np.float32)).cuda()
        y = torch.empty(N, device="cuda")
        nbytes = N * q4k_row_bytes(K)
        launches = 64
        with torch.cuda.stream(stream):
            for i in range(4):
                glc.gemv_q4k_dev(copies[i], x.data_ptr(), y.data_ptr(), K, N, s)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for i in range(launches):
                    glc.gemv_q4k_dev(copies[i % 4], x.data_ptr(), y.data_ptr(), K, N, s)
            graph.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda._sleep(200000)
            e0.record(stream)
            for _ in range(4):
                graph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            per = e0.elapsed_time(e1) / (4 * launches)
            single = []
            for i in range(20):
                e0.record(stream)
                glc.gemv_q4k_dev(copies[i % 4], x.data_ptr(), y.data_ptr(), K, N, s)
                e1.record(stream)
                torch.cuda.synchronize()
                single.append(e0.elapsed_time(e1))
        del graph
        # the chain: 64 GEMVs in one launch, each behind a grid-wide wait
        jobs = [dict(W=copies[i % 4], x=x.data_ptr(), y=y.data_ptr(), K=K, N=N, after_previous=i > 0)
                for i in range(launches)]
        with torch.cuda.stream(stream):
            glc.gemv_q4k_chain_dev(jobs, s)
            torch.cuda.synchronize()
            cgraph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(cgraph, stream=stream):
                glc.gemv_q4k_chain_dev(jobs, s)
            cgraph.replay()
            torch.cuda.synchronize()
            torch.cuda._sleep(200000)
            e0.record(stream)
            for _ in range(4):
                cgraph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            per_chain = e0.elapsed_time(e1) / (4 * launches)
        del cgraph
        glc.gemv_poll_error()
        gbs = nbytes / (per_chain * 1e-3) / 1e9
        res[name] = {"K": K, "N": N, "weight_bytes": nbytes, "ms_per_gemv": per_chain, "gbs": gbs,
                     "frac": gbs / peak,
                     "submission": f"glc_gemv_q4k_chain_dev: {launches} GEMVs over 4 rotating copies in one launch, "
                                   "each behind a grid-wide wait for the one before; CUDA graph replayed",
                     "separate_launches": {"ms_per_launch": per, "frac": nbytes / (per * 1e-3) / 1e9 / peak,
                                           "submission": f"glc_gemv_q4k_dev: CUDA graph of {launches} "
                                                         "programmatically serialised launches, replayed"},
                     "single_launch_ms_median": float(np.median(single)),
                     "single_launch_frac": nbytes / (float(np.median(single)) * 1e-3) / 1e9 / peak}
    return res


def measure_batched(torch, worker, w, stream, args):
    """The same layer on a 64-token batch (router, dispatch plan, operand split,
    grouped tcgen05 gate/up+SwiGLU, split, grouped down, combine): device time
    per batch and per kernel, CUDA events on the launching stream."""
    D, T = w["D"], BATCH_TOKENS
    rng = np.random.default_rng(w["seed"] + 1)
    xs = [torch.from_numpy(rng.standard_normal((T, D)).astype(np.float32)).cuda() for _ in range(4)]
    out = torch.empty(T, D, device="cuda")
    s = stream.cuda_stream
    reps = max(10, min(200, args.steps // 100))
    reps = (reps + 3) // 4 * 4
    with torch.cuda.stream(stream):
        for i in range(3):
            worker.forward_dev(0, xs[i % 4].data_ptr(), T, w["flags"], out.data_ptr(), stream=s)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(reps):
            worker.forward_dev(0, xs[i % 4].data_ptr(), T, w["flags"], out.data_ptr(), stream=s)
        e1.record(stream)
        torch.cuda.synchronize()
        ms_direct = e0.elapsed_time(e1) / reps
    # as the decode leg: four batches (the four inputs) captured in one CUDA
    # graph and replayed
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(4):
            worker.forward_dev(0, xs[i].data_ptr(), T, w["flags"], out.data_ptr(), stream=s)
    with torch.cuda.stream(stream):
        graph.replay()
        torch.cuda.synchronize()
        e0.record(stream)
        for i in range(reps // 4):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
    del graph
    with torch.cuda.stream(stream):
        worker.set_profiling(True)
        kt = []
        for i in range(reps):
            worker.forward_dev(0, xs[i % 4].data_ptr(), T, w["flags"], out.data_ptr(), stream=s)
            kt.append(worker.kernel_times_ms())
        worker.set_profiling(False)
    worker.poll_error()
    kt = np.array(kt).mean(axis=0)
    names = ["router", "dispatch_plan", "split_x", "grouped_gateup", "split_act", "grouped_down", "combine"]
    expert_bytes = 3 * w["F"] * q4k_row_bytes(w["D"])  # gate + up + down of one expert
    weight_bytes = w["E"] * expert_bytes  # a 64-token batch touches all 8 experts
    peak, _ = peaks()
    gu = kt[3] if len(kt) > 3 else float("nan")
    dn = kt[5] if len(kt) > 5 else float("nan")
    return {"workload": "mixtral8x7b_moe_layer_prefill_64", "tokens": T, "ms_per_batch": ms,
            "ms_per_batch_direct_launches": ms_direct,
            "submission": "4 batches captured in one CUDA graph and replayed (direct launches beside it)",
            "tokens_per_s": T / (ms * 1e-3), "weight_bytes": weight_bytes,
            "layer_gbs": weight_bytes / (ms * 1e-3) / 1e9,
            "grouped_gateup_gbs": (2 * w["E"] * w["F"] * q4k_row_bytes(D)) / (gu * 1e-3) / 1e9,
            "grouped_down_gbs": (w["E"] * D * q4k_row_bytes(w["F"])) / (dn * 1e-3) / 1e9,
            "peak_gbs": peak,
            "kernel_ms": {n: float(v) for n, v in zip(names, kt)}}


def measure_residency(glc, w, local):
    """Expert residency (glc_moe_set_expert_slots): the same Mixtral layer with
    HBM slots for 4 of its 8 experts, the others paged in from pinned host
    memory as the routing selects them (least recently used out); decode
    tokens through the host-buffer forward.  Host wall clock per synchronous
    call: the forward waits on the host for each call's routing."""
    D, F, E, k = w["D"], w["F"], w["E"], w["k"]
    slots = 4
    paged = glc.GpuExpertStageWorker(D, F, E, k, renormalize=True, device=local, max_tokens=1, expert_slots=slots)
    paged.synth_layer(0, w["seed"])
    toks = make_tokens(w, N_TOKENS)
    for i in range(3):
        paged.forward(0, toks[i], w["flags"])
    c0 = paged.expert_residency()
    n = 48
    t0 = time.perf_counter()
    for i in range(n):
        paged.forward(0, toks[i % N_TOKENS], w["flags"])
    el = time.perf_counter() - t0
    c1 = paged.expert_residency()
    paged.poll_error()
    paged.dispose()
    hits, tr = c1["hits"] - c0["hits"], c1["transfers"] - c0["transfers"]
    eb = 3 * F * q4k_row_bytes(D)
    return {"workload": "mixtral8x7b_moe_layer_decode_paged", "slots": slots, "experts": E, "tokens": n,
            "ms_per_token": el * 1e3 / n, "hit_rate": hits / max(hits + tr, 1), "transfers_per_token": tr / n,
            "expert_bytes": eb, "host_to_hbm_gbs": tr * eb / el / 1e9,
            "note": f"{N_TOKENS} rotating tokens; every miss copies one expert (gate, up, down) from pinned host memory"}


QWEN = dict(name="qwen2_57b_a14b_moe_layer", D=3584, F=2560, E=64, k=8, Fs=20480, seed=20241202, flags=3)
QWEN_T = (1, 16, 256)


def qwen_tokens(args):
    return tuple(int(t) for t in str(getattr(args, "qwen_tokens", "")).split(",") if t.strip()) or QWEN_T


def qwen_host_layer(glc, w, worker):
    """Host copies of the config's weights for the CPU port: the routed experts
    and router read back from the device, the shared expert from the same
    seeded generator (byte-identical to the device's, tested)."""
    from cuda.bindings import runtime as rt
    from oracle import oracle as o
    D, F, E, Fs = w["D"], w["F"], w["E"], w["Fs"]
    gb, db = E * F * q4k_row_bytes(D), E * D * q4k_row_bytes(F)
    L = {}
    for key, ptr, n in zip(("gate", "up", "down", "router"), worker.layer_device_ptrs(0), (gb, gb, db, 4 * D * E)):
        buf = np.empty(n, np.uint8)
        err, = rt.cudaMemcpy(buf.ctypes.data, ptr, n, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
        if int(err) != 0:
            raise RuntimeError(f"device-to-host copy of {key} failed: {err}")
        L[key] = buf if key != "router" else buf.view(np.float32)
    L["sh_gate"] = o.synth_q4k(w["seed"], o.expert_tag(65535, 0), Fs, D)
    L["sh_up"] = o.synth_q4k(w["seed"], o.expert_tag(65535, 1), Fs, D)
    L["sh_down"] = o.synth_q4k(w["seed"], o.expert_tag(65535, 2), D, Fs)
    L["sh_gate_vec"] = o.fill_normal(w["seed"], 3, 0.02, D)
    return o, L


def measure_qwen(torch, glc, args, stream, want_cpu, local=0):
    """Qwen2-57B-A14B-shaped MoE layer (hidden 3584, 64 experts top-8 softmax
    without renormalisation, SwiGLU experts 3584->2560->3584, a sigmoid-gated
    shared expert 3584->20480->3584, all Q4_K) at token batches of 1, 16 and
    256: device time per call (four rotating input batches captured in one CUDA
    graph and replayed), tokens/s, and the HBM roofline of the whole layer
    call, with algorithmic bytes = distinct experts the batch touches (counted
    from the ids the call returns) x 15,482,880 B + the shared expert's
    123,863,040 B + the router + activations."""
    w = QWEN
    D, F, E, k, Fs = w["D"], w["F"], w["E"], w["k"], w["Fs"]
    worker = glc.GpuExpertStageWorker(D, F, E, k, shared_ffn_dim=Fs, renormalize=False, device=local,
                                      max_tokens=max(qwen_tokens(args)))
    worker.synth_layer(0, w["seed"])
    s = stream.cuda_stream
    peak, _ = peaks()
    expert_bytes = 2 * F * q4k_row_bytes(D) + D * q4k_row_bytes(F)
    shared_bytes = 2 * Fs * q4k_row_bytes(D) + D * q4k_row_bytes(Fs)
    legs = {}
    rng = np.random.default_rng(w["seed"])
    for T in qwen_tokens(args):
        xs = [torch.from_numpy(rng.standard_normal((T, D)).astype(np.float32)).cuda() for _ in range(4)]
        out = torch.empty(T, D, device="cuda")
        ids = [torch.empty(T, k, dtype=torch.int32, device="cuda") for _ in range(4)]
        wts = torch.empty(T, k, device="cuda")
        with torch.cuda.stream(stream):
            for i in range(4):
                worker.forward_dev(0, xs[i].data_ptr(), T, w["flags"], out.data_ptr(), ids[i].data_ptr(),
                                   wts.data_ptr(), stream=s)
        torch.cuda.synchronize()
        worker.poll_error()
        distinct = [len(np.unique(t.cpu().numpy())) for t in ids]
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(4):
                worker.forward_dev(0, xs[i].data_ptr(), T, w["flags"], out.data_ptr(), stream=s)
        reps = max(5, min(100, int(2000 // (1 + T // 4))))
        with torch.cuda.stream(stream):
            graph.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda._sleep(200000)
            e0.record(stream)
            for _ in range(reps):
                graph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / (4 * reps)
        del graph
        worker.poll_error()
        # launches per call and each kernel's share, from the event marks
        worker.set_profiling(True)
        with torch.cuda.stream(stream):
            worker.forward_dev(0, xs[0].data_ptr(), T, w["flags"], out.data_ptr(), stream=s)
            torch.cuda.synchronize()
        kt = worker.kernel_times_ms()
        worker.set_profiling(False)
        act_bytes = 4 * T * D * 3 + 4 * T * k * (2 * F) + 4 * T * 2 * Fs
        alg = float(np.mean(distinct)) * expert_bytes + shared_bytes + 4 * D * E + 4 * D + act_bytes
        gbs = alg / (ms * 1e-3) / 1e9
        legs[f"T{T}"] = {"workload": f"qwen2_57b_moe_layer_T{T}", "tokens": T, "ms_per_call": ms,
                         "tokens_per_s": T / (ms * 1e-3), "distinct_experts_mean": float(np.mean(distinct)),
                         "algorithmic_bytes": alg, "achieved_gbs": gbs, "peak_gbs": peak, "frac": gbs / peak,
                         "launches_per_call": len(kt), "kernel_ms": [round(v, 4) for v in kt],
                         "submission": "4 calls (rotating inputs) captured in one CUDA graph and replayed"}
    cpu = None
    if want_cpu:
        o, L = qwen_host_layer(glc, w, worker)
        nthreads = os.cpu_count() or 1
        x = make_tokens(dict(w, T=1), 4)
        outh = np.empty(D, np.float32)
        n, t0 = 0, time.perf_counter()
        while n < 2 or time.perf_counter() - t0 < args.cpu_seconds / 3:
            o.lib().oc_cpu_moe_token_shared_fast(L["gate"], L["up"], L["down"], L["router"], L["sh_gate"],
                                                 L["sh_up"], L["sh_down"], L["sh_gate_vec"], D, F, E, k, Fs, 0,
                                                 w["flags"], x[n % 4][0], outh, nthreads)
            n += 1
        el = time.perf_counter() - t0
        cpu = {"value": n / el, "unit": UNIT, "cores": nthreads, "kind": "port",
               "sample": f"{n} tokens one at a time in {el:.1f} s through the CPU port of the reference CPU "
                         f"path (routed experts + shared expert), same layer"}
    worker.dispose()
    return {"legs": legs, "cpu_baseline": cpu}


EP_TOKENS = 8  # decode tokens per rank in the expert-parallel leg (Mixtral layer)
EP_QWEN_T = (16, 256)  # tokens per rank of the Qwen2-57B expert-parallel legs
EP_PHASES = ["route", "dispatch", "exchange_out", "experts", "exchange_back", "combine"]


def ep_communicator(glc, dist, world, rank, local):
    """The C ABI's own NCCL communicator (glc_comm_*): the exchange a host
    without torch.distributed uses.  torch.distributed only hands rank 0's id
    to the other ranks."""
    uid = glc.Communicator.unique_id() if rank == 0 else None
    if dist:
        box = [uid]
        dist.broadcast_object_list(box, src=0)
        uid = box[0]
    return glc.Communicator(uid, world, rank, local)


def ep_time(torch, dist, shard, comm, xs, T, flags, stream, steps):
    """Device time per expert-parallel step (max over ranks) and the mean of
    each phase (route, dispatch, exchange out, experts, exchange back, combine)."""
    D = xs[0].shape[1]
    out = torch.empty(T, D, device="cuda")
    s = stream.cuda_stream
    with torch.cuda.stream(stream):
        for i in range(3):
            shard.ep_forward_dev(comm, 0, xs[i % len(xs)].data_ptr(), T, flags, out.data_ptr(), stream=s)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(steps):
            shard.ep_forward_dev(comm, 0, xs[i % len(xs)].data_ptr(), T, flags, out.data_ptr(), stream=s)
        e1.record(stream)
        torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    shard.set_profiling(True)
    ph = []
    with torch.cuda.stream(stream):
        for i in range(8):
            shard.ep_forward_dev(comm, 0, xs[i % len(xs)].data_ptr(), T, flags, out.data_ptr(), stream=s)
            torch.cuda.synchronize()
            ph.append(shard.kernel_times_ms())
    shard.set_profiling(False)
    shard.poll_error()
    phases = {n: float(v) for n, v in zip(EP_PHASES, np.mean(np.array(ph), axis=0))}
    return float(t.item()), phases


DENSE = dict(name="qwen25_14b_decode", D=5120, FF=13824, Hq=40, Hkv=8, layers=48, vocab=152064, max_len=2048,
             seed=20241203)
DENSE_SPLITS = {1: [48], 2: [27, 21], 4: [12, 12, 12, 12], 8: [6] * 8}
DENSE_STEPS = 16


def dense_token_bytes(q, pos):
    """Bytes one token moves through the whole model: every layer's Q4_K
    matrices, its KV cache rows 0..pos (K and V, fp16), the embedding row and
    the LM head."""
    rb = lambda k: q4k_row_bytes(k)
    D, FF, Hq, Hkv = q["D"], q["FF"], q["Hq"], q["Hkv"]
    layer = (Hq + 2 * Hkv) * 128 * rb(D) + D * rb(Hq * 128) + 2 * FF * rb(D) + D * rb(FF)
    kv = 2 * Hkv * (pos + 1) * 128 * 2
    return q["layers"] * (layer + kv) + q["vocab"] * rb(D) + rb(D)


def measure_dense(torch, dist, glc, args, stream, world, rank, local):
    """Dense decoder decode (Qwen2.5-14B geometry: 48 layers, hidden 5120, FFN
    13824, 40 query / 8 KV heads, head dim 128, RoPE theta 1e6, vocab 152064,
    a 2048-position fp16 KV cache, batch 1), greedy: every layer as a
    DenseStage (glc_stage_forward_dev, one captured graph per stage step).
    N = 1: the whole model on one GPU.  N > 1: pipeline stages (27:21 at
    N = 2, even splits at 4 / 8), the activation crossing every boundary as a
    FusedActivationHeader + symmetric INT8 payload (glc_pp_send / glc_pp_recv,
    5,124 B per token), the arg-max token handed back from the last stage to
    the first (glc_comm_send / recv).  Decode steps at the last positions of
    the cache (attention over up to 2048 rows); device time per token, max
    over ranks."""
    q = DENSE
    split = DENSE_SPLITS.get(world) or [q["layers"] // world] * world
    begin, count = sum(split[:rank]), split[rank]
    first, last = rank == 0, rank == world - 1
    D = q["D"]
    st = glc.DenseStage(D, q["FF"], q["Hq"], q["Hkv"], begin, count, q["max_len"], 1e6, 1e-6, q["vocab"], first,
                        last, local)
    for l in range(count):
        st.synth_layer(l, q["seed"])
    st.synth_io(q["seed"])
    comm = ep_communicator(glc, dist, world, rank, local) if world > 1 else None
    s = stream.cuda_stream
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    x = torch.empty(D, device="cuda")
    hdr = glc.FusedActivationHeader(1, 0, begin + count, D, 2, 0, 1.0, 1)  # INT8 wire

    def step(pos):
        if first:
            st.forward_dev(pos, token_ptr=tok.data_ptr(), x_out_ptr=x.data_ptr(),
                           token_out_ptr=tok.data_ptr() if last else None, stream=s)
        else:
            comm.pp_recv(rank - 1, x.data_ptr(), 1, D, s)
            st.forward_dev(pos, x_in_ptr=x.data_ptr(), x_out_ptr=None if last else x.data_ptr(),
                           token_out_ptr=tok.data_ptr() if last else None, stream=s)
        if not last:
            comm.pp_send(rank + 1, hdr, x.data_ptr(), s)
        if world > 1 and last:
            comm.send(0, tok.data_ptr(), 4, s)
        if world > 1 and first:
            comm.recv(world - 1, tok.data_ptr(), 4, s)

    p0 = q["max_len"] - DENSE_STEPS - 3
    with torch.cuda.stream(stream):
        for i in range(3):
            step(p0 + i)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(DENSE_STEPS):
            step(p0 + 3 + i)
        e1.record(stream)
        torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / DENSE_STEPS], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    st.poll_error()
    st.dispose()
    if comm:
        comm.dispose()
    peak, _ = peaks()
    tb = dense_token_bytes(q, q["max_len"] - 1)
    gbs = tb / (ms * 1e-3) / 1e9
    return {"workload": f"{q['name']}_pp{world}", "layers": q["layers"], "stage_layers": split,
            "ms_per_token": ms, "tokens_per_s": 1000.0 / ms, "steps": DENSE_STEPS,
            "positions": [p0 + 3, p0 + 2 + DENSE_STEPS], "bytes_per_token": tb,
            "achieved_gbs_whole_model": gbs, "frac_of_one_gpu_peak": gbs / peak,
            "boundary": "FusedActivationHeader + INT8 payload (5,124 B / token) per stage boundary" if world > 1
                        else "single GPU", "submission": "one captured graph per stage step, replayed per token"}


MIXTRAL22B = dict(name="mixtral8x22b_decode", D=6144, F=16384, E=8, k=2, Hq=48, Hkv=8, layers=56, vocab=32768,
                  max_len=4096, seed=20241204)


def moe_token_bytes(q, pos):
    """Bytes one token moves through the whole mixture-of-experts model: every
    layer's attention matrices, its KV cache rows 0..pos, the router and the
    k routed experts' gate / up / down Q4_K rows, the embedding row and the LM
    head."""
    rb = q4k_row_bytes
    D, F, Hq, Hkv, E, k = q["D"], q["F"], q["Hq"], q["Hkv"], q["E"], q["k"]
    attn = (Hq + 2 * Hkv) * 128 * rb(D) + D * rb(Hq * 128)
    experts = k * (2 * F * rb(D) + D * rb(F))
    kv = 2 * Hkv * (pos + 1) * 128 * 2
    return q["layers"] * (attn + experts + D * E * 4 + kv) + q["vocab"] * rb(D) + rb(D)


def measure_mixtral22b(torch, glc, args, stream, local):
    """The whole Mixtral-8x22B-shaped model (56 layers of attention
    (48 query / 8 KV heads, a 4096-position fp16 cache) and a mixture-of-experts
    feed-forward of 8 SwiGLU experts, FFN 16384, top-2 renormalised, hidden 6144,
    vocab 32768; random-init Q4_K, ~80 GB resident) decoding greedily at batch
    1 at the last positions of the cache, one GPU: every layer through
    glc_stage_forward_dev (attention launch, O projection, router, routed
    gate/up and down GEMVs, next QKV), one captured graph per token."""
    q = MIXTRAL22B
    D = q["D"]
    st = glc.DenseStage(D, 0, q["Hq"], q["Hkv"], 0, q["layers"], q["max_len"], 1e6, 1e-5, q["vocab"], True, True,
                        local, num_experts=q["E"], top_k=q["k"], expert_ffn_dim=q["F"], moe_renormalize=True)
    t0 = time.perf_counter()
    for l in range(q["layers"]):
        st.synth_layer(l, q["seed"])
    st.synth_io(q["seed"])
    synth_s = time.perf_counter() - t0
    s = stream.cuda_stream
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    steps = 16
    p0 = q["max_len"] - steps - 3
    with torch.cuda.stream(stream):
        for i in range(3):
            st.forward_dev(p0 + i, token_ptr=tok.data_ptr(), token_out_ptr=tok.data_ptr(), stream=s)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(steps):
            st.forward_dev(p0 + 3 + i, token_ptr=tok.data_ptr(), token_out_ptr=tok.data_ptr(), stream=s)
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    st.poll_error()
    st.dispose()
    peak, _ = peaks()
    tb = moe_token_bytes(q, q["max_len"] - 1)
    gbs = tb / (ms * 1e-3) / 1e9
    return {"workload": f"{q['name']}_batch1", "layers": q["layers"], "ms_per_token": ms, "tokens_per_s": 1000.0 / ms,
            "steps": steps, "positions": [p0 + 3, p0 + 2 + steps], "bytes_per_token": tb,
            "achieved_gbs": gbs, "frac": gbs / peak, "weights_synthesised_s": round(synth_s, 1),
            "submission": "one captured graph per token (7 launches per layer), greedy token fed back on the device"}


def measure_ep(torch, dist, glc, w, stream, args, world, rank, local):
    """Expert parallelism through the C ABI (glc_moe_ep_forward, the call a C#
    host binds: NCCL inside the library, no torch.distributed on the data
    path): E / world experts per rank, fixed-size dispatch blocks exchanged
    with one grouped NCCL send/receive each way (no host read of the counts),
    grouped tensor-core experts on the rows each rank receives, k-ordered
    combine at home.  Every rank checks its output, ids and weights against
    its own single-GPU layer on the same tokens; device time per step as the
    max over ranks, with the per-phase breakdown."""
    D, F, E, k = w["D"], w["F"], w["E"], w["k"]
    epr = E // world
    comm = ep_communicator(glc, dist, world, rank, local)
    res = {"exchange": "fixed-size per-rank blocks (worst case T*k rows), one grouped ncclSend/ncclRecv each way, "
                       "counts read on the device only",
           "api": "glc_moe_ep_forward (C ABI, communicator glc_comm)"}
    flags = w["flags"] | GLC_FWD_BATCHED
    # ---- Mixtral-8x7B layer, EP_TOKENS decode tokens per rank
    T = EP_TOKENS
    shard = glc.GpuExpertStageWorker(D, F, E, k, renormalize=True, device=local, max_tokens=world * T,
                                     expert_begin=rank * epr, expert_count=epr)
    shard.synth_layer(0, w["seed"])
    rng = np.random.default_rng(w["seed"] + 100 + rank)
    xh = [rng.standard_normal((T, D)).astype(np.float32) for _ in range(4)]
    xs = [torch.from_numpy(x).cuda() for x in xh]
    # parity: this rank's tokens against its own single-GPU layer (batched path)
    full = glc.GpuExpertStageWorker(D, F, E, k, renormalize=True, device=local, max_tokens=T)
    full.synth_layer(0, w["seed"])
    out = torch.empty(T, D, device="cuda")
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    wts = torch.empty(T, k, device="cuda")
    shard.ep_forward_dev(comm, 0, xs[0].data_ptr(), T, flags, out.data_ptr(), ids.data_ptr(), wts.data_ptr())
    torch.cuda.synchronize()
    fo, fids, fw = full.forward(0, xh[0], flags)
    full.dispose()
    eo = out.cpu().numpy()
    exact = bool(np.array_equal(eo, fo) and np.array_equal(ids.cpu().numpy(), fids)
                 and np.array_equal(wts.cpu().numpy(), fw))
    ok = torch.tensor([1 if exact else 0], device="cuda")
    if dist:
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    peer = comm.peer_exchange_active()
    res["exchange"] = ("NVLink peer memory: the pack and repack kernels write each rank's blocks into the "
                       "destination's CUDA IPC window, an epoch flag per source, only routed rows cross"
                       if peer else res["exchange"])
    steps = max(20, min(args.steps // 10, 200))
    ms, phases = ep_time(torch, dist, shard, comm, xs, T, flags, stream, steps)
    nccl_ms = None
    if peer:  # the same step with the blocks through NCCL, for comparison
        comm.set_peer_exchange(False)
        nccl_ms, _ = ep_time(torch, dist, shard, comm, xs, T, flags, stream, steps)
        comm.set_peer_exchange(True)
    shard.dispose()
    res["mixtral"] = {"workload": f"mixtral8x7b_moe_layer_decode_ep{world}", "experts_per_rank": epr,
                      "tokens_per_rank": T, "ms_per_step": ms, "tokens_per_s": world * T / (ms * 1e-3),
                      "tokens_per_s_per_gpu": T / (ms * 1e-3), "steps": steps, "phases_ms": phases,
                      "nccl_exchange_ms_per_step": nccl_ms,
                      "parity": {"bit_exact_vs_single_gpu_all_ranks": bool(ok.item() == 1),
                                 "reference": "each rank's own single-GPU layer, batched path, same tokens"}}
    # ---- Qwen2-57B layer, 64 / world experts per rank + the shared expert
    if not args.skip_qwen:
        q = QWEN
        Dq, Fq, Eq, kq, Fsq = q["D"], q["F"], q["E"], q["k"], q["Fs"]
        eq = Eq // world
        for Tq in EP_QWEN_T:
            # a handle sized for this batch: the exchange blocks hold the worst
            # case of max_tokens / world tokens per rank
            shard = glc.GpuExpertStageWorker(Dq, Fq, Eq, kq, shared_ffn_dim=Fsq, renormalize=False, device=local,
                                             max_tokens=world * Tq, expert_begin=rank * eq, expert_count=eq)
            shard.synth_layer(0, q["seed"])
            xs = [torch.from_numpy(rng.standard_normal((Tq, Dq)).astype(np.float32)).cuda() for _ in range(2)]
            stq = max(5, min(steps, 2000 // Tq))
            ms, phases = ep_time(torch, dist, shard, comm, xs, Tq, q["flags"] | GLC_FWD_BATCHED, stream, stq)
            res[f"qwen2_57b_T{Tq}"] = {"workload": f"qwen2_57b_moe_layer_ep{world}_T{Tq}", "experts_per_rank": eq,
                                        "tokens_per_rank": Tq, "ms_per_step": ms,
                                        "tokens_per_s": world * Tq / (ms * 1e-3),
                                        "tokens_per_s_per_gpu": Tq / (ms * 1e-3), "steps": stq,
                                        "phases_ms": phases}
            shard.dispose()
    comm.dispose()
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--skip-cpu-baseline", action="store_true")
    ap.add_argument("--skip-batched", action="store_true")
    ap.add_argument("--skip-qwen", action="store_true")
    ap.add_argument("--qwen-tokens", default=",".join(map(str, QWEN_T)),
                    help="token batches of the Qwen2-57B layer leg (comma-separated)")
    ap.add_argument("--skip-ep", action="store_true")
    ap.add_argument("--skip-dense", action="store_true", help="skip the whole-model legs (Qwen2.5-14B dense, Mixtral-8x22B)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    w = dict(WORKLOAD)
    if args.impl == "reference":
        return run_reference(args, w)
    return run_ours(args, w)


if __name__ == "__main__":
    sys.exit(main())
