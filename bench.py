"""Benchmark of the B200 matmul path of MVLM (Q4_0 decode GEMV; prefill GEMMs).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one decode token through the GEMV path of Phi-1.5: for each of the 24 layers the
qkv (2048x6144), out (2048x2048), fc1 (2048x8192) and fc2 (8192x2048) GEMVs, then the
2048x51200 lm_head, M=1, fp32 activations, weights ~N(0, 0.02) quantised to GGUF Q4_0 and
kept packed in HBM (BASELINE config 1's layer + head shapes, repeated over the model's 24
layers).  The 738 MB of weights a step reads are ~6x the 126 MB L2, so every step streams
from HBM.  The step is captured once as a CUDA graph through the library's capture API.

value   = algorithmic bytes of a step (packed weights + x + y) / device time per step, GB/s.
e2e     = the same metric through the public C ABI with host buffers: every step copies the
          activations host->device and the outputs device->host.
roofline: the dominant kernel is gemv_q_stream: every one of the 97 launches of a step, back to
          back; achieved = average algorithmic bytes per launch / average launch duration over
          the timed region (CUDA events), against the measured HBM peak.  The lm_head launch
          alone is also reported (marker events captured around it inside the graph).
cpu_baseline: the CPU restatement of the reference's quantised path (dequantise + fp32 dot),
          OpenMP over all host cores, on a bounded sample of the same workload.
prefill : secondary metric: tcgen05 GEMM TFLOP/s on the Phi-1.5 prefill shapes (M=761, Q8_0
          weights dequantised to bf16 in the weight loads).
fused_epilogues: the Phi-1.5 prefill MLP GEMMs with their activation / gate product /
          residual add fused into the epilogue, each against the plain GEMM of the same shape.

With --gpus N (launched by torchrun, one process per GPU, NCCL): the lm_head is
column-sharded (51200/N output rows of W per rank) and the logits are all-gathered with NCCL
over NVLink after every step; the 24 layers' GEMVs are the same on every rank (replicas:
M=1 decode does not shard usefully).  Total work is fixed ("strong" scaling); each rank's
time is measured on its device and the max over ranks is reported.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

METRIC = "Q4_0 decode GEMV HBM GB/s (% peak); prefill GEMM TFLOP/s at 1/2/4/8 B200"
LAYERS = 24
LAYER_SHAPES = [("qkv", 2048, 6144), ("out", 2048, 2048), ("fc1", 2048, 8192), ("fc2", 8192, 2048)]  # (K, N)
HEAD = ("lm_head", 2048, 51200)
PREFILL_SHAPES = [(761, 2048, 6144), (761, 2048, 2048), (761, 2048, 8192), (761, 8192, 2048)]  # (M, K, N)
SEED = 0x4D564C4D


def measured_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def gemv_bytes(K: int, N: int) -> int:
    return N * (K // 32) * 18 + 4 * K + 4 * N


# --------------------------------------------------------------------------------------
# clocks sampled during the timed region
# --------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = os.path.join("/tmp", f"mvlm_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.remove(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# --------------------------------------------------------------------------------------
# CPU baseline: the oracle (test infrastructure) timed on the host cores
# --------------------------------------------------------------------------------------
def cpu_baseline(budget_s: float = 12.0) -> dict:
    import oracle as O
    # all the host threads this process may run on (torchrun sets OMP_NUM_THREADS=1 per rank;
    # only rank 0 runs this)
    O.set_threads(len(os.sched_getaffinity(0)))
    shapes = [(K, N) for _, K, N in LAYER_SHAPES] + [(HEAD[1], HEAD[2])]
    mats = []
    for i, (K, N) in enumerate(shapes):
        W = O.quantize(O.normal(N * K, SEED + 100 + i, 0.02), O.Q4_0)
        x = O.normal(K, SEED + 200 + i, 1.0)
        mats.append((K, N, W, x, np.empty(N, np.float32)))
    L = O.lib()
    nbytes = sum(gemv_bytes(K, N) for K, N, *_ in mats)
    # warm-up pass, then whole passes until the budget is spent
    for K, N, W, x, y in mats:
        L.ora_gemv_q_mt(O._p(x), O._p(W), O._p(y), N, K, O.Q4_0)
    t0 = time.perf_counter()
    passes = 0
    while True:
        for K, N, W, x, y in mats:
            L.ora_gemv_q_mt(O._p(x), O._p(W), O._p(y), N, K, O.Q4_0)
        passes += 1
        if time.perf_counter() - t0 >= budget_s or passes >= 200:
            break
    dt = time.perf_counter() - t0
    return {"value": round(nbytes * passes / dt / 1e9, 3), "unit": "GB/s", "cores": O.max_threads(),
            "kind": "port",
            "sample": f"{passes} passes over one layer (qkv, out, fc1, fc2) + lm_head, Q4_0, M=1, "
                      f"{nbytes / 1e6:.1f} MB per pass, {dt:.1f} s"}


# --------------------------------------------------------------------------------------
# our arm
# --------------------------------------------------------------------------------------
def run_ours(args, rank: int, world: int, local_rank: int) -> dict | None:
    import torch

    import mvlm_b200 as mg

    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    dev = mg.Device(local_rank)
    stream = torch.cuda.Stream()  # a real stream: the legacy default stream cannot be captured
    torch.cuda.set_stream(stream)
    dev.set_stream(stream.cuda_stream)
    dev.set_event_mode(0)
    peaks = measured_peaks()

    # ---------------- weights: generated and quantised on the device ----------------
    from mvlm_b200.shard import column_shard, gather_columns
    h0, h1 = column_shard(HEAD[2], world, rank)
    n_head = h1 - h0
    head_rows = [column_shard(HEAD[2], world, r)[0] for r in range(world)] + [HEAD[2]]
    max_el = max(max(K * N for _, K, N in LAYER_SHAPES), HEAD[1] * n_head)
    tmp = dev.empty(max_el, mg.F32)

    def make_q(K, N, seed):
        w = dev.create_buffer(N * (K // 32) * 18, None, mg.Q4_0, mg.LAYOUT_NK, N, K)
        dev.fill_normal(tmp, N * K, seed, 0.02)
        dev.quantize(tmp, w, N * K, mg.Q4_0)
        return w

    layers = []
    for l in range(LAYERS):
        mats = []
        for j, (name, K, N) in enumerate(LAYER_SHAPES):
            W = make_q(K, N, SEED + 1000 * l + j)
            x = dev.empty(K, mg.F32)
            dev.fill_normal(x, K, SEED + 7 + 1000 * l + j, 1.0)
            y = dev.empty(N, mg.F32)
            mats.append((name, K, N, W, x, y))
        layers.append(mats)
    # lm_head shard: this rank's rows [head_rows[r], head_rows[r+1]) of W[51200][2048]
    K_h = HEAD[1]
    Wh = make_q(K_h, n_head, SEED + 999_999 + rank)
    xh = dev.empty(K_h, mg.F32)
    dev.fill_normal(xh, K_h, SEED + 5, 1.0)
    y_full = torch.empty(HEAD[2], dtype=torch.float32, device="cuda")
    y_shard_t = torch.empty(n_head, dtype=torch.float32, device="cuda")
    yh = dev.wrap(y_shard_t.data_ptr(), n_head * 4, mg.F32)
    del tmp
    dev.finish()

    step_bytes = sum(gemv_bytes(K, N) for _, K, N in LAYER_SHAPES) * LAYERS + gemv_bytes(K_h, HEAD[2])
    launches_per_step = LAYERS * len(LAYER_SHAPES) + 1

    # ---------------- capture one step ----------------
    def enqueue_step():
        for mats in layers:
            for name, K, N, W, x, y in mats:
                mg.gemv_q(dev, x, W, y, N, K, mg.Q4_0)
        m0 = dev.record_event()
        mg.gemv_q(dev, xh, Wh, yh, n_head, K_h, mg.Q4_0)
        m1 = dev.record_event()
        return m0, m1

    enqueue_step()  # eager run first (validates arguments outside capture)
    dev.finish()
    dev.capture_begin()
    head0, head1 = enqueue_step()
    graph = dev.capture_end()

    def gather_logits():
        # one NCCL all-gather of the logit shards over NVLink (all_gather_into_tensor when the
        # shards are equal, as for 51200 / {1,2,4,8})
        if HEAD[2] % world == 0:
            dist.all_gather_into_tensor(y_full, y_shard_t)
        else:
            y_full.copy_(gather_columns(y_shard_t, HEAD[2]))

    def step():
        graph.launch()
        if world > 1:
            gather_logits()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.3)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms_total = ev0.elapsed_time(ev1)
    # lm_head launch duration: marker events captured around it inside the graph, read after
    # each of a few replays (the graph is the same one the timed loop replays)
    head_samples = []
    for _ in range(min(args.steps, 50)):
        step()
        torch.cuda.synchronize()
        head_samples.append(head0.elapsed_ms(head1))
    head_ms = statistics.mean(head_samples)

    ms = ms_total / args.steps
    if world > 1:
        t = torch.tensor([ms, head_ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, head_ms = float(t[0]), float(t[1])

    # ---------------- e2e through the C ABI with host buffers ----------------
    y_full_buf = dev.wrap(y_full.data_ptr(), HEAD[2] * 4, mg.F32) if world > 1 else None
    e2e = run_e2e(args, dev, mg, layers, xh, Wh, yh, n_head, K_h, step_bytes, world, dist, gather_logits, torch,
                  stream, y_full_buf)

    # ---------------- prefill GEMMs (secondary metric) ----------------
    prefill = run_prefill(dev, mg, torch, stream, peaks) if rank == 0 and not args.no_prefill else None
    # ---------------- the other BASELINE configs (secondary, one GPU) ----------------
    secondary = None
    if not args.no_secondary:
        if world == 1:
            secondary = {"fp32_gemv": run_fp32_gemv(dev, mg, torch, stream, peaks),
                         "batched_decode": run_batched_decode(dev, mg, torch, stream, peaks, layers, Wh, K_h, n_head),
                         # before SigLIP, whose seconds of dense MMAs can leave the clocks power-capped
                         "fused_epilogues": _guarded(run_fused_epilogues, dev, mg, torch, stream, peaks),
                         "siglip": run_siglip(dev, mg, torch, stream, peaks)}
        else:
            # every rank takes part (collectives); rank 0 reports
            secondary = {"batched_decode": run_batched_decode(dev, mg, torch, stream, peaks, layers, Wh, K_h, n_head,
                                                              world=world, dist=dist),
                         "siglip": run_siglip(dev, mg, torch, stream, peaks, batches=(8, 64), world=world, dist=dist)}

    graph = None
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return None

    head_bytes = gemv_bytes(K_h, n_head)
    achieved = head_bytes / (head_ms * 1e-3) / 1e9
    value = step_bytes / (ms * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "pct_of_peak": round(100.0 * value / peaks["hbm_gbs"], 1),
        "data": "synthetic: weights ~N(0,0.02) seeded, quantised to GGUF Q4_0 on the device; x ~N(0,1) fp32",
        "config": {"workload": "Q4_0 decode GEMV sweep, M=1: 24 layers x (qkv 2048x6144, out 2048x2048, "
                               "fc1 2048x8192, fc2 8192x2048) + lm_head 2048x51200 (BASELINE config 1 shapes "
                               "over the model's 24 layers)",
                   "bytes_per_step": step_bytes, "launches_per_step": launches_per_step,
                   "l2": "inputs larger than L2: 738 MB of packed weights per step vs 126 MB L2",
                   "parallelism": f"lm_head column-shard x{world} + NCCL all-gather; layers replicated"
                   if world > 1 else "single GPU", "seed": SEED, "prng": "SplitMix64 + Box-Muller (device)"},
        "roofline": {"bound": "hbm", "kernel": "gemv_q_stream", "launches_per_step": launches_per_step,
                     "achieved": round(value, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(value / peaks["hbm_gbs"], 4), "traffic": None,
                     "avg_launch_us": round(ms * 1e3 / launches_per_step, 3),
                     "bytes_per_launch_avg": step_bytes // launches_per_step, "peak_source": peaks["source"],
                     "basis": "every launch in the timed region is gemv_q_stream, back to back: average "
                              "algorithmic bytes per launch / average launch duration (CUDA events)"},
        "lm_head_launch": {"gbs": round(achieved, 1), "frac": round(achieved / peaks["hbm_gbs"], 4),
                           "bytes": head_bytes, "ms": round(head_ms, 5),
                           "basis": "marker events captured around the lm_head launch inside the graph",
                           "dram_traffic_bytes": 59059360 if world == 1 else None,
                           "dram_traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of this launch, "
                                                  "profiles/gemv_q_stream_q4_0_lm_head_2048x51200.md"},
        "e2e": e2e,
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
    }
    if prefill:
        line["prefill"] = prefill
    if secondary:
        line.update(secondary)
    if not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_baseline(args.cpu_budget)
    return line


def run_e2e(args, dev, mg, layers, xh, Wh, yh, n_head, K_h, step_bytes, world, dist, gather_logits, torch,
            stream, y_full_buf=None) -> dict:
    """The step through the public C ABI, from pinned host memory to pinned host memory, the way
    an engine drives it: the step's 97 activation vectors live in one device arena (views from
    mgpu_buf_view), so one mgpu_buf_write_async moves them all; the 97 mgpu_gemv_q dispatches
    are captured once with mgpu_capture_begin/end and replayed with mgpu_graph_launch; one
    mgpu_buf_read_async returns every layer output.  The logits: on one GPU they are in the same
    arena; on N GPUs each rank's shard is all-gathered (NCCL over NVLink) and the full logits
    are read back with a second mgpu_buf_read_async.  Device time of the whole loop, copies
    included, by CUDA events on the stream."""
    L = mg.lib()
    shapes = [(K, N, W) for mats in layers for (_, K, N, W, _, _) in mats] + [(K_h, n_head, Wh)]
    h2d = sum(K * 4 for K, _, _ in shapes)
    y_shapes = shapes if world == 1 else shapes[:-1]  # N>1: the logit shard goes to yh, then all-gathered
    y_bytes = sum(N * 4 for _, N, _ in y_shapes)
    logit_bytes = 0 if world == 1 else HEAD[2] * 4
    d2h = y_bytes + logit_bytes
    x_arena = dev.create_buffer(h2d, None, mg.F32)
    y_arena = dev.create_buffer(y_bytes, None, mg.F32)
    xv, yv = [], []
    xo = yo = 0
    for K, N, _ in shapes:
        xv.append(x_arena.view(xo, K * 4))
        xo += K * 4
    for _, N, _ in y_shapes:
        yv.append(y_arena.view(yo, N * 4))
        yo += N * 4
    if world > 1:
        yv.append(yh)
    hx = L.mgpu_host_alloc(h2d)
    hy = L.mgpu_host_alloc(d2h)
    try:
        host_x = np.ctypeslib.as_array((np.ctypeslib.ctypes.c_float * (h2d // 4)).from_address(hx))
        host_x[:] = np.random.default_rng(SEED).standard_normal(h2d // 4).astype(np.float32)

        def enqueue():
            for (K, N, W), x, y in zip(shapes, xv, yv):
                mg.gemv_q(dev, x, W, y, N, K, mg.Q4_0)

        enqueue()  # eager pass: validates arguments outside the capture
        dev.finish()
        dev.capture_begin()
        enqueue()
        graph = dev.capture_end()

        def one():
            mg._check(L.mgpu_buf_write_async(x_arena.h, 0, hx, h2d), "buf_write_async")
            graph.launch()
            mg._check(L.mgpu_buf_read_async(y_arena.h, 0, hy, y_bytes), "buf_read_async")
            if world > 1:
                gather_logits()
                mg._check(L.mgpu_buf_read_async(y_full_buf.h, 0, hy + y_bytes, logit_bytes), "buf_read_async")

        steps = max(3, min(args.steps, 2000))
        for _ in range(3):
            one()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            one()
        e1.record(stream)
        torch.cuda.synchronize()
        del graph
        ms = e0.elapsed_time(e1) / steps
        if world > 1:
            t = torch.tensor([ms], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t[0])
        return {"value": round(step_bytes / (ms * 1e-3) / 1e9, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(ms, 5), "steps": steps,
                "api": "mgpu_buf_write_async (all 97 inputs, one pinned buffer) + mgpu_graph_launch of the "
                       "captured 97 mgpu_gemv_q + mgpu_buf_read_async (all outputs"
                       + ("" if world == 1 else "; logits after an NCCL all-gather") + ")"}
    finally:
        L.mgpu_host_free(hx)
        L.mgpu_host_free(hy)


def run_prefill(dev, mg, torch, stream, peaks) -> dict:
    """tcgen05 GEMM on the Phi-1.5 prefill shapes: M=761, bf16 A, Q8_0 W (dequantised to bf16
    tiles inside the kernel), fp32 accumulate, bf16 C.  Rotates enough weight copies per shape
    that each pass over them is about 2x the L2.
    The kernels are timed as a captured graph of one launch per copy (at least 40), which is
    what an engine replaying its prefill graph sees; `eager_tflops` is the same loop dispatched
    call by call from Python, whose ~8 us of host time per call hides part of the kernel time."""
    out = {}
    tot_flop, tot_ms = 0.0, 0.0
    tmp_el = max(K * N for _, K, N in PREFILL_SHAPES)
    tmp = dev.empty(tmp_el, mg.F32)
    for M, K, N in PREFILL_SHAPES:
        wbytes = N * (K // 32) * 34
        ncopy = max(4, -(-256_000_000 // wbytes))
        iters = max(40, ncopy)
        A = dev.empty(M * K, mg.BF16)
        dev.fill_normal(A, M * K, SEED + K, 1.0)
        Ws = []
        for c in range(ncopy):
            w = dev.create_buffer(wbytes, None, mg.Q8_0, mg.LAYOUT_NK, N, K)
            dev.fill_normal(tmp, N * K, SEED + N + 17 * c, 0.02)
            dev.quantize(tmp, w, N * K, mg.Q8_0)
            Ws.append(w)
        C = dev.empty(M * N, mg.BF16)
        for w in Ws:
            mg.gemm_q(dev, A, w, C, M, N, K, mg.Q8_0)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(iters):
            mg.gemm_q(dev, A, Ws[i % ncopy], C, M, N, K, mg.Q8_0)
        e1.record(stream)
        torch.cuda.synchronize()
        ms_eager = e0.elapsed_time(e1) / iters
        dev.capture_begin()
        for i in range(iters):
            mg.gemm_q(dev, A, Ws[i % ncopy], C, M, N, K, mg.Q8_0)
        graph = dev.capture_end()
        for _ in range(3):
            graph.launch()
        torch.cuda.synchronize()
        reps = 5
        e0.record(stream)
        for _ in range(reps):
            graph.launch()
        e1.record(stream)
        torch.cuda.synchronize()
        del graph
        ms = e0.elapsed_time(e1) / (reps * iters)
        flop = 2.0 * M * K * N
        out[f"{K}x{N}"] = {"tflops": round(flop / (ms * 1e-3) / 1e12, 1), "us": round(ms * 1e3, 2),
                           "eager_tflops": round(flop / (ms_eager * 1e-3) / 1e12, 1), "weight_copies": ncopy}
        del Ws, A, C
        tot_flop += flop
        tot_ms += ms
    agg = tot_flop / (tot_ms * 1e-3) / 1e12
    return {"unit": "TFLOP/s", "M": 761, "weights": "Q8_0", "activations": "bf16", "shapes": out,
            "aggregate_tflops": round(agg, 1), "frac_of_peak": round(agg / peaks["bf16_tflops"], 4),
            "peak": peaks["bf16_tflops"], "peak_source": peaks["source"],
            "timing": "CUDA events around 5 replays of a captured graph of one launch per weight copy; "
                      "copies rotated so each pass reads ~256 MB of packed weights (2x L2)"}


def _guarded(fn, *args) -> dict:
    """Run a secondary measurement; a failure is reported in its place instead of losing the
    headline line."""
    try:
        return fn(*args)
    except Exception as e:  # noqa: BLE001
        return {"error": f"{type(e).__name__}: {e}"}


def run_fused_epilogues(dev, mg, torch, stream, peaks) -> dict:
    """The fused GEMM epilogues on the Phi-1.5 prefill MLP shapes (M=761, bf16 A, Q8_0 W, bf16
    C), each timed against the plain GEMM of the same shape: fc1 2048x8192 with bias + GELU,
    the SiLU-gated MLP's gate GEMM (silu(A.W^T) * up), and fc2 8192x2048 with the residual added
    in place.  Weight copies rotate through ~256 MB per pass (2x L2), one launch per copy in a
    captured graph.  `unfused_floor_us` = plain GEMM time + the HBM time of the elementwise
    passes the fusion removes (the reference's separate activation / multiply / add kernels at
    the measured copy bandwidth, launch cost not counted): a lower bound on the unfused chain."""
    M = 761
    out = {}
    tmp = dev.empty(8192 * 2048, mg.F32)
    for name, K, N, variant, extra in (("fc1_bias_gelu", 2048, 8192, "gelu", 2),
                                       ("gate_silu_mul_up", 2048, 8192, "silu_gate", 3),
                                       ("fc2_residual_in_place", 8192, 2048, "residual", 3)):
        wbytes = N * (K // 32) * 34
        ncopy = max(4, -(-256_000_000 // wbytes))
        A = dev.empty(M * K, mg.BF16)
        dev.fill_normal(A, M * K, SEED + 3 * K, 1.0)
        Ws = []
        for c in range(ncopy):
            w = dev.create_buffer(wbytes, None, mg.Q8_0, mg.LAYOUT_NK, N, K)
            dev.fill_normal(tmp, N * K, SEED + 5 * N + 13 * c, 0.02)
            dev.quantize(tmp, w, N * K, mg.Q8_0)
            Ws.append(w)
        C = dev.empty(M * N, mg.BF16)
        R = dev.empty(M * N, mg.BF16)
        dev.fill_normal(R, M * N, SEED + 7, 1.0)
        bias = dev.empty(N, mg.F32)
        dev.fill_normal(bias, N, SEED + 9, 0.5)

        def plain():
            for w in Ws:
                mg.gemm_q(dev, A, w, C, M, N, K, mg.Q8_0)

        def fused():
            for w in Ws:
                if variant == "gelu":
                    mg.gemm_fused(dev, A, w, C, M, N, K, bias, mg.ACT_GELU, None)
                elif variant == "silu_gate":
                    mg.gemm_silu_gate(dev, A, w, R, C, M, N, K)
                else:
                    mg.gemm_fused(dev, A, w, R, M, N, K, None, mg.ACT_NONE, R)

        us_plain = time_graph(dev, torch, stream, plain, reps=5) * 1e3 / ncopy
        us_fused = time_graph(dev, torch, stream, fused, reps=5) * 1e3 / ncopy
        saved = extra * M * N * 2
        floor = us_plain + saved / (peaks["hbm_gbs"] * 1e3)
        out[name] = {"K": K, "N": N, "plain_us": round(us_plain, 2), "fused_us": round(us_fused, 2),
                     "epilogue_overhead": round(us_fused / us_plain - 1.0, 4),
                     "hbm_bytes_saved": saved, "unfused_floor_us": round(floor, 2),
                     "speedup_vs_unfused_floor": round(floor / us_fused, 3)}
        del Ws, A, C, R
    return {"M": M, "weights": "Q8_0", "activations": "bf16", "out": "bf16", "shapes": out,
            "timing": "CUDA events around 5 replays of a captured graph of one launch per weight copy"}


def time_graph(dev, torch, stream, enqueue, reps: int, flush=None) -> float:
    """Capture enqueue() once as a graph through the library's capture API, replay it twice
    untimed, then return the mean device time (ms) of `reps` replays, each bracketed by its
    own CUDA events; `flush` (an L2-sized write) runs before each replay, outside the events."""
    enqueue()  # eager pass: validates arguments and sizes the workspace outside the capture
    dev.finish()
    dev.capture_begin()
    enqueue()
    graph = dev.capture_end()
    for _ in range(2):
        graph.launch()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for e0, e1 in evs:
        if flush is not None:
            flush()
        e0.record(stream)
        graph.launch()
        e1.record(stream)
    torch.cuda.synchronize()
    del graph
    return sum(e0.elapsed_time(e1) for e0, e1 in evs) / reps


def run_fp32_gemv(dev, mg, torch, stream, peaks) -> dict:
    """fp32 GEMV M=1, K=2048, N=8192, x and W [K][N] row-major ~U(-1,1)
    (the reference orientation), through dispatch_gemv.  Four weight copies (268 MB, > 2x L2)
    rotate, one launch each per replay."""
    K, N, copies = 2048, 8192, 4
    Ws = []
    for c in range(copies):
        w = dev.create_buffer(K * N * 4, None, mg.F32, mg.LAYOUT_KN, K, N)
        dev.fill_uniform(w, K * N, SEED + 300 + c)
        Ws.append(w)
    x = dev.empty(K, mg.F32)
    dev.fill_uniform(x, K, SEED + 301)
    y = dev.empty(N, mg.F32)

    def enqueue():
        for w in Ws:
            mg.dispatch_gemv(dev, None, x, w, y, N, K)

    ms = time_graph(dev, torch, stream, enqueue, 20) / copies
    nbytes = 4 * K * N + 4 * K + 4 * N
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"shape": f"{K}x{N}", "gbs": round(gbs, 1), "frac": round(gbs / peaks["hbm_gbs"], 4), "us": round(ms * 1e3, 2),
            "bytes": nbytes, "basis": "4 weight copies of 67 MB rotated; algorithmic bytes 4KN+4K+4N per launch"}


SIGLIP_LAYER = [(1152, 3456), (1152, 1152), (1152, 4304), (4304, 1152)]  # (K, N) per image token
SIGLIP_PROJ = [(2304, 8192), (8192, 2048)]


def run_siglip(dev, mg, torch, stream, peaks, batches=(1, 8, 64), world=1, dist=None) -> dict:
    """SigLIP encoder GEMMs at M = 729 * B with fp16 A ~N(0,1) and fp16
    weights ~N(0,0.02) in GGUF [N][K] order: one encoder layer (qkv, out, fc1, fc2) plus the
    projection MLP (2304->8192->2048), fp32 accumulate, fp16 C.  Each replay of the captured
    sequence follows a 256 MB write that evicts L2.  On N GPUs the images are batch-sharded
    (B/N per GPU, weights replicated, no exchange); the time is the maximum over ranks and the
    TFLOP/s are the whole batch's."""
    flush_buf = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")
    shapes = SIGLIP_LAYER + SIGLIP_PROJ
    tmp = dev.empty(max(K * N for K, N in shapes), mg.F32)
    Ws = []
    for i, (K, N) in enumerate(shapes):
        w = dev.create_buffer(N * K * 2, None, mg.F16, mg.LAYOUT_NK, N, K)
        dev.fill_normal(tmp, N * K, SEED + 400 + i, 0.02)
        dev.convert(tmp, w, N * K)
        Ws.append(w)
    del tmp
    out = {}
    for B in batches:
        if B % world:
            continue
        M = 729 * (B // world)
        A = dev.empty(M * max(K for K, _ in shapes), mg.F16)
        dev.fill_normal(A, M * max(K for K, _ in shapes), SEED + 500 + B, 1.0)
        C = dev.empty(M * max(N for _, N in shapes), mg.F16)

        def enqueue():
            for (K, N), w in zip(shapes, Ws):
                mg.gemm(dev, A, w, C, M, N, K)

        ms = time_graph(dev, torch, stream, enqueue, 5 if B >= 64 else 20, flush=lambda: flush_buf.zero_())
        if world > 1:
            t = torch.tensor([ms], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t[0])
        flop = sum(2.0 * M * K * N for K, N in shapes) * world
        tf = flop / (ms * 1e-3) / 1e12
        out[f"B{B}"] = {"M_per_gpu": M, "tflops": round(tf, 1), "frac": round(tf / (peaks["bf16_tflops"] * world), 4),
                        "ms": round(ms, 4), "gflop": round(flop / 1e9, 1)}
        del A, C
    return {"unit": "TFLOP/s", "dtype": "f16", "gemms": "layer qkv/out/fc1/fc2 + projection 2304x8192, 8192x2048",
            "peak": peaks["bf16_tflops"], "peak_source": peaks["source"], "batches": out,
            "parallelism": "single GPU" if world == 1 else f"batch-shard x{world} (B/{world} images per GPU)"}


def run_batched_decode(dev, mg, torch, stream, peaks, layers, Wh, K_h, n_head, seqs=(8, 32, 128), world=1,
                       dist=None) -> dict:
    """S concurrent decode sequences, i.e. GEMMs with M = S over the 24
    layers' Q4_0 weights (the same 738 MB as the GEMV sweep, > 5x L2) plus the lm_head; bf16
    activations ~N(0,1), bf16 outputs.  One replay = one decode step of all S sequences.
    On N GPUs the sequences are sharded for the layers (S/N per GPU, weights replicated); the
    hidden states are all-gathered and each GPU applies its column shard of the lm_head (Wh,
    51200/N rows) to all S, then the logit shards are all-gathered (NCCL).  The time is the
    maximum over ranks."""
    out = {}
    layer_bytes = sum(w.nbytes for mats in layers for (_, _, _, w, _, _) in mats)
    maxk = max(K for mats in layers for (_, K, _, _, _, _) in mats)
    maxn = max(N for mats in layers for (_, _, N, _, _, _) in mats)
    for S in seqs:
        if S % world:
            continue
        Sl = S // world
        A = dev.empty(Sl * maxk, mg.BF16)
        dev.fill_normal(A, Sl * maxk, SEED + 600 + S, 1.0)
        C = dev.empty(Sl * maxn, mg.BF16)
        hid_t = torch.empty(S * K_h, dtype=torch.bfloat16, device="cuda")
        hid = dev.wrap(hid_t.data_ptr(), S * K_h * 2, mg.BF16)
        hid_local = hid_t[:Sl * K_h] if world == 1 else torch.empty(Sl * K_h, dtype=torch.bfloat16, device="cuda")
        logit_t = torch.empty(S * n_head, dtype=torch.bfloat16, device="cuda")
        logits = dev.wrap(logit_t.data_ptr(), S * n_head * 2, mg.BF16)
        gathered = torch.empty(world * S * n_head, dtype=torch.bfloat16, device="cuda") if world > 1 else None

        def layers_enqueue():
            for mats in layers:
                for _, K, N, W, _, _ in mats:
                    mg.gemm_q(dev, A, W, C, Sl, N, K, mg.Q4_0)

        def head_enqueue():
            mg.gemm_q(dev, hid, Wh, logits, S, n_head, K_h, mg.Q4_0)

        if world == 1:
            def enqueue():
                layers_enqueue()
                head_enqueue()

            ms = time_graph(dev, torch, stream, enqueue, 10)
        else:
            # layers as one captured graph, the exchanges and the head between replays
            layers_enqueue()
            head_enqueue()
            dev.finish()
            dev.capture_begin()
            layers_enqueue()
            g_layers = dev.capture_end()

            def step():
                g_layers.launch()
                dist.all_gather_into_tensor(hid_t, hid_local)
                head_enqueue()
                dist.all_gather_into_tensor(gathered, logit_t)

            for _ in range(2):
                step()
            torch.cuda.synchronize()
            dist.barrier()
            reps = 10
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                step()
            e1.record(stream)
            torch.cuda.synchronize()
            del g_layers
            ms = e0.elapsed_time(e1) / reps
            t = torch.tensor([ms], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t[0])
        act = sum(2 * S * (K + N) for mats in layers for (_, K, N, _, _, _) in mats) + 2 * S * (K_h + n_head * world)
        flop = sum(2.0 * S * K * N for mats in layers for (_, K, N, _, _, _) in mats) + 2.0 * S * K_h * n_head * world
        # bytes every GPU streams per step: all layer weights (replicated) and its lm_head shard
        wbytes = (layer_bytes + Wh.nbytes) * world
        gbs = (wbytes + act) / (ms * 1e-3) / 1e9
        tf = flop / (ms * 1e-3) / 1e12
        out[f"S{S}"] = {"ms_per_step": round(ms, 4), "gbs": round(gbs, 1),
                        "hbm_frac": round(gbs / (peaks["hbm_gbs"] * world), 4),
                        "tflops": round(tf, 1), "tensor_frac": round(tf / (peaks["bf16_tflops"] * world), 4),
                        "launches": 4 * len(layers) + 1}
        del A, C
    return {"weights": "Q4_0", "activations": "bf16", "layers": len(layers), "steps": out,
            "parallelism": "single GPU" if world == 1 else
            f"sequences x{world} for the layers, lm_head column-shard x{world}, NCCL all-gathers",
            "basis": "roofline = min(HBM x AI, tensor peak); weights stream from HBM every step"}


# --------------------------------------------------------------------------------------
# reference arm: the reference's quantised path as its CPU restatement (the reference has no
# Q4_0 kernel of its own and no runnable OpenCL here), on the host cores
# --------------------------------------------------------------------------------------
def run_reference(args, rank: int, world: int) -> dict | None:
    if rank != 0:
        return None
    import oracle as O
    b = cpu_baseline(args.cpu_budget)
    # one bounded step per --steps, timed individually
    return {"metric": METRIC, "value": b["value"], "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "impl": "reference", "data": "synthetic (seeded, host)",
            "config": {"workload": "Q4_0 decode GEMV sweep (one layer + lm_head sample), M=1, host cores"},
            "cpu_baseline": {"value": b["value"], "unit": "GB/s", "cores": b["cores"], "kind": "port",
                             "sample": b["sample"]},
            "e2e": {"value": b["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "threads": O.max_threads()}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-budget", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the fp32 GEMV, batched-decode and SigLIP sections")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus if args.gpus == 1 else 1)))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank, world)
    else:
        line = run_ours(args, rank, world, local_rank)
    if line is not None and rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
