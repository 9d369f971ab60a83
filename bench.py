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

With --gpus N (launched by torchrun, one process per GPU, NCCL), as the path partitions: N
concurrent sequences, one per GPU, each GPU running its sequence's token through the 24 layers
(weights replicated, no exchange), then the lm_head column-sharded: the hidden states are
all-gathered (8 KB per GPU), each GPU applies its 51200/N rows to all N sequences (skinny GEMM,
M = N), and an all-to-all brings each sequence's per-shard (index, value) argmax pairs to its
GPU, which combines them into the token on the device.  Per-GPU work is fixed ("weak"
scaling); value counts N x the layer bytes + the lm_head once; each rank's time is measured on
its device and the max over ranks is reported.  The secondary paths shard too: SigLIP by
images, batched decode by sequences (lm_head column-sharded), prefill fc1 by columns.
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
DECODE_WORKLOAD = ("Q4_0 decode step, M=1: 24 layers x (qkv 2048x6144, out 2048x2048, fc1 2048x8192, fc2 8192x2048) "
                   "+ lm_head 2048x51200, each GEMV reading the previous one's output (BASELINE config 1 shapes over "
                   "the model's 24 layers)")
DECODE_WORKLOAD_MULTI = ("Q4_0 decode step of {n} concurrent sequences on {n} GPUs: per GPU one sequence's token "
                         "through the 24 layers (M=1 GEMVs, the same shapes as on one GPU); the 2048x51200 lm_head "
                         "column-sharded, each GPU applying its 51200/{n} rows to all {n} sequences")


def measured_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def driver_version() -> str | None:
    """The NVIDIA driver the box runs (the dependent-launch latency of the decode chain moved
    with it between driver builds), read with nvidia-smi."""
    try:
        out = subprocess.run(["nvidia-smi", "--query-gpu=driver_version", "--format=csv,noheader"],
                             capture_output=True, text=True, timeout=20).stdout.split()
        return out[0] if out else None
    except (OSError, subprocess.SubprocessError):
        return None


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
def qbytes(qt: int, K: int, N: int) -> int:
    """Algorithmic bytes of one quantised GEMV: packed weights + fp32 x + fp32 y."""
    return N * (K // 32) * (18 if qt == 2 else 34) + 4 * K + 4 * N


STEP_BYTES_Q4 = sum(qbytes(2, K, N) for _, K, N in LAYER_SHAPES) * LAYERS + qbytes(2, HEAD[1], HEAD[2])


def make_q(dev, mg, tmp, qt, K, N, seed):
    """Seeded ~N(0, 0.02) weights [N][K], quantised to qt on the device."""
    w = dev.create_buffer(N * (K // 32) * (18 if qt == mg.Q4_0 else 34), None, qt, mg.LAYOUT_NK, N, K)
    dev.fill_normal(tmp, N * K, seed, 0.02)
    dev.quantize(tmp, w, N * K, qt)
    return w


def head_seed(r: int) -> int:
    return SEED + 999_999 + r


def build_decode_step(dev, mg, tmp, qt, n_head, head_rank):
    """The decode step's GEMVs with the dataflow of a real decode token: the first link reads the
    token's hidden state x0, every later link reads (the first K values of) the previous link's
    output, and the lm_head (this rank's n_head rows) reads the last layer's output.
    Returns (links [(name, x, W, y, N, K)], x0)."""
    x0 = dev.empty(HEAD[1], mg.F32)
    dev.fill_normal(x0, HEAD[1], SEED + 5, 1.0)
    links, prev = [], None
    for l in range(LAYERS):
        for j, (name, K, N) in enumerate(LAYER_SHAPES):
            W = make_q(dev, mg, tmp, qt, K, N, SEED + 1000 * l + j + (0 if qt == mg.Q4_0 else 7_000_000))
            y = dev.empty(N, mg.F32)
            x = x0 if prev is None else prev.view(0, K * 4).set_format(mg.F32)
            links.append((name, x, W, y, N, K))
            prev = y
    Wh = make_q(dev, mg, tmp, qt, HEAD[1], n_head, head_seed(head_rank) + (0 if qt == mg.Q4_0 else 7_000_000))
    yh = dev.empty(n_head, mg.F32)
    links.append((HEAD[0], prev.view(0, HEAD[1] * 4).set_format(mg.F32), Wh, yh, n_head, HEAD[1]))
    return links, x0


def enqueue_links(dev, mg, qt, links):
    for _, x, W, y, N, K in links:
        mg.gemv_q(dev, x, W, y, N, K, qt)


def run_per_shape(dev, mg, torch, stream, peaks, qt, tmp) -> dict:
    """Each Phi-1.5 decode shape as its own chain of dependent GEMVs (every launch reads the
    previous launch's output, through PDL like the step), with enough links that a replay
    streams about 2x the L2 of packed weights; GB/s = links x algorithmic bytes / device time.
    fc2's input (K=8192) is a vector whose first 2048 values are the previous fc2's output."""
    out = {}
    bb = 18 if qt == mg.Q4_0 else 34
    for name, K, N in LAYER_SHAPES + [HEAD]:
        wbytes = N * (K // 32) * bb
        L = max(4, -(-256_000_000 // wbytes))
        links, prev = [], None
        xs = dev.empty(K, mg.F32)
        dev.fill_normal(xs, K, SEED + 77, 1.0)
        for i in range(L):
            W = make_q(dev, mg, tmp, qt, K, N, SEED + 50_000 + 31 * i + K + N)
            if K <= N:
                y = dev.empty(N, mg.F32)
                x = xs if prev is None else prev.view(0, K * 4).set_format(mg.F32)
                nxt = y
            else:
                # the next link's K-long input, whose first N values this link writes
                xn = dev.empty(K, mg.F32)
                dev.fill_normal(xn, K, SEED + 78 + i, 1.0)
                y = xn.view(0, N * 4).set_format(mg.F32)
                x = xs if prev is None else prev
                nxt = xn
            links.append((name, x, W, y, N, K))
            prev = nxt
        ms = time_graph(dev, torch, stream, lambda: enqueue_links(dev, mg, qt, links), 20)
        gbs = L * qbytes(qt, K, N) / (ms * 1e-3) / 1e9
        out[name] = {"K": K, "N": N, "links": L, "us_per_gemv": round(ms * 1e3 / L, 3), "gbs": round(gbs, 1),
                     "frac": round(gbs / peaks["hbm_gbs"], 4)}
        del links
    return out


def run_chain_kernel(dev, mg, torch, stream, peaks, qt, links, step_bytes) -> dict:
    """The same decode step through mgpu_gemv_chain (one cooperative launch for all links)."""
    chain = mg.GemvChain(dev, [(x, W, y, N, K) for _, x, W, y, N, K in links])
    try:
        ms = time_graph(dev, torch, stream, lambda: chain.run(), 20)
        ends = chain.run_timed()
        per = {}
        prev = 0.0
        for (name, _, _, _, N, K), t in zip(links, ends):
            d = per.setdefault(name, [0.0, 0])
            d[0] += t - prev
            d[1] += qbytes(qt, K, N)
            prev = t
        gbs = step_bytes / (ms * 1e-3) / 1e9
        return {"ms_per_step": round(ms, 5), "gbs": round(gbs, 1), "frac": round(gbs / peaks["hbm_gbs"], 4),
                "launches_per_step": 1,
                "per_shape_gbs": {k: round(v[1] / (v[0] * 1e-6) / 1e9, 1) for k, v in per.items()},
                "basis": "one cooperative launch over the step's links; per-shape figures from one run with "
                         "%globaltimer marks at each link's end (max over CTAs)"}
    finally:
        chain.destroy()


def run_decode_multi(args, dev, mg, torch, stream, dist, rank: int, world: int, qt, tmp) -> dict:
    """The decode step on N GPUs: N concurrent sequences, one per GPU, as the path partitions.
    - Layers: each rank runs its own sequence's token through the 24 layers (96 dependent
      gemv_q_stream launches, captured once as a graph); the weights are the same model on every
      rank (replicated), the activations its own; no exchange.
    - lm_head, column-sharded: each rank converts its final hidden state to bf16, the N of them
      are all-gathered over NVLink (mgpu_peer_allgather: stores into every peer's receive slots,
      4 KB per rank), and every rank applies its 51200/N rows of the lm_head to all N sequences
      (the skinny GEMM, M = N, fp32 logits).
    - Greedy token: mgpu_argmax_rows gives each sequence's {index, value} over this rank's
      columns; mgpu_peer_alltoall sends sequence s's pair to rank s (8 bytes per pair), and
      mgpu_argmax_combine turns the N pairs into that sequence's token on its own GPU.
    The whole step is one captured graph per rank (no collective-library call, no host round
    trip between the phases).  Whole-job bytes per step: N x the layer weights (each rank
    streams them for its sequence) + the lm_head once; the time is the max over ranks of the
    device time per step."""
    from mvlm_b200.shard import column_shard
    K_h, N_h = HEAD[1], HEAD[2]
    h0, h1 = column_shard(N_h, world, rank)
    n_head = h1 - h0
    # this rank's sequence: its own token input, the model's weights
    x0 = dev.empty(K_h, mg.F32)
    dev.fill_normal(x0, K_h, SEED + 5 + rank, 1.0)
    hid_t = torch.empty(K_h, dtype=torch.float32, device="cuda")
    hidden = dev.wrap(hid_t.data_ptr(), K_h * 4, mg.F32)
    links, prev = [], None
    for l in range(LAYERS):
        for j, (name, K, N) in enumerate(LAYER_SHAPES):
            W = make_q(dev, mg, tmp, qt, K, N, SEED + 1000 * l + j)
            last = l == LAYERS - 1 and j == len(LAYER_SHAPES) - 1
            y = hidden if last and N == K_h else dev.empty(N, mg.F32)
            x = x0 if prev is None else prev.view(0, K * 4).set_format(mg.F32)
            links.append((name, x, W, y, N, K))
            prev = y
    assert links[-1][3] is hidden
    Wh = make_q(dev, mg, tmp, qt, K_h, n_head, head_seed(rank))
    hb = dev.empty(K_h, mg.BF16)
    logits = dev.empty(world * n_head, mg.F32)
    pairs = dev.empty(2 * world, mg.F32)
    tok_t = torch.zeros(2, dtype=torch.int32, device="cuda")
    tok = dev.wrap(tok_t.data_ptr(), 8, mg.F32)
    # the two exchanges over peer memory (NVLink): receive slots mapped by every rank through
    # CUDA IPC, the 64-byte handles exchanged once with torch.distributed
    g_hid = mg.PeerGroup(dev, rank, world, K_h * 2)
    g_pair = mg.PeerGroup(dev, rank, world, 8)
    for grp in (g_hid, g_pair):
        handles = [None] * world
        dist.all_gather_object(handles, grp.handle())
        grp.connect(handles)
    Hall = g_hid.slots(mg.BF16)   # [world][K_h]: every sequence's hidden state
    recv = g_pair.slots(mg.F32)   # [world][2]: this sequence's pair from every rank

    # The lm_head shard over the N sequences: one GEMM with M = N (the skinny kernel), or N
    # M = 1 GEMVs (one per sequence, each reading its row of the gathered hidden states).  The
    # GEMV streams weights ~2x faster per byte than the skinny kernel but pays its fixed cost N
    # times; each rank times both once (its own graph replays, no collective) and keeps the
    # faster.
    head_rows = [(Hall.view(i * K_h * 2, K_h * 2).set_format(mg.BF16),
                  logits.view(i * n_head * 4, n_head * 4).set_format(mg.F32)) for i in range(world)]

    def head_gemm():
        mg.gemm_q(dev, Hall, Wh, logits, world, n_head, K_h, qt)

    def head_gemvs():
        for hx, ly in head_rows:
            mg.gemv_q(dev, hx, Wh, ly, n_head, K_h, qt)

    head_us = {name: time_graph(dev, torch, stream, fn, 20) * 1e3
               for name, fn in (("gemm_m_eq_n", head_gemm), ("gemv_per_sequence", head_gemvs))}
    head_kind = min(head_us, key=head_us.get)
    head = head_gemm if head_kind == "gemm_m_eq_n" else head_gemvs

    phases = [("layers_and_bf16", lambda: (enqueue_links(dev, mg, qt, links), dev.convert(hidden, hb, K_h))),
              ("hidden_all_gather", lambda: g_hid.allgather(hb, K_h * 2)),
              ("head_gemm_argmax", lambda: (head(), mg.argmax_rows(dev, logits, world, n_head, n_head, pairs))),
              ("pairs_all_to_all", lambda: g_pair.alltoall(pairs, 8)),
              ("combine", lambda: mg.argmax_combine(dev, recv, world, N_h, tok))]

    def step_enqueue():
        for _, fn in phases:
            fn()

    def capture(fn):
        # an eager pass first (every rank in the same order: the exchanges run in lockstep)
        fn()
        dev.finish()
        dev.capture_begin()
        fn()
        return dev.capture_end()

    g_step = capture(step_enqueue)

    def step():
        g_step.launch()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    sampler = ClockSampler(torch.cuda.current_device())
    sampler.start()
    time.sleep(0.3)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = ev0.elapsed_time(ev1) / args.steps
    t = torch.tensor([ms], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t[0])
    layer_bytes = sum(qbytes(qt, K, N) for _, K, N in LAYER_SHAPES) * LAYERS
    step_bytes = world * layer_bytes + qbytes(qt, K_h, N_h)

    # ---- where a step's time goes (untimed steps, each phase its own graph with CUDA events
    # between them, mean over the steps, max over ranks) ----
    g_phases = [capture(fn) for _, fn in phases]
    reps = 20
    marks = [[torch.cuda.Event(enable_timing=True) for _ in range(len(phases) + 1)] for _ in range(reps)]
    for ev in marks:
        ev[0].record(stream)
        for i, gph in enumerate(g_phases):
            gph.launch()
            ev[i + 1].record(stream)
    torch.cuda.synchronize()
    per = torch.tensor([sum(ev[i].elapsed_time(ev[i + 1]) for ev in marks) / reps * 1e3 for i in range(len(phases))],
                       dtype=torch.float64, device="cuda")
    dist.all_reduce(per, op=dist.ReduceOp.MAX)
    breakdown = {name: round(float(v), 2) for (name, _), v in zip(phases, per.tolist())}
    del g_phases

    # ---- parity, after the timed region: every sequence's full logits (the ranks' shards
    # gathered on rank 0) against the oracle's lm_head on the same bf16 hidden state, within the
    # fp32 tolerance; every rank's token against the argmax of its sequence's full row ----
    import oracle as O
    mine = torch.from_numpy(logits.read(np.float32)).cuda()
    pad = world * max(column_shard(N_h, world, r)[1] - column_shard(N_h, world, r)[0] for r in range(world))
    send = torch.zeros(pad, dtype=torch.float32, device="cuda")
    send[:mine.numel()] = mine
    got_all = [torch.zeros(pad, dtype=torch.float32, device="cuda") for _ in range(world)]
    dist.all_gather(got_all, send)
    toks = [torch.zeros(2, dtype=torch.int32, device="cuda") for _ in range(world)]
    dist.all_gather(toks, tok_t)
    parity = {"ok": True}
    if rank == 0:
        H = O.bf16_to_f32(Hall.read(np.uint16)).reshape(world, K_h)
        parts = []
        for r in range(world):
            a, b = column_shard(N_h, world, r)
            parts.append(make_q(dev, mg, tmp, qt, K_h, b - a, head_seed(r)).read(np.uint8))
        Wfull = np.concatenate(parts)
        full = np.zeros((world, N_h), np.float32)
        for r in range(world):
            a, b = column_shard(N_h, world, r)
            full[:, a:b] = got_all[r][:world * (b - a)].cpu().numpy().reshape(world, b - a)
        O.set_threads(len(os.sched_getaffinity(0)))
        ref = O.gemm_q(H.reshape(-1), Wfull, world, N_h, K_h, qt, threads=True).reshape(world, N_h)
        err = float(np.max(np.abs(full - ref)) / np.max(np.abs(ref)))
        tok_ok = all(int(toks[s_][0].item()) == int(np.argmax(full[s_])) for s_ in range(world))
        parity = {"tolerance": 1e-4, "logits_vs_oracle_rel_err": err, "tokens_are_row_argmax": tok_ok,
                  "sequences": world, "ok": bool(err <= 1e-4 and tok_ok)}

    # ---- e2e through the C ABI: each rank writes its token's hidden state from pinned host
    # memory and reads its 8-byte greedy result back ----
    L = mg.lib()
    h2d, d2h = K_h * 4, 8
    hx, hy = L.mgpu_host_alloc(h2d), L.mgpu_host_alloc(d2h)
    try:
        host_x = np.ctypeslib.as_array((ctypes_float() * (h2d // 4)).from_address(hx))
        host_x[:] = np.random.default_rng(SEED + rank).standard_normal(h2d // 4).astype(np.float32)

        # the copies from and to pinned memory captured with the step: one graph launch per token
        g_e2e = capture(lambda: (mg._check(L.mgpu_buf_write_async(x0.h, 0, hx, h2d), "buf_write_async"),
                                 step_enqueue(),
                                 mg._check(L.mgpu_buf_read_async(tok.h, 0, hy, d2h), "buf_read_async")))

        def one():
            g_e2e.launch()

        for _ in range(3):
            one()
        torch.cuda.synchronize()
        dist.barrier()
        e2e_steps = max(3, min(args.steps, 2000))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e2e_steps):
            one()
        e1.record(stream)
        torch.cuda.synchronize()
        ems = e0.elapsed_time(e1) / e2e_steps
        t = torch.tensor([ems], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ems = float(t[0])
        del g_e2e
    finally:
        L.mgpu_host_free(hx)
        L.mgpu_host_free(hy)
    del g_step
    e2e = {"value": round(step_bytes / (ems * 1e-3) / 1e9, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
           "d2h_bytes_per_step": d2h, "ms_per_step": round(ems, 5), "steps": e2e_steps,
           "api": "per rank, one mgpu_graph_launch per token of: mgpu_buf_write_async (its sequence's hidden state, "
                  "pinned), the 96 layer mgpu_gemv_q, mgpu_convert of the hidden state to bf16, mgpu_peer_allgather "
                  "(4 KB per GPU over NVLink), mgpu_gemm_q (lm_head shard, M = N), mgpu_argmax_rows, "
                  "mgpu_peer_alltoall (8 bytes per sequence and GPU), mgpu_argmax_combine, mgpu_buf_read_async (its "
                  "8-byte greedy result)"}
    g_hid.destroy()
    g_pair.destroy()
    return {"ms": ms, "step_bytes": step_bytes, "layer_bytes": layer_bytes, "n_head": n_head, "parity": parity,
            "e2e": e2e, "clocks": clocks,
            "launches_per_step": len(links) + 5 + (world if head_kind == "gemv_per_sequence" else 1),
            "links": links, "Wh": Wh, "breakdown_us": breakdown,
            "head": {"kind": head_kind, "us": {k: round(v, 2) for k, v in head_us.items()}}}


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
    qt = mg.Q4_0

    # ---------------- the decode step, weights generated and quantised on the device ----------------
    tmp = dev.empty(max(max(K * N for _, K, N in LAYER_SHAPES), HEAD[1] * HEAD[2]), mg.F32)
    K_h = HEAD[1]
    if world > 1:
        # N concurrent sequences, one per GPU, the lm_head column-sharded across the GPUs
        multi = run_decode_multi(args, dev, mg, torch, stream, dist, rank, world, qt, tmp)
        ms, step_bytes, parity, e2e, clocks = (multi["ms"], multi["step_bytes"], multi["parity"], multi["e2e"],
                                               multi["clocks"])
        links, Wh, n_head = multi["links"], multi["Wh"], multi["n_head"]
        launches_per_step = multi["launches_per_step"]
        secondary_multi = {"step_breakdown_us": multi["breakdown_us"], "lm_head_shard": multi["head"]}
    else:
        n_head = HEAD[2]
        links, x0 = build_decode_step(dev, mg, tmp, qt, n_head, 0)
        dev.finish()
        yh = links[-1][3]
        Wh = links[-1][2]
        step_bytes = sum(qbytes(qt, K, N) for _, K, N in LAYER_SHAPES) * LAYERS + qbytes(qt, K_h, HEAD[2])
        argbuf = dev.empty(2, mg.F32)

        def enqueue():
            enqueue_links(dev, mg, qt, links)

        enqueue()  # eager run first (validates arguments outside capture)
        dev.finish()
        dev.capture_begin()
        enqueue()
        graph = dev.capture_end()
        launches_per_step = len(links)

        for _ in range(args.warmup):
            graph.launch()
        torch.cuda.synchronize()
        sampler = ClockSampler(local_rank)
        sampler.start()
        time.sleep(0.3)
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for _ in range(args.steps):
            graph.launch()
        ev1.record(stream)
        torch.cuda.synchronize()
        clocks = sampler.stop()
        ms = ev0.elapsed_time(ev1) / args.steps
        del graph

        # ---------------- parity of the step's result ----------------
        parity = {"ok": None, "skipped": "--ncu"}
        e2e = None
        if not args.ncu:
            parity = check_decode_parity(mg, qt, links)
            # ---------------- e2e through the C ABI with host buffers ----------------
            e2e = run_e2e(args, dev, mg, torch, stream, qt, links, x0, argbuf, step_bytes)

    # ---------------- secondary measurements ----------------
    secondary = {} if world == 1 else dict(secondary_multi)
    if world == 1 and not args.no_secondary:
        per_launch_logits = yh.read(np.float32)
        secondary["chain_kernel"] = _guarded(run_chain_kernel, dev, mg, torch, stream, peaks, qt, links, step_bytes)
        secondary["chain_kernel"]["logits_equal_per_launch"] = bool(np.array_equal(yh.read(np.float32),
                                                                                  per_launch_logits))
        secondary["per_shape"] = run_per_shape(dev, mg, torch, stream, peaks, qt, tmp)
        secondary["q8_0_sweep"] = _guarded(run_q8_sweep, dev, mg, torch, stream, peaks, tmp)
    del tmp
    layers = [[(name, K, N, W, x, y) for name, x, W, y, N, K in links[4 * l:4 * l + 4]] for l in range(LAYERS)]
    prefill = None
    if not args.no_prefill:
        prefill = run_prefill(dev, mg, torch, stream, peaks, world, dist, rank)
    if not args.no_secondary:
        if world == 1:
            secondary.update({"fp32_gemv": run_fp32_gemv(dev, mg, torch, stream, peaks),
                              "batched_decode": run_batched_decode(dev, mg, torch, stream, peaks, layers, Wh, K_h,
                                                                   n_head),
                              # before SigLIP, whose seconds of dense MMAs can leave the clocks power-capped
                              "fused_epilogues": _guarded(run_fused_epilogues, dev, mg, torch, stream, peaks),
                              "siglip": run_siglip(dev, mg, torch, stream, peaks)})
        else:
            # every rank takes part (collectives); rank 0 reports
            secondary.update({"batched_decode": run_batched_decode(dev, mg, torch, stream, peaks, layers, Wh, K_h,
                                                                   n_head, world=world, dist=dist),
                              "siglip": run_siglip(dev, mg, torch, stream, peaks, batches=(8, 64), world=world,
                                                   dist=dist)})
    if "siglip" in secondary and "parity" in secondary["siglip"]:
        parity["siglip_rel_err"] = secondary["siglip"]["parity"]["rel_err"]
        parity["ok"] = parity["ok"] and secondary["siglip"]["parity"]["ok"]
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return None

    value = step_bytes / (ms * 1e-3) / 1e9
    # the roofline is per GPU: the bytes one GPU streams per step (its sequence's layers and, on N
    # GPUs, its lm_head shard) over the step's device time, against one GPU's HBM peak
    gpu_bytes = step_bytes if world == 1 else multi["layer_bytes"] + qbytes(qt, K_h, n_head)
    achieved = gpu_bytes / (ms * 1e-3) / 1e9
    traffic = profiled_traffic() if world == 1 else {}
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "pct_of_peak": round(100.0 * value / (peaks["hbm_gbs"] * world), 1),
        "data": "synthetic: weights ~N(0,0.02) seeded, quantised to GGUF Q4_0 on the device; x0 ~N(0,1) fp32",
        "config": {"workload": DECODE_WORKLOAD if world == 1 else DECODE_WORKLOAD_MULTI.format(n=world),
                   "bytes_per_step": step_bytes, "launches_per_step": launches_per_step,
                   "l2": "inputs larger than L2: 738 MB of packed weights per step vs 126 MB L2",
                   "parallelism": "single GPU" if world == 1 else
                   f"sequences x{world} (one per GPU, layer weights replicated); lm_head column-shard x{world} "
                   f"applied to all {world} sequences; all-gather of the bf16 hidden states (4 KB per GPU) and "
                   f"all-to-all of the greedy (index, value) pairs (8 bytes per sequence and GPU) over NVLink "
                   f"peer memory (mgpu_peer_allgather / mgpu_peer_alltoall), one graph per step",
                   "seed": SEED, "prng": "SplitMix64 + Box-Muller (device)"},
        "roofline": {"bound": "hbm", "kernel": "gemv_q_stream", "launches_per_step": len(links),
                     "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": traffic.get("bytes_per_step"),
                     "traffic_source": traffic.get("source"),
                     "avg_launch_us": round(ms * 1e3 / len(links), 3),
                     "bytes_per_launch_avg": gpu_bytes // len(links), "peak_source": peaks["source"],
                     "basis": "per GPU: every GEMV of the step is a gemv_q_stream launch, back to back under "
                              "programmatic dependent launch: algorithmic bytes one GPU streams per step / device "
                              "time of the step (CUDA events)" + ("" if world == 1 else
                              "; on N GPUs the step also holds the lm_head shard's skinny GEMM and the two NCCL "
                              "exchanges")},
        "parity": parity, "parity_ok": parity["ok"],
        "e2e": e2e,
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
        "driver": driver_version(),
    }
    if prefill:
        line["prefill"] = prefill
    if secondary:
        line.update(secondary)
    if not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_baseline(args.cpu_budget)
    return line


def check_decode_parity(mg, qt, links) -> dict:
    """The step's logits against the CPU oracle's lm_head (dequantise + fp32 dot, the
    reference's quantised path) applied to the same final hidden state, after the timed region,
    within the fp32 tolerance 1e-4 of the output's max-norm."""
    import oracle as O
    yh, hidden = links[-1][3], links[-2][3]
    K_h, N_h = HEAD[1], HEAD[2]
    h = hidden.read(np.float32)[:K_h].copy()
    got = yh.read(np.float32)
    O.set_threads(len(os.sched_getaffinity(0)))
    ref = O.gemm_q(h, links[-1][2].read(np.uint8), 1, N_h, K_h, qt, threads=True)
    err = float(np.max(np.abs(got - ref)) / np.max(np.abs(ref)))
    return {"tolerance": 1e-4, "logits_vs_oracle_rel_err": err, "ok": bool(err <= 1e-4)}


def run_e2e(args, dev, mg, torch, stream, qt, links, x0, argbuf, step_bytes) -> dict:
    """The step through the public C ABI, from pinned host memory to pinned host memory, as an
    engine drives a decode token: mgpu_buf_write_async of the token's hidden state (8 KB), the
    97 mgpu_gemv_q, the device argmax of the logits (mgpu_argmax) and one mgpu_buf_read_async of
    the 8-byte greedy result, all captured once (the copies from and to pinned memory become
    graph nodes) and replayed with mgpu_graph_launch, one launch per token.  Device time of the
    whole loop, copies included, by CUDA events on the stream."""
    L = mg.lib()
    yh = links[-1][3]
    n_head = links[-1][4]
    h2d, d2h = HEAD[1] * 4, 8
    hx = L.mgpu_host_alloc(h2d)
    hy = L.mgpu_host_alloc(d2h)
    try:
        host_x = np.ctypeslib.as_array((ctypes_float() * (h2d // 4)).from_address(hx))
        host_x[:] = np.random.default_rng(SEED).standard_normal(h2d // 4).astype(np.float32)

        def enqueue():
            mg._check(L.mgpu_buf_write_async(x0.h, 0, hx, h2d), "buf_write_async")
            enqueue_links(dev, mg, qt, links)
            mg.argmax(dev, yh, n_head, argbuf)
            mg._check(L.mgpu_buf_read_async(argbuf.h, 0, hy, d2h), "buf_read_async")

        enqueue()  # eager pass: validates arguments outside the capture
        dev.finish()
        dev.capture_begin()
        enqueue()
        graph = dev.capture_end()

        def one():
            graph.launch()

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
        return {"value": round(step_bytes / (ms * 1e-3) / 1e9, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(ms, 5), "steps": steps,
                "api": "one mgpu_graph_launch per token of the captured mgpu_buf_write_async (the token's hidden "
                       "state, pinned) + 97 mgpu_gemv_q + mgpu_argmax + mgpu_buf_read_async (the 8-byte greedy "
                       "result, pinned)"}
    finally:
        L.mgpu_host_free(hx)
        L.mgpu_host_free(hy)


def ctypes_float():
    import ctypes
    return ctypes.c_float


def run_q8_sweep(dev, mg, torch, stream, peaks, tmp) -> dict:
    """BASELINE config 1's Q8_0 half: the same decode step (24 layers + lm_head, each GEMV reading
    the previous output) with the weights quantised to Q8_0, then each shape's dependent chain."""
    qt = mg.Q8_0
    links, _ = build_decode_step(dev, mg, tmp, qt, HEAD[2], 0)
    step_bytes = sum(qbytes(qt, K, N) for _, K, N in LAYER_SHAPES) * LAYERS + qbytes(qt, HEAD[1], HEAD[2])
    ms = time_graph(dev, torch, stream, lambda: enqueue_links(dev, mg, qt, links), 50)
    del links
    gbs = step_bytes / (ms * 1e-3) / 1e9
    return {"bytes_per_step": step_bytes, "ms_per_step": round(ms, 5), "gbs": round(gbs, 1),
            "frac": round(gbs / peaks["hbm_gbs"], 4),
            "per_shape": run_per_shape(dev, mg, torch, stream, peaks, qt, tmp)}


def profiled_traffic() -> dict:
    """DRAM bytes per step of the decode step's kernels, from the committed ncu summary of the
    same workload (profiles/gemv_q_stream_decode_step_dram.md: the `bytes per step` row)."""
    path = os.path.join(ROOT, "profiles", "gemv_q_stream_decode_step_dram.md")
    if not os.path.exists(path):
        return {}
    with open(path) as f:
        for line in f:
            if line.startswith("| bytes per step"):
                cells = [c.strip() for c in line.strip().strip("|").split("|")]
                return {"bytes_per_step": int(cells[1].replace(",", "")), "source": os.path.relpath(path, ROOT)}
    return {}


def run_prefill(dev, mg, torch, stream, peaks, world=1, dist=None, rank=0) -> dict:
    """tcgen05 GEMM on the Phi-1.5 prefill shapes: M=761, bf16 A, Q8_0 W (dequantised to bf16
    tiles inside the kernel), fp32 accumulate, bf16 C.  Rotates enough weight copies per shape
    that each pass over them is about 2x the L2; the kernels are timed as a captured graph of
    one launch per copy (at least 40), replayed.
    On N GPUs fc1 (2048x8192) is column-sharded: each rank computes 8192/N output columns of
    every token and the shards are all-gathered with NCCL over NVLink into the [761][8192]
    activations (the gathered [rank][M][N/N] blocks are put in row order on the device); the
    other three GEMMs run whole on every rank (replicas).  Time = max over ranks; TFLOP/s count
    each GEMM's full 2MKN once."""
    import oracle as O
    from mvlm_b200.shard import column_shard
    out = {}
    tot_flop, tot_ms = 0.0, 0.0
    tmp = dev.empty(max(K * N for _, K, N in PREFILL_SHAPES), mg.F32)
    parity = {}
    for M, K, N in PREFILL_SHAPES:
        sharded = world > 1 and (K, N) == (2048, 8192)
        a, b = column_shard(N, world, rank) if sharded else (0, N)
        n_loc = b - a
        rb = (K // 32) * 34
        wbytes = N * rb
        ncopy = max(4, -(-256_000_000 // (n_loc * rb)))
        iters = max(40, ncopy)
        A = dev.empty(M * K, mg.BF16)
        dev.fill_normal(A, M * K, SEED + K, 1.0)
        Ws, Wfull = [], []
        for c in range(ncopy):
            w = dev.create_buffer(wbytes, None, mg.Q8_0, mg.LAYOUT_NK, N, K)
            dev.fill_normal(tmp, N * K, SEED + N + 17 * c, 0.02)
            dev.quantize(tmp, w, N * K, mg.Q8_0)
            Wfull.append(w)
            Ws.append(w.view(a * rb, n_loc * rb).set_format(mg.Q8_0, mg.LAYOUT_NK, n_loc, K) if sharded else w)
        C_t = torch.empty(M * n_loc, dtype=torch.bfloat16, device="cuda")
        C = dev.wrap(C_t.data_ptr(), M * n_loc * 2, mg.BF16)
        for w in Ws:  # eager pass first: validates the arguments outside the capture
            mg.gemm_q(dev, A, w, C, M, n_loc, K, mg.Q8_0)
        torch.cuda.synchronize()
        dev.capture_begin()
        for i in range(iters):
            mg.gemm_q(dev, A, Ws[i % ncopy], C, M, n_loc, K, mg.Q8_0)
        graph = dev.capture_end()
        if sharded:
            gath = torch.empty(world * M * n_loc, dtype=torch.bfloat16, device="cuda")
            full = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")

            def once():
                graph.launch()
                # every launch of the replay writes the same shard: one gather per replay, as a
                # layer's forward pays one
                dist.all_gather_into_tensor(gath, C_t)
                full.copy_(gath.view(world, M, n_loc).permute(1, 0, 2).reshape(M, N))
        else:
            def once():
                graph.launch()
        for _ in range(3):
            once()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        reps = 5
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            once()
        e1.record(stream)
        torch.cuda.synchronize()
        ms_all = e0.elapsed_time(e1) / reps
        if world > 1:
            t = torch.tensor([ms_all], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms_all = float(t[0])
        ms = ms_all / iters
        if sharded:
            # the gather's share: time the GEMM graph alone too, the difference is the exchange
            e0.record(stream)
            for _ in range(reps):
                graph.launch()
            e1.record(stream)
            torch.cuda.synchronize()
            g_ms = e0.elapsed_time(e1) / reps
            # and the two halves of the exchange on their own: the NCCL all-gather, the re-layout
            e0.record(stream)
            for _ in range(reps):
                dist.all_gather_into_tensor(gath, C_t)
            e1.record(stream)
            e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e2.record(stream)
            for _ in range(reps):
                full.copy_(gath.view(world, M, n_loc).permute(1, 0, 2).reshape(M, N))
            e3.record(stream)
            torch.cuda.synchronize()
            t = torch.tensor([g_ms, e0.elapsed_time(e1) / reps, e2.elapsed_time(e3) / reps], dtype=torch.float64,
                             device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            gemm_ms = float(t[0]) / iters
            gather_ms = ms_all - float(t[0])
            nccl_ms, relayout_ms = float(t[1]), float(t[2])
            ms = gemm_ms + gather_ms
        flop = 2.0 * M * K * N
        key = f"{K}x{N}"
        out[key] = {"tflops": round(flop / (ms * 1e-3) / 1e12, 1), "us": round(ms * 1e3, 2),
                    "weight_copies": ncopy}
        if sharded:
            out[key].update({"column_shard": f"{n_loc} of {N} columns per GPU", "gemm_us": round(gemm_ms * 1e3, 2),
                             "exchange_us": round(gather_ms * 1e3, 2), "nccl_all_gather_us": round(nccl_ms * 1e3, 2),
                             "relayout_us": round(relayout_ms * 1e3, 2),
                             "all_gather_bytes": world * M * n_loc * 2})
        if (K, N) == (2048, 8192) and rank == 0:
            # parity of the (gathered) fc1 output on a few tokens against the CPU oracle
            rows = [0, 1, 380, 760]
            got = (full.float().cpu().numpy() if sharded else
                   C_t.float().cpu().numpy().reshape(M, N))[rows]
            Ah = O.bf16_to_f32(A.read(np.uint16)).reshape(M, K)[rows]
            ref = O.gemm_q(np.ascontiguousarray(Ah), Wfull[(iters - 1) % ncopy].read(np.uint8), len(rows), N, K,
                           O.Q8_0, threads=True).reshape(len(rows), N)
            err = float(np.max(np.abs(got - ref)) / np.max(np.abs(ref)))
            parity = {"fc1_rows_checked": rows, "rel_err": err, "tolerance": 1e-2, "ok": err <= 1e-2}
        graph = None
        del Ws, Wfull, A, C, C_t
        tot_flop += flop
        tot_ms += ms
    agg = tot_flop / (tot_ms * 1e-3) / 1e12
    res = {"unit": "TFLOP/s", "M": 761, "weights": "Q8_0", "activations": "bf16", "n_gpus": world, "shapes": out,
           "aggregate_tflops": round(agg, 1), "frac_of_peak": round(agg / peaks["bf16_tflops"], 4),
           "peak": peaks["bf16_tflops"], "peak_source": peaks["source"],
           "parallelism": "single GPU" if world == 1 else
           f"fc1 column-shard x{world} + NCCL all-gather; qkv / out / fc2 replicated",
           "timing": "CUDA events around 5 replays of a captured graph of one launch per weight copy; "
                     "copies rotated so each pass reads ~256 MB of packed weights (2x L2)"}
    if parity:
        res["parity"] = parity
    return res


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
    parity = {}
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
        if B == max(batches):
            # parity: C holds the last GEMM (projection 8192 -> 2048) of this GPU's images; a few
            # of its rows against the CPU oracle, on every rank, worst error over the ranks
            import oracle as O
            K, N = shapes[-1]
            rows = [0, 1, M // 2, M - 1]
            Ah = O.f16_to_f32(A.read(np.uint16, M * K)).reshape(M, K)[rows]
            Cg = O.f16_to_f32(C.read(np.uint16, M * N)).reshape(M, N)[rows]
            ref = O.gemm_nk(np.ascontiguousarray(Ah), Ws[-1].read(np.uint16), mg.F16, len(rows), N, K).reshape(
                len(rows), N)
            err = float(np.max(np.abs(Cg - ref)) / np.max(np.abs(ref)))
            if world > 1:
                t = torch.tensor([err], dtype=torch.float64, device="cuda")
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                err = float(t[0])
            parity = {"batch": B, "rows_checked_per_gpu": rows, "gemm": f"{K}x{N}", "rel_err": err,
                      "tolerance": 1e-2, "ok": err <= 1e-2}
        del A, C
    res = {"unit": "TFLOP/s", "dtype": "f16", "gemms": "layer qkv/out/fc1/fc2 + projection 2304x8192, 8192x2048",
           "peak": peaks["bf16_tflops"], "peak_source": peaks["source"], "batches": out,
           "parallelism": "single GPU" if world == 1 else f"batch-shard x{world} (B/{world} images per GPU)"}
    if parity:
        res["parity"] = parity
    return res


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
def ncu_case_batched(args) -> dict:
    """Capture case for ncu: four back-to-back batched-decode GEMMs (S = 8 sequences against the
    qkv weights, Q4_0, bf16 activations and output), nothing else timed."""
    import torch

    import mvlm_b200 as mg
    dev = mg.Device(0)
    S, K, N = 8, 2048, 6144
    tmp = dev.empty(K * N, mg.F32)
    W = make_q(dev, mg, tmp, mg.Q4_0, K, N, SEED + 41)
    A = dev.empty(S * K, mg.BF16)
    dev.fill_normal(A, S * K, SEED + 42, 1.0)
    C = dev.empty(S * N, mg.BF16)
    for _ in range(4):
        mg.gemm_q(dev, A, W, C, S, N, K, mg.Q4_0)
    dev.finish()
    torch.cuda.synchronize()
    return {"ncu_case": args.ncu_case, "launches": 4, "S": S, "K": K, "N": N}


def run_reference(args, rank: int, world: int) -> dict | None:
    if rank != 0:
        return None
    import oracle as O
    b = cpu_baseline(args.cpu_budget)
    # one bounded step per --steps, timed individually
    return {"metric": METRIC, "value": b["value"], "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "impl": "reference", "data": "synthetic (seeded, host)",
            "config": {"workload": DECODE_WORKLOAD if world == 1 else DECODE_WORKLOAD_MULTI.format(n=world),
                       "bytes_per_step": STEP_BYTES_Q4 if world == 1 else
                       world * (STEP_BYTES_Q4 - qbytes(2, HEAD[1], HEAD[2])) + qbytes(2, HEAD[1], HEAD[2])},
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
    ap.add_argument("--ncu-case", choices=["decode", "batched_s8_qkv"], default="decode",
                    help="with --ncu: the decode step (default), or four launches of the batched-decode GEMM "
                         "(S=8, qkv 2048x6144, Q4_0, bf16) for a capture of that kernel")
    ap.add_argument("--ncu", action="store_true",
                    help="capture mode for ncu: only the decode step (3 timed steps), no e2e, parity or other "
                         "sections, so that a launch list or a capture holds the step's kernels alone")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.ncu:
        args.steps = min(args.steps, 3)
        args.no_secondary = args.no_prefill = args.no_cpu_baseline = True
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus if args.gpus == 1 else 1)))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank, world)
    elif args.ncu and args.ncu_case != "decode":
        line = ncu_case_batched(args)
    else:
        line = run_ours(args, rank, world, local_rank)
    if line is not None and rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
