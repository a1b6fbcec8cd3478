"""Benchmark of the attention hot path (prints ONE JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...   (N > 1)

Workload (Qwen3-32B layer): fused Q/K RMSNorm +
RoPE + KV-cache write followed by causal GQA prefill attention, S = 4096,
64 query / 8 KV heads, head_dim 128, f16, seeded N(0,1) inputs.  One step =
both kernels over one sequence.  value = attention FLOPs (4*D*Hq*S(S+1)/2)
per second of step time, whole job.  Multi-GPU: each rank runs its own
sequence (weak scaling; attention shards by sequence / KV head with no
collective).  Side measurements on rank 0 at N = 1: config 3's split-K
decode grid (HBM GB/s per cell) and config 1.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Attn decode HBM GB/s + prefill TFLOP/s (Qwen3-32B GQA)"
D = 128
HQ, HKV, S = 64, 8, 4096
EPS, THETA = 1e-6, 1.0e6
L2_FLUSH_BYTES = 256 << 20


class L2Flush:
    """Evicts L2 between timed steps: writes a 256 MB buffer (larger than the
    126 MB L2), then reads a second one so the dirty lines are written back
    before the timed region rather than inside it."""

    def __init__(self, device):
        import torch
        self.w = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)
        self.r = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)
        self.i = 0

    def __call__(self):
        self.i += 1
        self.w.fill_(float(self.i))
        self.sink = self.r.sum()
# DRAM bytes (read + write) of one prefill_kernel launch on this workload,
# taken from one ncu capture (dram__bytes_read.sum + dram__bytes_write.sum);
# bench.py cannot read DRAM counters itself, so the line labels it as such.
PREFILL_TRAFFIC_BYTES = 83_973_632 + 25_476_352


def prefill_flops(S_, hq=HQ, P=0):
    # causal, unmasked entries only: QK^T and PV, 2 flops per MAC each
    return 4.0 * D * hq * sum_visible(S_, P)


def sum_visible(S_, P=0):
    return S_ * P + S_ * (S_ + 1) / 2.0


def shard_kv_heads(hkv, world, rank):
    """KV heads [lo, hi) owned by `rank` when a layer is sharded by KV head
    (each rank also owns query heads [lo*G, hi*G)); no exchange is needed."""
    if hkv % world:
        raise ValueError(f"{hkv} KV heads do not split over {world} ranks")
    per = hkv // world
    return rank * per, (rank + 1) * per


def reduce_max(values, dist=None, device=None):
    """Max over ranks of a list of per-rank timings (ms)."""
    if dist is None:
        return list(values)
    import torch
    t = torch.tensor(values, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def job_tflops(flops_per_rank_step, steps, world, max_ms):
    """Whole-job throughput: every rank's work over the slowest rank's time."""
    return world * flops_per_rank_step * steps / (max_ms * 1e-3) / 1e12


def fused_bytes(S_, hq=HQ, hkv=HKV):
    return 2.0 * S_ * (hq + 2 * hkv) * D * 2


def peaks():
    p = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            m = json.load(f)
        p.update({k: m[k] for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained") if k in m})
        p["src"] = "measured"
    return p


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.index)], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.25)
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self):
        rows = []
        for line in (self.out or "").strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, x in enumerate(r) if x.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


def make_inputs(seed_base):
    from grout_b200 import synth
    q = synth.normal(seed_base + 1, S * HQ * D).reshape(S, HQ, D)
    k = synth.normal(seed_base + 2, S * HKV * D).reshape(S, HKV, D)
    v = synth.normal(seed_base + 3, S * HKV * D).reshape(S, HKV, D)
    qw = synth.norm_weight(seed_base + 4, D)
    kw = synth.norm_weight(seed_base + 5, D)
    return q, k, v, qw, kw


# ------------------------------------------------------------ CPU baseline
def cpu_baseline(rows_step=2):
    """The oracle (a C++ restatement of the reference's f32 CPU path) on a
    bounded sample of the same workload: the fused norm/RoPE/KV write over
    all 4096 tokens, and causal attention for every rows_step-th query row of
    all 64 heads.  TFLOP/s = attention FLOPs of the sampled rows / time of
    (sampled attention + fused write scaled to the same row fraction)."""
    import oracle
    oracle.set_num_threads(os.cpu_count() or 1)
    q, k, v, qw, kw = make_inputs(0)
    tab = oracle.rope_table(oracle.inv_freq(THETA, D), S)
    kc = np.zeros((HKV, S, D), np.float16)
    vc = np.zeros_like(kc)
    t0 = time.perf_counter()
    q_out = oracle.qk_norm_rope_kv_prefill(q, k, v, qw, kw, tab, kc, vc, 0, EPS)
    t_fused = time.perf_counter() - t0
    t0 = time.perf_counter()
    oracle.attn_prefill(q_out, kc, vc, np.array([0, S]), None, None, HQ, HKV, 0, D, S * D,
                        1.0 / math.sqrt(D), rows_step=rows_step)
    t_attn = time.perf_counter() - t0
    rows = np.arange(0, S, rows_step)
    flops = 4.0 * D * HQ * float(np.sum(rows + 1))
    frac = len(rows) / S
    t = t_attn + t_fused * frac
    return {"value": flops / t / 1e12, "unit": "TFLOP/s", "cores": oracle.num_threads(),
            "kind": "port",
            "sample": f"oracle: attention for every {rows_step}th query row ({len(rows)} of 4096) x 64 heads "
                      f"+ fused norm/RoPE/KV write (full, time scaled by {frac:.4f}); "
                      f"{t_attn:.2f}s + {t_fused:.2f}s"}


# ------------------------------------------------------------ GPU arm
def device_times(fns, reps, flush):
    """Median device time (ms) of each callable in `fns`, run in sequence,
    over `reps` repetitions with an L2 flush before each.  All repetitions
    are recorded into ONE CUDA graph with timing events between the calls
    (event-record nodes), so an interval holds the kernels' device time only:
    no host launch latency and no graph-launch gap (a graph replay costs
    ~4 us before its first kernel on B200)."""
    import torch
    cur = torch.cuda.current_stream()
    s = torch.cuda.Stream()
    s.wait_stream(cur)
    with torch.cuda.stream(s):
        for _ in range(2):
            for fn in fns:
                fn()
    cur.wait_stream(s)
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True, external=True) for _ in range(len(fns) + 1)]
          for _ in range(reps)]
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for r in range(reps):
            flush()
            ev[r][0].record()
            for i, fn in enumerate(fns):
                fn()
                ev[r][i + 1].record()
    graph.replay()
    torch.cuda.synchronize()
    return [statistics.median(ev[r][i].elapsed_time(ev[r][i + 1]) for r in range(reps))
            for i in range(len(fns))]


def e2e_pipelined(args, g, dev, stream, host_in, host_out, dev_in0, out0, consts, dist):
    import torch
    dqw, dkw, table, q_out, kc, vc = consts
    sets = [(dev_in0, out0), (tuple(torch.empty_like(t) for t in dev_in0), torch.empty_like(out0))]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = lambda: torch.cuda.Event()
    n = args.steps
    in_ready = [ev() for _ in range(n)]
    done = [ev() for _ in range(n)]
    out_read = [ev() for _ in range(n)]

    def run(n_steps, e0=None, e1=None):
        if e0 is not None:
            e0.record(stream)
            s_in.wait_stream(stream)
        for i in range(n_steps):
            (dq, dk, dv), out = sets[i % 2]
            with torch.cuda.stream(s_in):
                if i >= 2:
                    s_in.wait_event(done[i - 2])   # step i-2 finished reading this set
                for d, h in zip((dq, dk, dv), host_in):
                    d.copy_(h, non_blocking=True)
                in_ready[i].record(s_in)
            stream.wait_event(in_ready[i])
            if i >= 2:
                stream.wait_event(out_read[i - 2])  # out buffer of this set copied back
            g.qk_norm_rope_kv_prefill(dq, dk, dv, dqw, dkw, table, q_out, kc, vc, 0, EPS)
            g.attention_prefill(q_out, kc, vc, out, 0)
            done[i].record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(done[i])
                host_out.copy_(out, non_blocking=True)
                out_read[i].record(s_out)
        stream.wait_stream(s_out)
        if e1 is not None:
            e1.record(stream)

    run(min(n, 3))
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    run(n, e0, e1)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def copy_ceiling_ms(dev, host_in, host_out, dist, reps=5):
    """The e2e step's host-copy bound on this rank, all ranks copying at once:
    the same pinned H2D (inputs) and D2H (output) bytes as one e2e step, on
    two streams like e2e_pipelined, without any compute.  Median ms."""
    import torch
    dev_in = [torch.empty_like(h, device=dev) for h in host_in]
    dev_out = torch.empty_like(host_out, device=dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ts = []
    for _ in range(reps):
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        cur = torch.cuda.current_stream(dev)
        e0.record(cur)
        s_in.wait_stream(cur)
        s_out.wait_stream(cur)
        with torch.cuda.stream(s_in):
            for d, h in zip(dev_in, host_in):
                d.copy_(h, non_blocking=True)
        with torch.cuda.stream(s_out):
            host_out.copy_(dev_out, non_blocking=True)
        cur.wait_stream(s_in)
        cur.wait_stream(s_out)
        e1.record(cur)
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    return statistics.median(ts)


def hbm_read_gbs(dev, nbytes=4 << 30, reps=5):
    """Read-only HBM rate: a torch sum over an nbytes f32 buffer (decode is a
    pure read stream, which the copy-based peak understates)."""
    import torch
    x = torch.ones(nbytes // 4, dtype=torch.float32, device=dev)
    ts = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        x.sum()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    del x
    torch.cuda.empty_cache()
    return nbytes / (min(ts) * 1e-3) / 1e9


def run_ours(args, rank, world, local_rank):
    import torch
    import grout_b200 as g

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    g.init(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
    q, k, v, qw, kw = make_inputs(1000 * rank)
    pin = lambda a: torch.from_numpy(np.ascontiguousarray(a)).pin_memory()
    hq_, hk_, hv_ = pin(q), pin(k), pin(v)
    dq, dk, dv = hq_.to(dev), hk_.to(dev), hv_.to(dev)
    dqw, dkw = pin(qw).to(dev), pin(kw).to(dev)
    table = g.rope_table(THETA, S, dev)
    kc = torch.zeros(HKV, S, D, dtype=torch.float16, device=dev)
    vc = torch.zeros_like(kc)
    q_out = torch.empty_like(dq)
    out = torch.empty_like(dq)
    host_out = torch.empty(out.shape, dtype=torch.float16).pin_memory()
    flush = L2Flush(dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        g.qk_norm_rope_kv_prefill(dq, dk, dv, dqw, dkw, table, q_out, kc, vc, 0, EPS)
        g.attention_prefill(q_out, kc, vc, out, 0)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    g.check_device_error()

    # The K timed steps are recorded into one CUDA graph (as the engine
    # records its decode step): per step an L2 flush, then the fused write
    # and the prefill kernel with timing events recorded on the device
    # between them, so the intervals hold device work only, not the
    # Python/ctypes launch path or the graph-launch gap.
    fns = (lambda: g.qk_norm_rope_kv_prefill(dq, dk, dv, dqw, dkw, table, q_out, kc, vc, 0, EPS),
           lambda: g.attention_prefill(q_out, kc, vc, out, 0))
    for fn in fns:  # capture warm-up
        fn()
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True, external=True) for _ in range(3)]
          for _ in range(args.steps)]
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(args.steps):
            flush()  # L2 flush between timed steps (outside the events)
            ev[i][0].record()
            fns[0]()
            ev[i][1].record()
            fns[1]()
            ev[i][2].record()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        graph.replay()
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    step_ms = sum(e[0].elapsed_time(e[2]) for e in ev)
    fused_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / args.steps
    attn_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / args.steps
    g.check_device_error()

    # End to end through the public API with host buffers.  Every step copies
    # its own inputs in (pinned host -> device) and its output back; the copy
    # of step i+1's inputs and of step i-1's output run on their own streams,
    # double-buffered, while step i computes (PCIe is full duplex).
    e2e_ms = e2e_pipelined(args, g, dev, stream, (hq_, hk_, hv_), host_out,
                           (dq, dk, dv), out, (dqw, dkw, table, q_out, kc, vc), dist)

    copy_ms = copy_ceiling_ms(dev, (hq_, hk_, hv_), host_out, dist)
    step_ms, e2e_ms, attn_ms, fused_ms, copy_ms = reduce_max(
        [step_ms, e2e_ms, attn_ms, fused_ms, copy_ms], dist, dev)
    ragged = None if args.no_ragged else ragged_c4(args, dev, rank, world, dist)
    c5 = None if args.no_e2e_decode else config5(args, rank, world, dist)
    if rank != 0:
        return None

    pk = peaks()
    flops = prefill_flops(S)
    ms_per_step = step_ms / args.steps
    value = job_tflops(flops, args.steps, world, step_ms)
    achieved = flops / (attn_ms * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded N(0,1) f16 inputs; norm weights 1+N(0,0.02))",
        "config": {"workload": "C2: fused Q/K RMSNorm+RoPE+KV write -> causal GQA prefill, "
                               "Qwen3-32B layer, S=4096, Hq=64, Hkv=8, D=128, batch 1 per GPU",
                   "seq_len": S, "num_q_heads": HQ, "num_kv_heads": HKV, "head_dim": D,
                   "l2": "flushed between timed steps (256 MB write + 256 MB read, outside the events)",
                   "timing": "the K steps recorded in one CUDA graph, CUDA events recorded on the "
                             "device around each step's kernels (device time only)",
                   "parallelism": f"sequence-sharded x{world} (no collective)"},
        "roofline": {"bound": "tensor", "kernel": "prefill_kernel (tcgen05)",
                     "achieved": round(achieved, 1), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": round(achieved / pk["bf16_tflops"], 4),
                     "peak_src": pk["src"] + " bf16 burst (dense f16 == bf16 rate on B200)",
                     "traffic": PREFILL_TRAFFIC_BYTES,
                     "traffic_src": "ncu capture of prefill_kernel on this workload (not measured "
                                    "in this run); algorithmic bytes Q+K+V+O = 151 MB, the O "
                                    "writes still in L2 at kernel end are not counted by DRAM",
                     "kernel_ms": round(attn_ms, 4),
                     "algorithmic_flops": flops},
        "fused_norm_rope_kv": {"bound": "hbm", "ms": round(fused_ms, 4),
                               "gbs": round(fused_bytes(S) / (fused_ms * 1e-3) / 1e9, 1),
                               "frac": round(fused_bytes(S) / (fused_ms * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
                               "algorithmic_bytes": fused_bytes(S)},
        "e2e": {"value": round(job_tflops(flops, args.steps, world, e2e_ms), 2),
                "unit": "TFLOP/s", "h2d_bytes_per_step": int(hq_.numel() * 2 + hk_.numel() * 2 + hv_.numel() * 2),
                "d2h_bytes_per_step": int(host_out.numel() * 2),
                "ms_per_step": round(e2e_ms / args.steps, 4),
                # the host-copy bound: one step's H2D + D2H bytes copied by
                # every rank at once with no compute (max over ranks)
                "copy_ceiling": {"ms_per_step": round(copy_ms, 4),
                                 "value": round(job_tflops(flops, 1, world, copy_ms), 2),
                                 "unit": "TFLOP/s",
                                 "e2e_frac_of_ceiling": round(copy_ms / (e2e_ms / args.steps), 4)},
                "path": "grout_b200.qk_norm_rope_kv_prefill + attention_prefill, pinned host buffers; "
                        "each step's H2D and D2H copies on their own streams, overlapping the "
                        "neighbouring steps' compute"},
        "gpu_launches": 2 * args.steps,
        "clocks": clk.summary(),
    }
    if ragged is not None:
        # per GPU: the aggregate over N ranks against N GPUs' peak
        ragged["frac_per_gpu"] = round(ragged["tflops"] / (world * pk["bf16_tflops"]), 4)
        line["ragged_c4"] = ragged
    if c5 is not None:
        line["e2e_decode_c5"] = c5
    if world == 1 and not args.no_decode:
        pk["hbm_read_gbs"] = round(hbm_read_gbs(dev), 1)
        line["decode"] = decode_grid(args, dev, pk)
        line["decode_paged"] = decode_paged_cells(args, dev, pk)
        line["decode_fused"] = decode_fused_cells(args, dev, pk)
        line["tp_gemv"] = tp_gemv_cells(args, dev, pk)
        line["prefill_splitk"] = prefill_splitk_cell(args, dev, pk)
        line["qkv_proj_epilogue"] = qkv_proj_cell(args, dev, pk)
    if world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline()
    return line


def config5(args, rank, world, dist):
    """Config 5: Qwen3-32B greedy decode (random f16 weights), 8192-token
    prompt then 256 tokens under CUDA-graph replay, tensor-parallel over the
    N ranks (NCCL all-reduce after o_proj / down_proj).  Roofline tok/s =
    measured HBM GB/s / bytes each rank reads per token (its weight shard +
    its KV cache at the final position)."""
    import torch
    from grout_b200 import qwen3_tp
    c = qwen3_tp.Qwen3Shape()
    r = qwen3_tp.run_config5(rank, world, None, prompt_len=args.c5_prompt,
                             gen_tokens=args.c5_tokens, shape=c,
                             barrier=dist.barrier if dist else None,
                             fused_allreduce=not args.c5_nccl)
    dev = torch.device("cuda", torch.cuda.current_device())
    vals = reduce_max([r["decode_ms"], r["prefill_ms"], r["attn_ms_per_step"]], dist, dev)
    decode_ms, prefill_ms, attn_ms = vals
    torch.cuda.empty_cache()
    D, H = c.head_dim, c.hidden
    per_layer = (c.heads + 2 * c.kv_heads) * D * H + H * c.heads * D + 3 * H * c.inter
    w_bytes = 2.0 * (c.layers * per_layer + c.vocab * H) / world
    kv_bytes = 2.0 * c.layers * 2 * (c.kv_heads // world) * (args.c5_prompt + args.c5_tokens) * D
    step_ms = decode_ms / args.c5_tokens
    hbm = peaks()["hbm_gbs"]
    roof = hbm * 1e9 / (w_bytes + kv_bytes)
    return {"workload": f"C5: Qwen3-32B greedy decode, prompt {args.c5_prompt}, "
                        f"{args.c5_tokens} tokens, TP={world}, CUDA-graph replay",
            "tok_s": round(args.c5_tokens / (decode_ms * 1e-3), 2), "ms_per_token": round(step_ms, 4),
            "prefill_ms": round(prefill_ms, 2),
            "attention_ms_per_token": round(attn_ms, 4),
            "attention_share": round(attn_ms / step_ms, 4),
            "roofline_tok_s": round(roof, 1), "frac": round(args.c5_tokens / (decode_ms * 1e-3) / roof, 4),
            "bytes_per_token_per_rank": w_bytes + kv_bytes, "first_tokens": r["first_tokens"],
            "stage_ms_per_token_rank0": r["stage_ms_per_step"],
            "allreduce": r["allreduce"]}


def ragged_c4(args, dev, rank, world, dist):
    """Config 4: ragged causal prefill batch at Qwen3-8B heads (32 query / 8
    KV heads), 16 sequences with lengths uniform in [128, 8192] (seed 5),
    packed varlen K/V [tokens][8][128].  Across N ranks the layer is split by
    KV head (rank r owns KV heads [r*8/N, (r+1)*8/N) and their query heads):
    strong scaling, no collective.  FLOPs = 4*D*Hq*sum_i L_i(L_i+1)/2 for the
    whole batch; time = max over ranks of the per-rank kernel time."""
    import torch
    import grout_b200 as g
    from grout_b200 import synth
    hq, hkv = 32, 8
    lens = synth.ragged_lengths(5, 16, 128, 8192)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    tot = int(cu[-1])
    gen = torch.Generator(device=dev).manual_seed(5)
    q = torch.randn(tot, hq, D, device=dev, generator=gen).half()
    k = torch.randn(tot, hkv, D, device=dev, generator=gen).half()
    v = torch.randn(tot, hkv, D, device=dev, generator=gen).half()
    out = torch.empty_like(q)
    dcu = torch.from_numpy(cu).to(dev)
    ks = dcu[:-1].contiguous()
    lo, hi = shard_kv_heads(hkv, world, rank)
    flush = L2Flush(dev)
    (ms,) = device_times([lambda: g.attention_prefill_varlen(
        q, k, v, out, dcu, int(lens.max()), hkv, kv_row_stride=hkv * D, kv_head_stride=D,
        kv_rows=tot, kv_start=ks, kv_head_range=(lo, hi))], max(3, min(args.steps, 10)), flush)
    g.check_device_error()
    (ms,) = reduce_max([ms], dist, dev)
    flops = 4.0 * D * hq * float(np.sum(lens.astype(np.float64) * (lens + 1) / 2))
    return {"workload": "C4: 16 ragged sequences, L ~ U[128, 8192] (seed 5), Qwen3-8B heads 32/8",
            "tokens": tot, "lengths": lens.tolist(), "ms": round(ms, 4),
            "tflops": round(flops / (ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s",
            "sharding": f"KV heads split over {world} rank(s), strong scaling",
            "algorithmic_flops": flops}


def decode_grid(args, dev, pk):
    """Config 3: split-K decode over B x L cells (Qwen3-32B, 64/8 heads), and
    config 1 (Qwen3-4B, 32/8 heads, L = 1024).  HBM bytes per cell:
    B*(2*Hkv*L*D*2 + 2*Hq*D*2).  Each rep is timed alone with an L2 flush
    before it."""
    import torch
    import grout_b200 as g
    flush = L2Flush(dev)
    cells = []
    shapes = [(1, 32, 8, 1024)] + [(B, 64, 8, L) for B in (1, 8, 32, 64)
                                   for L in (2048, 8192, 16384, 32768)]
    if args.decode_cells:
        shapes = [(int(b), 64, 8, int(l)) for b, l in
                  (c.split("x") for c in args.decode_cells.split(","))]
    reps = max(3, min(args.steps, 10))
    for B, hq, hkv, L in shapes:
        kc = torch.randn(B, hkv, L, D, device=dev, dtype=torch.float16)
        vc = torch.randn_like(kc)
        q = torch.randn(B, hq, D, device=dev, dtype=torch.float16)
        out = torch.empty_like(q)
        pos = torch.full((B,), L - 1, dtype=torch.int32, device=dev)
        nks = g.decode_splits(B, L, hq, hkv, L)
        ws = torch.empty(max(16, g.decode_workspace_bytes(B, L, hq, hkv, L)), dtype=torch.uint8, device=dev)
        (ms,) = device_times([lambda: g.attention_decode(q, kc, vc, pos, out, L, workspace=ws)],
                             reps, flush)
        us = ms * 1e3
        nbytes = B * (2 * hkv * L * D * 2 + 2 * hq * D * 2)
        gbs = nbytes / (us * 1e-6) / 1e9
        cells.append({"B": B, "L": L, "hq": hq, "splits": nks, "us": round(us, 2),
                      "gbs": round(gbs, 1), "frac": round(gbs / pk["hbm_gbs"], 4),
                      "frac_read": round(gbs / pk["hbm_read_gbs"], 4)})
        del kc, vc
        torch.cuda.empty_cache()
    g.check_device_error()
    big = [c for c in cells if c["B"] * c["L"] >= 8 * 8192]
    return {"unit": "GB/s", "peak_gbs": pk["hbm_gbs"], "read_peak_gbs": pk["hbm_read_gbs"],
            "frac": "of the measured copy peak; frac_read: of the read-only rate measured "
                    "in this run (torch sum over 4 GiB)", "cells": cells,
            "mean_frac_large_cells": round(statistics.mean(c["frac"] for c in big), 4) if big else None}


def prefill_splitk_cell(args, dev, pk):
    """A launch with fewer work items than SMs (one sequence, S = 2048, 8/1
    heads: 64 items for 148 SMs) with and without the split-K path."""
    import ctypes
    import torch
    import grout_b200 as g
    flush = L2Flush(dev)
    S, hq, hkv = 2048, 8, 1
    q = torch.randn(S, hq, D, device=dev, dtype=torch.float16)
    k = torch.randn(hkv, S, D, device=dev, dtype=torch.float16)
    v = torch.randn_like(k)
    out = torch.empty_like(q)
    flops = 4.0 * D * hq * S * (S + 1) / 2
    nks = g.lib().grout_attn_prefill_splits(1, S, ctypes.byref(g.attn.make_dims(hq, hkv, S)))
    ws = torch.empty(max(16, g.lib().grout_attn_prefill_splitk_workspace_bytes(1, S, hq, nks)),
                     dtype=torch.uint8, device=dev)
    res = {"workload": "one sequence, S=2048, 8 query / 1 KV heads (64 items)", "splits": nks}
    for name, fn in (("unsplit", lambda: g.attention_prefill(q, k, v, out, 0)),
                     ("split", lambda: g.attention_prefill_splitk(
                         q, k, v, out, None, S, hkv, kv_row_stride=D, kv_head_stride=S * D,
                         kv_rows=S, num_splits=nks, workspace=ws))):
        (ms,) = device_times([fn], max(3, min(args.steps, 10)), flush)
        us = ms * 1e3
        res[name] = {"us": round(us, 2), "tflops": round(flops / (us * 1e-6) / 1e12, 1)}
    g.check_device_error()
    return res


def qkv_proj_cell(args, dev, pk):
    """Config 2's QKV projection (S = 4096, hidden 5120 -> 80 heads x 128)
    with the fused norm/RoPE/KV write as its epilogue, against the unfused
    pair it replaces (cuBLAS GEMM into an f16 activation + the fused kernel)."""
    import ctypes
    import torch
    import grout_b200 as g
    flush = L2Flush(dev)
    S, hidden, hq, hkv = 4096, 5120, 64, 8
    N = (hq + 2 * hkv) * D
    x = torch.randn(S, hidden, device=dev, dtype=torch.float16)
    w = (torch.randn(N, hidden, device=dev) * 0.02).half()
    ones = torch.ones(D, dtype=torch.float16, device=dev)
    table = g.rope_table(1.0e6, S, dev)
    q_out = torch.empty(S, hq, D, dtype=torch.float16, device=dev)
    kc = torch.zeros(hkv, S, D, dtype=torch.float16, device=dev)
    vc = torch.zeros_like(kc)
    qkv = torch.empty(S, N, dtype=torch.float16, device=dev)
    q_wide = torch.empty(S, N, dtype=torch.float16, device=dev)  # q_out shares q's row stride
    dims = g.attn.make_dims(hq, hkv, S, 1e-6)
    vp = ctypes.c_void_p

    def unfused():
        # the reference's pair: GEMM into the f16 activation, then the fused
        # kernel reading q/k/v straight out of it (row stride N)
        torch.matmul(x, w.t(), out=qkv)
        st = g.lib().grout_qk_norm_rope_kv_prefill(
            vp(qkv.data_ptr()), vp(qkv.data_ptr() + hq * D * 2), vp(qkv.data_ptr() + (hq + hkv) * D * 2),
            N, N, vp(ones.data_ptr()), vp(ones.data_ptr()), vp(table.data_ptr()), vp(q_wide.data_ptr()),
            vp(kc.data_ptr()), vp(vc.data_ptr()), S * D, 0, S, ctypes.byref(dims),
            vp(torch.cuda.current_stream().cuda_stream))
        if st != 0:
            raise RuntimeError(g.lib().grout_attn_last_error().decode())

    flops = 2.0 * S * hidden * N
    res = {"workload": "QKV projection S=4096, 5120 -> 10240, + norm/RoPE/KV write", "gemm_flops": flops}
    for name, fn in (("fused_epilogue", lambda: g.qkv_proj_norm_rope_kv_prefill(
                         x, w, ones, ones, table, q_out, kc, vc, 0, 1e-6)),
                     ("cublas_gemm_plus_fused_kernel", unfused)):
        (ms,) = device_times([fn], max(3, min(args.steps, 10)), flush)
        us = ms * 1e3
        res[name] = {"us": round(us, 2), "tflops": round(flops / (us * 1e-6) / 1e12, 1)}
    g.check_device_error()
    return res


def decode_fused_cells(args, dev, pk):
    """One decode step of a layer's attention at config 5's shapes (8192-token
    prompt + 256 tokens: position 8447) and config 1's: the fused write +
    split-K attention as one kernel (grout_attn_decode_fused) against the two
    launches it replaces (qk_norm_rope_kv_decode, then attention_decode).
    Bytes: the KV cache read plus the QKV row in and the K/V row and output
    out."""
    import torch
    import grout_b200 as g
    flush = L2Flush(dev)
    reps = max(3, min(args.steps, 10))
    cells = []
    for name, hq, hkv, L in (("C5 TP=1", 64, 8, 8448), ("C5 TP=8", 8, 1, 8448),
                             ("C1", 32, 8, 1024)):
        gen = torch.Generator(device=dev).manual_seed(hq + L)
        kc = torch.randn(1, hkv, L, D, device=dev, generator=gen).half()
        vc = torch.randn_like(kc)
        qkv = torch.randn(1, (hq + 2 * hkv) * D, device=dev, generator=gen).half()
        w = torch.ones(D, device=dev, dtype=torch.float16)
        table = g.rope_table(THETA, L, dev)
        q1 = torch.empty(1, hq, D, device=dev, dtype=torch.float16)
        out = torch.empty_like(q1)
        pos = torch.full((1,), L - 1, dtype=torch.int32, device=dev)
        ws = torch.empty(max(16, g.decode_workspace_bytes(1, L, hq, hkv, L)), dtype=torch.uint8,
                         device=dev)
        fused, sep_w, sep_a = device_times([
            lambda: g.attention_decode_fused(qkv, w, w, table, kc, vc, pos, out, L, EPS, workspace=ws),
            lambda: g.qk_norm_rope_kv_decode(qkv, w, w, table, q1, kc, vc, pos, hq, hkv, EPS),
            lambda: g.attention_decode(q1, kc, vc, pos, out, L, workspace=ws)], reps, flush)
        nbytes = 2 * hkv * L * D * 2 + (hq + 2 * hkv) * D * 2 + 2 * hkv * D * 2 + hq * D * 2
        cells.append({"cell": name, "hq": hq, "hkv": hkv, "L": L,
                      "splits": g.decode_splits(1, L, hq, hkv, L),
                      "fused_us": round(fused * 1e3, 2),
                      "separate_us": round((sep_w + sep_a) * 1e3, 2),
                      "fused_gbs": round(nbytes / (fused * 1e-3) / 1e9, 1),
                      "fused_frac": round(nbytes / (fused * 1e-3) / 1e9 / pk["hbm_gbs"], 4)})
        del kc, vc
        torch.cuda.empty_cache()
    g.check_device_error()
    return {"unit": "us", "timing": "device time of one call (events recorded inside one graph)",
            "cells": cells}


def tp_gemv_cells(args, dev, pk):
    """The row-parallel GEMV of grout_gemv_allreduce (one rank: the exchange
    is local) at config 5's o_proj / down_proj shard shapes, against torch's
    cuBLAS GEMV of the same shape.  Bytes: the weight shard; frac of the
    measured copy peak."""
    import torch
    from grout_b200 import tp
    flush = L2Flush(dev)
    reps = max(3, min(args.steps, 10))
    comm = tp.TPComm(0, 1, 5120, device=dev)
    cells = []
    for name, k in (("o_proj TP=8", 1024), ("down_proj TP=8", 3200), ("o_proj TP=2", 4096),
                    ("down_proj TP=2", 12800)):
        w = (torch.randn(5120, k, device=dev) * 0.02).half()
        x = torch.randn(k, device=dev).half()
        out = torch.empty(5120, device=dev, dtype=torch.float16)
        y = torch.empty(1, 5120, device=dev, dtype=torch.float16)
        t_ours, t_cub = device_times([lambda: comm.gemv_allreduce(w, x, out),
                                      lambda: torch.matmul(x.view(1, -1), w.t(), out=y)],
                                     reps, flush)
        nbytes = 5120 * k * 2
        cells.append({"cell": name, "k": k, "grout_us": round(t_ours * 1e3, 2),
                      "grout_frac": round(nbytes / (t_ours * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
                      "cublas_us": round(t_cub * 1e3, 2),
                      "cublas_frac": round(nbytes / (t_cub * 1e-3) / 1e9 / pk["hbm_gbs"], 4)})
    comm.close()
    return {"unit": "us", "cells": cells}


def decode_paged_cells(args, dev, pk):
    """The paged KV cache (page-pool layout [num_pages, Hkv, page_size, D],
    pages of each sequence shuffled across the pool) on config-3 cells, timed
    like decode_grid; bytes per cell are the same as the contiguous cell's."""
    import torch
    import grout_b200 as g
    flush = L2Flush(dev)
    reps = max(3, min(args.steps, 10))
    cells = []
    for B, L, ps in ((8, 8192, 64), (32, 16384, 128), (64, 32768, 256)):
        hq, hkv = 64, 8
        per = L // ps
        n = B * per
        gen = torch.Generator().manual_seed(7)
        table = torch.randperm(n, generator=gen).view(B, per).to(torch.int32).to(dev)
        kp = torch.randn(n, hkv, ps, D, device=dev, dtype=torch.float16)
        vp = torch.randn_like(kp)
        q = torch.randn(B, hq, D, device=dev, dtype=torch.float16)
        out = torch.empty_like(q)
        pos = torch.full((B,), L - 1, dtype=torch.int32, device=dev)
        ws = torch.empty(max(16, g.decode_workspace_bytes(B, L, hq, hkv, L)), dtype=torch.uint8, device=dev)
        (ms,) = device_times([lambda: g.attention_decode_paged(q, kp, vp, table, pos, out, L,
                                                               workspace=ws)], reps, flush)
        us = ms * 1e3
        nbytes = B * (2 * hkv * L * D * 2 + 2 * hq * D * 2)
        gbs = nbytes / (us * 1e-6) / 1e9
        cells.append({"B": B, "L": L, "page_size": ps, "us": round(us, 2), "gbs": round(gbs, 1),
                      "frac": round(gbs / pk["hbm_gbs"], 4)})
        del kp, vp
        torch.cuda.empty_cache()
    g.check_device_error()
    return {"unit": "GB/s", "layout": "page pool [num_pages, Hkv, page_size, 128], shuffled pages",
            "cells": cells}


# ------------------------------------------------------------ reference arm
def run_reference(args):
    """The reference's CPU path for the same workload (the oracle port; the
    Rust reference cannot be built here), all host threads, K timed steps
    each on the bounded sample (about 5 s of CPU work per step)."""
    import oracle
    oracle.set_num_threads(os.cpu_count() or 1)  # torchrun sets OMP_NUM_THREADS=1
    cpu_baseline(rows_step=512)  # warm-up: page in, spin up the thread pool
    vals = []
    last = None
    for _ in range(args.steps):
        last = cpu_baseline(rows_step=4)
        vals.append(last["value"])
    v = statistics.median(vals)
    return {"metric": METRIC, "value": round(v, 6), "unit": "TFLOP/s", "impl": "reference",
            "n_gpus": 0, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) f16 inputs)",
            "config": {"workload": "C2: fused Q/K RMSNorm+RoPE+KV write -> causal GQA prefill, "
                                   "Qwen3-32B layer, S=4096, Hq=64, Hkv=8, D=128",
                       "seq_len": S},
            "cpu_baseline": {"value": round(v, 6), "unit": "TFLOP/s", "cores": oracle.num_threads(),
                             "kind": "port", "sample": last["sample"]},
            "e2e": {"value": round(v, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def emit(line):
    """Writes the one JSON line to the real stdout (see main)."""
    os.write(_STDOUT_FD, (json.dumps(line) + "\n").encode())


def profile_case_qkv_proj():
    """Qwen3-32B prefill QKV projection + fused norm/RoPE/KV write, S = 4096:
    two launches on cuda:0, so `ncu -k <kernel> -s 1 -c 1` captures one warm
    launch."""
    import torch
    import grout_b200 as g
    g.init(0)
    hidden, N = 5120, (HQ + 2 * HKV) * D
    dev = torch.device("cuda", 0)
    x = torch.randn(S, hidden, device=dev).half()
    w = (torch.randn(N, hidden, device=dev) * 0.02).half()
    ones = torch.ones(D, dtype=torch.float16, device=dev)
    table = g.rope_table(THETA, S, dev)
    q_out = torch.empty(S, HQ, D, dtype=torch.float16, device=dev)
    kc = torch.zeros(HKV, S, D, dtype=torch.float16, device=dev)
    vc = torch.zeros_like(kc)
    for _ in range(2):
        g.qkv_proj_norm_rope_kv_prefill(x, w, ones, ones, table, q_out, kc, vc, 0, EPS)
    torch.cuda.synchronize()
    g.check_device_error()


def profile_case_decode_fused():
    """Config 5's decode step at TP = 1 (64/8 heads, position 8447): the
    fused norm/RoPE/KV write + split-K attention, two launches."""
    import torch
    import grout_b200 as g
    g.init(0)
    dev = torch.device("cuda", 0)
    hq, hkv, L = HQ, HKV, 8448
    kc = torch.randn(1, hkv, L, D, device=dev).half()
    vc = torch.randn_like(kc)
    qkv = torch.randn(1, (hq + 2 * hkv) * D, device=dev).half()
    w = torch.ones(D, device=dev, dtype=torch.float16)
    table = g.rope_table(THETA, L, dev)
    out = torch.empty(1, hq, D, device=dev, dtype=torch.float16)
    pos = torch.full((1,), L - 1, dtype=torch.int32, device=dev)
    for _ in range(2):
        g.attention_decode_fused(qkv, w, w, table, kc, vc, pos, out, L, EPS)
    torch.cuda.synchronize()
    g.check_device_error()


def profile_case_norm_rope():
    """Config 2's fused Q/K norm + RoPE + KV write (S = 4096): two launches."""
    import torch
    import grout_b200 as g
    g.init(0)
    dev = torch.device("cuda", 0)
    q = torch.randn(S, HQ, D, device=dev).half()
    k = torch.randn(S, HKV, D, device=dev).half()
    v = torch.randn_like(k)
    w = torch.ones(D, device=dev, dtype=torch.float16)
    table = g.rope_table(THETA, S, dev)
    q_out = torch.empty_like(q)
    kc = torch.zeros(HKV, S, D, dtype=torch.float16, device=dev)
    vc = torch.zeros_like(kc)
    for _ in range(2):
        g.qk_norm_rope_kv_prefill(q, k, v, w, w, table, q_out, kc, vc, 0, EPS)
    torch.cuda.synchronize()
    g.check_device_error()


def profile_case_tp_gemv():
    """grout_gemv_allreduce on one rank at config 5's TP = 2 down_proj shard
    (5120 x 12800): two launches."""
    import torch
    import grout_b200 as g
    from grout_b200 import tp
    g.init(0)
    dev = torch.device("cuda", 0)
    comm = tp.TPComm(0, 1, 5120, device=dev)
    w = (torch.randn(5120, 12800, device=dev) * 0.02).half()
    x = torch.randn(12800, device=dev).half()
    out = torch.empty(5120, device=dev, dtype=torch.float16)
    for _ in range(2):
        comm.gemv_allreduce(w, x, out)
    torch.cuda.synchronize()
    g.check_device_error()
    comm.close()


PROFILE_CASES = {"qkv_proj": profile_case_qkv_proj, "decode_fused": profile_case_decode_fused,
                 "norm_rope": profile_case_norm_rope, "tp_gemv": profile_case_tp_gemv}

_STDOUT_FD = 1


def main():
    # Everything else that reaches fd 1 (e.g. the NCCL version banner printed
    # when a communicator is created) goes to stderr: stdout carries only the
    # JSON line.
    global _STDOUT_FD
    sys.stdout.flush()
    _STDOUT_FD = os.dup(1)
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-ragged", action="store_true", help="skip the config-4 ragged batch")
    ap.add_argument("--no-e2e-decode", action="store_true", help="skip config 5 (Qwen3-32B decode)")
    ap.add_argument("--c5-prompt", type=int, default=8192)
    ap.add_argument("--c5-tokens", type=int, default=256)
    ap.add_argument("--c5-nccl", action="store_true",
                    help="config 5 with cuBLAS GEMV + NCCL all-reduce instead of the fused kernel")
    ap.add_argument("--no-prefill", action="store_true",
                    help="skip the prefill workload (decode grid only; for profiling)")
    ap.add_argument("--only", default="",
                    help="with --no-prefill: comma list of decode, decode_paged, decode_fused, "
                         "tp_gemv, prefill_splitk, qkv_proj_epilogue (default: all)")
    ap.add_argument("--decode-cells", default="",
                    help="comma list BxL of config-3 cells (default: the full grid + config 1)")
    ap.add_argument("--profile-case", choices=sorted(PROFILE_CASES),
                    help="run one small single-kernel workload for an ncu capture and exit "
                         "(prints no JSON line)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.profile_case:
        PROFILE_CASES[args.profile_case]()
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            emit(run_reference(args))
        return

    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    if args.no_prefill:
        import torch
        import grout_b200 as g
        dev = torch.device("cuda", local_rank)
        torch.cuda.set_device(dev)
        g.init(local_rank)
        if rank == 0:
            pk = peaks()
            pk["hbm_read_gbs"] = round(hbm_read_gbs(dev), 1)
            parts = {"decode": decode_grid, "decode_paged": decode_paged_cells,
                     "decode_fused": decode_fused_cells, "tp_gemv": tp_gemv_cells,
                     "prefill_splitk": prefill_splitk_cell,
                     "qkv_proj_epilogue": qkv_proj_cell}
            only = args.only.split(",") if args.only else list(parts)
            line = {k: parts[k](args, dev, pk) for k in only}
        else:
            line = None
    else:
        line = run_ours(args, rank, world, local_rank)
    if line is not None:
        emit(line)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
