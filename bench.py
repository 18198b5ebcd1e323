"""Benchmark of the sparse-MLA decode path (BASELINE config 2 by default).

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl dsv4|reference] [--config c2|c3|c4|c5|c5w]

A step is one decode token of the measured path — per-head norm + RoPE of q, the window index list,
the lightning-indexer scores + top-k over the compressed keys, sparse attention over the 640
gathered rows with the inverse RoPE fused — for every sequence of the config's batch (config 2:
batch 1 against a 32768-token context; config 3: batch 64 against 8192-token contexts).

Timing: `value` replays the step's CUDA graph with inputs resident in HBM, rotating over R replicas
of the whole state (R * footprint > 2 x L2, so no step finds its inputs in L2); K steps are
bracketed by a barrier + synchronize and timed with CUDA events, max over ranks. `e2e` runs the
same K steps through the public DecodeRunner.step_host: pinned host inputs copied in, the graph,
the output copied out, every step. N > 1: each rank runs its own replica set (decode batches split
across GPUs with no collective; weak scaling).
"""
import argparse
import json

import numpy as np
import os
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PKG = "deepseek-v4-flash-mlx_b200"
METRIC = "sparse-MLA decode tok/s at 32K ctx (indexer + top-k + sparse attention + RoPE)"
METRICS = {"c2": METRIC,
           "c3": "sparse-MLA batched decode tok/s (indexer + top-k + sparse attention + RoPE)",
           "c4": "sparse-MLA prefill tok/s at 64K ctx (compressors + indexer top-k + sparse attention)",
           "c5": "full attention block decode tok/s (projections + compressor + indexer + sparse MLA + o_proj)",
           "c5w": "window-only (ratio-128) attention block decode tok/s (projections + window attention + o_proj)"}
CONFIGS = {
    "c2": dict(batch=1, ctx=32768, top_k=512, seeds=lambda r, i: 1 + 7919 * r, strong=False,
               workload="config2: decode, batch 1, 32768-token context (8192 compressed + 128 window rows), "
                        "top-k 512, bf16 cache, fp32 indexer keys"),
    "c3": dict(batch=64, ctx=8192, top_k=512, seeds=lambda r, i: 100 + i, strong=True,
               workload="config3: batched decode, global batch 64 split across GPUs, 8192-token contexts "
                        "(2048 compressed + 128 window rows each), top-k 512"),
    "c4": dict(batch=1, ctx=65536, top_k=1024, seeds=lambda r, i: 2,
               workload="config4: long prefill, 65536 tokens: KV + indexer-key compressors (16384 rows), indexer "
                        "top-k 1024 causal, sparse attention over 128 window + 1024 rows; query-sharded with an NCCL "
                        "all-gather of compressed KV and keys"),
    "c5": dict(batch=32, ctx=16384, top_k=512, seeds=lambda r, i: 3 + i, strong=True,
               workload="config5: full attention block decode, global batch 32 split across GPUs, 16384-token "
                        "contexts, int8-g64 weights (bf16 scales), top-k 512"),
    "c5w": dict(batch=32, ctx=16384, top_k=0, seeds=lambda r, i: 3 + i, strong=True,
                workload="config5 block at a ratio-128 layer (window-only attention, as the reference runs "
                         "ratio-128 layers): global batch 32 split across GPUs, 16384-token contexts, 128-row "
                         "window rings, int8-g64 weights (bf16 scales)"),
}
L2_BYTES = 126 * 1024 * 1024

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the dominant op, from one
# ncu capture each on B200: config 2 on this bench's own command (score + select kernels of one
# step); config 4 on `--kernel-case attn_prefill` (4,096 of the 65,536 queries, every query with
# 1,152 list entries), scaled by 16 to the step's eight 8,192-query launches.
TRAFFIC = {"c2": {"indexer_topk": 4331264, "sparse_attn": 2138982},
           "c4": {"tc::attn_tc_kernel": 16 * 547425536}}


def _pkg():
    import importlib
    return importlib.import_module(PKG)


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML every ~10 ms (reading only)."""

    NAMES = {0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
             0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device_index):
        self.samples, self.reasons, self.ok = [], set(), False
        self.window = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None
        self._stop = threading.Event()

    def _run(self):
        while not self._stop.is_set():
            try:
                mhz = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((time.perf_counter(), mhz, r))
            except Exception:
                pass
            time.sleep(0.01)

    def start(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()

    def sample_while(self, event, period=0.001):
        """Sample on the calling thread, every `period` seconds, until `event` (the CUDA event that
        ends the timed region) has completed: a timed region shorter than the thread's 10 ms period
        still gets samples while the GPU works through the queued steps."""
        if not self.ok:
            return
        while not event.query():
            try:
                self.samples.append((time.perf_counter(), self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM),
                                     self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)))
            except Exception:
                pass
            time.sleep(period)

    def stop(self):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self, t0, t1):
        inside = [s for s in self.samples if t0 <= s[0] <= t1]
        use = inside or self.samples
        reasons = set()
        for _, _, r in use:
            for bit, name in self.NAMES.items():
                if r & bit:
                    reasons.add(name)
        mhz = [m for _, m, _ in use]
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(use), "samples_in_timed_region": len(inside),
                "source": "nvml"}


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _barrier_max(x, world, device):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


# ------------------------------------------------------------------------------ CPU reference leg
CPU_MIN_SECONDS = 10.0  # timed CPU work per reported number (a bounded sample of the workload)


def _cpu_threads(threads=None):
    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    return threads


def cpu_workload(cfg_name, samples):
    """Set up, once, a bounded sample of the config's workload for the CPU oracle (torch fp32 + the
    C indexer restatement). Returns (run, desc): run() performs one timed repetition and returns
    (tokens, seconds) of it."""
    from oracle import layer_ref as LR
    from oracle import norm_rope_ref as NR
    if cfg_name == "c4":
        return _cpu_prefill(samples)
    if cfg_name == "c5":
        return _cpu_block(samples)
    if cfg_name == "c5w":
        return _cpu_block_window(samples)
    cfgd = CONFIGS[cfg_name]
    C = __import__("importlib").import_module(PKG + ".configs")
    f = NR.precompute_freqs(64, 0, 65536, 160000.0, 16, 32, 1)
    batch = min(cfgd["batch"], samples)
    case = C.make_decode_case(batch, cfgd["ctx"], cfgd["top_k"], seeds=[cfgd["seeds"](0, i) for i in range(batch)],
                              device="cpu", shuffle_pages=True)
    pool, win_base, comp_rows = C.decode_case_host_pool(case)
    h = case.host

    def run():
        t0 = time.perf_counter()
        LR.decode_attention_ref(pool, win_base, comp_rows, h["k_idx"], h["q"], h["q_idx"], h["w_idx"], h["sink"],
                                h["positions"], cfgd["top_k"], f)
        return batch, time.perf_counter() - t0
    return run, f"{batch} decode token(s) of {cfg_name} per repetition through the CPU oracle"


def cpu_sample_size(cfg_name):
    """Tokens per repetition of the CPU sample: the block configs run their batch of 32 per call (the
    weights are read once per call, as a CPU implementation would), config 4 runs 64 queries, the
    attention-only decode configs one sequence (their oracle loops over sequences anyway)."""
    return {"c4": 64, "c5": 32, "c5w": 32}.get(cfg_name, 1)


def _dequantized(W):
    """The attention weights with every 8-bit grouped matrix dequantised to fp32 once, so that the
    CPU oracle's timed repetitions do not repeat the dequantisation."""
    from dataclasses import fields
    from oracle.layer_ref import _w
    return W.__class__(**{f.name: _w(getattr(W, f.name)) if hasattr(getattr(W, f.name), "scale")
                          else getattr(W, f.name) for f in fields(W)})


def timed_rate(run, min_seconds=CPU_MIN_SECONDS):
    """Repeat run() until at least min_seconds of timed work; returns (tok/s, repetitions, seconds)."""
    tok = sec = 0.0
    reps = 0
    while sec < min_seconds or reps == 0:
        t, dt = run()
        tok, sec, reps = tok + t, sec + dt, reps + 1
    return tok / sec, reps, sec


def cpu_reference(cfg_name, samples, threads=None, min_seconds=CPU_MIN_SECONDS):
    """Time the oracle port on the host cores: one warm-up repetition, then repetitions of the
    config's bounded sample until at least min_seconds of timed work; returns (tok/s, cores, description)."""
    threads = _cpu_threads(threads)
    run, desc = cpu_workload(cfg_name, samples)
    run()
    v, reps, sec = timed_rate(run, min_seconds)
    return v, threads, f"{desc}; {reps} repetitions, {sec:.1f} s of timed CPU work, {threads} threads"


def _cpu_prefill(nq):
    """Config 4 per-token CPU cost: the two compressors over a 4096-token slice (per token), plus
    the indexer over 16384 keys and attention over 1152 rows for nq queries in the middle of the
    65536-token sequence (per query)."""
    import importlib
    from oracle import compressor_ref as CR
    from oracle import indexer_ref as I
    from oracle import norm_rope_ref as NR
    from oracle import sparse_attn_ref as SA
    Lm = importlib.import_module(PKG + ".layer")
    W = Lm.make_attention_weights(2)
    g = torch.Generator().manual_seed(2)
    xs = torch.randn(4096, 4096, generator=g)
    s = 65536
    keys = torch.randn(16384, 128, generator=g)
    qi = torch.randn(nq, 64, 128, generator=g)
    wi = torch.randn(nq, 64, generator=g) / 8
    q = torch.randn(nq, 64, 512, generator=g)
    kvcat = torch.randn(s + 16384, 512, generator=g).to(torch.bfloat16).float()
    f = NR.precompute_freqs(64, 0, 65536, 160000.0, 16, 32, 1)
    pos = np.arange(s // 2 - nq, s // 2)   # mid-sequence queries: the average visible key count
    win = np.stack([np.arange(t - 127, t + 1) for t in pos])

    def run():
        t0 = time.perf_counter()
        CR.compressor_prefill(xs[None], W.c_wkv.float(), W.c_wgate.float(), W.c_ape, W.c_norm)
        CR.compressor_prefill(xs[None], W.i_wkv.float(), W.i_wgate.float(), W.i_ape, W.i_norm, head_dim=128)
        t_comp = time.perf_counter() - t0
        t0 = time.perf_counter()
        sel = I.indexer_topk(qi.numpy()[None], wi.numpy()[None], keys.numpy()[None], 1024, positions=pos[None],
                             ratio=4)[0]
        idx = torch.from_numpy(np.concatenate([win, sel + s], 1).astype(np.int64))
        o = SA.sparse_attn_chunked(q, kvcat, W.sinks, idx, 512 ** -0.5, chunk=16)
        NR.rope_at(o, torch.from_numpy(pos), f, inverse=True)
        t_q = time.perf_counter() - t0
        per_token = t_comp / 4096 + t_q / nq   # seconds of one prefill token: its compressor share + one query
        return (t_comp + t_q) / per_token, t_comp + t_q
    return run, (f"oracle port, per repetition: compressors over 4096 tokens + indexer/attention for {nq} queries at "
                 f"position 32K (the sequence's average), combined per token")


def _cpu_block_window(nseq):
    """Window-only (ratio-128) block per-token CPU cost: the oracle decode block without compression."""
    import importlib
    from oracle import layer_ref as LR
    Lm = importlib.import_module(PKG + ".layer")
    C = importlib.import_module(PKG + ".configs")
    W = _dequantized(Lm.make_attention_weights(3, dims=C.LayerDims(ratio=128), quant=True))
    g = torch.Generator().manual_seed(3)
    state = dict(pool=torch.randn(nseq * 128, 512, generator=g).to(torch.bfloat16).float(),
                 win_base=torch.arange(nseq) * 128)
    x = torch.randn(nseq, 4096, generator=g)
    pos = torch.full((nseq,), 16383, dtype=torch.int32)

    def run():
        t0 = time.perf_counter()
        LR.decode_block_ref(state, W, x, pos, ratio=128)
        return nseq, time.perf_counter() - t0
    return run, f"{nseq} token(s) of the window-only (ratio-128) block per repetition through the CPU oracle"


def _cpu_block(nseq):
    """Config 5 per-token CPU cost: the oracle decode block (dequantised int8 weights in fp32). Each
    repetition steps the same token again (same work; the state it writes is overwritten)."""
    import importlib
    from oracle import layer_ref as LR
    Lm = importlib.import_module(PKG + ".layer")
    C = importlib.import_module(PKG + ".configs")
    W = _dequantized(Lm.make_attention_weights(3, quant=True))
    case = C.make_decode_case(nseq, 16384, 512, seeds=[3 + i for i in range(nseq)], device="cpu")
    pool, win_base, comp_rows = C.decode_case_host_pool(case)
    c = case.cache
    state = dict(pool=pool.float(), win_base=win_base, comp_rows=comp_rows, k_idx=c.k_idx.clone(),
                 ring_kv=c.ring_kv.clone(), ring_score=c.ring_score.clone(), ring_k=c.ring_k_idx.clone(),
                 ring_s=c.ring_s_idx.clone())
    x = torch.randn(nseq, 4096, generator=torch.Generator().manual_seed(3))
    pos = torch.full((nseq,), 16383, dtype=torch.int32)

    def run():
        t0 = time.perf_counter()
        LR.decode_block_ref(state, W, x, pos, top_k=512)
        return nseq, time.perf_counter() - t0
    return run, f"{nseq} token(s) of the config-5 block per repetition through the CPU oracle"


def run_reference(args):
    """The reference arm: the reference's own CPU implementation of the path (its ref_torch code as
    restated in oracle/, since the reference cannot be installed as a package) on all host cores,
    on this config's workload. Rank 0 alone runs it; each step is a bounded sample of at least
    CPU_MIN_SECONDS of timed work."""
    world, rank, _ = _dist()
    if rank != 0:
        return
    cfgd = CONFIGS[args.config]
    threads = _cpu_threads()
    run, desc = cpu_workload(args.config, cpu_sample_size(args.config))
    warm = max(1, min(args.warmup, 3))
    for _ in range(warm):
        run()
    per_step, reps_total, sec_total = [], 0, 0.0
    for _ in range(min(args.steps, 3)):
        v, reps, sec = timed_rate(run)
        per_step.append(v)
        reps_total, sec_total = reps_total + reps, sec_total + sec
    v = statistics.median(per_step)
    desc = f"{desc}; {reps_total} repetitions over {len(per_step)} steps, {sec_total:.1f} s of timed CPU work"
    line = {"impl": "reference", "metric": METRICS[args.config],
            "value": v, "unit": "tok/s", "n_gpus": args.gpus, "steps": len(per_step), "warmup": warm,
            "ms_per_step": 1000.0 * (cfgd["ctx"] if args.config == "c4" else cfgd["batch"]) / v,
            "higher_is_better": True, "scaling": "strong" if cfgd.get("strong") or args.config == "c4" else "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": cfgd["workload"], "global_batch": cfgd["batch"], "ctx": cfgd["ctx"],
                       "parallelism": "cpu"},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": desc + "; the reference's ref_torch path restated in oracle/"},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------ GPU leg
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--impl", default="dsv4", choices=["dsv4", "reference"])
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS))
    ap.add_argument("--replicas", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kernel-case", default=None,
                    choices=["attn_prefill", "indexer_prefill", "block_decode", "block_decode_window", "hc"],
                    help="profiling aid: run one prefill kernel alone on a 4096-query slice of config 4 "
                         "(positions 60000..64095), or config 5's block step eagerly inside an NVTX range "
                         "(block_decode; block_decode_window: the same block at a ratio-128 layer), and print its "
                         "CUDA-event time; not a bench line")
    args = ap.parse_args()
    if args.kernel_case:
        return run_kernel_case(args)
    args.steps_given, args.warmup_given = args.steps is not None, args.warmup is not None
    if args.steps is None:
        args.steps = 2400
    if args.warmup is None:
        args.warmup = 240
    if args.impl == "reference":
        return run_reference(args)

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    dsv4 = _pkg()
    C = __import__("importlib").import_module(PKG + ".configs")
    cfgd = CONFIGS[args.config]
    if args.config == "c4":
        return bench_prefill(args, world, rank, local, dev)
    if args.config == "c5":
        return bench_block(args, world, rank, local, dev)
    if args.config == "c5w":
        return bench_block_window(args, world, rank, local, dev)
    batch, ctx, top_k = cfgd["batch"], cfgd["ctx"], cfgd["top_k"]
    if cfgd.get("strong"):
        batch = max(1, batch // world)

    # ---- replicas of the whole decode state, rotating so that no step starts with warm L2
    seed_of = (lambda i: cfgd["seeds"](rank, rank * batch + i)) if cfgd.get("strong") else (lambda i: cfgd["seeds"](rank, i))
    probe = C.make_decode_case(batch, ctx, top_k, seeds=[seed_of(i) for i in range(batch)], device=dev)
    c = probe.cache
    footprint = (c.kv_pool.numel() * 2 + c.k_idx.numel() * 4 + c.block_table.numel() * 4)
    R = args.replicas or max(2, -(-2 * L2_BYTES // footprint) + 1)
    cases = [probe] + [C.make_decode_case(batch, ctx, top_k, seeds=[seed_of(i) + 104729 * r for i in range(batch)],
                                          device=dev)
                       for r in range(1, R)]
    runners = []
    for cs in cases:
        r = dsv4.DecodeRunner(cs.cache, cs.sink, top_k, device=dev)
        r.q.copy_(cs.q), r.q_idx.copy_(cs.q_idx), r.w_idx.copy_(cs.w_idx), r.positions.copy_(cs.positions)
        r.capture()
        runners.append(r)
    stream = runners[0].stream
    for r in runners[1:]:
        r.stream = stream
    torch.cuda.synchronize()

    # ---- one graph holding R steps (one per replica): a replay = R decode tokens
    big = torch.cuda.CUDAGraph()
    with torch.cuda.graph(big, stream=stream):
        for r in runners:
            r._body()
    torch.cuda.synchronize()

    def run_steps(k):
        full, rest = divmod(k, R)
        with torch.cuda.stream(stream):
            for _ in range(full):
                big.replay()
            for i in range(rest):
                runners[i].graph.replay()

    run_steps(max(args.warmup, 3))
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.05)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record(stream)
    run_steps(args.steps)
    e1.record(stream)
    sampler.sample_while(e1)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    if world > 1:
        torch.distributed.barrier()
    ms = e0.elapsed_time(e1)
    ms = _barrier_max(ms, world, dev)
    sampler.stop()
    clocks = sampler.summary(t0, t1)
    ms_per_step = ms / args.steps
    value = world * batch * args.steps / (ms / 1000.0)

    # ---- e2e through the public host API: each step copies the token's inputs from pinned host
    # memory (the runner's host_inputs(), written once per replica here as a serving loop writes
    # each token's), runs the kernels and copies the output back, as one graph launch
    hin = []
    for r, cs in zip(runners, cases):
        for dst, key in zip(r.host_inputs(), ("q", "q_idx", "w_idx", "positions")):
            dst.copy_(cs.host[key])
        hin.append(r.host_inputs())
    for i in range(min(R, 4)):
        runners[i].step_host(*hin[i])
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for s in range(args.steps):
        i = s % R
        runners[i].step_host(*hin[i])
    f1.record(stream)
    torch.cuda.synchronize()
    ems = _barrier_max(f0.elapsed_time(f1), world, dev)
    e2e = {"value": world * batch * args.steps / (ems / 1000.0), "unit": "tok/s",
           "h2d_bytes_per_step": runners[0].h2d_bytes(), "d2h_bytes_per_step": runners[0].d2h_bytes(),
           "path": "DecodeRunner.step_host (pinned host in/out, copies and kernels in one CUDA graph)"}

    # ---- dominant-kernel timing: each kernel of the step, alone, over the replica rotation
    kern = kernel_times(dsv4, cases, runners, stream, dev, min(args.steps, 4 * R))
    peak, peak_kind = _peaks()
    top = max(kern, key=lambda k: kern[k]["us"])
    kb = kern[top]
    achieved = kb["bytes"] / (kb["us"] * 1e-6) / 1e9
    roofline = {"bound": "hbm", "kernel": top, "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "peak_source": peak_kind, "traffic": None,
                "per_kernel_us": {k: round(v["us"], 3) for k, v in kern.items()},
                "algorithmic_bytes_per_launch": kb["bytes"]}
    roofline["traffic"] = TRAFFIC.get(args.config, {}).get(top)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores, desc = cpu_reference(args.config, 1 if args.config == "c2" else 2)
        cpu = {"value": v, "unit": "tok/s", "cores": cores, "kind": "port", "sample": desc}

    if rank == 0:
        line = {"metric": METRICS[args.config],
                "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": ms_per_step, "higher_is_better": True,
                "scaling": "strong" if cfgd.get("strong") else "weak", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic",
                "config": {"workload": cfgd["workload"], "global_batch": batch * world, "ctx": ctx, "top_k": top_k,
                           "parallelism": f"batch-split x{world} (no collective)" if world > 1 else "single GPU",
                           "l2": f"inputs rotate over {R} replicas x {footprint / 2**20:.1f} MiB = "
                                 f"{R * footprint / 2**20:.0f} MiB > L2 (126 MB)",
                           "cuda_graph": True},
                "gpu_launches": decode_launches_per_step(runners[0]) * args.steps,
                "e2e": e2e, "roofline": roofline, "cpu_baseline": cpu, "clocks": clocks}
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


# ------------------------------------------------------------------------------ config 4 (long prefill)
def _phase_events(n):
    return [torch.cuda.Event(enable_timing=True) for _ in range(n)]


def bench_prefill(args, world, rank, local, dev):
    """Config 4: one step = the sparse-MLA prefill core over 65536 tokens (strong scaling: the
    same sequence split over the ranks; the compressed cache is all-gathered)."""
    import importlib
    P = importlib.import_module(PKG + ".prefill")
    Lm = importlib.import_module(PKG + ".layer")
    cfgd = CONFIGS["c4"]
    s, top_k = cfgd["ctx"], cfgd["top_k"]
    steps = args.steps if args.steps_given else 5
    warmup = max(3, args.warmup if args.warmup_given else 3)
    W = Lm.make_attention_weights(2).to(dev)
    cw = P.CompressorWeights.from_attention_weights(W)
    g = torch.Generator(device=dev).manual_seed(2)
    x = torch.randn(s, 4096, device=dev, generator=g).to(torch.bfloat16)
    q = torch.randn(s, 64, 512, device=dev, generator=g).to(torch.bfloat16)
    kv = torch.randn(s, 512, device=dev, generator=g).to(torch.bfloat16)
    qi = torch.randn(s, 64, 128, device=dev, generator=g)
    wi = torch.randn(s, 64, device=dev, generator=g) / 8
    sharded = P.ShardedPrefill() if world > 1 else None
    ranges = P.zigzag_ranges(s, world, rank) if world > 1 else [(0, s)]
    g0, g1 = P.block_range(s // 4, world, rank)
    phases = {"compress": 0.0, "gather": 0.0, "indexer+attention": 0.0}

    def step(record=False):
        ev = _phase_events(4) if record else None
        if ev:
            ev[0].record()
        comp_l, keys_l = P.compress_range(x, cw, g0, g1)
        if ev:
            ev[1].record()
        if sharded is not None:
            comp, keys = sharded.gather_cache(comp_l, keys_l, s // 4)
        else:
            comp, keys = comp_l, keys_l
        if ev:
            ev[2].record()
        outs = [P.attend_queries(q[a:b], qi[a:b], wi[a:b], kv, comp, keys, W.sinks, a, b, top_k, 8192)
                for a, b in ranges]
        if ev:
            ev[3].record()
        return outs, ev

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.05)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    sampler.sample_while(e1)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    if world > 1:
        torch.distributed.barrier()
    ms = _barrier_max(e0.elapsed_time(e1), world, dev) / steps
    sampler.stop()
    clocks = sampler.summary(t0, t1)
    _, ev = step(record=True)
    torch.cuda.synchronize()
    phases = {"compress": ev[0].elapsed_time(ev[1]), "gather": ev[1].elapsed_time(ev[2]),
              "indexer+attention": ev[2].elapsed_time(ev[3])}
    # attention-only timing on this rank's queries for the tensor roofline (indices precomputed)
    att_ms, att_flops = _prefill_attention_time(P, x, q, qi, wi, kv, W, cw, ranges, s, top_k, dev)
    peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(ROOT, "MEASURED_PEAKS.json")) else {"bf16_tflops": 1590.0}
    achieved = att_flops / (att_ms * 1e-3) / 1e12
    roofline = {"bound": "tensor", "kernel": "tc::attn_tc_kernel", "achieved": achieved,
                "peak": peaks["bf16_tflops"], "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
                "peak_source": "measured" if "when" in peaks else "fallback",
                "traffic": TRAFFIC["c4"]["tc::attn_tc_kernel"] // world,  # this rank's queries
                "algorithmic_flops_per_launch": att_flops, "phases_ms": phases}
    # e2e: this rank's inputs from pinned host memory, the step, its outputs back
    hx = x.cpu().pin_memory()
    hq = [q[a:b].cpu().pin_memory() for a, b in ranges]
    hqi = [qi[a:b].cpu().pin_memory() for a, b in ranges]
    hw = [wi[a:b].cpu().pin_memory() for a, b in ranges]
    hkv = kv.cpu().pin_memory()
    ho = [torch.empty((b - a, 64, 512), dtype=torch.bfloat16).pin_memory() for a, b in ranges]
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    h2d = d2h = 0
    for _ in range(steps):
        x.copy_(hx, non_blocking=True)
        kv.copy_(hkv, non_blocking=True)
        h2d = hx.numel() * 2 + hkv.numel() * 2
        for i, (a, b) in enumerate(ranges):
            q[a:b].copy_(hq[i], non_blocking=True)
            qi[a:b].copy_(hqi[i], non_blocking=True)
            wi[a:b].copy_(hw[i], non_blocking=True)
            h2d += hq[i].numel() * 2 + hqi[i].numel() * 4 + hw[i].numel() * 4
        outs, _ = step()
        d2h = 0
        for i, o in enumerate(outs):
            ho[i].copy_(o, non_blocking=True)
            d2h += o.numel() * 2
    f1.record()
    torch.cuda.synchronize()
    ems = _barrier_max(f0.elapsed_time(f1), world, dev) / steps
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores, desc = cpu_reference("c4", cpu_sample_size("c4"))
        cpu = {"value": v, "unit": "tok/s", "cores": cores, "kind": "port", "sample": desc}
    if rank == 0:
        line = {"metric": METRICS["c4"], "value": s / (ms / 1000.0), "unit": "tok/s", "n_gpus": world,
                "steps": steps, "warmup": warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": cfgd["workload"], "global_batch": 1, "seq_len": s, "top_k": top_k,
                           "parallelism": f"query-sharded x{world} (zig-zag) + NCCL all-gather" if world > 1
                           else "single GPU", "l2": "inputs (~7 GB) larger than L2"},
                "gpu_launches": None,
                "e2e": {"value": s / (ems / 1000.0), "unit": "tok/s", "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": d2h, "path": "host inputs -> prefill core -> host outputs"},
                "roofline": roofline, "cpu_baseline": cpu, "clocks": clocks}
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def _prefill_attention_time(P, x, q, qi, wi, kv, W, cw, ranges, s, top_k, dev):
    """CUDA-event time of the sparse attention kernels alone over this rank's queries (index lists
    built beforehand). FLOPs = sum over queries of 64 heads x valid rows x 512 x 4 (QK^T and PV)."""
    import importlib
    IX = importlib.import_module(PKG + ".indexer")
    SA = importlib.import_module(PKG + ".sparse_attn")
    NRm = importlib.import_module(PKG + ".norm_rope")
    comp, keys = P.compress_range(x, cw, 0, s // 4)
    kvcat = torch.cat([kv, comp])
    freqs = NRm.rope_freqs(64, dev)
    win_base = torch.zeros(1, dtype=torch.int64, device=dev)
    chunks = []
    for a, b in ranges:
        for c0 in range(a, b, 8192):
            c1 = min(b, c0 + 8192)
            pos = torch.arange(c0, c1, dtype=torch.int32, device=dev)
            idx = torch.empty((1, c1 - c0, 128 + top_k), dtype=torch.int32, device=dev)
            IX.indexer_topk_into(idx, qi[c0:c1][None], wi[c0:c1][None], keys[None], top_k, positions=pos[None],
                                 ratio=4, out_col=128, out_offset=s, win_base=win_base, window=128, window_linear=True)
            chunks.append((c0, c1, pos, idx[0]))
    flops = 0
    for c0, c1, _, _ in chunks:
        t = torch.arange(c0, c1, dtype=torch.int64)
        rows = torch.clamp(t + 1, max=128) + torch.clamp((t + 1) // 4, max=top_k)
        flops += int(rows.sum()) * 64 * 512 * 4
    for c0, c1, pos, idx in chunks:  # warm-up
        SA.sparse_attn_rope(q[c0:c1], kvcat, W.sinks, idx, 512 ** -0.5, pos, freqs, 64)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for c0, c1, pos, idx in chunks:
        SA.sparse_attn_rope(q[c0:c1], kvcat, W.sinks, idx, 512 ** -0.5, pos, freqs, 64)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1), flops


# ------------------------------------------------------------------------------ config 5 (decode block)
def bench_block(args, world, rank, local, dev):
    """Config 5: one step = the whole attention block for one token of each sequence (global batch
    32 split over the ranks), int8-g64 weights, captured in a CUDA graph."""
    import importlib
    Lm = importlib.import_module(PKG + ".layer")
    C = importlib.import_module(PKG + ".configs")
    M = importlib.import_module(PKG + ".mla")
    cfgd = CONFIGS["c5"]
    B, ctx, top_k = max(1, cfgd["batch"] // world), cfgd["ctx"], cfgd["top_k"]
    steps = args.steps if args.steps_given else 200
    warmup = max(3, args.warmup if args.warmup_given else 20)
    W = Lm.make_attention_weights(3, quant=True).to(dev)
    case = C.make_decode_case(B, ctx, top_k, seeds=[cfgd["seeds"](rank, rank * B + i) for i in range(B)], device=dev)
    blk = Lm.DecodeBlock(W, B, ctx, top_k=top_k, cache=case.cache)
    g = torch.Generator().manual_seed(3 + rank)
    x = torch.randn(B, 4096, generator=g).to(dev)
    pos = torch.full((B,), ctx - 1, dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        blk.step(x, pos)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        out = blk.step(x, pos)
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            graph.replay()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.05)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(steps):
            graph.replay()
    e1.record(stream)
    sampler.sample_while(e1)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    if world > 1:
        torch.distributed.barrier()
    ms = _barrier_max(e0.elapsed_time(e1), world, dev) / steps
    sampler.stop()
    clocks = sampler.summary(t0, t1)
    # e2e: this token's hidden states from pinned host memory, the graph, the block output back
    hx = x.cpu().pin_memory()
    ho = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(steps):
            x.copy_(hx, non_blocking=True)
            graph.replay()
            ho.copy_(out, non_blocking=True)
    f1.record(stream)
    torch.cuda.synchronize()
    ems = _barrier_max(f0.elapsed_time(f1), world, dev) / steps
    # algorithmic HBM bytes of one step: every weight once, the visible indexer keys, the gathered rows
    wbytes = 0
    for name in Lm.MATRICES:
        w = getattr(W, name)
        wbytes += (w.q.numel() + w.scale.numel() * 2) if isinstance(w, M.QuantWeight) else w.numel() * w.element_size()
    nvis = min(ctx // 4, case.cache.max_comp)
    step_bytes = wbytes + B * (nvis * 128 * 4 + (128 + top_k) * 1024)
    peak, peak_kind = _peaks()
    achieved = step_bytes / (ms * 1e-3) / 1e9
    roofline = {"bound": "hbm", "kernel": "whole block step", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "peak_source": peak_kind, "traffic": None,
                "algorithmic_bytes_per_launch": step_bytes}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores, desc = cpu_reference("c5", cpu_sample_size("c5"))
        cpu = {"value": v, "unit": "tok/s", "cores": cores, "kind": "port", "sample": desc}
    if rank == 0:
        line = {"metric": METRICS["c5"], "value": cfgd["batch"] / (ms / 1000.0), "unit": "tok/s", "n_gpus": world,
                "steps": steps, "warmup": warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": cfgd["workload"], "global_batch": cfgd["batch"], "ctx": ctx, "top_k": top_k,
                           "parallelism": f"batch-split x{world} (no collective)" if world > 1 else "single GPU",
                           "l2": f"weights + caches {step_bytes / 2**20:.0f} MiB per step > L2", "cuda_graph": True},
                "gpu_launches": None,
                "e2e": {"value": cfgd["batch"] / (ems / 1000.0), "unit": "tok/s", "h2d_bytes_per_step": hx.numel() * 4,
                        "d2h_bytes_per_step": ho.numel() * 4, "path": "host hidden states -> block graph -> host"},
                "roofline": roofline, "cpu_baseline": cpu, "clocks": clocks}
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def bench_block_window(args, world, rank, local, dev):
    """The config-5 block at a window-only (ratio-128) layer: one step = projections, this token's kv
    row into its window ring, attention over the 128-row window, grouped output projection, for one
    token of each sequence (global batch 32 split over the ranks), int8-g64 weights, one CUDA graph
    per replica. A replica's weights and rings (~114 MB) fit in L2, so the steps rotate over three
    replicas: a step's inputs were last touched two steps (~228 MB of other data) earlier."""
    import importlib
    Lm = importlib.import_module(PKG + ".layer")
    C = importlib.import_module(PKG + ".configs")
    M = importlib.import_module(PKG + ".mla")
    cfgd = CONFIGS["c5w"]
    dims = C.LayerDims(ratio=128)
    B, ctx = max(1, cfgd["batch"] // world), cfgd["ctx"]
    steps = args.steps if args.steps_given else 300
    warmup = max(3, args.warmup if args.warmup_given else 30)
    R = 3
    stream = torch.cuda.Stream(dev)
    blocks, graphs, xs, outs, Ws = [], [], [], [], []
    for r in range(R):
        W = Lm.make_attention_weights(3 + 7 * r, dims=dims, quant=True).to(dev)
        blk = Lm.DecodeBlock(W, B, ctx, dims=dims, device=dev)
        g = torch.Generator().manual_seed(cfgd["seeds"](rank, rank * B) + 104729 * r)
        blk.cache.kv_pool.copy_(torch.randn(blk.cache.kv_pool.shape, generator=g).to(torch.bfloat16))
        x = torch.randn(B, 4096, generator=g).to(dev)
        pos = torch.full((B,), ctx - 1, dtype=torch.int32, device=dev)
        with torch.cuda.stream(stream):
            blk.step(x, pos)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            out = blk.step(x, pos)
        blocks.append(blk), graphs.append(graph), xs.append(x), outs.append(out), Ws.append(W)
    with torch.cuda.stream(stream):
        for i in range(warmup):
            graphs[i % R].replay()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.05)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record(stream)
    with torch.cuda.stream(stream):
        for i in range(steps):
            graphs[i % R].replay()
    e1.record(stream)
    sampler.sample_while(e1)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    if world > 1:
        torch.distributed.barrier()
    ms = _barrier_max(e0.elapsed_time(e1), world, dev) / steps
    sampler.stop()
    clocks = sampler.summary(t0, t1)
    # e2e: this token's hidden states from pinned host memory, the graph, the block output back
    hx = [x.cpu().pin_memory() for x in xs]
    ho = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in outs]
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    with torch.cuda.stream(stream):
        for i in range(steps):
            r = i % R
            xs[r].copy_(hx[r], non_blocking=True)
            graphs[r].replay()
            ho[r].copy_(outs[r], non_blocking=True)
    f1.record(stream)
    torch.cuda.synchronize()
    ems = _barrier_max(f0.elapsed_time(f1), world, dev) / steps
    # algorithmic HBM bytes of one step: the five matrices the step reads, once, and the window rows
    W = Ws[0]
    wbytes = 0
    for name in ("wq_a", "wq_b", "wkv", "wo_a", "wo_b"):
        w = getattr(W, name)
        wbytes += (w.q.numel() + w.scale.numel() * 2) if isinstance(w, M.QuantWeight) else w.numel() * w.element_size()
    step_bytes = wbytes + B * 128 * 1024
    peak, peak_kind = _peaks()
    achieved = step_bytes / (ms * 1e-3) / 1e9
    roofline = {"bound": "hbm", "kernel": "whole block step", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "peak_source": peak_kind, "traffic": None,
                "algorithmic_bytes_per_launch": step_bytes}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores, desc = cpu_reference("c5w", cpu_sample_size("c5w"))
        cpu = {"value": v, "unit": "tok/s", "cores": cores, "kind": "port", "sample": desc}
    if rank == 0:
        line = {"metric": METRICS["c5w"], "value": cfgd["batch"] / (ms / 1000.0), "unit": "tok/s", "n_gpus": world,
                "steps": steps, "warmup": warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": cfgd["workload"], "global_batch": cfgd["batch"], "ctx": ctx,
                           "parallelism": f"batch-split x{world} (no collective)" if world > 1 else "single GPU",
                           "l2": f"{R} replicas of {step_bytes / 2**20:.0f} MiB rotated (> L2 between uses)",
                           "cuda_graph": True},
                "gpu_launches": None,
                "e2e": {"value": cfgd["batch"] / (ems / 1000.0), "unit": "tok/s", "h2d_bytes_per_step": hx[0].numel() * 4,
                        "d2h_bytes_per_step": ho[0].numel() * 4, "path": "host hidden states -> block graph -> host"},
                "roofline": roofline, "cpu_baseline": cpu, "clocks": clocks}
        print(json.dumps(line), flush=True)
    del graphs
    if world > 1:
        torch.distributed.destroy_process_group()


def decode_launches_per_step(runner):
    """Kernels one decode step launches: q's norm + RoPE, the indexer's scores (or its tensor-core
    filter), the top-k selection, sparse attention, and the split merge when the attention plan
    writes split partials. The plan writes them exactly when its workspace is non-zero; splits merged
    inside a thread-block cluster need none."""
    import ctypes
    import importlib
    L = importlib.import_module(PKG + "._lib")
    SA = importlib.import_module(PKG + ".sparse_attn")
    c = runner.cache
    qr = torch.empty((c.batch, 64, c.head_dim), dtype=torch.bfloat16, device=runner.idx.device)
    out = torch.empty(qr.shape, dtype=runner.out_dtype, device=qr.device)
    p = SA._attn_params(qr, c.kv_pool, runner.sink, runner.idx, out, c.head_dim ** -0.5, runner.freqs,
                        runner.positions, 64, win_base=c.win_base, window=c.window)
    merge = L.lib().dsv4_sparse_attn_workspace_size(ctypes.byref(p)) > 0
    return 4 + int(merge)


def kernel_times(dsv4, cases, runners, stream, dev, n):
    """Average duration of each kernel of the step, launched alone n times over the replica
    rotation inside a CUDA graph and timed with CUDA events on the launching stream."""
    import importlib
    L = importlib.import_module(PKG + "._lib")
    SA = importlib.import_module(PKG + ".sparse_attn")
    IX = importlib.import_module(PKG + ".indexer")
    R = len(cases)
    b = cases[0].cache.batch
    top_k = runners[0].top_k
    freqs = runners[0].freqs
    NRm = importlib.import_module(PKG + ".norm_rope")
    qn = [NRm.norm_rope(r.q, r.positions, freqs) for r in runners]
    torch.cuda.synchronize()
    nvis = [min((int(c.host["positions"][i]) + 1) // 4, c.cache.max_comp) for c in cases[:1] for i in range(b)]
    n_keys = sum(nvis)
    funcs = {
        # score + select (which also writes the window rows): k_idx read once, indices written
        "indexer_topk": (lambda i: IX.indexer_topk_into(runners[i].idx.view(b, 1, -1), runners[i].q_idx.view(b, 1, 64, 128),
                                                        runners[i].w_idx.view(b, 1, 64), cases[i].cache.k_idx, top_k,
                                                        runners[i].positions.view(b, 1), 4, out_col=0,
                                                        out_offset=cases[i].cache.comp_base,
                                                        block_table=cases[i].cache.block_table, page=cases[i].cache.page),
                         n_keys * 128 * 4 + b * (64 * 128 * 4 + 64 * 4 + top_k * 4)),
        # attention (+ split merge): gathered rows, normed q in, o out, indices
        "sparse_attn": (lambda i: SA.sparse_attn_rope(qn[i], cases[i].cache.kv_pool, cases[i].sink, runners[i].idx,
                                                      512 ** -0.5, runners[i].positions, freqs, 64,
                                                      win_base=cases[i].cache.win_base, window=128),
                        b * ((128 + top_k) * 512 * 2 + top_k * 4 + 64 * 512 * 2 * 2)),
    }
    out = {}
    for name, (fn, nbytes) in funcs.items():
        with torch.cuda.stream(stream):
            fn(0)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(R):
                fn(i)
        reps = max(1, n // R)
        with torch.cuda.stream(stream):
            g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(reps):
                g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        out[name] = {"us": e0.elapsed_time(e1) * 1000.0 / (reps * R), "bytes": nbytes}
    return out


def run_kernel_case(args):
    """One prefill kernel on a 4096-query slice of config 4 (queries at positions 60000..64095,
    65,536 window rows + 16,384 compressed rows, top-k 1024): the case the profiles under profiles/
    were captured on. Seeded synthetic inputs; prints one JSON line with the CUDA-event time."""
    import importlib
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    SA = importlib.import_module(PKG + ".sparse_attn")
    IX = importlib.import_module(PKG + ".indexer")
    NRm = importlib.import_module(PKG + ".norm_rope")
    if args.kernel_case in ("block_decode", "block_decode_window"):
        return run_block_case(args, dev)
    if args.kernel_case == "hc":
        return run_hc_case(args, dev)
    s, nwin, ncomp, top_k = 4096, 65536, 16384, 1024
    g = torch.Generator(device=dev).manual_seed(0)
    pos = torch.arange(60000, 60000 + s, dtype=torch.int32, device=dev)
    reps = args.steps if args.steps is not None else 3
    if args.kernel_case == "attn_prefill":
        q = torch.randn(s, 64, 512, device=dev, generator=g).bfloat16()
        kvcat = torch.randn(nwin + ncomp, 512, device=dev, generator=g).bfloat16()
        sink = torch.randn(64, device=dev, generator=g)
        idx = torch.randint(nwin, nwin + ncomp, (s, top_k), device=dev, generator=g, dtype=torch.int32)
        freqs = NRm.rope_freqs(64, dev)
        wb = torch.zeros(1, dtype=torch.int64, device=dev)
        fn = lambda: SA.sparse_attn_rope(q, kvcat, sink, idx, 512 ** -0.5, pos, freqs, 64, win_base=wb, window=128,
                                         window_linear=True, kernel=2)
        work = {"flop": s * 64 * (128 + top_k) * 512 * 4}
    else:
        qi = torch.randn(1, s, 64, 128, device=dev, generator=g)
        wi = torch.randn(1, s, 64, device=dev, generator=g) / 8
        keys = torch.randn(1, ncomp, 128, device=dev, generator=g)
        out = torch.empty((1, s, top_k), dtype=torch.int32, device=dev)
        fn = lambda: IX.indexer_topk_into(out, qi, wi, keys, top_k, positions=pos[None], ratio=4, mode=2)
        work = {"visible_pairs": int(((pos.long() + 1) // 4).clamp(max=ncomp).sum())}
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    print(json.dumps({"kernel_case": args.kernel_case, "queries": s, "ms_per_call": ms, **work}), flush=True)


def run_hc_case(args, dev):
    """The hyper-connection kernels around the block (dim 4096, hc 4): hc_pre with the block's
    RMSNorm fused (bf16 output) and hc_post, at config 5's decode batch (32 tokens; x and the
    weights stay in L2 between calls) and at a 4096-token prefill slice (x 268 MB, above L2), each
    timed as one replay of a CUDA graph of `--steps` calls (default 20).
    Algorithmic bytes per call: hc_pre reads x (16 dim B per token) and fn once (1.5 MB), writes the
    bf16 norm (2 dim B per token) and post / comb; hc_post reads x and the residual (20 dim B per
    token) and writes 16 dim B per token."""
    import importlib
    H = importlib.import_module(PKG + ".hc")
    dim = 4096
    g = torch.Generator(device=dev).manual_seed(0)
    fn_w = torch.randn(24, 4 * dim, device=dev, generator=g) * 0.02
    scale = torch.rand(3, device=dev, generator=g) + 0.5
    base = torch.randn(24, device=dev, generator=g) * 0.1
    nw = (torch.rand(dim, device=dev, generator=g) + 0.5).bfloat16()
    reps = args.steps if args.steps is not None else 20
    res = {}
    for tokens in (CONFIGS["c5"]["batch"], 4096):
        x = torch.randn(tokens, 4, dim, device=dev, generator=g)
        att = torch.randn(tokens, dim, device=dev, generator=g)
        _, post, comb, _ = H.hc_pre(x, fn_w, scale, base, norm_w=nw)
        cases = {
            "hc_pre_norm": (lambda: H._hc_call(x, fn_w, scale, base, 0, nw, want_y=False),
                            tokens * (16 * dim + 2 * dim + 80) + fn_w.numel() * 4),
            "hc_post": (lambda: H.hc_post(att, x, post, comb), tokens * (36 * dim + 80)),
        }
        for name, (fn, nbytes) in cases.items():
            # `reps` calls captured in one CUDA graph: the device time without the host's launch gaps
            fn()
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for _ in range(reps):
                    fn()
            graph.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            graph.replay()
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) / reps * 1000
            res[f"{name}_t{tokens}"] = {"us_per_call": round(us, 2), "alg_bytes": nbytes,
                                        "gbs": round(nbytes / us / 1000, 1)}
    print(json.dumps({"kernel_case": "hc", "dim": dim, **res}), flush=True)


def run_block_case(args, dev):
    """Config 5's block step (batch 32, 16384-token contexts, int8-g64 weights) launched eagerly:
    three warm-up steps, then `--steps` (default 2) steps inside the NVTX range "step", so that a
    profiler can take exactly those launches (`ncu --nvtx --nvtx-include "step/"`). With
    `block_decode_window` the block is a ratio-128 (window-only) layer's."""
    import importlib
    Lm = importlib.import_module(PKG + ".layer")
    C = importlib.import_module(PKG + ".configs")
    cfgd = CONFIGS["c5"]
    B, ctx, top_k = cfgd["batch"], cfgd["ctx"], cfgd["top_k"]
    if args.kernel_case == "block_decode_window":
        dims = C.LayerDims(ratio=128)
        W = Lm.make_attention_weights(3, dims=dims, quant=True).to(dev)
        blk = Lm.DecodeBlock(W, B, ctx, dims=dims, device=dev)
        blk.cache.kv_pool.copy_(torch.randn(blk.cache.kv_pool.shape, generator=torch.Generator().manual_seed(3))
                                .to(torch.bfloat16))
    else:
        W = Lm.make_attention_weights(3, quant=True).to(dev)
        case = C.make_decode_case(B, ctx, top_k, seeds=[cfgd["seeds"](0, i) for i in range(B)], device=dev)
        blk = Lm.DecodeBlock(W, B, ctx, top_k=top_k, cache=case.cache)
    x = torch.randn(B, 4096, generator=torch.Generator().manual_seed(3)).to(dev)
    pos = torch.full((B,), ctx - 1, dtype=torch.int32, device=dev)
    for _ in range(3):
        blk.step(x, pos)
    torch.cuda.synchronize()
    reps = args.steps if args.steps is not None else 2
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("step")
    e0.record()
    for _ in range(reps):
        out = blk.step(x, pos)
    e1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    print(json.dumps({"kernel_case": args.kernel_case, "batch": B, "ctx": ctx, "eager_ms_per_step": e0.elapsed_time(e1) / reps,
                      "checksum": float(out.abs().sum())}), flush=True)


if __name__ == "__main__":
    main()
