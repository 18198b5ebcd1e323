"""Benchmark of the B200 sparse-MLA attention path.

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl dsv4|reference] [--config all|c2|c3|c4|c5|c5w]

The default run (`--config all`) prints ONE JSON line: the headline, config 2 (decode of one token
against a 32768-token context), with configs 3, 4 and 5 measured in the same process under
`"configs"`, each entry carrying its own value, ms_per_step, roofline, clocks, e2e and CPU baseline:

  c2  one decode token (batch 1, 32K context): the per-head norm + RoPE of q, the lightning-indexer
      scores + top-k 512 over 8192 compressed keys, sparse attention over the 128 window + 512
      selected rows with the inverse RoPE fused. Does not shard: N GPUs run N replicas (weak).
  c3  one decode token of each of 64 sequences (8K contexts): the same kernels, batched. The
      batch is split across the N GPUs with no collective (strong scaling).
  c4  prefill of 65,536 tokens: the KV and indexer-key compressors, the indexer top-k 1024
      (causal), sparse attention over 128 + 1024 rows. Query-sharded across N GPUs with one NCCL
      all-gather of the compressed rows and keys (strong).
  c5  the full attention block decode of 32 sequences (16K contexts, int8-g64 weights): RMSNorm,
      projections, RoPE, compressor ring, indexer, sparse MLA, grouped output projection. Batch
      split across the N GPUs with no collective (strong).

Timing: a step is one decode token (c2, c3, c5: one CUDA graph launch per step; a decode loop
cannot batch successive tokens of a sequence into one launch) or one whole prefill (c4). Inputs
resident in HBM, larger than L2 between uses (the decode steps rotate over replicas of the whole
state). W untimed warm-up steps, then `repeats` regions of exactly K steps, each bracketed by a
barrier + synchronize and timed with CUDA events on the launching stream, max over ranks; the
reported ms_per_step is the median region / K. `e2e` is the same K steps through the public host
API (pinned host inputs copied in, the step, the result copied out, every step). SM clocks and
throttle reasons are sampled through NVML during the timed regions (reading only).
"""
import argparse
import ctypes
import gc
import json
import os
import statistics
import sys
import threading
import time

import numpy as np
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
    "c4": dict(batch=1, ctx=65536, top_k=1024, seeds=lambda r, i: 2, strong=True,
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
ALL = ("c2", "c3", "c4", "c5")
# steps of a sub-config region when the headline's K is larger (c4 steps are whole prefills)
SUB_STEPS = {"c2": 200, "c3": 100, "c4": 5, "c5": 100, "c5w": 100}
REPEATS = {"c2": 15, "c3": 9, "c4": 3, "c5": 9, "c5w": 9}
L2_BYTES = 126 * 1024 * 1024
L2_NOTE = {
    "c2": "inputs > L2 between uses: steps rotate over replicas of the whole decode state (> 2x L2 in total)",
    "c3": "inputs > L2 between uses: steps rotate over replicas of the whole decode state (> 2x L2 in total)",
    "c4": "inputs (~7 GB) larger than L2",
    "c5": "weights + caches read per step (~230 MB) larger than L2",
    "c5w": "steps rotate over 3 replicas of weights + windows (> 2x L2 between uses)",
}

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the dominant op, from one
# ncu capture each on B200: config 2 on this bench's own command (score + select kernels of one
# step); config 4 on `--kernel-case attn_prefill` (4,096 of the 65,536 queries, every query with
# 1,152 list entries), scaled by 16 to the step's eight 8,192-query launches.
TRAFFIC = {"c2": {"indexer_topk": 4319744, "sparse_attn": 777216},
           "c4": {"tc::attn_tc_kernel": 16 * 545708288}}


def _pkg():
    import importlib
    return importlib.import_module(PKG)


def _mod(name):
    import importlib
    return importlib.import_module(PKG + "." + name)


def _peaks():
    """(hbm GB/s, bf16 TFLOP/s burst, bf16 TFLOP/s sustained, source)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return (float(p["hbm_gbs"]), float(p["bf16_tflops"]),
                float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "measured")
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


def config_dict(name, world):
    """The workload description shared by both arms (the reference arm prints the same dict)."""
    c = CONFIGS[name]
    if name == "c2":
        par = f"replicas x{world} (batch 1 does not shard)" if world > 1 else "single GPU"
        gb = world
    elif name == "c4":
        par = f"query-sharded x{world} (zig-zag) + NCCL all-gather of compressed KV and keys" if world > 1 \
            else "single GPU"
        gb = 1
    else:
        par = f"batch-split x{world} (no collective)" if world > 1 else "single GPU"
        gb = c["batch"]
    d = {"workload": c["workload"], "global_batch": gb, "ctx": c["ctx"], "parallelism": par, "l2": L2_NOTE[name]}
    if c["top_k"]:
        d["top_k"] = c["top_k"]
    return d


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML every ~10 ms (reading only)."""

    NAMES = {0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
             0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device_index):
        self.samples, self.reasons, self.ok = [], set(), False
        self.windows = []
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

    def summary(self, t0=None, t1=None, windows=None):
        """Median SM clock and the union of throttle reasons over the samples inside the timed
        windows ([(t0, t1)], or the single window t0..t1); all samples if none fell inside."""
        windows = windows if windows is not None else [(t0, t1)]
        inside = [s for s in self.samples if any(a <= s[0] <= b for a, b in windows)]
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


def _barrier(world):
    if world > 1:
        torch.distributed.barrier()


class Env:
    """Per-process run context: ranks, device, step counts of the headline."""

    def __init__(self, args, world, rank, local, dev):
        self.args, self.world, self.rank, self.local, self.dev = args, world, rank, local, dev

    def steps_for(self, name, headline):
        a = self.args
        if headline and a.steps_given:
            return a.steps
        if a.steps_given:
            return min(a.steps, SUB_STEPS[name]) if name == "c4" else a.steps
        return SUB_STEPS[name]

    def warmup_for(self, name, headline):
        a = self.args
        w = a.warmup if a.warmup_given else (3 if name == "c4" else 20)
        return max(3, w)

    def repeats_for(self, name):
        return self.args.repeats or REPEATS[name]


def timed_regions(env, stream, run_k, k, repeats, sampler):
    """`repeats` regions of exactly k steps each: barrier + synchronize, CUDA events on `stream`
    around run_k(k), synchronize + barrier; per-region ms as the max over ranks. Returns
    (list of ms, wall windows for the clock summary)."""
    out, windows = [], []
    for _ in range(repeats):
        _barrier(env.world)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        e0.record(stream)
        run_k(k)
        e1.record(stream)
        sampler.sample_while(e1)
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        _barrier(env.world)
        out.append(_barrier_max(e0.elapsed_time(e1), env.world, env.dev))
        windows.append((t0, t1))
    return out, windows


def timing_summary(ms_list, k):
    return {"repeats": len(ms_list), "steps_per_region": k,
            "region_ms": [round(m, 4) for m in ms_list],
            "ms_per_step_min": min(ms_list) / k, "ms_per_step_max": max(ms_list) / k}


# ------------------------------------------------------------------------------ graph launch counts
_cuda_drv = None


def _drv():
    global _cuda_drv
    if _cuda_drv is None:
        _cuda_drv = ctypes.CDLL("libcuda.so.1")
    return _cuda_drv


def graph_kernel_nodes(graph):
    """(kernel nodes, of which this library's) in a captured torch CUDAGraph (keep_graph=True), read
    through the driver API: cuGraphGetNodes / cuGraphNodeGetType and, for the names, the kernel
    node's function (cuGraphKernelNodeGetParams, cuFuncGetName). Returns (None, None) when the
    driver does not answer."""
    try:
        d = _drv()
        g = ctypes.c_void_p(graph.raw_cuda_graph())
        n = ctypes.c_size_t(0)
        if d.cuGraphGetNodes(g, None, ctypes.byref(n)) != 0:
            return None, None
        nodes = (ctypes.c_void_p * n.value)()
        if d.cuGraphGetNodes(g, nodes, ctypes.byref(n)) != 0:
            return None, None
        kernels, ours = 0, 0

        class KParams(ctypes.Structure):  # CUDA_KERNEL_NODE_PARAMS_v2
            _fields_ = [("func", ctypes.c_void_p), ("gx", ctypes.c_uint), ("gy", ctypes.c_uint),
                        ("gz", ctypes.c_uint), ("bx", ctypes.c_uint), ("by", ctypes.c_uint), ("bz", ctypes.c_uint),
                        ("smem", ctypes.c_uint), ("params", ctypes.c_void_p), ("extra", ctypes.c_void_p),
                        ("kern", ctypes.c_void_p), ("ctx", ctypes.c_void_p)]
        named = 0
        for i in range(n.value):
            t = ctypes.c_int(-1)
            d.cuGraphNodeGetType(ctypes.c_void_p(nodes[i]), ctypes.byref(t))
            if t.value != 0:   # CU_GRAPH_NODE_TYPE_KERNEL
                continue
            kernels += 1
            kp = KParams()
            name = ctypes.c_char_p()
            try:
                if d.cuGraphKernelNodeGetParams_v2(ctypes.c_void_p(nodes[i]), ctypes.byref(kp)) == 0 and kp.func and \
                        d.cuFuncGetName(ctypes.byref(name), ctypes.c_void_p(kp.func)) == 0 and name.value:
                    named += 1
                    if name.value.startswith(b"_ZN4dsv4"):   # every kernel of libdsv4.so is in namespace dsv4
                        ours += 1
            except Exception:
                pass
        return kernels, (ours if named == kernels else None)
    except Exception:
        return None, None


def _count_launches(graph, steps_per_graph=1):
    k, ours = graph_kernel_nodes(graph)
    if k is None:
        return None
    per = (ours if ours is not None else k) / steps_per_graph
    return per


# ------------------------------------------------------------------------------ CPU reference leg
CPU_MIN_SECONDS = 10.0  # timed CPU work per reported number (a bounded sample of the workload)
CPU_SUB_SECONDS = 5.0   # the same for the configs reported beside the headline


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
    C = _mod("configs")
    f = NR.precompute_freqs(64, 0, 65536, 160000.0, 16, 32, 1)
    batch = samples
    case = C.make_decode_case(batch, cfgd["ctx"], cfgd["top_k"], seeds=[cfgd["seeds"](i, i) for i in range(batch)],
                              device="cpu", shuffle_pages=True)
    pool, win_base, comp_rows = C.decode_case_host_pool(case)
    h = case.host

    def run():
        t0 = time.perf_counter()
        LR.decode_attention_ref(pool, win_base, comp_rows, h["k_idx"], h["q"], h["q_idx"], h["w_idx"], h["sink"],
                                h["positions"], cfgd["top_k"], f)
        return batch, time.perf_counter() - t0
    return run, f"{batch} decode token(s) of {cfg_name} per repetition through the CPU oracle"


def cpu_sample_size(cfg_name, world=1):
    """Tokens per repetition of the CPU sample: config 2 runs the arm's global batch (one sequence
    per GPU replica), the block configs their batch of 32 per call (the weights are read once per
    call, as a CPU implementation would), config 4 runs 64 queries, config 3 two sequences (the
    oracle loops over sequences, so tok/s does not depend on the sample's batch)."""
    return {"c2": world, "c3": 2, "c4": 64, "c5": 32, "c5w": 32}[cfg_name]


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


def _cpu_baseline(env, name, headline):
    if env.rank != 0 or env.world != 1 or env.args.no_cpu_baseline:
        return None
    v, cores, desc = cpu_reference(name, cpu_sample_size(name), min_seconds=CPU_MIN_SECONDS if headline
                                   else CPU_SUB_SECONDS)
    return {"value": v, "unit": "tok/s", "cores": cores, "kind": "port", "sample": desc}


def _cpu_prefill(nq):
    """Config 4 per-token CPU cost: the two compressors over a 4096-token slice (per token), plus
    the indexer over 16384 keys and attention over 1152 rows for nq queries in the middle of the
    65536-token sequence (per query)."""
    from oracle import compressor_ref as CR
    from oracle import indexer_ref as I
    from oracle import norm_rope_ref as NR
    from oracle import sparse_attn_ref as SA
    Lm = _mod("layer")
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
    from oracle import layer_ref as LR
    Lm, C = _mod("layer"), _mod("configs")
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
    from oracle import layer_ref as LR
    Lm, C = _mod("layer"), _mod("configs")
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


def _tokens_per_step(name, world):
    c = CONFIGS[name]
    if name == "c2":
        return world
    if name == "c4":
        return c["ctx"]
    return c["batch"]


def reference_line(name, steps, warmup, world, per_step_seconds):
    """One config through the reference's CPU path (its ref_torch code as restated in oracle/) on all
    host cores: `warmup` untimed repetitions, then `steps` timed steps, each a bounded sample of at
    least per_step_seconds of CPU work."""
    threads = _cpu_threads()
    run, desc = cpu_workload(name, cpu_sample_size(name, world))
    for _ in range(max(1, warmup)):
        run()
    per_step, reps_total, sec_total = [], 0, 0.0
    for _ in range(steps):
        v, reps, sec = timed_rate(run, per_step_seconds)
        per_step.append(v)
        reps_total, sec_total = reps_total + reps, sec_total + sec
    v = statistics.median(per_step)
    desc = f"{desc}; {reps_total} repetitions over {steps} steps, {sec_total:.1f} s of timed CPU work"
    return {"impl": "reference", "metric": METRICS[name],
            "value": v, "unit": "tok/s", "n_gpus": world, "steps": steps, "warmup": max(1, warmup),
            "ms_per_step": 1000.0 * _tokens_per_step(name, world) / v,
            "higher_is_better": True, "scaling": "weak" if name == "c2" else "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_dict(name, world),
            "execution": f"CPU, {threads} host threads (rank 0 of {world})",
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": desc + "; the reference's ref_torch path restated in oracle/"},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_reference(args):
    """The reference arm: the reference's own CPU implementation of the path (its ref_torch code as
    restated in oracle/, since the reference cannot be installed as a package) on all host cores,
    on the same configs (same `config` dicts) as the GPU arm at this N. Rank 0 alone runs it. The
    headline runs K timed steps, each a bounded sample sized so the whole run stays within a few
    minutes; the other configs get one bounded sample each under "configs"."""
    world, rank, _ = _dist()
    if rank != 0:
        return
    names = ALL if args.config == "all" else (args.config,)
    per_step = min(CPU_MIN_SECONDS, max(0.5, 90.0 / args.steps))
    head = reference_line(names[0], args.steps, min(args.warmup, 3), world, per_step)
    if len(names) > 1:
        head["configs"] = {n: reference_line(n, 1, 1, world, CPU_SUB_SECONDS) for n in names[1:]}
    print(json.dumps(head), flush=True)


# ------------------------------------------------------------------------------ configs 2 and 3 (decode attention)
def bench_decode(env, name, headline):
    """Configs 2 and 3: a step is one decode token of every sequence of this rank's batch, one CUDA
    graph launch (q's norm + RoPE, indexer scores + top-k, sparse attention + inverse RoPE)."""
    dsv4, C = _pkg(), _mod("configs")
    cfgd = CONFIGS[name]
    world, rank, dev = env.world, env.rank, env.dev
    K, W, reps = env.steps_for(name, headline), env.warmup_for(name, headline), env.repeats_for(name)
    batch, ctx, top_k = cfgd["batch"], cfgd["ctx"], cfgd["top_k"]
    if cfgd.get("strong"):
        batch = max(1, batch // world)
    seed_of = (lambda i: cfgd["seeds"](rank, rank * batch + i)) if cfgd.get("strong") else (lambda i: cfgd["seeds"](rank, i))
    probe = C.make_decode_case(batch, ctx, top_k, seeds=[seed_of(i) for i in range(batch)], device=dev)
    c = probe.cache
    footprint = (c.kv_pool.numel() * 2 + c.k_idx.numel() * 4 + c.block_table.numel() * 4 +
                 sum(t.numel() * t.element_size() for t in c.key_image))
    R = env.args.replicas or max(2, -(-2 * L2_BYTES // footprint) + 1)
    cases = [probe] + [C.make_decode_case(batch, ctx, top_k, seeds=[seed_of(i) + 104729 * r for i in range(batch)],
                                          device=dev)
                       for r in range(1, R)]
    runners = []
    stream = torch.cuda.Stream(dev)
    for cs in cases:
        r = dsv4.DecodeRunner(cs.cache, cs.sink, top_k, device=dev, q_dtype=torch.bfloat16, stream=stream,
                              keep_graph=True)
        r.q.copy_(cs.q), r.q_idx.copy_(cs.q_idx), r.w_idx.copy_(cs.w_idx), r.positions.copy_(cs.positions)
        r.capture()
        runners.append(r)
    torch.cuda.synchronize()
    cursor = [0]

    def run_k(k):  # one graph launch per decode step, rotating over the replicas
        with torch.cuda.stream(stream):
            for _ in range(k):
                runners[cursor[0] % R].graph.replay()
                cursor[0] += 1

    run_k(max(W, 2 * R))   # at least W, and every replica's graph replayed (uploaded) before timing
    torch.cuda.synchronize()
    sampler = ClockSampler(env.local)
    sampler.start()
    time.sleep(0.05)
    ms_list, windows = timed_regions(env, stream, run_k, K, reps, sampler)
    sampler.stop()
    clocks = sampler.summary(windows=windows)
    ms_per_step = statistics.median(ms_list) / K
    value = world * batch / (ms_per_step / 1000.0)

    # ---- e2e through the public host API: each step copies the token's inputs from pinned host
    # memory (the runner's host_inputs(), written once per replica here as a serving loop writes
    # each token's), runs the kernels and copies the output back, as one graph launch
    hin = []
    for r, cs in zip(runners, cases):
        for dst, key in zip(r.host_inputs(), ("q", "q_idx", "w_idx", "positions")):
            dst.copy_(cs.host[key])
        hin.append(r.host_inputs())
    ecur = [0]

    def run_host(k):
        for _ in range(k):
            i = ecur[0] % R
            runners[i].step_host(*hin[i])
            ecur[0] += 1

    run_host(R)
    torch.cuda.synchronize()
    ems_list, _ = timed_regions(env, stream, run_host, K, reps, _NoSampler())
    ems = statistics.median(ems_list) / K
    e2e = {"value": world * batch / (ems / 1000.0), "unit": "tok/s", "ms_per_step": ems,
           "h2d_bytes_per_step": runners[0].h2d_bytes(), "d2h_bytes_per_step": runners[0].d2h_bytes(),
           "path": "DecodeRunner.step_host (pinned host in/out, q in bf16; the copies and the step in one CUDA "
                   "graph: " + ("copy kernels in, the attention's own stores out" if batch < _mod("decode").FUSED_Q_MAX_BATCH
                                else "copy-engine transfers in, q's beside the indexer; the merge kernel's own stores out") + ")"}

    # ---- dominant-kernel timing: each kernel of the step, alone, over the replica rotation
    kern = kernel_times(cases, runners, stream, min(max(K, 20), 4 * R))
    hbm, _, _, peak_kind = _peaks()
    top = max((k for k in kern if not k.startswith("alt:")), key=lambda k: kern[k]["us"])
    kb = kern[top]
    achieved = kb["bytes"] / (kb["us"] * 1e-6) / 1e9
    roofline = {"bound": "hbm", "kernel": top, "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm, "peak_source": peak_kind,
                "traffic": TRAFFIC.get(name, {}).get(top),
                "per_kernel_us": {k: round(v["us"], 3) for k, v in kern.items()},
                "algorithmic_bytes_per_launch": kb["bytes"]}
    launches = _count_launches(runners[0].graph)
    line = {"metric": METRICS[name], "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "strong" if cfgd.get("strong") else "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic", "config": config_dict(name, world),
            "timing": dict(timing_summary(ms_list, K), replicas=R, replica_mib=round(footprint / 2**20, 1),
                           graph="one CUDA graph launch per decode step"),
            "gpu_launches": None if launches is None else int(round(launches * K)),
            "gpu_launches_per_step": launches,
            "e2e": e2e, "roofline": roofline, "cpu_baseline": _cpu_baseline(env, name, headline), "clocks": clocks}
    for r in runners:
        r.release()
    return line


class _NoSampler:
    def sample_while(self, event, period=0.001):
        return


def kernel_times(cases, runners, stream, n):
    """Average duration of each op of the step, launched alone n times over the replica rotation
    inside a CUDA graph and timed with CUDA events on the launching stream."""
    SA, IX, NRm = _mod("sparse_attn"), _mod("indexer"), _mod("norm_rope")
    R = len(cases)
    b = cases[0].cache.batch
    top_k = runners[0].top_k
    freqs = runners[0].freqs
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
                                                        block_table=cases[i].cache.block_table, page=cases[i].cache.page,
                                                        key_image=cases[i].cache.key_image),
                         n_keys * 128 * 4 + b * (64 * 128 * 4 + 64 * 4 + top_k * 4)),
        # attention (+ split merge): gathered rows, normed q in, o out, indices
        "sparse_attn": (lambda i: SA.sparse_attn_rope(qn[i], cases[i].cache.kv_pool, cases[i].sink, runners[i].idx,
                                                      512 ** -0.5, runners[i].positions, freqs, 64,
                                                      win_base=cases[i].cache.win_base, window=128),
                        b * ((128 + top_k) * 512 * 2 + top_k * 4 + 64 * 512 * 2 * 2)),
    }
    # the tensor-core filter + exact band (mode 2) on the same call, for comparison (not in the step)
    funcs["alt:indexer_topk_mode2"] = (
        lambda i: IX.indexer_topk_into(runners[i].idx.view(b, 1, -1), runners[i].q_idx.view(b, 1, 64, 128),
                                       runners[i].w_idx.view(b, 1, 64), cases[i].cache.k_idx, top_k,
                                       runners[i].positions.view(b, 1), 4, out_col=0,
                                       out_offset=cases[i].cache.comp_base, block_table=cases[i].cache.block_table,
                                       page=cases[i].cache.page, key_image=cases[i].cache.key_image, mode=2),
        funcs["indexer_topk"][1])
    # the other attention kernels on the same call (kernel 1: 64-head mma.sync, 2: tcgen05, 3: head groups)
    for kern_id in (1, 2, 3):
        funcs[f"alt:sparse_attn_kernel{kern_id}"] = (
            (lambda k: lambda i: SA.sparse_attn_rope(qn[i], cases[i].cache.kv_pool, cases[i].sink, runners[i].idx,
                                                     512 ** -0.5, runners[i].positions, freqs, 64,
                                                     win_base=cases[i].cache.win_base, window=128, kernel=k))(kern_id),
            funcs["sparse_attn"][1])
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
        del g
    return out


# ------------------------------------------------------------------------------ config 4 (long prefill)
def bench_prefill(env, name, headline):
    """Config 4: one step = the sparse-MLA prefill core over 65536 tokens (strong scaling: the
    same sequence split over the ranks by query; the compressed cache is all-gathered)."""
    P, Lm = _mod("prefill"), _mod("layer")
    cfgd = CONFIGS["c4"]
    world, rank, dev = env.world, env.rank, env.dev
    s, top_k = cfgd["ctx"], cfgd["top_k"]
    K, Wm, reps = env.steps_for("c4", headline), env.warmup_for("c4", headline), env.repeats_for("c4")
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
    stream = torch.cuda.current_stream(dev)

    def step(record=False):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)] if record else None
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

    def run_k(k):
        for _ in range(k):
            step()

    run_k(Wm)
    torch.cuda.synchronize()
    sampler = ClockSampler(env.local)
    sampler.start()
    time.sleep(0.05)
    ms_list, windows = timed_regions(env, stream, run_k, K, reps, sampler)
    sampler.stop()
    clocks = sampler.summary(windows=windows)
    ms = statistics.median(ms_list) / K
    _barrier(world)
    _, ev = step(record=True)
    torch.cuda.synchronize()
    phases = {"compress": ev[0].elapsed_time(ev[1]), "gather": ev[1].elapsed_time(ev[2]),
              "indexer+attention": ev[2].elapsed_time(ev[3])}
    phases = {k: _barrier_max(v, world, dev) for k, v in phases.items()}
    # attention-only timing on this rank's queries for the tensor roofline (indices precomputed)
    att_ms, att_flops = _prefill_attention_time(P, x, q, qi, wi, kv, W, cw, ranges, s, top_k, dev)
    att_ms = _barrier_max(att_ms, world, dev)
    _, burst, sustained, src = _peaks()
    achieved = att_flops / (att_ms * 1e-3) / 1e12
    roofline = {"bound": "tensor", "kernel": "tc::attn_tc_kernel", "achieved": achieved,
                "peak": sustained, "unit": "TFLOP/s", "frac": achieved / sustained,
                "peak_source": f"{src} (bf16 sustained: the kernel runs for ~{att_ms:.0f} ms back to back)",
                "frac_of_burst": achieved / burst,
                "traffic": TRAFFIC["c4"]["tc::attn_tc_kernel"] // world,  # this rank's queries
                "algorithmic_flops_per_launch": att_flops, "attention_ms": att_ms, "phases_ms": phases}
    # e2e: this rank's inputs from pinned host memory, the step, its outputs back
    hx = x.cpu().pin_memory()
    hq = [q[a:b].cpu().pin_memory() for a, b in ranges]
    hqi = [qi[a:b].cpu().pin_memory() for a, b in ranges]
    hw = [wi[a:b].cpu().pin_memory() for a, b in ranges]
    hkv = kv.cpu().pin_memory()
    ho = [torch.empty((b - a, 64, 512), dtype=torch.bfloat16).pin_memory() for a, b in ranges]
    io = {"h2d": 0, "d2h": 0}
    staging = P.PrefillStaging(8192, dev)

    def run_host(k):
        # x and the window rows first (the compressors need x), then per 8192-query chunk the
        # inputs in and the output out on two copy streams around the compute (attend_queries_host)
        for _ in range(k):
            x.copy_(hx, non_blocking=True)
            kv.copy_(hkv, non_blocking=True)
            h2d = hx.numel() * 2 + hkv.numel() * 2
            comp_l, keys_l = P.compress_range(x, cw, g0, g1)
            if sharded is not None:
                comp, keys = sharded.gather_cache(comp_l, keys_l, s // 4)
            else:
                comp, keys = comp_l, keys_l
            d2h = 0
            for i, (a, b) in enumerate(ranges):
                P.attend_queries_host(hq[i], hqi[i], hw[i], kv, comp, keys, W.sinks, a, b, ho[i], top_k, 8192,
                                      staging)
                h2d += hq[i].numel() * 2 + hqi[i].numel() * 4 + hw[i].numel() * 4
                d2h += ho[i].numel() * 2
            io["h2d"], io["d2h"] = h2d, d2h

    ems_list, _ = timed_regions(env, stream, run_host, K, 1, _NoSampler())
    ems = ems_list[0] / K
    line = {"metric": METRICS["c4"], "value": s / (ms / 1000.0), "unit": "tok/s", "n_gpus": world,
            "steps": K, "warmup": Wm, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": config_dict("c4", world),
            "timing": dict(timing_summary(ms_list, K), graph="eager launches (chunks of 8192 queries)"),
            "gpu_launches": None,
            "e2e": {"value": s / (ems / 1000.0), "unit": "tok/s", "ms_per_step": ems, "h2d_bytes_per_step": io["h2d"],
                    "d2h_bytes_per_step": io["d2h"],
                    "path": "pinned host inputs -> prefill core -> pinned host outputs; per query chunk the copies "
                            "overlap the neighbouring chunks' compute (attend_queries_host)"},
            "roofline": roofline, "cpu_baseline": _cpu_baseline(env, "c4", headline), "clocks": clocks}
    return line


def _prefill_attention_time(P, x, q, qi, wi, kv, W, cw, ranges, s, top_k, dev):
    """CUDA-event time of the sparse attention kernels alone over this rank's queries (index lists
    built beforehand). FLOPs = sum over queries of 64 heads x valid rows x 512 x 4 (QK^T and PV)."""
    IX, SA, NRm = _mod("indexer"), _mod("sparse_attn"), _mod("norm_rope")
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
def _step_bytes_block(W, B, ctx, top_k, max_comp, names):
    M = _mod("mla")
    wbytes = 0
    for n in names:
        w = getattr(W, n)
        wbytes += (w.q.numel() + w.scale.numel() * 2) if isinstance(w, M.QuantWeight) else w.numel() * w.element_size()
    nvis = min(ctx // 4, max_comp)
    return wbytes + B * (nvis * 128 * 4 + (128 + top_k) * 1024) if top_k else wbytes + B * 128 * 1024


def bench_block(env, name, headline):
    """Config 5 (and 5w): one step = the whole attention block for one token of each sequence
    (global batch 32 split over the ranks), int8-g64 weights, one CUDA graph per step. Config 5w is
    the block of a ratio-128 (window-only) layer."""
    Lm, C = _mod("layer"), _mod("configs")
    cfgd = CONFIGS[name]
    world, rank, dev = env.world, env.rank, env.dev
    K, Wm, reps = env.steps_for(name, headline), env.warmup_for(name, headline), env.repeats_for(name)
    B, ctx, top_k = max(1, cfgd["batch"] // world), cfgd["ctx"], cfgd["top_k"]
    window_only = name == "c5w"
    stream = torch.cuda.Stream(dev)
    R = 3 if window_only else 1   # a window-only replica fits in L2: rotate three
    blocks, graphs, xs, outs, Ws = [], [], [], [], []
    for r in range(R):
        if window_only:
            dims = C.LayerDims(ratio=128)
            W = Lm.make_attention_weights(3 + 7 * r, dims=dims, quant=True).to(dev)
            blk = Lm.DecodeBlock(W, B, ctx, dims=dims, device=dev)
            g = torch.Generator().manual_seed(cfgd["seeds"](rank, rank * B) + 104729 * r)
            blk.cache.kv_pool.copy_(torch.randn(blk.cache.kv_pool.shape, generator=g).to(torch.bfloat16))
        else:
            W = Lm.make_attention_weights(3, quant=True).to(dev)
            case = C.make_decode_case(B, ctx, top_k, seeds=[cfgd["seeds"](rank, rank * B + i) for i in range(B)],
                                      device=dev)
            blk = Lm.DecodeBlock(W, B, ctx, top_k=top_k, cache=case.cache)
            g = torch.Generator().manual_seed(3 + rank)
        x = torch.randn(B, 4096, generator=g).to(dev)
        pos = torch.full((B,), ctx - 1, dtype=torch.int32, device=dev)
        with torch.cuda.stream(stream):
            blk.step(x, pos)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph(keep_graph=True)
        with torch.cuda.graph(graph, stream=stream):
            out = blk.step(x, pos)
        blocks.append(blk), graphs.append(graph), xs.append(x), outs.append(out), Ws.append(W)
    cursor = [0]

    def run_k(k):
        with torch.cuda.stream(stream):
            for _ in range(k):
                graphs[cursor[0] % R].replay()
                cursor[0] += 1

    run_k(max(Wm, 2 * R))
    torch.cuda.synchronize()
    sampler = ClockSampler(env.local)
    sampler.start()
    time.sleep(0.05)
    ms_list, windows = timed_regions(env, stream, run_k, K, reps, sampler)
    sampler.stop()
    clocks = sampler.summary(windows=windows)
    ms = statistics.median(ms_list) / K
    # e2e: through BlockRunner, one graph per token holding the copy of this token's hidden states
    # and positions in from pinned host memory, the block, and the copy of its output back
    runners = [Lm.BlockRunner(blk, stream=stream) for blk in blocks]
    for r in range(R):
        hx_r, hp_r = runners[r].host_inputs()
        hx_r.copy_(xs[r].cpu())
        hp_r.fill_(ctx - 1)
    ecur = [0]

    def run_host(k):
        for _ in range(k):
            runners[ecur[0] % R].step_host()
            ecur[0] += 1

    run_host(max(3, 2 * R))
    torch.cuda.synchronize()
    ems_list, _ = timed_regions(env, stream, run_host, K, reps, _NoSampler())
    ems = statistics.median(ems_list) / K
    names = ("wq_a", "wq_b", "wkv", "wo_a", "wo_b") if window_only else Lm.MATRICES
    max_comp = 0 if window_only else blocks[0].cache.max_comp
    step_bytes = _step_bytes_block(Ws[0], B, ctx, top_k, max_comp, names)
    hbm, _, _, peak_kind = _peaks()
    achieved = step_bytes / (ms * 1e-3) / 1e9
    roofline = {"bound": "hbm", "kernel": "whole block step", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm, "peak_source": peak_kind, "traffic": None,
                "algorithmic_bytes_per_launch": step_bytes}
    launches = _count_launches(graphs[0])
    line = {"metric": METRICS[name], "value": cfgd["batch"] / (ms / 1000.0), "unit": "tok/s", "n_gpus": world,
            "steps": K, "warmup": Wm, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": config_dict(name, world),
            "timing": dict(timing_summary(ms_list, K), replicas=R, graph="one CUDA graph launch per decode step"),
            "gpu_launches": None if launches is None else int(round(launches * K)),
            "gpu_launches_per_step": launches,
            "e2e": {"value": cfgd["batch"] / (ems / 1000.0), "unit": "tok/s", "ms_per_step": ems,
                    "h2d_bytes_per_step": runners[0].h2d_bytes(), "d2h_bytes_per_step": runners[0].d2h_bytes(),
                    "path": "pinned host hidden states + positions -> BlockRunner graph (copy kernels in and "
                            "out) -> pinned host output"},
            "roofline": roofline, "cpu_baseline": _cpu_baseline(env, name, headline), "clocks": clocks}
    for rn in runners:
        rn.release()
    del graphs
    return line


BENCH = {"c2": bench_decode, "c3": bench_decode, "c4": bench_prefill, "c5": bench_block, "c5w": bench_block}


# ------------------------------------------------------------------------------ GPU leg
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--repeats", type=int, default=0, help="timed regions of K steps per config (median reported)")
    ap.add_argument("--impl", default="dsv4", choices=["dsv4", "reference"])
    ap.add_argument("--config", default="all", choices=["all"] + sorted(CONFIGS))
    ap.add_argument("--replicas", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kernel-case", default=None,
                    choices=["attn_prefill", "indexer_prefill", "compressor_prefill", "gemm_prefill",
                             "block_decode", "block_decode_window", "hc"],
                    help="profiling aid: run one prefill kernel alone on a 4096-query slice of config 4 "
                         "(positions 60000..64095), the two compressors on a 16384-token slice "
                         "(compressor_prefill), the projection GEMM's two kernels on prefill shapes "
                         "(gemm_prefill), or config 5's block step eagerly inside an NVTX range "
                         "(block_decode; block_decode_window: the same block at a ratio-128 layer), and print its "
                         "CUDA-event time; not a bench line")
    args = ap.parse_args()
    if args.kernel_case:
        return run_kernel_case(args)
    args.steps_given, args.warmup_given = args.steps is not None, args.warmup is not None
    if args.steps is None:
        args.steps = SUB_STEPS["c2"] if args.config == "all" else SUB_STEPS[args.config]
    if args.warmup is None:
        args.warmup = 20
    if args.impl == "reference":
        return run_reference(args)

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    _pkg()
    env = Env(args, world, rank, local, dev)
    names = ALL if args.config == "all" else (args.config,)
    results = {}
    for i, name in enumerate(names):
        results[name] = BENCH[name](env, name, i == 0)
        gc.collect()
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    head = results[names[0]]
    if len(names) > 1:
        head["configs"] = {n: results[n] for n in names[1:]}
    if rank == 0:
        print(json.dumps(head), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def run_kernel_case(args):
    """One prefill kernel on a 4096-query slice of config 4 (queries at positions 60000..64095,
    65,536 window rows + 16,384 compressed rows, top-k 1024): the case the profiles under profiles/
    were captured on. Seeded synthetic inputs; prints one JSON line with the CUDA-event time."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    SA, IX, NRm = _mod("sparse_attn"), _mod("indexer"), _mod("norm_rope")
    if args.kernel_case in ("block_decode", "block_decode_window"):
        return run_block_case(args, dev)
    if args.kernel_case == "hc":
        return run_hc_case(args, dev)
    if args.kernel_case == "compressor_prefill":
        return run_compressor_case(args, dev)
    if args.kernel_case == "gemm_prefill":
        return run_gemm_case(args, dev)
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


def run_compressor_case(args, dev):
    """The two compressors of config 4 on 16,384 tokens (x [16384, 4096] bf16, 128 MB, above L2):
    per compressor the projection pair (x wkv^T, x wgate^T in one tcgen05 launch, fp32 out) and the
    pooling kernel (softmax over 8 slots, RMSNorm, RoPE, the cache rounding), each timed with CUDA
    events over `--steps` calls. Prints one JSON line; not a bench line."""
    mla, C = _mod("mla"), _mod("compressor")
    NRm = _mod("norm_rope")
    s, dim = 16384, 4096
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(s, dim, device=dev, generator=g).bfloat16()
    reps = args.steps if args.steps is not None else 3
    freqs = NRm.rope_freqs(64, dev)
    res = {}
    for tag, hd, aq, odt in (("main", 512, 1, torch.bfloat16), ("indexer", 128, 2, torch.float32)):
        ws = [(torch.randn(2 * hd, dim, device=dev, generator=g) * 0.02).bfloat16() for _ in range(2)]
        ape = torch.randn(4, 2 * hd, device=dev, generator=g) * 0.1
        nw = torch.ones(hd, device=dev)
        kv, sc = mla.linear_multi(x, ws, torch.float32)
        out = torch.empty(1, s // 4, hd, dtype=odt, device=dev)
        proj = lambda: mla.linear_multi(x, ws, torch.float32)
        pool = lambda: C._pool(kv[None], sc[None], ape, nw, out, hd, 4, 64, freqs, pos0=0, act_quant=aq)
        for name, fn in (("proj", proj), ("pool", pool)):
            fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                fn()
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / reps
            if name == "proj":
                res[f"{tag}_proj"] = {"ms": ms, "tflops": 2 * 2 * s * 2 * hd * dim / ms / 1e9}
            else:
                nbytes = 2 * kv.numel() * 4 + out.numel() * out.element_size()
                res[f"{tag}_pool"] = {"ms": ms, "gbs": nbytes / ms / 1e6, "bytes": nbytes}
    print(json.dumps({"kernel_case": "compressor_prefill", "tokens": s, **res}), flush=True)


def run_gemm_case(args, dev):
    """dsv4_linear on prefill shapes (bf16 x and W, fp32 y) with the tcgen05 kernel (kernel 2) and
    the mma.sync kernel (kernel 1): median CUDA-event time of `--steps` calls (default 10) after 3
    warm-up calls. Shapes: config 4's compressor projection over all 65,536 tokens and its indexer
    twin, an 8,192-token chunk, q_up's width on 4,096 tokens, and config 1's 512 tokens."""
    import ctypes
    L = _mod("_lib")
    reps = args.steps if args.steps is not None else 10
    g = torch.Generator(device=dev).manual_seed(0)
    rows = []
    for m, n, k in ((65536, 1024, 4096), (65536, 256, 4096), (8192, 1024, 4096), (4096, 32768, 1024),
                    (512, 1024, 4096)):
        x = torch.randn(m, k, device=dev, generator=g).bfloat16()
        w = (torch.randn(n, k, device=dev, generator=g) * 0.02).bfloat16()
        y = torch.empty(m, n, device=dev)
        for kern in (2, 1):
            p = L.LinearParams()
            p.x, p.w, p.y = L.ptr(x), L.ptr(w), L.ptr(y)
            p.m, p.n, p.k, p.groups, p.group = m, n, k, 1, 64
            p.x_dtype, p.w_dtype, p.y_dtype, p.kernel = L.BF16, L.BF16, L.F32, kern
            nb = L.lib().dsv4_linear_workspace_size(ctypes.byref(p))
            ws = torch.empty(max(nb, 16), dtype=torch.uint8, device=dev)
            p.workspace, p.workspace_bytes = L.ptr(ws), nb
            st = L.stream_of(x)
            fn = lambda: L.check(L.lib().dsv4_linear(ctypes.byref(p), st))
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            ts = []
            for _ in range(reps):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                fn()
                e1.record()
                torch.cuda.synchronize()
                ts.append(e0.elapsed_time(e1))
            ms = sorted(ts)[len(ts) // 2]
            rows.append({"m": m, "n": n, "k": k, "kernel": "tcgen05" if kern == 2 else "mma.sync", "ms": ms,
                         "tflops": 2 * m * n * k / ms / 1e9})
        del x, w, y
    print(json.dumps({"kernel_case": "gemm_prefill", "calls": rows}), flush=True)


def run_hc_case(args, dev):
    """The hyper-connection kernels around the block (dim 4096, hc 4): hc_pre with the block's
    RMSNorm fused (bf16 output) and hc_post, at config 5's decode batch (32 tokens; x and the
    weights stay in L2 between calls) and at a 4096-token prefill slice (x 268 MB, above L2), each
    timed as one replay of a CUDA graph of `--steps` calls (default 20).
    Algorithmic bytes per call: hc_pre reads x (16 dim B per token) and fn once (1.5 MB), writes the
    bf16 norm (2 dim B per token) and post / comb; hc_post reads x and the residual (20 dim B per
    token) and writes 16 dim B per token."""
    H = _mod("hc")
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
    Lm, C = _mod("layer"), _mod("configs")
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
