"""Benchmark of the sparse-MLA decode path (BASELINE config 2 by default).

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl dsv4|reference] [--config c2|c3]

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
CONFIGS = {
    "c2": dict(batch=1, ctx=32768, top_k=512, seeds=lambda r, i: 1 + 7919 * r,
               workload="config2: decode, batch 1, 32768-token context (8192 compressed + 128 window rows), "
                        "top-k 512, bf16 cache, fp32 indexer keys"),
    "c3": dict(batch=64, ctx=8192, top_k=512, seeds=lambda r, i: 100 + i + 7919 * r,
               workload="config3: batched decode, batch 64, 8192-token contexts (2048 compressed + 128 window "
                        "rows each), top-k 512"),
}
L2_BYTES = 126 * 1024 * 1024
# kernels of one decode step: q norm/rope, indexer scores, top-k selection, sparse attention, split merge
LAUNCHES_PER_STEP = 5


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
def cpu_reference(cfg_name, samples, threads=None):
    """Time the oracle port (torch fp32 + the C indexer restatement) on the host cores for a bounded
    sample of decode tokens of the config; returns (tok/s, cores, description)."""
    from oracle import layer_ref as LR
    from oracle import norm_rope_ref as NR
    cfgd = CONFIGS[cfg_name]
    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    C = __import__("importlib").import_module(PKG + ".configs")
    batch = min(cfgd["batch"], samples)
    case = C.make_decode_case(batch, cfgd["ctx"], cfgd["top_k"], seeds=[cfgd["seeds"](0, i) for i in range(batch)],
                              device="cpu", shuffle_pages=True)
    pool, win_base, comp_rows = C.decode_case_host_pool(case)
    f = NR.precompute_freqs(64, 0, 65536, 160000.0, 16, 32, 1)
    h = case.host
    LR.decode_attention_ref(pool, win_base, comp_rows, h["k_idx"][:1], h["q"][:1], h["q_idx"][:1], h["w_idx"][:1],
                            h["sink"], h["positions"][:1], cfgd["top_k"], f)  # warm-up
    t0 = time.perf_counter()
    LR.decode_attention_ref(pool, win_base, comp_rows, h["k_idx"], h["q"], h["q_idx"], h["w_idx"], h["sink"],
                            h["positions"], cfgd["top_k"], f)
    dt = time.perf_counter() - t0
    return batch / dt, threads, f"{batch} decode token(s) of {cfg_name} through the CPU oracle ({dt:.2f} s)"


def run_reference(args):
    world, rank, _ = _dist()
    if rank != 0:
        return
    cfgd = CONFIGS[args.config]
    per_step = []
    n_tok = 1
    for _ in range(max(1, args.warmup // 100)):
        cpu_reference(args.config, n_tok)
    for _ in range(min(args.steps, 3)):
        v, cores, desc = cpu_reference(args.config, n_tok)
        per_step.append(v)
    v = statistics.median(per_step)
    line = {"impl": "reference", "metric": METRIC if args.config == "c2" else METRIC.replace("at 32K ctx", "batched"),
            "value": v, "unit": "tok/s", "n_gpus": args.gpus, "steps": len(per_step), "warmup": args.warmup,
            "ms_per_step": 1000.0 * n_tok / v * (cfgd["batch"] // n_tok if args.config == "c3" else 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": cfgd["workload"], "global_batch": cfgd["batch"], "ctx": cfgd["ctx"],
                       "parallelism": "cpu"},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": "port",
                             "sample": desc + "; the reference's ref_torch path restated in oracle/"},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------ GPU leg
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2400)
    ap.add_argument("--warmup", type=int, default=240)
    ap.add_argument("--impl", default="dsv4", choices=["dsv4", "reference"])
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS))
    ap.add_argument("--replicas", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
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
    batch, ctx, top_k = cfgd["batch"], cfgd["ctx"], cfgd["top_k"]

    # ---- replicas of the whole decode state, rotating so that no step starts with warm L2
    probe = C.make_decode_case(batch, ctx, top_k, seeds=[cfgd["seeds"](rank, i) for i in range(batch)], device=dev)
    c = probe.cache
    footprint = (c.kv_pool.numel() * 2 + c.k_idx.numel() * 4 + c.block_table.numel() * 4)
    R = args.replicas or max(2, -(-2 * L2_BYTES // footprint) + 1)
    cases = [probe] + [C.make_decode_case(batch, ctx, top_k, seeds=[cfgd["seeds"](rank, i) + 104729 * r
                                                                   for i in range(batch)], device=dev)
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

    # ---- e2e through the public host API (pinned inputs, graph, output back, every step)
    hq = [cs.host["q"].pin_memory() for cs in cases]
    hqi = [cs.host["q_idx"].pin_memory() for cs in cases]
    hw = [cs.host["w_idx"].pin_memory() for cs in cases]
    hp = [cs.host["positions"].pin_memory() for cs in cases]
    for i in range(min(R, 4)):
        runners[i].step_host(hq[i], hqi[i], hw[i], hp[i])
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for s in range(args.steps):
        i = s % R
        runners[i].step_host(hq[i], hqi[i], hw[i], hp[i])
    f1.record(stream)
    torch.cuda.synchronize()
    ems = _barrier_max(f0.elapsed_time(f1), world, dev)
    e2e = {"value": world * batch * args.steps / (ems / 1000.0), "unit": "tok/s",
           "h2d_bytes_per_step": runners[0].h2d_bytes(), "d2h_bytes_per_step": runners[0].d2h_bytes(),
           "path": "DecodeRunner.step_host (pinned host in/out, CUDA graph)"}

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
    prof = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(prof):
        try:
            roofline["traffic"] = json.load(open(prof)).get(args.config, {}).get(top)
        except Exception:
            pass

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores, desc = cpu_reference(args.config, 1 if args.config == "c2" else 2)
        cpu = {"value": v, "unit": "tok/s", "cores": cores, "kind": "port", "sample": desc}

    if rank == 0:
        line = {"metric": METRIC if args.config == "c2" else METRIC.replace("at 32K ctx", "batched"),
                "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic",
                "config": {"workload": cfgd["workload"], "global_batch": batch * world, "ctx": ctx, "top_k": top_k,
                           "parallelism": f"batch-split x{world} (no collective)" if world > 1 else "single GPU",
                           "l2": f"inputs rotate over {R} replicas x {footprint / 2**20:.1f} MiB = "
                                 f"{R * footprint / 2**20:.0f} MiB > L2 (126 MB)",
                           "cuda_graph": True},
                "gpu_launches": LAUNCHES_PER_STEP * args.steps,
                "e2e": e2e, "roofline": roofline, "cpu_baseline": cpu, "clocks": clocks}
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


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
    torch.cuda.synchronize()
    nvis = [min((int(c.host["positions"][i]) + 1) // 4, c.cache.max_comp) for c in cases[:1] for i in range(b)]
    n_keys = sum(nvis)
    funcs = {
        # score + select (which also writes the window rows): k_idx read once, indices written
        "indexer_topk": (lambda i: IX.indexer_topk_into(runners[i].idx.view(b, 1, -1), runners[i].q_idx.view(b, 1, 64, 128),
                                                        runners[i].w_idx.view(b, 1, 64), cases[i].cache.k_idx, top_k,
                                                        runners[i].positions.view(b, 1), 4, out_col=128,
                                                        out_offset=cases[i].cache.comp_base,
                                                        block_table=cases[i].cache.block_table, page=cases[i].cache.page,
                                                        win_base=cases[i].cache.win_base, window=128),
                         n_keys * 128 * 4 + b * (64 * 128 * 4 + 64 * 4 + (128 + top_k) * 4)),
        # attention (+ split merge): gathered rows, raw q in, o out, indices
        "sparse_attn": (lambda i: SA.sparse_attn_decode(runners[i].q, cases[i].cache.kv_pool, cases[i].sink,
                                                        runners[i].idx, 512 ** -0.5, runners[i].positions, freqs, 64),
                        b * ((128 + top_k) * (512 * 2 + 4) + 64 * 512 * 4 + 64 * 512 * 2)),
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


if __name__ == "__main__":
    main()
