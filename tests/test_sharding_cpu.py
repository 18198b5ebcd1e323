"""Host logic of the multi-GPU paths on CPU ranks (gloo, world size 2): query zig-zag coverage and
balance, compressed-block ranges, and the all-gather that assembles the compressed cache."""
import importlib
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

P = importlib.import_module("deepseek-v4-flash-mlx_b200.prefill")


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_zigzag_covers_queries_once_and_balances_causal_work(world):
    s = 65536
    seen = torch.zeros(s, dtype=torch.int32)
    work = []
    for r in range(world):
        w = 0
        for a, b in P.zigzag_ranges(s, world, r):
            seen[a:b] += 1
            w += sum(t // 4 for t in (a, b - 1)) * (b - a) / 2   # trapezoid of visible keys
        work.append(w)
    assert torch.all(seen == 1)
    assert max(work) / min(work) < 1.02
    n_blocks = s // 4
    blocks = [P.block_range(n_blocks, world, r) for r in range(world)]
    assert blocks[0][0] == 0 and blocks[-1][1] == n_blocks
    assert all(blocks[i][1] == blocks[i + 1][0] for i in range(world - 1))


def _gather_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sp = P.ShardedPrefill()
        n_blocks = 8 * world
        g0, g1 = P.block_range(n_blocks, world, rank)
        comp = torch.arange(g0, g1, dtype=torch.float32)[:, None].repeat(1, 4).to(torch.bfloat16)
        keys = torch.arange(g0, g1, dtype=torch.float32)[:, None].repeat(1, 3) * 10
        full_c, full_k = sp.gather_cache(comp, keys, n_blocks)
        ok = bool(torch.equal(full_c[:, 0].float(), torch.arange(n_blocks, dtype=torch.float32))) and \
            bool(torch.equal(full_k[:, 1], torch.arange(n_blocks, dtype=torch.float32) * 10))
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_cache_all_gather_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}


def _lost_rank_worker(rank, world, port, q):
    """Rank 1 joins, then leaves between steps (nothing of it in flight); rank 0 then runs the cache
    exchange and must get an error from the short process-group timeout or the closed connection,
    not wait for ever."""
    import datetime
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        q.put((rank, "left"))
        q.close()
        q.join_thread()  # the item is in the pipe before the process goes
        os._exit(0)  # leaves without the exchange and without tearing the group down
    t0 = time.perf_counter()
    try:
        sp = P.ShardedPrefill()
        comp = torch.zeros(8, 4, dtype=torch.bfloat16)
        keys = torch.zeros(8, 3)
        sp.gather_cache(comp, keys, 16)
        q.put((rank, "no error"))
    except Exception as e:  # the collective fails: a timeout or a closed peer connection
        q.put((rank, f"error after {time.perf_counter() - t0:.1f} s: {type(e).__name__}"))
    finally:
        q.close()
        q.join_thread()
        os._exit(0)


def test_lost_rank_ends_exchange_with_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 30500 + os.getpid() % 1000
    procs = [ctx.Process(target=_lost_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert res[1] == "left"
    assert res[0].startswith("error after"), res[0]
    assert float(res[0].split()[2]) < 60, res[0]
