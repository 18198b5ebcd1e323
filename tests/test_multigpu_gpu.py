"""Multi-GPU paths on 2 GPUs (NCCL): the query-sharded long prefill equals the single-GPU result, and
batch-split decode is independent per rank. Skipped with fewer than 2 GPUs."""
import importlib
import os

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
PKG = "deepseek-v4-flash-mlx_b200"


def _worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        P = importlib.import_module(PKG + ".prefill")
        Lm = importlib.import_module(PKG + ".layer")
        C = importlib.import_module(PKG + ".configs")
        s = 4096
        g = torch.Generator().manual_seed(9)
        W = Lm.make_attention_weights(9, dims=C.LayerDims(dim=1024)).to("cuda")
        x = torch.randn(s, 1024, generator=g).cuda()
        qq = torch.randn(s, 64, 512, generator=g).to(torch.bfloat16).cuda()
        kv = torch.randn(s, 512, generator=g).to(torch.bfloat16).cuda()
        qi = torch.randn(s, 64, 128, generator=g).cuda()
        wi = (torch.randn(s, 64, generator=g) / 8).cuda()
        cw = P.CompressorWeights.from_attention_weights(W)
        full = P.sparse_mla_prefill(x, qq, kv, qi, wi, W.sinks, cw, top_k=256, chunk=1024)
        outs = P.ShardedPrefill().run(x, qq, kv, qi, wi, W.sinks, cw, top_k=256, chunk=1024)
        ok = all(torch.equal(o, full[a:b]) for a, b, o in outs)
        dist.barrier()
        q.put((rank, ok, sum(b - a for a, b, _ in outs)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_prefill_equals_single_gpu():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
    assert all(ok for _, ok, _ in res), res
    assert sum(n for _, _, n in res) == 4096


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_one_process_two_devices():
    """Kernel attributes (shared-memory limits, non-portable cluster sizes) are per device: one
    process that runs the attention kernels and the indexer on GPU 0 and then on GPU 1 gets the
    same results on both."""
    dsv4 = importlib.import_module(PKG)
    g = torch.Generator().manual_seed(17)
    q = torch.randn(20, 64, 512, generator=g).to(torch.bfloat16)
    kv = torch.randn(3000, 512, generator=g).to(torch.bfloat16)
    sink = torch.randn(64, generator=g)
    idx = torch.randint(0, 3000, (20, 640), generator=g, dtype=torch.int32)
    q1 = q[:1]
    qi = torch.randn(1, 256, 64, 128, generator=g)
    wi = torch.randn(1, 256, 64, generator=g) / 8
    keys = torch.randn(1, 2000, 128, generator=g)
    res = []
    for d in (0, 1):
        dev = torch.device("cuda", d)
        with torch.cuda.device(dev):
            r = [dsv4.sparse_attn(q.to(dev), kv.to(dev), sink.to(dev), idx.to(dev), 512 ** -0.5, kernel=k).cpu()
                 for k in (1, 2)]
            # one query: the mma.sync kernel's splits run as one (non-portable, 10-CTA) cluster
            r.append(dsv4.sparse_attn(q1.to(dev), kv.to(dev), sink.to(dev), idx[:1].to(dev), 512 ** -0.5).cpu())
            r.append(dsv4.indexer_topk(qi.to(dev), wi.to(dev), keys.to(dev), 256, mode=2).cpu())
            torch.cuda.synchronize(dev)
        res.append(r)
    for a, b in zip(*res):
        assert torch.equal(a, b)
