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
