"""The dsv4 ops are opaque to torch.compile: compressor_prefill -> sparse_attn, and a decode step
(compressor_decode_step + decode_attention), traced with fullgraph=True (a graph break raises),
give exactly the eager results (same kernels, so bit for bit).

The backend is aot_eager: it traces through every op's fake (shape) implementation and
functionalises the mutating ops, and runs the captured graph without generating code."""
import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_compile_fullgraph_compressor_then_sparse_attn(dsv4, cuda_dev):
    torch._dynamo.reset()
    g = torch.Generator(device=cuda_dev).manual_seed(11)
    s, dim, n_win, t = 64, 4096, 64, 96
    x = torch.randn(1, s, dim, device=cuda_dev, generator=g).bfloat16()
    wkv = (torch.randn(1024, dim, device=cuda_dev, generator=g) * 0.02).bfloat16()
    wgate = (torch.randn(1024, dim, device=cuda_dev, generator=g) * 0.02).bfloat16()
    ape = torch.randn(4, 1024, device=cuda_dev, generator=g) * 0.1
    norm_w = 1 + torch.randn(512, device=cuda_dev, generator=g) * 0.1
    q = torch.randn(s, 64, 512, device=cuda_dev, generator=g).bfloat16()
    kvwin = torch.randn(n_win, 512, device=cuda_dev, generator=g).bfloat16()
    sink = torch.randn(64, device=cuda_dev, generator=g)
    idx = torch.randint(-1, n_win + s // 4, (s, t), device=cuda_dev, generator=g, dtype=torch.int32)

    def f(x, wkv, wgate, ape, norm_w, q, kvwin, sink, idx):
        comp, state = dsv4.compressor_prefill(x, wkv, wgate, ape, norm_w, out_dtype=torch.bfloat16)
        kv = torch.cat([kvwin, comp[0]])
        return dsv4.sparse_attn(q, kv, sink, idx, 512 ** -0.5), state["ring_kv"], state["score"]

    want = f(x, wkv, wgate, ape, norm_w, q, kvwin, sink, idx)
    got = torch.compile(f, fullgraph=True, backend="aot_eager")(x, wkv, wgate, ape, norm_w, q, kvwin, sink, idx)
    torch.cuda.synchronize()
    for a, b in zip(got, want):
        assert torch.equal(a, b)


def test_compile_fullgraph_decode_step(dsv4, cuda_dev):
    """One decode step of the compressed layer: the compressor ring step (mutating the ring and the
    cache rows) then decode attention, compiled whole against the same step run eagerly."""
    torch._dynamo.reset()
    C = importlib.import_module("deepseek-v4-flash-mlx_b200.configs")
    NRm = importlib.import_module("deepseek-v4-flash-mlx_b200.norm_rope")
    b, ctx = 2, 2048
    case = C.make_decode_case(b, ctx, 256, seeds=[31, 32], device=cuda_dev)
    g = torch.Generator(device=cuda_dev).manual_seed(12)
    kvp = torch.randn(b, 1024, device=cuda_dev, generator=g)
    scp = torch.randn(b, 1024, device=cuda_dev, generator=g)
    ape = torch.randn(4, 1024, device=cuda_dev, generator=g) * 0.1
    norm_w = 1 + torch.randn(512, device=cuda_dev, generator=g) * 0.1
    wdummy = torch.zeros(1024, 4096, device=cuda_dev, dtype=torch.bfloat16)
    x = torch.zeros(b, 4096, device=cuda_dev)
    freqs = NRm.rope_freqs(64, cuda_dev)
    pos = torch.full((b,), ctx - 1, dtype=torch.int32, device=cuda_dev)   # (p+1) % 4 == 0: the ring emits
    rows = torch.stack([case.cache.comp_rows(i, torch.tensor(ctx // 4 - 1, device=cuda_dev)) for i in range(b)])

    def step(cache, q, q_idx, w_idx, sink, pos, rows):
        dsv4.compressor_decode_step(x, wdummy, wdummy, ape, norm_w, cache.ring_kv, cache.ring_score, pos,
                                    cache.kv_pool, rows, freqs=freqs, proj=(kvp, scp))
        return dsv4.decode_attention(cache, q, q_idx, w_idx, sink, pos, 256, freqs=freqs)

    c_eager, c_comp = case.cache, case.cache.clone()
    want = step(c_eager, case.q, case.q_idx, case.w_idx, case.sink, pos, rows)
    got = torch.compile(step, fullgraph=True, backend="aot_eager")(c_comp, case.q, case.q_idx, case.w_idx, case.sink,
                                                                   pos, rows)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert torch.equal(c_comp.ring_kv, c_eager.ring_kv) and torch.equal(c_comp.ring_score, c_eager.ring_score)
    assert torch.equal(c_comp.kv_pool, c_eager.kv_pool)
