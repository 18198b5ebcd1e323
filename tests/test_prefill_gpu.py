"""The long-prefill core (config 4 shapes, reduced length) against the oracle."""
import importlib

import numpy as np
import pytest
import torch

from helpers import assert_close_bf16
from oracle import compressor_ref as CR
from oracle import indexer_ref as I
from oracle import norm_rope_ref as NR
from oracle import sparse_attn_ref as SA

pytestmark = pytest.mark.gpu
PKG = "deepseek-v4-flash-mlx_b200"


def _inputs(s, seed, dim=1024):
    g = torch.Generator().manual_seed(seed)
    Lm = importlib.import_module(PKG + ".layer")
    W = Lm.make_attention_weights(seed, dims=importlib.import_module(PKG + ".configs").LayerDims(dim=dim))
    x = torch.randn(s, dim, generator=g)
    q = torch.randn(s, 64, 512, generator=g).to(torch.bfloat16)
    kv = torch.randn(s, 512, generator=g).to(torch.bfloat16)
    q_idx = torch.randn(s, 64, 128, generator=g)
    w_idx = torch.randn(s, 64, generator=g) / 8
    return W, x, q, kv, q_idx, w_idx


def test_compress_range_slices_equal_full_compression():
    P = importlib.import_module(PKG + ".prefill")
    W, x, *_ = _inputs(1024, 4)
    Wd = W.to("cuda")
    cw = P.CompressorWeights.from_attention_weights(Wd)
    comp, keys = P.compress_range(x.cuda(), cw, 0, 256)
    for g0, g1 in [(0, 64), (64, 128), (200, 256)]:
        c, k = P.compress_range(x.cuda(), cw, g0, g1)
        assert torch.equal(c, comp[g0:g1]) and torch.equal(k, keys[g0:g1]), (g0, g1)
    # against the oracle on the same (bf16-rounded) operands
    xb = x.to(torch.bfloat16).float()
    ref, _ = CR.compressor_prefill(xb[None], W.c_wkv.float(), W.c_wgate.float(), W.c_ape, W.c_norm)
    assert_close_bf16(comp, ref[0], what="compressed rows")
    refk, _ = CR.compressor_prefill(xb[None], W.i_wkv.float(), W.i_wgate.float(), W.i_ape, W.i_norm, head_dim=128)
    assert_close_bf16(keys, refk[0], what="indexer keys")


def test_sparse_mla_prefill_matches_oracle():
    P = importlib.import_module(PKG + ".prefill")
    s, top_k = 2048, 96
    W, x, q, kv, q_idx, w_idx = _inputs(s, 5)
    Wd = W.to("cuda")
    cw = P.CompressorWeights.from_attention_weights(Wd)
    o = P.sparse_mla_prefill(x.cuda(), q.cuda(), kv.cuda(), q_idx.cuda(), w_idx.cuda(), Wd.sinks, cw, top_k=top_k,
                             chunk=512)
    o_small = P.sparse_mla_prefill(x.cuda(), q.cuda(), kv.cuda(), q_idx.cuda(), w_idx.cuda(), Wd.sinks, cw,
                                   top_k=top_k, chunk=2048)
    assert torch.equal(o, o_small)                     # chunking does not change the result
    comp, keys = P.compress_range(x.cuda(), cw, 0, s // 4)
    pos = np.arange(s)
    sel = I.indexer_topk(q_idx.numpy()[None], w_idx.numpy()[None], keys.cpu().numpy()[None], top_k,
                         positions=pos[None], ratio=4)[0]
    win = np.stack([[max(0, t - 127) + c if max(0, t - 127) + c <= t else -1 for c in range(128)] for t in range(s)])
    idx = torch.from_numpy(np.concatenate([win, np.where(sel >= 0, sel + s, -1)], 1).astype(np.int64))
    kvcat = torch.cat([kv.float(), comp.float().cpu()])
    f = NR.precompute_freqs(64, 0, 65536, 160000.0, 16, 32, 1)
    ref = NR.rope_at(SA.sparse_attn_chunked(q.float(), kvcat, W.sinks, idx, 512 ** -0.5), torch.arange(s), f,
                     inverse=True)
    assert_close_bf16(o.float(), ref, what="prefill attention output")


def test_host_prefill_matches_device_prefill():
    """The pinned-host path (per-chunk copies on two copy streams around the compute stream, two
    device slots reused across chunks and across calls) gives the device path's bits, for a range
    that starts mid-sequence and ends in a partial chunk."""
    P = importlib.import_module(PKG + ".prefill")
    s, top_k, chunk = 2048, 96, 384
    W, x, q, kv, q_idx, w_idx = _inputs(s, 6)
    Wd = W.to("cuda")
    cw = P.CompressorWeights.from_attention_weights(Wd)
    x = x.to(torch.bfloat16)
    want = P.sparse_mla_prefill(x.cuda(), q.cuda(), kv.cuda(), q_idx.cuda(), w_idx.cuda(), Wd.sinks, cw, top_k=top_k,
                                chunk=chunk)
    pin = [t.contiguous().pin_memory() for t in (x, q, kv, q_idx, w_idx)]
    h_out = torch.full((s, 64, 512), float("nan"), dtype=torch.bfloat16).pin_memory()
    staging = P.PrefillStaging(chunk, "cuda")
    for _ in range(2):   # the second call reuses the staging slots
        h_out.fill_(float("nan"))
        P.sparse_mla_prefill_host(*pin[:2], pin[2], *pin[3:], Wd.sinks, cw, h_out, top_k=top_k, chunk=chunk,
                                  staging=staging)
        torch.cuda.synchronize()
        assert torch.equal(h_out, want.cpu())
    # a mid-sequence range [a, b) against attend_queries over the same range
    comp, keys = P.compress_range(x.cuda(), cw, 0, s // 4)
    a, b = 640, 1900
    ref = P.attend_queries(q[a:b].cuda(), q_idx[a:b].cuda(), w_idx[a:b].cuda(), kv.cuda(), comp, keys, Wd.sinks, a, b,
                           top_k, chunk)
    part = torch.empty((b - a, 64, 512), dtype=torch.bfloat16).pin_memory()
    P.attend_queries_host(pin[1][a:b], pin[3][a:b], pin[4][a:b], kv.cuda(), comp, keys, Wd.sinks, a, b, part, top_k,
                          chunk, staging)
    torch.cuda.synchronize()
    assert torch.equal(part, ref.cpu())
    with pytest.raises(ValueError):
        P.attend_queries_host(q[a:b], pin[3][a:b], pin[4][a:b], kv.cuda(), comp, keys, Wd.sinks, a, b, part, top_k,
                              chunk, staging)   # q not pinned
