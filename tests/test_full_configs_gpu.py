"""Configs 3, 4 and 5 at their full shapes against the CPU oracle.

  c3  batched decode: 64 sequences, each with its own 8192-token context (2048 compressed rows),
      top-k 512, sequence i seeded 100 + i: every sequence's attention index list bit for bit and
      the attention outputs at the attention tolerance (ref_torch/sparse_attn.py:23-34,
      oracle/v4_fast.py:108-119 with the indexer's selection).
  c4  prefill of 65,536 tokens, hidden 4096, top-k 1024, seed 2, through the same path the bench
      times (prefill.sparse_mla_prefill): compressed rows and indexer keys sampled around positions
      16K, 32K and 64K against the oracle compressor (ref_torch/compressor.py:21-50) on the same bf16
      hidden states; the selections of ~100 queries there, taken from the production chunk calls,
      bit for bit against the oracle indexer on the GPU's own keys; their attention outputs against
      the oracle attention over the GPU's own cached rows.
  c5  the full attention block decode: 32 sequences of 16,384-token contexts, int8-g64 weights,
      top-k 512, seed 3 (oracle/v4_fast.py:82-122) against the oracle block.
"""
import importlib

import numpy as np
import pytest
import torch

from helpers import assert_close_bf16, rel_rms
from oracle import compressor_ref as CR
from oracle import indexer_ref as I
from oracle import layer_ref as LR
from oracle import norm_rope_ref as NR
from oracle import sparse_attn_ref as SA

pytestmark = pytest.mark.gpu
PKG = "deepseek-v4-flash-mlx_b200"
BLOCK_REL = 1e-2   # the block output's tolerance (seven bf16 roundings on the way; see test_layer_gpu)


def _m(name):
    return importlib.import_module(PKG + "." + name)


def test_config3_full_shape(dsv4):
    C = _m("configs")
    b, ctx, top_k = 64, 8192, 512
    case = C.make_decode_case(b, ctx, top_k, seeds=[100 + i for i in range(b)])
    runner = dsv4.DecodeRunner(case.cache, case.sink, top_k)
    runner.q.copy_(case.q), runner.q_idx.copy_(case.q_idx), runner.w_idx.copy_(case.w_idx)
    runner.positions.copy_(case.positions)
    out = runner.step_device().float()          # the benchmarked path: one graph launch
    torch.cuda.synchronize()
    pool, win_base, comp_rows = C.decode_case_host_pool(case)
    f = NR.precompute_freqs(64, 0, 65536, 160000.0, 16, 32, 1)
    h = case.host
    ref, ref_idx = LR.decode_attention_ref(pool, win_base, comp_rows, h["k_idx"], h["q"], h["q_idx"], h["w_idx"],
                                           h["sink"], h["positions"], top_k, f, return_indices=True)
    # the graph's index buffer holds the selected pool rows (the window rows are implicit)
    np.testing.assert_array_equal(runner.idx.cpu().numpy(), ref_idx.numpy()[:, 128:])
    assert_close_bf16(out, ref, what="config 3 decode attention")


def test_config4_full_shape(dsv4):
    P, Lm, IX = _m("prefill"), _m("layer"), _m("indexer")
    dev = torch.device("cuda")
    s, top_k, chunk = 65536, 1024, 8192
    W = Lm.make_attention_weights(2)
    Wd = W.to(dev)
    cw = P.CompressorWeights.from_attention_weights(Wd)
    g = torch.Generator(device=dev).manual_seed(2)
    x = torch.randn(s, 4096, device=dev, generator=g).to(torch.bfloat16)
    q = torch.randn(s, 64, 512, device=dev, generator=g).to(torch.bfloat16)
    kv = torch.randn(s, 512, device=dev, generator=g).to(torch.bfloat16)
    qi = torch.randn(s, 64, 128, device=dev, generator=g)
    wi = torch.randn(s, 64, device=dev, generator=g) / 8
    o = P.sparse_mla_prefill(x, q, kv, qi, wi, Wd.sinks, cw, top_k=top_k, chunk=chunk)
    comp, keys = P.compress_range(x, cw, 0, s // 4)
    torch.cuda.synchronize()

    # compressed rows and keys of blocks around 16K, 32K and 64K: the oracle on x slices (a block
    # reads its 4 tokens and the 4 before them), roped at the blocks' absolute positions
    for j0, j1 in [(4090, 4102), (8186, 8198), (16372, 16384)]:
        lo = 4 * (j0 - 1)
        xs = x[lo:4 * j1].float().cpu()[None]
        rows, _ = CR.compressor_prefill(xs, W.c_wkv.float(), W.c_wgate.float(), W.c_ape, W.c_norm, pos0=lo)
        assert_close_bf16(comp[j0:j1].float(), rows[0, 1:], what=f"compressed rows {j0}..{j1}")
        kr, _ = CR.compressor_prefill(xs, W.i_wkv.float(), W.i_wgate.float(), W.i_ape, W.i_norm, head_dim=128,
                                      pos0=lo)
        assert_close_bf16(keys[j0:j1], kr[0, 1:], what=f"indexer keys {j0}..{j1}")

    # sampled queries: the first and last ones of the chunks that hold 16K, 32K and 64K
    picks = np.concatenate([np.arange(16384, 16400), np.arange(24560, 24576), np.arange(32768, 32784),
                            np.arange(40944, 40960), np.arange(57344, 57360), np.arange(65520, 65536)])
    f = NR.precompute_freqs(64, 0, 65536, 160000.0, 16, 32, 1)
    keys_h = keys.cpu().numpy()
    kvcat = torch.cat([kv.float().cpu(), comp.float().cpu()])
    win_base = torch.zeros(1, dtype=torch.int64, device=dev)
    for c0 in sorted({int(t) // chunk * chunk for t in picks}):
        c1 = c0 + chunk
        ts = picks[(picks >= c0) & (picks < c1)]
        # the production call for the whole chunk (the tensor-core filter + exact band)
        pos = torch.arange(c0, c1, dtype=torch.int32, device=dev)
        idx = torch.empty((1, c1 - c0, 128 + top_k), dtype=torch.int32, device=dev)
        IX.indexer_topk_into(idx, qi[c0:c1][None], wi[c0:c1][None], keys[None], top_k, positions=pos[None], ratio=4,
                             out_col=128, out_offset=s, win_base=win_base, window=128, window_linear=True)
        got = idx[0, ts - c0].cpu().numpy()
        sel = I.indexer_topk(qi[ts].cpu().numpy()[None], wi[ts].cpu().numpy()[None], keys_h[None], top_k,
                             positions=ts[None], ratio=4)[0]
        win = np.stack([np.arange(t - 127, t + 1) for t in ts])
        want = np.concatenate([win, np.where(sel >= 0, sel + s, -1)], 1)
        np.testing.assert_array_equal(got, want)
        ref = SA.sparse_attn(q[ts].float().cpu(), kvcat, W.sinks, torch.from_numpy(want.astype(np.int64)),
                             512 ** -0.5)
        ref = NR.rope_at(ref, torch.from_numpy(ts), f, inverse=True)
        assert_close_bf16(o[ts].float(), ref, what=f"prefill attention, queries {ts[0]}..{ts[-1]}")


def test_config5_full_shape(dsv4):
    Lm, C = _m("layer"), _m("configs")
    b, ctx, top_k = 32, 16384, 512
    case = C.make_decode_case(b, ctx, top_k, seeds=[3 + i for i in range(b)])
    W = Lm.make_attention_weights(3, quant=True)
    cache = case.cache
    g = torch.Generator().manual_seed(3)
    cache.ring_kv.copy_(torch.randn(cache.ring_kv.shape, generator=g))
    cache.ring_score.copy_(torch.randn(cache.ring_score.shape, generator=g))
    cache.ring_k_idx.copy_(torch.randn(cache.ring_k_idx.shape, generator=g))
    cache.ring_s_idx.copy_(torch.randn(cache.ring_s_idx.shape, generator=g))
    # every sequence at the context's last position (16383 closes a compression block), as the bench
    pos = torch.full((b,), ctx - 1, dtype=torch.int32)
    x = torch.randn(b, 4096, generator=g)
    pool, win_base, comp_rows = C.decode_case_host_pool(case)
    state = dict(pool=pool.float(), win_base=win_base, comp_rows=comp_rows, k_idx=cache.k_idx.cpu().clone(),
                 ring_kv=cache.ring_kv.cpu().clone(), ring_score=cache.ring_score.cpu().clone(),
                 ring_k=cache.ring_k_idx.cpu().clone(), ring_s=cache.ring_s_idx.cpu().clone())
    blk = Lm.DecodeBlock(W.to("cuda"), b, ctx, top_k=top_k, cache=cache)
    aux = {}
    out = blk.step(x.cuda(), pos.cuda(), aux=aux)
    torch.cuda.synchronize()
    # With 4096 visible keys and top-k 512 the selection is sensitive to the indexer's inputs, which
    # the GPU computes from bf16 activations (the oracle from fp32): the oracle selects on the GPU's
    # own q_idx, w_idx and keys, and must then pick exactly the GPU's rows; the rest of the block
    # (projections, ring, attention, output projection) stays the oracle's fp32 chain.
    keys_gpu = cache.k_idx.cpu().clone()
    oaux = {}
    ref = LR.decode_block_ref(state, W, x, pos, top_k=top_k, aux=oaux,
                              indexer_inputs=(aux["q_idx"].cpu().float(), aux["w_idx"].cpu().float(), keys_gpu))
    np.testing.assert_array_equal(aux["idx"].cpu().numpy(), oaux["idx"].numpy()[:, 128:])
    rr = rel_rms(out, ref)
    assert rr <= BLOCK_REL, f"config 5 block rel_rms={rr:.3e}"
    assert_close_bf16(cache.k_idx.cpu(), state["k_idx"], what="indexer keys after the step")
    assert_close_bf16(cache.ring_kv.cpu(), state["ring_kv"], what="compressor ring after the step")
