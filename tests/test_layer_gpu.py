"""The full attention block (config 1 prefill, config 5 decode) against the CPU oracle."""
import importlib

import numpy as np
import pytest
import torch

from helpers import assert_close_bf16, rel_rms
from oracle import indexer_ref as I
from oracle import layer_ref as LR

pytestmark = pytest.mark.gpu
PKG = "deepseek-v4-flash-mlx_b200"
# Tolerance of the block output (after o_grouped): the GPU rounds seven activations to bf16 on the
# way (x_n, q_a, q, kv rows, compressed rows, o, the o_grouped midpoint) where the oracle stays in
# fp32; each rounding contributes ~1e-3 relative, so the block output is held to rel-RMS 1e-2.
BLOCK_REL = 1e-2


def _layer():
    return importlib.import_module(PKG + ".layer")


def test_prefill_layer_config1():
    """Config 1: 512 tokens, hidden 4096, x ~N(0,1), weights ~N(0,0.02), seed 0. top_k 512 exceeds the
    visible compressed rows, so the index list is the reference's (window + all visible rows)."""
    Lm = _layer()
    W = Lm.make_attention_weights(0)
    x = torch.randn(512, 4096, generator=torch.Generator().manual_seed(0))
    out, aux = Lm.prefill_layer(x.cuda(), W.to("cuda"), top_k=512, return_aux=True)
    ref, idx_ref, o_ref = LR.prefill_layer_ref(x, W, top_k=512)
    np.testing.assert_array_equal(aux["idx"].cpu().numpy(), idx_ref.numpy())
    assert_close_bf16(aux["o"], o_ref, what="attention output")
    rr = rel_rms(out, ref)
    assert rr <= BLOCK_REL, f"block output rel_rms={rr:.3e}"


def test_prefill_layer_selection_bit_exact():
    """top_k below the visible count: the GPU's selection equals the oracle's on the same indexer inputs."""
    Lm = _layer()
    W = Lm.make_attention_weights(1)
    s = 384
    x = torch.randn(s, 4096, generator=torch.Generator().manual_seed(1))
    _, aux = Lm.prefill_layer(x.cuda(), W.to("cuda"), top_k=24, return_aux=True)
    sel = I.indexer_topk(aux["q_idx"].cpu().numpy()[None], aux["w_idx"].cpu().numpy()[None],
                         aux["k_idx"].cpu().numpy(), 24, positions=np.arange(s)[None], ratio=4)[0]
    got = aux["idx"].cpu().numpy()[:, 128:]
    np.testing.assert_array_equal(got, np.where(sel >= 0, sel + s, -1))


@pytest.mark.parametrize("quant", [False, True])
def test_decode_block_config5(quant):
    """Config 5 shape (reduced batch/context): one decode step of the whole block, 8-bit g64 weights
    in the quantised case; sequences at positions that do and do not close a compression block."""
    Lm = _layer()
    C = importlib.import_module(PKG + ".configs")
    b, ctx = 3, 1024
    case = C.make_decode_case(b, ctx, 512, seeds=[300 + i for i in range(b)])
    W = Lm.make_attention_weights(3, quant=quant)
    Wd = W.to("cuda")
    cache = case.cache
    g = torch.Generator().manual_seed(5)
    cache.ring_kv.copy_(torch.randn(cache.ring_kv.shape, generator=g))
    cache.ring_score.copy_(torch.randn(cache.ring_score.shape, generator=g))
    cache.ring_k_idx.copy_(torch.randn(cache.ring_k_idx.shape, generator=g))
    cache.ring_s_idx.copy_(torch.randn(cache.ring_s_idx.shape, generator=g))
    # the new tokens: positions 1023 (closes a block), 1021 and 1022; the block's entry (p+1)//4-1 is
    # written by the step for p = 1023
    pos = torch.tensor([ctx - 1, ctx - 3, ctx - 2], dtype=torch.int32)
    x = torch.randn(b, 4096, generator=g)
    pool, win_base, comp_rows = C.decode_case_host_pool(case)
    state = dict(pool=pool.float(), win_base=win_base, comp_rows=comp_rows, k_idx=cache.k_idx.cpu().clone(),
                 ring_kv=cache.ring_kv.cpu().clone(), ring_score=cache.ring_score.cpu().clone(),
                 ring_k=cache.ring_k_idx.cpu().clone(), ring_s=cache.ring_s_idx.cpu().clone())
    blk = Lm.DecodeBlock(Wd, b, ctx, top_k=512, cache=cache)
    out = blk.step(x.cuda(), pos.cuda())
    ref = LR.decode_block_ref(state, W, x, pos, top_k=512)
    rr = rel_rms(out, ref)
    assert rr <= BLOCK_REL, f"decode block rel_rms={rr:.3e}"
    # the state the step wrote: this token's window rows, the emitted compressed row and indexer key
    assert_close_bf16(cache.kv_pool.float().cpu(), state["pool"], what="pool after step")
    # keys come from bf16 GEMM operands on the GPU (fp32 in the oracle): bf16-level tolerance
    assert_close_bf16(cache.k_idx.cpu(), state["k_idx"], what="indexer keys after step")
    assert_close_bf16(cache.ring_kv.cpu(), state["ring_kv"], what="compressor ring")
    # the key image the step kept current (the emitted key appended by the compressor) is the one a
    # full rebuild from the keys gives, byte for byte; its norm maximum still bounds every key
    IX = importlib.import_module(PKG + ".indexer")
    img, inv, nmax = cache.key_image
    fresh = IX.build_key_image(cache.k_idx, IX.key_image_buffers(b, cache.max_comp, "cuda"))
    assert torch.equal(img, fresh[0])
    assert torch.equal(inv, fresh[1])
    assert (nmax >= fresh[2] * (1 - 1e-6)).all()


def test_decode_block_act_quant():
    """The block step with the reference's fp8 act-quant simulation of the cached kv and compressed
    rows (oracle/decode_engine.py:82, 105) against the oracle doing the same."""
    Lm = _layer()
    C = importlib.import_module(PKG + ".configs")
    b, ctx = 2, 1024
    case = C.make_decode_case(b, ctx, 512, seeds=[310, 311])
    W = Lm.make_attention_weights(5, quant=True)
    cache = case.cache
    g = torch.Generator().manual_seed(7)
    cache.ring_kv.copy_(torch.randn(cache.ring_kv.shape, generator=g))
    cache.ring_score.copy_(torch.randn(cache.ring_score.shape, generator=g))
    pos = torch.tensor([ctx - 1, ctx - 2], dtype=torch.int32)
    x = torch.randn(b, 4096, generator=g)
    pool, win_base, comp_rows = C.decode_case_host_pool(case)
    state = dict(pool=pool.float(), win_base=win_base, comp_rows=comp_rows, k_idx=cache.k_idx.cpu().clone(),
                 ring_kv=cache.ring_kv.cpu().clone(), ring_score=cache.ring_score.cpu().clone(),
                 ring_k=cache.ring_k_idx.cpu().clone(), ring_s=cache.ring_s_idx.cpu().clone())
    blk = Lm.DecodeBlock(W.to("cuda"), b, ctx, top_k=512, cache=cache, act_quant=True)
    out = blk.step(x.cuda(), pos.cuda())
    ref = LR.decode_block_ref(state, W, x, pos, top_k=512, act_quant=True)
    rr = rel_rms(out, ref)
    assert rr <= BLOCK_REL, f"decode block (act quant) rel_rms={rr:.3e}"
    # the rows this step cached carry fp8 values on their nope dims: at most 16 distinct magnitudes
    # per 64-dim block once the block scale is divided out (e4m3 has 3 mantissa bits and 16 binades)
    win_row = cache.kv_pool[int(cache.win_base[0]) + (ctx - 1) % 128].float().cpu()
    blk0 = win_row[:64]
    e = int(torch.ceil(torch.log2(blk0.abs().max().clamp(min=1e-4) / 448)))
    assert torch.equal(blk0, (blk0 / 2.0 ** e).to(torch.float8_e4m3fn).float() * 2.0 ** e)


def test_decode_block_hc():
    """The block step inside hc_pre / hc_post (oracle/v4_fast.py:85, 122), with hc_pre and the
    attention norm fused in one kernel, against the oracle chain. The residual term
    sum_i comb[i, j] x[i] is removed from both sides before the block tolerance is applied, so the
    check sees the attention output's share."""
    from oracle import hc_ref as H
    Lm = _layer()
    C = importlib.import_module(PKG + ".configs")
    b, ctx = 2, 1024
    case = C.make_decode_case(b, ctx, 512, seeds=[320, 321])
    W = Lm.make_attention_weights(6, quant=True)
    cache = case.cache
    g = torch.Generator().manual_seed(8)
    cache.ring_kv.copy_(torch.randn(cache.ring_kv.shape, generator=g))
    cache.ring_score.copy_(torch.randn(cache.ring_score.shape, generator=g))
    pos = torch.tensor([ctx - 1, ctx - 2], dtype=torch.int32)
    x = torch.randn(b, 4, 4096, generator=g)
    hc_fn = torch.randn(24, 4 * 4096, generator=g) * 0.02
    hc_scale, hc_base = torch.rand(3, generator=g) + 0.5, torch.randn(24, generator=g) * 0.1
    pool, win_base, comp_rows = C.decode_case_host_pool(case)
    state = dict(pool=pool.float(), win_base=win_base, comp_rows=comp_rows, k_idx=cache.k_idx.cpu().clone(),
                 ring_kv=cache.ring_kv.cpu().clone(), ring_score=cache.ring_score.cpu().clone(),
                 ring_k=cache.ring_k_idx.cpu().clone(), ring_s=cache.ring_s_idx.cpu().clone())
    blk = Lm.DecodeBlock(W.to("cuda"), b, ctx, top_k=512, cache=cache)
    out = blk.step_hc(x.cuda(), pos.cuda(), hc_fn.cuda(), hc_scale.cuda(), hc_base.cuda())
    assert out.shape == (b, 4, 4096) and out.dtype == torch.float32
    ref, post, comb = LR.decode_block_hc_ref(state, W, x, pos, hc_fn, hc_scale, hc_base, top_k=512)
    resid = torch.from_numpy(H.hc_post(np.zeros((b, 4096)), x.numpy(), np.zeros((b, 4)), comb))
    rr = rel_rms(out.double().cpu() - resid, ref - resid)
    assert rr <= BLOCK_REL, f"decode block (hc) rel_rms={rr:.3e}"
    assert_close_bf16(cache.kv_pool.float().cpu(), state["pool"], what="pool after hc step")


def test_decode_block_steps_keep_key_image():
    """Eight decode steps (two block closings per sequence): the incrementally kept key image
    matches a rebuild, and the indexer reading it selects what the split-every-call path selects."""
    Lm = _layer()
    C = importlib.import_module(PKG + ".configs")
    IX = importlib.import_module(PKG + ".indexer")
    b, ctx = 4, 2048
    case = C.make_decode_case(b, ctx, 512, seeds=[400 + i for i in range(b)])
    W = Lm.make_attention_weights(4, quant=True).to("cuda")
    blk = Lm.DecodeBlock(W, b, ctx + 16, top_k=512, cache=case.cache)
    g = torch.Generator().manual_seed(6)
    for step in range(8):  # rewrites entries near the end of the cache (positions below its capacity)
        pos = torch.tensor([ctx - 40 + step + i for i in range(b)], dtype=torch.int32).cuda()
        blk.step(torch.randn(b, 4096, generator=g).cuda(), pos)
    c = case.cache
    fresh = IX.build_key_image(c.k_idx, IX.key_image_buffers(b, c.max_comp, "cuda"))
    assert torch.equal(c.key_image[0], fresh[0])
    assert torch.equal(c.key_image[1], fresh[1])
    q = torch.randn(b, 1, 64, 128, generator=g).cuda()
    w = (torch.randn(b, 1, 64, generator=g) / 8).cuda()
    pos = torch.full((b, 1), ctx + 4, dtype=torch.int32).cuda()
    outs = []
    for kimg, mode in ((c.key_image, 2), (None, 2), (None, 1)):
        out = torch.full((b, 1, 256), -7, dtype=torch.int32, device="cuda")
        IX.indexer_topk_into(out, q, w, c.k_idx, 256, positions=pos, ratio=4, mode=mode, key_image=kimg)
        outs.append(out.cpu())
    assert torch.equal(outs[0], outs[2]) and torch.equal(outs[1], outs[2])


@pytest.mark.parametrize("ratio", [4, 128])
def test_block_runner_host_steps_match_eager_steps(ratio):
    """BlockRunner (pinned host x and positions in, one graph launch per token, pinned host output
    out) against DecodeBlock.step on an identical block, token by token: the same bits, including
    the first, eager, call and the replays after it, and the same cache afterwards."""
    Lm = _layer()
    C = importlib.import_module(PKG + ".configs")
    b, ctx = 3, 2048
    blocks = []
    for _ in range(2):
        if ratio == 4:
            case = C.make_decode_case(b, ctx, 512, seeds=[500 + i for i in range(b)])
            W = Lm.make_attention_weights(8, quant=True).to("cuda")
            blocks.append(Lm.DecodeBlock(W, b, ctx + 16, top_k=512, cache=case.cache))
        else:
            dims = C.LayerDims(ratio=128)
            W = Lm.make_attention_weights(9, dims=dims, quant=True).to("cuda")
            blk = Lm.DecodeBlock(W, b, ctx + 16, dims=dims)
            g = torch.Generator().manual_seed(12)
            blk.cache.kv_pool.copy_(torch.randn(blk.cache.kv_pool.shape, generator=g).to(torch.bfloat16))
            blocks.append(blk)
    eager, hosted = blocks
    runner = Lm.BlockRunner(hosted)
    g = torch.Generator().manual_seed(7)
    for step in range(6):   # positions cross a compressor block end
        x = torch.randn(b, 4096, generator=g)
        pos = torch.tensor([ctx - 30 + step + 5 * i for i in range(b)], dtype=torch.int32)
        want = eager.step(x.cuda(), pos.cuda()).cpu()
        if step % 2:
            hx, hp = runner.host_inputs()
            hx.copy_(x), hp.copy_(pos)
            got = runner.step_host()
        else:
            got = runner.step_host(x, pos)
        runner.synchronize()
        assert torch.equal(got, want), f"step {step}"
    assert torch.equal(eager.cache.kv_pool, hosted.cache.kv_pool)
    if ratio == 4:
        assert torch.equal(eager.cache.ring_kv, hosted.cache.ring_kv)
        assert torch.equal(eager.cache.k_idx, hosted.cache.k_idx)
    runner.release()
