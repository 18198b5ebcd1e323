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
