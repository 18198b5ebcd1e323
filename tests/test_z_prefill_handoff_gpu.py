"""Prefill -> decode hand-off of the attention block on the GPU (oracle/decode_engine.py:86-95):
prefill_layer, DecodeBlock.load_prefill, then decode steps, against the oracle doing the same."""
import importlib

import pytest
import torch

from helpers import rel_rms
from oracle import layer_ref as LR

pytestmark = pytest.mark.gpu
PKG = "deepseek-v4-flash-mlx_b200"
# Prefill then decode passes the roundings twice: the state the GPU prefill leaves (bf16 operands and
# rows) moves the oracle's own decode output by 3.5e-3 rel-RMS (measured on the CPU by rounding the
# oracle's prefill the way the GPU does), and the decode pass adds its own (a single block pass is
# held to 1e-2).
HANDOFF_REL = 1.5e-2


def _layer():
    return importlib.import_module(PKG + ".layer")


@pytest.mark.parametrize("ratio", [4, 128])
def test_prefill_then_decode_block(ratio):
    """The hand-off the reference makes between its prefill and its decode steps
    (oracle/decode_engine.py:86-95): prefill_layer over 300 tokens, DecodeBlock.load_prefill, then
    six decode steps (two close a compression block), against the oracle's prefill state loaded
    into a CPU cache and its decode steps."""
    Lm = _layer()
    C = importlib.import_module(PKG + ".configs")
    D = importlib.import_module(PKG + ".decode")
    dims = C.LayerDims(ratio=ratio)
    window_only = C.window_only(dims)
    W = Lm.make_attention_weights(12, dims=dims)
    Wd = W.to("cuda")
    s, k = 300, 6
    x = torch.randn(s + k, 4096, generator=torch.Generator().manual_seed(13))
    _, aux = Lm.prefill_layer(x[:s].cuda(), Wd, dims=dims, return_aux=True)
    blk = Lm.DecodeBlock(Wd, 1, 2048, top_k=512, dims=dims)
    blk.load_prefill(0, aux)
    _, _, _, st = LR.prefill_layer_ref(x[:s], W, top_k=512, ratio=ratio, return_state=True)
    cache = D.SparseMLACache(1, 0 if window_only else 512, ratio=ratio, device="cpu")
    if window_only:
        cache.load_prefill(0, st["kv"])
        state = dict(pool=cache.kv_pool.float(), win_base=cache.win_base)
    else:
        cache.load_prefill(0, st["kv"], st["comp"], st["k_idx"], ring=st["ring"], key_ring=st["key_ring"])
        state = dict(pool=cache.kv_pool.float(), win_base=cache.win_base, comp_rows=cache.comp_rows,
                     k_idx=cache.k_idx.clone(), ring_kv=cache.ring_kv.clone(), ring_score=cache.ring_score.clone(),
                     ring_k=cache.ring_k_idx.clone(), ring_s=cache.ring_s_idx.clone())
    for t in range(s, s + k):
        pos = torch.tensor([t], dtype=torch.int32)
        out = blk.step(x[t:t + 1].cuda(), pos.cuda())
        ref = LR.decode_block_ref(state, W, x[t:t + 1], pos, top_k=512, ratio=ratio)
        rr = rel_rms(out, ref)
        assert rr <= HANDOFF_REL, f"ratio {ratio}, position {t}: rel_rms={rr:.3e}"
