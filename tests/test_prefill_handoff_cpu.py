"""Prefill -> decode hand-off on the CPU, through the oracle and a CPU-resident cache: the state a
prefill of s tokens leaves (window rows, compressed rows, indexer keys, both compressors' rings),
loaded with SparseMLACache.load_prefill, lets k decode steps reproduce what a prefill of s + k tokens
computes for those tokens (oracle/decode_engine.py:86-95 and :96-118 describe the same layer)."""
import importlib

import pytest
import torch

from helpers import rel_rms
from oracle import layer_ref as LR

PKG = "deepseek-v4-flash-mlx_b200"
# the decode state holds bf16 rows where the prefill keeps fp32 ones: a few 1e-3 of difference
TOL = 1e-2


@pytest.mark.parametrize("ratio", [4, 128])
def test_prefill_then_decode_equals_longer_prefill(ratio):
    Lm = importlib.import_module(PKG + ".layer")
    C = importlib.import_module(PKG + ".configs")
    D = importlib.import_module(PKG + ".decode")
    dims = C.LayerDims(dim=512, q_lora=256, ratio=ratio)
    W = Lm.make_attention_weights(11, dims=dims)
    s, k = 130, 6  # the window has wrapped; the decode steps close two compression blocks (p = 131, 135)
    x = torch.randn(s + k, 512, generator=torch.Generator().manual_seed(12))
    full, _, _ = LR.prefill_layer_ref(x, W, top_k=512, ratio=ratio)
    _, _, _, st = LR.prefill_layer_ref(x[:s], W, top_k=512, ratio=ratio, return_state=True)
    window_only = C.window_only(dims)
    cache = D.SparseMLACache(1, 0 if window_only else 64, ratio=ratio, device="cpu",
                             page_order=None if window_only else torch.tensor([0]))
    if window_only:
        cache.load_prefill(0, st["kv"])
        state = dict(pool=cache.kv_pool.float(), win_base=cache.win_base)
    else:
        cache.load_prefill(0, st["kv"], st["comp"], st["k_idx"], ring=st["ring"], key_ring=st["key_ring"])
        state = dict(pool=cache.kv_pool.float(), win_base=cache.win_base, comp_rows=cache.comp_rows,
                     k_idx=cache.k_idx.clone(), ring_kv=cache.ring_kv.clone(), ring_score=cache.ring_score.clone(),
                     ring_k=cache.ring_k_idx.clone(), ring_s=cache.ring_s_idx.clone())
    for t in range(s, s + k):
        out = LR.decode_block_ref(state, W, x[t:t + 1], torch.tensor([t], dtype=torch.int32), top_k=512, ratio=ratio)
        rr = rel_rms(out[0], full[t])
        assert rr <= TOL, f"ratio {ratio}, position {t}: rel_rms={rr:.3e}"


def test_load_prefill_places_rows_keys_and_rings():
    """Where load_prefill puts each part: the last 128 kv rows in ring slots p % 128, compressed
    entry j at its block-table row, keys at entry j, the rings of sequence b."""
    D = importlib.import_module(PKG + ".decode")
    g = torch.Generator().manual_seed(4)
    perm = torch.randperm(2 * 2, generator=g).to(torch.int32)
    c = D.SparseMLACache(2, 100, device="cpu", page_order=perm)
    s = 300
    rows = torch.randn(s, 512, generator=g).to(torch.bfloat16)
    comp = torch.randn(s // 4 - 5, 512, generator=g).to(torch.bfloat16)
    keys = torch.randn(comp.shape[0], 128, generator=g)
    ring = (torch.randn(1, 8, 1024, generator=g), torch.randn(1, 8, 1024, generator=g))
    kring = (torch.randn(1, 8, 256, generator=g), torch.randn(1, 8, 256, generator=g))
    c.load_prefill(1, rows, comp, keys, ring=ring, key_ring=kring)
    for p in (s - 128, s - 1, 250):
        assert torch.equal(c.kv_pool[int(c.win_base[1]) + p % 128], rows[p])
    for j in (0, 63, 64, comp.shape[0] - 1):
        assert torch.equal(c.kv_pool[int(c.comp_rows(1, torch.tensor(j)))], comp[j])
    assert torch.equal(c.k_idx[1, :comp.shape[0]], keys) and c.image_stale
    assert torch.equal(c.ring_kv[1], ring[0][0]) and torch.equal(c.ring_s_idx[1], kring[1][0])
    assert torch.equal(c.ring_kv[0], torch.zeros(8, 1024))  # the other sequence is untouched
    with pytest.raises(ValueError):
        c.load_prefill(0, rows, torch.zeros(101, 512), torch.zeros(101, 128))


def test_block_load_prefill_rejects_a_window_only_state():
    Lm = importlib.import_module(PKG + ".layer")
    C = importlib.import_module(PKG + ".configs")
    dims = C.LayerDims(dim=256, q_lora=128)
    blk = Lm.DecodeBlock(Lm.make_attention_weights(0, dims=dims), 1, 256, dims=dims, device="cpu")
    aux = dict(q=torch.zeros(10, 64, 512), kvcat=torch.zeros(10, 512))   # what a window-only prefill returns
    with pytest.raises(ValueError, match="window-only"):
        blk.load_prefill(0, aux)
