"""The decode attention path (configs 2 and 3, reduced context) against the CPU oracle."""
import importlib

import numpy as np
import pytest
import torch

from helpers import assert_close_bf16
from oracle import layer_ref as LR
from oracle import norm_rope_ref as NR

pytestmark = pytest.mark.gpu


def _cfg():
    return importlib.import_module("deepseek-v4-flash-mlx_b200.configs")


@pytest.mark.parametrize("batch,ctx,top_k", [(1, 32768, 512), (4, 8192, 512), (3, 1000, 512), (2, 60, 16),
                                             (2, 2048, 64)])
def test_decode_attention_matches_oracle(dsv4, batch, ctx, top_k):
    C = _cfg()
    case = C.make_decode_case(batch, ctx, top_k, seeds=[100 + i for i in range(batch)])
    if ctx < 128:  # young sequences: only positions 0..ctx-1 of the window ring are valid
        pass
    out = dsv4.decode_attention(case.cache, case.q, case.q_idx, case.w_idx, case.sink, case.positions, top_k,
                                out_dtype=torch.float32)
    pool, win_base, comp_rows = C.decode_case_host_pool(case)
    f = NR.precompute_freqs(64, 0, 65536, 160000.0, 16, 32, 1)
    h = case.host
    ref = LR.decode_attention_ref(pool, win_base, comp_rows, h["k_idx"], h["q"], h["q_idx"], h["w_idx"], h["sink"],
                                  h["positions"], top_k, f)
    assert_close_bf16(out, ref, what=f"decode b={batch} ctx={ctx}")


def test_decode_indices_bit_exact(dsv4):
    """The attention index list: window rows in the reference's ring order (written by the selection
    kernel's window option) + the indexer's selection mapped through the block table."""
    C = _cfg()
    case = C.make_decode_case(2, 8192, 512, seeds=[100, 101])
    b = 2
    idx = torch.empty((b, 128 + 512), dtype=torch.int32, device="cuda")
    pos = case.positions
    dsv4.indexer_topk_into(idx.view(b, 1, -1), case.q_idx.view(b, 1, 64, 128), case.w_idx.view(b, 1, 64),
                           case.cache.k_idx, 512, pos.view(b, 1), 4, out_col=128, out_offset=case.cache.comp_base,
                           block_table=case.cache.block_table, page=case.cache.page, win_base=case.cache.win_base,
                           window=128)
    pool, win_base, comp_rows = C.decode_case_host_pool(case)
    f = NR.precompute_freqs(64, 0, 65536, 160000.0, 16, 32, 1)
    h = case.host
    _, ref_idx = LR.decode_attention_ref(pool, win_base, comp_rows, h["k_idx"], h["q"], h["q_idx"], h["w_idx"],
                                         h["sink"], h["positions"], 512, f, return_indices=True)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_idx.numpy())


def test_implicit_window_equals_explicit_list(dsv4):
    """sparse attention with the window computed in the kernel equals the same list given explicitly."""
    C = _cfg()
    for ctx in (8192, 77, 4096):
        case = C.make_decode_case(2, ctx, 64 if ctx != 4096 else 512, seeds=[7, 8])
        b = 2
        k = 64 if ctx != 4096 else 512
        full = torch.empty((b, 128 + k), dtype=torch.int32, device="cuda")
        dsv4.indexer_topk_into(full.view(b, 1, -1), case.q_idx.view(b, 1, 64, 128), case.w_idx.view(b, 1, 64),
                               case.cache.k_idx, k, case.positions.view(b, 1), 4, out_col=128,
                               out_offset=case.cache.comp_base, block_table=case.cache.block_table,
                               page=case.cache.page, win_base=case.cache.win_base, window=128)
        f = dsv4.rope_freqs(64, "cuda")
        q = torch.randn(b, 64, 512, device="cuda").to(torch.bfloat16)
        # same split count on both sides (the accumulation order then matches exactly); splits 1-3 put
        # window and selected rows in one CTA (a range spanning the window boundary)
        for splits in (0, 1, 2, 3):
            a = dsv4.sparse_attn_rope(q, case.cache.kv_pool, case.sink, full, 512 ** -0.5, case.positions, f,
                                      out_dtype=torch.float32, num_splits=splits)
            bb = dsv4.sparse_attn_rope(q, case.cache.kv_pool, case.sink, full[:, 128:].contiguous(), 512 ** -0.5,
                                       case.positions, f, out_dtype=torch.float32, win_base=case.cache.win_base,
                                       window=128, num_splits=splits)
            torch.testing.assert_close(a, bb, rtol=0, atol=0, msg=f"ctx={ctx} splits={splits}")


@pytest.mark.parametrize("b", [1, 20])   # the fused three-kernel step; the side-stream split step
def test_decode_runner_graph_and_host_path(dsv4, b):
    C = _cfg()
    case = C.make_decode_case(b, 4096, 512, seeds=list(range(1, b + 1)))
    r = dsv4.DecodeRunner(case.cache, case.sink, 512, out_dtype=torch.float32)
    r.q.copy_(case.q), r.q_idx.copy_(case.q_idx), r.w_idx.copy_(case.w_idx), r.positions.copy_(case.positions)
    dev_out = r.step_device().clone()
    ref = dsv4.decode_attention(case.cache, case.q, case.q_idx, case.w_idx, case.sink, case.positions, 512,
                                out_dtype=torch.float32)
    torch.testing.assert_close(dev_out, ref, rtol=0, atol=0)
    h = case.host
    out = r.step_host(h["q"], h["q_idx"], h["w_idx"], h["positions"])   # staged through host_inputs()
    r.synchronize()
    torch.testing.assert_close(out, ref.cpu(), rtol=0, atol=0)
    # the zero-copy path: inputs written straight into the runner's pinned block
    r.synchronize()
    out.zero_()
    for dst, key in zip(r.host_inputs(), ("q", "q_idx", "w_idx", "positions")):
        dst.copy_(h[key])
    out = r.step_host(*r.host_inputs())
    r.synchronize()
    torch.testing.assert_close(out, ref.cpu(), rtol=0, atol=0)


def test_decode_rows_bookkeeping(dsv4):
    """One launch computes this step's window slot, compressed row and indexer key row for every
    sequence, as the cache's own host-side formulas; an entry past the cache raises the device
    error word and is clamped."""
    D = importlib.import_module("deepseek-v4-flash-mlx_b200.decode")
    L = importlib.import_module("deepseek-v4-flash-mlx_b200._lib")
    g = torch.Generator().manual_seed(9)
    b, max_comp = 6, 700
    perm = torch.randperm(6 * 11, generator=g)
    cache = D.SparseMLACache(b, max_comp, page=64, page_order=perm)
    pos = torch.tensor([0, 1, 2, 3, 4 * max_comp - 1, 1234], dtype=torch.int32)
    L.device_error()
    win, comp, key = (t.cpu() for t in D.decode_rows(cache, pos.cuda()))
    assert L.device_error() == 0
    entry = torch.clamp((pos.long() + 1) // 4 - 1, min=0)
    bt = cache.block_table.cpu().long()
    seq = torch.arange(b)
    assert torch.equal(win, cache.win_base.cpu() + pos.long() % cache.window)
    assert torch.equal(comp, cache.comp_base + bt[seq, entry // 64] * 64 + entry % 64)
    assert torch.equal(key, seq * max_comp + entry)
    over = torch.tensor([4 * max_comp + 3], dtype=torch.int32)     # entry max_comp: outside the cache
    D.decode_rows(D.SparseMLACache(1, max_comp), over.cuda())
    assert L.device_error() == 4


def test_copy_kernel_between_pinned_host_and_device(dsv4):
    """dsv4_copy moves bytes between pinned host memory and the device by kernel loads and stores
    (the serving step's staging); misaligned sizes are refused."""
    L = importlib.import_module("deepseek-v4-flash-mlx_b200._lib")
    src = torch.arange(100_000, dtype=torch.int32).pin_memory()
    dev = torch.empty(100_000, dtype=torch.int32, device="cuda")
    back = torch.zeros(100_000, dtype=torch.int32).pin_memory()
    L.copy_(dev, src)
    L.copy_(back, dev)
    torch.cuda.synchronize()
    assert torch.equal(dev.cpu(), src) and torch.equal(back, src)
    with pytest.raises(L.Dsv4Error):
        L.copy_(dev[:3], src[:3])     # 12 bytes: not a multiple of 16
