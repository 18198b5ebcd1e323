"""The allocation-free indexer entry point, called through the C ABI.

Some callers cannot allocate device memory while they run the indexer: an engine that hands out
all GPU memory from its own pool, a plugin that must not synchronise mid-step (cudaMalloc and
cudaFree may), or code running while another component's stream capture is open.
dsv4_indexer_topk_noalloc serves them with a scratch array built into the library. This test checks
that, on two calls in a row with different inputs, it returns exactly what the allocating entry
point dsv4_indexer_topk returns (index selections are compared bit for bit, the tolerance every
indexer test uses), and that a request larger than the built-in scratch is refused.
This file is collected last so that a stopped-at-first-failure run has already run everything else.
"""
import ctypes
import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu
L = importlib.import_module("deepseek-v4-flash-mlx_b200._lib")


def _inputs(b, s, n, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, s, 64, 128, generator=g).cuda()
    w = (torch.randn(b, s, 64, generator=g) / 8).cuda()
    k = torch.randn(b, n, 128, generator=g).cuda()
    pos = torch.randint(4 * n // 2, 4 * n + 8, (b, s), generator=g).to(torch.int32).cuda()
    return q, w, k, pos


def _params(q, w, k, pos, out, top_k, ws=None):
    p = L.IndexerParams()
    p.q, p.w, p.k, p.out = q.data_ptr(), w.data_ptr(), k.data_ptr(), out.data_ptr()
    p.scores_out = None
    p.batch, p.s, p.heads, p.n_keys, p.top_k = q.shape[0], q.shape[1], 64, k.shape[1], top_k
    p.k_batch_stride = k.shape[1]
    p.positions, p.ratio = pos.data_ptr(), 4
    p.out_stride, p.out_col, p.out_offset = out.shape[-1], 0, 0
    p.block_table, p.table_stride, p.page = None, 0, 0
    p.workspace = ws.data_ptr() if ws is not None else None
    p.workspace_bytes = ws.numel() if ws is not None else 0
    return p


def _decode_layout(p, b, n, page=64, window=128, out_col=128, seed=0):
    """A decode engine's call: keys mapped through a shuffled block table into pool rows after each
    sequence's window ring, the window rows written to the first `window` columns."""
    g = torch.Generator().manual_seed(seed)
    pages = (n + page - 1) // page
    table = torch.randperm(b * pages, generator=g).to(torch.int32).reshape(b, pages).cuda()
    win_base = (torch.arange(b, dtype=torch.int64) * window).cuda()
    p.block_table, p.table_stride, p.page = table.data_ptr(), pages, page
    p.out_col, p.out_offset = out_col, b * window
    p.win_base, p.window, p.window_linear = win_base.data_ptr(), window, 0
    return table, win_base


CASES = [  # (batch, queries per row, keys, top_k, seed, mode of the allocating call, decode layout)
    (2, 3, 3000, 512, 21, 0, False),
    (1, 2, 8192, 512, 22, 0, False),
    (1, 128, 4096, 512, 23, 1, False),  # s >= 64: the allocating call takes the query-tiled score kernel
    (3, 1, 2048, 512, 24, 0, True),     # block table, window columns, out_col > 0
]


def test_noalloc_indexer_matches_allocating_entry_point():
    lib = L.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call, (b, s, n, top_k, seed, mode, decode) in enumerate(CASES):
        q, w, k, pos = _inputs(b, s, n, seed)
        width = top_k + (128 if decode else 0)
        ref = torch.full((b, s, width), -7, dtype=torch.int32, device="cuda")
        p_ref = _params(q, w, k, pos, ref, top_k)
        p_ref.mode = mode
        keep = _decode_layout(p_ref, b, n, seed=seed) if decode else None
        ws = torch.empty(max(1, lib.dsv4_indexer_topk_workspace_size(ctypes.byref(p_ref))), dtype=torch.uint8,
                         device="cuda")
        p_ref.workspace, p_ref.workspace_bytes = ws.data_ptr(), ws.numel()
        assert lib.dsv4_indexer_topk(ctypes.byref(p_ref), stream) == 0, lib.dsv4_last_error()
        for rep in range(2):   # two calls in a row on the shared scratch
            got = torch.full((b, s, width), -7, dtype=torch.int32, device="cuda")
            p = _params(q, w, k, pos, got, top_k)
            if decode:
                p.block_table, p.table_stride, p.page = p_ref.block_table, p_ref.table_stride, p_ref.page
                p.out_col, p.out_offset = p_ref.out_col, p_ref.out_offset
                p.win_base, p.window, p.window_linear = p_ref.win_base, p_ref.window, 0
            assert lib.dsv4_indexer_topk_noalloc(ctypes.byref(p), stream) == 0, lib.dsv4_last_error()
            torch.cuda.synchronize()
            assert torch.equal(got, ref), f"case {call} call {rep}: allocation-free selection differs"
            assert (got >= -1).all()
        del keep


def test_noalloc_indexer_rejects_oversized_requests():
    lib = L.load()
    q, w, k, pos = _inputs(1, 1, 64, 5)
    out = torch.empty((1, 1, 8), dtype=torch.int32, device="cuda")
    p = _params(q, w, k, pos, out, 8)
    p.batch, p.s, p.n_keys = 200, 100, 8192            # 163,840,000 scores > 1 Mi scratch
    p.k_batch_stride = 8192                             # refused on size, before any launch
    assert lib.dsv4_indexer_topk_noalloc(ctypes.byref(p), None) == 6
    assert b"exceeds the built-in scratch" in lib.dsv4_last_error()
    ws = torch.empty(16, dtype=torch.uint8, device="cuda")
    p2 = _params(q, w, k, pos, out, 8, ws)
    assert lib.dsv4_indexer_topk_noalloc(ctypes.byref(p2), None) == 1   # workspace must be NULL
    p3 = _params(q, w, k, pos, out, 8)
    p3.mode = 3                                                          # unknown mode, as the allocating call
    assert lib.dsv4_indexer_topk_noalloc(ctypes.byref(p3), None) == 1
    p4 = _params(q, w, k, pos, out, 8)
    p4.key_image = k.data_ptr()                                          # half of the key-image triple
    assert lib.dsv4_indexer_topk_noalloc(ctypes.byref(p4), None) == 1
    assert b"go together" in lib.dsv4_last_error()
