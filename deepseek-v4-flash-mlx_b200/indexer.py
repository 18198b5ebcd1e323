"""Lightning indexer + top-k selection.

The reference has no indexer: it attends to every visible compressed row
(oracle/decode_engine.py:112-114, oracle/v4_fast.py:114-117). This op scores the visible
compressed keys, score[j] = sum_h w[h] * relu(q[h] . k[j]) in fp32 with a fixed rounding order,
and keeps the top_k keys by (score desc, index asc), written in ascending key order and padded
with -1. When top_k >= the visible count it returns exactly the reference's list.
"""
import ctypes

import torch

from . import _lib as L


def _params(q, w, k, out, top_k, positions, ratio, out_col, out_offset, block_table, page, scores_out,
            win_base=None, window=0, window_linear=False, mode=0, key_image=None):
    b, s, h, di = q.shape
    p = L.IndexerParams()
    p.q, p.w, p.k, p.out = L.ptr(q), L.ptr(w), L.ptr(k), L.ptr(out)
    p.scores_out = L.ptr(scores_out) if scores_out is not None else None
    p.batch, p.s, p.heads, p.n_keys, p.top_k = b, s, h, k.shape[1], top_k
    p.k_batch_stride = k.shape[1]
    p.positions = L.ptr(positions) if positions is not None else None
    p.ratio = ratio
    p.out_stride, p.out_col, p.out_offset = out.shape[-1], out_col, out_offset
    p.block_table = L.ptr(block_table) if block_table is not None else None
    p.table_stride = block_table.shape[-1] if block_table is not None else 0
    p.page = page
    p.win_base = L.ptr(win_base) if win_base is not None else None
    p.window = window
    p.window_linear = int(window_linear)
    p.mode = mode
    if key_image is not None:
        img, inv, nmax = key_image
        p.key_image, p.key_inv, p.key_norm_max = L.ptr(img), L.ptr(inv), L.ptr(nmax)
    return p


def key_image_buffers(batch, max_keys, device):
    """Zeroed buffers of a decode cache's key image for `max_keys` keys per batch entry:
    (image uint8 [batch * tiles * 64 KB], inverse scales fp32 [batch, tiles * 128], norm max fp32 [batch])."""
    tiles = (max_keys + 127) // 128
    img = torch.zeros(batch * tiles * L.KEY_TILE_BYTES, dtype=torch.uint8, device=device)
    return img, torch.zeros(batch, tiles * 128, dtype=torch.float32, device=device), \
        torch.zeros(batch, dtype=torch.float32, device=device)


def build_key_image(k_idx, key_image, n_keys=None):
    """(Re)build the key image (dsv4_indexer_key_image) of keys [0, n_keys) of every batch entry of
    k_idx [batch, max_keys, 128] fp32 into the buffers of key_image_buffers."""
    L.require_cuda(k_idx)
    img, inv, nmax = key_image
    b, stride = k_idx.shape[0], k_idx.shape[1]
    p = L.KeyImageParams()
    p.k, p.batch, p.n_keys, p.k_batch_stride = L.ptr(k_idx), b, stride if n_keys is None else int(n_keys), stride
    p.image, p.inv, p.norm_max = L.ptr(img), L.ptr(inv), L.ptr(nmax)
    L.check(L.lib().dsv4_indexer_key_image(ctypes.byref(p), L.stream_of(k_idx)))
    return key_image


def _run(p, device, stream_ref):
    nbytes = L.lib().dsv4_indexer_topk_workspace_size(ctypes.byref(p))
    ws = L.workspace(nbytes, device)
    p.workspace, p.workspace_bytes = L.ptr(ws), nbytes
    L.check(L.lib().dsv4_indexer_topk(ctypes.byref(p), L.stream_of(stream_ref)))


@torch.library.custom_op("dsv4::indexer_topk", mutates_args=(), device_types="cuda")
def _indexer_op(q_idx: torch.Tensor, w: torch.Tensor, k_idx: torch.Tensor, top_k: int,
                positions: torch.Tensor | None, ratio: int, mode: int = 0) -> torch.Tensor:
    b, s = q_idx.shape[0], q_idx.shape[1]
    out = torch.empty((b, s, top_k), dtype=torch.int32, device=q_idx.device)
    p = _params(q_idx, w, k_idx, out, top_k, positions, ratio, 0, 0, None, 0, None, mode=mode)
    _run(p, q_idx.device, q_idx)
    return out


@_indexer_op.register_fake
def _(q_idx, w, k_idx, top_k, positions, ratio, mode=0):
    return torch.empty((q_idx.shape[0], q_idx.shape[1], top_k), dtype=torch.int32, device=q_idx.device)


def _prep(q_idx, w, k_idx, positions):
    L.require_cuda(q_idx, w, k_idx, positions)
    squeeze = q_idx.dim() == 3
    if squeeze:  # [s, h, d] -> [1, s, h, d]
        q_idx, w, k_idx = q_idx[None], w[None], k_idx[None]
        if positions is not None:
            positions = positions.reshape(1, -1)
    if q_idx.dtype != torch.float32 or w.dtype != torch.float32 or k_idx.dtype != torch.float32:
        raise TypeError("indexer: q_idx, w and k_idx must be float32 (scores are computed in fp32)")
    if positions is not None:
        positions = positions.to(torch.int32).contiguous()
    return q_idx.contiguous(), w.contiguous(), k_idx.contiguous(), positions, squeeze


def indexer_topk(q_idx, w, k_idx, top_k, positions=None, ratio=4, mode=0):
    """q_idx [b, s, 64, 128] (or [s, 64, 128]), w [b, s, 64], k_idx [b, n, 128] fp32 ->
    int32 [b, s, top_k] key indices. With `positions`, query i sees keys j < (positions[i]+1)//ratio
    (the causal compressed-block rule of oracle/decode_engine.py:112). `mode`: 1 scores every key
    in the fixed fp32 order, 2 filters with tensor-core scores and rescores the uncertain band
    exactly, 0 picks (2 for prefill-shaped calls); the result is the same bit for bit."""
    q_idx, w, k_idx, positions, squeeze = _prep(q_idx, w, k_idx, positions)
    out = _indexer_op(q_idx, w, k_idx, int(top_k), positions, int(ratio), int(mode))
    return out[0] if squeeze else out


def indexer_scores(q_idx, w, k_idx, positions=None, ratio=4, mode=1):
    """Raw fp32 scores [b, s, n] (entries beyond each query's visible range are left undefined);
    exposed for verification against the CPU oracle. mode 1: the exact scores; mode 2: the
    tensor-core approximate scores of the filter stage."""
    q_idx, w, k_idx, positions, squeeze = _prep(q_idx, w, k_idx, positions)
    b, s = q_idx.shape[0], q_idx.shape[1]
    scores = torch.full((b, s, k_idx.shape[1]), float("nan"), dtype=torch.float32, device=q_idx.device)
    out = torch.empty((b, s, 1), dtype=torch.int32, device=q_idx.device)
    p = _params(q_idx, w, k_idx, out, 1, positions, ratio, 0, 0, None, 0, scores, mode=int(mode))
    _run(p, q_idx.device, q_idx)
    return scores[0] if squeeze else scores


def indexer_topk_into(out, q_idx, w, k_idx, top_k, positions=None, ratio=4, out_col=0, out_offset=0,
                      block_table=None, page=0, win_base=None, window=0, window_linear=False, mode=0,
                      key_image=None):
    """Write the selection into columns [out_col, out_col+top_k) of an existing int32 index buffer
    out [b, s, T], mapping key j to pool row out_offset + j, or through a block table
    (block_table[b, j // page] * page + j % page + out_offset). Used by the decode and prefill
    pipelines to build the attention index list without a copy. With `win_base` (int64 [b]) the
    window rows of each query also go to columns [out_col - window, out_col): the decode ring order
    at positions[b], or with window_linear the prefill rows win_base + max(0, p-window+1) .. p.
    `key_image` (the buffers of key_image_buffers, kept current for k_idx) lets the tensor-core
    filter read the keys' split form instead of splitting them on every call."""
    q_idx, w, k_idx, positions, _ = _prep(q_idx, w, k_idx, positions)
    if out.dtype != torch.int32 or not out.is_contiguous():
        raise TypeError("indexer_topk_into: out must be a contiguous int32 tensor")
    p = _params(q_idx, w, k_idx, out, int(top_k), positions, int(ratio), int(out_col), int(out_offset),
                block_table, int(page), None, win_base, int(window), window_linear, int(mode), key_image)
    _run(p, q_idx.device, q_idx)
    return out
