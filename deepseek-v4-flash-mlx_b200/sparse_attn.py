"""Sparse MLA attention ops (reference: ref_torch/sparse_attn.py, v4mlx/sparse_attn.py).

`sparse_attn(q, kv, attn_sink, topk_idxs, scale)` and `get_window_topk_idxs(...)` keep the
reference signatures. kv is consumed as bf16 (the cache format); an fp32 kv is rounded to bf16
once by the library's cast kernel. q may be fp32 or bf16; the output has q's dtype.
"""
import ctypes

import torch

from . import _lib as L


def _attn_params(q, kv, sink, idx, out, scale, freqs=None, positions=None, rope_dim=0, num_splits=0,
                 q_norm_rope=False, q_eps=1e-6, win_base=None, window=0, window_linear=False, kernel=0,
                 pre_wait=False):
    p = L.SparseAttnParams()
    p.q, p.kv, p.sink, p.idx, p.out = L.ptr(q), L.ptr(kv), L.ptr(sink), L.ptr(idx), L.ptr(out)
    p.s, p.n, p.h, p.d, p.t = q.shape[0], kv.shape[0], q.shape[1], q.shape[2], idx.shape[-1]
    p.q_dtype, p.idx_dtype, p.out_dtype = L.dtype_code(q), L.dtype_code(idx), L.dtype_code(out)
    p.scale = scale
    p.rope_freqs = L.ptr(freqs) if freqs is not None else None
    p.positions = L.ptr(positions) if positions is not None else None
    p.rope_dim = rope_dim
    p.num_splits = num_splits
    p.q_norm_rope = int(q_norm_rope)
    p.q_eps = q_eps
    p.win_base = L.ptr(win_base) if win_base is not None else None
    p.win_stride = 1 if (win_base is not None and win_base.numel() > 1) else 0
    p.window = window
    p.window_linear = int(window_linear)
    p.kernel = kernel
    p.pre_wait = int(pre_wait)
    return p


@torch.library.custom_op("dsv4::sparse_attn", mutates_args=(), device_types="cuda")
def _sparse_attn_op(q: torch.Tensor, kv: torch.Tensor, attn_sink: torch.Tensor, topk_idxs: torch.Tensor,
                    scale: float, out_dtype: torch.dtype, rope_freqs: torch.Tensor | None,
                    positions: torch.Tensor | None, rope_dim: int, num_splits: int,
                    q_norm_rope: bool = False, q_eps: float = 1e-6, win_base: torch.Tensor | None = None,
                    window: int = 0, window_linear: bool = False, kernel: int = 0,
                    pre_wait: bool = False) -> torch.Tensor:
    out = torch.empty(q.shape, dtype=out_dtype, device=q.device)
    sparse_attn_into(out, q, kv, attn_sink, topk_idxs, scale, rope_freqs, positions, rope_dim, num_splits, q_norm_rope,
                     q_eps, win_base, window, window_linear, kernel, pre_wait)
    return out


def sparse_attn_into(out, q, kv, attn_sink, topk_idxs, scale, rope_freqs=None, positions=None, rope_dim=0,
                     num_splits=0, q_norm_rope=False, q_eps=1e-6, win_base=None, window=0, window_linear=False,
                     kernel=0, pre_wait=False):
    """The body of `dsv4::sparse_attn` into a caller-owned `out` (q's shape, bf16 or fp32). `out`
    may be pinned host memory (a unified-address pointer): the kernel then stores the result over
    the bus itself, which a decode step captured with its host copies uses to skip the copy back."""
    q = q.contiguous()
    kv = kv.contiguous()
    if kv.dtype != torch.bfloat16:
        kv16 = torch.empty(kv.shape, dtype=torch.bfloat16, device=kv.device)
        L.check(L.lib().dsv4_cast(L.ptr(kv), L.dtype_code(kv), L.ptr(kv16), L.BF16, kv.numel(), L.stream_of(q)))
        kv = kv16
    sink = attn_sink.float().contiguous()
    idx = topk_idxs.contiguous()
    p = _attn_params(q, kv, sink, idx, out, scale, rope_freqs, positions, rope_dim, num_splits, q_norm_rope, q_eps,
                     win_base, window, window_linear, kernel, pre_wait)
    nbytes = L.lib().dsv4_sparse_attn_workspace_size(ctypes.byref(p))
    ws = L.workspace(nbytes, q.device)
    p.workspace, p.workspace_bytes = L.ptr(ws), nbytes
    L.check(L.lib().dsv4_sparse_attn(ctypes.byref(p), L.stream_of(q)))
    return out


@_sparse_attn_op.register_fake
def _(q, kv, attn_sink, topk_idxs, scale, out_dtype, rope_freqs, positions, rope_dim, num_splits, q_norm_rope=False,
      q_eps=1e-6, win_base=None, window=0, window_linear=False, kernel=0, pre_wait=False):
    return torch.empty(q.shape, dtype=out_dtype, device=q.device)


def sparse_attn(q, kv, attn_sink, topk_idxs, scale, kernel=0):
    """q [s,h,d], kv [n,d], attn_sink [h], topk_idxs [s,T] (-1 masked) -> o [s,h,d].

    o = sum_t softmax-numerator_t kv[idx_t] / (sum_t numerator_t + exp(sink_h - rowmax)),
    the reference's dense-gather formula (ref_torch/sparse_attn.py:23-34). `kernel` picks the
    implementation (0 automatic, 1 mma.sync split-K, 2 tcgen05; same function)."""
    L.require_cuda(q, kv, attn_sink, topk_idxs)
    if topk_idxs.dim() == 3 and topk_idxs.shape[0] == 1:
        topk_idxs = topk_idxs[0]
    if topk_idxs.dtype not in (torch.int32, torch.int64):
        topk_idxs = topk_idxs.long()
    return _sparse_attn_op(q, kv, attn_sink, topk_idxs, float(scale), q.dtype, None, None, 0, 0, kernel=int(kernel))


def sparse_attn_rope(q, kv, attn_sink, topk_idxs, scale, positions, freqs, rope_dim=64,
                     out_dtype=torch.bfloat16, num_splits=0, win_base=None, window=0, window_linear=False,
                     kernel=0):
    """sparse_attn followed by the inverse rope of the output's last rope_dim dims at `positions`
    (oracle/decode_engine.py:118, oracle/v4_fast.py:119), fused into the attention epilogue. With
    `win_base` (int64, one per query or a single value) the list of query i is [window rows | topk_idxs[i]],
    the window rows computed in the kernel (decode ring order, or linear with window_linear)."""
    L.require_cuda(q, kv, attn_sink, topk_idxs, positions, freqs, win_base)
    return _sparse_attn_op(q, kv, attn_sink, topk_idxs, float(scale), out_dtype, freqs.float().contiguous(),
                           positions.to(torch.int32).contiguous(), int(rope_dim), int(num_splits), False, 1e-6,
                           win_base, int(window), bool(window_linear), int(kernel))


def sparse_attn_decode(q_raw, kv, attn_sink, topk_idxs, scale, positions, freqs, rope_dim=64, eps=1e-6,
                       out_dtype=torch.bfloat16, num_splits=0, kernel=0):
    """The decode attention of oracle/v4_fast.py:88-119 in one op: q_raw (the q_up output) gets the
    weightless per-head norm and RoPE at `positions` while it is staged, then sparse attention over
    topk_idxs, then the inverse RoPE of the output in the epilogue."""
    L.require_cuda(q_raw, kv, attn_sink, topk_idxs, positions, freqs)
    return _sparse_attn_op(q_raw, kv, attn_sink, topk_idxs, float(scale), out_dtype, freqs.float().contiguous(),
                           positions.to(torch.int32).contiguous(), int(rope_dim), int(num_splits), True, float(eps),
                           kernel=int(kernel))


@torch.library.custom_op("dsv4::get_window_topk_idxs", mutates_args=(), device_types="cuda")
def _window_op(anchor: torch.Tensor, window_size: int, bsz: int, seqlen: int, start_pos: int) -> torch.Tensor:
    cols = window_size if start_pos > 0 else min(seqlen, window_size)
    out = torch.empty((bsz, seqlen, cols), dtype=torch.int32, device=anchor.device)
    L.check(L.lib().dsv4_window_topk_idxs(window_size, bsz, seqlen, start_pos, L.ptr(out), L.stream_of(anchor)))
    return out


@_window_op.register_fake
def _(anchor, window_size, bsz, seqlen, start_pos):
    cols = window_size if start_pos > 0 else min(seqlen, window_size)
    return torch.empty((bsz, seqlen, cols), dtype=torch.int32, device=anchor.device)


def get_window_topk_idxs(window_size, bsz, seqlen, start_pos, device="cuda"):
    """Window index matrix of ref_torch/sparse_attn.py:9-20 (all three branches), int32 on device.
    Shape [bsz, seqlen, cols]; for start_pos > 0 the reference's single row is repeated per query."""
    anchor = torch.empty(0, device=device)
    L.require_cuda(anchor)
    return _window_op(anchor, int(window_size), int(bsz), int(seqlen), int(start_pos))
