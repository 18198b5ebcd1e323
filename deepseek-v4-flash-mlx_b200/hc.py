"""Hyper-connections around the attention block (reference: ref_torch/hc.py:18-80, the official
Block.hc_pre / hc_post and ParallelHead.hc_head), with the reference signatures.

The residual stream carries hc = 4 copies of the hidden state per token. `hc_pre` mixes them into
the block input (a 24-way projection of the normalised copies, sigmoid gates and a 4x4 Sinkhorn
matrix) in one kernel per token, optionally also producing the block's RMSNorm of that input in
bf16 (the projections' operand); `hc_post` folds the block output back into the 4 copies.
"""
import ctypes

import torch

from . import _lib as L


def _hc_call(x, hc_fn, hc_scale, hc_base, head, norm_w=None, norm_eps=1e-6, hc_eps=1e-6, sinkhorn_iters=20,
             y_norm_dtype=torch.bfloat16, y_norm_eps=1e-6, want_y=True):
    L.require_cuda(x, hc_fn, hc_scale, hc_base, norm_w)
    shape = x.shape
    hc, dim = shape[-2], shape[-1]
    xf = x.float().contiguous()
    rows = xf.numel() // (hc * dim)
    dev = x.device
    y = torch.empty((*shape[:-2], dim), dtype=torch.float32, device=dev) if want_y else None
    post = None if head else torch.empty((*shape[:-2], hc), dtype=torch.float32, device=dev)
    comb = None if head else torch.empty((*shape[:-2], hc, hc), dtype=torch.float32, device=dev)
    y_norm = torch.empty((*shape[:-2], dim), dtype=y_norm_dtype, device=dev) if norm_w is not None else None
    p = L.HcParams()
    keep = (hc_fn.float().contiguous(), hc_scale.float().contiguous(), hc_base.float().contiguous())
    p.x, p.fn, p.scale, p.base = L.ptr(xf), L.ptr(keep[0]), L.ptr(keep[1]), L.ptr(keep[2])
    p.y, p.post, p.comb = L.ptr(y), L.ptr(post), L.ptr(comb)
    if norm_w is not None:
        nw = norm_w if norm_w.dtype in (torch.float32, torch.bfloat16) else norm_w.float()
        keep = keep + (nw.contiguous(),)
        p.norm_w, p.norm_dtype = L.ptr(keep[-1]), L.dtype_code(keep[-1])
        p.y_norm, p.y_norm_dtype = L.ptr(y_norm), L.dtype_code(y_norm)
    p.rows, p.hc, p.dim, p.sinkhorn_iters, p.head = rows, hc, dim, int(sinkhorn_iters), int(head)
    nbytes = L.lib().dsv4_hc_workspace_size(rows, hc, dim, int(head))
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=dev)
    p.workspace, p.workspace_bytes = L.ptr(ws), ws.numel()
    p.norm_eps, p.hc_eps, p.y_norm_eps = float(norm_eps), float(hc_eps), float(y_norm_eps)
    L.check(L.lib().dsv4_hc_pre(ctypes.byref(p), L.stream_of(x)))
    return y, post, comb, y_norm


def hc_pre(x, hc_fn, hc_scale, hc_base, hc=4, norm_eps=1e-6, sinkhorn_iters=20, hc_eps=1e-6, norm_w=None,
           y_norm_eps=1e-6):
    """ref_torch/hc.py:46 hc_pre: x [b, s, hc, dim] -> (y [b, s, dim], post [b, s, hc], comb [b, s, hc, hc]).
    With `norm_w` (the block's attn_norm weight) a fourth output is the block's RMSNorm of y in
    bf16, computed in the same launch."""
    if x.shape[-2] != hc:
        raise ValueError("hc_pre: x's hc axis does not match hc")
    y, post, comb, yn = _hc_call(x, hc_fn, hc_scale, hc_base, 0, norm_w, norm_eps, hc_eps, sinkhorn_iters,
                                 y_norm_eps=y_norm_eps)
    return (y, post, comb) if norm_w is None else (y, post, comb, yn)


def hc_head(x, hc_fn, hc_scale, hc_base, hc=4, norm_eps=1e-6, hc_eps=1e-6):
    """ref_torch/hc.py:72 hc_head: x [b, s, hc, dim] -> y [b, s, dim] (pre gates only)."""
    return _hc_call(x, hc_fn, hc_scale, hc_base, 1, None, norm_eps, hc_eps)[0]


def hc_post(x, residual, post, comb):
    """ref_torch/hc.py:63 hc_post: x [b, s, dim], residual [b, s, hc, dim], post [b, s, hc],
    comb [b, s, hc, hc] -> [b, s, hc, dim]."""
    L.require_cuda(x, residual, post, comb)
    hc, dim = residual.shape[-2], residual.shape[-1]
    xf, rf = x.float().contiguous(), residual.float().contiguous()
    pf, cf = post.float().contiguous(), comb.float().contiguous()
    out = torch.empty(rf.shape, dtype=torch.float32, device=x.device)
    rows = xf.numel() // dim
    L.check(L.lib().dsv4_hc_post(L.ptr(xf), L.ptr(rf), L.ptr(pf), L.ptr(cf), L.ptr(out), rows, hc, dim,
                                 L.stream_of(x)))
    return out
