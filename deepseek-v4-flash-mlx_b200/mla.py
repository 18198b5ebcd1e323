"""MLA projections (reference: v4mlx/mla.py:16-56; 8-bit weights as oracle/v4_fast.py:31-34).

Weights are [out, in] and y = x @ W.T as in the reference. A weight is either a bf16 tensor or a
`QuantWeight` (int8 values with one bf16 scale per row and 64-wide group of inputs: symmetric
8-bit g64, the block format of the full-block decode config). All products run in libdsv4.so.
"""
import ctypes
from dataclasses import dataclass

import torch

from . import _lib as L

N_HEADS, HEAD_DIM, ROPE_HD = 64, 512, 64
N_GROUPS, O_LORA = 8, 1024


@dataclass
class QuantWeight:
    q: torch.Tensor       # int8 [out, in]
    scale: torch.Tensor   # bf16 [out, in // 64]

    @property
    def shape(self):
        return self.q.shape

    def dequantize(self):
        s = self.scale.float().repeat_interleave(64, dim=-1)
        return self.q.float() * s


def quantize_int8_g64(w):
    """Symmetric 8-bit quantisation with one bf16 scale per (row, 64 inputs)."""
    out_f, in_f = w.shape
    g = w.float().reshape(out_f, in_f // 64, 64)
    scale = (g.abs().amax(-1) / 127.0).clamp(min=1e-12).to(torch.bfloat16)
    q = torch.clamp(torch.round(g / scale.float()[..., None]), -127, 127).to(torch.int8)
    return QuantWeight(q.reshape(out_f, in_f).contiguous(), scale.contiguous())


def _as_bf16(x):
    if x.dtype == torch.bfloat16:
        return x.contiguous()
    x = x.contiguous()
    y = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    L.check(L.lib().dsv4_cast(L.ptr(x), L.dtype_code(x), L.ptr(y), L.BF16, x.numel(), L.stream_of(x)))
    return y


@torch.library.custom_op("dsv4::linear", mutates_args=(), device_types="cuda")
def _linear_op(x: torch.Tensor, w: torch.Tensor, w_scale: torch.Tensor | None, groups: int,
               out_dtype: torch.dtype) -> torch.Tensor:
    xb = _as_bf16(x)
    n_total, k = w.shape
    n = n_total // groups
    lead = x.shape[:-1]
    m = xb.numel() // (groups * k)
    y = torch.empty((*lead, groups * n), dtype=out_dtype, device=x.device)
    p = L.LinearParams()
    p.x, p.w, p.y = L.ptr(xb), L.ptr(w), L.ptr(y)
    p.w_scale = L.ptr(w_scale) if w_scale is not None else None
    p.m, p.n, p.k, p.groups, p.group = m, n, k, groups, 64
    p.x_dtype, p.w_dtype, p.y_dtype = L.BF16, L.dtype_code(w), L.dtype_code(y)
    nbytes = L.lib().dsv4_linear_workspace_size(ctypes.byref(p))
    ws = L.workspace(nbytes, x.device)
    p.workspace, p.workspace_bytes = L.ptr(ws), nbytes
    L.check(L.lib().dsv4_linear(ctypes.byref(p), L.stream_of(x)))
    return y


@_linear_op.register_fake
def _(x, w, w_scale, groups, out_dtype):
    n = w.shape[0] // groups
    return torch.empty((*x.shape[:-1], groups * n), dtype=out_dtype, device=x.device)


def linear(x, W, out_dtype=torch.float32, groups=1):
    """y = x @ W.T with W [out, in] (bf16, fp32 rounded to bf16 once, or QuantWeight).
    With groups > 1, x [..., groups*in] and W [groups*out, in]: y[..., g*out:(g+1)*out] = x_g W_g^T."""
    if isinstance(W, QuantWeight):
        L.require_cuda(x, W.q, W.scale)
        return _linear_op(x, W.q, W.scale, int(groups), out_dtype)
    L.require_cuda(x, W)
    if W.dtype != torch.bfloat16:
        W = _as_bf16(W)
    return _linear_op(x, W.contiguous(), None, int(groups), out_dtype)


@torch.library.custom_op("dsv4::linear_multi", mutates_args=(), device_types="cuda")
def _linear_multi_op(x: torch.Tensor, ws: list[torch.Tensor], scales: list[torch.Tensor],
                     out_dtype: torch.dtype) -> list[torch.Tensor]:
    xb = _as_bf16(x)
    k = ws[0].shape[1]
    lead = x.shape[:-1]
    m = xb.numel() // k
    ys = [torch.empty((*lead, w.shape[0]), dtype=out_dtype, device=x.device) for w in ws]
    p = L.LinearMultiParams()
    p.x, p.m, p.k, p.group, p.count = L.ptr(xb), m, k, 64, len(ws)
    p.x_dtype, p.w_dtype = L.BF16, L.dtype_code(ws[0])
    for i, (w, y) in enumerate(zip(ws, ys)):
        o = p.outs[i]
        o.w, o.y, o.n, o.y_dtype = L.ptr(w), L.ptr(y), w.shape[0], L.dtype_code(y)
        o.w_scale = L.ptr(scales[i]) if scales else None
    L.check(L.lib().dsv4_linear_multi(ctypes.byref(p), L.stream_of(x)))
    return ys


@_linear_multi_op.register_fake
def _(x, ws, scales, out_dtype):
    return [x.new_empty((*x.shape[:-1], w.shape[0]), dtype=out_dtype) for w in ws]


def linear_multi(x, Ws, out_dtype=torch.float32):
    """[x @ W.T for W in Ws] in one launch (up to 8 projections of the same x, all bf16 or all
    QuantWeight, same input width): the decode block's projections that read the same activations."""
    if not 1 <= len(Ws) <= L.LINEAR_MULTI_MAX:
        raise ValueError(f"linear_multi takes 1..{L.LINEAR_MULTI_MAX} weights")
    quant = isinstance(Ws[0], QuantWeight)
    if any(isinstance(W, QuantWeight) != quant for W in Ws):
        raise ValueError("linear_multi: mixed weight kinds")
    if quant:
        L.require_cuda(x, *[W.q for W in Ws])
        return _linear_multi_op(x, [W.q for W in Ws], [W.scale for W in Ws], out_dtype)
    L.require_cuda(x, *Ws)
    return _linear_multi_op(x, [(W if W.dtype == torch.bfloat16 else _as_bf16(W)).contiguous() for W in Ws], [],
                            out_dtype)


def q_down(x, wq_a, out_dtype=torch.float32):
    """x [..., dim] -> q_lora [..., q_lora_rank] (v4mlx/mla.py:21)."""
    return linear(x, wq_a, out_dtype)


def q_up(qln, wq_b, out_dtype=torch.float32):
    """q_lora_norm [..., q_lora_rank] -> [..., N_HEADS, HEAD_DIM] (v4mlx/mla.py:31-34)."""
    q = linear(qln, wq_b, out_dtype)
    return q.reshape(*q.shape[:-1], N_HEADS, HEAD_DIM)


def kv_proj(x, wkv, out_dtype=torch.float32):
    """x [..., dim] -> single MLA latent [..., HEAD_DIM] (v4mlx/mla.py:37-39)."""
    return linear(x, wkv, out_dtype)


def perhead_norm(q, eps=1e-6):
    from .norm_rope import perhead_norm as _phn
    return _phn(q, eps)


def o_grouped(o, wo_a, wo_b, out_dtype=torch.float32):
    """Grouped low-rank output projection (v4mlx/mla.py:42-56).
    o [..., N_HEADS*HEAD_DIM] -> [..., 8, 4096] . wo_a[g] [1024, 4096]^T -> [..., 8192] . wo_b^T."""
    mid = linear(o, wo_a, torch.bfloat16, groups=N_GROUPS)
    return linear(mid, wo_b, out_dtype)
