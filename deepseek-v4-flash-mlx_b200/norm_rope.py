"""RMSNorm + RoPE/YaRN ops (reference: ref_torch/norm_rope.py, v4mlx/norm_rope.py, v4mlx/mla.py:26).

Public functions keep the reference call signatures. `precompute_freqs` / `precompute_freqs_cis`
are host-side table builders (a 32-entry fp32 table); every per-element op runs in libdsv4.so.
"""
import ctypes
import math

import torch

from . import _lib as L


# ---- host-side YaRN frequency table -----------------------------------------------------------

def precompute_freqs(dim, seqlen, original_seq_len, base, factor, beta_fast, beta_slow):
    """YaRN angular frequencies [dim/2] in fp32 (ref_torch/norm_rope.py:19-43).

    The base table is computed on a float32 tensor exactly as the reference forms it, so the
    device kernels see bit-identical frequencies. `seqlen` is unused (kept for the signature)."""
    freqs = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
    if original_seq_len > 0:
        def corr(rot):
            return dim * math.log(original_seq_len / (rot * 2 * math.pi)) / (2 * math.log(base))
        low = max(math.floor(corr(beta_fast)), 0)
        high = min(math.ceil(corr(beta_slow)), dim - 1)
        if low == high:
            high += 0.001
        ramp = torch.clamp((torch.arange(dim // 2, dtype=torch.float32) - low) / (high - low), 0, 1)
        smooth = 1 - ramp
        freqs = freqs / factor * (1 - smooth) + freqs * smooth
    return freqs


def precompute_freqs_cis(dim, seqlen, original_seq_len, base, factor, beta_fast, beta_slow):
    """complex64 [seqlen, dim/2] table e^{i t f} (ref_torch/norm_rope.py:46-50)."""
    f = precompute_freqs(dim, seqlen, original_seq_len, base, factor, beta_fast, beta_slow)
    ang = torch.outer(torch.arange(seqlen), f)
    return torch.polar(torch.ones_like(ang), ang)


# YaRN settings of the compressed-attention layers and of the ratio-0 layers
# (oracle/decode_engine.py:47; ref_torch/compressor.py:21 defaults)
YARN_COMPRESSED = dict(original_seq_len=65536, base=160000.0, factor=16, beta_fast=32, beta_slow=1)
ROPE_PLAIN = dict(original_seq_len=0, base=10000.0, factor=40, beta_fast=32, beta_slow=1)

_freq_cache = {}


def rope_freqs(rope_dim=64, device="cuda", **yarn):
    """Device copy of the YaRN frequency table (cached per device and settings)."""
    cfg = dict(YARN_COMPRESSED)
    cfg.update(yarn)
    key = (rope_dim, str(torch.device(device)), tuple(sorted(cfg.items())))
    t = _freq_cache.get(key)
    if t is None:
        t = precompute_freqs(rope_dim, 0, cfg["original_seq_len"], cfg["base"], cfg["factor"],
                             cfg["beta_fast"], cfg["beta_slow"]).to(device)
        _freq_cache[key] = t
    return t


# ---- custom ops ---------------------------------------------------------------------------------

@torch.library.custom_op("dsv4::rmsnorm", mutates_args=(), device_types="cuda")
def _rmsnorm_op(x: torch.Tensor, weight: torch.Tensor | None, eps: float,
                out_dtype: torch.dtype | None = None) -> torch.Tensor:
    x = x.contiguous()
    out = torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
    p = L.RmsNormParams()
    p.x, p.out = L.ptr(x), L.ptr(out)
    p.weight = L.ptr(weight.contiguous()) if weight is not None else None
    p.rows = x.numel() // x.shape[-1] if x.numel() else 0
    p.dim = x.shape[-1]
    p.x_dtype, p.out_dtype = L.dtype_code(x), L.dtype_code(out)
    p.w_dtype = L.dtype_code(weight) if weight is not None else L.F32
    p.eps = eps
    L.check(L.lib().dsv4_rmsnorm(ctypes.byref(p), L.stream_of(x)))
    return out


@_rmsnorm_op.register_fake
def _(x, weight, eps, out_dtype=None):
    return torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)


def rmsnorm(x, weight, eps=1e-6, out_dtype=None):
    """RMSNorm.forward (ref_torch/norm_rope.py:10-16): fp32 math, result in x.dtype (or out_dtype:
    one rounding of the fp32 result, the operand a bf16 projection consumes)."""
    L.require_cuda(x, weight)
    if weight is not None and weight.dtype not in (torch.float32, torch.bfloat16):
        weight = weight.float()
    return _rmsnorm_op(x, weight, float(eps), out_dtype)


def perhead_norm(q, eps=1e-6):
    """Weightless per-head RMS (v4mlx/mla.py:26-28): q * rsqrt(mean(q^2, -1) + eps)."""
    L.require_cuda(q)
    return _rmsnorm_op(q, None, float(eps))


@torch.library.custom_op("dsv4::apply_rotary_emb", mutates_args=(), device_types="cuda")
def _rope_cis_op(x: torch.Tensor, cis: torch.Tensor, inverse: bool) -> torch.Tensor:
    x = x.contiguous()
    out = torch.empty_like(x)
    heads = x.shape[2] if x.dim() == 4 else 1
    rows = x.numel() // (x.shape[-1] * heads)
    table = torch.view_as_real(cis.to(x.device)).float().contiguous() if cis.is_complex() else cis.float().contiguous()
    p = L.RopeParams()
    p.x, p.out = L.ptr(x), L.ptr(out)
    p.s, p.heads, p.dim, p.rope_dim = rows, heads, x.shape[-1], x.shape[-1]
    p.x_dtype, p.out_dtype = L.dtype_code(x), L.dtype_code(out)
    p.cis, p.cis_rows = L.ptr(table), table.shape[0]
    p.freqs, p.positions, p.pos_offset, p.inverse = None, None, 0, int(inverse)
    L.check(L.lib().dsv4_rope(ctypes.byref(p), L.stream_of(x)))
    return out


@_rope_cis_op.register_fake
def _(x, cis, inverse):
    return torch.empty_like(x)


def apply_rotary_emb(x, freqs_cis, inverse=False):
    """apply_rotary_emb (ref_torch/norm_rope.py:53-62): x [b, s, d] or [b, s, h, d]; the last dim is
    the rope sub-vector, interleaved (real, imag) pairs; freqs_cis complex [s, d/2]."""
    L.require_cuda(x)
    if x.dim() not in (3, 4):
        raise ValueError("apply_rotary_emb: x must be [b, s, d] or [b, s, h, d]")
    if freqs_cis.shape[0] != x.shape[1]:
        raise ValueError("apply_rotary_emb: freqs_cis rows must equal seqlen")
    return _rope_cis_op(x, freqs_cis, bool(inverse))


@torch.library.custom_op("dsv4::rope_positions", mutates_args=(), device_types="cuda")
def _rope_pos_op(x: torch.Tensor, freqs: torch.Tensor, positions: torch.Tensor, rope_dim: int,
                 inverse: bool) -> torch.Tensor:
    x = x.contiguous()
    out = torch.empty_like(x)
    rows = positions.numel()
    heads = x.numel() // (rows * x.shape[-1])
    p = L.RopeParams()
    p.x, p.out = L.ptr(x), L.ptr(out)
    p.s, p.heads, p.dim, p.rope_dim = rows, heads, x.shape[-1], rope_dim
    p.x_dtype, p.out_dtype = L.dtype_code(x), L.dtype_code(out)
    p.cis, p.cis_rows = None, 0
    p.freqs, p.positions = L.ptr(freqs), L.ptr(positions)
    p.pos_offset, p.inverse = 0, int(inverse)
    L.check(L.lib().dsv4_rope(ctypes.byref(p), L.stream_of(x)))
    return out


@_rope_pos_op.register_fake
def _(x, freqs, positions, rope_dim, inverse):
    return torch.empty_like(x)


def rope(x, positions, freqs, rope_dim=64, inverse=False):
    """RoPE of the last rope_dim dims of rows x[..., pos_row, (heads,), dim] at int32 positions."""
    L.require_cuda(x, positions, freqs)
    return _rope_pos_op(x, freqs.float().contiguous(), positions.to(torch.int32).contiguous(),
                        int(rope_dim), bool(inverse))


@torch.library.custom_op("dsv4::norm_rope", mutates_args=(), device_types="cuda")
def _norm_rope_op(x: torch.Tensor, weight: torch.Tensor | None, freqs: torch.Tensor,
                  positions: torch.Tensor, rope_dim: int, eps: float, out_dtype: torch.dtype,
                  act_quant: bool = False) -> torch.Tensor:
    x = x.contiguous()
    out = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    rows = positions.numel()
    heads = x.numel() // (rows * x.shape[-1])
    p = L.NormRopeParams()
    p.x, p.out, p.out_rows = L.ptr(x), L.ptr(out), None
    p.weight = L.ptr(weight) if weight is not None else None
    p.rows, p.heads, p.dim, p.rope_dim = rows, heads, x.shape[-1], rope_dim
    p.x_dtype, p.out_dtype = L.dtype_code(x), L.dtype_code(out)
    p.w_dtype = L.dtype_code(weight) if weight is not None else L.F32
    p.eps = eps
    p.freqs, p.positions = L.ptr(freqs), L.ptr(positions)
    p.act_quant = int(act_quant)
    L.check(L.lib().dsv4_norm_rope(ctypes.byref(p), L.stream_of(x)))
    return out


@_norm_rope_op.register_fake
def _(x, weight, freqs, positions, rope_dim, eps, out_dtype, act_quant=False):
    return torch.empty(x.shape, dtype=out_dtype, device=x.device)


def norm_rope(x, positions, freqs, weight=None, rope_dim=64, eps=1e-6, out_dtype=torch.bfloat16, act_quant=False):
    """Fused RMSNorm (weight given) or weightless per-head norm (weight None) over the last dim,
    then RoPE of its last rope_dim dims at `positions` (one per leading row), then a cast.
    This is the q / kv chain of oracle/decode_engine.py:77-81 and oracle/v4_fast.py:87-91.
    `act_quant`: the fp8-e4m3 act-quant simulation of the kv row's nope dims (blocks of 64,
    power-of-two scales) that the reference applies before caching (oracle/decode_engine.py:82)."""
    L.require_cuda(x, positions, freqs, weight)
    return _norm_rope_op(x, weight, freqs.float().contiguous(), positions.to(torch.int32).contiguous(),
                         int(rope_dim), float(eps), out_dtype, bool(act_quant))
