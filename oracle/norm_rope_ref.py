"""Oracle: RMSNorm / YaRN / RoPE (restating ref_torch/norm_rope.py and v4mlx/mla.py:26). Test-only."""
import math

import torch


def rmsnorm(x, weight, eps=1e-6):
    """ref_torch/norm_rope.py:10-16: fp32 mean of squares, rsqrt, weight multiply, cast back."""
    dt = x.dtype
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    if weight is not None:
        y = weight.float() * y
    return y.to(dt)


def perhead_norm(q, eps=1e-6):
    """v4mlx/mla.py:26-28 (no weight)."""
    return rmsnorm(q, None, eps)


def precompute_freqs(dim, seqlen, original_seq_len, base, factor, beta_fast, beta_slow):
    """ref_torch/norm_rope.py:19-43: base frequencies in fp32, YaRN ramp between the correction
    dims of beta_fast and beta_slow."""
    f = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
    if original_seq_len > 0:
        cd = lambda r: dim * math.log(original_seq_len / (r * 2 * math.pi)) / (2 * math.log(base))
        lo = max(math.floor(cd(beta_fast)), 0)
        hi = min(math.ceil(cd(beta_slow)), dim - 1)
        if lo == hi:
            hi += 0.001
        ramp = ((torch.arange(dim // 2, dtype=torch.float32) - lo) / (hi - lo)).clamp(0, 1)
        keep = 1 - ramp
        f = f / factor * (1 - keep) + f * keep
    return f


def precompute_freqs_cis(dim, seqlen, original_seq_len, base, factor, beta_fast, beta_slow):
    """ref_torch/norm_rope.py:46-50."""
    f = precompute_freqs(dim, seqlen, original_seq_len, base, factor, beta_fast, beta_slow)
    ang = torch.outer(torch.arange(seqlen), f)
    return torch.polar(torch.ones_like(ang), ang)


def apply_rotary_emb(x, freqs_cis, inverse=False):
    """ref_torch/norm_rope.py:53-62: interleaved pairs as complex numbers times e^{+-i theta}."""
    z = torch.view_as_complex(x.float().reshape(*x.shape[:-1], -1, 2).contiguous())
    f = freqs_cis.conj() if inverse else freqs_cis
    f = f.reshape(1, z.shape[1], z.shape[-1]) if z.dim() == 3 else f.reshape(1, z.shape[1], 1, z.shape[-1])
    return torch.view_as_real(z * f).flatten(-2).to(x.dtype)


def rope_at(x, positions, freqs, rope_dim=64, inverse=False):
    """RoPE of the last rope_dim dims of x[..., row, (h,), d] with one position per row (the cos/sin
    rows the reference gathers at cos[cpos], oracle/decode_engine.py:79)."""
    pos = positions.long().reshape(-1)
    ang = pos.float()[:, None] * freqs[None, :]                          # [rows, rope/2]
    cis = torch.polar(torch.ones_like(ang), ang)
    if inverse:
        cis = cis.conj()
    lead = x.shape[:-1]
    rows = pos.numel()
    xr = x.float().reshape(rows, -1, x.shape[-1])
    z = torch.view_as_complex(xr[..., -rope_dim:].reshape(rows, xr.shape[1], -1, 2).contiguous())
    zr = torch.view_as_real(z * cis[:, None, :]).flatten(-2)
    out = torch.cat([xr[..., :-rope_dim], zr], -1)
    return out.reshape(*lead, x.shape[-1])
