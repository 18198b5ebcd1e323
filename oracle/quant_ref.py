"""Oracle (test infrastructure only): the act-quant simulation of cached rows.

Restates the blockwise fp8-e4m3 round trip of the reference (`aq` in oracle/decode_engine.py:52-54,
`act_quant_sim` in v4mlx/compressor.py:11-20): per block of 64 values, amax = max(|x|, 1e-4),
s = 2^ceil(log2(amax / 448)), and each value becomes e4m3(clip(x / s, -448, 448)) * s, where e4m3
rounds to the nearest value of the format (ties to even): 4 exponent bits (bias 7), 3 mantissa bits,
largest finite 448, subnormal spacing 2^-9. The reference applies it to the nope dims (all but the
last 64 rope dims) of the current token's kv row (decode_engine.py:82) and of every emitted
compressed row (decode_engine.py:105; the prefill compressor, v4mlx/compressor.py:60-62).

The indexer compressor's variant (`compressor_prefill(..., rotate=True)`, v4mlx/compressor.py:57-59,
with v4mlx/qat.py:8-31) instead rotates every dim of the row with the normalised Walsh-Hadamard
transform (Sylvester order, butterflies of width 1, 2, 4, ... in float32, then a multiply by
float32(n^-0.5)) and takes a blockwise fp4-e2m1 round trip: per block of 32, amax = max(|x|,
6 * 2^-126), s = 2^ceil(log2(amax / 6)), each value e2m1(clip(x / s, -6, 6)) * s, where e2m1 holds
0, 0.5, 1, 1.5, 2, 3, 4, 6 (ties to the even mantissa).

The exponent ceil(log2(q)) is taken exactly from the bits of the fp32 quotient q = amax / 448 (the
reference evaluates np.log2 in float32, which can round to an integer for quotients within a few
ulps above a power of two; on seeded normal data no block comes that close, and the fixture test
pins the two against each other).
"""
import numpy as np
import torch

FP8_MAX = 448.0


def _e4m3_round(y):
    """Nearest e4m3 value (ties to even) of float32 y, |y| <= 448."""
    y = np.asarray(y, dtype=np.float32)
    a = np.abs(y).astype(np.float64)
    # the spacing of the format at |y|: 2^(floor(log2|y|) - 3) for normals, 2^-9 below 2^-6
    e = np.floor(np.log2(np.where(a > 0, a, 1.0)))
    e = np.maximum(e, -6.0)
    step = np.exp2(e - 3.0)
    r = np.rint(a / step) * step  # rint: half to even; a / step is exact (power of two)
    return (np.sign(y) * np.minimum(r, FP8_MAX)).astype(np.float32)


def block_exp(amax):
    """ceil(log2(max(amax, 1e-4) / 448)) from the float32 quotient's bits."""
    q = (np.maximum(np.asarray(amax, dtype=np.float32), np.float32(1e-4)) / np.float32(FP8_MAX)).astype(np.float32)
    bits = q.view(np.uint32).astype(np.int64)
    return ((bits >> 23) & 0xFF) - 127 + ((bits & 0x7FFFFF) != 0)


def act_quant_sim(x, block=64):
    """Blockwise fp8-e4m3 round trip along the last dim (a multiple of `block`); returns float32."""
    a = np.asarray(x, dtype=np.float32)
    sh = a.shape
    ab = a.reshape(*sh[:-1], sh[-1] // block, block)
    e = block_exp(np.abs(ab).max(-1, keepdims=True))
    s = np.exp2(e.astype(np.float64)).astype(np.float32)
    q = _e4m3_round(np.clip(ab / s, -FP8_MAX, FP8_MAX))
    return (q * s).reshape(sh).astype(np.float32)


def act_quant_rows(t, rope_dim=64, block=64):
    """The cached-row form: act_quant_sim on every dim but the last rope_dim (torch in, torch out)."""
    a = t.detach().float().cpu().numpy()
    out = a.copy()
    out[..., :-rope_dim] = act_quant_sim(a[..., :-rope_dim], block)
    return torch.from_numpy(out).to(t.device)


FP4_MAX = 6.0


def hadamard_rotate(x):
    """Normalised Walsh-Hadamard transform along the last dim (a power of two), float32 throughout:
    at width h the pair (i, i + h) of each 2h-block becomes (x_i + x_{i+h}, x_i - x_{i+h})."""
    a = np.array(x, dtype=np.float32, copy=True)
    n = a.shape[-1]
    assert n & (n - 1) == 0
    h = 1
    while h < n:
        v = a.reshape(*a.shape[:-1], n // (2 * h), 2, h)
        lo, hi = v[..., 0, :].copy(), v[..., 1, :].copy()
        v[..., 0, :] = lo + hi
        v[..., 1, :] = lo - hi
        a = v.reshape(*a.shape[:-1], n)
        h *= 2
    return (a * np.float32(n ** -0.5)).astype(np.float32)


def _e2m1_round(y):
    """Nearest e2m1 value (ties to the even mantissa) of float32 y, |y| <= 6: spacing 0.5 below 2,
    1 in [2, 4), 2 in [4, 6]."""
    y = np.asarray(y, dtype=np.float32)
    a = np.abs(y)
    q = np.where(a < 2, np.rint(a * 2) / 2, np.where(a < 4, np.rint(a), np.rint(a / 2) * 2)).astype(np.float32)
    return np.copysign(q, y).astype(np.float32)


def fp4_exp(amax):
    """ceil(log2(max(amax, 6 * 2^-126) / 6)) from the float32 quotient's bits."""
    q = (np.maximum(np.asarray(amax, dtype=np.float32), np.float32(6 * 2.0 ** -126)) / np.float32(FP4_MAX))
    bits = q.astype(np.float32).view(np.uint32).astype(np.int64)
    return ((bits >> 23) & 0xFF) - 127 + ((bits & 0x7FFFFF) != 0)


def fp4_act_quant(x, block=32):
    """Blockwise fp4-e2m1 round trip with power-of-two scales along the last dim; float32."""
    a = np.asarray(x, dtype=np.float32)
    sh = a.shape
    ab = a.reshape(*sh[:-1], sh[-1] // block, block)
    e = fp4_exp(np.abs(ab).max(-1, keepdims=True))
    s = np.exp2(e.astype(np.float64)).astype(np.float32)
    q = _e2m1_round(np.clip(ab / s, -FP4_MAX, FP4_MAX))
    return (q * s).reshape(sh).astype(np.float32)


def rotate_quant_rows(t):
    """The indexer compressor's key form: fp4_act_quant(hadamard_rotate(row)) (torch in, torch out)."""
    a = t.detach().float().cpu().numpy()
    return torch.from_numpy(fp4_act_quant(hadamard_rotate(a))).to(t.device)
