"""Oracle (test infrastructure only): the act-quant simulation of cached rows.

Restates the blockwise fp8-e4m3 round trip of the reference (`aq` in oracle/decode_engine.py:52-54,
`act_quant_sim` in v4mlx/compressor.py:11-20): per block of 64 values, amax = max(|x|, 1e-4),
s = 2^ceil(log2(amax / 448)), and each value becomes e4m3(clip(x / s, -448, 448)) * s, where e4m3
rounds to the nearest value of the format (ties to even): 4 exponent bits (bias 7), 3 mantissa bits,
largest finite 448, subnormal spacing 2^-9. The reference applies it to the nope dims (all but the
last 64 rope dims) of the current token's kv row (decode_engine.py:82) and of every emitted
compressed row (decode_engine.py:105; the prefill compressor, v4mlx/compressor.py:60-62).

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
