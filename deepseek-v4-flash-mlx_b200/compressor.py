"""KV block compressor (reference: ref_torch/compressor.py:21-50; decode ring
oracle/decode_engine.py:85-105, oracle/v4_fast.py:97-106).

`compressor_prefill` keeps the reference signature and returns (kv_compressed, state): the two
projections run on the projection GEMM (bf16 operands, fp32 accumulate), then one kernel pools each
4-token block with the 8-slot softmax gate, applies RMSNorm and RoPE and stores the row. `state`
holds the reference's hand-off tensors plus the device ring used by `compressor_decode_step`.
"""
import ctypes

import torch

from . import _lib as L
from .mla import linear
from .norm_rope import rope_freqs


def _pool(kv, score, ape, norm_w, out, head_dim, ratio, rope_dim, freqs, ring_kv=None, ring_score=None,
          out_rows=None, pos0=0, eps=1e-6, act_quant=False):
    b, s = kv.shape[0], kv.shape[1]
    p = L.CompressorParams()
    p.kv, p.score, p.ape = L.ptr(kv), L.ptr(score), L.ptr(ape)
    p.norm_w = L.ptr(norm_w) if norm_w is not None else None
    p.out = L.ptr(out)
    p.out_rows = L.ptr(out_rows) if out_rows is not None else None
    p.b, p.s, p.head_dim, p.ratio, p.rope_dim = b, s, head_dim, ratio, rope_dim
    p.norm_dtype = L.dtype_code(norm_w) if norm_w is not None else L.F32
    p.out_dtype = L.dtype_code(out)
    p.eps = eps
    p.freqs, p.pos0 = L.ptr(freqs), pos0
    p.ring_kv = L.ptr(ring_kv) if ring_kv is not None else None
    p.ring_score = L.ptr(ring_score) if ring_score is not None else None
    p.act_quant = int(act_quant)
    L.check(L.lib().dsv4_compressor_pool(ctypes.byref(p), L.stream_of(kv)))


def compressor_prefill(x, wkv, wgate, ape, norm_w, head_dim=512, ratio=4, rope_head_dim=64,
                       base=160000.0, original_seq_len=65536, factor=16, beta_fast=32, beta_slow=1,
                       out_dtype=torch.float32, pos0=0, act_quant=False, rotate=False):
    """x [b, s, dim] -> (kv [b, s//ratio, head_dim] post-rope, state).

    state: "kv" / "score" = the last full block's kv and score+ape [b, ratio, 2*head_dim] (when
    s >= ratio), "kv_rem" = the remainder rows, and "ring_kv" / "ring_score" [b, 2*ratio, 2*head_dim]
    the device ring that `compressor_decode_step` continues from (ref_torch/compressor.py:67-74).
    `pos0` is the position of x's first token (a slice of a longer sequence): row g is roped at
    pos0 + ratio*g. `act_quant`: the fp8-e4m3 act-quant simulation of each row's nope dims (the
    reference's default for the main compressor, v4mlx/compressor.py:60-62). `rotate` (head_dim
    128, the indexer compressor; v4mlx/compressor.py:57-59): instead, every dim of each row is
    rotated by the normalised Walsh-Hadamard transform and rounded to fp4-e2m1 in blocks of 32."""
    L.require_cuda(x, wkv, wgate, ape, norm_w)
    b, s, _ = x.shape
    d2 = 2 * head_dim
    kv = linear(x, wkv, torch.float32)
    score = linear(x, wgate, torch.float32)
    freqs = rope_freqs(rope_head_dim, x.device, original_seq_len=original_seq_len, base=base, factor=factor,
                       beta_fast=beta_fast, beta_slow=beta_slow)
    groups = s // ratio
    out = torch.empty((b, groups, head_dim), dtype=out_dtype, device=x.device)
    ring_kv = torch.empty((b, 2 * ratio, d2), dtype=torch.float32, device=x.device)
    ring_score = torch.empty_like(ring_kv)
    nw = norm_w if norm_w.dtype in (torch.float32, torch.bfloat16) else norm_w.float()
    _pool(kv, score, ape.float().contiguous(), nw.contiguous(), out, head_dim, ratio, rope_head_dim, freqs,
          ring_kv, ring_score, pos0=pos0, act_quant=2 if rotate else act_quant)
    cutoff = s - s % ratio
    state = {"ring_kv": ring_kv, "ring_score": ring_score}
    if cutoff >= ratio:
        state["kv"] = ring_kv[:, :ratio]
        state["score"] = ring_score[:, :ratio]
    if s % ratio:
        state["kv_rem"] = kv[:, cutoff:]
    return out, state


def compressor_decode_step(x, wkv, wgate, ape, norm_w, ring_kv, ring_score, positions, out, out_rows,
                           head_dim=512, ratio=4, rope_head_dim=64, freqs=None, eps=1e-6,
                           proj=None, key_image=None, act_quant=False, rotate=False):
    """One decode token per sequence (oracle/decode_engine.py:96-105): write this token's kv / score
    into the device ring; sequences whose position p has (p+1) % ratio == 0 emit a pooled, normed,
    roped row into out[out_rows[b]] and shift the ring. x [b, dim]; positions int32 [b].
    `proj` may pass precomputed projections (kv, score) [b, 2*head_dim] fp32. `key_image`
    (image, inv, norm_max, keys_per_entry) also adds each emitted indexer key (out viewed as
    [entries * keys_per_entry, 128] fp32) to a decode cache's key image. `act_quant`: the fp8-e4m3
    act-quant simulation of the emitted row's nope dims (oracle/decode_engine.py:105). `rotate`
    (head_dim 128): the Hadamard + fp4-e2m1 key simulation of `compressor_prefill(rotate=True)`."""
    L.require_cuda(x, ring_kv, ring_score, positions, out, out_rows)
    if proj is None:
        kvp = linear(x, wkv, torch.float32)
        scp = linear(x, wgate, torch.float32)
    else:
        kvp, scp = proj
    if freqs is None:
        freqs = rope_freqs(rope_head_dim, x.device)
    p = L.CompressorDecodeParams()
    p.kv, p.score, p.ape = L.ptr(kvp.contiguous()), L.ptr(scp.contiguous()), L.ptr(ape)
    p.norm_w = L.ptr(norm_w) if norm_w is not None else None
    p.ring_kv, p.ring_score = L.ptr(ring_kv), L.ptr(ring_score)
    p.positions = L.ptr(positions)
    p.out, p.out_rows = L.ptr(out), L.ptr(out_rows)
    p.b, p.head_dim, p.ratio, p.rope_dim = kvp.shape[0], head_dim, ratio, rope_head_dim
    p.norm_dtype = L.dtype_code(norm_w) if norm_w is not None else L.F32
    p.out_dtype = L.dtype_code(out)
    p.eps = eps
    p.freqs = L.ptr(freqs)
    p.act_quant = 2 if rotate else int(act_quant)
    if key_image is not None:
        img, inv, nmax, stride = key_image
        p.key_image, p.key_inv, p.key_norm_max, p.image_stride = L.ptr(img), L.ptr(inv), L.ptr(nmax), int(stride)
    L.check(L.lib().dsv4_compressor_decode(ctypes.byref(p), L.stream_of(x)))
