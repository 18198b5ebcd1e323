"""KV block compressor (reference: ref_torch/compressor.py:21-50; decode ring
oracle/decode_engine.py:85-105, oracle/v4_fast.py:97-106).

`compressor_prefill` keeps the reference signature and returns (kv_compressed, state): the two
projections run on the projection GEMM (bf16 operands, fp32 accumulate), then one kernel pools each
4-token block with the 8-slot softmax gate, applies RMSNorm and RoPE and stores the row. `state`
holds the reference's hand-off tensors plus the device ring used by `compressor_decode_step`.
"""
import ctypes
from typing import NamedTuple

import torch

from . import _lib as L
from .mla import QuantWeight, linear, linear_multi
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


def _w_parts(W):
    """(tensor, scale or None) of a weight: bf16 / fp32 tensor, or QuantWeight's int8 values + scales."""
    if isinstance(W, QuantWeight):
        return W.q, W.scale
    return W, None


def _w_join(w, scale):
    return QuantWeight(w, scale) if scale is not None else w


@torch.library.custom_op("dsv4::compressor_prefill", mutates_args=(), device_types="cuda")
def _compressor_prefill_op(x: torch.Tensor, wkv: torch.Tensor, wkv_scale: torch.Tensor | None, wgate: torch.Tensor,
                           wgate_scale: torch.Tensor | None, ape: torch.Tensor, norm_w: torch.Tensor, head_dim: int,
                           ratio: int, rope_head_dim: int, base: float, original_seq_len: int, factor: float,
                           beta_fast: float, beta_slow: float, out_dtype: torch.dtype, pos0: int,
                           act_quant: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    b, s, _ = x.shape
    d2 = 2 * head_dim
    if b * s > 64 and wkv_scale is None and wgate_scale is None:
        kv, score = linear_multi(x, [wkv, wgate], torch.float32)  # one tcgen05 launch, x read once
    else:
        kv = linear(x, _w_join(wkv, wkv_scale), torch.float32)
        score = linear(x, _w_join(wgate, wgate_scale), torch.float32)
    freqs = rope_freqs(rope_head_dim, x.device, original_seq_len=original_seq_len, base=base, factor=factor,
                       beta_fast=beta_fast, beta_slow=beta_slow)
    out = torch.empty((b, s // ratio, head_dim), dtype=out_dtype, device=x.device)
    ring_kv = torch.empty((b, 2 * ratio, d2), dtype=torch.float32, device=x.device)
    ring_score = torch.empty_like(ring_kv)
    nw = norm_w if norm_w.dtype in (torch.float32, torch.bfloat16) else norm_w.float()
    _pool(kv, score, ape.float().contiguous(), nw.contiguous(), out, head_dim, ratio, rope_head_dim, freqs,
          ring_kv, ring_score, pos0=pos0, act_quant=act_quant)
    cutoff = s - s % ratio
    return out, ring_kv, ring_score, kv[:, cutoff:].clone()


@_compressor_prefill_op.register_fake
def _(x, wkv, wkv_scale, wgate, wgate_scale, ape, norm_w, head_dim, ratio, rope_head_dim, base, original_seq_len,
      factor, beta_fast, beta_slow, out_dtype, pos0, act_quant):
    b, s, _ = x.shape
    ring = x.new_empty((b, 2 * ratio, 2 * head_dim), dtype=torch.float32)
    return (x.new_empty((b, s // ratio, head_dim), dtype=out_dtype), ring, torch.empty_like(ring),
            x.new_empty((b, s % ratio, 2 * head_dim), dtype=torch.float32))


def compressor_prefill(x, wkv, wgate, ape, norm_w, head_dim=512, ratio=4, rope_head_dim=64,
                       base=160000.0, original_seq_len=65536, factor=16, beta_fast=32, beta_slow=1,
                       out_dtype=torch.float32, pos0=0, act_quant=False, rotate=False):
    """x [b, s, dim] -> (kv [b, s//ratio, head_dim] post-rope, state).

    The reference signature (ref_torch/compressor.py:21) over the custom op `dsv4::compressor_prefill`
    (opaque to torch.compile / FakeTensor tracing; weights bf16, fp32, or QuantWeight).
    state: "kv" / "score" = the last full block's kv and score+ape [b, ratio, 2*head_dim] (when
    s >= ratio), "kv_rem" = the remainder rows, and "ring_kv" / "ring_score" [b, 2*ratio, 2*head_dim]
    the device ring that `compressor_decode_step` continues from (ref_torch/compressor.py:67-74).
    `pos0` is the position of x's first token (a slice of a longer sequence): row g is roped at
    pos0 + ratio*g. `act_quant`: the fp8-e4m3 act-quant simulation of each row's nope dims (the
    reference's default for the main compressor, v4mlx/compressor.py:60-62). `rotate` (head_dim
    128, the indexer compressor; v4mlx/compressor.py:57-59): instead, every dim of each row is
    rotated by the normalised Walsh-Hadamard transform and rounded to fp4-e2m1 in blocks of 32."""
    wkv_t, wkv_s = _w_parts(wkv)
    wg_t, wg_s = _w_parts(wgate)
    L.require_cuda(x, wkv_t, wg_t, ape, norm_w)
    s = x.shape[1]
    out, ring_kv, ring_score, rem = _compressor_prefill_op(
        x, wkv_t, wkv_s, wg_t, wg_s, ape, norm_w, int(head_dim), int(ratio), int(rope_head_dim), float(base),
        int(original_seq_len), float(factor), float(beta_fast), float(beta_slow), out_dtype, int(pos0),
        2 if rotate else int(act_quant))
    state = {"ring_kv": ring_kv, "ring_score": ring_score}
    if s - s % ratio >= ratio:
        state["kv"] = ring_kv[:, :ratio]
        state["score"] = ring_score[:, :ratio]
    if s % ratio:
        state["kv_rem"] = rem
    return out, state


@torch.library.custom_op("dsv4::compressor_decode_step",
                         mutates_args=("ring_kv", "ring_score", "out", "key_image", "key_inv", "key_norm_max"),
                         device_types="cuda")
def _compressor_decode_op(x: torch.Tensor, wkv: torch.Tensor, wkv_scale: torch.Tensor | None, wgate: torch.Tensor,
                          wgate_scale: torch.Tensor | None, ape: torch.Tensor, norm_w: torch.Tensor | None,
                          ring_kv: torch.Tensor, ring_score: torch.Tensor, positions: torch.Tensor,
                          out: torch.Tensor, out_rows: torch.Tensor, head_dim: int, ratio: int, rope_head_dim: int,
                          freqs: torch.Tensor, eps: float, proj_kv: torch.Tensor | None,
                          proj_score: torch.Tensor | None, key_image: torch.Tensor | None,
                          key_inv: torch.Tensor | None, key_norm_max: torch.Tensor | None, image_stride: int,
                          act_quant: int) -> None:
    if proj_kv is None:
        kvp = linear(x, _w_join(wkv, wkv_scale), torch.float32)
        scp = linear(x, _w_join(wgate, wgate_scale), torch.float32)
    else:
        kvp, scp = proj_kv, proj_score
    p = _decode_params(kvp, scp, ape, norm_w, ring_kv, ring_score, positions, out, out_rows, head_dim, ratio,
                       rope_head_dim, freqs, eps, key_image, key_inv, key_norm_max, image_stride, act_quant)
    L.check(L.lib().dsv4_compressor_decode(ctypes.byref(p), L.stream_of(x)))


def _decode_params(kvp, scp, ape, norm_w, ring_kv, ring_score, positions, out, out_rows, head_dim, ratio,
                   rope_head_dim, freqs, eps, key_image, key_inv, key_norm_max, image_stride, act_quant):
    """dsv4_compressor_decode_params of one compressor's decode step."""
    kvp, scp = kvp.contiguous(), scp.contiguous()
    p = L.CompressorDecodeParams()
    p.kv, p.score, p.ape = L.ptr(kvp), L.ptr(scp), L.ptr(ape)
    p.norm_w = L.ptr(norm_w) if norm_w is not None else None
    p.ring_kv, p.ring_score = L.ptr(ring_kv), L.ptr(ring_score)
    p.positions = L.ptr(positions)
    p.out, p.out_rows = L.ptr(out), L.ptr(out_rows)
    p.b, p.head_dim, p.ratio, p.rope_dim = kvp.shape[0], head_dim, ratio, rope_head_dim
    p.norm_dtype = L.dtype_code(norm_w) if norm_w is not None else L.F32
    p.out_dtype = L.dtype_code(out)
    p.eps = eps
    p.freqs = L.ptr(freqs)
    p.act_quant = act_quant
    if key_image is not None:
        p.key_image, p.key_inv, p.key_norm_max = L.ptr(key_image), L.ptr(key_inv), L.ptr(key_norm_max)
        p.image_stride = image_stride
    return p


@_compressor_decode_op.register_fake
def _(x, wkv, wkv_scale, wgate, wgate_scale, ape, norm_w, ring_kv, ring_score, positions, out, out_rows, head_dim,
      ratio, rope_head_dim, freqs, eps, proj_kv, proj_score, key_image, key_inv, key_norm_max, image_stride,
      act_quant):
    return None


def compressor_decode_step(x, wkv, wgate, ape, norm_w, ring_kv, ring_score, positions, out, out_rows,
                           head_dim=512, ratio=4, rope_head_dim=64, freqs=None, eps=1e-6,
                           proj=None, key_image=None, act_quant=False, rotate=False):
    """One decode token per sequence (oracle/decode_engine.py:96-105): write this token's kv / score
    into the device ring; sequences whose position p has (p+1) % ratio == 0 emit a pooled, normed,
    roped row into out[out_rows[b]] and shift the ring. x [b, dim]; positions int32 [b].
    The custom op `dsv4::compressor_decode_step` (it mutates the ring, `out` and the key image).
    `proj` may pass precomputed projections (kv, score) [b, 2*head_dim] fp32. `key_image`
    (image, inv, norm_max, keys_per_entry) also adds each emitted indexer key (out viewed as
    [entries * keys_per_entry, 128] fp32) to a decode cache's key image. `act_quant`: the fp8-e4m3
    act-quant simulation of the emitted row's nope dims (oracle/decode_engine.py:105). `rotate`
    (head_dim 128): the Hadamard + fp4-e2m1 key simulation of `compressor_prefill(rotate=True)`."""
    wkv_t, wkv_s = _w_parts(wkv)
    wg_t, wg_s = _w_parts(wgate)
    L.require_cuda(x, ring_kv, ring_score, positions, out, out_rows)
    if freqs is None:
        freqs = rope_freqs(rope_head_dim, x.device)
    pk, ps = proj if proj is not None else (None, None)
    img, inv, nmax, stride = key_image if key_image is not None else (None, None, None, 0)
    _compressor_decode_op(x, wkv_t, wkv_s, wg_t, wg_s, ape, norm_w, ring_kv, ring_score, positions, out, out_rows,
                          int(head_dim), int(ratio), int(rope_head_dim), freqs, float(eps), pk, ps, img, inv, nmax,
                          int(stride), 2 if rotate else int(act_quant))


class CompressorStep(NamedTuple):
    """One compressor's share of `compressor_decode_pair`: its projections of this token
    (kv, score) fp32 [b, 2*head_dim], its weights, ring and output rows, as `compressor_decode_step`
    takes them."""
    proj: tuple
    ape: torch.Tensor
    norm_w: torch.Tensor | None
    ring_kv: torch.Tensor
    ring_score: torch.Tensor
    out: torch.Tensor
    out_rows: torch.Tensor
    head_dim: int
    key_image: tuple | None = None
    act_quant: int = 0


@torch.library.custom_op("dsv4::compressor_decode_pair",
                         mutates_args=("a_ring_kv", "a_ring_score", "a_out", "b_ring_kv", "b_ring_score", "b_out",
                                       "b_key_image", "b_key_inv", "b_key_norm_max"),
                         device_types="cuda")
def _compressor_decode_pair_op(positions: torch.Tensor, ratio: int, rope_head_dim: int, freqs: torch.Tensor,
                               eps: float, a_kv: torch.Tensor, a_score: torch.Tensor, a_ape: torch.Tensor,
                               a_norm_w: torch.Tensor | None, a_ring_kv: torch.Tensor, a_ring_score: torch.Tensor,
                               a_out: torch.Tensor, a_out_rows: torch.Tensor, a_head_dim: int, a_act_quant: int,
                               b_kv: torch.Tensor, b_score: torch.Tensor, b_ape: torch.Tensor,
                               b_norm_w: torch.Tensor | None, b_ring_kv: torch.Tensor, b_ring_score: torch.Tensor,
                               b_out: torch.Tensor, b_out_rows: torch.Tensor, b_head_dim: int, b_act_quant: int,
                               b_key_image: torch.Tensor | None, b_key_inv: torch.Tensor | None,
                               b_key_norm_max: torch.Tensor | None, b_image_stride: int) -> None:
    pa = _decode_params(a_kv, a_score, a_ape, a_norm_w, a_ring_kv, a_ring_score, positions, a_out, a_out_rows,
                        a_head_dim, ratio, rope_head_dim, freqs, eps, None, None, None, 0, a_act_quant)
    pb = _decode_params(b_kv, b_score, b_ape, b_norm_w, b_ring_kv, b_ring_score, positions, b_out, b_out_rows,
                        b_head_dim, ratio, rope_head_dim, freqs, eps, b_key_image, b_key_inv, b_key_norm_max,
                        b_image_stride, b_act_quant)
    L.check(L.lib().dsv4_compressor_decode_pair(ctypes.byref(pa), ctypes.byref(pb), L.stream_of(positions)))


@_compressor_decode_pair_op.register_fake
def _(positions, ratio, rope_head_dim, freqs, eps, a_kv, a_score, a_ape, a_norm_w, a_ring_kv, a_ring_score, a_out,
      a_out_rows, a_head_dim, a_act_quant, b_kv, b_score, b_ape, b_norm_w, b_ring_kv, b_ring_score, b_out, b_out_rows,
      b_head_dim, b_act_quant, b_key_image, b_key_inv, b_key_norm_max, b_image_stride):
    return None


def compressor_decode_pair(a: CompressorStep, b: CompressorStep, positions, ratio=4, rope_head_dim=64, freqs=None,
                           eps=1e-6):
    """Two compressors' decode steps for the same tokens (a decode block's main and indexer
    compressors, oracle/decode_engine.py:96-105 each) in one launch: each is
    `compressor_decode_step(proj=..., key_image=..., act_quant=...)` with its own weights, ring and
    output rows, and the results are the same. Only the second step may carry a key image. The
    custom op `dsv4::compressor_decode_pair`."""
    if a.key_image is not None:
        raise ValueError("compressor_decode_pair: only the second step may append to a key image")
    L.require_cuda(positions, a.ring_kv, a.ring_score, a.out, a.out_rows, b.ring_kv, b.ring_score, b.out, b.out_rows)
    if freqs is None:
        freqs = rope_freqs(rope_head_dim, positions.device)
    img, inv, nmax, stride = b.key_image if b.key_image is not None else (None, None, None, 0)
    _compressor_decode_pair_op(positions, int(ratio), int(rope_head_dim), freqs, float(eps),
                               a.proj[0], a.proj[1], a.ape, a.norm_w, a.ring_kv, a.ring_score, a.out, a.out_rows,
                               int(a.head_dim), int(a.act_quant),
                               b.proj[0], b.proj[1], b.ape, b.norm_w, b.ring_kv, b.ring_score, b.out, b.out_rows,
                               int(b.head_dim), int(b.act_quant), img, inv, nmax, int(stride))
