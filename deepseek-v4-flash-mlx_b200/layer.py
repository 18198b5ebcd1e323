"""The compressed sparse-MLA attention block: prefill (config 1) and decode (config 5).

Prefill follows oracle/decode_engine.py:75-119 (without the hyper-connection mixing around it):
  xn = RMSNorm(x); qa = RMSNorm(x_n Wq_a); q = RoPE(per-head-norm(qa Wq_b))
  kv = RoPE(RMSNorm(xn Wkv))                       -> the window rows (token t is row t)
  comp = compressor_prefill(xn, ...)               -> compressed rows (row s + j)
  indexer: k_idx = compressor_prefill(xn, ... 128-wide), q_idx = RoPE(qa Wq_idx), w = xn Wproj
  index list of query t = [rows max(0,t-127)..t | s + top-k compressed entries visible at t]
  o = inverse-RoPE(sparse_attn(q, [kv; comp], sinks, list)); out = o_grouped(o, Wo_a, Wo_b)
With top_k at least the visible count the list is exactly the reference's (all visible rows).

Decode follows oracle/v4_fast.py:82-122: the token's kv row goes into its window ring slot, the
compressor rings emit a compressed row (and an indexer key) every 4th token, then decode attention
over the device-resident cache and the grouped output projection. Weights may be bf16 or
8-bit grouped (`QuantWeight`, config 5).

Window-only layers (`dims.ratio` 0 or 128): the reference compresses only at ratio 4; its ratio-128
layers keep no compressor ring and no compressed rows, and ratio-0 layers none either
(oracle/v4_fast.py:42-43, 114; oracle/decode_engine.py:87, 112). Their list is the window alone, and
the RoPE table is YaRN(160000, 16, 65536) for ratio 128 and the plain base-10000 table for ratio 0
(oracle/decode_engine.py:47, 73).
"""
import math
from dataclasses import dataclass, fields

import torch

from . import _lib as L
from .compressor import CompressorStep, compressor_decode_pair, compressor_prefill
from .configs import DIMS, LayerDims, window_only
from .decode import SparseMLACache, decode_attention, decode_rows, window_attention
from .hc import hc_post, hc_pre
from .indexer import indexer_topk_into
from .mla import QuantWeight, linear, linear_multi, o_grouped, quantize_int8_g64
from .norm_rope import ROPE_PLAIN, norm_rope, rmsnorm, rope, rope_freqs
from .sparse_attn import get_window_topk_idxs, sparse_attn_rope


@dataclass
class AttentionWeights:
    attn_norm: torch.Tensor     # [dim]
    wq_a: object                # [q_lora, dim]
    q_a_norm: torch.Tensor      # [q_lora]
    wq_b: object                # [heads*head_dim, q_lora]
    wkv: object                 # [head_dim, dim]
    kv_a_norm: torch.Tensor     # [head_dim]
    sinks: torch.Tensor         # [heads]
    wo_a: object                # [groups*o_lora, heads*head_dim/groups]
    wo_b: object                # [dim, groups*o_lora]
    c_wkv: object               # [2*head_dim, dim]  compressor
    c_wgate: object             # [2*head_dim, dim]
    c_ape: torch.Tensor         # [ratio, 2*head_dim]
    c_norm: torch.Tensor        # [head_dim]
    i_wq: object                # [idx_heads*idx_dim, q_lora]  indexer queries
    i_wproj: object             # [idx_heads, dim]             indexer head weights
    i_wkv: object               # [2*idx_dim, dim]             indexer-key compressor
    i_wgate: object             # [2*idx_dim, dim]
    i_ape: torch.Tensor         # [ratio, 2*idx_dim]
    i_norm: torch.Tensor        # [idx_dim]

    def to(self, device):
        def mv(v):
            if isinstance(v, QuantWeight):
                return QuantWeight(v.q.to(device), v.scale.to(device))
            return v.to(device)
        return AttentionWeights(**{f.name: mv(getattr(self, f.name)) for f in fields(self)})


MATRICES = ("wq_a", "wq_b", "wkv", "wo_a", "wo_b", "c_wkv", "c_wgate", "i_wq", "i_wproj", "i_wkv", "i_wgate")


def make_attention_weights(seed, dims: LayerDims = DIMS, quant=False):
    """Synthetic weights on the CPU: matrices ~N(0, 0.02) rounded to bf16 (or int8-g64 when
    `quant`), norm weights 1 + N(0, 0.1), ape ~N(0, 0.1), sinks ~N(0, 1). The indexer head-weight
    matrix carries the 1/sqrt(heads*idx_dim) score scale."""
    g = torch.Generator().manual_seed(seed)
    d, hd, ql = dims.dim, dims.head_dim, dims.q_lora

    def mat(o, i, scale=0.02):
        w = (torch.randn(o, i, generator=g) * scale).to(torch.bfloat16)
        return quantize_int8_g64(w.float()) if quant else w

    def vec(n, base=1.0, scale=0.1):
        return base + torch.randn(n, generator=g) * scale

    return AttentionWeights(
        attn_norm=vec(d), wq_a=mat(ql, d), q_a_norm=vec(ql), wq_b=mat(dims.n_heads * hd, ql),
        wkv=mat(hd, d), kv_a_norm=vec(hd), sinks=torch.randn(dims.n_heads, generator=g),
        wo_a=mat(dims.n_groups * dims.o_lora, dims.n_heads * hd // dims.n_groups),
        wo_b=mat(d, dims.n_groups * dims.o_lora),
        c_wkv=mat(2 * hd, d), c_wgate=mat(2 * hd, d), c_ape=torch.randn(dims.ratio, 2 * hd, generator=g) * 0.1,
        c_norm=vec(hd),
        i_wq=mat(dims.idx_heads * dims.idx_dim, ql), i_wproj=mat(dims.idx_heads, d, 0.02 / math.sqrt(dims.idx_heads * dims.idx_dim) * 8),
        i_wkv=mat(2 * dims.idx_dim, d), i_wgate=mat(2 * dims.idx_dim, d),
        i_ape=torch.randn(dims.ratio, 2 * dims.idx_dim, generator=g) * 0.1, i_norm=vec(dims.idx_dim),
    )


def prefill_layer(x, W: AttentionWeights, top_k=512, dims: LayerDims = DIMS, return_aux=False, act_quant=False):
    """x [s, dim] (one sequence from position 0) -> out [s, dim] fp32 (and the int32 index list
    [s, window + top_k] plus intermediates with return_aux). `act_quant`: the fp8 act-quant
    simulation of the cached kv rows and compressed rows (oracle/decode_engine.py:82,
    v4mlx/compressor.py:60-62). The aux dict also carries the state a decode continues from
    (kv rows and compressed rows in `kvcat`, keys in `k_idx`, the compressors' rings in `ring` and
    `key_ring`): `DecodeBlock.load_prefill` takes it."""
    L.require_cuda(x)
    s = x.shape[0]
    dev = x.device
    freqs = layer_rope_freqs(dims, dev)
    pos = torch.arange(s, dtype=torch.int32, device=dev)
    xn = rmsnorm(x, W.attn_norm)
    qa = rmsnorm(linear(xn, W.wq_a, torch.float32), W.q_a_norm)
    qraw = linear(qa, W.wq_b, torch.float32).view(s, dims.n_heads, dims.head_dim)
    q = norm_rope(qraw, pos, freqs, weight=None, rope_dim=dims.rope_dim)                  # bf16
    if window_only(dims):
        # the window alone (oracle/decode_engine.py:111-114 with nvis = 0): query t attends to rows
        # max(0, t-127)..t, the list of ref_torch/sparse_attn.py:15-18 as an explicit index tensor
        kv = norm_rope(linear(xn, W.wkv, torch.float32), pos, freqs, weight=W.kv_a_norm, rope_dim=dims.rope_dim,
                       act_quant=act_quant)
        idx = get_window_topk_idxs(dims.window, 1, s, 0, device=dev)[0]
        o = sparse_attn_rope(q, kv, W.sinks, idx, dims.head_dim ** -0.5, pos, freqs, dims.rope_dim)
        out = o_grouped(o.reshape(s, -1), W.wo_a, W.wo_b)
        if return_aux:
            return out, dict(idx=idx, o=o, kvcat=kv, q=q)
        return out
    n_comp = s // dims.ratio
    kvcat = torch.empty((s + n_comp, dims.head_dim), dtype=torch.bfloat16, device=dev)
    kvcat[:s] = norm_rope(linear(xn, W.wkv, torch.float32), pos, freqs, weight=W.kv_a_norm, rope_dim=dims.rope_dim,
                          act_quant=act_quant)
    comp, cstate = compressor_prefill(xn[None], W.c_wkv, W.c_wgate, W.c_ape, W.c_norm, head_dim=dims.head_dim,
                                      ratio=dims.ratio, rope_head_dim=dims.rope_dim, out_dtype=torch.bfloat16,
                                      act_quant=act_quant)
    kvcat[s:] = comp[0]
    k_idx, kstate = compressor_prefill(xn[None], W.i_wkv, W.i_wgate, W.i_ape, W.i_norm, head_dim=dims.idx_dim,
                                       ratio=dims.ratio, rope_head_dim=dims.rope_dim, out_dtype=torch.float32)
    q_idx = rope(linear(qa, W.i_wq, torch.float32).view(s, dims.idx_heads, dims.idx_dim), pos, freqs,
                 dims.rope_dim)
    w_idx = linear(xn, W.i_wproj, torch.float32)
    idx = torch.empty((1, s, dims.window + top_k), dtype=torch.int32, device=dev)
    win_base = torch.zeros(1, dtype=torch.int64, device=dev)
    indexer_topk_into(idx, q_idx[None], w_idx[None], k_idx.reshape(1, n_comp, dims.idx_dim), top_k,
                      positions=pos[None], ratio=dims.ratio, out_col=dims.window, out_offset=s,
                      win_base=win_base, window=dims.window, window_linear=True)
    o = sparse_attn_rope(q, kvcat, W.sinks, idx[0], dims.head_dim ** -0.5, pos, freqs, dims.rope_dim)
    out = o_grouped(o.reshape(s, -1), W.wo_a, W.wo_b)
    if return_aux:
        return out, dict(idx=idx[0], o=o, q_idx=q_idx, w_idx=w_idx, k_idx=k_idx, kvcat=kvcat, q=q,
                         ring=(cstate["ring_kv"], cstate["ring_score"]),
                         key_ring=(kstate["ring_kv"], kstate["ring_score"]))
    return out


class DecodeBlock:
    """Device-resident decode state of one layer for a batch of sequences plus its weights
    (config 5): `step(x, positions)` runs the whole attention block for one token per sequence."""

    def __init__(self, W: AttentionWeights, batch, max_ctx, top_k=512, dims: LayerDims = DIMS, device="cuda",
                 page=64, cache=None, act_quant=False):
        self.W, self.dims, self.top_k = W, dims, top_k
        self.act_quant = act_quant  # the fp8 act-quant simulation of cached rows (oracle/decode_engine.py:82, 105)
        self.window_only = window_only(dims)
        self.cache = cache if cache is not None else SparseMLACache(
            batch, 0 if self.window_only else max_ctx // dims.ratio, window=dims.window, head_dim=dims.head_dim,
            idx_dim=dims.idx_dim, ratio=dims.ratio, page=page, device=device)
        if self.window_only and self.cache.compressed:
            raise ValueError("DecodeBlock: a window-only layer (ratio 0 or 128) takes a cache without compressed rows")
        self.freqs = layer_rope_freqs(dims, device)
        self.batch = batch
        b = torch.arange(batch, device=device)
        self._seq = b

    def load_prefill(self, b, aux):
        """Continue sequence b from a `prefill_layer(..., return_aux=True)` of its first s tokens
        (same weights and dims): its window rows, compressed rows, indexer keys and compressor rings
        go into the cache, as the reference's prefill leaves its layer state for the decode steps
        (oracle/decode_engine.py:86-95). The next `step` for b is at position s."""
        s = aux["q"].shape[0]
        if self.window_only:
            self.cache.load_prefill(b, aux["kvcat"][:s])
            return
        if "ring" not in aux:
            raise ValueError("DecodeBlock.load_prefill: the prefill state comes from a window-only layer, this block "
                             "compresses (its dims.ratio is 4)")
        self.cache.load_prefill(b, aux["kvcat"][:s], aux["kvcat"][s:], aux["k_idx"].reshape(-1, self.dims.idx_dim),
                                ring=aux["ring"], key_ring=aux["key_ring"])

    def step(self, x, positions, aux=None):
        """x [b, dim] fp32/bf16, positions int32 [b] (position of this token) -> out [b, dim] fp32.
        `aux` (a dict, for verification) receives the indexer's inputs ("q_idx" after RoPE, "w_idx")
        and the selected pool rows ("idx") of a compressed layer's step."""
        # the normed activations feed only bf16 projections: rounded to bf16 once, by the norm
        return self._attend(rmsnorm(x, self.W.attn_norm, out_dtype=torch.bfloat16), positions, aux)

    def step_hc(self, x, positions, hc_fn, hc_scale, hc_base, sinkhorn_iters=20, hc_eps=1e-6):
        """The block inside its hyper-connections (the decode layer's hc_pre -> attn_norm -> attention
        -> hc_post, oracle/v4_fast.py:85-86, 122): x [b, hc, dim] fp32 residual copies -> [b, hc, dim].
        hc_pre and the attention norm run as one kernel (bf16 output for the projections)."""
        _, post, comb, xn = hc_pre(x, hc_fn, hc_scale, hc_base, sinkhorn_iters=sinkhorn_iters, hc_eps=hc_eps,
                                   norm_w=self.W.attn_norm)
        return hc_post(self._attend(xn, positions), x, post, comb)

    def _attend(self, xn, positions, aux=None):
        d, W, c = self.dims, self.W, self.cache
        b = xn.shape[0]
        pos = positions.to(torch.int32).contiguous()
        if self.window_only:
            # oracle/v4_fast.py:87-92, 110-119 without the ring (w.r4 false): q and kv projections,
            # this token's row into its window slot, attention over the window ring
            qa_p, kvp = linear_multi(xn, [W.wq_a, W.wkv], torch.float32)
            qa = rmsnorm(qa_p, W.q_a_norm, out_dtype=torch.bfloat16)
            qraw = linear(qa, W.wq_b, torch.float32).view(b, d.n_heads, d.head_dim)
            win_rows, _, _ = decode_rows(c, pos)
            _norm_rope_into(kvp, W.kv_a_norm, pos, self.freqs, c.kv_pool, win_rows, d.rope_dim, self.act_quant)
            o = window_attention(c, qraw, W.sinks, pos, freqs=self.freqs)
            return o_grouped(o.reshape(b, -1), W.wo_a, W.wo_b)
        # the seven projections of xn run as one launch, the two of qa as another
        qa_p, kvp, c_kv, c_sc, w_idx, i_kv, i_sc = linear_multi(
            xn, [W.wq_a, W.wkv, W.c_wkv, W.c_wgate, W.i_wproj, W.i_wkv, W.i_wgate], torch.float32)
        qa = rmsnorm(qa_p, W.q_a_norm, out_dtype=torch.bfloat16)
        qraw, qi = linear_multi(qa, [W.wq_b, W.i_wq], torch.float32)
        qraw = qraw.view(b, d.n_heads, d.head_dim)
        # this token's window slot, and where the compressors emit (when (p+1) % ratio == 0)
        win_rows, comp_rows, key_rows = decode_rows(c, pos)
        _norm_rope_into(kvp, W.kv_a_norm, pos, self.freqs, c.kv_pool, win_rows, d.rope_dim, self.act_quant)
        # the main and indexer compressors' ring steps in one launch
        compressor_decode_pair(
            CompressorStep((c_kv, c_sc), W.c_ape, W.c_norm, c.ring_kv, c.ring_score, c.kv_pool, comp_rows,
                           d.head_dim, act_quant=int(self.act_quant)),
            CompressorStep((i_kv, i_sc), W.i_ape, W.i_norm, c.ring_k_idx, c.ring_s_idx, c.k_idx.view(-1, d.idx_dim),
                           key_rows, d.idx_dim, key_image=(*c.key_image, c.max_comp)),
            pos, ratio=d.ratio, rope_head_dim=d.rope_dim, freqs=self.freqs)
        q_idx = rope(qi.view(b, d.idx_heads, d.idx_dim), pos, self.freqs, d.rope_dim)
        idx_buf = None
        if aux is not None:
            idx_buf = torch.empty((b, self.top_k), dtype=torch.int32, device=xn.device)
            aux.update(q_idx=q_idx, w_idx=w_idx, idx=idx_buf)
        o = decode_attention(c, qraw, q_idx, w_idx, W.sinks, pos, self.top_k, freqs=self.freqs, idx_buf=idx_buf)
        return o_grouped(o.reshape(b, -1), W.wo_a, W.wo_b)


def layer_rope_freqs(dims: LayerDims, device):
    """RoPE table of a layer: plain base 10000 for ratio 0, YaRN(160000, 16, 65536) otherwise
    (oracle/decode_engine.py:47, 73; oracle/v4_fast.py:83)."""
    if dims.ratio == 0:
        return rope_freqs(dims.rope_dim, device, **ROPE_PLAIN)
    return rope_freqs(dims.rope_dim, device)


def _norm_rope_into(x, weight, positions, freqs, pool, rows, rope_dim, act_quant=False):
    """RMSNorm(weight) + RoPE of x [b, dim] written as bf16 into pool rows `rows` (int64 [b])."""
    p = L.NormRopeParams()
    p.x, p.weight, p.out, p.out_rows = L.ptr(x), L.ptr(weight), L.ptr(pool), L.ptr(rows)
    p.rows, p.heads, p.dim, p.rope_dim = x.shape[0], 1, x.shape[-1], rope_dim
    p.x_dtype, p.w_dtype, p.out_dtype = L.dtype_code(x), L.dtype_code(weight), L.BF16
    p.eps = 1e-6
    p.freqs, p.positions = L.ptr(freqs), L.ptr(positions)
    p.act_quant = int(act_quant)
    L.check(L.lib().dsv4_norm_rope(ctypes_byref(p), L.stream_of(x)))


def ctypes_byref(p):
    import ctypes
    return ctypes.byref(p)


class BlockRunner:
    """A `DecodeBlock`'s step from pinned host memory to pinned host memory, one CUDA graph launch
    per token (the serving-loop form of config 5): the graph holds a copy kernel that brings this
    token's hidden states and positions in from one pinned block (x [b, dim] fp32 and positions
    int32 [b] at fixed offsets), the block's kernels, and a copy kernel that stores the block's
    output [b, dim] fp32 into a pinned host tensor.

    The block's step changes its cache (this token's window row, the compressors' rings), so the
    first `step_host` runs eagerly, as the token it is, and only then captures the graph that the
    later calls replay. Callers that write their inputs straight into `host_inputs()` skip the
    host-side staging copy. The returned output is valid after `synchronize()` and until the next
    step."""

    def __init__(self, block: DecodeBlock, stream=None):
        self.block = block
        b, dim = block.batch, block.dims.dim
        dev = block.cache.kv_pool.device
        x_bytes = -(-b * dim * 4 // 256) * 256
        self._in_bytes = x_bytes + -(-b * 4 // 256) * 256
        self.d_in = torch.zeros(self._in_bytes, dtype=torch.uint8, device=dev)
        self.h_in = torch.zeros(self._in_bytes, dtype=torch.uint8).pin_memory()
        self.x = self.d_in[:b * dim * 4].view(torch.float32).view(b, dim)
        self.positions = self.d_in[x_bytes:x_bytes + b * 4].view(torch.int32)
        self.h_x = self.h_in[:b * dim * 4].view(torch.float32).view(b, dim)
        self.h_pos = self.h_in[x_bytes:x_bytes + b * 4].view(torch.int32)
        self.h_out = torch.empty((b, dim), dtype=torch.float32).pin_memory()
        self.stream = stream or torch.cuda.Stream(dev)
        self.graph = None
        self._done = None

    def _body(self):
        L.copy_(self.d_in, self.h_in)
        out = self.block.step(self.x, self.positions)
        L.copy_(self.h_out, out)

    def host_inputs(self):
        """The pinned host views (x, positions) that `step_host` copies from."""
        return self.h_x, self.h_pos

    def step_host(self, x=None, positions=None):
        """Host x [b, dim] and positions [b] in (or None: the `host_inputs()` views as they are),
        the block's output [b, dim] fp32 out, in pinned host memory."""
        if x is not None or positions is not None:
            if self._done is not None:
                self._done.synchronize()   # the previous step has read the pinned block
            if x is not None:
                self.h_x.copy_(x)
            if positions is not None:
                self.h_pos.copy_(positions)
        with torch.cuda.stream(self.stream):
            if self.graph is None:
                self._body()               # this token, eagerly; then the graph for the next ones
                self.graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(self.graph, stream=self.stream):
                    self._body()
            else:
                self.graph.replay()
            if self._done is None:
                self._done = torch.cuda.Event()
            self._done.record(self.stream)
        return self.h_out

    def h2d_bytes(self):
        return self._in_bytes

    def d2h_bytes(self):
        return self.h_out.numel() * 4

    def synchronize(self):
        self.stream.synchronize()

    def release(self):
        """Drop the captured graph (its memory returns to torch's graph pool)."""
        self.stream.synchronize()
        self.graph = None
