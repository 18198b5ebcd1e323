"""Long-prefill sparse-MLA core (config 4), on one GPU or query-sharded across GPUs.

For one sequence of s tokens:
  1. KV compressor and indexer-key compressor over the hidden states x (ref_torch/compressor.py:21)
     -> comp [s/4, 512] bf16 and k_idx [s/4, 128] fp32;
  2. per chunk of queries, the indexer top-k over the compressed keys visible at each query
     (causal: j < (t+1)/4), written straight into the attention index list after the 128 window
     rows (the prefill branch of ref_torch/sparse_attn.py:17-19);
  3. sparse attention over [window rows | selected compressed rows] with the inverse RoPE fused.
The q, window kv rows, q_idx and w inputs are the outputs of the projections (layer.py makes them
from x); here they are given.

Multi-GPU (`ShardedPrefill`): the compressor is sequence-sharded — rank r pools compressed rows
[r*G/P, (r+1)*G/P) from its x slice plus one 4-token halo block before it (the overlap slots of a
block read the previous block) — and the compressed rows and indexer keys are all-gathered with
NCCL (`all_gather_into_tensor`), the only exchange. Queries are sharded in zig-zag order (rank r
takes query chunks r and 2P-1-r) so that every rank sees the same causal work; each rank runs steps
2-3 for its own queries against the full gathered cache.
"""
import torch

from . import _lib as L
from .compressor import compressor_prefill
from .indexer import indexer_topk_into
from .norm_rope import rope_freqs
from .sparse_attn import sparse_attn_into

WINDOW = 128


class CompressorWeights:
    """The two compressors of the layer (kv: 512-wide rows; indexer keys: 128-wide)."""

    def __init__(self, c_wkv, c_wgate, c_ape, c_norm, i_wkv, i_wgate, i_ape, i_norm):
        self.c = (c_wkv, c_wgate, c_ape, c_norm)
        self.i = (i_wkv, i_wgate, i_ape, i_norm)

    @classmethod
    def from_attention_weights(cls, W):
        return cls(W.c_wkv, W.c_wgate, W.c_ape, W.c_norm, W.i_wkv, W.i_wgate, W.i_ape, W.i_norm)


def compress_range(x, cw, g0, g1, head_dim=512, idx_dim=128, ratio=4, rope_dim=64):
    """Compressed rows and indexer keys of blocks [g0, g1) of a sequence whose hidden states are x
    (all s tokens, or any slice that covers tokens [4*g0 - 4, 4*g1)); returns (comp bf16, keys fp32)."""
    lo = max(0, ratio * (g0 - 1))
    xs = x[lo:ratio * g1][None]
    comp, _ = compressor_prefill(xs, *cw.c, head_dim=head_dim, ratio=ratio, rope_head_dim=rope_dim,
                                 out_dtype=torch.bfloat16, pos0=lo)
    keys, _ = compressor_prefill(xs, *cw.i, head_dim=idx_dim, ratio=ratio, rope_head_dim=rope_dim,
                                 out_dtype=torch.float32, pos0=lo)
    drop = 1 if g0 > 0 else 0  # the halo block is pooled without its own predecessor: discarded
    return comp[0, drop:], keys[0, drop:]


def attend_queries(q, q_idx, w_idx, kv_rows, comp, keys, sinks, t_begin, t_end, top_k=1024, chunk=8192,
                   out=None, freqs=None, scale=512 ** -0.5):
    """Steps 2-3 for queries [t_begin, t_end) of the sequence. kv_rows [s, 512] bf16 are the window rows
    (token t is row t), comp/keys the full compressed cache. q [n, 64, 512] bf16 (normed, roped),
    q_idx [n, 64, 128] fp32, w_idx [n, 64] fp32 for those queries. Returns o [n, 64, 512] bf16."""
    dev = q.device
    n = t_end - t_begin
    ctx = _Context(kv_rows, comp, keys, sinks, freqs, scale, top_k)
    if out is None:
        out = torch.empty((n, q.shape[1], q.shape[2]), dtype=torch.bfloat16, device=dev)
    for c0 in range(0, n, chunk):
        c1 = min(n, c0 + chunk)
        ctx.attend(out[c0:c1], q[c0:c1], q_idx[c0:c1], w_idx[c0:c1], t_begin + c0)
    return out


class _Context:
    """What every query chunk of one attend call shares: the window rows and the compressed rows in
    one pool (window row t at t, compressed row j at s + j), the keys, the RoPE table."""

    def __init__(self, kv_rows, comp, keys, sinks, freqs, scale, top_k):
        dev = kv_rows.device
        self.s = kv_rows.shape[0]
        n_comp = comp.shape[0]
        self.kvcat = torch.empty((self.s + n_comp, kv_rows.shape[1]), dtype=torch.bfloat16, device=dev)
        self.kvcat[:self.s] = kv_rows
        self.kvcat[self.s:] = comp
        self.keys3 = keys.reshape(1, n_comp, -1)
        self.sinks = sinks.float().contiguous()
        self.freqs = (freqs if freqs is not None else rope_freqs(64, dev)).float().contiguous()
        self.scale, self.top_k = scale, top_k
        self.win_base = torch.zeros(1, dtype=torch.int64, device=dev)

    def attend(self, out, q, q_idx, w_idx, p0):
        """Queries at positions p0 .. p0 + len(q) - 1: the indexer's top-k written after the 128
        window columns of the index list, then the attention with the inverse RoPE, into `out`."""
        m = q.shape[0]
        dev = q.device
        pos = torch.arange(p0, p0 + m, dtype=torch.int32, device=dev)
        idx = torch.empty((1, m, WINDOW + self.top_k), dtype=torch.int32, device=dev)
        indexer_topk_into(idx, q_idx[None], w_idx[None], self.keys3, self.top_k, positions=pos[None], ratio=4,
                          out_col=WINDOW, out_offset=self.s, win_base=self.win_base, window=WINDOW,
                          window_linear=True)
        sparse_attn_into(out, q, self.kvcat, self.sinks, idx[0], self.scale, self.freqs, pos, 64)


class PrefillStaging:
    """Device slots and copy streams for `attend_queries_host`: two slots of each per-chunk buffer
    (q, q_idx, w_idx and the output), so that one chunk computes while the next chunk's inputs and
    the previous chunk's output cross the bus. Reusable across calls on one device."""

    def __init__(self, chunk, device, heads=64, head_dim=512, idx_dim=128):
        dev = torch.device(device)
        self.chunk = chunk
        self.q = [torch.empty((chunk, heads, head_dim), dtype=torch.bfloat16, device=dev) for _ in range(2)]
        self.q_idx = [torch.empty((chunk, heads, idx_dim), dtype=torch.float32, device=dev) for _ in range(2)]
        self.w_idx = [torch.empty((chunk, heads), dtype=torch.float32, device=dev) for _ in range(2)]
        self.o = [torch.empty((chunk, heads, head_dim), dtype=torch.bfloat16, device=dev) for _ in range(2)]
        self.h2d = torch.cuda.Stream(dev)
        self.d2h = torch.cuda.Stream(dev)
        self.free = None  # recorded on the compute stream when the last call's slots are free


def attend_queries_host(h_q, h_q_idx, h_w_idx, kv_rows, comp, keys, sinks, t_begin, t_end, h_out, top_k=1024,
                        chunk=8192, staging=None, freqs=None, scale=512 ** -0.5):
    """`attend_queries` for queries whose inputs and output are in pinned host memory (h_q
    [n, 64, 512] bf16, h_q_idx [n, 64, 128] fp32, h_w_idx [n, 64] fp32 -> h_out [n, 64, 512] bf16):
    per chunk, the inputs cross the bus on one copy stream, the indexer and the attention run on the
    current stream, and the output returns on another copy stream, so that chunk c + 1's inputs and
    chunk c - 1's output move while chunk c computes. The same kernels and chunking as
    `attend_queries`, so h_out holds the same bits. h_out is complete once the current stream has
    synchronized. `staging` (a `PrefillStaging`) can be reused across calls."""
    for name, t in (("h_q", h_q), ("h_q_idx", h_q_idx), ("h_w_idx", h_w_idx), ("h_out", h_out)):
        if t.is_cuda or not t.is_pinned() or not t.is_contiguous():
            raise ValueError(f"attend_queries_host: {name} must be a contiguous pinned host tensor")
    L.require_cuda(kv_rows, comp, keys, sinks)
    dev = kv_rows.device
    n = t_end - t_begin
    if not (h_q.shape[0] == h_q_idx.shape[0] == h_w_idx.shape[0] == h_out.shape[0] == n):
        raise ValueError(f"attend_queries_host: the host tensors must hold the {n} queries of the range")
    st = staging if staging is not None else PrefillStaging(chunk, dev)
    if st.chunk < chunk:
        raise ValueError(f"attend_queries_host: staging slots of {st.chunk} queries for chunks of {chunk}")
    comp_stream = torch.cuda.current_stream(dev)
    ctx = _Context(kv_rows, comp, keys, sinks, freqs, scale, top_k)
    if st.free is not None:
        st.h2d.wait_event(st.free)  # the previous call's chunks are done with the slots
    comp_done, d2h_done = [], []
    for i, c0 in enumerate(range(0, n, chunk)):
        c1 = min(n, c0 + chunk)
        m, k = c1 - c0, i % 2
        with torch.cuda.stream(st.h2d):
            if i >= 2:
                st.h2d.wait_event(comp_done[i - 2])  # chunk i - 2 has read this slot's inputs
            st.q[k][:m].copy_(h_q[c0:c1], non_blocking=True)
            st.q_idx[k][:m].copy_(h_q_idx[c0:c1], non_blocking=True)
            st.w_idx[k][:m].copy_(h_w_idx[c0:c1], non_blocking=True)
            landed = torch.cuda.Event()
            landed.record(st.h2d)
        comp_stream.wait_event(landed)
        if i >= 2:
            comp_stream.wait_event(d2h_done[i - 2])  # chunk i - 2's output has left this slot
        ctx.attend(st.o[k][:m], st.q[k][:m], st.q_idx[k][:m], st.w_idx[k][:m], t_begin + c0)
        ev = torch.cuda.Event()
        ev.record(comp_stream)
        comp_done.append(ev)
        with torch.cuda.stream(st.d2h):
            st.d2h.wait_event(ev)
            h_out[c0:c1].copy_(st.o[k][:m], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(st.d2h)
            d2h_done.append(ev)
    if d2h_done:
        comp_stream.wait_event(d2h_done[-1])  # the copy stream runs in order: every chunk is back
    st.free = torch.cuda.Event()
    st.free.record(comp_stream)
    return h_out


def sparse_mla_prefill(x, q, kv_rows, q_idx, w_idx, sinks, cw, top_k=1024, chunk=8192):
    """Single-GPU config 4: the whole sequence. Returns o [s, 64, 512] bf16."""
    L.require_cuda(x, q, kv_rows, q_idx, w_idx, sinks)
    s = x.shape[0]
    comp, keys = compress_range(x, cw, 0, s // 4)
    return attend_queries(q, q_idx, w_idx, kv_rows, comp, keys, sinks, 0, s, top_k, chunk)


def sparse_mla_prefill_host(h_x, h_q, h_kv_rows, h_q_idx, h_w_idx, sinks, cw, h_out, top_k=1024, chunk=8192,
                            staging=None):
    """`sparse_mla_prefill` from pinned host inputs to a pinned host output: x and the window rows
    cross the bus first (the compressors need x), then `attend_queries_host` overlaps each query
    chunk's transfers with its neighbours' compute. h_out is complete once the current stream has
    synchronized."""
    L.require_cuda(sinks)
    dev = sinks.device
    x = h_x.to(dev, non_blocking=True)
    kv_rows = h_kv_rows.to(dev, non_blocking=True)
    s = x.shape[0]
    comp, keys = compress_range(x, cw, 0, s // 4)
    return attend_queries_host(h_q, h_q_idx, h_w_idx, kv_rows, comp, keys, sinks, 0, s, h_out, top_k, chunk,
                               staging)


def zigzag_ranges(s, world, rank, align=64):
    """Query ranges of `rank`: chunks r and 2P-1-r of 2P equal chunks (causal load balance)."""
    n = 2 * world
    size = (s + n - 1) // n
    size = (size + align - 1) // align * align
    out = []
    for c in (rank, n - 1 - rank):
        a, b = c * size, min(s, (c + 1) * size)
        if a < b:
            out.append((a, b))
    return out


def block_range(n_blocks, world, rank):
    per = n_blocks // world
    return rank * per, (rank + 1) * per


class ShardedPrefill:
    """Query-sharded config 4 over a torch.distributed process group (NCCL on GPUs, gloo on CPU for
    the host-logic tests). Every rank holds the full x / kv rows / inputs it needs; the compressed
    cache is built cooperatively and all-gathered."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def gather_cache(self, comp_local, keys_local, n_blocks):
        """All-gather the per-rank compressed rows and keys into the full cache (rank order)."""
        dev = comp_local.device
        out = []
        for t in (comp_local.contiguous(), keys_local.contiguous()):
            full = torch.empty((n_blocks, t.shape[1]), dtype=t.dtype, device=dev)
            if self.dist.get_backend(self.group) == "nccl":
                self.dist.all_gather_into_tensor(full, t, group=self.group)
            else:  # gloo (host-logic tests): list form
                parts = list(full.chunk(self.world))
                self.dist.all_gather(parts, t, group=self.group)
                full = torch.cat(parts)
            out.append(full)
        return out[0], out[1]

    def run(self, x, q_full, kv_rows, q_idx_full, w_full, sinks, cw, top_k=1024, chunk=8192):
        """Returns [(t_begin, t_end, o)] for this rank's query ranges."""
        s = x.shape[0]
        n_blocks = s // 4
        if n_blocks % self.world:
            raise ValueError("the compressed block count must divide evenly across ranks")
        g0, g1 = block_range(n_blocks, self.world, self.rank)
        comp_l, keys_l = compress_range(x, cw, g0, g1)
        comp, keys = self.gather_cache(comp_l, keys_l, n_blocks)
        outs = []
        for a, b in zigzag_ranges(s, self.world, self.rank):
            o = attend_queries(q_full[a:b], q_idx_full[a:b], w_full[a:b], kv_rows, comp, keys, sinks, a, b,
                               top_k, chunk)
            outs.append((a, b, o))
        return outs
