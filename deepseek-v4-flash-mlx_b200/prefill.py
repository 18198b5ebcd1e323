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
from .sparse_attn import sparse_attn_rope

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
    s = kv_rows.shape[0]
    n_comp = comp.shape[0]
    if freqs is None:
        freqs = rope_freqs(64, dev)
    kvcat = torch.empty((s + n_comp, kv_rows.shape[1]), dtype=torch.bfloat16, device=dev)
    kvcat[:s] = kv_rows
    kvcat[s:] = comp
    if out is None:
        out = torch.empty((n, q.shape[1], q.shape[2]), dtype=torch.bfloat16, device=dev)
    win_base = torch.zeros(1, dtype=torch.int64, device=dev)
    keys3 = keys.reshape(1, n_comp, -1)
    for c0 in range(0, n, chunk):
        c1 = min(n, c0 + chunk)
        pos = torch.arange(t_begin + c0, t_begin + c1, dtype=torch.int32, device=dev)
        idx = torch.empty((1, c1 - c0, WINDOW + top_k), dtype=torch.int32, device=dev)
        indexer_topk_into(idx, q_idx[c0:c1][None], w_idx[c0:c1][None], keys3, top_k, positions=pos[None], ratio=4,
                          out_col=WINDOW, out_offset=s, win_base=win_base, window=WINDOW, window_linear=True)
        out[c0:c1] = sparse_attn_rope(q[c0:c1], kvcat, sinks, idx[0], scale, pos, freqs, 64)
    return out


def sparse_mla_prefill(x, q, kv_rows, q_idx, w_idx, sinks, cw, top_k=1024, chunk=8192):
    """Single-GPU config 4: the whole sequence. Returns o [s, 64, 512] bf16."""
    L.require_cuda(x, q, kv_rows, q_idx, w_idx, sinks)
    s = x.shape[0]
    comp, keys = compress_range(x, cw, 0, s // 4)
    return attend_queries(q, q_idx, w_idx, kv_rows, comp, keys, sinks, 0, s, top_k, chunk)


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
