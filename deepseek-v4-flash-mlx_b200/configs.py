"""Layer dimensions and seeded synthetic inputs for the benchmark configurations.

Shapes follow the reference defaults (v4mlx/mla.py:12-13; ref_torch/compressor.py:21;
oracle/decode_engine.py:17,47,111): 64 query heads, a 512-wide latent row whose last 64 dims carry
RoPE, compression ratio 4, a 128-token window, YaRN(160000, 16, 65536). The indexer has 64 heads of
128 dims. All data is synthetic (there is no dataset or checkpoint): torch.Generator on the CPU,
seeded per configuration, so the oracle and the GPU see identical values.
"""
from dataclasses import dataclass

import torch

from .decode import SparseMLACache


@dataclass(frozen=True)
class LayerDims:
    dim: int = 4096
    n_heads: int = 64
    head_dim: int = 512
    rope_dim: int = 64
    q_lora: int = 1024
    window: int = 128
    ratio: int = 4
    idx_heads: int = 64
    idx_dim: int = 128
    n_groups: int = 8
    o_lora: int = 1024


DIMS = LayerDims()

# Ratios whose layers attend over the sliding window alone: ratio 0 (the dense-attention layers, RoPE
# base 10000 without YaRN) and ratio 128, which the reference engine runs with neither a compressor
# ring nor compressed rows (oracle/v4_fast.py:42-43, 114; oracle/decode_engine.py:17, 47, 112).
WINDOW_ONLY_RATIOS = (0, 128)


def window_only(dims: LayerDims) -> bool:
    return dims.ratio in WINDOW_ONLY_RATIOS


@dataclass
class DecodeCase:
    """A batch of decode tokens against pre-filled caches (configs 2 and 3)."""
    cache: SparseMLACache
    q: torch.Tensor          # [b, 64, 512] fp32 (before the per-head norm)
    q_idx: torch.Tensor      # [b, 64, 128] fp32
    w_idx: torch.Tensor      # [b, 64] fp32
    sink: torch.Tensor       # [64] fp32
    positions: torch.Tensor  # [b] int32
    top_k: int
    host: dict               # CPU copies for the oracle


def make_decode_case(batch, ctx, top_k=512, seeds=None, device="cuda", page=64, shuffle_pages=True, dims=DIMS):
    """Every sequence has `ctx` tokens of context: ctx // ratio compressed rows (bf16 ~N(0,1)),
    a full 128-row window ring (bf16 ~N(0,1)) and fp32 ~N(0,1) indexer keys; the new token sits at
    position ctx - 1. q ~N(0,1), q_idx ~N(0,1), w ~N(0,1)/8, sink ~N(0,1). Sequence b uses
    seeds[b]. With shuffle_pages the block table maps compressed pages to a permuted pool order."""
    seeds = seeds if seeds is not None else list(range(batch))
    n_comp = ctx // dims.ratio
    pages_per_seq = (n_comp + page - 1) // page
    order = None
    if shuffle_pages:
        order = torch.randperm(batch * pages_per_seq, generator=torch.Generator().manual_seed(12345))
    cache = SparseMLACache(batch, n_comp, window=dims.window, head_dim=dims.head_dim, idx_dim=dims.idx_dim,
                           ratio=dims.ratio, page=page, device=device, page_order=order)
    qs, qis, ws, comp_h, win_h, keys_h = [], [], [], [], [], []
    sink = None
    for b in range(batch):
        g = torch.Generator().manual_seed(int(seeds[b]))
        comp = torch.randn(n_comp, dims.head_dim, generator=g).to(torch.bfloat16)
        win = torch.randn(dims.window, dims.head_dim, generator=g).to(torch.bfloat16)
        keys = torch.randn(n_comp, dims.idx_dim, generator=g)
        q = torch.randn(dims.n_heads, dims.head_dim, generator=g)
        q_idx = torch.randn(dims.idx_heads, dims.idx_dim, generator=g)
        w = torch.randn(dims.idx_heads, generator=g) / 8
        if b == 0:
            sink = torch.randn(dims.n_heads, generator=g)
        cache.fill_compressed(b, comp.to(device), keys.to(device))
        cache.fill_window(b, torch.arange(dims.window, device=device), win.to(device))
        qs.append(q), qis.append(q_idx), ws.append(w)
        comp_h.append(comp), win_h.append(win), keys_h.append(keys)
    if str(device).startswith("cuda"):
        cache.refresh_key_image()
    positions = torch.full((batch,), ctx - 1, dtype=torch.int32)
    host = dict(q=torch.stack(qs), q_idx=torch.stack(qis), w_idx=torch.stack(ws), sink=sink, positions=positions,
                k_idx=torch.stack(keys_h))
    return DecodeCase(cache, host["q"].to(device), host["q_idx"].to(device), host["w_idx"].to(device),
                      sink.to(device), positions.to(device), top_k, host)


def decode_case_host_pool(case):
    """CPU copies of the pool and the addressing used by the oracle."""
    c = case.cache
    pool = c.kv_pool.cpu()
    bt = c.block_table.cpu().long()

    def comp_rows(b, j):
        return c.comp_base + bt[b][j // c.page] * c.page + j % c.page

    return pool, c.win_base.cpu(), comp_rows
