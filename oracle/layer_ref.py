"""Oracle: attention-block compositions (test infrastructure only).

decode_attention_ref restates the per-token attention of oracle/v4_fast.py:83-119 (and
oracle/step12_glue.py ATTN_NEW): q per-head norm + rope, the window rows in ring order
(ref_torch/sparse_attn.py:11-13), the compressed rows chosen by the indexer (which, with top_k at
least the visible count, is the reference's "all visible rows" list, oracle/v4_fast.py:114-117),
sparse attention, inverse rope of the output.
"""
import torch

from . import indexer_ref as I
from .norm_rope_ref import perhead_norm, rope_at
from .sparse_attn_ref import sparse_attn


def window_slots(p, window=128):
    """Ring slots attended by the token at position p (ref_torch/sparse_attn.py:11-15)."""
    if p >= window - 1:
        sp = p % window
        return list(range(sp + 1, window)) + list(range(0, sp + 1))
    return list(range(0, p + 1)) + [-1] * (window - p - 1)


def decode_attention_ref(kv_pool, win_base, comp_rows, k_idx, q, q_idx, w_idx, sink, positions, top_k, freqs,
                         window=128, ratio=4, scale=512 ** -0.5, return_indices=False):
    """kv_pool [rows, 512] (bf16 values), win_base [b], comp_rows(b, j) -> pool rows, k_idx [b, n, 128],
    q [b, 64, 512], q_idx [b, 64, 128], w_idx [b, 64], sink [64], positions [b] -> o [b, 64, 512] fp32."""
    pool = kv_pool.float()
    outs, all_idx = [], []
    for b in range(q.shape[0]):
        p = int(positions[b])
        qn = rope_at(perhead_norm(q[b].float())[None], torch.tensor([p]), freqs)[0]
        slots = window_slots(p, window)
        rows = [int(win_base[b]) + s if s >= 0 else -1 for s in slots]
        nvis = min((p + 1) // ratio, k_idx.shape[1])
        sc = I.scores(q_idx[b].numpy(), w_idx[b].numpy(), k_idx[b, :nvis].numpy())
        sel = I.select(sc, top_k)
        sel_t = torch.from_numpy(sel.astype("int64"))
        crow = torch.where(sel_t >= 0, comp_rows(b, sel_t.clamp(min=0)), torch.full_like(sel_t, -1))
        idx = torch.tensor(rows + crow.tolist(), dtype=torch.int64)
        o = sparse_attn(qn[None], pool, sink, idx[None], scale)[0]
        outs.append(rope_at(o[None], torch.tensor([p]), freqs, inverse=True)[0])
        all_idx.append(idx)
    out = torch.stack(outs)
    return (out, torch.stack(all_idx)) if return_indices else out
