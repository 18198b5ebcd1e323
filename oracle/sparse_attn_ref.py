"""Oracle: sparse attention and window indices (restating ref_torch/sparse_attn.py). Test-only."""
import torch


def get_window_topk_idxs(window_size, bsz, seqlen, start_pos):
    """ref_torch/sparse_attn.py:9-20, all three branches, int64 [bsz, seqlen|1, cols]."""
    if start_pos >= window_size - 1:
        sp = start_pos % window_size
        row = torch.cat([torch.arange(sp + 1, window_size), torch.arange(0, sp + 1)])
        mat = row[None]
    elif start_pos > 0:
        row = torch.full((window_size,), -1, dtype=torch.int64)
        row[: start_pos + 1] = torch.arange(start_pos + 1)
        mat = row[None]
    else:
        i = torch.arange(seqlen)[:, None]
        cols = min(seqlen, window_size)
        mat = (i - window_size + 1).clamp(min=0) + torch.arange(cols)[None]
        mat = torch.where(mat > i, torch.full_like(mat, -1), mat)
    return mat[None].expand(bsz, -1, -1)


def sparse_attn(q, kv, attn_sink, topk_idxs, scale):
    """ref_torch/sparse_attn.py:23-34: masked dense-gather softmax with the sink in the denominator.
    q [s,h,d], kv [n,d], attn_sink [h], topk_idxs [s,T] -> [s,h,d] (fp32)."""
    q, kv, attn_sink = q.float(), kv.float(), attn_sink.float()
    ok = topk_idxs >= 0
    rows = kv[topk_idxs.clamp(min=0).long()]                      # [s, T, d]
    logits = torch.einsum("shd,std->sht", q, rows) * scale
    logits = logits.masked_fill(~ok[:, None, :], float("-inf"))
    m = logits.amax(-1, keepdim=True)
    e = torch.exp(logits - m)
    den = e.sum(-1, keepdim=True) + torch.exp(attn_sink[None, :, None] - m)
    return torch.einsum("sht,std->shd", e, rows) / den


def sparse_attn_chunked(q, kv, attn_sink, topk_idxs, scale, chunk=256):
    """Same result in query chunks (bounded memory for long prefill)."""
    outs = [sparse_attn(q[i:i + chunk], kv, attn_sink, topk_idxs[i:i + chunk], scale)
            for i in range(0, q.shape[0], chunk)]
    return torch.cat(outs) if outs else q.float().clone()
