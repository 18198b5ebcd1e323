"""Oracle: KV compressor prefill and decode ring (restating ref_torch/compressor.py:12-50 and
oracle/decode_engine.py:85-105). Test-only."""
import torch

from .norm_rope_ref import apply_rotary_emb, precompute_freqs, precompute_freqs_cis, rmsnorm, rope_at


def overlap_transform(t, ratio, d, fill):
    """ref_torch/compressor.py:12-18: [b,g,ratio,2d] -> [b,g,2*ratio,d]; slots ratio.. take the group's
    own upper half, slots ..ratio the previous group's lower half (fill for group 0)."""
    b, g = t.shape[0], t.shape[1]
    out = t.new_full((b, g, 2 * ratio, d), fill)
    out[:, :, ratio:] = t[:, :, :, d:]
    out[:, 1:, :ratio] = t[:, :-1, :, :d]
    return out


def compressor_prefill(x, wkv, wgate, ape, norm_w, head_dim=512, ratio=4, rope_head_dim=64,
                       base=160000.0, original_seq_len=65536, factor=16, beta_fast=32, beta_slow=1, pos0=0):
    """ref_torch/compressor.py:21-50 -> (rows [b, s//ratio, head_dim], state). `pos0` (test aid, 0 in
    the reference): x is a slice of a longer sequence starting at position pos0, so row g is roped at
    pos0 + ratio * g (the angles t * freq do not depend on the table's length)."""
    b, s, _ = x.shape
    x = x.float()
    kv = x @ wkv.float().T
    sc = x @ wgate.float().T
    rem = s % ratio
    cut = s - rem
    state = {}
    if cut >= ratio:
        state["kv"] = kv[:, cut - ratio:cut].clone()
        state["score"] = (sc[:, cut - ratio:cut] + ape.float()).clone()
    if rem:
        state["kv_rem"] = kv[:, cut:]
    kv, sc = kv[:, :cut], sc[:, :cut]
    kv = kv.reshape(b, -1, ratio, kv.shape[-1])
    sc = sc.reshape(b, -1, ratio, sc.shape[-1]) + ape.float()
    kv = overlap_transform(kv, ratio, head_dim, 0.0)
    sc = overlap_transform(sc, ratio, head_dim, float("-inf"))
    rows = (kv * sc.softmax(dim=2)).sum(dim=2)
    rows = rmsnorm(rows, norm_w.float())
    cis = precompute_freqs_cis(rope_head_dim, pos0 + s, original_seq_len, base, factor, beta_fast,
                               beta_slow)[pos0:pos0 + cut:ratio]
    rd = rope_head_dim
    rows = torch.cat([rows[..., :-rd], apply_rotary_emb(rows[..., -rd:], cis)], -1)
    return rows, state


def ring_from_prefill(kv_proj, score_proj, ape, s, ratio=4):
    """Decode ring seeded from prefill projections (oracle/decode_engine.py:91-95):
    rows 0..ratio-1 = last full block (kv, score+ape), rows ratio.. = the remainder, rest 0/-inf."""
    b, _, d2 = kv_proj.shape
    rk = torch.zeros(b, 2 * ratio, d2)
    rs = torch.full((b, 2 * ratio, d2), float("-inf"))
    cut = s - s % ratio
    if cut >= ratio:
        rk[:, :ratio] = kv_proj[:, cut - ratio:cut]
        rs[:, :ratio] = score_proj[:, cut - ratio:cut] + ape
    rem = s % ratio
    if rem:
        rk[:, ratio:ratio + rem] = kv_proj[:, cut:]
        rs[:, ratio:ratio + rem] = score_proj[:, cut:] + ape[:rem]
    return rk, rs


def decode_ring_step(ring_kv, ring_score, kv_tok, score_tok, ape, norm_w, pos, freqs, ratio=4, rope_dim=64,
                     eps=1e-6):
    """oracle/decode_engine.py:96-105 for one sequence: writes row ratio + pos%ratio; on a block end
    returns the emitted row (pooled, normed, roped at pos+1-ratio) and shifts the ring. In place."""
    d2 = ring_kv.shape[-1]
    d = d2 // 2
    ring_kv[ratio + pos % ratio] = kv_tok
    ring_score[ratio + pos % ratio] = score_tok + ape[pos % ratio]
    if (pos + 1) % ratio != 0:
        return None
    kve = torch.cat([ring_kv[:ratio, :d], ring_kv[ratio:, d:]], 0)
    sce = torch.cat([ring_score[:ratio, :d], ring_score[ratio:, d:]], 0)
    row = (kve * torch.softmax(sce, 0)).sum(0)
    row = rmsnorm(row[None], norm_w.float(), eps)[0]
    row = rope_at(row[None], torch.tensor([pos + 1 - ratio]), freqs, rope_dim)[0]
    ring_kv[:ratio] = ring_kv[ratio:].clone()
    ring_score[:ratio] = ring_score[ratio:].clone()
    return row
