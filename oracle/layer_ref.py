"""Oracle: attention-block compositions (test infrastructure only).

decode_attention_ref restates the per-token attention of oracle/v4_fast.py:83-119 (and
oracle/step12_glue.py ATTN_NEW): q per-head norm + rope, the window rows in ring order
(ref_torch/sparse_attn.py:11-13), the compressed rows chosen by the indexer (which, with top_k at
least the visible count, is the reference's "all visible rows" list, oracle/v4_fast.py:114-117),
sparse attention, inverse rope of the output. window_attention_ref is the same for the window-only
layers (ratio 0 and 128), whose list holds the window rows alone (oracle/decode_engine.py:112).
"""
import torch

from . import indexer_ref as I
from .norm_rope_ref import perhead_norm, rope_at
from .sparse_attn_ref import sparse_attn, sparse_attn_chunked


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


def window_attention_ref(kv_pool, win_base, q, sink, positions, freqs, window=128, scale=512 ** -0.5):
    """Decode attention of a window-only layer (ratio 0 or 128): oracle/v4_fast.py:110-119 with
    nvis = 0, i.e. q per-head norm + rope, the window rows alone in ring order, sparse attention,
    inverse rope of the output. kv_pool [rows, 512], win_base [b], q [b, 64, 512] -> o [b, 64, 512]."""
    pool = kv_pool.float()
    outs = []
    for b in range(q.shape[0]):
        p = int(positions[b])
        qn = rope_at(perhead_norm(q[b].float())[None], torch.tensor([p]), freqs)[0]
        rows = [int(win_base[b]) + s if s >= 0 else -1 for s in window_slots(p, window)]
        o = sparse_attn(qn[None], pool, sink, torch.tensor([rows], dtype=torch.int64), scale)[0]
        outs.append(rope_at(o[None], torch.tensor([p]), freqs, inverse=True)[0])
    return torch.stack(outs)


def layer_freqs(ratio, rope_dim=64):
    """The layer's RoPE table (oracle/decode_engine.py:47, 73): base 10000 without YaRN at ratio 0,
    YaRN(160000, factor 16, original 65536, beta 32/1) for the compressed-table layers (ratio 4, 128)."""
    from .norm_rope_ref import precompute_freqs
    if ratio == 0:
        return precompute_freqs(rope_dim, 0, 0, 10000.0, 40, 32, 1)
    return precompute_freqs(rope_dim, 0, 65536, 160000.0, 16, 32, 1)


def is_window_only(ratio):
    """The reference compresses only at ratio 4 (oracle/v4_fast.py:42: "ring/comp ONLY at ratio 4");
    ratio-0 and ratio-128 layers attend over the window alone (oracle/decode_engine.py:112)."""
    return ratio in (0, 128)


# ---------------------------------------------------------------------------- full block
def _w(v):
    """fp32 value of a weight (bf16 tensor or an 8-bit grouped weight)."""
    if hasattr(v, "q") and hasattr(v, "scale"):
        return v.q.float() * v.scale.float().repeat_interleave(64, dim=-1)
    return v.float()


def prefill_layer_ref(x, W, top_k=512, window=128, ratio=4, heads=64, head_dim=512, idx_heads=64, idx_dim=128,
                      rope_dim=64, groups=8, indexer_inputs=None, act_quant=False, return_state=False):
    """fp32 restatement of oracle/decode_engine.py:75-119 plus the indexer selection.
    indexer_inputs=(q_idx, w_idx, k_idx) lets a test score the selection on given inputs.
    Returns (out [s, dim], idx [s, window + top_k], o [s, heads, head_dim]); with return_state also
    the state the reference's prefill leaves for its decode steps (oracle/decode_engine.py:86-95):
    dict(kv [s, head_dim] rows, comp [s//ratio, head_dim] rows, k_idx keys, ring / key_ring =
    (ring_kv, ring_score) [1, 2*ratio, 2*dim] seeded from the compressors' projections)."""
    from .compressor_ref import compressor_prefill
    from .mla_ref import o_grouped
    from .norm_rope_ref import rmsnorm
    s = x.shape[0]
    f = layer_freqs(ratio, rope_dim)
    pos = torch.arange(s)
    xn = rmsnorm(x.float(), W.attn_norm)
    qa = rmsnorm(xn @ _w(W.wq_a).T, W.q_a_norm)
    q = rope_at(perhead_norm((qa @ _w(W.wq_b).T).reshape(s, heads, head_dim)), pos, f, rope_dim)
    kv = rope_at(rmsnorm(xn @ _w(W.wkv).T, W.kv_a_norm), pos, f, rope_dim)
    win = torch.stack([torch.tensor([max(0, t - window + 1) + c if max(0, t - window + 1) + c <= t else -1
                                     for c in range(window)]) for t in range(s)])
    if is_window_only(ratio):
        # oracle/decode_engine.py:108-116 with nvis = 0: the window rows alone (widx)
        if act_quant:
            from .quant_ref import act_quant_rows
            kv = act_quant_rows(kv, rope_dim)
        idx = win[:, :min(s, window)]
        o = sparse_attn_chunked(q, kv, W.sinks, idx, head_dim ** -0.5)
        o = rope_at(o, pos, f, rope_dim, inverse=True)
        res = (o_grouped(o.reshape(s, -1), _w(W.wo_a), _w(W.wo_b), groups=groups), idx, o)
        return (*res, dict(kv=kv)) if return_state else res
    comp, _ = compressor_prefill(xn[None], _w(W.c_wkv), _w(W.c_wgate), W.c_ape, W.c_norm, head_dim=head_dim,
                                 ratio=ratio, rope_head_dim=rope_dim)
    if act_quant:  # oracle/decode_engine.py:82 (kv rows) and the compressor's sim (v4mlx/compressor.py:60-62)
        from .quant_ref import act_quant_rows
        kv = act_quant_rows(kv, rope_dim)
        comp = act_quant_rows(comp, rope_dim)
    if indexer_inputs is None:
        k_idx, _ = compressor_prefill(xn[None], _w(W.i_wkv), _w(W.i_wgate), W.i_ape, W.i_norm, head_dim=idx_dim,
                                      ratio=ratio, rope_head_dim=rope_dim)
        q_idx = rope_at((qa @ _w(W.i_wq).T).reshape(s, idx_heads, idx_dim), pos, f, rope_dim)
        w_idx = xn @ _w(W.i_wproj).T
        k_idx = k_idx[0]
    else:
        q_idx, w_idx, k_idx = indexer_inputs
    sel = I.indexer_topk(q_idx.numpy()[None], w_idx.numpy()[None], k_idx.numpy()[None], top_k,
                         positions=pos.numpy()[None], ratio=ratio)[0]
    sel_t = torch.from_numpy(sel.astype("int64"))
    idx = torch.cat([win, torch.where(sel_t >= 0, sel_t + s, sel_t)], 1)
    kvcat = torch.cat([kv, comp[0]], 0)
    o = sparse_attn_chunked(q, kvcat, W.sinks, idx, head_dim ** -0.5)
    o = rope_at(o, pos, f, rope_dim, inverse=True)
    out = o_grouped(o.reshape(s, -1), _w(W.wo_a), _w(W.wo_b), groups=groups)
    if not return_state:
        return out, idx, o
    from .compressor_ref import ring_from_prefill
    ring = ring_from_prefill((xn @ _w(W.c_wkv).T)[None], (xn @ _w(W.c_wgate).T)[None], W.c_ape, s, ratio)
    key_ring = ring_from_prefill((xn @ _w(W.i_wkv).T)[None], (xn @ _w(W.i_wgate).T)[None], W.i_ape, s, ratio)
    return out, idx, o, dict(kv=kv, comp=comp[0], k_idx=k_idx, ring=ring, key_ring=key_ring)


def decode_block_ref(state, W, x, positions, top_k=512, window=128, ratio=4, heads=64, head_dim=512, idx_heads=64,
                     idx_dim=128, rope_dim=64, groups=8, act_quant=False, indexer_inputs=None, aux=None):
    """One decode token per sequence on host copies of the cache (oracle/v4_fast.py:82-122,
    oracle/decode_engine.py:96-105). `state` = dict(pool, win_base, comp_rows(b, j), k_idx, ring_kv, ring_score,
    ring_k, ring_s) and is updated in place. Returns out [b, dim]. With act_quant the token's kv row and
    the emitted compressed rows take the fp8 act-quant simulation on their nope dims before they are
    cached (oracle/decode_engine.py:82, 105). indexer_inputs=(q_idx after RoPE [b, 64, 128], w_idx [b, 64],
    k_idx [b, n, 128]) lets a test select on given indexer inputs (the rest of the block stays the
    oracle's); `aux` (a dict) receives the attention index lists under "idx"."""
    from .quant_ref import act_quant_rows
    from .compressor_ref import decode_ring_step
    from .mla_ref import o_grouped
    from .norm_rope_ref import rmsnorm
    f = layer_freqs(ratio, rope_dim)
    b = x.shape[0]
    xn = rmsnorm(x.float(), W.attn_norm)
    qa = rmsnorm(xn @ _w(W.wq_a).T, W.q_a_norm)
    qraw = (qa @ _w(W.wq_b).T).reshape(b, heads, head_dim)
    kvp = rmsnorm(xn @ _w(W.wkv).T, W.kv_a_norm)
    if is_window_only(ratio):
        # oracle/v4_fast.py:87-96, 110-122 without the ring (w.r4 false): state = dict(pool, win_base)
        for i in range(b):
            p = int(positions[i])
            row = rope_at(kvp[i][None], torch.tensor([p]), f, rope_dim)[0]
            if act_quant:
                row = act_quant_rows(row, rope_dim)
            state["pool"][int(state["win_base"][i]) + p % window] = row.to(torch.bfloat16).float()
        o = window_attention_ref(state["pool"], state["win_base"], qraw, W.sinks, positions, f, window=window,
                                 scale=head_dim ** -0.5)
        return o_grouped(o.reshape(b, -1), _w(W.wo_a), _w(W.wo_b), groups=groups)
    ckv, cgt = xn @ _w(W.c_wkv).T, xn @ _w(W.c_wgate).T
    ikv, igt = xn @ _w(W.i_wkv).T, xn @ _w(W.i_wgate).T
    q_idx = (qa @ _w(W.i_wq).T).reshape(b, idx_heads, idx_dim)
    w_idx = xn @ _w(W.i_wproj).T
    for i in range(b):
        p = int(positions[i])
        row = rope_at(kvp[i][None], torch.tensor([p]), f, rope_dim)[0]
        if act_quant:
            row = act_quant_rows(row, rope_dim)
        state["pool"][int(state["win_base"][i]) + p % window] = row.to(torch.bfloat16).float()
        emitted = decode_ring_step(state["ring_kv"][i], state["ring_score"][i], ckv[i], cgt[i], W.c_ape, W.c_norm, p, f,
                                   ratio, rope_dim)
        if emitted is not None:
            if act_quant:
                emitted = act_quant_rows(emitted, rope_dim)
            e = (p + 1) // ratio - 1
            state["pool"][int(state["comp_rows"](i, torch.tensor(e)))] = emitted.to(torch.bfloat16).float()
        key = decode_ring_step(state["ring_k"][i], state["ring_s"][i], ikv[i], igt[i], W.i_ape, W.i_norm, p, f, ratio,
                               rope_dim)
        if key is not None:
            state["k_idx"][i, (p + 1) // ratio - 1] = key
        q_idx[i] = rope_at(q_idx[i][None], torch.tensor([p]), f, rope_dim)[0]
    keys = state["k_idx"]
    if indexer_inputs is not None:
        q_idx, w_idx, keys = indexer_inputs
    o, idx = decode_attention_ref(state["pool"], state["win_base"], state["comp_rows"], keys, qraw, q_idx, w_idx,
                                  W.sinks, positions, top_k, f, window=window, ratio=ratio, scale=head_dim ** -0.5,
                                  return_indices=True)
    if aux is not None:
        aux["idx"] = idx
    return o_grouped(o.reshape(b, -1), _w(W.wo_a), _w(W.wo_b), groups=groups)


def decode_block_hc_ref(state, W, x, positions, hc_fn, hc_scale, hc_base, **kw):
    """The block inside its hyper-connections (oracle/v4_fast.py:85, 122): x [b, hc, dim] ->
    hc_post(block(hc_pre(x)), x) [b, hc, dim], in float64 for the mixes (hc_ref) and the block's
    own oracle in between. Returns (out, post, comb) as torch float32 / float64."""
    from . import hc_ref as H
    y, post, comb = H.hc_pre(x.numpy(), hc_fn.numpy(), hc_scale.numpy(), hc_base.numpy())
    att = decode_block_ref(state, W, torch.from_numpy(y).float(), positions, **kw)
    out = H.hc_post(att.double().numpy(), x.numpy(), post, comb)
    return torch.from_numpy(out), post, comb
