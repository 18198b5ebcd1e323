"""Generate tests/golden/mla_golden.npz from the reference's own v4mlx/mla.py and v4mlx/sparse_attn.py
on seeded inputs.

Run where a checkout of the reference project is available:
    python tests/golden/make_mla_golden.py <reference checkout>
The module imports mlx, which is absent here (no Apple GPU). Its projection functions use only `@`,
`.T`, `reshape`, `.square()`, `mean`, `mx.rsqrt` and `mx.stack`, so they run unchanged on numpy
arrays given a small stand-in for `mlx.core` that provides those two functions. The module's shape
constants (heads, head dim, groups, o_lora) are read when a function runs, so they are set to small
values for small fixtures; the code path is the reference's own. Recorded (inputs included):
q_down, q_up, perhead_norm, kv_proj and o_grouped (v4mlx/mla.py:16-56); the MLX twin of sparse
attention and of the prefill window list (v4mlx/sparse_attn.py:16-39), which need `arange`,
`maximum`, `where`, `einsum`, `exp` and `inf` from the stand-in; and the MLX twin of the compressor
(v4mlx/compressor.py:32-63) without and with its fp8 simulation, and as the indexer-key compressor
with `rotate`, for which the stand-in also gives `float32`, `full`, `array`, `concatenate`, `clip`,
`cos`, `sin` and a softmax along one axis; and the MLX twin of the hyper-connections
(v4mlx/hc.py: hc_pre, hc_post, hc_head), which adds `sigmoid` and `sum`; and the MLX twin of the
norm and RoPE (v4mlx/norm_rope.py: precompute_freqs, the cos/sin rotation forward and inverse,
rmsnorm).
"""
import os
import sys
import types

import numpy as np

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "mla_golden.npz")


class _Array(np.ndarray):
    """numpy array with the one array method the module calls that numpy lacks."""

    def square(self):
        return np.square(self)


def _install_mlx_stand_in():
    core = types.ModuleType("mlx.core")
    core.rsqrt = lambda x: (1.0 / np.sqrt(x)).astype(np.float32)
    core.stack = np.stack
    core.arange, core.maximum, core.where, core.einsum, core.exp = np.arange, np.maximum, np.where, np.einsum, np.exp
    core.inf = np.float32(np.inf)
    core.float32, core.clip, core.cos, core.sin = np.float32, np.clip, np.cos, np.sin

    def wrap(fn):  # results keep the array method the reference code calls (`.square()`)
        return lambda *a, **k: np.asarray(fn(*a, **k)).view(_Array)

    def softmax(a, axis):
        e = np.exp(a - a.max(axis=axis, keepdims=True))
        return e / e.sum(axis=axis, keepdims=True)
    core.full, core.array, core.concatenate, core.softmax = (wrap(np.full), wrap(np.asarray),
                                                             wrap(np.concatenate), wrap(softmax))
    core.sigmoid = wrap(lambda a: 1.0 / (1.0 + np.exp(-a)))
    core.sum = wrap(np.sum)
    pkg = types.ModuleType("mlx")
    pkg.core = core
    sys.modules["mlx"], sys.modules["mlx.core"] = pkg, core


def main(ref_root):
    _install_mlx_stand_in()
    sys.path.insert(0, ref_root)
    from v4mlx import mla as M

    M.N_HEADS, M.HEAD_DIM, M.N_GROUPS, M.O_LORA = 8, 32, 8, 16
    rng = np.random.default_rng(20)

    def arr(*shape, scale=1.0):
        return (rng.standard_normal(shape) * scale).astype(np.float32).view(_Array)

    dim, q_lora, s = 64, 32, 3
    x = arr(s, dim)
    wq_a, wq_b = arr(q_lora, dim, scale=0.1), arr(M.N_HEADS * M.HEAD_DIM, q_lora, scale=0.1)
    wkv = arr(M.HEAD_DIM, dim, scale=0.1)
    o = arr(s, M.N_HEADS * M.HEAD_DIM)
    wo_a = arr(M.N_GROUPS * M.O_LORA, M.N_HEADS * M.HEAD_DIM // M.N_GROUPS, scale=0.1)
    wo_b = arr(dim, M.N_GROUPS * M.O_LORA, scale=0.1)
    qa = M.q_down(x, wq_a)
    qraw = M.q_up(qa, wq_b)
    g = dict(mla_x=x, mla_wq_a=wq_a, mla_wq_b=wq_b, mla_wkv=wkv, mla_o=o, mla_wo_a=wo_a, mla_wo_b=wo_b,
             mla_q_down=qa, mla_q_up=qraw, mla_perhead_norm=M.perhead_norm(qraw), mla_kv_proj=M.kv_proj(x, wkv),
             mla_o_grouped=M.o_grouped(o, wo_a, wo_b),
             mla_shape=np.array([M.N_HEADS, M.HEAD_DIM, M.N_GROUPS, M.O_LORA], dtype=np.int64))
    from v4mlx import sparse_attn as SA
    n, sq, t = 200, 5, 48
    sq_q, sq_kv = rng.standard_normal((sq, 16, 512)).astype(np.float32), rng.standard_normal((n, 512)).astype(np.float32)
    sink = rng.standard_normal(16).astype(np.float32)
    idx = rng.integers(0, n, (sq, t))
    idx[0, 3:9] = -1
    idx[2, ::4] = -1
    g.update(mlxsa_q=sq_q, mlxsa_kv=sq_kv, mlxsa_sink=sink, mlxsa_idx=idx,
             mlxsa_out=SA.sparse_attn(sq_q, sq_kv, sink, idx, np.float32(512 ** -0.5)),
             mlxsa_win_20_8=SA.get_window_topk_idxs(8, 20), mlxsa_win_5_128=SA.get_window_topk_idxs(128, 5))
    from v4mlx import compressor as CMP
    dim_c = 48
    cx = rng.standard_normal((1, 18, dim_c)).astype(np.float32).view(_Array)  # 4 full blocks, remainder 2
    for hd, tag in ((512, "cmp"), (128, "icmp")):
        wkv = (rng.standard_normal((2 * hd, dim_c)) * 0.1).astype(np.float32)
        wgate = (rng.standard_normal((2 * hd, dim_c)) * 0.1).astype(np.float32)
        ape = (rng.standard_normal((4, 2 * hd)) * 0.1).astype(np.float32)
        nw = (rng.random(hd) + 0.5).astype(np.float32)
        g.update({f"mlx{tag}_x": cx, f"mlx{tag}_wkv": wkv, f"mlx{tag}_wgate": wgate, f"mlx{tag}_ape": ape,
                  f"mlx{tag}_nw": nw,
                  f"mlx{tag}_rows": CMP.compressor_prefill(cx, wkv, wgate, ape, nw, head_dim=hd, apply_sim=False)})
        if hd == 512:
            g["mlxcmp_rows_sim"] = CMP.compressor_prefill(cx, wkv, wgate, ape, nw, head_dim=hd, apply_sim=True)
        else:
            g["mlxicmp_rows_rotate"] = CMP.compressor_prefill(cx, wkv, wgate, ape, nw, head_dim=hd, rotate=True)
    from v4mlx import hc as HC
    hdim = 32
    hx = rng.standard_normal((1, 3, 4, hdim)).astype(np.float32).view(_Array)
    hfn = (rng.standard_normal((24, 4 * hdim)) * 0.05).astype(np.float32)
    hscale = (rng.random(3) + 0.5).astype(np.float32)
    hbase = (rng.standard_normal(24) * 0.1).astype(np.float32)
    y, post, comb = HC.hc_pre(hx, hfn, hscale, hbase)
    att = rng.standard_normal((1, 3, hdim)).astype(np.float32).view(_Array)
    head_fn = (rng.standard_normal((4, 4 * hdim)) * 0.05).astype(np.float32)
    g.update(mlxhc_x=hx, mlxhc_fn=hfn, mlxhc_scale=hscale, mlxhc_base=hbase, mlxhc_y=y, mlxhc_post=post,
             mlxhc_comb=comb, mlxhc_att=att, mlxhc_post_y=HC.hc_post(att, hx, post, comb), mlxhc_head_fn=head_fn,
             mlxhc_head_y=HC.hc_head(hx, head_fn, hscale[:1], hbase[:4]))
    from v4mlx import norm_rope as NRM
    cos, sin = NRM.rope_cos_sin(64, 16, 65536, 160000.0, 16, 32, 1)
    rx3 = rng.standard_normal((1, 16, 64)).astype(np.float32).view(_Array)
    rx4 = rng.standard_normal((1, 16, 4, 64)).astype(np.float32).view(_Array)
    nx = rng.standard_normal((3, 512)).astype(np.float32).view(_Array)
    nwt = (rng.standard_normal(512) * 0.1 + 1).astype(np.float32)
    g.update(mlxnr_freqs_yarn=NRM.precompute_freqs(64, 65536, 160000.0, 16, 32, 1),
             mlxnr_freqs_plain=NRM.precompute_freqs(64, 0, 10000.0, 40, 32, 1),
             mlxnr_x3=rx3, mlxnr_x4=rx4, mlxnr_x3_fwd=NRM.apply_rotary_emb(rx3, cos, sin),
             mlxnr_x3_inv=NRM.apply_rotary_emb(rx3, cos, sin, inverse=True),
             mlxnr_x4_fwd=NRM.apply_rotary_emb(rx4, cos, sin), mlxnr_nx=nx, mlxnr_nw=nwt,
             mlxnr_rms=NRM.rmsnorm(nx, nwt))
    np.savez_compressed(OUT, **{k: np.asarray(v) for k, v in g.items()})
    print("wrote", OUT, sorted(g))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_mla_golden.py <reference checkout>")
    main(sys.argv[1])
