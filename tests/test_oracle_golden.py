"""The CPU oracle against the reference's own ref_torch outputs (tests/golden/make_golden.py)."""
import numpy as np
import torch

from oracle import compressor_ref as C
from oracle import norm_rope_ref as NR
from oracle import sparse_attn_ref as SA


def test_window_indices_all_branches(golden):
    i = 0
    while f"win_{i}_args" in golden:
        w, b, s, sp = (int(v) for v in golden[f"win_{i}_args"])
        got = SA.get_window_topk_idxs(w, b, s, sp).numpy()
        np.testing.assert_array_equal(got, golden[f"win_{i}_out"], err_msg=f"case {(w, b, s, sp)}")
        i += 1
    assert i >= 9


def test_sparse_attn_matches_reference(golden):
    q, kv, sink, idx = (torch.from_numpy(golden[k]) for k in ("sa_q", "sa_kv", "sa_sink", "sa_idx"))
    out = SA.sparse_attn(q, kv, sink, idx, float(golden["sa_scale"])).numpy()
    ref = golden["sa_out"]
    assert np.isnan(ref[5]).all() and np.isnan(out[5]).all()  # all-masked query -> NaN in both
    np.testing.assert_allclose(out[:5], ref[:5], rtol=1e-4, atol=1e-5)


def test_norm_rope_matches_reference(golden):
    np.testing.assert_allclose(NR.rmsnorm(torch.from_numpy(golden["rms_x"]), torch.from_numpy(golden["rms_w"])).numpy(),
                               golden["rms_out"], rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(NR.precompute_freqs(64, 0, 65536, 160000.0, 16, 32, 1).numpy(), golden["freqs_yarn"])
    np.testing.assert_array_equal(NR.precompute_freqs(64, 0, 0, 10000.0, 40, 32, 1).numpy(), golden["freqs_plain"])
    cis = NR.precompute_freqs_cis(64, 16, 65536, 160000.0, 16, 32, 1)
    np.testing.assert_array_equal(torch.view_as_real(cis).numpy(), golden["cis_real"])
    x3, x4 = torch.from_numpy(golden["rope_x3"]), torch.from_numpy(golden["rope_x4"])
    np.testing.assert_allclose(NR.apply_rotary_emb(x3, cis).numpy(), golden["rope_x3_fwd"], atol=1e-6)
    np.testing.assert_allclose(NR.apply_rotary_emb(x3, cis, True).numpy(), golden["rope_x3_inv"], atol=1e-6)
    np.testing.assert_allclose(NR.apply_rotary_emb(x4, cis).numpy(), golden["rope_x4_fwd"], atol=1e-6)
    # the per-position form used by the pipelines equals the table form
    f = NR.precompute_freqs(64, 0, 65536, 160000.0, 16, 32, 1)
    np.testing.assert_allclose(NR.rope_at(x3[0], torch.arange(16), f).numpy(), golden["rope_x3_fwd"][0], atol=1e-6)


def test_compressor_matches_reference(golden):
    wkv, wgate, ape, nw = (torch.from_numpy(golden[k]) for k in ("cmp_wkv", "cmp_wgate", "cmp_ape", "cmp_nw"))
    for s in (18, 16):
        x = torch.from_numpy(golden[f"cmp{s}_x"])
        rows, st = C.compressor_prefill(x, wkv, wgate, ape, nw)
        np.testing.assert_allclose(rows.numpy(), golden[f"cmp{s}_rows"], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(st["kv"].numpy(), golden[f"cmp{s}_state_kv"], rtol=1e-6, atol=1e-6)
        np.testing.assert_allclose(st["score"].numpy(), golden[f"cmp{s}_state_score"], rtol=1e-6, atol=1e-6)
        if f"cmp{s}_state_kv_rem" in golden:
            np.testing.assert_allclose(st["kv_rem"].numpy(), golden[f"cmp{s}_state_kv_rem"], rtol=1e-6, atol=1e-6)


def test_decode_ring_continues_prefill(golden):
    """Stepping the decode ring over tokens 16..19 emits the row prefill would produce for them."""
    wkv, wgate, ape, nw = (torch.from_numpy(golden[k]) for k in ("cmp_wkv", "cmp_wgate", "cmp_ape", "cmp_nw"))
    x = torch.from_numpy(golden["cmp18_x"])[:1]
    torch.manual_seed(0)
    x20 = torch.cat([x, torch.randn(1, 2, x.shape[-1])], 1)   # 20 tokens
    full, _ = C.compressor_prefill(x20, wkv, wgate, ape, nw)  # 5 rows
    kvp, scp = x20.float() @ wkv.T, x20.float() @ wgate.T
    rk, rs = C.ring_from_prefill(kvp[:, :16], scp[:, :16], ape, 16)
    f = NR.precompute_freqs(64, 0, 65536, 160000.0, 16, 32, 1)
    row = None
    for p in range(16, 20):
        row = C.decode_ring_step(rk[0], rs[0], kvp[0, p], scp[0, p], ape, nw, p, f)
        assert (row is None) == (p != 19)
    np.testing.assert_allclose(row.numpy(), full[0, 4].numpy(), rtol=1e-4, atol=1e-5)


def _qat_golden():
    import os
    return np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "qat_golden.npz"))


def test_act_quant_matches_reference():
    """The fp8-e4m3 act-quant oracle against the reference's own `aq` (oracle/decode_engine.py:52-54)
    on rows spanning 1e-6..1e3, an all-zero block and a block of exact powers of two: bit for bit."""
    from oracle import quant_ref as Q
    g = _qat_golden()
    got = Q.act_quant_sim(g["aq_x"])
    np.testing.assert_array_equal(got.view(np.uint32), g["aq_y"].view(np.uint32))


def test_hc_matches_reference():
    """hc_pre / hc_post / hc_head oracle against the reference's ref_torch/hc.py outputs."""
    from oracle import hc_ref as H
    g = _qat_golden()
    y, post, comb = H.hc_pre(g["hc_x"], g["hc_fn"], g["hc_scale"], g["hc_base"])
    np.testing.assert_allclose(y, g["hc_y"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(post, g["hc_post"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(comb, g["hc_comb"], rtol=1e-5, atol=1e-6)
    # the Sinkhorn result is doubly stochastic to within its eps terms
    np.testing.assert_allclose(comb.sum(-2), 1.0, atol=1e-4)
    np.testing.assert_allclose(comb.sum(-1), 1.0, atol=1e-4)
    out = H.hc_post(g["hc_att"], g["hc_x"], g["hc_post"], g["hc_comb"])
    np.testing.assert_allclose(out, g["hc_post_y"], rtol=1e-5, atol=1e-5)
    yh = H.hc_head(g["hc_x"], g["hc_head_fn"], g["hc_head_scale"], g["hc_head_base"])
    np.testing.assert_allclose(yh, g["hc_head_y"], rtol=1e-5, atol=1e-6)


def test_hadamard_fp4_matches_reference():
    """The indexer-key simulation (v4mlx/qat.py:8-31) against the reference's own outputs, bit for
    bit: the float32 Hadamard rotation and the fp4-e2m1 block round trip."""
    from oracle import quant_ref as Q
    g = _qat_golden()
    had = Q.hadamard_rotate(g["fp4_x"])
    np.testing.assert_array_equal(had.view(np.uint32), g["had_y"].view(np.uint32))
    q = Q.fp4_act_quant(had)
    np.testing.assert_array_equal(q.view(np.uint32), g["fp4_y"].view(np.uint32))
    # every value is an e2m1 value times its block's power-of-two scale
    blk = q.reshape(-1, 32)
    e = Q.fp4_exp(np.abs(had.reshape(-1, 32)).max(-1, keepdims=True))
    grid = {0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0}
    assert set(np.abs(blk / np.exp2(e.astype(np.float64))).ravel().tolist()) <= grid


def test_e2m1_round_ties_and_edges():
    """e2m1 rounding on the tie points and the range ends (planted against a table of the format)."""
    from oracle import quant_ref as Q
    x = np.array([0.0, -0.0, 0.2, 0.25, 0.26, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 5.01, 6.0, -1.25, -5.0], np.float32)
    want = np.array([0.0, -0.0, 0.0, 0.0, 0.5, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0, 6.0, 6.0, -1.0, -4.0], np.float32)
    got = Q._e2m1_round(x)
    np.testing.assert_array_equal(got, want)
    assert np.signbit(got[1]) and np.signbit(Q._e2m1_round(np.float32(-0.2)))


def test_mla_projections_match_reference():
    """oracle/mla_ref.py and the per-head norm against the reference's own v4mlx/mla.py functions
    (run on numpy arrays with a stand-in for mlx.core, at reduced shapes; tests/golden/make_mla_golden.py)."""
    import os

    import torch

    from oracle import mla_ref as M
    from oracle.norm_rope_ref import perhead_norm
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "mla_golden.npz"))
    heads, head_dim, groups, _ = (int(v) for v in g["mla_shape"])
    t = {k: torch.from_numpy(g[k]) for k in g.files}
    tol = dict(rtol=1e-5, atol=1e-6)  # fp32 matmuls, summed in a different order than numpy's
    qa = M.linear(t["mla_x"], t["mla_wq_a"])
    np.testing.assert_allclose(qa.numpy(), g["mla_q_down"], **tol)
    q = M.q_up(t["mla_q_down"], t["mla_wq_b"], heads=heads, head_dim=head_dim)
    np.testing.assert_allclose(q.numpy(), g["mla_q_up"], **tol)
    np.testing.assert_allclose(perhead_norm(t["mla_q_up"]).numpy(), g["mla_perhead_norm"], **tol)
    np.testing.assert_allclose(M.linear(t["mla_x"], t["mla_wkv"]).numpy(), g["mla_kv_proj"], **tol)
    out = M.o_grouped(t["mla_o"], t["mla_wo_a"], t["mla_wo_b"], groups=groups)
    np.testing.assert_allclose(out.numpy(), g["mla_o_grouped"], **tol)


def test_sparse_attn_matches_reference_mlx_twin():
    """The oracle's sparse attention and prefill window list against the reference's MLX twin
    (v4mlx/sparse_attn.py, run on numpy with a stand-in for mlx.core; tests/golden/make_mla_golden.py):
    the two reference forms and the oracle agree."""
    import os

    import torch

    from oracle import sparse_attn_ref as SA
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "mla_golden.npz"))
    out = SA.sparse_attn(torch.from_numpy(g["mlxsa_q"]), torch.from_numpy(g["mlxsa_kv"]),
                         torch.from_numpy(g["mlxsa_sink"]), torch.from_numpy(g["mlxsa_idx"]), 512 ** -0.5)
    np.testing.assert_allclose(out.numpy(), g["mlxsa_out"], rtol=2e-5, atol=2e-6)
    for key, (w, s) in (("mlxsa_win_20_8", (8, 20)), ("mlxsa_win_5_128", (128, 5))):
        np.testing.assert_array_equal(SA.get_window_topk_idxs(w, 1, s, 0)[0].numpy(), g[key])


def test_compressor_matches_reference_mlx_twin():
    """The oracle's compressor against the reference's MLX twin (v4mlx/compressor.py, run on numpy
    with a stand-in for mlx.core; tests/golden/make_mla_golden.py): the rows before any simulation
    to fp32 accuracy, and the twin's fp8 (main compressor) and Hadamard + fp4 (indexer compressor,
    `rotate`) rows equal bit for bit to the oracle's simulations applied to the twin's own rows, which
    pins where the twin applies them (after the norm and RoPE; fp8 on the nope dims only)."""
    import os

    import torch

    from oracle import compressor_ref as CR
    from oracle import quant_ref as Q
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "mla_golden.npz"))
    for tag, hd in (("cmp", 512), ("icmp", 128)):
        t = {k: torch.from_numpy(g[f"mlx{tag}_{k}"]) for k in ("x", "wkv", "wgate", "ape", "nw")}
        rows, _ = CR.compressor_prefill(t["x"], t["wkv"], t["wgate"], t["ape"], t["nw"], head_dim=hd)
        np.testing.assert_allclose(rows.numpy(), g[f"mlx{tag}_rows"], rtol=1e-4, atol=2e-5)
    twin = torch.from_numpy(g["mlxcmp_rows"])
    sim = Q.act_quant_rows(twin, 64).numpy()
    np.testing.assert_array_equal(sim.view(np.uint32), g["mlxcmp_rows_sim"].view(np.uint32))
    rot = Q.rotate_quant_rows(torch.from_numpy(g["mlxicmp_rows"])).numpy()
    np.testing.assert_array_equal(rot.view(np.uint32), g["mlxicmp_rows_rotate"].astype(np.float32).view(np.uint32))


def test_hyper_connections_match_reference_mlx_twin():
    """The float64 hyper-connection oracle against the reference's MLX twin (v4mlx/hc.py, run in
    float32 on numpy with a stand-in for mlx.core; tests/golden/make_mla_golden.py)."""
    import os

    from oracle import hc_ref as H
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "mla_golden.npz"))
    tol = dict(rtol=2e-5, atol=2e-6)  # the twin runs in float32, the oracle in float64
    y, post, comb = H.hc_pre(g["mlxhc_x"], g["mlxhc_fn"], g["mlxhc_scale"], g["mlxhc_base"])
    np.testing.assert_allclose(y, g["mlxhc_y"], **tol)
    np.testing.assert_allclose(post, g["mlxhc_post"], **tol)
    np.testing.assert_allclose(comb, g["mlxhc_comb"], **tol)
    np.testing.assert_allclose(H.hc_post(g["mlxhc_att"], g["mlxhc_x"], g["mlxhc_post"], g["mlxhc_comb"]),
                               g["mlxhc_post_y"], **tol)
    yh = H.hc_head(g["mlxhc_x"], g["mlxhc_head_fn"], g["mlxhc_scale"][:1], g["mlxhc_base"][:4])
    np.testing.assert_allclose(yh, g["mlxhc_head_y"], **tol)


def test_norm_rope_match_reference_mlx_twin():
    """The oracle's YaRN tables, RoPE (forward and inverse, with and without a head axis) and RMSNorm
    against the reference's MLX twin (v4mlx/norm_rope.py on numpy with a stand-in for mlx.core,
    whose cos/sin tables are float32 where ref_torch builds complex64 ones)."""
    import os

    import torch

    from oracle import norm_rope_ref as NR
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "mla_golden.npz"))
    fy = NR.precompute_freqs(64, 0, 65536, 160000.0, 16, 32, 1)
    np.testing.assert_allclose(fy.numpy(), g["mlxnr_freqs_yarn"], rtol=1e-6)
    np.testing.assert_allclose(NR.precompute_freqs(64, 0, 0, 10000.0, 40, 32, 1).numpy(), g["mlxnr_freqs_plain"],
                               rtol=1e-6)
    pos = torch.arange(16)
    tol = dict(rtol=1e-5, atol=1e-5)
    x3, x4 = torch.from_numpy(g["mlxnr_x3"]), torch.from_numpy(g["mlxnr_x4"])
    np.testing.assert_allclose(NR.rope_at(x3[0], pos, fy).numpy(), g["mlxnr_x3_fwd"][0], **tol)
    np.testing.assert_allclose(NR.rope_at(x3[0], pos, fy, inverse=True).numpy(), g["mlxnr_x3_inv"][0], **tol)
    np.testing.assert_allclose(NR.rope_at(x4[0], pos, fy).numpy(), g["mlxnr_x4_fwd"][0], **tol)
    rms = NR.rmsnorm(torch.from_numpy(g["mlxnr_nx"]), torch.from_numpy(g["mlxnr_nw"]))
    np.testing.assert_allclose(rms.numpy(), g["mlxnr_rms"], rtol=1e-5, atol=1e-6)


def test_decode_ring_matches_reference_code():
    """The oracle's decode ring step against the reference's own inline ring code
    (oracle/decode_engine.py:96-105, run from the file's syntax tree; tests/golden/make_ring_golden.py):
    the ring after every step, the emitted rows before the fp8 simulation, and the simulation of the
    reference's own rows equal to its final rows bit for bit (emission at (p+1) % 4 == 0, RoPE at p-3,
    fp8 on the nope dims after the norm and RoPE)."""
    import os

    import torch

    from oracle import compressor_ref as CR
    from oracle import norm_rope_ref as NR
    from oracle import quant_ref as Q
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ring_golden.npz"))
    t = {k: torch.from_numpy(g[f"ring_{k}"]) for k in ("wkv", "wgate", "ape", "nw")}
    rk, rs = torch.from_numpy(g["ring_kv0"]).clone(), torch.from_numpy(g["ring_sc0"]).clone()
    f = NR.precompute_freqs(64, 0, 65536, 160000.0, 16, 32, 1)
    emitted = 0
    for i, p in enumerate(g["ring_pos"]):
        x = torch.from_numpy(g["ring_x"][i])
        row = CR.decode_ring_step(rk, rs, x @ t["wkv"].T, x @ t["wgate"].T, t["ape"], t["nw"], int(p), f)
        np.testing.assert_allclose(rk.numpy(), g["ring_kvs"][i], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(rs.numpy(), g["ring_scs"][i], rtol=1e-5, atol=1e-6)
        raw = g["ring_raw_rows"][i]
        if np.isnan(raw).all():
            assert row is None, p
            continue
        emitted += 1
        np.testing.assert_allclose(row.numpy(), raw, rtol=1e-4, atol=1e-5)
        sim = Q.act_quant_rows(torch.from_numpy(raw), 64).numpy()
        np.testing.assert_array_equal(sim.view(np.uint32), g["ring_q_rows"][i].view(np.uint32))
    assert emitted == 2


def test_decode_attention_matches_reference_code():
    """The oracle's decode attention (window rows in ring order + every visible compressed row) and
    its window-only attention against the reference's own inline decode attention
    (oracle/v4_fast.py:108-119 run from the file's syntax tree with the MLX twins on numpy;
    tests/golden/make_decode_attention_golden.py): a wrapped window with 75 visible rows, a partial
    window, and a layer without compression."""
    import os

    import torch

    from oracle import layer_ref as LR
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "decode_attention_golden.npz"))
    f = LR.layer_freqs(4)
    for tag in ("r4", "r4p", "w"):
        winr, comp = torch.from_numpy(g[f"da_{tag}_winr"]), torch.from_numpy(g[f"da_{tag}_comp"])
        q = torch.from_numpy(g[f"da_{tag}_qraw"])[None]
        sink, pos = torch.from_numpy(g[f"da_{tag}_sinks"]), torch.tensor([int(g[f"da_{tag}_p"])])
        pool, win_base = torch.cat([winr, comp]), torch.zeros(1, dtype=torch.int64)
        if bool(g[f"da_{tag}_r4"]):
            rng = np.random.default_rng(0)   # the indexer inputs do not matter: top_k covers every visible row
            k_idx = torch.from_numpy(rng.standard_normal((1, comp.shape[0], 128)).astype(np.float32))
            q_idx = torch.from_numpy(rng.standard_normal((1, 64, 128)).astype(np.float32))
            w_idx = torch.from_numpy(rng.standard_normal((1, 64)).astype(np.float32))
            o = LR.decode_attention_ref(pool, win_base, lambda b, j: 128 + j, k_idx, q, q_idx, w_idx, sink, pos, 512, f)
        else:
            o = LR.window_attention_ref(pool, win_base, q, sink, pos, f)
        np.testing.assert_allclose(o[0].numpy(), g[f"da_{tag}_o"], rtol=1e-4, atol=2e-5, err_msg=tag)
