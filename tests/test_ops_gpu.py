"""Each dsv4 op on the GPU against the CPU oracle (same seeded inputs)."""
import ctypes
import importlib

import numpy as np
import pytest
import torch

from helpers import assert_close_bf16, rel_rms
from oracle import compressor_ref as C
from oracle import indexer_ref as I
from oracle import mla_ref as M
from oracle import norm_rope_ref as NR
from oracle import sparse_attn_ref as SA

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _bf16(x):
    return x.to(torch.bfloat16).float()


# ---------------------------------------------------------------- sparse attention
def test_sparse_attn_golden_inputs(dsv4, golden):
    q, kv, sink, idx = (torch.from_numpy(golden[k]) for k in ("sa_q", "sa_kv", "sa_sink", "sa_idx"))
    kvb = _bf16(kv)
    ref = SA.sparse_attn(q, kvb, sink, idx, float(golden["sa_scale"]))
    out = dsv4.sparse_attn(q.to(DEV), kvb.to(DEV), sink.to(DEV), idx.to(DEV), float(golden["sa_scale"]))
    assert out.dtype == torch.float32
    assert torch.isnan(out[5]).all()                     # all-masked query -> NaN like the reference
    assert_close_bf16(out, ref, what="golden")


@pytest.mark.parametrize("s,t,n,h,idx_dtype,splits", [
    (1, 640, 8320, 64, torch.int32, 0),      # C2-like decode (split-K + combine)
    (3, 640, 2176, 64, torch.int64, 0),
    (1, 100, 500, 64, torch.int32, 1),        # t not a multiple of 64, single split
    (1, 1152, 4000, 64, torch.int32, 5),      # explicit splits
    (40, 256, 700, 64, torch.int32, 0),       # prefill-like, one CTA per query
    (2, 200, 300, 128, torch.int32, 0),       # two head blocks
    (2, 64, 300, 32, torch.int32, 0),         # fewer heads than a block
])
def test_sparse_attn_shapes(dsv4, s, t, n, h, idx_dtype, splits):
    g = torch.Generator().manual_seed(s * 1000 + t)
    q = torch.randn(s, h, 512, generator=g)
    kv = _bf16(torch.randn(n, 512, generator=g))
    sink = torch.randn(h, generator=g)
    idx = torch.randint(0, n, (s, t), generator=g)
    idx[:, ::7] = -1
    ref = SA.sparse_attn(q, kv, sink, idx, 512 ** -0.5)
    L = __import__("importlib").import_module("deepseek-v4-flash-mlx_b200.sparse_attn")
    out = L._sparse_attn_op(q.to(DEV), kv.to(DEV).bfloat16(), sink.to(DEV), idx.to(DEV, idx_dtype), 512 ** -0.5,
                            torch.float32, None, None, 0, splits)
    assert_close_bf16(out, ref, what=f"s={s} t={t}")


def test_sparse_attn_known_answers(dsv4):
    """One-hot rows, sink-only mass, duplicate indices."""
    h, n = 64, 128
    kv = torch.zeros(n, 512)
    kv[torch.arange(n), torch.arange(n)] = 1.0
    q = torch.zeros(1, h, 512)
    sink = torch.full((h,), -1e4)
    idx = torch.tensor([[5, 9, -1, 9]])
    out = dsv4.sparse_attn(q.to(DEV), kv.to(DEV), sink.to(DEV), idx.to(DEV), 1.0).cpu()
    # equal logits (0): weights 1/3 each over rows 5, 9, 9
    assert torch.allclose(out[0, :, 5], torch.full((h,), 1 / 3), atol=1e-3)
    assert torch.allclose(out[0, :, 9], torch.full((h,), 2 / 3), atol=1e-3)
    sink2 = torch.full((h,), 30.0)                         # sink dominates the denominator
    out2 = dsv4.sparse_attn(q.to(DEV), kv.to(DEV), sink2.to(DEV), idx.to(DEV), 1.0).cpu()
    assert out2.abs().max() < 1e-9


def test_sparse_attn_inverse_rope_fused(dsv4):
    g = torch.Generator().manual_seed(5)
    s, t, n = 4, 300, 1000
    q = torch.randn(s, 64, 512, generator=g)
    kv = _bf16(torch.randn(n, 512, generator=g))
    sink = torch.randn(64, generator=g)
    idx = torch.randint(0, n, (s, t), generator=g)
    pos = torch.tensor([0, 7, 4095, 32767], dtype=torch.int32)
    f = NR.precompute_freqs(64, 0, 65536, 160000.0, 16, 32, 1)
    ref = NR.rope_at(SA.sparse_attn(q, kv, sink, idx, 512 ** -0.5), pos, f, 64, inverse=True)
    for splits in (0, 1):
        L = __import__("importlib").import_module("deepseek-v4-flash-mlx_b200.sparse_attn")
        out = L._sparse_attn_op(q.to(DEV), kv.to(DEV).bfloat16(), sink.to(DEV), idx.to(DEV), 512 ** -0.5,
                                torch.float32, f.to(DEV), pos.to(DEV), 64, splits)
        assert_close_bf16(out, ref, what=f"rope splits={splits}")


def test_sparse_attn_out_of_range_index_flags_device_error(dsv4):
    L = __import__("importlib").import_module("deepseek-v4-flash-mlx_b200._lib")
    L.device_error()  # clear
    q = torch.randn(1, 64, 512, device=DEV)
    kv = torch.randn(10, 512, device=DEV).bfloat16()
    idx = torch.tensor([[1, 2, 10_000]], device=DEV)       # 10000 >= n: treated as masked and flagged
    out = dsv4.sparse_attn(q, kv, torch.zeros(64, device=DEV), idx, 0.05)
    assert torch.isfinite(out).all()
    assert L.device_error() == 4
    assert L.device_error() == 0


def test_window_indices_gpu(dsv4, golden):
    i = 0
    while f"win_{i}_args" in golden:
        w, b, s, sp = (int(v) for v in golden[f"win_{i}_args"])
        got = dsv4.get_window_topk_idxs(w, b, s, sp).cpu().numpy()
        ref = golden[f"win_{i}_out"]
        ref = np.broadcast_to(ref, got.shape) if ref.shape[1] == 1 else ref
        np.testing.assert_array_equal(got, ref, err_msg=str((w, b, s, sp)))
        i += 1


# ---------------------------------------------------------------- norm / rope
def test_rmsnorm_and_perhead(dsv4):
    g = torch.Generator().manual_seed(1)
    x = torch.randn(37, 1024, generator=g) * 3
    w = torch.randn(1024, generator=g)
    assert rel_rms(dsv4.rmsnorm(x.to(DEV), w.to(DEV)), NR.rmsnorm(x, w)) < 1e-6
    xb = x.bfloat16()
    out = dsv4.rmsnorm(xb.to(DEV), w.to(DEV))
    assert out.dtype == torch.bfloat16
    assert rel_rms(out, NR.rmsnorm(xb, w)) < 8e-3
    q = torch.randn(5, 64, 512, generator=g)
    assert rel_rms(dsv4.perhead_norm(q.to(DEV)), NR.perhead_norm(q)) < 1e-6


@pytest.mark.parametrize("rows,dim,out_dtype", [(32, 4096, torch.bfloat16), (32, 1024, torch.float32),
                                                 (3, 4100, torch.float32), (7, 130, torch.bfloat16),
                                                 (1000, 512, torch.float32), (1, 8192, torch.bfloat16)])
def test_rmsnorm_row_shapes(dsv4, rows, dim, out_dtype):
    """Decode-sized batches (one CTA per row, the row in registers) and the one-warp-per-row form
    (many rows, or a dim that is not a multiple of 4), fp32 input with a bf16 or fp32 result."""
    g = torch.Generator().manual_seed(rows + dim)
    x = torch.randn(rows, dim, generator=g) * 2
    w = torch.randn(dim, generator=g)
    out = dsv4.rmsnorm(x.to(DEV), w.to(DEV), out_dtype=out_dtype)
    assert out.dtype == out_dtype
    ref = NR.rmsnorm(x, w)
    assert rel_rms(out.float(), ref) < (4e-3 if out_dtype == torch.bfloat16 else 1e-6)
    if out_dtype == torch.bfloat16:   # one rounding of the fp32 result
        assert torch.equal(out.cpu(), dsv4.rmsnorm(x.to(DEV), w.to(DEV)).cpu().bfloat16())


def test_apply_rotary_emb_table_form(dsv4, golden):
    cis = NR.precompute_freqs_cis(64, 16, 65536, 160000.0, 16, 32, 1)
    x3, x4 = torch.from_numpy(golden["rope_x3"]), torch.from_numpy(golden["rope_x4"])
    np.testing.assert_allclose(dsv4.apply_rotary_emb(x3.to(DEV), cis).cpu().numpy(), golden["rope_x3_fwd"], atol=2e-6)
    np.testing.assert_allclose(dsv4.apply_rotary_emb(x3.to(DEV), cis, inverse=True).cpu().numpy(),
                               golden["rope_x3_inv"], atol=2e-6)
    np.testing.assert_allclose(dsv4.apply_rotary_emb(x4.to(DEV), cis).cpu().numpy(), golden["rope_x4_fwd"], atol=2e-6)
    xb = torch.randn(3, 16, 64)
    ref = NR.apply_rotary_emb(xb, cis)
    assert rel_rms(dsv4.apply_rotary_emb(xb.to(DEV), cis), ref) < 1e-6


def test_norm_rope_fused(dsv4):
    g = torch.Generator().manual_seed(2)
    f = NR.precompute_freqs(64, 0, 65536, 160000.0, 16, 32, 1)
    pos = torch.tensor([0, 1, 5000, 32767, 65535], dtype=torch.int32)
    q = torch.randn(5, 64, 512, generator=g) * 0.7
    ref = NR.rope_at(NR.perhead_norm(q), pos, f)
    out = dsv4.norm_rope(q.to(DEV), pos.to(DEV), f.to(DEV), weight=None, out_dtype=torch.float32)
    assert rel_rms(out, ref) < 2e-6
    kv = torch.randn(5, 512, generator=g)
    w = torch.rand(512, generator=g) + 0.5
    ref2 = NR.rope_at(NR.rmsnorm(kv, w), pos, f)
    out2 = dsv4.norm_rope(kv.to(DEV), pos.to(DEV), f.to(DEV), weight=w.to(DEV))
    assert out2.dtype == torch.bfloat16
    assert_close_bf16(out2, ref2, what="kv norm_rope")


# ---------------------------------------------------------------- indexer
def _idx_inputs(b, s, n, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, s, 64, 128, generator=g)
    w = torch.randn(b, s, 64, generator=g) / 8
    k = torch.randn(b, n, 128, generator=g)
    return q, w, k


def test_indexer_scores_bit_exact(dsv4):
    q, w, k = _idx_inputs(1, 3, 1000, 7)
    got = dsv4.indexer_scores(q.to(DEV), w.to(DEV), k.to(DEV)).cpu().numpy()
    for i in range(3):
        ref = I.scores(q[0, i].numpy(), w[0, i].numpy(), k[0].numpy())
        np.testing.assert_array_equal(got[0, i].view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("b,s,n,k,causal", [(1, 1, 8192, 512, False), (4, 1, 2048, 512, False),
                                            (1, 40, 700, 64, True), (2, 3, 300, 512, False),
                                            (1, 200, 300, 32, True), (2, 130, 1000, 64, False),
                                            (1, 64, 20000, 1024, False)])
def test_indexer_topk_bit_exact(dsv4, b, s, n, k, causal):
    q, w, keys = _idx_inputs(b, s, n, b * 100 + s)
    pos = None
    if causal:
        pos = torch.arange(n * 4 - s * 37, n * 4, 37)[:s].repeat(b, 1).to(torch.int32)
    got = dsv4.indexer_topk(q.to(DEV), w.to(DEV), keys.to(DEV), k, None if pos is None else pos.to(DEV)).cpu().numpy()
    ref = I.indexer_topk(q.numpy(), w.numpy(), keys.numpy(), k, None if pos is None else pos.numpy())
    np.testing.assert_array_equal(got, ref)


def test_indexer_scores_tiled_prefill_bit_exact(dsv4):
    """The query-tiled (prefill) score kernel: causal visibility, partial query and key tiles."""
    q, w, k = _idx_inputs(1, 150, 333, 17)
    pos = torch.arange(1000, 1150, dtype=torch.int32)[None]       # visible counts 250..287
    got = dsv4.indexer_scores(q.to(DEV), w.to(DEV), k.to(DEV), pos.to(DEV)).cpu().numpy()
    for i in range(150):
        nv = min((1000 + i + 1) // 4, 333)
        ref = I.scores(q[0, i].numpy(), w[0, i].numpy(), k[0, :nv].numpy())
        np.testing.assert_array_equal(got[0, i, :nv].view(np.uint32), ref.view(np.uint32), err_msg=f"query {i}")


def test_indexer_ties_and_padding(dsv4):
    """Duplicate keys give exactly equal scores: the lower index must win the boundary."""
    q, w, keys = _idx_inputs(1, 1, 300, 9)
    keys[0, 200:] = keys[0, 100:200]                      # rows 200..299 duplicate rows 100..199
    got = dsv4.indexer_topk(q.to(DEV), w.to(DEV), keys.to(DEV), 77).cpu().numpy()
    ref = I.indexer_topk(q.numpy(), w.numpy(), keys.numpy(), 77)
    np.testing.assert_array_equal(got, ref)
    pos = torch.tensor([[39]], dtype=torch.int32)           # 10 visible keys, k = 16
    got2 = dsv4.indexer_topk(q.to(DEV), w.to(DEV), keys.to(DEV), 16, pos.to(DEV)).cpu().numpy()
    np.testing.assert_array_equal(got2[0, 0], list(range(10)) + [-1] * 6)


def test_indexer_heavy_ties_fallback(dsv4):
    """All scores equal (zero weights): more than 1024 keys share the boundary bin, so the radix
    fallback runs; the answer is the lowest indices. Also a crowded bin with distinct scores."""
    q, w, keys = _idx_inputs(1, 2, 5000, 13)
    w[0, 0] = 0.0                                           # query 0: every score is +0
    got = dsv4.indexer_topk(q.to(DEV), w.to(DEV), keys.to(DEV), 512).cpu().numpy()
    np.testing.assert_array_equal(got[0, 0], np.arange(512))
    ref = I.indexer_topk(q.numpy(), w.numpy(), keys.numpy(), 512)
    np.testing.assert_array_equal(got, ref)
    # scores crowded into one 12-bit bin: keys nearly identical
    keys2 = keys.clone()
    keys2[0] = keys[0, :1] + 1e-4 * torch.randn(5000, 128, generator=torch.Generator().manual_seed(1))
    got2 = dsv4.indexer_topk(q.to(DEV), w.to(DEV), keys2.to(DEV), 512).cpu().numpy()
    ref2 = I.indexer_topk(q.numpy(), w.numpy(), keys2.numpy(), 512)
    np.testing.assert_array_equal(got2, ref2)
    # 450 near-identical keys: one 12-bit bin of 450 (at most the CTA's 512 threads), ranked directly
    keys3 = keys[:, :450].clone()
    keys3[0] = keys[0, :1] + 1e-4 * torch.randn(450, 128, generator=torch.Generator().manual_seed(2))
    keys3[0, 300:310] = keys3[0, 100:110]                   # exact ties inside the ranked bin
    got3 = dsv4.indexer_topk(q.to(DEV), w.to(DEV), keys3.to(DEV), 200).cpu().numpy()
    ref3 = I.indexer_topk(q.numpy(), w.numpy(), keys3.numpy(), 200)
    np.testing.assert_array_equal(got3, ref3)


# ---------------------------------------------------------------- projections
def test_linear_bf16_and_grouped(dsv4):
    g = torch.Generator().manual_seed(3)
    x = _bf16(torch.randn(70, 256, generator=g))
    W = _bf16(torch.randn(192, 256, generator=g) * 0.05)
    ref = M.linear(x, W)
    out = dsv4.linear(x.to(DEV).bfloat16(), W.to(DEV).bfloat16())
    assert rel_rms(out, ref) < 1e-5
    o = _bf16(torch.randn(3, 8 * 128, generator=g))
    wa = _bf16(torch.randn(8 * 64, 128, generator=g) * 0.1)
    wb = _bf16(torch.randn(96, 8 * 64, generator=g) * 0.1)
    ref2 = M.o_grouped(o, wa, wb, groups=8)
    out2 = dsv4.o_grouped(o.to(DEV), wa.to(DEV).bfloat16(), wb.to(DEV).bfloat16())
    assert rel_rms(out2, ref2) < 5e-3


def test_linear_int8_g64(dsv4):
    g = torch.Generator().manual_seed(4)
    x = _bf16(torch.randn(32, 512, generator=g))
    qw = dsv4.quantize_int8_g64(torch.randn(384, 512, generator=g) * 0.02)
    ref = M.linear(x, M.dequant_int8_g64(qw.q, qw.scale))
    qd = type(qw)(qw.q.to(DEV), qw.scale.to(DEV))
    out = dsv4.linear(x.to(DEV).bfloat16(), qd)
    assert rel_rms(out, ref) < 1e-5


@pytest.mark.parametrize("m,n,k,groups,quant,split", [
    (32, 1024, 4096, 1, True, True),      # wq_a at batch 32: 8 output tiles, k split
    (5, 512, 4096, 1, False, True),       # ragged m, bf16 weights
    (32, 256, 1600, 4, True, True),       # grouped, k tiles not a multiple of the split
    (1, 64, 4096, 1, True, True),         # one output tile (the indexer head weights)
    (40, 19200, 128, 1, True, False),     # 64-token tiles, enough output tiles: no split
    (12, 19200, 256, 1, False, False),    # 16-token tiles, bf16
    (100, 256, 4096, 1, True, True),      # the tiled kernel (m > 64, int8) with k split
])
def test_linear_split_k_decode_shapes(dsv4, m, n, k, groups, quant, split):
    """Decode-shaped projections (the weight-streaming kernel for m <= 64), with k split across
    CTAs and a fixed-order fp32 sum of the partials where the output tiles alone leave SMs idle
    (`split`): close to the fp64 product and bit-identical from call to call."""
    L = importlib.import_module("deepseek-v4-flash-mlx_b200._lib")
    p = L.LinearParams()
    p.m, p.n, p.k, p.groups, p.w_dtype = m, n, k, groups, L.I8 if quant else L.BF16
    # m <= 64 sums its k split inside a thread-block cluster (no workspace); the tiled kernel
    # writes fp32 partials to the workspace
    assert (L.lib().dsv4_linear_workspace_size(ctypes.byref(p)) > 0) == (split and m > 64)
    g = torch.Generator().manual_seed(m + n + k)
    x = _bf16(torch.randn(m, groups * k, generator=g))
    w = torch.randn(groups * n, k, generator=g) * 0.02
    if quant:
        qw = dsv4.quantize_int8_g64(w)
        wd = M.dequant_int8_g64(qw.q, qw.scale)
        wdev = type(qw)(qw.q.to(DEV), qw.scale.to(DEV))
    else:
        wd = _bf16(w)
        wdev = wd.to(DEV).bfloat16()
    ref = torch.einsum("mgk,gnk->mgn", x.double().view(m, groups, k), wd.double().view(groups, n, k)).reshape(m, -1)
    out = dsv4.linear(x.to(DEV).bfloat16(), wdev, groups=groups)
    assert rel_rms(out, ref.float()) < 1e-5
    again = dsv4.linear(x.to(DEV).bfloat16(), wdev, groups=groups)
    assert torch.equal(out, again)
    outb = dsv4.linear(x.to(DEV).bfloat16(), wdev, torch.bfloat16, groups=groups)
    assert rel_rms(outb.float(), ref.float()) < 4e-3


@pytest.mark.parametrize("m,quant", [(32, True), (7, False), (64, True), (100, True)])
def test_linear_multi_matches_separate_projections(dsv4, m, quant):
    """Several projections of one x in one launch (ragged n, a tile shared by none): each output
    close to the fp64 product and to its own dsv4.linear; m > 64 runs one tiled call per output."""
    g = torch.Generator().manual_seed(m)
    k = 1024
    ns = [1024, 512, 64, 256, 130]
    x = _bf16(torch.randn(m, k, generator=g))
    Ws, ref = [], []
    for n in ns:
        w = torch.randn(n, k, generator=g) * 0.02
        if quant:
            qw = dsv4.quantize_int8_g64(w)
            ref.append(x.double() @ M.dequant_int8_g64(qw.q, qw.scale).double().T)
            Ws.append(type(qw)(qw.q.to(DEV), qw.scale.to(DEV)))
        else:
            ref.append(x.double() @ _bf16(w).double().T)
            Ws.append(w.to(DEV).bfloat16())
    outs = dsv4.linear_multi(x.to(DEV).bfloat16(), Ws)
    for o, r, W in zip(outs, ref, Ws):
        assert o.shape == r.shape
        assert rel_rms(o, r.float()) < 1e-5
        assert rel_rms(o, dsv4.linear(x.to(DEV).bfloat16(), W)) < 1e-6


# ---------------------------------------------------------------- compressor
def test_compressor_prefill_golden_inputs(dsv4, golden):
    wkv, wgate, ape, nw = (torch.from_numpy(golden[k]) for k in ("cmp_wkv", "cmp_wgate", "cmp_ape", "cmp_nw"))
    for s in (18, 16):
        x = torch.from_numpy(golden[f"cmp{s}_x"])
        # the GPU consumes bf16 operands: compare with the oracle on the same rounded operands
        ref, st = C.compressor_prefill(_bf16(x), _bf16(wkv), _bf16(wgate), ape, nw)
        out, gst = dsv4.compressor_prefill(x.to(DEV), wkv.to(DEV).bfloat16(), wgate.to(DEV).bfloat16(),
                                           ape.to(DEV), nw.to(DEV))
        assert_close_bf16(out, ref, 2e-3, 1e-4, what=f"cmp{s}")
        assert_close_bf16(gst["kv"], st["kv"], 1e-4, 1e-5, what="state kv")
        assert_close_bf16(gst["score"], st["score"], 1e-4, 1e-5, what="state score")
        # and against the reference itself (fp32 operands): bf16 operand rounding only
        assert_close_bf16(out, torch.from_numpy(golden[f"cmp{s}_rows"]), what=f"cmp{s} vs ref")


@pytest.mark.parametrize("hd,b", [(128, 3), (512, 5), (1024, 2)])
def test_compressor_decode_state_and_rows(dsv4, hd, b):
    """Eight decode steps of b sequences at staggered positions from a random ring: every emitted
    row and the whole ring state after each step against the oracle's ring step."""
    g = torch.Generator().manual_seed(hd + b)
    d2 = 2 * hd
    rk = torch.randn(b, 8, d2, generator=g)
    rs = torch.randn(b, 8, d2, generator=g)
    ape = torch.randn(4, d2, generator=g) * 0.1
    nw = torch.rand(hd, generator=g) + 0.5
    f = NR.precompute_freqs(64, 0, 65536, 160000.0, 16, 32, 1)
    grk, grs = rk.clone().to(DEV), rs.clone().to(DEV)
    pos0 = torch.tensor([100 + 3 * i for i in range(b)], dtype=torch.int32)
    pool = torch.zeros(b * 8, hd, device=DEV)
    for step in range(8):
        pos = pos0 + step
        kv = torch.randn(b, d2, generator=g)
        sc = torch.randn(b, d2, generator=g)
        rows = torch.arange(b) * 8 + step
        dsv4.compressor_decode_step(kv.to(DEV), None, None, ape.to(DEV), nw.to(DEV), grk, grs,
                                    pos.to(DEV), pool, rows.to(DEV), head_dim=hd, freqs=f.to(DEV),
                                    proj=(kv.to(DEV), sc.to(DEV)))
        for i in range(b):
            ref = C.decode_ring_step(rk[i], rs[i], kv[i], sc[i], ape, nw, int(pos[i]), f)
            if ref is not None:
                assert_close_bf16(pool[rows[i]], ref, 2e-3, 1e-4, what=f"hd={hd} seq {i} step {step}")
        torch.testing.assert_close(grk.cpu(), rk, rtol=0, atol=0)
        torch.testing.assert_close(grs.cpu(), rs, rtol=1e-6, atol=1e-6)


def test_norm_rope_act_quant(dsv4):
    """The kv row's fp8 act-quant simulation fused into the norm + rope kernel: the quantised output
    is the oracle's act-quant of the unquantised output (bit for bit, fp32 and bf16 outputs)."""
    from oracle import quant_ref as Q
    g = torch.Generator().manual_seed(31)
    f = NR.precompute_freqs(64, 0, 65536, 160000.0, 16, 32, 1).to(DEV)
    kv = (torch.randn(9, 512, generator=g) * torch.exp2(torch.randint(-12, 8, (9, 1), generator=g).float())).to(DEV)
    w = (torch.rand(512, generator=g) + 0.5).to(DEV)
    pos = torch.tensor([0, 1, 7, 100, 4095, 32767, 5, 6, 65535], dtype=torch.int32, device=DEV)
    plain = dsv4.norm_rope(kv, pos, f, weight=w, out_dtype=torch.float32)
    quant = dsv4.norm_rope(kv, pos, f, weight=w, out_dtype=torch.float32, act_quant=True)
    ref = Q.act_quant_rows(plain.cpu())
    np.testing.assert_array_equal(quant.cpu().numpy().view(np.uint32), ref.numpy().view(np.uint32))
    qb = dsv4.norm_rope(kv, pos, f, weight=w, out_dtype=torch.bfloat16, act_quant=True).float().cpu()
    assert torch.equal(qb[:, :448], ref[:, :448])      # fp8 values times powers of two are exact in bf16
    assert torch.equal(qb[:, 448:], ref[:, 448:].bfloat16().float())   # the rope dims: one bf16 rounding


def test_compressor_act_quant(dsv4):
    """Prefill rows and decode-emitted rows with the fp8 act-quant simulation of their nope dims:
    the oracle's act-quant of the same kernels' unquantised rows."""
    from oracle import quant_ref as Q
    g = torch.Generator().manual_seed(32)
    x = torch.randn(2, 24, 256, generator=g)
    wkv = torch.randn(1024, 256, generator=g) * 0.05
    wgate = torch.randn(1024, 256, generator=g) * 0.05
    ape = torch.randn(4, 1024, generator=g) * 0.1
    nw = torch.rand(512, generator=g) + 0.5
    args = (x.to(DEV), wkv.to(DEV).bfloat16(), wgate.to(DEV).bfloat16(), ape.to(DEV), nw.to(DEV))
    plain, st0 = dsv4.compressor_prefill(*args)
    quant, st1 = dsv4.compressor_prefill(*args, act_quant=True)
    np.testing.assert_array_equal(quant.cpu().numpy().view(np.uint32), Q.act_quant_rows(plain.cpu()).numpy().view(np.uint32))
    # decode: identical rings, one emission each
    f = NR.precompute_freqs(64, 0, 65536, 160000.0, 16, 32, 1).to(DEV)
    kvp, scp = torch.randn(2, 1024, generator=g).to(DEV), torch.randn(2, 1024, generator=g).to(DEV)
    outs = []
    for aq in (False, True):
        rk, rs = st0["ring_kv"].clone(), st0["ring_score"].clone()
        pool = torch.zeros(2, 512, device=DEV)
        dsv4.compressor_decode_step(kvp, None, None, ape.to(DEV), nw.to(DEV), rk, rs,
                                    torch.tensor([27, 27], dtype=torch.int32, device=DEV), pool,
                                    torch.tensor([0, 1], device=DEV), freqs=f, proj=(kvp, scp), act_quant=aq)
        outs.append(pool.cpu())
    np.testing.assert_array_equal(outs[1].numpy().view(np.uint32), Q.act_quant_rows(outs[0]).numpy().view(np.uint32))


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_compressor_rotate(dsv4, out_dtype):
    """The indexer compressor's Hadamard + fp4-e2m1 key simulation (v4mlx/compressor.py:57-59):
    prefill rows and decode-emitted rows equal the oracle's rotation and round trip of the same
    kernels' plain rows, bit for bit (bf16 output: after one more rounding of both)."""
    from oracle import quant_ref as Q
    g = torch.Generator().manual_seed(33)
    x = torch.randn(2, 40, 256, generator=g)
    wkv = torch.randn(256, 256, generator=g) * 0.05
    wgate = torch.randn(256, 256, generator=g) * 0.05
    ape = torch.randn(4, 256, generator=g) * 0.1
    nw = torch.rand(128, generator=g) + 0.5
    args = (x.to(DEV), wkv.to(DEV).bfloat16(), wgate.to(DEV).bfloat16(), ape.to(DEV), nw.to(DEV))
    plain, st0 = dsv4.compressor_prefill(*args, head_dim=128)
    rot, _ = dsv4.compressor_prefill(*args, head_dim=128, rotate=True, out_dtype=out_dtype)
    want = Q.rotate_quant_rows(plain.cpu())
    if out_dtype == torch.float32:
        np.testing.assert_array_equal(rot.cpu().numpy().view(np.uint32), want.numpy().view(np.uint32))
    else:
        assert torch.equal(rot.cpu(), want.to(torch.bfloat16))
    # the rows hold fp4 values times a power of two per 32-dim block
    blk = want.reshape(-1, 32).double()
    scale = 2.0 ** torch.from_numpy(Q.fp4_exp(Q.hadamard_rotate(plain.cpu().numpy()).reshape(-1, 32).__abs__().max(-1, keepdims=True))).double()
    assert set((blk / scale).abs().unique().tolist()) <= {0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0}
    # decode: identical rings, one emission each (ratio-4 kernel, key image kept in step)
    f = NR.precompute_freqs(64, 0, 65536, 160000.0, 16, 32, 1).to(DEV)
    kvp, scp = torch.randn(2, 256, generator=g).to(DEV), torch.randn(2, 256, generator=g).to(DEV)
    outs = []
    for rotate in (False, True):
        rk, rs = st0["ring_kv"].clone(), st0["ring_score"].clone()
        pool = torch.zeros(2, 128, device=DEV)
        dsv4.compressor_decode_step(kvp, None, None, ape.to(DEV), nw.to(DEV), rk, rs,
                                    torch.tensor([43, 43], dtype=torch.int32, device=DEV), pool,
                                    torch.tensor([0, 1], device=DEV), head_dim=128, freqs=f, proj=(kvp, scp),
                                    rotate=rotate)
        outs.append(pool.cpu())
    np.testing.assert_array_equal(outs[1].numpy().view(np.uint32), Q.rotate_quant_rows(outs[0]).numpy().view(np.uint32))
    with pytest.raises(RuntimeError):
        dsv4.compressor_prefill(*args[:3], torch.randn(4, 1024, device=DEV), torch.rand(512, device=DEV) + 0.5,
                                rotate=True)


def test_compressor_decode_ring(dsv4):
    g = torch.Generator().manual_seed(8)
    dim, s0 = 128, 13
    wkv = _bf16(torch.randn(1024, dim, generator=g) * 0.05)
    wgate = _bf16(torch.randn(1024, dim, generator=g) * 0.05)
    ape = torch.randn(4, 1024, generator=g) * 0.1
    nw = torch.rand(512, generator=g) + 0.5
    x = _bf16(torch.randn(1, s0 + 7, dim, generator=g))
    f = NR.precompute_freqs(64, 0, 65536, 160000.0, 16, 32, 1)
    kvp, scp = x @ wkv.T, x @ wgate.T
    rk, rs = C.ring_from_prefill(kvp[:, :s0], scp[:, :s0], ape, s0)
    _, st = dsv4.compressor_prefill(x[:, :s0].to(DEV), wkv.to(DEV).bfloat16(), wgate.to(DEV).bfloat16(), ape.to(DEV),
                                    nw.to(DEV))
    assert_close_bf16(st["ring_kv"], rk, 1e-4, 1e-5, what="ring kv")
    pool = torch.zeros(8, 512, device=DEV)
    for p in range(s0, s0 + 7):
        row = C.decode_ring_step(rk[0], rs[0], kvp[0, p], scp[0, p], ape, nw, p, f)
        dsv4.compressor_decode_step(x[:, p].to(DEV), wkv.to(DEV).bfloat16(), wgate.to(DEV).bfloat16(), ape.to(DEV),
                                    nw.to(DEV), st["ring_kv"], st["ring_score"],
                                    torch.tensor([p], dtype=torch.int32, device=DEV), pool,
                                    torch.tensor([p // 4], device=DEV), freqs=f.to(DEV))
        if row is not None:
            assert_close_bf16(pool[p // 4], row, 2e-3, 1e-4, what=f"emit p={p}")
