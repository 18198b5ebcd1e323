"""The tcgen05 (tensor-memory) attention kernel against the CPU oracle and the mma.sync kernel.

kernel=2 forces the tcgen05 kernel on any 64-head bf16 call, so small cases exercise it too: list
lengths around the 128-row tile, masked rows, all-masked queries, int64 indices, fp32 output,
scores whose running maximum jumps by far more than the lazy-rescale threshold, the implicit
prefill window with the fused inverse RoPE, and the fused q norm/rope prologue."""
import importlib

import pytest
import torch

from helpers import assert_close_bf16
from oracle import norm_rope_ref as NR
from oracle import sparse_attn_ref as SA

pytestmark = pytest.mark.gpu
DEV = "cuda"
SCALE = 512 ** -0.5


def _sa():
    return importlib.import_module("deepseek-v4-flash-mlx_b200.sparse_attn")


def _bf16(x):
    return x.to(torch.bfloat16).float()


def _case(s, t, n, seed, mask_every=7):
    g = torch.Generator().manual_seed(seed)
    q = _bf16(torch.randn(s, 64, 512, generator=g))
    kv = _bf16(torch.randn(n, 512, generator=g))
    sink = torch.randn(64, generator=g)
    idx = torch.randint(0, n, (s, t), generator=g)
    if mask_every:
        idx[:, ::mask_every] = -1
    return q, kv, sink, idx


@pytest.mark.parametrize("s,t,n,idx_dtype,out_dtype", [
    (3, 1, 50, torch.int32, torch.float32),
    (5, 127, 400, torch.int32, torch.float32),
    (5, 128, 400, torch.int64, torch.float32),
    (4, 129, 400, torch.int32, torch.bfloat16),
    (6, 300, 1000, torch.int32, torch.float32),
    (2, 1152, 5000, torch.int32, torch.bfloat16),
])
def test_tc_against_oracle(dsv4, s, t, n, idx_dtype, out_dtype):
    q, kv, sink, idx = _case(s, t, n, seed=s * 7919 + t, mask_every=7 if t > 1 else 0)
    ref = SA.sparse_attn(q, kv, sink, idx, SCALE)
    out = _sa()._sparse_attn_op(q.to(DEV).bfloat16(), kv.to(DEV).bfloat16(), sink.to(DEV), idx.to(DEV, idx_dtype),
                                SCALE, out_dtype, None, None, 0, 0, kernel=2)
    assert out.dtype == out_dtype
    assert_close_bf16(out, ref, what=f"tc s={s} t={t}")


def test_tc_all_masked_query_is_nan(dsv4):
    q, kv, sink, idx = _case(3, 200, 300, seed=5, mask_every=0)
    idx[1] = -1
    out = _sa().sparse_attn(q.to(DEV).bfloat16(), kv.to(DEV).bfloat16(), sink.to(DEV), idx.to(DEV), SCALE,
                            kernel=2).float().cpu()
    assert torch.isnan(out[1]).all()
    ref = SA.sparse_attn(q, kv, sink, idx, SCALE)
    assert_close_bf16(out[[0, 2]], ref[[0, 2]], what="neighbours of a masked query")


@pytest.mark.parametrize("growth", [4.0, 9.0, 20.0])
def test_tc_growing_maximum_rescales(dsv4, growth):
    """Every 128-row tile scores `growth` log2 units above the previous one, so the running maximum
    grows past the lazy-rescale threshold (8) at every tile for growth 9 and 20, and stays under it
    for 4 (p up to 2^4 accumulated unrescaled). q = b*u + noise, kv rows = tile*a*u + noise, with
    the noise orthogonal to the unit vector u."""
    s, t = 4, 640
    g = torch.Generator().manual_seed(11)
    u = torch.randn(512, generator=g)
    u = u / u.norm()

    def orth(x):
        return x - (x @ u)[..., None] * u

    a = 0.5
    b = growth / (a * SCALE * 1.4426950408889634)
    q = _bf16(b * u + 0.5 * orth(torch.randn(s, 64, 512, generator=g)))
    tiles = (torch.arange(t) // 128).float()
    kv = _bf16(tiles[:, None] * a * u + 0.5 * orth(torch.randn(t, 512, generator=g)))
    sink = torch.randn(64, generator=g)
    idx = torch.arange(t)[None].repeat(s, 1)
    idx[:, 5::9] = -1
    ref = SA.sparse_attn(q, kv, sink, idx, SCALE)
    for kern in (1, 2):
        out = _sa().sparse_attn(q.to(DEV).bfloat16(), kv.to(DEV).bfloat16(), sink.to(DEV), idx.to(DEV), SCALE,
                                kernel=kern)
        assert_close_bf16(out, ref, what=f"growth={growth} kernel={kern}")


def test_tc_equals_mma_prefill_window_rope(dsv4):
    """Prefill shape: implicit linear window of 128 rows + 512 selected rows, fused inverse rope;
    the two kernels agree to fp32 summation-order noise (bf16 output)."""
    S = _sa()
    s, n_win, n_comp, top_k = 300, 300, 75, 512
    g = torch.Generator().manual_seed(3)
    q = torch.randn(s, 64, 512, generator=g).bfloat16().to(DEV)
    kvcat = torch.randn(n_win + n_comp, 512, generator=g).bfloat16().to(DEV)
    sink = torch.randn(64, generator=g).to(DEV)
    idx = torch.randint(n_win, n_win + n_comp, (s, top_k), generator=g, dtype=torch.int32)
    idx[:, 200:] = -1
    idx = idx.to(DEV)
    pos = torch.arange(s, dtype=torch.int32, device=DEV)
    freqs = importlib.import_module("deepseek-v4-flash-mlx_b200.norm_rope").rope_freqs(64, DEV)
    wb = torch.zeros(1, dtype=torch.int64, device=DEV)
    outs = [S.sparse_attn_rope(q, kvcat, sink, idx, SCALE, pos, freqs, 64, win_base=wb, window=128,
                               window_linear=True, kernel=k).float() for k in (1, 2)]
    assert_close_bf16(outs[1], outs[0], max_abs_tol=1.6e-2, rel_tol=4e-3, what="tc vs mma")
    # and against the oracle on a few queries
    rows = [0, 1, 127, 128, 299]
    ql, kl = q.float().cpu(), kvcat.float().cpu()
    lists = []
    for i in rows:
        lo = max(0, i - 127)
        win = list(range(lo, i + 1)) + [-1] * (128 - (i + 1 - lo))
        lists.append(torch.tensor(win + idx[i].cpu().tolist()))
    ref = SA.sparse_attn(ql[rows], kl, sink.cpu(), torch.stack(lists), SCALE)
    ref = NR.rope_at(ref, pos.cpu()[rows], freqs.cpu(), 64, inverse=True)
    assert_close_bf16(outs[1][rows], ref, what="tc window+rope vs oracle")


def test_tc_fused_q_prologue(dsv4):
    S = _sa()
    s, t, n = 160, 256, 2000
    g = torch.Generator().manual_seed(9)
    q_raw = torch.randn(s, 64, 512, generator=g).bfloat16().to(DEV)
    kv = torch.randn(n, 512, generator=g).bfloat16().to(DEV)
    sink = torch.randn(64, generator=g).to(DEV)
    idx = torch.randint(0, n, (s, t), generator=g, dtype=torch.int32).to(DEV)
    pos = torch.randint(0, 60000, (s,), generator=g, dtype=torch.int32).to(DEV)
    freqs = importlib.import_module("deepseek-v4-flash-mlx_b200.norm_rope").rope_freqs(64, DEV)
    outs = [S.sparse_attn_decode(q_raw, kv, sink, idx, SCALE, pos, freqs, kernel=k).float() for k in (1, 2)]
    assert_close_bf16(outs[1], outs[0], max_abs_tol=1.6e-2, rel_tol=4e-3, what="prologue tc vs mma")


def test_tc_rejects_unsupported_shape(dsv4):
    q, kv, sink, idx = _case(2, 64, 100, seed=1)
    L = importlib.import_module("deepseek-v4-flash-mlx_b200._lib")
    with pytest.raises(L.Dsv4Error):
        _sa().sparse_attn(q[:, :32].to(DEV).bfloat16().contiguous(), kv.to(DEV).bfloat16(), sink[:32].to(DEV),
                          idx.to(DEV), SCALE, kernel=2)
    with pytest.raises(L.Dsv4Error):
        _sa().sparse_attn(q.to(DEV), kv.to(DEV).bfloat16(), sink.to(DEV), idx.to(DEV), SCALE, kernel=2)  # fp32 q


@pytest.mark.parametrize("splits", [1, 2, 3, 5])
def test_tc_split_partials_against_oracle(dsv4, splits):
    """The tcgen05 kernel split over ranges of 128-row tiles (partials merged by the combine kernel),
    with the implicit decode window (ring order) and the fused inverse rope."""
    S = _sa()
    s, n, t = 20, 4000, 512
    g = torch.Generator().manual_seed(40 + splits)
    q = _bf16(torch.randn(s, 64, 512, generator=g))
    kv = _bf16(torch.randn(n, 512, generator=g))
    sink = torch.randn(64, generator=g)
    idx = torch.randint(128 * s, n, (s, t), generator=g, dtype=torch.int32)
    idx[:, 400:] = -1
    pos = torch.randint(0, 5000, (s,), generator=g, dtype=torch.int32)
    wb = torch.arange(s, dtype=torch.int64) * 128
    freqs = importlib.import_module("deepseek-v4-flash-mlx_b200.norm_rope").rope_freqs(64, DEV)
    out = S.sparse_attn_rope(q.to(DEV).bfloat16(), kv.to(DEV).bfloat16(), sink.to(DEV), idx.to(DEV), SCALE,
                             pos.to(DEV), freqs, 64, out_dtype=torch.float32, num_splits=splits,
                             win_base=wb.to(DEV), window=128, kernel=2)
    # the decode ring order of the window (ref_torch/sparse_attn.py:11-15) and the oracle
    lists = []
    for i in range(s):
        p = int(pos[i])
        if p >= 127:
            sp = p % 128
            win = [int(wb[i]) + (sp + 1 + u if u < 127 - sp else u - (127 - sp)) for u in range(128)]
        else:
            win = [int(wb[i]) + u if u <= p else -1 for u in range(128)]
        lists.append(torch.tensor(win + idx[i].tolist()))
    ref = SA.sparse_attn(q, kv, sink, torch.stack(lists), SCALE)
    ref = NR.rope_at(ref, pos, freqs.cpu(), 64, inverse=True)
    assert_close_bf16(out, ref, what=f"splits={splits}")
