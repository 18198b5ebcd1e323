"""The head-group decode attention kernel (kernel=3: 16 heads per CTA, the 64-row tiles of a query
split over up to 16 CTAs merged as one thread-block cluster, q's norm + RoPE fused) against the CPU
oracle (ref_torch/sparse_attn.py:23-34 restated) and the other kernels.

Cases: list lengths around the 64-row tile, masked rows, all-masked queries, int64 indices, fp32 and
bf16 outputs, 16 / 32 / 64 heads, every split count from one CTA (online softmax across tiles) to 16,
the implicit decode window in ring order with the inverse RoPE, the fused q prologue from fp32 and
bf16 raw q, running maxima that jump between tiles, and out-of-range indices."""
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


def _freqs():
    return importlib.import_module("deepseek-v4-flash-mlx_b200.norm_rope").rope_freqs(64, DEV)


def _bf16(x):
    return x.to(torch.bfloat16).float()


def _case(s, t, n, seed, h=64, mask_every=7):
    g = torch.Generator().manual_seed(seed)
    q = _bf16(torch.randn(s, h, 512, generator=g))
    kv = _bf16(torch.randn(n, 512, generator=g))
    sink = torch.randn(h, generator=g)
    idx = torch.randint(0, n, (s, t), generator=g)
    if mask_every:
        idx[:, ::mask_every] = -1
    return q, kv, sink, idx


@pytest.mark.parametrize("s,t,n,h,idx_dtype,out_dtype,splits", [
    (1, 1, 50, 64, torch.int32, torch.float32, 0),
    (1, 63, 400, 64, torch.int32, torch.float32, 0),
    (2, 64, 400, 64, torch.int64, torch.float32, 0),
    (3, 65, 400, 32, torch.int32, torch.bfloat16, 0),
    (1, 640, 9000, 64, torch.int32, torch.bfloat16, 0),
    (1, 640, 9000, 64, torch.int32, torch.float32, 1),
    (4, 640, 9000, 16, torch.int32, torch.float32, 3),
    (2, 1152, 5000, 64, torch.int32, torch.bfloat16, 16),
    (15, 300, 3000, 64, torch.int32, torch.float32, 0),
])
def test_hg_against_oracle(dsv4, s, t, n, h, idx_dtype, out_dtype, splits):
    q, kv, sink, idx = _case(s, t, n, seed=s * 7919 + t + h, h=h, mask_every=7 if t > 1 else 0)
    ref = SA.sparse_attn(q, kv, sink, idx, SCALE)
    out = _sa()._sparse_attn_op(q.to(DEV).bfloat16(), kv.to(DEV).bfloat16(), sink.to(DEV), idx.to(DEV, idx_dtype),
                                SCALE, out_dtype, None, None, 0, splits, kernel=3)
    assert out.dtype == out_dtype
    assert_close_bf16(out, ref, what=f"hg s={s} t={t} h={h} splits={splits}")


def test_hg_all_masked_query_is_nan(dsv4):
    q, kv, sink, idx = _case(3, 640, 3000, seed=5, mask_every=0)
    idx[1] = -1
    idx[2, 64:] = -1   # a query whose later splits hold no valid row
    out = _sa().sparse_attn(q.to(DEV).bfloat16(), kv.to(DEV).bfloat16(), sink.to(DEV), idx.to(DEV), SCALE,
                            kernel=3).float().cpu()
    assert torch.isnan(out[1]).all()
    ref = SA.sparse_attn(q, kv, sink, idx, SCALE)
    assert_close_bf16(out[[0, 2]], ref[[0, 2]], what="neighbours of a masked query")


@pytest.mark.parametrize("growth", [4.0, 20.0])
@pytest.mark.parametrize("splits", [1, 10])
def test_hg_growing_maximum(dsv4, growth, splits):
    """Every 64-row tile scores `growth` log2 units above the previous one: with one split the
    online softmax rescales at every tile, with ten the cluster merge weighs very different maxima."""
    s, t = 2, 640
    g = torch.Generator().manual_seed(11)
    u = torch.randn(512, generator=g)
    u = u / u.norm()

    def orth(x):
        return x - (x @ u)[..., None] * u

    a = 0.5
    b = growth / (a * SCALE * 1.4426950408889634)
    q = _bf16(b * u + 0.5 * orth(torch.randn(s, 64, 512, generator=g)))
    tiles = (torch.arange(t) // 64).float()
    kv = _bf16(tiles[:, None] * a * u + 0.5 * orth(torch.randn(t, 512, generator=g)))
    sink = torch.randn(64, generator=g)
    idx = torch.arange(t)[None].repeat(s, 1)
    idx[:, 5::9] = -1
    ref = SA.sparse_attn(q, kv, sink, idx, SCALE)
    out = _sa()._sparse_attn_op(q.to(DEV).bfloat16(), kv.to(DEV).bfloat16(), sink.to(DEV), idx.to(DEV), SCALE,
                                torch.float32, None, None, 0, splits, kernel=3)
    assert_close_bf16(out, ref, what=f"growth={growth} splits={splits}")


@pytest.mark.parametrize("q_dtype", [torch.float32, torch.bfloat16])
def test_hg_decode_window_prologue_rope(dsv4, q_dtype):
    """The decode call: raw q (per-head norm + RoPE fused in the kernel), the implicit window in ring
    order at positions on both sides of 127, 512 selected rows, the inverse RoPE of the output;
    against the oracle and the mma.sync kernel with its separate prologue."""
    S = _sa()
    s, n, t = 5, 6000, 512
    g = torch.Generator().manual_seed(77)
    q_raw = torch.randn(s, 64, 512, generator=g).to(q_dtype)
    kv = _bf16(torch.randn(n, 512, generator=g))
    sink = torch.randn(64, generator=g)
    idx = torch.randint(128 * s, n, (s, t), generator=g, dtype=torch.int32)
    idx[:, 450:] = -1
    pos = torch.tensor([5, 126, 127, 128, 40000], dtype=torch.int32)
    wb = torch.arange(s, dtype=torch.int64) * 128
    freqs = _freqs()
    args = (q_raw.to(DEV), kv.to(DEV).bfloat16(), sink.to(DEV), idx.to(DEV), SCALE, torch.float32, freqs,
            pos.to(DEV), 64, 0, True, 1e-6, wb.to(DEV), 128, False)
    out3 = S._sparse_attn_op(*args, kernel=3)
    out1 = S._sparse_attn_op(*args, kernel=1)
    assert_close_bf16(out3, out1, max_abs_tol=1.6e-2, rel_tol=4e-3, what="hg vs mma.sync")
    lists = []
    for i in range(s):
        p = int(pos[i])
        if p >= 127:
            sp = p % 128
            win = [int(wb[i]) + (sp + 1 + u if u < 127 - sp else u - (127 - sp)) for u in range(128)]
        else:
            win = [int(wb[i]) + u if u <= p else -1 for u in range(128)]
        lists.append(torch.tensor(win + idx[i].tolist()))
    qn = NR.rope_at(NR.perhead_norm(q_raw.float()), pos, freqs.cpu(), 64)
    ref = SA.sparse_attn(_bf16(qn), kv, sink, torch.stack(lists), SCALE)
    ref = NR.rope_at(ref, pos, freqs.cpu(), 64, inverse=True)
    assert_close_bf16(out3, ref, what=f"hg decode call, q {q_dtype}")


def test_hg_out_of_range_index_flags_device_error(dsv4):
    L = importlib.import_module("deepseek-v4-flash-mlx_b200._lib")
    L.device_error()   # clear
    q, kv, sink, idx = _case(1, 200, 300, seed=3, mask_every=0)
    idx[0, 17] = 300   # one past the pool
    out = _sa().sparse_attn(q.to(DEV).bfloat16(), kv.to(DEV).bfloat16(), sink.to(DEV), idx.to(DEV), SCALE,
                            kernel=3).float().cpu()
    assert L.device_error() == 4   # DSV4_ERR_INDEX_OUT_OF_RANGE, and the row was masked
    idx[0, 17] = -1
    ref = SA.sparse_attn(q, kv, sink, idx, SCALE)
    assert_close_bf16(out, ref, what="masked out-of-range row")
