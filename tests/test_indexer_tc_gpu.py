"""The tensor-core filter of the indexer (mode 2): approximate tcgen05 scores within the proven bound,
and the selected sets bit-identical to the CPU oracle and to the all-exact path (mode 1)."""
import numpy as np
import pytest
import torch

from oracle import indexer_ref as I

pytestmark = pytest.mark.gpu
DEV = "cuda"
EPS_C = 2.0 ** -14


def _inputs(b, s, n, seed, spread=False):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, s, 64, 128, generator=g)
    w = torch.randn(b, s, 64, generator=g) / 8
    k = torch.randn(b, n, 128, generator=g)
    if spread:  # elements spanning 2^-8 .. 2^8 within every vector
        q = q * torch.exp2(torch.randint(-8, 9, q.shape, generator=g).float())
        k = k * torch.exp2(torch.randint(-8, 9, k.shape, generator=g).float())
    return q, w, k


@pytest.mark.parametrize("spread", [False, True])
def test_approx_scores_within_bound(dsv4, spread):
    """|A - score| <= eps = C * sum_h |w_h| ||q_h|| * max_j ||k_j|| for every visible entry; the
    observed worst case is reported against the bound (the filter's safety margin)."""
    q, w, k = _inputs(1, 260, 3000, 5 + spread, spread)
    qd, wd, kd = q.to(DEV), w.to(DEV), k.to(DEV)
    approx = dsv4.indexer_scores(qd, wd, kd, mode=2).cpu().double()
    exact = dsv4.indexer_scores(qd, wd, kd, mode=1).cpu().double()
    kmax = k[0].double().norm(dim=-1).max()
    wq = (w[0].double().abs() * q[0].double().norm(dim=-1)).sum(-1)          # [s]
    eps = EPS_C * wq * kmax
    ratio = ((approx[0] - exact[0]).abs() / eps[:, None]).max().item()
    print(f"max |A - score| / eps = {ratio:.3e} (spread={spread})")
    assert ratio <= 0.25, ratio


@pytest.mark.parametrize("b,s,n,k,causal", [
    (1, 300, 2000, 512, True),
    (2, 260, 1000, 64, False),
    (1, 256, 16384, 1024, True),
    (1, 257, 777, 100, False),
    (12, 2, 3000, 512, True),     # two queries per batch entry: the per-sequence walk, causal
    (40, 1, 9000, 512, False),    # decode batch, a walk that crosses queries inside a CTA
])
def test_mode2_selection_bit_exact(dsv4, b, s, n, k, causal):
    q, w, keys = _inputs(b, s, n, b * 31 + s + n)
    pos = None
    if causal:
        pos = torch.arange(n * 4 - s, n * 4, dtype=torch.int32)[None].repeat(b, 1)
    args = (q.to(DEV), w.to(DEV), keys.to(DEV), k, None if pos is None else pos.to(DEV))
    got2 = dsv4.indexer_topk(*args, mode=2).cpu().numpy()
    got1 = dsv4.indexer_topk(*args, mode=1).cpu().numpy()
    np.testing.assert_array_equal(got2, got1)
    # the same filter reading a key image built once (as a decode cache keeps it)
    mod = __import__("importlib").import_module("deepseek-v4-flash-mlx_b200.indexer")
    kd = keys.to(DEV)
    image = mod.build_key_image(kd, mod.key_image_buffers(b, n, DEV))
    outi = torch.full((b, s, k), -7, dtype=torch.int32, device=DEV)
    mod.indexer_topk_into(outi, q.to(DEV), w.to(DEV), kd, k, positions=None if pos is None else pos.to(DEV), ratio=4,
                          mode=2, key_image=image)
    np.testing.assert_array_equal(outi.cpu().numpy(), got1)
    rows = range(s) if s * n <= 300 * 2000 else range(0, s, 16)
    ref = I.indexer_topk(q[:, list(rows)].numpy(), w[:, list(rows)].numpy(), keys.numpy(), k,
                         None if pos is None else pos[:, list(rows)].numpy())
    np.testing.assert_array_equal(got2[:, list(rows)], ref)


def test_mode2_ties_and_wide_band(dsv4):
    """Duplicated keys (exact ties across the band) and a query whose scores are all equal (every
    key in the band: several rescoring rounds; the lowest indices win)."""
    q, w, keys = _inputs(1, 256, 1500, 77)
    keys[0, 750:] = keys[0, :750]
    w[0, 3] = 0.0                      # query 3: every score is +0
    args = (q.to(DEV), w.to(DEV), keys.to(DEV), 300)
    got = dsv4.indexer_topk(*args, mode=2).cpu().numpy()
    np.testing.assert_array_equal(got, dsv4.indexer_topk(*args, mode=1).cpu().numpy())
    np.testing.assert_array_equal(got[0, 3], np.arange(300))
    ref = I.indexer_topk(q[:, :8].numpy(), w[:, :8].numpy(), keys.numpy(), 300)
    np.testing.assert_array_equal(got[:, :8], ref)


def test_mode2_spread_inputs_bit_exact(dsv4):
    q, w, keys = _inputs(1, 256, 2500, 91, spread=True)
    args = (q.to(DEV), w.to(DEV), keys.to(DEV), 256)
    np.testing.assert_array_equal(dsv4.indexer_topk(*args, mode=2).cpu().numpy(),
                                  dsv4.indexer_topk(*args, mode=1).cpu().numpy())


def test_mode2_into_window_and_offset(dsv4):
    """The prefill call shape: index list with the linear window columns and a row offset."""
    mod = __import__("importlib").import_module("deepseek-v4-flash-mlx_b200.indexer")
    s, n, k = 512, 400, 128
    q, w, keys = _inputs(1, s, n, 12)
    pos = torch.arange(1024, 1024 + s, dtype=torch.int32)[None]
    outs = []
    for mode in (1, 2):
        out = torch.full((1, s, 128 + k), -7, dtype=torch.int32, device=DEV)
        mod.indexer_topk_into(out, q.to(DEV), w.to(DEV), keys.to(DEV), k, positions=pos.to(DEV), ratio=4, out_col=128,
                              out_offset=5000, win_base=torch.zeros(1, dtype=torch.int64, device=DEV), window=128,
                              window_linear=True, mode=mode)
        outs.append(out.cpu().numpy())
    np.testing.assert_array_equal(outs[1], outs[0])


def test_mode2_row_scales_bit_exact(dsv4):
    """Rows of very different magnitude (2^-40 .. 2^40 per query head and per key): the per-row
    power-of-two scaling keeps the fp16 split exact up to its rounding; the sets match mode 1."""
    q, w, keys = _inputs(1, 256, 2000, 55)
    g = torch.Generator().manual_seed(56)
    q = q * torch.exp2(torch.randint(-40, 41, (1, 256, 64, 1), generator=g).float())
    keys = keys * torch.exp2(torch.randint(-40, 41, (1, 2000, 1), generator=g).float())
    args = (q.to(DEV), w.to(DEV), keys.to(DEV), 200)
    got = dsv4.indexer_topk(*args, mode=2).cpu().numpy()
    np.testing.assert_array_equal(got, dsv4.indexer_topk(*args, mode=1).cpu().numpy())
    ref = I.indexer_topk(q[:, :6].numpy(), w[:, :6].numpy(), keys.numpy(), 200)
    np.testing.assert_array_equal(got[:, :6], ref)


@pytest.mark.parametrize("b,n,k", [(20, 3000, 512), (64, 2048, 512), (17, 700, 100)])
def test_mode2_decode_batch_bit_exact(dsv4, b, n, k):
    """Decode batches (one query per sequence): the one-query-per-CTA tensor-core filter, causal
    visibility per sequence, block-table output mapping and the window columns, against mode 1 and
    the oracle."""
    mod = __import__("importlib").import_module("deepseek-v4-flash-mlx_b200.indexer")
    q, w, keys = _inputs(b, 1, n, 1000 + b)
    g = torch.Generator().manual_seed(b)
    pos = torch.randint(4 * k, 4 * n + 8, (b, 1), generator=g, dtype=torch.int32)   # some see all n keys
    page = 64
    pages = (n + page - 1) // page
    table = torch.stack([torch.randperm(pages, generator=g) for _ in range(b)]).to(torch.int32)
    outs = []
    image = mod.build_key_image(keys.to(DEV), mod.key_image_buffers(b, n, DEV))
    for mode, kimg in ((1, None), (2, None), (2, image)):
        out = torch.full((b, 1, 128 + k), -7, dtype=torch.int32, device=DEV)
        mod.indexer_topk_into(out, q.to(DEV), w.to(DEV), keys.to(DEV), k, positions=pos.to(DEV), ratio=4, out_col=128,
                              out_offset=333, block_table=table.to(DEV), page=page,
                              win_base=torch.arange(b, dtype=torch.int64, device=DEV) * 128, window=128, mode=mode,
                              key_image=kimg)
        outs.append(out.cpu().numpy())
    np.testing.assert_array_equal(outs[1], outs[0])
    np.testing.assert_array_equal(outs[2], outs[0])   # the filter reading a kept key image
    ref = I.indexer_topk(q.numpy(), w.numpy(), keys.numpy(), k, pos.numpy())          # [b, 1, k] key indices
    sel = ref[:, 0]
    mapped = np.where(sel >= 0, table.numpy()[np.arange(b)[:, None], np.maximum(sel, 0) // page] * page
                      + np.maximum(sel, 0) % page + 333, -1)
    np.testing.assert_array_equal(np.sort(outs[1][:, 0, 128:], axis=1), np.sort(mapped, axis=1))
