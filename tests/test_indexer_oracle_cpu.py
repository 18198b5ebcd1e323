"""The canonical-order indexer oracle (C) on the CPU: scores, selection rule, ties, padding."""
import numpy as np

from oracle import indexer_ref as I


def _rand(n, seed=0):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((64, 128)).astype(np.float32)
    w = (rng.standard_normal(64) / 8).astype(np.float32)
    k = rng.standard_normal((n, 128)).astype(np.float32)
    return q, w, k


def test_scores_track_float64():
    q, w, k = _rand(2048)
    s = I.scores(q, w, k)
    s64 = I.scores_f64(q, w, k)
    assert np.abs(s - s64).max() <= 1e-5 * np.abs(s64).max() + 1e-5


def test_selection_is_top_k_by_score_then_index():
    q, w, k = _rand(3000, 1)
    s = I.scores(q, w, k)
    sel = I.select(s, 512)
    assert (np.diff(sel) > 0).all()
    order = np.lexsort((np.arange(s.size), -s.astype(np.float64)))
    np.testing.assert_array_equal(np.sort(order[:512]), sel)


def test_ties_break_on_lower_index():
    s = np.zeros(100, dtype=np.float32)
    s[[3, 50, 70, 90]] = 2.0
    s[[10, 20, 30, 40]] = 1.0            # four-way tie at the boundary, two are taken
    sel = I.select(s, 6)
    np.testing.assert_array_equal(sel, [3, 10, 20, 50, 70, 90])
    s2 = np.full(10, -1.0, dtype=np.float32)
    s2[7] = -0.0
    s2[2] = 0.0                           # +0 ranks above -0 (order-preserving image of the bits)
    np.testing.assert_array_equal(I.select(s2, 1), [2])


def test_fewer_visible_than_k_pads():
    q, w, k = _rand(64, 2)
    out = I.indexer_topk(q[None, None], w[None, None], k[None], top_k=16, positions=np.array([[39]]), ratio=4)
    np.testing.assert_array_equal(out[0, 0], list(range(10)) + [-1] * 6)


def test_causal_visibility_per_query():
    rng = np.random.default_rng(3)
    s, n = 12, 16
    q = rng.standard_normal((1, s, 64, 128)).astype(np.float32)
    w = rng.standard_normal((1, s, 64)).astype(np.float32)
    k = rng.standard_normal((1, n, 128)).astype(np.float32)
    pos = np.arange(30, 30 + s)
    out = I.indexer_topk(q, w, k, top_k=4, positions=pos[None], ratio=4)
    for i in range(s):
        nv = min((pos[i] + 1) // 4, n)
        sc = I.scores(q[0, i], w[0, i], k[0, :nv])
        np.testing.assert_array_equal(out[0, i], I.select(sc, 4))
        assert out[0, i].max() < nv
