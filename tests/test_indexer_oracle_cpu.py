"""The canonical-order indexer oracle (C) on the CPU: scores, selection rule, ties, padding."""
from fractions import Fraction

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


def _round_f32(x):
    """The float32 nearest to the rational x, ties to the even significand (IEEE round-to-nearest)."""
    c = np.float32(float(x))  # within one ulp of the answer (float64 then float32 may round twice)
    best = None
    for cand in (np.nextafter(c, np.float32(-np.inf)), c, np.nextafter(c, np.float32(np.inf))):
        d = abs(Fraction(float(cand)) - x)
        even = (int(np.array(cand, dtype=np.float32).view(np.uint32)) & 1) == 0
        if best is None or d < best[0] or (d == best[0] and even):
            best = (d, cand)
    return np.float32(best[1])


def _fmaf(a, b, c):
    return _round_f32(Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c)))


def _score_exact(q, w, k, fused=True):
    """The documented canonical order, with each fmaf rounded once from its exact value (fused), or
    as a rounded product then a rounded sum (not fused)."""
    step = _fmaf if fused else (lambda a, b, c: np.float32(np.float32(a * b) + c))
    part = []
    for m in range(16):
        p = np.float32(0.0)
        for h in range(4 * m, 4 * m + 4):
            d = np.float32(0.0)
            for i in range(128):
                d = step(q[h, i], k[i], d)
            p = step(w[h], d if d > 0 else np.float32(0.0), p)
        part.append(p)
    while len(part) > 1:
        part = [np.float32(part[2 * t] + part[2 * t + 1]) for t in range(len(part) // 2)]
    return part[0]


def test_c_oracle_is_the_canonical_fma_order():
    """The C oracle (which the GPU score kernels match bit for bit) against an independent Python
    restatement of its documented order with exactly rounded fmaf: equal bit for bit, and different
    from the same order without fused multiply-adds (so the comparison can tell them apart)."""
    q, w, k = _rand(4, 5)
    got = I.scores(q, w, k)
    fused = np.array([_score_exact(q, w, k[j]) for j in range(4)], dtype=np.float32)
    plain = np.array([_score_exact(q, w, k[j], fused=False) for j in range(4)], dtype=np.float32)
    np.testing.assert_array_equal(got.view(np.uint32), fused.view(np.uint32))
    assert (plain.view(np.uint32) != fused.view(np.uint32)).any()
