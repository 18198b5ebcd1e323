"""Oracle (test infrastructure only): the hyper-connection mixes around the attention block.

Restates ref_torch/hc.py:18-80 (the official Block.hc_pre / hc_post and ParallelHead.hc_head) in
numpy, in float64 so it can stand as the checker of an fp32 kernel. The residual stream holds
hc = 4 copies of a token's hidden state, x [..., hc, dim]:
  r      = 1 / sqrt(mean over all hc*dim values of x^2 + norm_eps)
  mixes  = (x flattened) . fn^T * r                     fn [(2+hc)*hc, hc*dim]   (hc.py:55-56)
  pre    = sigmoid(mixes[0:hc] s0 + b[0:hc]) + eps                               (hc.py:30)
  post   = 2 sigmoid(mixes[hc:2hc] s1 + b[hc:2hc])                               (hc.py:31)
  comb   = row softmax(mixes[2hc:] s2 + b[2hc:], as [hc, hc]) + eps, then the columns divided by
           their sum + eps; then iters-1 rounds of rows / (row sum + eps), columns / (column sum
           + eps)                                                                (hc.py:32-40)
  y      = sum_k pre[k] x[k]                                                     (hc.py:58)
  hc_post: out[j] = post[j] x + sum_i comb[i, j] residual[i]                     (hc.py:67-68)
  hc_head: fn [hc, hc*dim], one scale; pre only                                  (hc.py:75-80)
"""
import numpy as np


def _sigmoid(v):
    return 1.0 / (1.0 + np.exp(-v))


def _mixes(x, fn, norm_eps):
    xf = np.asarray(x, np.float64).reshape(*x.shape[:-2], -1)
    r = 1.0 / np.sqrt(np.mean(xf * xf, axis=-1, keepdims=True) + norm_eps)
    return (xf @ np.asarray(fn, np.float64).T) * r


def sinkhorn_split(mixes, scale, base, hc=4, iters=20, eps=1e-6):
    """mixes [..., (2+hc)*hc] -> pre [..., hc], post [..., hc], comb [..., hc, hc] (hc.py:18-41)."""
    s = np.asarray(scale, np.float64)
    b = np.asarray(base, np.float64)
    pre = _sigmoid(mixes[..., :hc] * s[0] + b[:hc]) + eps
    post = 2.0 * _sigmoid(mixes[..., hc:2 * hc] * s[1] + b[hc:2 * hc])
    c = (mixes[..., 2 * hc:] * s[2] + b[2 * hc:]).reshape(*mixes.shape[:-1], hc, hc)
    c = np.exp(c - c.max(axis=-1, keepdims=True))
    c = c / c.sum(axis=-1, keepdims=True) + eps
    c = c / (c.sum(axis=-2, keepdims=True) + eps)
    for _ in range(iters - 1):
        c = c / (c.sum(axis=-1, keepdims=True) + eps)
        c = c / (c.sum(axis=-2, keepdims=True) + eps)
    return pre, post, c


def hc_pre(x, fn, scale, base, hc=4, norm_eps=1e-6, iters=20, hc_eps=1e-6):
    """x [..., hc, dim] -> y [..., dim], post [..., hc], comb [..., hc, hc] (float64)."""
    pre, post, comb = sinkhorn_split(_mixes(x, fn, norm_eps), scale, base, hc, iters, hc_eps)
    y = np.einsum("...k,...kd->...d", pre, np.asarray(x, np.float64))
    return y, post, comb


def hc_head(x, fn, scale, base, hc=4, norm_eps=1e-6, hc_eps=1e-6):
    """x [..., hc, dim] -> y [..., dim] (float64)."""
    m = _mixes(x, fn, norm_eps)
    pre = _sigmoid(m * float(np.asarray(scale).reshape(-1)[0]) + np.asarray(base, np.float64)) + hc_eps
    return np.einsum("...k,...kd->...d", pre, np.asarray(x, np.float64))


def hc_post(x, residual, post, comb):
    """x [..., dim], residual [..., hc, dim], post [..., hc], comb [..., hc, hc] -> [..., hc, dim]."""
    x = np.asarray(x, np.float64)
    res = np.asarray(residual, np.float64)
    return (np.asarray(post, np.float64)[..., :, None] * x[..., None, :]
            + np.einsum("...ij,...id->...jd", np.asarray(comb, np.float64), res))


def rmsnorm(y, w=None, eps=1e-6):
    """The attention block's first norm of hc_pre's y (float64)."""
    y = np.asarray(y, np.float64)
    o = y / np.sqrt(np.mean(y * y, axis=-1, keepdims=True) + eps)
    return o if w is None else o * np.asarray(w, np.float64)
