"""Hyper-connection kernels (hc_pre / hc_post / hc_head, ref_torch/hc.py:18-80) on the GPU against
the float64 oracle and the reference's own outputs.

Tolerances: the kernels compute in fp32 (24 dot products of length hc*dim as per-thread FMA chains
and block reductions, sigmoid/exp through CUDA's expf); against the float64 oracle that is a
relative error of a few 1e-6 on mixes, so y / post / comb are checked at rtol 2e-5, atol 2e-6
(comb after 20 Sinkhorn rounds included). The bf16 RMSNorm output is checked to one bf16 rounding
(rtol 2^-8) against the oracle's norm of the kernel's own fp32 y."""
import numpy as np
import pytest
import torch

from oracle import hc_ref as H

pytestmark = pytest.mark.gpu
DEV = "cuda"
RTOL, ATOL = 2e-5, 2e-6


def _qat():
    import os
    return np.load(os.path.join(os.path.dirname(__file__), "golden", "qat_golden.npz"))


def _inputs(rows, dim, seed, head=False):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, 4, dim, generator=g)
    nm = 4 if head else 24
    fn = torch.randn(nm, 4 * dim, generator=g) * 0.02
    scale = torch.rand(1 if head else 3, generator=g) + 0.5
    base = torch.randn(nm, generator=g) * 0.1
    return x, fn, scale, base


def test_hc_golden(dsv4):
    z = _qat()
    t = {k: torch.from_numpy(z[k]).to(DEV) for k in z.files if k.startswith("hc_")}
    y, post, comb = dsv4.hc_pre(t["hc_x"], t["hc_fn"], t["hc_scale"], t["hc_base"])
    np.testing.assert_allclose(y.cpu().numpy(), z["hc_y"], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(post.cpu().numpy(), z["hc_post"], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(comb.cpu().numpy(), z["hc_comb"], rtol=RTOL, atol=ATOL)
    out = dsv4.hc_post(t["hc_att"], t["hc_x"], t["hc_post"], t["hc_comb"])
    np.testing.assert_allclose(out.cpu().numpy(), z["hc_post_y"], rtol=RTOL, atol=1e-5)
    yh = dsv4.hc_head(t["hc_x"], t["hc_head_fn"], t["hc_head_scale"], t["hc_head_base"])
    np.testing.assert_allclose(yh.cpu().numpy(), z["hc_head_y"], rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("rows,dim", [(1, 4096), (7, 4096), (64, 4096), (3, 3072), (5, 260), (2, 1024), (300, 512),
                                      (600, 4096), (257, 260)])
def test_hc_pre_shapes(dsv4, rows, dim):
    x, fn, scale, base = _inputs(rows, dim, 10 + rows + dim)
    y, post, comb = dsv4.hc_pre(x.to(DEV), fn.to(DEV), scale.to(DEV), base.to(DEV))
    ry, rp, rc = H.hc_pre(x.numpy(), fn.numpy(), scale.numpy(), base.numpy())
    np.testing.assert_allclose(post.cpu().numpy(), rp, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(comb.cpu().numpy(), rc, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(y.cpu().numpy(), ry, rtol=RTOL, atol=1e-5)


def test_hc_pre_sinkhorn_iters_and_eps(dsv4):
    x, fn, scale, base = _inputs(9, 512, 3)
    for iters, eps in ((1, 1e-6), (3, 1e-3), (20, 0.0)):
        y, post, comb = dsv4.hc_pre(x.to(DEV), fn.to(DEV), scale.to(DEV), base.to(DEV), sinkhorn_iters=iters,
                                    hc_eps=eps, norm_eps=1e-5)
        ry, rp, rc = H.hc_pre(x.numpy(), fn.numpy(), scale.numpy(), base.numpy(), iters=iters, hc_eps=eps,
                              norm_eps=1e-5)
        np.testing.assert_allclose(comb.cpu().numpy(), rc, rtol=RTOL, atol=ATOL, err_msg=f"iters {iters}")
        np.testing.assert_allclose(y.cpu().numpy(), ry, rtol=RTOL, atol=1e-5, err_msg=f"iters {iters}")


@pytest.mark.parametrize("w_dtype", [torch.bfloat16, torch.float32, None])
def test_hc_pre_fused_norm(dsv4, w_dtype):
    """hc_pre with the block's attn_norm in the same launch: bf16 RMSNorm(y) * w."""
    x, fn, scale, base = _inputs(6, 4096, 21)
    w = None if w_dtype is None else (torch.rand(4096) + 0.5).to(w_dtype)
    args = (x.to(DEV), fn.to(DEV), scale.to(DEV), base.to(DEV))
    if w is None:
        # no weight: pass a ones vector through the op layer's norm_w argument contract
        w = torch.ones(4096)
    y, post, comb, yn = dsv4.hc_pre(*args, norm_w=w.to(DEV))
    assert yn.dtype == torch.bfloat16
    ref = H.rmsnorm(y.cpu().numpy(), w.float().numpy())
    np.testing.assert_allclose(yn.float().cpu().numpy(), ref, rtol=2 ** -8, atol=1e-6)
    y2, _, _ = dsv4.hc_pre(*args)
    assert torch.equal(y, y2)


@pytest.mark.parametrize("rows,dim", [(3, 256), (64, 4096), (1, 4), (400, 1024)])
def test_hc_head_shapes(dsv4, rows, dim):
    x, fn, scale, base = _inputs(rows, dim, 5 + dim, head=True)
    y = dsv4.hc_head(x.to(DEV), fn.to(DEV), scale.to(DEV), base.to(DEV))
    np.testing.assert_allclose(y.cpu().numpy(), H.hc_head(x.numpy(), fn.numpy(), scale.numpy(), base.numpy()),
                               rtol=RTOL, atol=1e-5)


@pytest.mark.parametrize("rows,dim", [(1, 4096), (37, 4096), (5, 260)])
def test_hc_post_shapes(dsv4, rows, dim):
    g = torch.Generator().manual_seed(rows + dim)
    x = torch.randn(rows, dim, generator=g)
    res = torch.randn(rows, 4, dim, generator=g)
    post = torch.rand(rows, 4, generator=g) * 2
    comb = torch.rand(rows, 4, 4, generator=g)
    out = dsv4.hc_post(x.to(DEV), res.to(DEV), post.to(DEV), comb.to(DEV))
    np.testing.assert_allclose(out.cpu().numpy(), H.hc_post(x.numpy(), res.numpy(), post.numpy(), comb.numpy()),
                               rtol=1e-6, atol=1e-6)


def test_hc_round_trip_layer_shapes(dsv4):
    """hc_pre -> (a stand-in block output) -> hc_post over a [b, s] batch, against the oracle chain."""
    g = torch.Generator().manual_seed(77)
    x = torch.randn(2, 3, 4, 512, generator=g)
    fn = torch.randn(24, 2048, generator=g) * 0.02
    scale, base = torch.rand(3, generator=g) + 0.5, torch.randn(24, generator=g) * 0.1
    y, post, comb = dsv4.hc_pre(x.to(DEV), fn.to(DEV), scale.to(DEV), base.to(DEV))
    assert y.shape == (2, 3, 512) and post.shape == (2, 3, 4) and comb.shape == (2, 3, 4, 4)
    att = torch.tanh(y)
    out = dsv4.hc_post(att, x.to(DEV), post, comb)
    ry, rp, rc = H.hc_pre(x.numpy(), fn.numpy(), scale.numpy(), base.numpy())
    ro = H.hc_post(np.tanh(ry), x.numpy(), rp, rc)
    np.testing.assert_allclose(out.cpu().numpy(), ro, rtol=1e-4, atol=1e-5)


def test_hc_errors(dsv4):
    x, fn, scale, base = _inputs(2, 256, 1)
    with pytest.raises(ValueError):
        dsv4.hc_pre(x.to(DEV), fn.to(DEV), scale.to(DEV), base.to(DEV), hc=2)
    bad = torch.randn(2, 4, 258, device=DEV)
    with pytest.raises(RuntimeError):
        dsv4.hc_pre(bad, torch.randn(24, 4 * 258, device=DEV), scale.to(DEV), base.to(DEV))
    with pytest.raises(RuntimeError):
        dsv4.hc_post(torch.randn(2, 258, device=DEV), torch.randn(2, 4, 258, device=DEV), torch.rand(2, 4, device=DEV),
                     torch.rand(2, 4, 4, device=DEV))
    with pytest.raises(RuntimeError):
        dsv4.hc_pre(x.cpu(), fn, scale, base)
