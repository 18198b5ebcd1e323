import torch

# tolerance of a bf16 path against the fp32 oracle (the north-star bar for attention outputs)
MAX_ABS = 2e-2
REL_RMS = 5e-3


def rel_rms(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).norm() / b.norm().clamp(min=1e-30)).item()


def max_abs(a, b):
    return (a.double().cpu() - b.double().cpu()).abs().max().item()


def assert_close_bf16(got, ref, max_abs_tol=MAX_ABS, rel_tol=REL_RMS, what=""):
    got, ref = got.float().cpu(), ref.float().cpu()
    assert got.shape == ref.shape, (got.shape, ref.shape)
    finite = torch.isfinite(ref)
    assert torch.equal(torch.isfinite(got), finite), f"{what}: non-finite pattern differs"
    g, r = got[finite], ref[finite]
    ma, rr = max_abs(g, r), rel_rms(g, r)
    assert ma <= max_abs_tol and rr <= rel_tol, f"{what}: max_abs={ma:.3e} rel_rms={rr:.3e}"
    return ma, rr
