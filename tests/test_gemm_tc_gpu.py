"""The tcgen05 projection GEMM (TMA-fed, fp32 accumulator in tensor memory) against the fp64
product of the same bf16 operands, the mma.sync kernels, and itself.

kernel=2 forces it at any m; m > 64 with bf16 weights selects it automatically. Cases cover one
k step, ragged m and n (the zero-filled rows of a partial tile, n not a multiple of the vector
width), grouped weights narrower than a tile, bf16 output, several projections in one launch, and
the compressor's prefill shapes (v4mlx/mla.py:16-56, ref_torch/compressor.py:27-28)."""
import ctypes
import importlib

import pytest
import torch

from helpers import rel_rms

pytestmark = pytest.mark.gpu
DEV = "cuda"
PKG = "deepseek-v4-flash-mlx_b200"


def _L():
    return importlib.import_module(PKG + "._lib")


def _linear(x, w, groups, out_dtype, kernel):
    """dsv4_linear with an explicit kernel choice (x [m, groups*k] bf16, w [groups*n, k] bf16)."""
    L = _L()
    m, k = x.shape[0], w.shape[1]
    n = w.shape[0] // groups
    y = torch.empty(m, groups * n, dtype=out_dtype, device=DEV)
    p = L.LinearParams()
    p.x, p.w, p.y = L.ptr(x), L.ptr(w), L.ptr(y)
    p.m, p.n, p.k, p.groups, p.group = m, n, k, groups, 64
    p.x_dtype, p.w_dtype, p.y_dtype = L.BF16, L.BF16, L.dtype_code(y)
    p.kernel = kernel
    nbytes = L.lib().dsv4_linear_workspace_size(ctypes.byref(p))
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=DEV)
    p.workspace, p.workspace_bytes = L.ptr(ws), nbytes
    L.check(L.lib().dsv4_linear(ctypes.byref(p), L.stream_of(x)))
    return y


def _operands(m, n, k, groups, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, groups * k, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(groups * n, k, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    ref = torch.einsum("mgk,gnk->mgn", x.double().view(m, groups, k), w.double().view(groups, n, k)).reshape(m, -1)
    return x, w, ref


@pytest.mark.parametrize("m,n,k,groups,out_dtype", [
    (65, 256, 64, 1, torch.float32),       # one tile, one k step
    (200, 198, 128, 1, torch.float32),     # ragged m and n; rows of 198 floats: scalar stores
    (300, 1024, 4096, 1, torch.float32),   # the main compressor's projection width
    (129, 64, 512, 8, torch.float32),      # grouped, 64 rows per group (the tile reads past the group)
    (1000, 130, 1024, 1, torch.bfloat16),  # bf16 output, a partial weight tile
    (1, 512, 256, 1, torch.float32),       # forced at one token
    (4096, 1024, 4096, 1, torch.float32),  # a prefill chunk
    (8192, 256, 4096, 1, torch.float32),   # the indexer compressor's width over 8,192 tokens
])
def test_tcgen05_linear_matches_fp64(dsv4, m, n, k, groups, out_dtype):
    x, w, ref = _operands(m, n, k, groups, m + n + k + groups)
    out = _linear(x, w, groups, out_dtype, kernel=2)
    tol = 1e-5 if out_dtype == torch.float32 else 4e-3
    assert rel_rms(out, ref) < tol
    err = (out.double() - ref).abs().max().item()
    assert err <= (1e-5 if out_dtype == torch.float32 else 8e-3) * ref.abs().max().item()
    again = _linear(x, w, groups, out_dtype, kernel=2)
    assert torch.equal(out, again)
    if m > 64:  # the automatic choice is this kernel
        assert torch.equal(out, _linear(x, w, groups, out_dtype, kernel=0))
    old = _linear(x, w, groups, out_dtype, kernel=1)
    assert rel_rms(out, old) < (1e-5 if out_dtype == torch.float32 else 4e-3)


def test_tcgen05_rows_do_not_depend_on_m(dsv4):
    """A row's result is the same bits whether it is computed among 1,000 rows or 129 (the
    sharded prefill's slices rely on it; slices of 64 rows or fewer run the weight-streaming
    kernel instead)."""
    x, w, _ = _operands(1000, 768, 1024, 1, 5)
    full = _linear(x, w, 1, torch.float32, kernel=0)
    part = _linear(x[300:429].contiguous(), w, 1, torch.float32, kernel=0)
    assert torch.equal(full[300:429], part)
    tail = _linear(x[872:].contiguous(), w, 1, torch.float32, kernel=0)
    assert torch.equal(full[872:], tail)


def test_tcgen05_multi_one_launch(dsv4):
    """Several projections of one x in one tcgen05 launch (ragged widths): each output equals its
    own dsv4.linear bit for bit and is close to the fp64 product."""
    g = torch.Generator().manual_seed(11)
    m, k = 300, 1024
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(DEV)
    ns = [1024, 512, 64, 256, 130]
    Ws = [(torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16).to(DEV) for n in ns]
    outs = dsv4.linear_multi(x, Ws)
    for o, W in zip(outs, Ws):
        ref = x.double() @ W.double().T
        assert rel_rms(o, ref) < 1e-5
        assert torch.equal(o, dsv4.linear(x, W))


def test_compressor_projections_share_one_launch(dsv4):
    """compressor_prefill at prefill size runs both projections in one tcgen05 launch; its rows
    equal those of the two separate projections (same kernel, same summation order)."""
    from oracle import compressor_ref as C
    g = torch.Generator().manual_seed(12)
    s, dim, hd = 512, 1024, 512
    x = (torch.randn(1, s, dim, generator=g)).to(torch.bfloat16)
    wkv = (torch.randn(2 * hd, dim, generator=g) * 0.03).to(torch.bfloat16)
    wgate = (torch.randn(2 * hd, dim, generator=g) * 0.03).to(torch.bfloat16)
    ape = torch.randn(4, 2 * hd, generator=g) * 0.1
    nw = 1 + 0.1 * torch.randn(hd, generator=g)
    out, _ = dsv4.compressor_prefill(x.to(DEV), wkv.to(DEV), wgate.to(DEV), ape.to(DEV), nw.to(DEV))
    ref, _ = C.compressor_prefill(x.float(), wkv.float(), wgate.float(), ape, nw)
    assert rel_rms(out, ref) < 1e-4
