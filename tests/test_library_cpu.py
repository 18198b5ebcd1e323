"""The C ABI library without a GPU: loads, exports every declared symbol, validates arguments."""
import ctypes
import os
import re

import pytest

from conftest import ROOT


def _declared():
    src = open(os.path.join(ROOT, "include", "dsv4.h")).read()
    return sorted(set(re.findall(r"DSV4_API\s+[\w\s\*]+?\b(dsv4_\w+)\s*\(", src)))


def test_header_and_binding_agree(dsv4):
    from importlib import import_module
    L = import_module("deepseek-v4-flash-mlx_b200._lib")
    assert _declared() == sorted(L.SIGNATURES), "include/dsv4.h and the ctypes binding list differ"


def test_library_exports_every_symbol(dsv4):
    lib = dsv4.library()
    for name in _declared():
        assert hasattr(lib, name), name
    assert lib.dsv4_abi_version() == 1


def test_argument_validation_without_gpu(dsv4):
    """Shape/dtype checks run on the host before any CUDA call and return a status + message."""
    from importlib import import_module
    L = import_module("deepseek-v4-flash-mlx_b200._lib")
    lib = dsv4.library()
    p = L.SparseAttnParams()
    assert lib.dsv4_sparse_attn(ctypes.byref(p), None) == 1
    assert b"NULL" in lib.dsv4_last_error()
    p.q = p.kv = p.sink = p.idx = p.out = ctypes.c_void_p(16)
    p.d, p.h, p.s, p.t, p.n = 256, 64, 1, 8, 10
    assert lib.dsv4_sparse_attn(ctypes.byref(p), None) == 1
    assert b"head dim" in lib.dsv4_last_error()
    p.d, p.q_dtype = 512, 3
    assert lib.dsv4_sparse_attn(ctypes.byref(p), None) == 2  # unsupported q dtype
    ip = L.IndexerParams()
    ip.q = ip.w = ip.k = ip.out = ctypes.c_void_p(16)
    ip.heads, ip.batch, ip.s, ip.n_keys, ip.top_k, ip.out_stride = 32, 1, 1, 10, 4, 4
    assert lib.dsv4_indexer_topk(ctypes.byref(ip), None) == 1
    ip.heads = 64
    assert lib.dsv4_indexer_topk(ctypes.byref(ip), None) == 6  # workspace missing
    lp = L.LinearParams()
    lp.x = lp.w = lp.y = ctypes.c_void_p(16)
    lp.m, lp.n, lp.k, lp.groups, lp.x_dtype, lp.w_dtype = 4, 8, 100, 1, 1, 1
    assert lib.dsv4_linear(ctypes.byref(lp), None) == 1
    assert b"multiple of 64" in lib.dsv4_last_error()
    lp.m, lp.k, lp.kernel = 0, 128, 3  # kernel choices are 0, 1, 2
    assert lib.dsv4_linear(ctypes.byref(lp), None) == 1
    assert b"kernel=3" in lib.dsv4_last_error()
    lp.kernel, lp.w_dtype, lp.w_scale, lp.group = 2, L.I8, ctypes.c_void_p(16), 64
    assert lib.dsv4_linear(ctypes.byref(lp), None) == 1  # the tcgen05 kernel takes bf16 weights
    assert b"bf16 weights" in lib.dsv4_last_error()


def test_ops_refuse_cpu_tensors(dsv4):
    import torch
    q = torch.zeros(1, 64, 512)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        dsv4.sparse_attn(q, torch.zeros(4, 512), torch.zeros(64), torch.zeros(1, 4, dtype=torch.long), 0.1)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        dsv4.rmsnorm(q, torch.ones(512))


def test_yarn_table_matches_reference_formula(dsv4, golden):
    import numpy as np
    lib = dsv4.library()
    f = (ctypes.c_float * 32)()
    assert lib.dsv4_yarn_freqs(64, 65536, 160000.0, 16.0, 32.0, 1.0, f) == 0
    np.testing.assert_array_equal(np.array(list(f), dtype=np.float32), golden["freqs_yarn"])
    np.testing.assert_array_equal(dsv4.precompute_freqs(64, 0, 65536, 160000.0, 16, 32, 1).numpy(),
                                  golden["freqs_yarn"])
    np.testing.assert_array_equal(dsv4.precompute_freqs(64, 0, 0, 10000.0, 40, 32, 1).numpy(), golden["freqs_plain"])
