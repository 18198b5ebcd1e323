"""The failure path on the GPU, without a fault: a bounded wait runs out, the kernel records the
timeout on the device error word and returns, the host reads the status, and the context keeps
running kernels."""
import ctypes
import importlib
import time

import pytest
import torch

from helpers import assert_close_bf16
from oracle import sparse_attn_ref as SAR

pytestmark = pytest.mark.gpu
PKG = "deepseek-v4-flash-mlx_b200"


def test_wait_timeout_reported_and_context_usable(dsv4):
    L = importlib.import_module(PKG + "._lib")
    torch.cuda.init()
    assert L.device_error() == 0  # nothing pending from earlier calls (the read also clears it)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    t0 = time.perf_counter()
    L.check(L.lib().dsv4_selftest_wait_timeout(stream))
    code = L.device_error()
    dt = time.perf_counter() - t0
    assert L.STATUS[code] == "WAIT_TIMEOUT"
    assert 0.5 < dt < 30, dt  # the wait's limit is 1 s of %globaltimer
    assert L.device_error() == 0  # read once, then cleared
    # the context still runs the library's kernels, with correct results
    g = torch.Generator().manual_seed(5)
    q = torch.randn(3, 64, 512, generator=g)
    kv = torch.randn(500, 512, generator=g).to(torch.bfloat16).float()
    sink = torch.randn(64, generator=g)
    idx = torch.randint(-1, 500, (3, 200), generator=g)
    out = dsv4.sparse_attn(q.cuda(), kv.cuda(), sink.cuda(), idx.cuda(), 512 ** -0.5)
    assert_close_bf16(out, SAR.sparse_attn(q, kv, sink, idx, 512 ** -0.5), what="attention after a timeout")
    assert L.device_error() == 0
