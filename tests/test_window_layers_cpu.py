"""Window-only layers (ratio 0 and 128) without a GPU: the RoPE table each ratio uses, the oracle's
window attention against its compressed-layer attention with nothing visible, the window-only cache
and the row-bookkeeping entry point's host-side checks."""
import ctypes
import importlib
import os

import numpy as np
import pytest
import torch

from oracle import layer_ref as LR

PKG = "deepseek-v4-flash-mlx_b200"
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_torch_golden.npz")


def test_layer_rope_tables_are_the_references():
    """Ratio 0 uses the plain base-10000 table, ratios 4 and 128 the YaRN table
    (oracle/decode_engine.py:47, 73); both pinned to ref_torch's precompute_freqs outputs."""
    g = np.load(GOLDEN)
    C = importlib.import_module(PKG + ".configs")
    Lm = importlib.import_module(PKG + ".layer")
    np.testing.assert_array_equal(LR.layer_freqs(0).numpy(), g["freqs_plain"])
    np.testing.assert_array_equal(LR.layer_freqs(128).numpy(), g["freqs_yarn"])
    np.testing.assert_array_equal(LR.layer_freqs(4).numpy(), g["freqs_yarn"])
    np.testing.assert_array_equal(Lm.layer_rope_freqs(C.LayerDims(ratio=0), "cpu").numpy(), g["freqs_plain"])
    np.testing.assert_array_equal(Lm.layer_rope_freqs(C.LayerDims(ratio=128), "cpu").numpy(), g["freqs_yarn"])
    assert C.window_only(C.LayerDims(ratio=0)) and C.window_only(C.LayerDims(ratio=128))
    assert not C.window_only(C.LayerDims())


def test_window_attention_ref_equals_attention_with_nothing_visible():
    """With no compressed row visible the compressed layer's list is the window plus masked
    entries, which add nothing: the two oracle paths agree bit for bit."""
    g = torch.Generator().manual_seed(3)
    b, n = 3, 3 * 128
    pool = torch.randn(n, 512, generator=g).bfloat16().float()
    win_base = torch.arange(b) * 128
    q = torch.randn(b, 64, 512, generator=g)
    sink = torch.randn(64, generator=g)
    pos = torch.tensor([3, 127, 400])
    f = LR.layer_freqs(128)
    a = LR.window_attention_ref(pool, win_base, q, sink, pos, f)
    k_idx = torch.zeros(b, 0, 128)
    bref = LR.decode_attention_ref(pool, win_base, lambda bb, j: j, k_idx, q, torch.randn(b, 64, 128, generator=g),
                                   torch.randn(b, 64, generator=g), sink, pos, 8, f)
    assert torch.equal(a, bref)


def test_window_only_cache_and_block_checks():
    D = importlib.import_module(PKG + ".decode")
    C = importlib.import_module(PKG + ".configs")
    Lm = importlib.import_module(PKG + ".layer")
    c = D.SparseMLACache(2, 0, device="cpu")
    assert not c.compressed and c.k_idx is None and c.ring_kv is None
    assert c.kv_pool.shape == (256, 512) and c.block_table.shape == (2, 0)
    W = Lm.make_attention_weights(0, dims=C.LayerDims(dim=256, ratio=128))
    with pytest.raises(ValueError):
        Lm.DecodeBlock(W, 2, 1024, dims=C.LayerDims(dim=256, ratio=128), device="cpu",
                       cache=D.SparseMLACache(2, 16, device="cpu"))


def test_decode_rows_window_only_validation(dsv4):
    """dsv4_decode_rows: a window-only cache (max_comp 0) needs no block table; a cache with
    compressed rows still does. Only the host-side checks run here."""
    L = importlib.import_module(PKG + "._lib")
    lib = dsv4.library()
    p = L.DecodeRowsParams()
    p.positions = p.win_base = p.win_rows = p.comp_rows = p.key_rows = ctypes.c_void_p(256)
    p.b, p.window, p.ratio, p.page, p.bt_stride, p.max_comp = 1, 128, 4, 64, 1, 64
    assert lib.dsv4_decode_rows(ctypes.byref(p), None) == 1
    assert b"NULL" in lib.dsv4_last_error()
    p.max_comp, p.window = 0, 0
    assert lib.dsv4_decode_rows(ctypes.byref(p), None) == 1
    assert b"bad sizes" in lib.dsv4_last_error()
    p.b = 0
    p.window = 128
    assert lib.dsv4_decode_rows(ctypes.byref(p), None) == 0  # empty batch: nothing launched


def test_decode_runner_refuses_window_only_cache():
    D = importlib.import_module(PKG + ".decode")
    with pytest.raises(ValueError, match="window-only"):
        D.DecodeRunner(D.SparseMLACache(2, 0, device="cpu"), torch.zeros(64), device="cpu")
