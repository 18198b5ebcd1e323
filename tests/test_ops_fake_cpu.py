"""Every dsv4 custom op has a fake (shape-only) implementation, so FakeTensor tracing (torch.compile,
torch.export) sees each op as one opaque call. Runs on the CPU: the public wrappers are called on
fake CUDA tensors, which never reach libdsv4.so."""
import importlib

import torch
from torch._subclasses.fake_tensor import FakeTensorMode

PKG = "deepseek-v4-flash-mlx_b200"


def _e(*shape, dtype=torch.float32):
    return torch.empty(*shape, dtype=dtype, device="cuda")


def test_every_dsv4_op_has_a_fake():
    importlib.import_module(PKG)
    from torch._library.simple_registry import singleton
    for name in ("sparse_attn", "indexer_topk", "compressor_prefill", "compressor_decode_step", "compressor_decode_pair",
                 "decode_attention",
                 "linear", "linear_multi", "rmsnorm", "norm_rope", "rope_positions", "apply_rotary_emb",
                 "get_window_topk_idxs"):
        assert hasattr(torch.ops.dsv4, name), name
        assert singleton.find(f"dsv4::{name}").fake_impl.kernel is not None, name


def test_wrappers_trace_on_fake_tensors():
    dsv4 = importlib.import_module(PKG)
    D = importlib.import_module(PKG + ".decode")
    with FakeTensorMode():
        x = _e(1, 64, 4096, dtype=torch.bfloat16)
        w = _e(1024, 4096, dtype=torch.bfloat16)
        comp, state = dsv4.compressor_prefill(x, w, w, _e(4, 1024), _e(512), out_dtype=torch.bfloat16)
        assert comp.shape == (1, 16, 512) and comp.dtype == torch.bfloat16
        assert state["ring_kv"].shape == (1, 8, 1024) and state["kv"].shape == (1, 4, 1024)
        _, st2 = dsv4.compressor_prefill(_e(1, 66, 4096), w, w, _e(4, 1024), _e(512))
        assert st2["kv_rem"].shape == (1, 2, 1024)

        o = dsv4.sparse_attn(_e(10, 64, 512, dtype=torch.bfloat16), _e(100, 512, dtype=torch.bfloat16), _e(64),
                             torch.empty(10, 40, dtype=torch.int32, device="cuda"), 512 ** -0.5)
        assert o.shape == (10, 64, 512) and o.dtype == torch.bfloat16

        sel = dsv4.indexer_topk(_e(1, 5, 64, 128), _e(1, 5, 64), _e(1, 300, 128), 32)
        assert sel.shape == (1, 5, 32) and sel.dtype == torch.int32

        cache = D.SparseMLACache(2, 512, device="cuda")
        b = 2
        pos = torch.empty(b, dtype=torch.int32, device="cuda")
        dsv4.compressor_decode_step(_e(b, 4096), w, w, _e(4, 1024), _e(512), cache.ring_kv, cache.ring_score, pos,
                                    cache.kv_pool, torch.empty(b, dtype=torch.int64, device="cuda"), freqs=_e(32),
                                    proj=(_e(b, 1024), _e(b, 1024)))
        ib = torch.empty(b, dtype=torch.int64, device="cuda")
        dsv4.compressor_decode_pair(
            dsv4.CompressorStep((_e(b, 1024), _e(b, 1024)), _e(4, 1024), _e(512), cache.ring_kv, cache.ring_score,
                                cache.kv_pool, ib, 512),
            dsv4.CompressorStep((_e(b, 256), _e(b, 256)), _e(4, 256), _e(128), cache.ring_k_idx, cache.ring_s_idx,
                                cache.k_idx.view(-1, 128), ib, 128, key_image=(*cache.key_image, cache.max_comp)),
            pos, freqs=_e(32))
        o = dsv4.decode_attention(cache, _e(b, 64, 512), _e(b, 64, 128), _e(b, 64), _e(64), pos, 128, freqs=_e(32))
        assert o.shape == (b, 64, 512) and o.dtype == torch.bfloat16

