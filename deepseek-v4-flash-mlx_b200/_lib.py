"""ctypes binding of libdsv4.so (the C ABI declared in include/dsv4.h).

This module is the only place that touches the shared library. It fails loudly: if libdsv4.so
is missing (and cannot be built here) every op raises; there is no CPU or PyTorch fallback.
"""
import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdsv4.so")

F32, BF16, I32, I64, I8 = 0, 1, 2, 3, 4
_DTYPE = {torch.float32: F32, torch.bfloat16: BF16, torch.int32: I32, torch.int64: I64,
          torch.int8: I8}

STATUS = {0: "OK", 1: "INVALID_ARGUMENT", 2: "UNSUPPORTED_DTYPE", 3: "CUDA", 4: "INDEX_OUT_OF_RANGE",
          5: "WAIT_TIMEOUT", 6: "WORKSPACE"}

vp, i32, i64, f32, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t


class SparseAttnParams(ctypes.Structure):
    _fields_ = [("q", vp), ("kv", vp), ("sink", vp), ("idx", vp), ("out", vp),
                ("s", i64), ("n", i64), ("h", i32), ("d", i32), ("t", i32),
                ("q_dtype", i32), ("idx_dtype", i32), ("out_dtype", i32), ("scale", f32),
                ("rope_freqs", vp), ("positions", vp), ("rope_dim", i32), ("num_splits", i32),
                ("workspace", vp), ("workspace_bytes", sz), ("q_norm_rope", i32), ("q_eps", f32),
                ("win_base", vp), ("win_stride", i32), ("window", i32), ("window_linear", i32),
                ("kernel", i32), ("pre_wait", i32)]


class RmsNormParams(ctypes.Structure):
    _fields_ = [("x", vp), ("weight", vp), ("out", vp), ("rows", i64), ("dim", i32),
                ("x_dtype", i32), ("w_dtype", i32), ("out_dtype", i32), ("eps", f32)]


class RopeParams(ctypes.Structure):
    _fields_ = [("x", vp), ("out", vp), ("s", i64), ("heads", i32), ("dim", i32), ("rope_dim", i32),
                ("x_dtype", i32), ("out_dtype", i32), ("cis", vp), ("cis_rows", i64), ("freqs", vp),
                ("positions", vp),
                ("pos_offset", i32), ("inverse", i32)]


class NormRopeParams(ctypes.Structure):
    _fields_ = [("x", vp), ("weight", vp), ("out", vp), ("out_rows", vp), ("rows", i64),
                ("heads", i32), ("dim", i32), ("rope_dim", i32), ("x_dtype", i32), ("w_dtype", i32),
                ("out_dtype", i32), ("eps", f32), ("freqs", vp), ("positions", vp), ("act_quant", i32)]


class IndexerParams(ctypes.Structure):
    _fields_ = [("q", vp), ("w", vp), ("k", vp), ("out", vp), ("scores_out", vp),
                ("batch", i32), ("s", i32), ("heads", i32), ("n_keys", i32), ("top_k", i32),
                ("k_batch_stride", i64), ("positions", vp), ("ratio", i32),
                ("out_stride", i32), ("out_col", i32), ("out_offset", i64),
                ("block_table", vp), ("table_stride", i32), ("page", i32),
                ("workspace", vp), ("workspace_bytes", sz), ("win_base", vp), ("window", i32),
                ("window_linear", i32), ("mode", i32), ("key_image", vp), ("key_inv", vp), ("key_norm_max", vp)]


KEY_TILE_BYTES = 65536


class KeyImageParams(ctypes.Structure):
    _fields_ = [("k", vp), ("batch", i32), ("n_keys", i32), ("k_batch_stride", i64), ("image", vp), ("inv", vp),
                ("norm_max", vp)]


class CompressorParams(ctypes.Structure):
    _fields_ = [("kv", vp), ("score", vp), ("ape", vp), ("norm_w", vp), ("out", vp), ("out_rows", vp),
                ("b", i32), ("s", i32), ("head_dim", i32), ("ratio", i32), ("rope_dim", i32),
                ("norm_dtype", i32), ("out_dtype", i32), ("eps", f32), ("freqs", vp), ("pos0", i32),
                ("ring_kv", vp), ("ring_score", vp), ("act_quant", i32)]


class CompressorDecodeParams(ctypes.Structure):
    _fields_ = [("kv", vp), ("score", vp), ("ape", vp), ("norm_w", vp), ("ring_kv", vp),
                ("ring_score", vp), ("positions", vp), ("out", vp), ("out_rows", vp),
                ("b", i32), ("head_dim", i32), ("ratio", i32), ("rope_dim", i32),
                ("norm_dtype", i32), ("out_dtype", i32), ("eps", f32), ("freqs", vp),
                ("key_image", vp), ("key_inv", vp), ("key_norm_max", vp), ("image_stride", i64),
                ("act_quant", i32)]


class LinearParams(ctypes.Structure):
    _fields_ = [("x", vp), ("w", vp), ("w_scale", vp), ("y", vp), ("m", i64), ("n", i32), ("k", i32),
                ("groups", i32), ("group", i32), ("x_dtype", i32), ("w_dtype", i32), ("y_dtype", i32),
                ("workspace", vp), ("workspace_bytes", sz), ("kernel", i32)]


class HcParams(ctypes.Structure):
    _fields_ = [("x", vp), ("fn", vp), ("scale", vp), ("base", vp), ("y", vp), ("post", vp), ("comb", vp),
                ("norm_w", vp), ("y_norm", vp), ("workspace", vp), ("workspace_bytes", ctypes.c_size_t), ("rows", i64), ("hc", i32), ("dim", i32), ("sinkhorn_iters", i32),
                ("head", i32), ("norm_dtype", i32), ("y_norm_dtype", i32), ("norm_eps", f32), ("hc_eps", f32),
                ("y_norm_eps", f32)]


LINEAR_MULTI_MAX = 8


class LinearOut(ctypes.Structure):
    _fields_ = [("w", vp), ("w_scale", vp), ("y", vp), ("n", i32), ("y_dtype", i32)]


class LinearMultiParams(ctypes.Structure):
    _fields_ = [("x", vp), ("m", i64), ("k", i32), ("group", i32), ("x_dtype", i32), ("w_dtype", i32),
                ("count", i32), ("outs", LinearOut * LINEAR_MULTI_MAX), ("kernel", i32)]


class DecodeRowsParams(ctypes.Structure):
    _fields_ = [("positions", vp), ("win_base", vp), ("block_table", vp), ("win_rows", vp), ("comp_rows", vp),
                ("key_rows", vp), ("comp_base", i64), ("b", i32), ("window", i32), ("ratio", i32), ("page", i32),
                ("bt_stride", i32), ("max_comp", i32)]


# every symbol include/dsv4.h declares, with its ctypes signature
SIGNATURES = {
    "dsv4_last_error": (ctypes.c_char_p, []),
    "dsv4_abi_version": (ctypes.c_int, []),
    "dsv4_device_error": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int), vp]),
    "dsv4_selftest_wait_timeout": (ctypes.c_int, [vp]),
    "dsv4_sparse_attn_workspace_size": (sz, [ctypes.POINTER(SparseAttnParams)]),
    "dsv4_sparse_attn": (ctypes.c_int, [ctypes.POINTER(SparseAttnParams), vp]),
    "dsv4_window_topk_idxs": (ctypes.c_int, [i32, i32, i32, i32, vp, vp]),
    "dsv4_rmsnorm": (ctypes.c_int, [ctypes.POINTER(RmsNormParams), vp]),
    "dsv4_rope": (ctypes.c_int, [ctypes.POINTER(RopeParams), vp]),
    "dsv4_norm_rope": (ctypes.c_int, [ctypes.POINTER(NormRopeParams), vp]),
    "dsv4_yarn_freqs": (ctypes.c_int, [i32, i64, ctypes.c_double, ctypes.c_double, ctypes.c_double,
                                       ctypes.c_double, ctypes.POINTER(ctypes.c_float)]),
    "dsv4_indexer_topk_workspace_size": (sz, [ctypes.POINTER(IndexerParams)]),
    "dsv4_indexer_topk": (ctypes.c_int, [ctypes.POINTER(IndexerParams), vp]),
    "dsv4_indexer_topk_noalloc": (ctypes.c_int, [ctypes.POINTER(IndexerParams), vp]),
    "dsv4_decode_window_indices": (ctypes.c_int, [i32, i32, vp, vp, vp, i32, vp]),
    "dsv4_compressor_pool": (ctypes.c_int, [ctypes.POINTER(CompressorParams), vp]),
    "dsv4_compressor_decode": (ctypes.c_int, [ctypes.POINTER(CompressorDecodeParams), vp]),
    "dsv4_compressor_decode_pair": (ctypes.c_int, [ctypes.POINTER(CompressorDecodeParams),
                                                   ctypes.POINTER(CompressorDecodeParams), vp]),
    "dsv4_decode_rows": (ctypes.c_int, [ctypes.POINTER(DecodeRowsParams), vp]),
    "dsv4_hc_pre": (ctypes.c_int, [ctypes.POINTER(HcParams), vp]),
    "dsv4_hc_workspace_size": (ctypes.c_size_t, [i64, i32, i32, i32]),
    "dsv4_hc_post": (ctypes.c_int, [vp, vp, vp, vp, vp, i64, i32, i32, vp]),
    "dsv4_indexer_key_image": (ctypes.c_int, [ctypes.POINTER(KeyImageParams), vp]),
    "dsv4_linear_workspace_size": (sz, [ctypes.POINTER(LinearParams)]),
    "dsv4_linear": (ctypes.c_int, [ctypes.POINTER(LinearParams), vp]),
    "dsv4_linear_multi": (ctypes.c_int, [ctypes.POINTER(LinearMultiParams), vp]),
    "dsv4_cast": (ctypes.c_int, [vp, i32, vp, i32, i64, vp]),
    "dsv4_copy": (ctypes.c_int, [vp, vp, sz, vp]),
    "dsv4_copy_beside": (ctypes.c_int, [vp, vp, sz, vp]),
}

_lib = None


def load(path=LIB_PATH):
    """Load libdsv4.so once. Raises RuntimeError when it is absent or incomplete."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(
            f"libdsv4.so not found at {path}: build it with the package's build.py "
            "(nvcc for sm_100a); the dsv4 ops have no fallback")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)  # AttributeError if a declared symbol is missing
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def lib():
    return load()


class Dsv4Error(RuntimeError):
    def __init__(self, status, msg):
        super().__init__(f"dsv4 {STATUS.get(status, status)}: {msg}")
        self.status = status


def check(status):
    if status != 0:
        msg = lib().dsv4_last_error()
        raise Dsv4Error(status, msg.decode() if msg else "")


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def dtype_code(t):
    try:
        return _DTYPE[t.dtype]
    except KeyError:
        raise TypeError(f"dsv4: unsupported dtype {t.dtype}") from None


def stream_of(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("dsv4 ops run on CUDA tensors only (no CPU fallback)")


def workspace(nbytes, device):
    if nbytes == 0:
        return None
    return torch.empty(int(nbytes), dtype=torch.uint8, device=device)


def device_error(stream=None):
    """Synchronise and return (and clear) the device error word: 0 or a status code."""
    code = ctypes.c_int(0)
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream if stream is None else stream)
    check(lib().dsv4_device_error(ctypes.byref(code), s))
    return code.value


def copy_beside_(dst, src, stream=None):
    """dst <- src as `copy_`, overlapped with the kernel launched before it (dsv4_copy_beside)."""
    nbytes = src.numel() * src.element_size()
    if dst.numel() * dst.element_size() != nbytes or not (dst.is_contiguous() and src.is_contiguous()):
        raise ValueError("dsv4 copy_beside_: contiguous tensors of the same size in bytes")
    s = stream if stream is not None else ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    check(lib().dsv4_copy_beside(ptr(dst), ptr(src), nbytes, s))
    return dst


def copy_(dst, src, stream=None):
    """dst <- src (same number of bytes, contiguous, 16-byte aligned; device or pinned host tensors)
    by a kernel on the current stream (dsv4_copy)."""
    nbytes = src.numel() * src.element_size()
    if dst.numel() * dst.element_size() != nbytes or not (dst.is_contiguous() and src.is_contiguous()):
        raise ValueError("dsv4 copy_: contiguous tensors of the same size in bytes")
    s = stream if stream is not None else ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    check(lib().dsv4_copy(ptr(dst), ptr(src), nbytes, s))
    return dst
