"""Oracle: ctypes wrapper of indexer_canon.c (test infrastructure only).

build_oracle() compiles the C restatement with gcc into oracle/_build/ (git-ignored); the built
.so travels with the repository snapshot to the GPU box like the library itself.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "indexer_canon.c")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(BUILD, "libdsv4_oracle.so")
CFLAGS = ["-O2", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-shared", "-fPIC", "-std=c11"]

_lib = None


def build_oracle(force=False):
    os.makedirs(BUILD, exist_ok=True)
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        subprocess.run(["gcc", *CFLAGS, SRC, "-o", LIB, "-lm"], check=True)
    return LIB


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build_oracle()
        lib = ctypes.CDLL(LIB)
        P = ctypes.c_void_p
        lib.dsv4_oracle_scores.argtypes = [P, P, P, ctypes.c_int64, P]
        lib.dsv4_oracle_select.argtypes = [P, ctypes.c_int64, ctypes.c_int32, P]
        lib.dsv4_oracle_indexer_topk.argtypes = [P, P, P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, P,
                                                 ctypes.c_int32, P]
        _lib = lib
    return _lib


def _f32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def scores(q, w, keys):
    """q [64,128], w [64], keys [n,128] -> fp32 [n] in the canonical order."""
    q, w, keys = _f32(q), _f32(w), _f32(keys)
    out = np.empty(keys.shape[0], dtype=np.float32)
    _load().dsv4_oracle_scores(q.ctypes.data, w.ctypes.data, keys.ctypes.data, keys.shape[0], out.ctypes.data)
    return out


def select(scores_, top_k):
    s = _f32(scores_)
    out = np.empty(top_k, dtype=np.int32)
    _load().dsv4_oracle_select(s.ctypes.data, s.shape[0], top_k, out.ctypes.data)
    return out


def indexer_topk(q, w, keys, top_k, positions=None, ratio=4):
    """q [b,s,64,128], w [b,s,64], keys [b,n,128] -> int32 [b,s,top_k] (ascending, -1 padded)."""
    q, w, keys = _f32(q), _f32(w), _f32(keys)
    b, s = q.shape[0], q.shape[1]
    n = keys.shape[1]
    if positions is None:
        nvis = np.full(b * s, n, dtype=np.int32)
    else:
        nvis = np.minimum((np.asarray(positions, dtype=np.int64).reshape(-1) + 1) // ratio, n).astype(np.int32)
    out = np.empty((b, s, top_k), dtype=np.int32)
    _load().dsv4_oracle_indexer_topk(q.ctypes.data, w.ctypes.data, keys.ctypes.data, b, s, n, nvis.ctypes.data,
                                     top_k, out.ctypes.data)
    return out


def scores_f64(q, w, keys):
    """Independent float64 evaluation of the same formula (sanity check of the fp32 order)."""
    q, w, keys = np.asarray(q, np.float64), np.asarray(w, np.float64), np.asarray(keys, np.float64)
    dots = keys @ q.T                                  # [n, 64]
    return (np.maximum(dots, 0.0) * w[None, :]).sum(-1)
