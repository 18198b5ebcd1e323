"""The ctypes mirrors of the C ABI structs match include/dsv4.h field for field (offsets and sizes),
checked by compiling a small C program against the header with the host compiler."""
import ctypes
import importlib
import os
import shutil
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
L = importlib.import_module("deepseek-v4-flash-mlx_b200._lib")

PAIRS = {
    "dsv4_sparse_attn_params": L.SparseAttnParams,
    "dsv4_rmsnorm_params": L.RmsNormParams,
    "dsv4_rope_params": L.RopeParams,
    "dsv4_norm_rope_params": L.NormRopeParams,
    "dsv4_indexer_params": L.IndexerParams,
    "dsv4_compressor_params": L.CompressorParams,
    "dsv4_compressor_decode_params": L.CompressorDecodeParams,
    "dsv4_linear_params": L.LinearParams,
    "dsv4_decode_rows_params": L.DecodeRowsParams,
    "dsv4_linear_out": L.LinearOut,
    "dsv4_linear_multi_params": L.LinearMultiParams,
    "dsv4_key_image_params": L.KeyImageParams,
    "dsv4_hc_params": L.HcParams,
}


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs a host C compiler")
def test_struct_layouts_match_header():
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "dsv4.h"', "int main(void) {"]
    for cname, py in PAIRS.items():
        lines.append(f'  printf("{cname} sizeof %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'  printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines.append("  return 0;\n}")
    with tempfile.TemporaryDirectory() as d:
        src, exe = os.path.join(d, "layout.c"), os.path.join(d, "layout")
        open(src, "w").write("\n".join(lines))
        subprocess.run(["gcc", "-std=c11", "-I", os.path.join(ROOT, "include"), src, "-o", exe], check=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout.split("\n")
    got = {}
    for ln in out:
        if ln:
            c, f, v = ln.split()
            got[(c, f)] = int(v)
    for cname, py in PAIRS.items():
        assert got[(cname, "sizeof")] == ctypes.sizeof(py), cname
        for fname, _ in py._fields_:
            assert got[(cname, fname)] == getattr(py, fname).offset, (cname, fname)
