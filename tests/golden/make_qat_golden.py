"""Generate tests/golden/qat_golden.npz from the reference's own code on seeded inputs.

Run where a checkout of the reference project is available:
    python tests/golden/make_qat_golden.py <reference checkout>
Recorded (inputs included), for tests/test_oracle_golden.py and the GPU parity tests:
  * `aq` (oracle/decode_engine.py:52-54), the fp8-e4m3 act-quant simulation of cached rows; the
    module imports mlx, so the function is taken from the file's syntax tree and run alone with
    numpy and ml_dtypes;
  * `hadamard_rotate` and `fp4_act_quant` (v4mlx/qat.py:8-31), the indexer-key simulation;
  * `hc_pre`, `hc_post`, `hc_head` (ref_torch/hc.py:18-80), the hyper-connection mixes.
"""
import ast
import os
import sys

import numpy as np
import torch

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "qat_golden.npz")


def _function_from_file(path, name, env):
    tree = ast.parse(open(path).read())
    node = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == name)
    code = compile(ast.Module(body=[node], type_ignores=[]), path, "exec")
    exec(code, env)
    return env[name]


def main(ref_root):
    sys.path.insert(0, ref_root)
    import ml_dtypes
    from ref_torch import hc as HC
    from v4mlx import qat as Q

    g = {}
    aq = _function_from_file(os.path.join(ref_root, "oracle", "decode_engine.py"), "aq",
                             {"np": np, "ml_dtypes": ml_dtypes})
    rng = np.random.default_rng(20)
    x = rng.standard_normal((8, 448)).astype(np.float32)
    x *= np.float32(10.0) ** rng.integers(-6, 4, size=(8, 1)).astype(np.float32)   # 1e-6 .. 1e3 per row
    x[0, :64] = 0.0                                                                 # an all-zero block
    x[1, 64:128] = np.float32(448.0) * np.float32(2.0) ** np.arange(-3, 61, dtype=np.float32)[:64] / 2 ** 60
    g["aq_x"], g["aq_y"] = x, aq(x, 64).astype(np.float32)

    k = rng.standard_normal((6, 128)).astype(np.float32)
    g["fp4_x"] = k
    g["had_y"] = Q.hadamard_rotate(k).astype(np.float32)
    g["fp4_y"] = Q.fp4_act_quant(Q.hadamard_rotate(k), 32).astype(np.float32)

    tg = torch.Generator().manual_seed(21)
    b, s, hc, dim = 1, 3, 4, 256
    xh = torch.randn(b, s, hc, dim, generator=tg)
    hc_fn = torch.randn(24, hc * dim, generator=tg) * 0.02
    hc_scale = torch.rand(3, generator=tg) + 0.5
    hc_base = torch.randn(24, generator=tg) * 0.1
    y, post, comb = HC.hc_pre(xh, hc_fn, hc_scale, hc_base)
    att = torch.randn(b, s, dim, generator=tg)
    yp = HC.hc_post(att, xh, post, comb)
    head_fn = torch.randn(hc, hc * dim, generator=tg) * 0.02
    head_scale = torch.rand(1, generator=tg) + 0.5
    head_base = torch.randn(hc, generator=tg) * 0.1
    yh = HC.hc_head(xh, head_fn, head_scale, head_base)
    for key, t in dict(hc_x=xh, hc_fn=hc_fn, hc_scale=hc_scale, hc_base=hc_base, hc_y=y, hc_post=post, hc_comb=comb,
                       hc_att=att, hc_post_y=yp, hc_head_fn=head_fn, hc_head_scale=head_scale, hc_head_base=head_base,
                       hc_head_y=yh).items():
        g[key] = t.numpy().astype(np.float32)
    np.savez_compressed(OUT, **g)
    print("wrote", OUT, sorted(g))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_qat_golden.py <reference checkout>")
    main(sys.argv[1])
