"""Generate tests/golden/decode_attention_golden.npz: the reference's own decode attention on seeded
inputs, for a compressing (ratio 4) and a window-only layer.

Run where a checkout of the reference project is available:
    python tests/golden/make_decode_attention_golden.py <reference checkout>
The decode attention is inline code of `layer_step` (oracle/v4_fast.py:108-119): the window rows in
ring order plus every visible compressed row (none when the layer does not compress), the MLX
`sparse_attn`, and the inverse RoPE of the output. Those statements are taken from the file's syntax
tree and run alone, on numpy, with the MLX twins (v4mlx/sparse_attn.py, v4mlx/norm_rope.py) loaded
under the stand-in for mlx.core of make_mla_golden.py. q is prepared as layer_step does before them
(oracle/v4_fast.py:88-89: the per-head norm and the RoPE of v4mlx). Recorded (inputs included): the
raw q, the window ring, the compressed rows, the sinks, positions and the outputs.
"""
import ast
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "decode_attention_golden.npz")
SRC = os.path.join("oracle", "v4_fast.py")


def _attention_statements(path):
    """layer_step's statements from `wlo = ...` to the inverse-RoPE assignment of `o`."""
    tree = ast.parse(open(path).read())
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "layer_step")
    body = fn.body
    start = next(i for i, n in enumerate(body) if isinstance(n, ast.Assign) and ast.unparse(n.targets[0]) == "wlo")
    end = next(i for i, n in enumerate(body) if i > start and isinstance(n, ast.Assign)
               and ast.unparse(n.targets[0]) == "o" and "apply_rotary_emb" in ast.unparse(n.value))
    return compile(ast.Module(body=body[start:end + 1], type_ignores=[]), path, "exec")


def main(ref_root):
    sys.path.insert(0, HERE)
    from make_mla_golden import _Array, _install_mlx_stand_in
    _install_mlx_stand_in()
    sys.path.insert(0, ref_root)
    from v4mlx import mla as MLA
    from v4mlx import norm_rope as NR
    from v4mlx import sparse_attn as SA

    code = _attention_statements(os.path.join(ref_root, SRC))
    mx = sys.modules["mlx.core"]
    cos1, sin1 = NR.rope_cos_sin(64, 512, 65536, 160000.0, 16, 32, 1)   # the YaRN table (ratio 4 and 128)
    rng = np.random.default_rng(41)
    g = {}
    # (tag, compresses, position, compressed rows held): wrapped window with 75 visible rows, a partial
    # window with 12 visible rows, and a window-only layer
    for tag, r4, p, ncomp in (("r4", True, 300, 80), ("r4p", True, 50, 12), ("w", False, 300, 0)):
        winr = rng.standard_normal((128, 512)).astype(np.float32)
        comp = rng.standard_normal((max(ncomp, 1), 512)).astype(np.float32)[:ncomp]
        qraw = rng.standard_normal((64, 512)).astype(np.float32).view(_Array)
        sinks = rng.standard_normal(64).astype(np.float32)
        cp, sp = cos1[p:p + 1], sin1[p:p + 1]
        q = MLA.perhead_norm(qraw.reshape(1, 1, 64, 512))           # oracle/v4_fast.py:88-89
        q = mx.concatenate([q[..., :-64], NR.apply_rotary_emb(q[..., -64:], cp, sp)], axis=-1)[0]
        st = types.SimpleNamespace(winr=winr, comp=list(comp))
        env = {"np": np, "mx": mx, "SA": SA, "NR": NR, "st": st, "p": p, "q": q, "cp": cp, "sp": sp, "RD": 64,
               "w": types.SimpleNamespace(r4=r4, sinks=sinks)}
        exec(code, env)
        g.update({f"da_{tag}_winr": winr, f"da_{tag}_comp": comp, f"da_{tag}_qraw": np.asarray(qraw),
                  f"da_{tag}_sinks": sinks, f"da_{tag}_p": np.array(p), f"da_{tag}_r4": np.array(r4),
                  f"da_{tag}_o": np.asarray(env["o"])[0, 0].astype(np.float32)})
    np.savez_compressed(OUT, **g)
    print("wrote", OUT, sorted(g))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_decode_attention_golden.py <reference checkout>")
    main(sys.argv[1])
