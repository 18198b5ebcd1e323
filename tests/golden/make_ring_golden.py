"""Generate tests/golden/ring_golden.npz: the reference's own decode ring step on seeded inputs.

Run where a checkout of the reference project is available:
    python tests/golden/make_ring_golden.py <reference checkout>
The ring step is inline code of `layer_fwd` (oracle/decode_engine.py:96-105), in a module that
imports MLX and loads a checkpoint at import. The statements of that branch are taken from the
file's syntax tree and run alone, in a namespace that gives them what the module would: the
weight lookup `W`, the layer's ring state `st`, the rope table `freqsC` and ref_torch's
`apply_rotary_emb` (as the module does), the module's own `aq`, and `mx.float32`. Recorded per
decode step (inputs included): the ring after the step, and the emitted row once with the module's
`aq` and once with `aq` replaced by the identity (the row before the fp8 simulation).
"""
import ast
import os
import sys
import types

import numpy as np

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ring_golden.npz")
SRC = os.path.join("oracle", "decode_engine.py")


def _decode_branch(tree):
    """The statements of the `else:` (decode step) branch of `if decode_pos is None:` in layer_fwd."""
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "layer_fwd")
    for node in ast.walk(fn):
        if (isinstance(node, ast.If) and isinstance(node.test, ast.Compare)
                and isinstance(node.test.left, ast.Name) and node.test.left.id == "decode_pos"):
            return node.orelse
    raise LookupError("decode branch of layer_fwd not found")


def _function(tree, name):
    return next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == name)


def main(ref_root):
    sys.path.insert(0, ref_root)
    import ml_dtypes
    import torch
    from ref_torch.norm_rope import apply_rotary_emb, precompute_freqs

    path = os.path.join(ref_root, SRC)
    tree = ast.parse(open(path).read())
    env_aq = {"np": np, "ml_dtypes": ml_dtypes}
    exec(compile(ast.Module(body=[_function(tree, "aq")], type_ignores=[]), path, "exec"), env_aq)
    branch = compile(ast.Module(body=_decode_branch(tree), type_ignores=[]), path, "exec")

    rng = np.random.default_rng(31)
    dim, L = 32, 2
    weights = {f"blk.{L}.attn_compressor_kv.weight": (rng.standard_normal((1024, dim)) * 0.1).astype(np.float32),
               f"blk.{L}.attn_compressor_gate.weight": (rng.standard_normal((1024, dim)) * 0.1).astype(np.float32),
               f"blk.{L}.attn_compressor_ape.weight": (rng.standard_normal((4, 1024)) * 0.1).astype(np.float32),
               f"blk.{L}.attn_compressor_norm.weight": (rng.random(512) + 0.5).astype(np.float32)}
    freqs = precompute_freqs(64, 64, 65536, 160000.0, 16, 32, 1).numpy().astype(np.float32)
    ring_kv0 = rng.standard_normal((8, 1024)).astype(np.float32)
    ring_sc0 = rng.standard_normal((8, 1024)).astype(np.float32)
    positions = np.arange(101, 109)                      # emits at 103 and 107
    xs = rng.standard_normal((len(positions), dim)).astype(np.float32)
    g = {"ring_x": xs, "ring_pos": positions, "ring_kv0": ring_kv0, "ring_sc0": ring_sc0,
         "ring_wkv": weights[f"blk.{L}.attn_compressor_kv.weight"],
         "ring_wgate": weights[f"blk.{L}.attn_compressor_gate.weight"],
         "ring_ape": weights[f"blk.{L}.attn_compressor_ape.weight"],
         "ring_nw": weights[f"blk.{L}.attn_compressor_norm.weight"]}
    for tag, aq in (("q", env_aq["aq"]), ("raw", lambda x, b=64: x)):
        st = types.SimpleNamespace(kvs=ring_kv0.copy(), scs=ring_sc0.copy(), comp=[])
        kvs, scs, rows = [], [], []
        for x, p in zip(xs, positions):
            env = {"np": np, "torch": torch, "mx": types.SimpleNamespace(float32=np.float32), "L": L, "RD": 64,
                   "W": lambda n, twod=True: weights[n], "xn": x[None, None], "decode_pos": int(p), "st": st,
                   "freqsC": freqs, "rope_t": apply_rotary_emb, "aq": aq}
            n_before = len(st.comp)
            exec(branch, env)
            kvs.append(st.kvs.copy()), scs.append(st.scs.copy())
            rows.append(st.comp[-1].astype(np.float32) if len(st.comp) > n_before else np.full(512, np.nan, np.float32))
        g[f"ring_{tag}_rows"] = np.stack(rows)
        if tag == "raw":  # the ring itself does not depend on the simulation of emitted rows
            g["ring_kvs"], g["ring_scs"] = np.stack(kvs), np.stack(scs)
    np.savez_compressed(OUT, **g)
    print("wrote", OUT, sorted(g))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_ring_golden.py <reference checkout>")
    main(sys.argv[1])
