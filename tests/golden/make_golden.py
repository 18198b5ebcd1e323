"""Generate tests/golden/ref_torch_golden.npz from the reference's own ref_torch functions.

Run where a checkout of the reference project is available:
    python tests/golden/make_golden.py <reference checkout>
The reference is not available on the GPU box, so its outputs on seeded inputs are recorded here
(inputs included) and the oracle restatements are checked against them by
tests/test_oracle_golden.py. Functions used: ref_torch/sparse_attn.py:9 get_window_topk_idxs,
:23 sparse_attn; ref_torch/compressor.py:21 compressor_prefill; ref_torch/norm_rope.py:10 rmsnorm,
:19 precompute_freqs, :46 precompute_freqs_cis, :53 apply_rotary_emb.
"""
import os
import sys

import numpy as np
import torch

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ref_torch_golden.npz")


def main(ref_root):
    sys.path.insert(0, ref_root)
    from ref_torch import compressor as C
    from ref_torch import norm_rope as NR
    from ref_torch import sparse_attn as SA

    g = {}
    # window indices: all three branches
    cases = [(128, 2, 5, 0), (8, 1, 20, 0), (8, 1, 1, 0), (8, 2, 1, 3), (8, 1, 1, 6), (8, 1, 1, 7),
             (8, 1, 1, 13), (128, 1, 1, 32767), (128, 1, 1, 200)]
    for i, (w, b, s, sp) in enumerate(cases):
        g[f"win_{i}_args"] = np.array([w, b, s, sp], dtype=np.int64)
        g[f"win_{i}_out"] = SA.get_window_topk_idxs(w, b, s, sp).numpy().astype(np.int64)

    # sparse attention (fp32), including masked entries, int64 indices and one all-masked query
    gen = torch.Generator().manual_seed(11)
    s, h, d, n, t = 6, 16, 512, 300, 40
    q = torch.randn(s, h, d, generator=gen)
    kv = torch.randn(n, d, generator=gen)
    sink = torch.randn(h, generator=gen)
    idx = torch.randint(0, n, (s, t), generator=gen)
    idx[0, 5:9] = -1
    idx[1, ::3] = -1
    idx[5, :] = -1  # all masked -> NaN row in the reference
    scale = d ** -0.5
    g["sa_q"], g["sa_kv"], g["sa_sink"], g["sa_idx"] = q.numpy(), kv.numpy(), sink.numpy(), idx.numpy()
    g["sa_scale"] = np.array(scale, dtype=np.float64)
    g["sa_out"] = SA.sparse_attn(q, kv, sink, idx, scale).numpy()

    # norm / rope
    x = torch.randn(3, 512, generator=gen)
    wn = torch.randn(512, generator=gen) * 0.1 + 1
    g["rms_x"], g["rms_w"], g["rms_out"] = x.numpy(), wn.numpy(), NR.rmsnorm(x, wn).numpy()
    g["freqs_yarn"] = NR.precompute_freqs(64, 0, 65536, 160000.0, 16, 32, 1).numpy()
    g["freqs_plain"] = NR.precompute_freqs(64, 0, 0, 10000.0, 40, 32, 1).numpy()
    cis = NR.precompute_freqs_cis(64, 16, 65536, 160000.0, 16, 32, 1)
    g["cis_real"] = torch.view_as_real(cis).numpy()
    x3 = torch.randn(1, 16, 64, generator=gen)
    x4 = torch.randn(1, 16, 4, 64, generator=gen)
    g["rope_x3"], g["rope_x4"] = x3.numpy(), x4.numpy()
    g["rope_x3_fwd"] = NR.apply_rotary_emb(x3, cis).numpy()
    g["rope_x3_inv"] = NR.apply_rotary_emb(x3, cis, inverse=True).numpy()
    g["rope_x4_fwd"] = NR.apply_rotary_emb(x4, cis).numpy()

    # compressor prefill: s = 18 (remainder 2) and s = 16 (no remainder), dim 64
    dim = 64
    wkv = torch.randn(1024, dim, generator=gen) * 0.05
    wgate = torch.randn(1024, dim, generator=gen) * 0.05
    ape = torch.randn(4, 1024, generator=gen) * 0.1
    nw = torch.randn(512, generator=gen) * 0.1 + 1
    g["cmp_wkv"], g["cmp_wgate"], g["cmp_ape"], g["cmp_nw"] = wkv.numpy(), wgate.numpy(), ape.numpy(), nw.numpy()
    for s_ in (18, 16):
        xx = torch.randn(2, s_, dim, generator=gen)
        rows, st = C.compressor_prefill(xx, wkv, wgate, ape, nw)
        g[f"cmp{s_}_x"] = xx.numpy()
        g[f"cmp{s_}_rows"] = rows.numpy()
        g[f"cmp{s_}_state_kv"] = st["kv"].numpy()
        g[f"cmp{s_}_state_score"] = st["score"].numpy()
        if "kv_rem" in st:
            g[f"cmp{s_}_state_kv_rem"] = st["kv_rem"].numpy()
    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT} ({os.path.getsize(OUT) / 1e6:.2f} MB, {len(g)} arrays)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference checkout>")
    main(sys.argv[1])
