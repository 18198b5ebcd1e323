"""CPU oracle for the compressed sparse-MLA path — TEST INFRASTRUCTURE ONLY.

Restatements of the reference's algorithms (each function cites the reference file:line it
follows), used as the checker by tests/, by __graft_entry__.smoke() and by bench.py's CPU
baseline leg. The product package never imports this directory.

  sparse_attn_ref.py   ref_torch/sparse_attn.py        (torch fp32)
  norm_rope_ref.py     ref_torch/norm_rope.py, v4mlx/mla.py:26  (torch fp32)
  compressor_ref.py    ref_torch/compressor.py, oracle/decode_engine.py:85-105 (torch fp32)
  mla_ref.py           v4mlx/mla.py (torch fp32; the reference has no torch version)
  indexer_canon.c      lightning-indexer scores + top-k in the library's fixed fp32 order (C)
  indexer_ref.py       ctypes wrapper of indexer_canon.c, built by build_oracle()
  layer_ref.py         the attention block compositions of oracle/decode_engine.py:75-119 and
                       oracle/v4_fast.py:83-122 (prefill and decode)

Pinning: tests/golden/make_golden.py imports the reference's own ref_torch (available only in
the development container) and records its outputs on seeded inputs; tests/test_oracle_golden.py
checks these restatements against those fixtures. The indexer has no reference implementation,
so its parity is pinned only by self-consistency (exact agreement with an independent float64
check of the same formula, up to fp32 rounding) — "parity unpinned" for the indexer selection.
"""
