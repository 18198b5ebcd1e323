"""B200-native compressed sparse-MLA attention path of DeepSeek-V4-Flash.

Drop-in ops with the reference's call signatures (ref_torch / v4mlx), each a torch custom op
(namespace `dsv4`) backed by sm_100a kernels in libdsv4.so through the C ABI of include/dsv4.h:

  sparse_attn, get_window_topk_idxs          ref_torch/sparse_attn.py
  compressor_prefill (+ decode ring step)     ref_torch/compressor.py, oracle/decode_engine.py:85-105
  rmsnorm, apply_rotary_emb, precompute_*     ref_torch/norm_rope.py
  q_down, perhead_norm, q_up, kv_proj,        v4mlx/mla.py
  o_grouped
  indexer_topk                                lightning-indexer selection (absent from the reference)

There is no CPU path: the ops raise on CPU tensors and when libdsv4.so is missing.
"""
from . import _lib
from .compressor import CompressorStep, compressor_decode_pair, compressor_decode_step, compressor_prefill
from .decode import DecodeRunner, SparseMLACache, decode_attention, window_attention
from .hc import hc_head, hc_post, hc_pre
from .indexer import indexer_scores, indexer_topk, indexer_topk_into
from .layer import (AttentionWeights, BlockRunner, DecodeBlock, layer_rope_freqs, make_attention_weights,
                    prefill_layer)
from .prefill import (CompressorWeights, PrefillStaging, ShardedPrefill, attend_queries_host, sparse_mla_prefill,
                      sparse_mla_prefill_host)
from .mla import (N_GROUPS, N_HEADS, HEAD_DIM, O_LORA, ROPE_HD, QuantWeight, kv_proj, linear, linear_multi, o_grouped,
                  q_down, q_up, quantize_int8_g64)
from .norm_rope import (apply_rotary_emb, norm_rope, perhead_norm, precompute_freqs, precompute_freqs_cis,
                        rmsnorm, rope, rope_freqs)
from .sparse_attn import get_window_topk_idxs, sparse_attn, sparse_attn_rope

__all__ = [
    "sparse_attn", "sparse_attn_rope", "get_window_topk_idxs", "compressor_prefill", "compressor_decode_step",
    "compressor_decode_pair", "CompressorStep",
    "rmsnorm", "perhead_norm", "apply_rotary_emb", "precompute_freqs", "precompute_freqs_cis", "norm_rope",
    "rope", "rope_freqs", "indexer_topk", "indexer_scores", "indexer_topk_into", "linear", "linear_multi", "q_down", "q_up",
    "kv_proj", "o_grouped", "QuantWeight", "quantize_int8_g64", "SparseMLACache", "decode_attention", "DecodeRunner",
    "AttentionWeights", "DecodeBlock", "BlockRunner", "make_attention_weights", "prefill_layer", "CompressorWeights", "ShardedPrefill",
    "sparse_mla_prefill", "sparse_mla_prefill_host", "attend_queries_host", "PrefillStaging", "hc_pre", "hc_post", "hc_head", "window_attention", "layer_rope_freqs",
]


def library():
    """The loaded libdsv4.so (raises if it is missing)."""
    return _lib.load()
