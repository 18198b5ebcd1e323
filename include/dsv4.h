/*
 * dsv4.h — C ABI of the B200 (sm_100a) compressed sparse-MLA attention path of DeepSeek-V4-Flash.
 *
 * Every entry point takes plain pointers, sizes and a cudaStream_t passed as `void*`; no torch
 * type crosses this boundary. Tensors are borrowed: the caller owns every buffer, including the
 * workspace (query its size with the matching *_workspace_size call). The library never frees and
 * never calls cudaMalloc on these paths. Every call is asynchronous on `stream` and returns a
 * dsv4_status; on a non-zero status dsv4_last_error() returns a message for the calling thread.
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   dsv4_sparse_attn          <- ref_torch/sparse_attn.py:23  sparse_attn(q, kv, attn_sink, topk_idxs, scale)
 *                                (MLX twin v4mlx/sparse_attn.py:26)
 *   dsv4_window_topk_idxs     <- ref_torch/sparse_attn.py:9   get_window_topk_idxs(window_size, bsz, seqlen, start_pos)
 *   dsv4_rmsnorm              <- ref_torch/norm_rope.py:10    rmsnorm(x, weight, eps)
 *                                and v4mlx/mla.py:26          perhead_norm(q, eps) (weight == NULL)
 *   dsv4_rope                 <- ref_torch/norm_rope.py:53    apply_rotary_emb(x, freqs_cis, inverse)
 *   dsv4_norm_rope            <- the rmsnorm -> rope -> cast chains of oracle/decode_engine.py:77-81
 *                                and oracle/v4_fast.py:87-91 (fused)
 *   dsv4_yarn_freqs           <- ref_torch/norm_rope.py:19    precompute_freqs(...)
 *   dsv4_compressor_pool      <- ref_torch/compressor.py:21   compressor_prefill(...) after its two projections
 *   dsv4_compressor_decode    <- oracle/decode_engine.py:96-105 (decode ring step; MLX twin oracle/v4_fast.py:97-106)
 *   dsv4_linear               <- v4mlx/mla.py:16-42           linear / q_down / q_up / kv_proj / o_grouped
 *                                (8-bit grouped weights as oracle/v4_fast.py:31-34 qz/qmm, symmetric here)
 *   dsv4_indexer_topk         <- no reference code: the reference attends to every visible compressed row
 *                                (oracle/decode_engine.py:112-114); this is the lightning-indexer selection
 *                                that replaces that list when more than top_k rows are visible.
 *   dsv4_decode_window_indices<- oracle/v4_fast.py:108-117 (window rows of the attended list, ring order
 *                                of ref_torch/sparse_attn.py:11-13)
 */
#ifndef DSV4_H_
#define DSV4_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DSV4_ABI_VERSION 1

#if defined(__GNUC__)
#define DSV4_API __attribute__((visibility("default")))
#else
#define DSV4_API
#endif

typedef enum {
  DSV4_OK = 0,
  DSV4_ERR_INVALID_ARGUMENT = 1,  /* bad shape, null pointer, unsupported size */
  DSV4_ERR_UNSUPPORTED_DTYPE = 2,
  DSV4_ERR_CUDA = 3,              /* a CUDA runtime call failed; message carries cudaGetErrorString */
  DSV4_ERR_INDEX_OUT_OF_RANGE = 4,/* device error word: a gathered index was outside [-1, n) */
  DSV4_ERR_WAIT_TIMEOUT = 5,      /* device error word: a bounded wait ran out */
  DSV4_ERR_WORKSPACE = 6          /* workspace pointer missing or smaller than *_workspace_size */
} dsv4_status;

typedef enum { DSV4_F32 = 0, DSV4_BF16 = 1, DSV4_I32 = 2, DSV4_I64 = 3, DSV4_I8 = 4 } dsv4_dtype;

/* ---- status ------------------------------------------------------------------------------ */
DSV4_API const char* dsv4_last_error(void);
DSV4_API int dsv4_abi_version(void);
/* Reads (and clears) the device error word of the current device after synchronising `stream`.
 * *code receives 0 or a dsv4_status raised by a kernel (index out of range, wait timeout). */
DSV4_API int dsv4_device_error(int* code, void* stream);
/* Self-test of the failure path (no counterpart in the reference, which has no kernels): one kernel
 * waits, with the same bounded wait the tcgen05 kernels use (1 s of %globaltimer), on an mbarrier
 * that nothing arrives on; it records DSV4_ERR_WAIT_TIMEOUT on the device error word and returns.
 * dsv4_device_error then reports the timeout, and the context stays usable. */
DSV4_API int dsv4_selftest_wait_timeout(void* stream);

/* ---- a1: sparse attention --------------------------------------------------------------------
 * o[i,h,:] = sum_t p[i,h,t] kv[idx[i,t],:] / (sum_t p[i,h,t] + exp(sink[h] - m[i,h]))
 * with p = exp(scale * q[i,h,:].kv[idx[i,t],:] - m[i,h]), m the max over valid t, idx < 0 masked.
 * A query whose indices are all masked yields NaN, as the reference does. */
typedef struct {
  const void* q;          /* [s, h, d], q_dtype (F32 or BF16) */
  const void* kv;         /* [n, d] BF16 */
  const float* sink;      /* [h] */
  const void* idx;        /* [s, t], idx_dtype (I32 or I64); -1 = masked */
  void* out;              /* [s, h, d], out_dtype (F32 or BF16) */
  int64_t s;              /* queries */
  int64_t n;              /* kv rows */
  int32_t h;              /* heads, multiple of 16 */
  int32_t d;              /* head dim, 512 */
  int32_t t;              /* indices per query */
  int32_t q_dtype, idx_dtype, out_dtype;
  float scale;
  /* optional fused inverse rope on the last rope_dim dims of the output (freqs == NULL: off) */
  const float* rope_freqs;      /* [rope_dim/2] angular frequencies */
  const int32_t* positions;     /* [s] rope position per query */
  int32_t rope_dim;
  int32_t num_splits;           /* 0 = automatic split of t across CTAs */
  void* workspace;
  size_t workspace_bytes;
  /* optional fused q prologue: weightless per-head RMS norm (eps q_eps) of each q row, then RoPE of
   * its last rope_dim dims at positions[i] with rope_freqs, applied while q is staged (the decode q
   * chain of oracle/v4_fast.py:88-89); q is then the raw projection output */
  int32_t q_norm_rope;
  float q_eps;
  /* optional implicit window (win_base == NULL: off): the list of query i is then
   * [window rows | idx[i, 0:t]], the window rows computed from positions[i] as in
   * dsv4_indexer_params (ring order, or linear with window_linear), pool row win_base[i*win_stride] + slot.
   * window must be a multiple of 64. Window tiles need nothing from the kernel launched before, so
   * under programmatic dependent launch they run while that kernel (the top-k selection) finishes. */
  const int64_t* win_base;
  int32_t win_stride;
  int32_t window;
  int32_t window_linear;
  /* kernel choice: 0 = automatic (the tcgen05 kernel, 128-row tiles, split-K over tile ranges, for
   * calls of at least 16 queries with 64 heads and bf16 q or the fused q prologue; below 16 queries
   * the head-group kernel, else the mma.sync split-K kernel), 1 = the mma.sync kernel (64 heads per
   * CTA), 2 = the tcgen05 kernel (64 heads and bf16 q or the fused prologue, else
   * DSV4_ERR_INVALID_ARGUMENT), 3 = the head-group decode kernel (16 heads per CTA, the 64-row tiles of
   * a query split over up to 16 CTAs that merge as one thread-block cluster; the q prologue fused in
   * the kernel; falls back to 1 where such a cluster cannot be scheduled). All compute the same
   * function (num_splits counts 64-row tiles for 1 and 3, 128-row tiles for 2); the choice is for
   * tests and measurements. */
  int32_t kernel;
  /* 1: the caller guarantees that no kernel still running when this one launches writes q,
   * positions, win_base or the implicit window's pool rows (only idx may come from the kernel launched
   * just before, e.g. the indexer's selection after its score kernel, which waits for all earlier work
   * before it lets later kernels launch); the head-group kernel then stages q and computes its window
   * tiles before the programmatic-dependency wait. 0: every read follows the wait. */
  int32_t pre_wait;
} dsv4_sparse_attn_params;

DSV4_API size_t dsv4_sparse_attn_workspace_size(const dsv4_sparse_attn_params* p);
DSV4_API int dsv4_sparse_attn(const dsv4_sparse_attn_params* p, void* stream);

/* ---- a2: window indices (int32 [bsz, seqlen, cols]); cols = window if start_pos > 0 else
 * min(seqlen, window), exactly the three branches of the reference. */
DSV4_API int dsv4_window_topk_idxs(int32_t window, int32_t bsz, int32_t seqlen, int32_t start_pos,
                          int32_t* out, void* stream);

/* ---- a5: RMSNorm / RoPE ---------------------------------------------------------------------- */
typedef struct {
  const void* x;          /* [rows, dim], x_dtype */
  const void* weight;     /* [dim] w_dtype, or NULL for the weightless per-head norm */
  void* out;              /* [rows, dim], out_dtype */
  int64_t rows;
  int32_t dim;
  int32_t x_dtype, w_dtype, out_dtype;
  float eps;
} dsv4_rmsnorm_params;
DSV4_API int dsv4_rmsnorm(const dsv4_rmsnorm_params* p, void* stream);

typedef struct {
  const void* x;          /* [s, heads, dim] rows (x_stride elements apart), rope on the LAST rope_dim */
  void* out;              /* same shape, out_dtype, out_stride */
  int64_t s;              /* positions (rows of the table) */
  int32_t heads;          /* rows sharing one position */
  int32_t dim;            /* full row length */
  int32_t rope_dim;
  int32_t x_dtype, out_dtype;
  /* exactly one of the two angle sources: */
  const float* cis;             /* [cis_rows, rope_dim/2, 2] (cos, sin) (a freqs_cis table);
                                   position row r uses table row r % cis_rows */
  int64_t cis_rows;
  const float* freqs;           /* [rope_dim/2]; angle = float(pos) * freqs[i] */
  const int32_t* positions;     /* [s] with freqs; NULL means pos = pos_offset + row */
  int32_t pos_offset;
  int32_t inverse;              /* conjugate rotation */
} dsv4_rope_params;
DSV4_API int dsv4_rope(const dsv4_rope_params* p, void* stream);

/* fused RMSNorm (or weightless per-head norm) + RoPE on the last rope_dim dims + cast. */
typedef struct {
  const void* x;          /* [rows, heads, dim] */
  const void* weight;     /* [dim] or NULL (per-head weightless norm) */
  void* out;              /* [rows, heads, dim] out_dtype; or, with out_rows, scattered rows */
  const int64_t* out_rows;/* optional [rows]: destination row index (in units of heads*dim) */
  int64_t rows;
  int32_t heads, dim, rope_dim;
  int32_t x_dtype, w_dtype, out_dtype;
  float eps;
  const float* freqs;     /* [rope_dim/2] */
  const int32_t* positions; /* [rows] */
  /* 1: the act-quant simulation of the cached rows (oracle/decode_engine.py:52-54, 82, 105;
   * v4mlx/compressor.py:11-20, 60-62): dims [0, dim - rope_dim) are rounded to fp8-e4m3 (nearest
   * even, saturating) in blocks of 64 with a power-of-two scale 2^ceil(log2(max(amax, 1e-4) / 448)),
   * after the norm and rope, before the store. (dim - rope_dim) must be a multiple of 64. 0: off. */
  int32_t act_quant;
} dsv4_norm_rope_params;
DSV4_API int dsv4_norm_rope(const dsv4_norm_rope_params* p, void* stream);

/* YaRN frequency table (host, fp32), the reference's precompute_freqs; out has dim/2 floats. */
DSV4_API int dsv4_yarn_freqs(int32_t dim, int64_t original_seq_len, double base, double factor,
                    double beta_fast, double beta_slow, float* out_host);

/* ---- a7: lightning indexer + top-k ---------------------------------------------------------------
 * score[j] = sum_h w[h] * relu(q[h,:] . k[j,:]) in a fixed fp32 order (per head a sequential fmaf
 * chain over the 128 dims; heads folded four at a time, sequentially, into 16 partials that are
 * summed by a balanced binary tree). Selection: the top_k visible keys by (score desc, index asc),
 * written in ascending key order, padded with -1. */
typedef struct {
  const float* q;         /* [batch, s, heads, 128] */
  const float* w;         /* [batch, s, heads] */
  const float* k;         /* [batch, n_keys, 128] (k_batch_stride rows apart) */
  int32_t* out;           /* [batch, s, out_stride]; top_k columns written from out_col */
  float* scores_out;      /* optional [batch, s, n_keys] raw scores (testing); NULL = off */
  int32_t batch, s, heads, n_keys, top_k;
  int64_t k_batch_stride; /* in rows */
  /* visibility: query i of batch b sees keys j < min(n_keys, n_vis) with
   * n_vis = (positions[b*s+i] + 1) / ratio if positions != NULL, else n_keys */
  const int32_t* positions;
  int32_t ratio;
  /* output mapping: out[b, i, out_col + r] = map(key j) where map(j) = j + out_offset, or, with a
   * block table, table[b*table_stride + j / page] * page + j % page + out_offset */
  int32_t out_stride, out_col;
  int64_t out_offset;
  const int32_t* block_table;
  int32_t table_stride, page;
  void* workspace;
  size_t workspace_bytes;
  /* optional: also write the window rows of query i into out columns [out_col - window, out_col):
   * window_linear == 0: the decode ring order of ref_torch/sparse_attn.py:11-15 at position
   *   positions[i], pool row win_base[b] + slot, -1 for slots not yet written;
   * window_linear == 1: the prefill branch (ref_torch/sparse_attn.py:17-19), rows
   *   win_base[b] + max(0, p - window + 1) + c, -1 where that exceeds p = positions[i] */
  const int64_t* win_base;
  int32_t window;
  int32_t window_linear;
  /* scoring method (the selected sets are the same, bit for bit):
   * 1 = every score in the fixed fp32 order above on the FMA pipe;
   * 2 = tensor-core filter: approximate scores A from a two-term fp16 split of q and k (each row
   *     scaled by a power of two) on tcgen05 with fp32 accumulation, the bound
   *     |A - score| <= eps = 2^-14 * sum_h |w[h]| * ||q[h,:]|| * max_j ||k[j,:]|| (the rounding
   *     analysis gives about 2^-15.7 for finite inputs whose nonzero rows peak within 2^+-86), and
   *     exact fp32 rescoring (the order above) of the keys whose A lies within 2 eps of the k-th
   *     largest A; keys above that band are in the top_k, keys below it are not. n_keys <= 16384.
   *     With scores_out, the approximate scores are written there.
   * 0 = automatic: 2 for prefill-shaped calls (batch * s >= 256) and decode batches (batch >= 16),
   *     when n_keys > top_k and n_keys <= 16384, else 1. The allocation-free entry point below
   *     always uses 1. */
  int32_t mode;
  /* optional, mode 2: the keys' tile image kept by a decode cache (dsv4_indexer_key_image, and the
   * compressor decode step for the keys it appends): the filter reads it instead of splitting the
   * keys on every call. All three or none; k_batch_stride keys per batch entry in the image. */
  const uint8_t* key_image;
  const float* key_inv;
  const float* key_norm_max;
} dsv4_indexer_params;

/* The decode cache's form of the indexer keys for the tensor-core filter: per batch entry,
 * ceil(k_batch_stride / 128) tiles of DSV4_KEY_TILE_BYTES (the scaled fp16 hi / lo split of 128 keys,
 * laid out as the MMA reads it), one inverse power-of-two scale per key ([batch, tiles * 128] fp32),
 * and a running maximum key norm per entry (an upper bound for the filter's error bound). This call
 * (re)builds keys [0, n_keys) of every entry and sets the norm maximum over them; keys a compressor
 * decode step appends later are added by that step (dsv4_compressor_decode_params). */
#define DSV4_KEY_TILE_BYTES 65536
typedef struct {
  const float* k;         /* [batch, k_batch_stride, 128] */
  int32_t batch, n_keys;
  int64_t k_batch_stride;
  uint8_t* image;         /* [batch, ceil(k_batch_stride / 128), DSV4_KEY_TILE_BYTES] */
  float* inv;             /* [batch, ceil(k_batch_stride / 128) * 128] */
  float* norm_max;        /* [batch] */
} dsv4_key_image_params;
DSV4_API int dsv4_indexer_key_image(const dsv4_key_image_params* p, void* stream);

DSV4_API size_t dsv4_indexer_topk_workspace_size(const dsv4_indexer_params* p);
DSV4_API int dsv4_indexer_topk(const dsv4_indexer_params* p, void* stream);

/* Allocation-free variant of dsv4_indexer_topk, for callers that cannot allocate device memory:
 * a host engine that hands out all GPU memory from its own pool and forbids other allocations, a
 * plugin invoked inside a step that must not synchronise (cudaMalloc and cudaFree can), or code that
 * runs while someone else's stream capture is open. It has no counterpart in the reference.
 * Same parameters and results as dsv4_indexer_topk; `workspace` and `scores_out` must be NULL. Every
 * valid `mode` (0, 1, 2) gives the same selection, and this path always computes it from the exact
 * fp32 scores (mode 1): it ignores key_image / key_inv / key_norm_max, which must still be all set or
 * all NULL. The score scratch is a fixed device array inside the library of DSV4_INDEXER_NOALLOC_MAX_SCORES floats
 * (4 MiB), present on every GPU that loads the library until the process exits; requests with
 * batch * s * round_up(n_keys, 4) above that are rejected with DSV4_ERR_WORKSPACE. The first call on a
 * device looks up that array's device address (cudaGetSymbolAddress) with the device current, so make
 * it before any stream capture; the address is looked up again if the device's context changes (after
 * cudaDeviceReset), so make the first call after a reset outside a capture too. All calls share the one array: calls that overlap on the GPU (on
 * different streams, or on one stream from different host threads without ordering) race. */
#define DSV4_INDEXER_NOALLOC_MAX_SCORES (1 << 20)
DSV4_API int dsv4_indexer_topk_noalloc(const dsv4_indexer_params* p, void* stream);

/* decode attention index list: out[b, 0:window] = window ring rows for position pos[b] in the
 * reference's ring order (ref_torch/sparse_attn.py:11-15), mapped to pool rows
 * win_base[b] + slot; masked slots are -1. Columns window.. are left to dsv4_indexer_topk. */
DSV4_API int dsv4_decode_window_indices(int32_t batch, int32_t window, const int32_t* positions,
                               const int64_t* win_base, int32_t* out, int32_t out_stride,
                               void* stream);

/* ---- a3/a4: KV compressor --------------------------------------------------------------------- */
typedef struct {
  const float* kv;        /* [b, s, 2*head_dim] projection x.wkv^T (fp32) */
  const float* score;     /* [b, s, 2*head_dim] projection x.wgate^T (fp32), before ape */
  const float* ape;       /* [ratio, 2*head_dim] */
  const void* norm_w;     /* [head_dim], norm_dtype */
  void* out;              /* [b, s/ratio, head_dim] out_dtype, or pool rows through out_rows */
  const int64_t* out_rows;/* optional [b, s/ratio] destination row (of head_dim elements) */
  int32_t b, s, head_dim, ratio, rope_dim;
  int32_t norm_dtype, out_dtype;
  float eps;
  const float* freqs;     /* [rope_dim/2]; compressed row g is roped at position ratio*g + pos0 */
  int32_t pos0;
  /* optional decode hand-off state (ref_torch/compressor.py:67-74): ring [b, 2*ratio, 2*head_dim]
   * for kv (0) and score+ape (-inf) seeded from the last full block and the remainder */
  float* ring_kv;
  float* ring_score;
  /* 1: the act-quant simulation of the cached rows (oracle/decode_engine.py:52-54, 82, 105;
   * v4mlx/compressor.py:11-20, 60-62): dims [0, dim - rope_dim) are rounded to fp8-e4m3 (nearest
   * even, saturating) in blocks of 64 with a power-of-two scale 2^ceil(log2(max(amax, 1e-4) / 448)),
   * after the norm and rope, before the store. (dim - rope_dim) must be a multiple of 64.
   * 2: the indexer compressor's key simulation (compressor_prefill(..., rotate=True),
   * v4mlx/compressor.py:57-59, v4mlx/qat.py:8-31), head_dim 128: after the norm and rope the whole
   * row is rotated by the normalised Walsh-Hadamard transform (Sylvester order, fp32 butterflies,
   * then * fp32(128^-0.5)) and rounded to fp4-e2m1 (nearest even) in blocks of 32 with a scale
   * 2^ceil(log2(max(amax, 6 * 2^-126) / 6)). 0: off. */
  int32_t act_quant;
} dsv4_compressor_params;
DSV4_API int dsv4_compressor_pool(const dsv4_compressor_params* p, void* stream);

typedef struct {
  const float* kv;        /* [b, 2*head_dim] this token's x.wkv^T */
  const float* score;     /* [b, 2*head_dim] this token's x.wgate^T (before ape) */
  const float* ape;       /* [ratio, 2*head_dim] */
  const void* norm_w;     /* [head_dim] */
  float* ring_kv;         /* [b, 2*ratio, 2*head_dim] */
  float* ring_score;      /* [b, 2*ratio, 2*head_dim] */
  const int32_t* positions; /* [b] decode position p of this token */
  void* out;              /* pool base [*, head_dim] out_dtype */
  const int64_t* out_rows;/* [b] pool row where the emitted row goes (written only when (p+1)%ratio==0) */
  int32_t b, head_dim, ratio, rope_dim;
  int32_t norm_dtype, out_dtype;
  float eps;
  const float* freqs;
  /* optional (indexer keys: head_dim 128, fp32 out): also add each emitted row to a key image
   * (dsv4_key_image_params layout) as key j = out_rows[b] % image_stride of entry
   * out_rows[b] / image_stride, and raise that entry's norm maximum. NULL = off. */
  uint8_t* key_image;
  float* key_inv;
  float* key_norm_max;
  int64_t image_stride;
  /* 1: the act-quant simulation of the cached rows (oracle/decode_engine.py:52-54, 82, 105;
   * v4mlx/compressor.py:11-20, 60-62): dims [0, dim - rope_dim) are rounded to fp8-e4m3 (nearest
   * even, saturating) in blocks of 64 with a power-of-two scale 2^ceil(log2(max(amax, 1e-4) / 448)),
   * after the norm and rope, before the store. (dim - rope_dim) must be a multiple of 64.
   * 2: the Hadamard + fp4-e2m1 key simulation of dsv4_compressor_params.act_quant (head_dim 128),
   * also applied to the row added to the key image. 0: off. */
  int32_t act_quant;
} dsv4_compressor_decode_params;
DSV4_API int dsv4_compressor_decode(const dsv4_compressor_decode_params* p, void* stream);
/* Two decode steps (two compressors, the same batch) in one launch: a decode block's main and
 * indexer compressors read the same token's projections and write disjoint rings and rows, so one
 * grid serves both (each as dsv4_compressor_decode with its own params). Pairs that do not share
 * the batch or the ratio-4 fast path run as two launches. No reference counterpart: the reference
 * runs its compressors one after the other (oracle/decode_engine.py:96-105). */
DSV4_API int dsv4_compressor_decode_pair(const dsv4_compressor_decode_params* a,
                                         const dsv4_compressor_decode_params* b, void* stream);

/* ---- decode-step row bookkeeping of the device-resident state (pool of bf16 rows: per-sequence
 * window rings at win_base[i], then pages of compressed rows from comp_base through block_table;
 * indexer keys [b, max_comp, 128]). For sequence i at position p = positions[i]:
 *   win_rows[i]  = win_base[i] + p % window                      (this token's window slot)
 *   entry        = max((p + 1) / ratio - 1, 0)                   (compressed entry the step emits)
 *   comp_rows[i] = comp_base + block_table[i*bt_stride + entry/page]*page + entry % page
 *   key_rows[i]  = i * max_comp + entry
 * An entry >= max_comp raises DSV4_ERR_INDEX_OUT_OF_RANGE on the device error word (clamped).
 * max_comp == 0 is a window-only cache (the ratio-0 and ratio-128 layers, which keep no compressed
 * rows, oracle/v4_fast.py:42-43, 114): comp_rows and key_rows are -1 and block_table may be NULL.
 * Replaces the host-side ring and kvbuf bookkeeping of oracle/v4_fast.py:93-118. */
typedef struct {
  const int32_t* positions;   /* [b] */
  const int64_t* win_base;    /* [b] */
  const int32_t* block_table; /* [b, bt_stride] */
  int64_t* win_rows;          /* [b] out */
  int64_t* comp_rows;         /* [b] out */
  int64_t* key_rows;          /* [b] out */
  int64_t comp_base;
  int32_t b, window, ratio, page, bt_stride, max_comp;
} dsv4_decode_rows_params;
DSV4_API int dsv4_decode_rows(const dsv4_decode_rows_params* p, void* stream);

/* ---- a6: projections. y[m, n] = sum_k x[m, k] * W[n, k] (W row-major [n, k] as the reference)
 * W is BF16, or I8 with BF16 scales per (row, group of `group` k). x BF16 or F32, y F32 or BF16.
 * `groups` > 1 runs a grouped projection: x viewed as [m, groups, k], W as [groups, n, k], y as
 * [m, groups, n] (the o_grouped first stage, v4mlx/mla.py:42-56). */
typedef struct {
  const void* x;
  const void* w;
  const void* w_scale;    /* [groups*n, k/group] BF16 when w_dtype == I8 */
  void* y;
  int64_t m;
  int32_t n, k, groups, group;
  int32_t x_dtype, w_dtype, y_dtype;
  /* m <= 64 (decode batches) runs a weight-streaming kernel; when its output tiles leave SMs
   * idle it splits k over a thread-block cluster and sums the partials in shared memory, no
   * workspace. Larger m with few output tiles and a long k splits k across CTAs and sums fp32
   * partials from this workspace (dsv4_linear_workspace_size bytes); NULL with 0 bytes runs it
   * without the split. Both sums run in a fixed order: results are deterministic. */
  void* workspace;
  size_t workspace_bytes;
  /* kernel choice (a choice of implementation, not of result beyond fp32 summation order):
   * 0 = automatic: bf16 weights with m > 64 run the tcgen05 kernel (TMA-fed, fp32 accumulator in
   * tensor memory, persistent grid, no workspace; a row's result does not depend on m), everything
   * else the kernels below; 1 = the mma.sync kernels (weight-streaming for m <= 64,
   * tiled above); 2 = the tcgen05 kernel for any m (bf16 weights only, else
   * DSV4_ERR_INVALID_ARGUMENT). */
  int32_t kernel;
} dsv4_linear_params;
DSV4_API size_t dsv4_linear_workspace_size(const dsv4_linear_params* p);
DSV4_API int dsv4_linear(const dsv4_linear_params* p, void* stream);

/* Several projections of the same x in one launch (the decode block's q_down, kv_proj, the two
 * compressors' projections and the indexer head weights all read the normed hidden states): output
 * i is y_i[m, n_i] = x[m, k] . W_i[n_i, k]^T, each W_i as in dsv4_linear (groups 1), one weight
 * dtype for all. m <= 64 runs them as one grid of the weight-streaming kernel; larger m runs them
 * as one tcgen05 launch (bf16 weights) or one dsv4_linear per output. Fuses the projections of v4mlx/mla.py:16-42 that share their input. */
#define DSV4_LINEAR_MULTI_MAX 8
typedef struct {
  const void* w;          /* [n, k] */
  const void* w_scale;    /* [n, k/64] BF16 when w_dtype == I8 */
  void* y;                /* [m, n] y_dtype */
  int32_t n, y_dtype;
} dsv4_linear_out;
typedef struct {
  const void* x;          /* [m, k] BF16 */
  int64_t m;
  int32_t k, group, x_dtype, w_dtype, count;
  dsv4_linear_out outs[DSV4_LINEAR_MULTI_MAX];
  /* as dsv4_linear_params.kernel; for m > 64 the tcgen05 kernel runs all outputs in one launch,
   * so the CTAs working on one token tile at the same time share it through L2 */
  int32_t kernel;
} dsv4_linear_multi_params;
DSV4_API int dsv4_linear_multi(const dsv4_linear_multi_params* p, void* stream);

/* ---- hyper-connections around the attention block (ref_torch/hc.py:18-80) -----------------------
 * hc_pre (head == 0): x [rows, hc, dim] fp32 (the hc = 4 residual copies of a token) ->
 *   mixes = (x . fn^T) * rsqrt(mean(x^2) + norm_eps), fn [(2 + hc) * hc, hc * dim];
 *   pre = sigmoid(mixes[0:hc] * scale[0] + base[0:hc]) + hc_eps, post = 2 sigmoid(mixes[hc:2hc] *
 *   scale[1] + base[hc:2hc]), comb = Sinkhorn(mixes[2hc:] * scale[2] + base[2hc:]) [hc, hc] (row
 *   softmax + hc_eps, column normalise, then sinkhorn_iters - 1 rounds of row and column
 *   normalisation, each dividing by the sum + hc_eps), y[d] = sum_k pre[k] x[k, d].
 * hc_head (head == 1): fn [hc, hc * dim], scale [1]: pre only, y as above (ParallelHead.hc_head).
 * Optional in the same launch: y_norm = RMSNorm(y) * norm_w (the attention block's first norm;
 * eps y_norm_eps) in y_norm_dtype. hc == 4, dim a multiple of 4 and at most 4096. Two launches: the
 * split-K mixes into the workspace, then the split, y and the norm, one CTA per token. */
typedef struct {
  const float* x;
  const float* fn;
  const float* scale;
  const float* base;
  float* y;               /* [rows, dim] or NULL */
  float* post;            /* [rows, hc] (hc_pre) */
  float* comb;            /* [rows, hc, hc] (hc_pre) */
  const void* norm_w;     /* [dim] norm_dtype, or NULL (no weight) */
  void* y_norm;           /* [rows, dim] y_norm_dtype, or NULL */
  void* workspace;        /* the split-K partial mixes; dsv4_hc_workspace_size bytes */
  size_t workspace_bytes;
  int64_t rows;
  int32_t hc, dim, sinkhorn_iters, head;
  int32_t norm_dtype, y_norm_dtype;
  float norm_eps, hc_eps, y_norm_eps;
} dsv4_hc_params;
DSV4_API int dsv4_hc_pre(const dsv4_hc_params* p, void* stream);
DSV4_API size_t dsv4_hc_workspace_size(int64_t rows, int32_t hc, int32_t dim, int32_t head);
/* hc_post: out[row, j, d] = post[row, j] x[row, d] + sum_i comb[row, i, j] residual[row, i, d];
 * x [rows, dim], residual [rows, hc, dim], all fp32 (Block.hc_post). */
DSV4_API int dsv4_hc_post(const float* x, const float* residual, const float* post, const float* comb, float* out,
                          int64_t rows, int32_t hc, int32_t dim, void* stream);

/* ---- casts used by the op layer (fp32 <-> bf16) ---- */
DSV4_API int dsv4_cast(const void* x, int32_t x_dtype, void* y, int32_t y_dtype, int64_t numel, void* stream);

/* ---- copy by a kernel, for the serving loop's host <-> device staging (no reference counterpart:
 * the reference uploads its host-built buffers with MLX array constructors, oracle/v4_fast.py:108-118).
 * dst and src are device or pinned (cudaHostAlloc'd) host memory, addressed by their unified pointers;
 * both 16-byte aligned, bytes a multiple of 16. A pinned buffer read or written this way moves over the
 * bus as the SMs load or store it, which for the tens of KB of a decode step's inputs and outputs costs
 * less than a copy-engine transfer. Ordered in the stream like any kernel (programmatic dependent
 * launch: it waits for the kernel before it). */
DSV4_API int dsv4_copy(void* dst, const void* src, size_t bytes, void* stream);
/* As dsv4_copy, but overlapped with the kernel launched before it on the stream (programmatic
 * dependent launch): the copy starts without waiting for that kernel, lets the next kernel launch
 * only once its own stores are visible, and waits for that kernel before it completes, so the next
 * kernel's dependency wait covers both. The kernel before must neither read nor write dst or src.
 * A decode step uses it to bring q in beside the top-k selection (no reference counterpart). */
DSV4_API int dsv4_copy_beside(void* dst, const void* src, size_t bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* DSV4_H_ */
