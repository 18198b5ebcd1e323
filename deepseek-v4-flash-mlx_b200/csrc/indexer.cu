// Lightning indexer + top-k selection for B200.
//
// Scores (fp32 on the FMA pipe, never tensor cores, so the order of every rounding is fixed):
//   dot[h,j]  = fmaf chain over the 128 dims in ascending order, starting from +0
//   r[h,j]    = dot > 0 ? dot : +0
//   P_m[j]    = fmaf chain over heads 4m..4m+3 (ascending) of w[h] * r[h,j], starting from +0
//   score[j]  = balanced binary tree over P_0..P_15: ((P0+P1)+(P2+P3)) + ((P4+P5)+(P6+P7)) ...
// The CPU oracle (oracle/indexer_canon.c) performs the identical sequence of IEEE operations, so
// scores and therefore the selected index sets are bit-exact.
//
// Selection: keys ordered by (score desc, index asc) with the score compared through its
// order-preserving 32-bit image; the top_k visible keys are written in ascending key order,
// padded with -1. The reference attends to all visible compressed rows (oracle/decode_engine.py
// :112-114); with top_k >= visible rows this selection returns exactly that list.
#include "common.cuh"

namespace dsv4 {
namespace idx {

constexpr int DI = 128;         // indexer head dim
constexpr int HI = 64;          // indexer heads
constexpr int KT = 64;          // keys per score CTA
constexpr int THREADS = 256;

struct ScoreSmem {
  alignas(16) float q[HI * DI];   // swizzled 16-byte chunks
  alignas(16) float k[KT * DI];
  float w[HI];
  float red[4][KT];
};

__device__ __forceinline__ int swz_chunk(int r, int c) { return c ^ ((r >> 2) & 7); }

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g, bool valid) {
  int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(saddr), "l"(g), "r"(sz));
}

struct ScoreParams {
  const float* q;
  const float* w;
  const float* k;
  float* scores;          // [batch*s, n_pad]
  int32_t batch, s, n_keys, n_pad;
  int64_t k_batch_stride;
  const int32_t* positions;
  int32_t ratio;
};

__device__ __forceinline__ int visible_keys(const int32_t* positions, int64_t qrow, int ratio,
                                            int n_keys) {
  if (positions == nullptr) return n_keys;
  int nv = (positions[qrow] + 1) / ratio;
  return nv < n_keys ? (nv < 0 ? 0 : nv) : n_keys;
}

// grid: (batch*s, key tiles). Thread layout: lane = hq_lo<<3 | jq_lo, warp = hq_hi<<1 | jq_hi,
// so a thread owns heads 4*hq..4*hq+3 and keys 4*jq..4*jq+3 of the tile.
__global__ void __launch_bounds__(THREADS) score_kernel(ScoreParams P) {
  extern __shared__ __align__(16) uint8_t score_smem[];
  ScoreSmem& sm = *reinterpret_cast<ScoreSmem*>(score_smem);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t qrow = blockIdx.x;
  const int b = static_cast<int>(qrow / P.s);
  const int nvis = visible_keys(P.positions, qrow, P.ratio, P.n_keys);
  const int j0 = blockIdx.y * KT;
  if (j0 >= nvis) return;

  const float* qg = P.q + qrow * (HI * DI);
  const float* kg = P.k + static_cast<int64_t>(b) * P.k_batch_stride * DI;
  const uint32_t qs = static_cast<uint32_t>(__cvta_generic_to_shared(sm.q));
  const uint32_t ks = static_cast<uint32_t>(__cvta_generic_to_shared(sm.k));
  for (int c = tid; c < HI * DI / 4; c += THREADS) {
    int r = c >> 5, ch = c & 31;
    cp_async16(qs + (r * 32 + swz_chunk(r, ch)) * 16, qg + r * DI + ch * 4, true);
  }
  for (int c = tid; c < KT * DI / 4; c += THREADS) {
    int r = c >> 5, ch = c & 31;
    bool valid = (j0 + r) < nvis;
    const float* src = kg + static_cast<int64_t>(valid ? j0 + r : 0) * DI + ch * 4;
    cp_async16(ks + (r * 32 + swz_chunk(r, ch)) * 16, src, valid);
  }
  asm volatile("cp.async.commit_group;\n" ::);
  if (tid < HI) sm.w[tid] = P.w[qrow * HI + tid];
  asm volatile("cp.async.wait_group 0;\n" ::);
  __syncthreads();

  const int hq = ((warp >> 1) << 2) | (lane >> 3);
  const int jq = ((warp & 1) << 3) | (lane & 7);
  float acc[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[a][c] = 0.f;

#pragma unroll 2
  for (int ch = 0; ch < DI / 4; ++ch) {
    float4 qv[4], kv[4];
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      int r = hq * 4 + a;
      qv[a] = *reinterpret_cast<const float4*>(&sm.q[(r * 32 + swz_chunk(r, ch)) * 4]);
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      int r = jq * 4 + c;
      kv[c] = *reinterpret_cast<const float4*>(&sm.k[(r * 32 + swz_chunk(r, ch)) * 4]);
    }
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        acc[a][c] = __fmaf_rn(qv[a].x, kv[c].x, acc[a][c]);
        acc[a][c] = __fmaf_rn(qv[a].y, kv[c].y, acc[a][c]);
        acc[a][c] = __fmaf_rn(qv[a].z, kv[c].z, acc[a][c]);
        acc[a][c] = __fmaf_rn(qv[a].w, kv[c].w, acc[a][c]);
      }
  }
  // fold this thread's four heads (ascending) per key
  float part[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    float p = 0.f;
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      float d = acc[a][c];
      float r = d > 0.f ? d : 0.f;
      p = __fmaf_rn(sm.w[hq * 4 + a], r, p);
    }
    part[c] = p;
  }
  // tree levels 0 and 1 over hq bits 0,1 (lane bits 3,4)
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    part[c] = __fadd_rn(part[c], __shfl_xor_sync(0xffffffffu, part[c], 8));
    part[c] = __fadd_rn(part[c], __shfl_xor_sync(0xffffffffu, part[c], 16));
  }
  // levels 2 and 3 over hq bits 2,3 (warp bits 1,2)
  if ((lane >> 3) == 0) {
#pragma unroll
    for (int c = 0; c < 4; ++c) sm.red[warp >> 1][jq * 4 + c] = part[c];
  }
  __syncthreads();
  if (tid < KT) {
    const int j = j0 + tid;
    float v = __fadd_rn(__fadd_rn(sm.red[0][tid], sm.red[1][tid]), __fadd_rn(sm.red[2][tid], sm.red[3][tid]));
    if (j < nvis) P.scores[qrow * P.n_pad + j] = v;
  }
}

// order-preserving image of an fp32 value (larger float -> larger unsigned)
__device__ __forceinline__ uint32_t ordered_bits(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

struct SelectParams {
  const float* scores;
  int32_t* out;
  int32_t batch, s, n_keys, n_pad, top_k;
  const int32_t* positions;
  int32_t ratio;
  int32_t out_stride, out_col;
  int64_t out_offset;
  const int32_t* block_table;
  int32_t table_stride, page;
};

constexpr int SEL_THREADS = 1024;
constexpr int SEL_MAX_KEYS = 32768;

__device__ __forceinline__ int32_t map_key(const SelectParams& P, int b, int j) {
  int64_t row;
  if (P.block_table != nullptr) {
    int pg = j / P.page;
    row = static_cast<int64_t>(P.block_table[static_cast<int64_t>(b) * P.table_stride + pg]) * P.page +
          (j % P.page);
  } else {
    row = j;
  }
  return static_cast<int32_t>(row + P.out_offset);
}

// One CTA per query: radix select (4 passes of 8 bits) of the k-th largest ordered score, then
// an index-ordered compaction that keeps keys above it and the lowest-index keys equal to it.
__global__ void __launch_bounds__(SEL_THREADS) select_kernel(SelectParams P) {
  extern __shared__ uint32_t keys[];  // [nvis] ordered scores
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_prefix, s_kleft;
  __shared__ uint32_t warp_cnt[2][SEL_THREADS / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t qrow = blockIdx.x;
  const int b = static_cast<int>(qrow / P.s);
  const int nvis = visible_keys(P.positions, qrow, P.ratio, P.n_keys);
  int32_t* out = P.out + qrow * P.out_stride + P.out_col;
  const int k = P.top_k;

  if (nvis <= k) {
    for (int r = tid; r < k; r += SEL_THREADS) out[r] = r < nvis ? map_key(P, b, r) : -1;
    return;
  }
  for (int j = tid; j < nvis; j += SEL_THREADS) keys[j] = ordered_bits(P.scores[qrow * P.n_pad + j]);
  if (tid == 0) {
    s_prefix = 0;
    s_kleft = k;
  }
  __syncthreads();
  // MSB-first radix select of the k-th largest key
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += SEL_THREADS) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix;
    const uint32_t mask_hi = (shift == 24) ? 0u : (0xffffffffu << (shift + 8));
    for (int j = tid; j < nvis; j += SEL_THREADS) {
      uint32_t key = keys[j];
      if ((key & mask_hi) == prefix) atomicAdd(&hist[(key >> shift) & 0xff], 1u);
    }
    __syncthreads();
    if (warp == 0) {
      // walk the 256 bins from the top: each lane owns 8 consecutive bins (descending)
      uint32_t kleft = s_kleft;
      uint32_t c[8], tot = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        c[e] = hist[255 - (lane * 8 + e)];
        tot += c[e];
      }
      // exclusive prefix of totals across lanes (in descending-bin order)
      uint32_t incl = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      uint32_t excl = incl - tot;
      // the lane whose range contains the kleft-th key finds the bin
      if (excl < kleft && kleft <= incl) {
        uint32_t run = excl;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (run + c[e] >= kleft) {
            int bin = 255 - (lane * 8 + e);
            s_prefix = prefix | (static_cast<uint32_t>(bin) << shift);
            s_kleft = kleft - run;
            break;
          }
          run += c[e];
        }
      }
    }
    __syncthreads();
  }
  const uint32_t tau = s_prefix;      // k-th largest ordered key
  const uint32_t need_eq = s_kleft;   // how many keys equal to tau are taken (lowest index first)

  // index-ordered compaction: each thread scans a contiguous chunk
  const int per = (nvis + SEL_THREADS - 1) / SEL_THREADS;
  const int jb = tid * per, je = min(nvis, jb + per);
  uint32_t n_gt = 0, n_eq = 0;
  for (int j = jb; j < je; ++j) {
    uint32_t key = keys[j];
    n_gt += key > tau;
    n_eq += key == tau;
  }
  // block exclusive scans of n_gt and n_eq
  uint32_t ig = n_gt, ie = n_eq;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    uint32_t vg = __shfl_up_sync(0xffffffffu, ig, o);
    uint32_t ve = __shfl_up_sync(0xffffffffu, ie, o);
    if (lane >= o) {
      ig += vg;
      ie += ve;
    }
  }
  if (lane == 31) {
    warp_cnt[0][warp] = ig;
    warp_cnt[1][warp] = ie;
  }
  __syncthreads();
  if (warp == 0) {
    uint32_t vg = warp_cnt[0][lane], ve = warp_cnt[1][lane];
    uint32_t sg = vg, se = ve;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      uint32_t tg = __shfl_up_sync(0xffffffffu, sg, o);
      uint32_t te = __shfl_up_sync(0xffffffffu, se, o);
      if (lane >= o) {
        sg += tg;
        se += te;
      }
    }
    warp_cnt[0][lane] = sg - vg;
    warp_cnt[1][lane] = se - ve;
  }
  __syncthreads();
  uint32_t gt_before = warp_cnt[0][warp] + ig - n_gt;
  uint32_t eq_before = warp_cnt[1][warp] + ie - n_eq;
  for (int j = jb; j < je; ++j) {
    uint32_t key = keys[j];
    bool take = false;
    if (key > tau) {
      take = true;
    } else if (key == tau) {
      take = eq_before < need_eq;
      ++eq_before;
    }
    if (take) {
      // output slot = (#taken with lower index) = gt_before + min(eq_before_excl, need_eq)
      uint32_t eq_taken = min(eq_before - (key == tau ? 1u : 0u), need_eq);
      out[gt_before + eq_taken] = map_key(P, b, j);
    }
    if (key > tau) ++gt_before;
  }
}

__global__ void decode_window_kernel(int32_t batch, int32_t window, const int32_t* positions,
                                     const int64_t* win_base, int32_t* out, int32_t out_stride) {
  const int b = blockIdx.x;
  const int p = positions[b];
  for (int c = threadIdx.x; c < window; c += blockDim.x) {
    int slot;
    if (p >= window - 1) {
      int sp = p % window;
      slot = (c < window - sp - 1) ? (sp + 1 + c) : (c - (window - sp - 1));
    } else {
      slot = (c <= p) ? c : -1;
    }
    out[static_cast<int64_t>(b) * out_stride + c] =
        slot < 0 ? -1 : static_cast<int32_t>(win_base[b] + slot);
  }
}

}  // namespace idx
DSV4_ERROR_READER(indexer)

}  // namespace dsv4

using namespace dsv4;

extern "C" size_t dsv4_indexer_topk_workspace_size(const dsv4_indexer_params* p) {
  if (!p || p->batch <= 0 || p->s <= 0 || p->n_keys <= 0) return 0;
  const int64_t n_pad = (p->n_keys + 3) / 4 * 4;
  return static_cast<size_t>(static_cast<int64_t>(p->batch) * p->s * n_pad * sizeof(float));
}

extern "C" int dsv4_indexer_topk(const dsv4_indexer_params* p, void* stream) {
  DSV4_CHECK_ARG(p != nullptr, "dsv4_indexer_topk: params is NULL");
  DSV4_CHECK_ARG(p->q && p->w && p->k && p->out, "dsv4_indexer_topk: NULL tensor");
  DSV4_CHECK_ARG(p->heads == idx::HI, "dsv4_indexer_topk: %d heads unsupported (64 only)", p->heads);
  DSV4_CHECK_ARG(p->batch > 0 && p->s > 0 && p->n_keys > 0 && p->top_k > 0,
                 "dsv4_indexer_topk: bad sizes");
  DSV4_CHECK_ARG(p->n_keys <= idx::SEL_MAX_KEYS, "dsv4_indexer_topk: n_keys %d above %d", p->n_keys,
                 idx::SEL_MAX_KEYS);
  DSV4_CHECK_ARG(p->positions == nullptr || p->ratio > 0, "dsv4_indexer_topk: ratio must be > 0");
  DSV4_CHECK_ARG(p->out_col >= 0 && p->out_col + p->top_k <= p->out_stride,
                 "dsv4_indexer_topk: out_col + top_k exceeds out_stride");
  DSV4_CHECK_ARG(p->block_table == nullptr || (p->page > 0 && p->table_stride > 0),
                 "dsv4_indexer_topk: block table needs page and table_stride");
  DSV4_CHECK_ARG(p->k_batch_stride >= p->n_keys || p->batch == 1,
                 "dsv4_indexer_topk: k_batch_stride smaller than n_keys");
  const int64_t rows = static_cast<int64_t>(p->batch) * p->s;
  DSV4_CHECK_ARG(rows <= 2147483647LL, "dsv4_indexer_topk: too many queries");
  const size_t need = dsv4_indexer_topk_workspace_size(p);
  if (p->workspace == nullptr || p->workspace_bytes < need) {
    set_error("dsv4_indexer_topk: workspace of %zu bytes needed, %zu given", need, p->workspace_bytes);
    return DSV4_ERR_WORKSPACE;
  }
  float* scores = p->scores_out ? p->scores_out : reinterpret_cast<float*>(p->workspace);
  const int n_pad = p->scores_out ? p->n_keys : (p->n_keys + 3) / 4 * 4;

  idx::ScoreParams S;
  S.q = p->q;
  S.w = p->w;
  S.k = p->k;
  S.scores = scores;
  S.batch = p->batch;
  S.s = p->s;
  S.n_keys = p->n_keys;
  S.n_pad = n_pad;
  S.k_batch_stride = p->k_batch_stride;
  S.positions = p->positions;
  S.ratio = p->ratio;
  dim3 g1(static_cast<unsigned>(rows), (p->n_keys + idx::KT - 1) / idx::KT);
  static bool score_attr = false;
  if (!score_attr) {
    DSV4_CUDA_CHECK(cudaFuncSetAttribute(idx::score_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         sizeof(idx::ScoreSmem)));
    score_attr = true;
  }
  idx::score_kernel<<<g1, idx::THREADS, sizeof(idx::ScoreSmem), as_stream(stream)>>>(S);
  DSV4_LAUNCH_CHECK("indexer score_kernel");

  idx::SelectParams L;
  L.scores = scores;
  L.out = p->out;
  L.batch = p->batch;
  L.s = p->s;
  L.n_keys = p->n_keys;
  L.n_pad = n_pad;
  L.top_k = p->top_k;
  L.positions = p->positions;
  L.ratio = p->ratio;
  L.out_stride = p->out_stride;
  L.out_col = p->out_col;
  L.out_offset = p->out_offset;
  L.block_table = p->block_table;
  L.table_stride = p->table_stride;
  L.page = p->page;
  const int smem = p->n_keys * 4;
  static int attr_smem = 0;
  if (smem > 48 * 1024 && smem > attr_smem) {
    DSV4_CUDA_CHECK(cudaFuncSetAttribute(idx::select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         idx::SEL_MAX_KEYS * 4));
    attr_smem = idx::SEL_MAX_KEYS * 4;
  }
  idx::select_kernel<<<static_cast<unsigned>(rows), idx::SEL_THREADS, smem, as_stream(stream)>>>(L);
  DSV4_LAUNCH_CHECK("indexer select_kernel");
  return DSV4_OK;
}

extern "C" int dsv4_decode_window_indices(int32_t batch, int32_t window, const int32_t* positions,
                                          const int64_t* win_base, int32_t* out, int32_t out_stride,
                                          void* stream) {
  DSV4_CHECK_ARG(batch > 0 && window > 0 && positions && win_base && out && out_stride >= window,
                 "dsv4_decode_window_indices: bad arguments");
  idx::decode_window_kernel<<<batch, 128, 0, as_stream(stream)>>>(batch, window, positions, win_base,
                                                                    out, out_stride);
  DSV4_LAUNCH_CHECK("decode_window_kernel");
  return DSV4_OK;
}
