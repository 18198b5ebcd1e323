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
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "indexer_tc.cuh"

namespace dsv4 {
namespace idx {

constexpr int DI = 128;         // indexer head dim
constexpr int HI = 64;          // indexer heads
// keys per score CTA (decode): 56, so that 8192 keys take 147 CTAs, one per SM of the 148; the
// thread layout covers 64 key slots, the last eight of which are zero-filled and never stored
constexpr int KT = 56;
constexpr int KT_SLOTS = 64;
constexpr int THREADS = 256;

constexpr int SROW = DI + 4;   // padded row (floats): the 16 keys a half-warp reads hit distinct banks

struct ScoreSmem {
  alignas(16) float q[HI * SROW];        // [head][dim]
  alignas(16) float k[KT_SLOTS * SROW];  // [key slot][dim]
  alignas(16) float w[HI];
  float red[THREADS / 32][KT_SLOTS];     // tree level 0 per warp and key slot
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

// grid: (batch*s, key tiles of KT = 56). 256 threads: thread = (head quad hq, key lane kq) with
// lane = (hq & 1) << 4 | kq, warp = hq >> 1: a thread owns heads 4hq..4hq+3 and key slots kq, kq+16,
// kq+32, kq+48 of the tile, 16 accumulators; q and key rows are padded to 132 floats, so a half-warp's
// 16 keys read distinct banks. A 4-dim step loads 4 q chunks (two distinct per warp: shared-memory
// broadcasts) and 4 key chunks for 64 FMAs, so the step is bound by the FMA pipe rather than by
// shared-memory bandwidth. Per (head, key) the dot product is one sequential fmaf chain over the
// 128 dims; the thread's four heads fold (ascending) into the partial P[hq] of the canonical order,
// whose balanced tree is level 0 across lane bit 4 and levels 1-3 across warps.
__device__ __forceinline__ void score_tile(const ScoreParams& P, ScoreSmem& sm) {
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
  // four stages of 32 dims (eight 16-byte chunks of every q and key row), so the dot products
  // start on the first 32 dims while the rest are in flight
  // the head weights ride in the first group (a plain load would hold the thread until it lands)
  if (tid < HI / 4)
    cp_async16(static_cast<uint32_t>(__cvta_generic_to_shared(sm.w)) + tid * 16, P.w + qrow * HI + tid * 4, true);
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    for (int c = tid; c < HI * 8; c += THREADS) {
      const int r = c >> 3, ch = g * 8 + (c & 7);
      cp_async16(qs + (r * SROW + ch * 4) * 4, qg + r * DI + ch * 4, true);
    }
    for (int c = tid; c < KT_SLOTS * 8; c += THREADS) {
      const int r = c >> 3, ch = g * 8 + (c & 7);
      const bool valid = r < KT && (j0 + r) < nvis;
      const float* src = kg + static_cast<int64_t>(valid ? j0 + r : 0) * DI + ch * 4;
      cp_async16(ks + (r * SROW + ch * 4) * 4, src, valid);
    }
    asm volatile("cp.async.commit_group;\n" ::);
  }

  // thread: heads 4 hq .. 4 hq + 3, key slots kq, kq + 16, kq + 32, kq + 48
  const int hq = (warp << 1) | (lane >> 4), kq = lane & 15;
  const float* qrow_s = sm.q + hq * 4 * SROW;
  const float* krow_s = sm.k + kq * SROW;
  float acc[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[a][c] = 0.f;
  // (loops kept rolled: a kernel of a few microseconds runs on SMs whose instruction caches are
  // cold, and straight-line code would be fetched line by line)
#pragma unroll 1
  for (int g = 0; g < 4; ++g) {
    switch (g) {  // stage g has landed (with w in the first group)
      case 0: asm volatile("cp.async.wait_group 3;\n" ::); break;
      case 1: asm volatile("cp.async.wait_group 2;\n" ::); break;
      case 2: asm volatile("cp.async.wait_group 1;\n" ::); break;
      default: asm volatile("cp.async.wait_group 0;\n" ::); break;
    }
    __syncthreads();
#pragma unroll 2
    for (int st = 0; st < 8; ++st) {
      const int d = (g * 8 + st) * 4;
      float4 qv[4], kv[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) qv[a] = *reinterpret_cast<const float4*>(qrow_s + a * SROW + d);
#pragma unroll
      for (int c = 0; c < 4; ++c) kv[c] = *reinterpret_cast<const float4*>(krow_s + c * 16 * SROW + d);
      // dimension-major: x of all 16 (head, key) pairs, then y, z, w; every pair's chain still
      // runs over the dims in ascending order
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[a][c] = __fmaf_rn(qv[a].x, kv[c].x, acc[a][c]);
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[a][c] = __fmaf_rn(qv[a].y, kv[c].y, acc[a][c]);
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[a][c] = __fmaf_rn(qv[a].z, kv[c].z, acc[a][c]);
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[a][c] = __fmaf_rn(qv[a].w, kv[c].w, acc[a][c]);
    }
  }
  // P[hq] per key: the thread's four heads, ascending; tree level 0 across hq bit 0 (lane bit 4)
  float part[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    float p = 0.f;
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const float d = acc[a][c];
      p = __fmaf_rn(sm.w[hq * 4 + a], d > 0.f ? d : 0.f, p);
    }
    part[c] = __fadd_rn(p, __shfl_xor_sync(0xffffffffu, p, 16));
  }
  if (lane < 16) {
#pragma unroll
    for (int c = 0; c < 4; ++c) sm.red[warp][kq + 16 * c] = part[c];
  }
  __syncthreads();
  if (tid < KT) {  // levels 1-3: hq bits 1-3 are the warp's bits 0-2
    const int j = j0 + tid;
    const float l1a = __fadd_rn(sm.red[0][tid], sm.red[1][tid]), l1b = __fadd_rn(sm.red[2][tid], sm.red[3][tid]);
    const float l1c = __fadd_rn(sm.red[4][tid], sm.red[5][tid]), l1d = __fadd_rn(sm.red[6][tid], sm.red[7][tid]);
    const float v = __fadd_rn(__fadd_rn(l1a, l1b), __fadd_rn(l1c, l1d));
    if (j < nvis) P.scores[qrow * P.n_pad + j] = v;
  }
}

__global__ void __launch_bounds__(THREADS) score_kernel(ScoreParams P) {
  extern __shared__ __align__(16) uint8_t score_smem[];
  // wait first, then let the next kernel launch: the kernels launched after the scores (the
  // selection, then a decode attention that stages q and the window rows before its own wait) find
  // everything written before the scores complete
  pdl_wait();
  pdl_trigger();
  score_tile(P, *reinterpret_cast<ScoreSmem*>(score_smem));
}

// Query-tiled scores for prefill: one CTA per (64 queries, 64 keys) of one batch row, skipping tiles
// the causal rule hides entirely. The 64x128 key tile stays in shared memory while the 64 heads
// stream through: per head the query tile q[t0..t0+63][h][:] is staged with cp.async (double
// buffered); each thread computes 4 queries x 4 keys of dot products with sequential fmaf chains
// over the 128 dims and folds w[t][h] * relu(dot) into its head-group partial. Every four heads the
// partial enters a binary-counter tree, which forms exactly the balanced tree over the 16 partials
// of the canonical order (same pairs, same left/right operands).
constexpr int TQ = 64, TK = 64;

struct TiledSmem {
  alignas(16) float k[TK * DI];          // swizzled 16-byte chunks
  alignas(16) float q[2][TQ * DI];       // one head's query tile, double buffered
  float w[TQ * HI];                      // w[t][h] of the query tile
  int nvis[TQ];
};

__device__ __forceinline__ void add4x4(float (&dst)[4][4], const float (&a)[4][4], const float (&b)[4][4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) dst[i][j] = __fadd_rn(a[i][j], b[i][j]);
}

__global__ void __launch_bounds__(THREADS, 1) score_tiled_kernel(ScoreParams P) {
  extern __shared__ __align__(16) uint8_t tiled_smem[];
  TiledSmem& sm = *reinterpret_cast<TiledSmem*>(tiled_smem);
  // wait first, then let the next kernel launch: the kernels launched after the scores (the
  // selection, then a decode attention that stages q and the window rows before its own wait) find
  // everything written before the scores complete
  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.z;
  const int t0 = blockIdx.y * TQ;
  const int j0 = blockIdx.x * TK;
  const int64_t row0 = static_cast<int64_t>(b) * P.s + t0;           // first query row of the tile
  const int t_cnt = min(TQ, P.s - t0);
  if (tid < TQ) sm.nvis[tid] = tid < t_cnt ? visible_keys(P.positions, row0 + tid, P.ratio, P.n_keys) : 0;
  __syncthreads();
  int nvis_max = 0;
#pragma unroll 8
  for (int r = 0; r < TQ; ++r) nvis_max = max(nvis_max, sm.nvis[r]);
  if (j0 >= nvis_max) return;

  const float* kg = P.k + static_cast<int64_t>(b) * P.k_batch_stride * DI;
  const uint32_t ks = static_cast<uint32_t>(__cvta_generic_to_shared(sm.k));
  for (int c = tid; c < TK * DI / 4; c += THREADS) {
    const int r = c >> 5, ch = c & 31;
    const bool valid = (j0 + r) < nvis_max;
    cp_async16(ks + (r * 32 + swz_chunk(r, ch)) * 16, kg + static_cast<int64_t>(valid ? j0 + r : 0) * DI + ch * 4,
               valid);
  }
  const uint32_t qs0 = static_cast<uint32_t>(__cvta_generic_to_shared(sm.q[0]));
  const uint32_t qs1 = static_cast<uint32_t>(__cvta_generic_to_shared(sm.q[1]));
  auto stage_q = [&](int h, uint32_t qs) {
    for (int c = tid; c < TQ * DI / 4; c += THREADS) {
      const int r = c >> 5, ch = c & 31;
      const bool valid = r < t_cnt;
      const float* src = P.q + ((row0 + (valid ? r : 0)) * HI + h) * DI + ch * 4;
      cp_async16(qs + (r * 32 + swz_chunk(r, ch)) * 16, src, valid);
    }
  };
  stage_q(0, qs0);
  asm volatile("cp.async.commit_group;\n" ::);
  for (int c = tid; c < TQ * HI; c += THREADS) sm.w[c] = (c / HI) < t_cnt ? P.w[(row0 + c / HI) * HI + c % HI] : 0.f;

  // 16 x 16 thread grid; a warp covers 4 query groups x 8 key groups, so its shared-memory reads hit
  // 4 (broadcast) query rows and 8 key rows in distinct bank groups
  const int tq = ((warp >> 1) << 2) | (lane >> 3);
  const int tk = ((warp & 1) << 3) | (lane & 7);
  float part[4][4], l0[4][4], l1[4][4], l2[4][4], l3[4][4], fin[4][4];
#pragma unroll 1
  for (int h = 0; h < HI; ++h) {
    if (h + 1 < HI) {
      stage_q(h + 1, (h & 1) ? qs0 : qs1);
      asm volatile("cp.async.commit_group;\n" ::);
      asm volatile("cp.async.wait_group 1;\n" ::);
    } else {
      asm volatile("cp.async.wait_group 0;\n" ::);
    }
    __syncthreads();
    const float* qt = sm.q[h & 1];
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
        const int r = tq * 4 + a;
        qv[a] = *reinterpret_cast<const float4*>(&qt[(r * 32 + swz_chunk(r, ch)) * 4]);
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int r = tk * 4 + c;
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
    // fold this head into the group partial (heads 4m..4m+3, from +0)
    if ((h & 3) == 0) {
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int c = 0; c < 4; ++c) part[a][c] = 0.f;
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const float wv = sm.w[(tq * 4 + a) * HI + h];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float d = acc[a][c];
        part[a][c] = __fmaf_rn(wv, d > 0.f ? d : 0.f, part[a][c]);
      }
    }
    if ((h & 3) == 3) {
      const int m = h >> 2;  // head group just completed: binary-counter insert
      if (!(m & 1)) {
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int c = 0; c < 4; ++c) l0[a][c] = part[a][c];
      } else {
        add4x4(part, l0, part);
        if (!(m & 2)) {
#pragma unroll
          for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int c = 0; c < 4; ++c) l1[a][c] = part[a][c];
        } else {
          add4x4(part, l1, part);
          if (!(m & 4)) {
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
              for (int c = 0; c < 4; ++c) l2[a][c] = part[a][c];
          } else {
            add4x4(part, l2, part);
            if (!(m & 8)) {
#pragma unroll
              for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int c = 0; c < 4; ++c) l3[a][c] = part[a][c];
            } else {
              add4x4(fin, l3, part);
            }
          }
        }
      }
    }
    __syncthreads();  // q buffer (h & 1) is restaged two heads later
  }
  // write the visible scores of this thread's 4 queries x 4 keys
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int t = tq * 4 + a;
    if (t >= t_cnt) continue;
    const int nv = sm.nvis[t];
    const int j = j0 + tk * 4;
    float* dst = P.scores + (row0 + t) * P.n_pad + j;
    if (j + 4 <= nv && (P.n_pad & 3) == 0) {
      *reinterpret_cast<float4*>(dst) = make_float4(fin[a][0], fin[a][1], fin[a][2], fin[a][3]);
    } else {
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (j + c < nv) dst[c] = fin[a][c];
    }
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
  const int64_t* win_base;
  int32_t window, window_linear;
  // refinement of approximate scores (tensor-core filter): exact rescoring of the uncertain band
  int32_t refine;
  const float* q;         // [rows, 64, 128]
  const float* w;         // [rows, 64]
  const float* k;         // [batch, n_keys, 128], k_batch_stride rows apart
  int64_t k_batch_stride;
  const float* kmax;      // [batch] max key norm
  float eps_c;            // bound constant C of eps = C * sum_h |w_h| ||q_h|| * kmax
};

// window rows of a query at position p: decode ring order, or the prefill (linear) branch
__device__ __forceinline__ int32_t window_row(const SelectParams& P, int b, int p, int c) {
  const int W = P.window;
  int slot;
  if (P.window_linear) {
    const int lo = p - W + 1 > 0 ? p - W + 1 : 0;
    slot = (lo + c <= p) ? lo + c : -1;
  } else if (p >= W - 1) {
    const int sp = p % W;
    slot = (c < W - sp - 1) ? (sp + 1 + c) : (c - (W - sp - 1));
  } else {
    slot = (c <= p) ? c : -1;
  }
  return slot < 0 ? -1 : static_cast<int32_t>(P.win_base[b] + slot);
}

constexpr int SEL_THREADS = 512;
constexpr int SEL_MAX_KEYS = 32768;
constexpr int SEL_BINS = 4096;
constexpr int SEL_RANK_MAX = 1024;   // candidates resolved by O(c^2) rank counting up to this many
static_assert(SEL_BINS % SEL_THREADS == 0, "whole bins per thread");

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

// map_key for the PER contiguous keys j0 .. j0 + PER - 1 of one thread: with pages of at least PER
// keys they lie on at most two pages, whose table entries are read once up front (the writes of the
// selection then need no dependent global loads)
struct KeyMap {
  int64_t off0 = 0, off1 = 0;  // pool row - key index on the first / second page, + out_offset
  int split = 0x7fffffff;      // first key index on the second page
  bool direct;                 // false: map through map_key
  __device__ __forceinline__ KeyMap(const SelectParams& P, int b, int j0, int per) {
    direct = P.block_table == nullptr || P.page >= per;
    if (P.block_table == nullptr) {
      off0 = off1 = P.out_offset;
    } else if (direct) {
      const int last = max(0, P.table_stride - 1);
      const int pg0 = min(j0 / P.page, last);
      const int pg1 = min((j0 + per - 1) / P.page, last);
      const int32_t* t = P.block_table + static_cast<int64_t>(b) * P.table_stride;
      off0 = (static_cast<int64_t>(__ldg(t + pg0)) - pg0) * P.page + P.out_offset;
      off1 = (static_cast<int64_t>(__ldg(t + pg1)) - pg1) * P.page + P.out_offset;
      split = (pg0 + 1) * P.page;
    }
  }
  __device__ __forceinline__ int32_t map(const SelectParams& P, int b, int j) const {
    if (!direct) return map_key(P, b, j);
    return static_cast<int32_t>(j + (j < split ? off0 : off1));
  }
};

struct SelShared {
  uint32_t hist[SEL_BINS];
  uint32_t warp_sum[SEL_THREADS / 32];
  uint32_t cand_key[SEL_RANK_MAX];
  int32_t cand_idx[SEL_RANK_MAX];
  uint32_t n_cand, bin, need, tau;
  int32_t tau_last;
  uint32_t total;
};

// exclusive prefix sum over the block (3 barriers); sh.total receives the block sum
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, SelShared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) sh.warp_sum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const uint32_t w = lane < SEL_THREADS / 32 ? sh.warp_sum[lane] : 0u;
    uint32_t wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += t;
    }
    if (lane < SEL_THREADS / 32) sh.warp_sum[lane] = wi - w;
    if (lane == 31) sh.total = wi;
  }
  __syncthreads();
  const uint32_t r = sh.warp_sum[warp] + incl - v;
  __syncthreads();
  return r;
}

// One CTA per query. (1) the visible scores are loaded (independent vector loads) into shared memory
// as order-preserving keys; (2) a 4096-bin histogram of their top 12 bits gives the boundary bin:
// keys in higher bins are taken, lower bins dropped; (3) the boundary bin is resolved exactly — by
// rank counting over (key desc, index asc) when it holds at most 1024 keys, else by radix passes
// over its remaining bits; (4) the taken keys are written in ascending index order through a block
// prefix sum, mapped to pool rows.
__global__ void __launch_bounds__(SEL_THREADS) select_kernel(SelectParams P) {
  extern __shared__ uint32_t keys[];  // [nvis] ordered scores
  __shared__ SelShared sh;
  pdl_trigger();
  pdl_wait();
  const int tid = threadIdx.x;
  const int64_t qrow = blockIdx.x;
  const int b = static_cast<int>(qrow / P.s);
  const int nvis = visible_keys(P.positions, qrow, P.ratio, P.n_keys);
  int32_t* out = P.out + qrow * P.out_stride + P.out_col;
  const int k = P.top_k;

  if (P.win_base != nullptr)
    for (int c = tid; c < P.window; c += SEL_THREADS) out[c - P.window] = window_row(P, b, P.positions[qrow], c);
  if (nvis <= k) {
    for (int r = tid; r < k; r += SEL_THREADS) out[r] = r < nvis ? map_key(P, b, r) : -1;
    return;
  }
  // (1) load
  const float* sc = P.scores + qrow * P.n_pad;
  if ((P.n_pad & 3) == 0) {
    const int n4 = nvis >> 2;
#pragma unroll 4
    for (int c = tid; c < n4; c += SEL_THREADS) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(sc) + c);
      *reinterpret_cast<uint4*>(keys + 4 * c) =
          make_uint4(ordered_bits(v.x), ordered_bits(v.y), ordered_bits(v.z), ordered_bits(v.w));
    }
    for (int j = 4 * n4 + tid; j < nvis; j += SEL_THREADS) keys[j] = ordered_bits(__ldcg(sc + j));
  } else {
#pragma unroll 4
    for (int j = tid; j < nvis; j += SEL_THREADS) keys[j] = ordered_bits(__ldcg(sc + j));
  }
#pragma unroll
  for (int i = 0; i < SEL_BINS / SEL_THREADS; ++i) sh.hist[tid + i * SEL_THREADS] = 0;
  if (tid == 0) sh.n_cand = 0;
  __syncthreads();
  // (2) histogram of the top 12 bits, then the boundary bin
  for (int j = tid; j < nvis; j += SEL_THREADS) atomicAdd(&sh.hist[keys[j] >> 20], 1u);
  __syncthreads();
  {
    constexpr int PER = SEL_BINS / SEL_THREADS;  // bins per thread, descending
    uint32_t c[PER], tot = 0;
#pragma unroll
    for (int e = 0; e < PER; ++e) {
      c[e] = sh.hist[SEL_BINS - 1 - (tid * PER + e)];
      tot += c[e];
    }
    const uint32_t before = block_exclusive_scan(tot, sh);
    if (before < static_cast<uint32_t>(k) && static_cast<uint32_t>(k) <= before + tot) {
      uint32_t run = before;
#pragma unroll
      for (int e = 0; e < PER; ++e) {
        if (run + c[e] >= static_cast<uint32_t>(k)) {
          sh.bin = SEL_BINS - 1 - (tid * PER + e);
          sh.need = k - run;
          break;
        }
        run += c[e];
      }
    }
  }
  __syncthreads();
  const uint32_t bin = sh.bin;
  const uint32_t need = sh.need;
  // (3) resolve the boundary bin
  if (sh.hist[bin] <= SEL_RANK_MAX) {
    for (int j = tid; j < nvis; j += SEL_THREADS) {
      const uint32_t key = keys[j];
      if ((key >> 20) == bin) {
        const uint32_t slot = atomicAdd(&sh.n_cand, 1u);
        sh.cand_key[slot] = key;
        sh.cand_idx[slot] = j;
      }
    }
    __syncthreads();
    const uint32_t c = sh.n_cand;
    for (uint32_t i = tid; i < c; i += SEL_THREADS) {
      const uint32_t ki = sh.cand_key[i];
      const int32_t ii = sh.cand_idx[i];
      uint32_t rank = 0;
#pragma unroll 4
      for (uint32_t m = 0; m < c; ++m) {
        const uint32_t km = sh.cand_key[m];
        rank += (km > ki) || (km == ki && sh.cand_idx[m] < ii);
      }
      if (rank == need - 1) {  // the last key taken
        sh.tau = ki;
        sh.tau_last = ii;      // keys equal to tau are taken up to this index
      }
    }
  } else {
    // a crowded boundary bin (e.g. heavy ties): radix passes over its bits 19..12, 11..4, 3..0
    uint32_t prefix = bin << 20, kleft = need;
    const int shifts[3] = {12, 4, 0}, widths[3] = {8, 8, 4};
#pragma unroll 1
    for (int ps = 0; ps < 3; ++ps) {
      const int shift = shifts[ps], width = widths[ps], hi = shift + width;
      const uint32_t mask = (1u << width) - 1u;
      if (tid < 256) sh.hist[tid] = 0;
      __syncthreads();
      for (int j = tid; j < nvis; j += SEL_THREADS) {
        const uint32_t key = keys[j];
        if ((key >> hi) == (prefix >> hi)) atomicAdd(&sh.hist[(key >> shift) & mask], 1u);
      }
      __syncthreads();
      if (tid == 0) {
        uint32_t run = 0;
        for (int d = static_cast<int>(mask); d >= 0; --d) {
          if (run + sh.hist[d] >= kleft) {
            sh.bin = d;
            sh.need = kleft - run;
            break;
          }
          run += sh.hist[d];
        }
      }
      __syncthreads();
      prefix |= sh.bin << shift;
      kleft = sh.need;
      __syncthreads();
    }
    // the kleft-th key (in index order) equal to prefix is the last one taken
    const int per = (nvis + SEL_THREADS - 1) / SEL_THREADS;
    const int jb = tid * per, je = min(nvis, jb + per);
    uint32_t ne = 0;
    for (int j = jb; j < je; ++j) ne += keys[j] == prefix;
    const uint32_t before = block_exclusive_scan(ne, sh);
    if (before < kleft && kleft <= before + ne) {
      uint32_t seen = before;
      for (int j = jb; j < je; ++j)
        if (keys[j] == prefix && ++seen == kleft) {
          sh.tau_last = j;
          break;
        }
    }
    if (tid == 0) sh.tau = prefix;
  }
  __syncthreads();
  const uint32_t tau = sh.tau;
  const int32_t tau_last = sh.tau_last;
  // (4) index-ordered compaction of {key > tau} U {key == tau, index <= tau_last}
  const int per = (nvis + SEL_THREADS - 1) / SEL_THREADS;
  const int jb = tid * per, je = min(nvis, jb + per);
  uint32_t cnt = 0;
  for (int j = jb; j < je; ++j) {
    const uint32_t key = keys[j];
    cnt += (key > tau) || (key == tau && j <= tau_last);
  }
  uint32_t pos = block_exclusive_scan(cnt, sh);
  for (int j = jb; j < je; ++j) {
    const uint32_t key = keys[j];
    if ((key > tau) || (key == tau && j <= tau_last)) out[pos++] = map_key(P, b, j);
  }
}

// Register-resident selection for up to SEL_THREADS * PER visible keys: thread t holds keys
// [t*PER, t*PER + PER) in registers (so every pass is in index order without shared-memory
// traffic). MSB-first radix over the order-preserving key: 12 bits, then 8, 8 and 4 more, each level
// histogramming only the keys that still match the prefix (shared-memory atomics). A level
// whose boundary bin is taken whole ends the search early; otherwise after all 32 bits the keys equal
// to the threshold are taken lowest index first. The taken keys are written in ascending order.
struct SelRegShared {
  alignas(16) uint32_t hist[SEL_BINS];
  uint32_t warp_sum[SEL_THREADS / 32];
  uint32_t total, bin, need;
  int32_t tau_last;
  uint32_t ncand, tau_key;
};

__device__ __forceinline__ uint32_t block_scan_reg(uint32_t v, SelRegShared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) sh.warp_sum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const uint32_t w = lane < SEL_THREADS / 32 ? sh.warp_sum[lane] : 0u;
    uint32_t wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += t;
    }
    if (lane < SEL_THREADS / 32) sh.warp_sum[lane] = wi - w;
    if (lane == 31) sh.total = wi;
  }
  __syncthreads();
  const uint32_t r = sh.warp_sum[warp] + incl - v;
  __syncthreads();
  return r;
}

// add 1 to hist[bin] when bin < nbins (plain shared atomics: grouping lanes by bin first with
// __match_any_sync measured several times slower on B200 than the conflicting atomics it saves)
__device__ __forceinline__ void warp_hist_add(uint32_t* hist, uint32_t bin, uint32_t nbins) {
  if (bin < nbins) atomicAdd(&hist[bin], 1u);
}

// Radix levels over the order-preserving keys (12, 8, 8 and 4 bits, most significant first) that
// locate the boundary of the top k. With stop_whole, a level whose boundary bin is taken whole ends
// the search (prefix then fixes the bits at and above shift); without it the search runs down to
// shift 0 and prefix is the k-th largest key itself. kleft = keys still needed from the boundary.
// max_levels < 4 stops early: the k-th largest key then lies in [prefix, prefix + 2^shift).
template <int PER>
__device__ __forceinline__ void radix_levels(const uint32_t (&key)[PER], int nv, uint32_t k, bool stop_whole,
                                             SelRegShared& sh, uint32_t& prefix, uint32_t& shift, uint32_t& kleft,
                                             bool& whole, int max_levels = 4) {
  const int tid = threadIdx.x, lane = tid & 31;

#pragma unroll
  for (int i = 0; i < SEL_BINS / SEL_THREADS; ++i) sh.hist[tid + i * SEL_THREADS] = 0;
  __syncthreads();
  // level 1: top 12 bits
#pragma unroll
  for (int e = 0; e < PER; ++e) warp_hist_add(sh.hist, e < nv ? (key[e] >> 20) : 0xffffffffu, SEL_BINS);
  __syncthreads();
  shift = 20;
  whole = false;
  {
    constexpr int PB = SEL_BINS / SEL_THREADS;
    static_assert(PB == 8, "two 16-byte reads per thread");
    uint32_t c[PB], tot = 0;
    {
      // this thread's 8 bins, highest first, read as two 16-byte vectors
      const uint4* h4 = reinterpret_cast<const uint4*>(sh.hist + SEL_BINS - PB * (tid + 1));
      const uint4 lo4 = h4[0], hi4 = h4[1];
      c[0] = hi4.w; c[1] = hi4.z; c[2] = hi4.y; c[3] = hi4.x;
      c[4] = lo4.w; c[5] = lo4.z; c[6] = lo4.y; c[7] = lo4.x;
#pragma unroll
      for (int e = 0; e < PB; ++e) tot += c[e];
    }
    const uint32_t before = block_scan_reg(tot, sh);
    if (before < k && k <= before + tot) {
      uint32_t run = before;
#pragma unroll
      for (int e = 0; e < PB; ++e) {
        if (run + c[e] >= k) {
          const uint32_t bn = SEL_BINS - 1 - (tid * PB + e);
          sh.bin = bn;
          sh.need = (k - run) | ((c[e] == k - run) ? 0x80000000u : 0u);  // top bit: bin taken whole
          break;
        }
        run += c[e];
      }
    }
    __syncthreads();
    prefix = sh.bin << 20;
    kleft = sh.need & 0x7fffffffu;
    whole = (sh.need >> 31) != 0;
  }
  // levels 2..4 over the keys inside the boundary bin: bits 19..12, 11..4, 3..0
#pragma unroll 1
  for (int level = 0; level < max_levels - 1 && !(whole && stop_whole); ++level) {
    const uint32_t width = level < 2 ? 8u : 4u;
    const uint32_t nshift = shift - width;
    const uint32_t nb = 1u << width;
    if (tid < 256) sh.hist[tid] = 0;
    __syncthreads();
#pragma unroll
    for (int e = 0; e < PER; ++e) {
      const bool in = e < nv && (key[e] >> shift) == (prefix >> shift);
      warp_hist_add(sh.hist, in ? ((key[e] >> nshift) & (nb - 1)) : 0xffffffffu, nb);
    }
    __syncthreads();
    if (tid < 32) {
      // lane l owns sub-bins [nb-1-l*8, nb-8-l*8] (descending); nb <= 256
      const int per = (nb + 31) / 32;
      uint32_t cnt[8], tot = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int d = static_cast<int>(nb) - 1 - (lane * per + e);
        cnt[e] = (e < per && d >= 0) ? sh.hist[d] : 0u;
        tot += cnt[e];
      }
      uint32_t incl = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      const uint32_t before = incl - tot;
      if (before < kleft && kleft <= incl) {
        uint32_t run = before;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (e < per && run + cnt[e] >= kleft) {
            sh.bin = static_cast<uint32_t>(static_cast<int>(nb) - 1 - (lane * per + e));
            sh.need = (kleft - run) | ((cnt[e] == kleft - run) ? 0x80000000u : 0u);
            break;
          }
          run += cnt[e];
        }
      }
    }
    __syncthreads();
    prefix |= sh.bin << nshift;
    kleft = sh.need & 0x7fffffffu;
    whole = (sh.need >> 31) != 0;
    shift = nshift;
    __syncthreads();
  }
}


constexpr int BAND_CAP = 512;  // band keys rescored per round
constexpr int STAGE_ROWS = 128;  // band key rows staged in shared memory at a time (128: every
                                // thread has a 4-key x 4-head task, and most bands take one round)
constexpr int OUT_STAGE = 2048;  // selections up to this size leave through shared memory
constexpr float EPS_C = 0x1p-14f;

struct RefineSmem {
  float4 q[HI * DI / 4];   // the query's 64 x 128 indexer q; chunk c of head h at c ^ ((h / 4) % 8)
  float w[HI];
  float wq[HI];
  float4 krow[STAGE_ROWS][DI / 4];  // band key rows staged for the exact rescoring
  int32_t band_idx[BAND_CAP];
  float band_e[BAND_CAP];
  uint8_t band_take[BAND_CAP];
  int32_t out_stage[OUT_STAGE];
  float eps;
};

__device__ __forceinline__ float from_ordered(uint32_t u) {
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

// Exact refinement of approximate scores A with |A - score| <= eps for every key (eps from the
// query's |w_h| ||q_h|| and the largest key norm). With v the k-th largest A, bracketed as
// lo <= v <= hi by two radix levels (20 of the 32 key bits):
//  - a key with A > hi + 2 eps is in the top k: any key that ties or beats it has
//    A >= score - eps >= its score - eps > v, and fewer than k keys have A > v;
//  - a key with A < lo - 2 eps is not: the k keys with A >= v all have score >= v - eps > its score.
// Keys in between (the band; at least k minus the certain count of them, since every key with
// A >= v is there or certain) get their exact score in the canonical fp32 order. When the band fits
// one round (BAND_CAP keys) the missing keys are taken from it by rank, (score desc, index asc), and
// the result is written here (returns true). A wider band leaves the certain keys pinned to the
// largest / smallest ordered key and the band keys holding their exact scores, for the ordinary
// selection that follows (returns false). Valid for finite inputs (see the error analysis of the
// approximate scores).
// Exact scores of band entries rs.band_idx[0, cnt) into rs.band_e (the canonical fp32 order),
// STAGE_ROWS key rows at a time staged in shared memory: task = (4 band entries, head quad); the
// 16 lanes of a quad set form the partial tree. Each thread keeps 4 heads x 4 keys of fmaf chains,
// so a q chunk serves 4 keys and a key chunk 4 heads. Ends with the block synchronised.
__device__ __forceinline__ void rescore_band(const float* kb, int cnt, RefineSmem& rs) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int s0 = 0; s0 < cnt; s0 += STAGE_ROWS) {
    const int rows = min(STAGE_ROWS, cnt - s0);
    {
      const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(&rs.krow[0][0]));
      for (int i = tid; i < rows * (DI / 4); i += SEL_THREADS) {
        const int r = i >> 5, c = i & 31;
        cp_async16(dst + static_cast<uint32_t>(i) * 16,
                   kb + static_cast<int64_t>(rs.band_idx[s0 + r]) * DI + c * 4, true);
      }
      asm volatile("cp.async.commit_group;\n" ::);
      asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    }
    __syncthreads();
    const int n_groups = (rows + 3) >> 2;
    for (int base = warp * 32; base < n_groups * 16; base += SEL_THREADS) {
      const int task = base + lane;
      const int grp = task >> 4, quad = task & 15;
      const bool valid = grp < n_groups;
      const int m0 = grp * 4;  // within the stage
      int rr[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) rr[e] = (valid && m0 + e < rows) ? m0 + e : 0;
      const int h0 = quad * 4, sw = quad & 7;
      float d[4][4];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int e = 0; e < 4; ++e) d[a][e] = 0.f;
      if (valid) {
#pragma unroll 4
        for (int c = 0; c < DI / 4; ++c) {
          float4 kv[4], qv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) kv[e] = rs.krow[rr[e]][c];
#pragma unroll
          for (int a = 0; a < 4; ++a) qv[a] = rs.q[(h0 + a) * 32 + (c ^ sw)];
#pragma unroll
          for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              d[a][e] = __fmaf_rn(qv[a].x, kv[e].x, d[a][e]);
              d[a][e] = __fmaf_rn(qv[a].y, kv[e].y, d[a][e]);
              d[a][e] = __fmaf_rn(qv[a].z, kv[e].z, d[a][e]);
              d[a][e] = __fmaf_rn(qv[a].w, kv[e].w, d[a][e]);
            }
        }
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float part = 0.f;
#pragma unroll
        for (int a = 0; a < 4; ++a) part = __fmaf_rn(rs.w[h0 + a], d[a][e] > 0.f ? d[a][e] : 0.f, part);
        // balanced tree over the 16 partials: pairs (2t, 2t+1) at every level
        part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, 1));
        part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, 2));
        part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, 4));
        part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, 8));
        if (valid && quad == 0 && m0 + e < rows) rs.band_e[s0 + m0 + e] = part;
      }
    }
    __syncthreads();  // krow reuse
  }
  __syncthreads();
}

template <int PER>
__device__ __forceinline__ bool refine_band(const SelectParams& P, int64_t qrow, int b, int k, uint32_t (&key)[PER],
                                            int nv, int j0, SelRegShared& sh, RefineSmem& rs, int32_t* out,
                                            const KeyMap& km) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // the query's q (64 x 128) streams into shared memory while the radix runs
  {
    const float* qg = P.q + qrow * (HI * DI);
    const uint32_t qs = static_cast<uint32_t>(__cvta_generic_to_shared(rs.q));
    for (int i = tid; i < HI * DI / 4; i += SEL_THREADS) {
      const int h = i >> 5, c = i & 31;
      cp_async16(qs + static_cast<uint32_t>(h * 32 + (c ^ ((h >> 2) & 7))) * 16, qg + i * 4, true);
    }
    asm volatile("cp.async.commit_group;\n" ::);
  }
  if (tid < HI) rs.w[tid] = P.w[qrow * HI + tid];
  // bracket [lo, hi] of the k-th largest approximate score: the first two radix levels (20 bits)
  uint32_t pfx, shift, kleft;
  bool whole;
  radix_levels<PER>(key, nv, static_cast<uint32_t>(k), false, sh, pfx, shift, kleft, whole, 2);
  const float lo = from_ordered(pfx), hi = from_ordered(pfx | ((1u << shift) - 1u));
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
  __syncthreads();
  {  // |w_h| * ||q_h||: 8 threads per head
    const int h = tid >> 3, part = tid & 7;
    float ss = 0.f;
#pragma unroll
    for (int c = part * 4; c < part * 4 + 4; ++c) {
      const float4 v = rs.q[h * 32 + (c ^ ((h >> 2) & 7))];
      ss = fmaf(v.x, v.x, ss);
      ss = fmaf(v.y, v.y, ss);
      ss = fmaf(v.z, v.z, ss);
      ss = fmaf(v.w, v.w, ss);
    }
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
    ss += __shfl_xor_sync(0xffffffffu, ss, 4);
    if (part == 0) rs.wq[h] = fabsf(rs.w[h]) * sqrtf(ss);
  }
  __syncthreads();
  if (warp == 0) {
    float t = rs.wq[lane] + rs.wq[lane + 32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    // the factor covers the fp32 rounding of the norms and sums above
    if (lane == 0) rs.eps = P.eps_c * t * P.kmax[b] * (1.f + 0x1p-10f) + 1e-30f;
  }
  __syncthreads();
  const float e2 = 2.f * rs.eps;
  const float upper = __fadd_ru(hi, e2), lower = __fsub_rd(lo, e2);
  uint32_t band = 0, inm = 0, nb = 0, nin = 0;
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    if (e < nv) {
      const float a = from_ordered(key[e]);
      if (a > upper) {
        key[e] = 0xffffffffu;
        inm |= 1u << e;
        ++nin;
      } else if (a < lower) {
        key[e] = 0u;
      } else {
        band |= 1u << e;
        ++nb;
      }
    }
  }
  // one scan of both counts (band in the low 16 bits, certain in the high 16; each <= 16384)
  const uint32_t both = block_scan_reg(nb | (nin << 16), sh);
  const uint32_t pos0 = both & 0xffffu;
  const uint32_t n_band = sh.total & 0xffffu;
  const uint32_t n_in = sh.total >> 16;
  const float* kb = P.k + static_cast<int64_t>(b) * P.k_batch_stride * DI;
  if (n_band <= static_cast<uint32_t>(BAND_CAP)) {
    // one round; from here on the per-key state is the two bit masks
    {
      uint32_t pos = pos0;
#pragma unroll
      for (int e = 0; e < PER; ++e)
        if ((band >> e) & 1u) rs.band_idx[pos++] = j0 + e;
    }
    __syncthreads();
    rescore_band(kb, static_cast<int>(n_band), rs);
    // take the (k - n_in) best band entries by (score desc, index asc); entries are in ascending key
    // order, so the index order is the entry order. Warp w ranks entries w, w + 16, ...; its lanes
    // split the comparisons.
    const uint32_t need = static_cast<uint32_t>(k) - n_in;
    for (int m = warp; m < static_cast<int>(n_band); m += SEL_THREADS / 32) {
      const uint32_t km = ordered_bits(rs.band_e[m]);
      uint32_t rank = 0;
      for (int m2 = lane; m2 < static_cast<int>(n_band); m2 += 32) {
        const uint32_t k2 = ordered_bits(rs.band_e[m2]);
        rank += (k2 > km) || (k2 == km && m2 < m);
      }
      rank = __reduce_add_sync(0xffffffffu, rank);
      if (lane == 0) rs.band_take[m] = rank < need ? 1 : 0;
    }
    __syncthreads();
    // the taken keys in ascending order (certain ones and the chosen band entries), staged in shared
    // memory so that the list leaves in coalesced stores
    uint32_t take = inm;
    {
      uint32_t pos = pos0;
#pragma unroll
      for (int e = 0; e < PER; ++e)
        if ((band >> e) & 1u) {
          if (rs.band_take[pos]) take |= 1u << e;
          ++pos;
        }
    }
    uint32_t o = block_scan_reg(static_cast<uint32_t>(__popc(take)), sh);
    const bool staged = k <= OUT_STAGE;
#pragma unroll
    for (int e = 0; e < PER; ++e)
      if ((take >> e) & 1u) {
        const int32_t v = km.map(P, b, j0 + e);
        if (staged) rs.out_stage[o] = v;
        else out[o] = v;
        ++o;
      }
    if (staged) {
      __syncthreads();
      for (int r = tid; r < k; r += SEL_THREADS) out[r] = rs.out_stage[r];
    }
    return true;
  }
  // a wide band (many equal or near-equal scores): rounds of BAND_CAP, the band keys taking their
  // exact scores, for the ordinary selection that follows over the pinned keys
  for (uint32_t r0 = 0; r0 < n_band; r0 += BAND_CAP) {
    const uint32_t cnt = min(static_cast<uint32_t>(BAND_CAP), n_band - r0);
    {
      uint32_t pos = pos0;
#pragma unroll
      for (int e = 0; e < PER; ++e)
        if ((band >> e) & 1u) {
          if (pos >= r0 && pos < r0 + cnt) rs.band_idx[pos - r0] = j0 + e;
          ++pos;
        }
    }
    __syncthreads();
    rescore_band(kb, static_cast<int>(cnt), rs);
    {
      uint32_t pos = pos0;
#pragma unroll
      for (int e = 0; e < PER; ++e)
        if ((band >> e) & 1u) {
          if (pos >= r0 && pos < r0 + cnt) key[e] = ordered_bits(rs.band_e[pos - r0]);
          ++pos;
        }
    }
    __syncthreads();
  }
  return false;
}

template <int PER, bool REFINE>
__global__ void __launch_bounds__(SEL_THREADS) select_reg_kernel(SelectParams P) {
  __shared__ SelRegShared sh;
  extern __shared__ __align__(16) uint8_t sel_dyn[];
  pdl_trigger();
  pdl_wait();
  const int tid = threadIdx.x;
  const int64_t qrow = blockIdx.x;
  const int b = static_cast<int>(qrow / P.s);
  const int j0 = tid * PER;
  // the scores and the block table entries load before the visible count is known (the three
  // global reads overlap): reads stay inside the row's n_pad entries, and keys at or past the
  // visible count are never counted
  const float* sc = P.scores + qrow * P.n_pad + j0;
  uint32_t key[PER];
  if ((P.n_pad & 3) == 0 && j0 + PER <= P.n_pad) {
#pragma unroll
    for (int e = 0; e < PER; e += 4) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(sc + e));
      key[e] = ordered_bits(v.x);
      key[e + 1] = ordered_bits(v.y);
      key[e + 2] = ordered_bits(v.z);
      key[e + 3] = ordered_bits(v.w);
    }
  } else {
#pragma unroll
    for (int e = 0; e < PER; ++e) key[e] = (j0 + e < P.n_pad) ? ordered_bits(__ldcg(sc + e)) : 0u;
  }
  const KeyMap km(P, b, j0, PER);
  if (tid == 0) sh.ncand = 0;  // ordered before its use by the radix level's barriers
  const int nvis = visible_keys(P.positions, qrow, P.ratio, P.n_keys);
  int32_t* out = P.out + qrow * P.out_stride + P.out_col;
  const int k = P.top_k;

  if (P.win_base != nullptr)
    for (int c = tid; c < P.window; c += SEL_THREADS) out[c - P.window] = window_row(P, b, P.positions[qrow], c);
  if (nvis <= k) {
    for (int r = tid; r < k; r += SEL_THREADS) out[r] = r < nvis ? map_key(P, b, r) : -1;
    return;
  }
  // number of valid keys of this thread (the rest are padding and never counted)
  const int nv = max(0, min(PER, nvis - j0));
  if constexpr (REFINE) {
    if (refine_band<PER>(P, qrow, b, k, key, nv, j0, sh, *reinterpret_cast<RefineSmem*>(sel_dyn), out, km)) return;
  }
  uint32_t prefix, kleft, shift;
  bool whole;
  int32_t tau_last = 0x7fffffff;
  // The top 12 bits first. When the boundary bin holds at most SEL_THREADS keys (the usual case:
  // ~n / 4096 keys per bin), its keys are ranked directly by (key desc, index asc) instead of
  // histogramming the lower bits: the kleft-th of them is the threshold (key, index).
  radix_levels<PER>(key, nv, static_cast<uint32_t>(k), true, sh, prefix, shift, kleft, whole, 1);
  bool ranked = false;
  if (!whole) {
    uint64_t* cand = reinterpret_cast<uint64_t*>(sh.hist);  // the histogram is free after the level
    const uint32_t top = prefix >> shift;
#pragma unroll
    for (int e = 0; e < PER; ++e)
      if (e < nv && (key[e] >> shift) == top) {
        const uint32_t slot = atomicAdd(&sh.ncand, 1u);
        if (slot < SEL_THREADS)
          cand[slot] = (static_cast<uint64_t>(key[e]) << 32) | static_cast<uint32_t>(~static_cast<uint32_t>(j0 + e));
      }
    __syncthreads();
    const uint32_t nc = sh.ncand;
    if (nc <= SEL_THREADS) {
      if (tid < static_cast<int>(nc)) {
        const uint64_t v = cand[tid];
        uint32_t rank = 0;
        for (uint32_t m = 0; m < nc; ++m) rank += cand[m] > v;
        if (rank == kleft - 1) {
          sh.tau_key = static_cast<uint32_t>(v >> 32);
          sh.tau_last = static_cast<int32_t>(~static_cast<uint32_t>(v));
        }
      }
      __syncthreads();
      prefix = sh.tau_key;
      tau_last = sh.tau_last;
      shift = 0;
      ranked = true;
    } else {  // a crowded bin (many equal or near-equal scores): the remaining radix levels
      radix_levels<PER>(key, nv, static_cast<uint32_t>(k), true, sh, prefix, shift, kleft, whole);
    }
  }
  // keys equal to the full 32-bit prefix (shift == 0, not whole): the kleft lowest indices
  if (!whole && !ranked) {
    uint32_t ne = 0;
#pragma unroll
    for (int e = 0; e < PER; ++e) ne += (e < nv && key[e] == prefix);
    const uint32_t before = block_scan_reg(ne, sh);
    if (before < kleft && kleft <= before + ne) {
      uint32_t seen = before;
#pragma unroll
      for (int e = 0; e < PER; ++e)
        if (e < nv && key[e] == prefix && ++seen == kleft) sh.tau_last = j0 + e;
    }
    __syncthreads();
    tau_last = sh.tau_last;
  }
  // take: (key >> shift) above the prefix, or equal to it and (whole, or index <= tau_last)
  const uint32_t hi = prefix >> shift;
  uint32_t take = 0;
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    const uint32_t kh = key[e] >> shift;
    take |= static_cast<uint32_t>((e < nv) && (kh > hi || (kh == hi && (whole || j0 + e <= tau_last)))) << e;
  }
  uint32_t pos = block_scan_reg(static_cast<uint32_t>(__popc(take)), sh);
  while (take) {  // the taken keys in ascending order
    const int e = __ffs(take) - 1;
    take &= take - 1;
    out[pos++] = km.map(P, b, j0 + e);
  }
}

// ---- selection for decode-sized calls (few query rows): one 1024-thread CTA per row ----------
// The keys' order-preserving images are binned linearly over [min, max] of the visible keys (a
// shift of key - min into 12 bits) instead of by their top 12 bits: the top bits of fp32 scores
// put most keys of a row into a handful of bins (3 mantissa bits per binade), while the linear bins
// leave a few keys in the boundary bin, which are then ranked directly by (key desc, index asc).
// A boundary bin with more than LIN_CAND keys narrows the range to that bin and bins again; a range
// of one value (equal scores) takes its kleft lowest indices. Same set as the oracle's sort, written
// in ascending key order.
constexpr int LIN_THREADS = 512;     // threads of the selection CTA (16 to 32 warps both work)
constexpr int LIN_BINS = 4096;
constexpr int LIN_CAND = 1024;
constexpr int LIN_MAX_ROWS = 32;     // rows per call served by this kernel

struct LinShared {
  alignas(16) uint32_t hist[LIN_BINS];
  unsigned long long cand[LIN_CAND];
  uint32_t wa[32], wb[32];
  uint32_t bin, kleft, count, ncand;
  unsigned long long thr;
  int32_t tau_idx;
};

// exclusive prefix sum over the NT threads (2 barriers, plus one before the scratch is reused)
template <int NT>
__device__ __forceinline__ uint32_t lin_scan(uint32_t v, LinShared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) sh.wa[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const uint32_t w = lane < NT / 32 ? sh.wa[lane] : 0u;
    uint32_t wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += t;
    }
    sh.wb[lane] = wi - w;
  }
  __syncthreads();
  return sh.wb[warp] + incl - v;
}

// the selection of query row qrow by the NT threads of a CTA, PER keys per thread
template <int PER, int NT>
__device__ __forceinline__ void select_lin_row(const SelectParams& P, int64_t qrow, LinShared& sh) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = static_cast<int>(qrow / P.s);
  const int j0 = tid * PER;
  const int nvis = visible_keys(P.positions, qrow, P.ratio, P.n_keys);
  const float* sc = P.scores + qrow * P.n_pad + j0;
  uint32_t key[PER];
  if ((P.n_pad & 3) == 0 && j0 + PER <= P.n_pad) {
#pragma unroll
    for (int e = 0; e < PER; e += 4) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(sc + e));
      key[e] = ordered_bits(v.x);
      key[e + 1] = ordered_bits(v.y);
      key[e + 2] = ordered_bits(v.z);
      key[e + 3] = ordered_bits(v.w);
    }
  } else {
#pragma unroll
    for (int e = 0; e < PER; ++e) key[e] = (j0 + e < P.n_pad) ? ordered_bits(__ldcg(sc + e)) : 0u;
  }
  const KeyMap km(P, b, j0, PER);
  int32_t* out = P.out + qrow * P.out_stride + P.out_col;
  const uint32_t k = static_cast<uint32_t>(P.top_k);
  if (P.win_base != nullptr)
    for (int c = tid; c < P.window; c += NT) out[c - P.window] = window_row(P, b, P.positions[qrow], c);
  if (nvis <= P.top_k) {
    for (int r = tid; r < P.top_k; r += NT) out[r] = r < nvis ? map_key(P, b, r) : -1;
    return;
  }
  const int nv = max(0, min(PER, nvis - j0));  // this thread's visible keys; the rest never count

  // min and max of the visible keys
  uint32_t mn = 0xffffffffu, mx = 0u;
#pragma unroll
  for (int e = 0; e < PER; ++e)
    if (e < nv) {
      mn = min(mn, key[e]);
      mx = max(mx, key[e]);
    }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  if (lane == 0) {
    sh.wa[warp] = mn;
    sh.wb[warp] = mx;
  }
#pragma unroll
  for (int i = tid; i < LIN_BINS; i += NT) sh.hist[i] = 0;
  __syncthreads();
  // every warp folds the per-warp partials itself (lane w takes warp w's), no second barrier
  uint32_t lo = lane < NT / 32 ? sh.wa[lane] : 0xffffffffu;
  uint32_t hi = lane < NT / 32 ? sh.wb[lane] : 0u;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  uint32_t kleft = k;
  unsigned long long thr = 0;   // (key << 32) | ~index of the k-th largest: take every key >= it
  bool found = false;
  // each pass narrows [lo, hi] to the boundary bin (a 4096th of the range or less); at most 4 passes
  // reach a single value
  for (int pass = 0; pass < 4 && !found && lo != hi; ++pass) {
    const uint32_t range = hi - lo;
    const int bits = 32 - __clz(range);
    const int shift = bits > 12 ? bits - 12 : 0;   // (key - lo) >> shift < 4096
    if (pass > 0) {
      __syncthreads();   // every thread is done with the previous pass's histogram
#pragma unroll
      for (int i = tid; i < LIN_BINS; i += NT) sh.hist[i] = 0;
      __syncthreads();
    }
#pragma unroll
    for (int e = 0; e < PER; ++e)
      if (e < nv && key[e] >= lo && key[e] <= hi) atomicAdd(&sh.hist[(key[e] - lo) >> shift], 1u);
    __syncthreads();
    // boundary bin: thread t owns the BPT bins below LIN_BINS - BPT t (highest first)
    constexpr int BPT = LIN_BINS / NT;
    uint32_t c[BPT], tot = 0;
#pragma unroll
    for (int q4 = 0; q4 < BPT / 4; ++q4) {
      const uint4 h4 = *reinterpret_cast<const uint4*>(&sh.hist[LIN_BINS - BPT * (tid + 1) + 4 * (BPT / 4 - 1 - q4)]);
      c[4 * q4] = h4.w;
      c[4 * q4 + 1] = h4.z;
      c[4 * q4 + 2] = h4.y;
      c[4 * q4 + 3] = h4.x;
    }
#pragma unroll
    for (int e = 0; e < BPT; ++e) tot += c[e];
    const uint32_t before = lin_scan<NT>(tot, sh);
    if (before < kleft && kleft <= before + tot) {
      uint32_t run = before;
#pragma unroll
      for (int e = 0; e < BPT; ++e) {
        if (run + c[e] >= kleft) {
          sh.bin = LIN_BINS - 1 - (BPT * tid + e);
          sh.kleft = kleft - run;
          sh.count = c[e];
          break;
        }
        run += c[e];
      }
    }
    if (tid == 0) sh.ncand = 0;
    __syncthreads();
    const uint32_t bin = sh.bin, cnt = sh.count;
    kleft = sh.kleft;
    const uint32_t blo = lo + (bin << shift);
    const uint32_t bhi = static_cast<uint32_t>(
        min(static_cast<unsigned long long>(hi), static_cast<unsigned long long>(blo) + ((1ull << shift) - 1ull)));
    if (cnt <= LIN_CAND) {
#pragma unroll
      for (int e = 0; e < PER; ++e)
        if (e < nv && key[e] >= blo && key[e] <= bhi) {
          const uint32_t slot = atomicAdd(&sh.ncand, 1u);
          sh.cand[slot] = (static_cast<unsigned long long>(key[e]) << 32) |
                          static_cast<uint32_t>(~static_cast<uint32_t>(j0 + e));
        }
      __syncthreads();
      for (int i = tid; i < static_cast<int>(cnt); i += NT) {
        const unsigned long long v = sh.cand[i];
        uint32_t rank = 0;
        for (uint32_t m = 0; m < cnt; ++m) rank += sh.cand[m] > v;
        if (rank == kleft - 1) sh.thr = v;
      }
      __syncthreads();
      thr = sh.thr;
      found = true;
    } else {
      lo = blo;
      hi = bhi;
    }
  }
  if (!found) {
    // [lo, hi] is one value: every key above it is taken and the kleft lowest indices equal to it
    uint32_t ne = 0;
#pragma unroll
    for (int e = 0; e < PER; ++e) ne += (e < nv && key[e] == lo);
    __syncthreads();
    const uint32_t before = lin_scan<NT>(ne, sh);
    if (before < kleft && kleft <= before + ne) {
      uint32_t seen = before;
#pragma unroll
      for (int e = 0; e < PER; ++e)
        if (e < nv && key[e] == lo && ++seen == kleft) sh.tau_idx = j0 + e;
    }
    __syncthreads();
    thr = (static_cast<unsigned long long>(lo) << 32) | static_cast<uint32_t>(~static_cast<uint32_t>(sh.tau_idx));
  }
  uint32_t take = 0;
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    const unsigned long long v =
        (static_cast<unsigned long long>(key[e]) << 32) | static_cast<uint32_t>(~static_cast<uint32_t>(j0 + e));
    take |= static_cast<uint32_t>(e < nv && v >= thr) << e;
  }
  __syncthreads();   // the scan scratch is free
  uint32_t pos = lin_scan<NT>(static_cast<uint32_t>(__popc(take)), sh);
  while (take) {  // the taken keys in ascending order
    const int e = __ffs(take) - 1;
    take &= take - 1;
    out[pos++] = km.map(P, b, j0 + e);
  }
}

template <int PER>
__global__ void __launch_bounds__(LIN_THREADS) select_lin_kernel(SelectParams P) {
  __shared__ LinShared sh;
  pdl_trigger();
  pdl_wait();
  select_lin_row<PER, LIN_THREADS>(P, blockIdx.x, sh);
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

// the query-tiled kernel when a batch row holds many queries (prefill), else one CTA per query
inline cudaError_t launch_scores(const ScoreParams& S, cudaStream_t st) {
  if (S.s >= TQ) {
    static PerDeviceOnce attr;
    const cudaError_t e = set_smem_once(attr, score_tiled_kernel, static_cast<int>(sizeof(TiledSmem)));
    if (e != cudaSuccess) return e;
    const dim3 g((S.n_keys + TK - 1) / TK, (S.s + TQ - 1) / TQ, S.batch);
    return launch_pdl(score_tiled_kernel, g, dim3(THREADS), sizeof(TiledSmem), st, S);
  }
  static PerDeviceOnce attr1;
  const cudaError_t e = set_smem_once(attr1, score_kernel, static_cast<int>(sizeof(ScoreSmem)));
  if (e != cudaSuccess) return e;
  const dim3 g(static_cast<unsigned>(static_cast<int64_t>(S.batch) * S.s), (S.n_keys + KT - 1) / KT);
  return launch_pdl(score_kernel, g, dim3(THREADS), sizeof(ScoreSmem), st, S);
}

// the register-resident kernel up to 16384 visible keys, the shared-memory one above
inline cudaError_t launch_select(const SelectParams& L, unsigned rows, cudaStream_t st) {
  const dim3 g(rows), blk(SEL_THREADS);
  if (!L.refine && rows <= static_cast<unsigned>(LIN_MAX_ROWS) && L.n_keys <= LIN_THREADS * 32) {
    const dim3 lb(LIN_THREADS);
    if (L.n_keys <= LIN_THREADS * 4) return launch_pdl(select_lin_kernel<4>, g, lb, 0, st, L);
    if (L.n_keys <= LIN_THREADS * 8) return launch_pdl(select_lin_kernel<8>, g, lb, 0, st, L);
    if (L.n_keys <= LIN_THREADS * 16) return launch_pdl(select_lin_kernel<16>, g, lb, 0, st, L);
    return launch_pdl(select_lin_kernel<32>, g, lb, 0, st, L);
  }
  if (L.refine) {
    constexpr size_t rsm = sizeof(RefineSmem);
    static PerDeviceOnce rattr;
    const cudaError_t e = rattr([&] {
      for (auto fn : {select_reg_kernel<4, true>, select_reg_kernel<8, true>, select_reg_kernel<16, true>,
                      select_reg_kernel<32, true>}) {
        const cudaError_t r = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(rsm));
        if (r != cudaSuccess) return r;
      }
      return cudaSuccess;
    });
    if (e != cudaSuccess) return e;
    if (L.n_keys <= SEL_THREADS * 4) return launch_pdl(select_reg_kernel<4, true>, g, blk, rsm, st, L);
    if (L.n_keys <= SEL_THREADS * 8) return launch_pdl(select_reg_kernel<8, true>, g, blk, rsm, st, L);
    if (L.n_keys <= SEL_THREADS * 16) return launch_pdl(select_reg_kernel<16, true>, g, blk, rsm, st, L);
    return launch_pdl(select_reg_kernel<32, true>, g, blk, rsm, st, L);
  }
  if (L.n_keys <= SEL_THREADS * 4) return launch_pdl(select_reg_kernel<4, false>, g, blk, 0, st, L);
  if (L.n_keys <= SEL_THREADS * 8) return launch_pdl(select_reg_kernel<8, false>, g, blk, 0, st, L);
  if (L.n_keys <= SEL_THREADS * 16) return launch_pdl(select_reg_kernel<16, false>, g, blk, 0, st, L);
  if (L.n_keys <= SEL_THREADS * 32) return launch_pdl(select_reg_kernel<32, false>, g, blk, 0, st, L);
  static PerDeviceOnce attr;
  const cudaError_t e = set_smem_once(attr, select_kernel, SEL_MAX_KEYS * 4);
  if (e != cudaSuccess) return e;
  return launch_pdl(select_kernel, g, blk, static_cast<size_t>(L.n_keys) * 4, st, L);
}

}  // namespace idx

DSV4_ERROR_READER(indexer)

}  // namespace dsv4

using namespace dsv4;

namespace {
// scoring method for a call: 1 exact FMA scores, 2 tensor-core filter + exact band; -1 unavailable
int resolve_mode(const dsv4_indexer_params* p) {
  if (p->mode == 1) return 1;
  const bool tc_ok = p->heads == idx::HI && p->n_keys <= idx::SEL_THREADS * 32;
  if (p->mode == 2) return tc_ok ? 2 : -1;
  if (p->mode != 0) return -1;
  // prefill-shaped calls, and decode batches large enough that the exact selection's latency per
  // query is hidden behind the others
  const bool many = itc::row_kernel(p->s) ? p->batch >= 16 : static_cast<int64_t>(p->batch) * p->s >= 256;
  return (tc_ok && many && p->n_keys > p->top_k) ? 2 : 1;
}
size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
// workspace: [scores rows x n_pad fp32] then, for mode 2, [key tile images] [key scales]
// [max key norm per batch]
size_t workspace_layout(const dsv4_indexer_params* p, int mode, size_t* off_kimg, size_t* off_kmax) {
  const int64_t n_pad = (p->n_keys + 3) / 4 * 4;
  const size_t sc = static_cast<size_t>(static_cast<int64_t>(p->batch) * p->s * n_pad * sizeof(float));
  if (mode != 2 || p->key_image != nullptr) {  // a cache-kept image brings its own scales and norms
    *off_kimg = *off_kmax = sc;
    return sc;
  }
  *off_kimg = round_up(sc, 1024);
  *off_kmax = *off_kimg;
  if (!itc::row_kernel(p->s)) *off_kmax += itc::kimg_bytes(p->batch, p->n_keys) + itc::kinv_bytes(p->batch, p->n_keys);
  return *off_kmax + round_up(sizeof(float) * p->batch, 256);
}
}  // namespace

extern "C" size_t dsv4_indexer_topk_workspace_size(const dsv4_indexer_params* p) {
  if (!p || p->batch <= 0 || p->s <= 0 || p->n_keys <= 0) return 0;
  size_t a = 0, b = 0;
  const int mode = resolve_mode(p);
  return workspace_layout(p, mode < 0 ? 1 : mode, &a, &b);
}

extern "C" int dsv4_indexer_topk(const dsv4_indexer_params* p, void* stream) {
  DSV4_CHECK_ARG(p != nullptr, "dsv4_indexer_topk: params is NULL");
  DSV4_CHECK_ARG(p->q && p->w && p->k && p->out, "dsv4_indexer_topk: NULL tensor");
  DSV4_CHECK_ARG(p->heads == idx::HI, "dsv4_indexer_topk: %d heads unsupported (64 only)", p->heads);
  DSV4_CHECK_ARG((reinterpret_cast<uintptr_t>(p->q) | reinterpret_cast<uintptr_t>(p->w) |
                  reinterpret_cast<uintptr_t>(p->k)) % 16 == 0,
                 "dsv4_indexer_topk: q, w and k must be 16-byte aligned");
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
  DSV4_CHECK_ARG(p->win_base == nullptr || (p->positions != nullptr && p->window > 0 &&
                                            p->out_col >= p->window),
                 "dsv4_indexer_topk: window columns need positions and out_col >= window");
  const int64_t rows = static_cast<int64_t>(p->batch) * p->s;
  DSV4_CHECK_ARG(rows <= 2147483647LL, "dsv4_indexer_topk: too many queries");
  DSV4_CHECK_ARG((p->key_image == nullptr) == (p->key_inv == nullptr) &&
                     (p->key_image == nullptr) == (p->key_norm_max == nullptr),
                 "dsv4_indexer_topk: key_image, key_inv and key_norm_max go together");
  DSV4_CHECK_ARG(p->key_image == nullptr || p->k_batch_stride >= p->n_keys,
                 "dsv4_indexer_topk: a key image needs k_batch_stride >= n_keys");
  DSV4_CHECK_ARG(p->key_image == nullptr || reinterpret_cast<uintptr_t>(p->key_image) % 16 == 0,
                 "dsv4_indexer_topk: key image must be 16-byte aligned");
  const int mode = resolve_mode(p);
  DSV4_CHECK_ARG(mode > 0, "dsv4_indexer_topk: mode %d unavailable (mode 2 needs n_keys <= %d)", p->mode,
                 idx::SEL_THREADS * 32);
  size_t off_kimg = 0, off_kmax = 0;
  const size_t need = workspace_layout(p, mode, &off_kimg, &off_kmax);
  if (p->workspace == nullptr || p->workspace_bytes < need) {
    set_error("dsv4_indexer_topk: workspace of %zu bytes needed, %zu given", need, p->workspace_bytes);
    return DSV4_ERR_WORKSPACE;
  }
  float* scores = p->scores_out ? p->scores_out : reinterpret_cast<float*>(p->workspace);
  const int n_pad = p->scores_out ? p->n_keys : (p->n_keys + 3) / 4 * 4;
  float* kmax = nullptr;
  if (mode == 2) {
    itc::ApproxArgs A = {};
    A.q = p->q;
    A.w = p->w;
    A.k = p->k;
    A.scores = scores;
    A.batch = p->batch;
    A.s = p->s;
    A.n_keys = p->n_keys;
    A.n_pad = n_pad;
    A.k_batch_stride = p->k_batch_stride;
    A.positions = p->positions;
    A.ratio = p->ratio;
    if (p->key_image) {
      A.kimg = const_cast<uint8_t*>(p->key_image);
      A.kinv = const_cast<float*>(p->key_inv);
      A.kmax = kmax = const_cast<float*>(p->key_norm_max);
      A.img_tiles = itc::key_tiles(static_cast<int>(std::min<int64_t>(p->k_batch_stride, 1 << 30)));
      A.img_ready = 1;
    } else {
      if (!itc::row_kernel(p->s)) {
        A.kimg = static_cast<uint8_t*>(p->workspace) + off_kimg;
        A.kinv = reinterpret_cast<float*>(A.kimg + itc::kimg_bytes(p->batch, p->n_keys));
      }
      A.kmax = kmax = reinterpret_cast<float*>(static_cast<uint8_t*>(p->workspace) + off_kmax);
      A.img_tiles = itc::key_tiles(p->n_keys);
    }
    DSV4_CUDA_CHECK(itc::launch_approx_scores(A, as_stream(stream)));
  }

  idx::ScoreParams S = {};
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
  idx::SelectParams L = {};
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
  L.win_base = p->win_base;
  L.window = p->window;
  L.window_linear = p->window_linear;
  if (mode == 2) {
    L.refine = 1;
    L.q = p->q;
    L.w = p->w;
    L.k = p->k;
    L.k_batch_stride = p->k_batch_stride;
    L.kmax = kmax;
    L.eps_c = idx::EPS_C;
  }
  if (mode == 1) DSV4_CUDA_CHECK(idx::launch_scores(S, as_stream(stream)));
  DSV4_CUDA_CHECK(idx::launch_select(L, static_cast<unsigned>(rows), as_stream(stream)));
  return DSV4_OK;
}

extern "C" int dsv4_indexer_key_image(const dsv4_key_image_params* p, void* stream) {
  DSV4_CHECK_ARG(p && p->k && p->image && p->inv && p->norm_max, "dsv4_indexer_key_image: NULL tensor");
  DSV4_CHECK_ARG(p->batch > 0 && p->n_keys >= 0 && p->k_batch_stride >= p->n_keys && p->k_batch_stride < (1 << 30),
                 "dsv4_indexer_key_image: bad sizes");
  DSV4_CHECK_ARG(reinterpret_cast<uintptr_t>(p->image) % 16 == 0, "dsv4_indexer_key_image: image not 16-byte aligned");
  itc::ApproxArgs A = {};
  A.k = p->k;
  A.batch = p->batch;
  A.n_keys = p->n_keys;
  A.k_batch_stride = p->k_batch_stride;
  A.kimg = p->image;
  A.kinv = p->inv;
  A.kmax = p->norm_max;
  A.img_tiles = itc::key_tiles(static_cast<int>(p->k_batch_stride));
  if (p->n_keys == 0) {
    DSV4_CUDA_CHECK(cudaMemsetAsync(p->norm_max, 0, sizeof(float) * p->batch, as_stream(stream)));
    return DSV4_OK;
  }
  DSV4_CUDA_CHECK(itc::launch_key_image(A, as_stream(stream)));
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

// ---- allocation-free entry point -------------------------------------------------------------
// Score scratch of dsv4_indexer_topk_noalloc: a fixed array in the library's device image, so that
// a caller that cannot allocate device memory can still run the indexer. Every GPU that loads the
// library holds these 4 MiB until the process exits. Host code must not use `g_noalloc_scores`
// as a pointer (on the host it names a stand-in, not the device array); it passes the address that
// cudaGetSymbolAddress returns for the current device.
static __device__ __align__(256) float g_noalloc_scores[DSV4_INDEXER_NOALLOC_MAX_SCORES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kMaxDevices] = {};
unsigned long long g_noalloc_ctx[kMaxDevices] = {};

// Unique id of the current CUDA context (cuCtxGetCurrent + cuCtxGetId, reached through the
// runtime's driver entry points so that the library needs no link to libcuda), 0 if unavailable.
// Ids are never reused within a process, so a context recreated after cudaDeviceReset (where the
// library's device image, and with it the scratch array, may load at another address) differs.
unsigned long long current_context_id() {
  using GetCurrent = int (*)(void**);
  using GetId = int (*)(void*, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static bool looked_up = false;
  if (!looked_up) {  // called with g_noalloc_mu held
    looked_up = true;
    cudaDriverEntryPointQueryResult q1, q2;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", reinterpret_cast<void**>(&get_current), 12000,
                                         cudaEnableDefault, &q1) != cudaSuccess || q1 != cudaDriverEntryPointSuccess)
      get_current = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", reinterpret_cast<void**>(&get_id), 12000,
                                         cudaEnableDefault, &q2) != cudaSuccess || q2 != cudaDriverEntryPointSuccess)
      get_id = nullptr;
    cudaGetLastError();
  }
  void* ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != 0 || ctx == nullptr || get_id(ctx, &id) != 0) return 0;
  return id;
}

// Device address of the scratch array on the current device: looked up at the first call on each
// device (with that device current), and again only when the device's context has changed.
int noalloc_scratch(float** out) {
  int dev = 0;
  DSV4_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("dsv4_indexer_topk_noalloc: device ordinal %d unsupported", dev);
    return DSV4_ERR_INVALID_ARGUMENT;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  const unsigned long long ctx = current_context_id();
  if (g_noalloc_ptr[dev] == nullptr || ctx != g_noalloc_ctx[dev]) {
    void* ptr = nullptr;
    DSV4_CUDA_CHECK(cudaGetSymbolAddress(&ptr, g_noalloc_scores));
    g_noalloc_ptr[dev] = static_cast<float*>(ptr);
    g_noalloc_ctx[dev] = ctx;
  }
  *out = g_noalloc_ptr[dev];
  return DSV4_OK;
}
}  // namespace

extern "C" int dsv4_indexer_topk_noalloc(const dsv4_indexer_params* p, void* stream) {
  DSV4_CHECK_ARG(p != nullptr, "dsv4_indexer_topk_noalloc: params is NULL");
  DSV4_CHECK_ARG(p->q && p->w && p->k && p->out, "dsv4_indexer_topk_noalloc: NULL tensor");
  DSV4_CHECK_ARG(p->workspace == nullptr && p->scores_out == nullptr,
                 "dsv4_indexer_topk_noalloc: workspace and scores_out must be NULL (the scratch is built in)");
  DSV4_CHECK_ARG(p->mode >= 0 && p->mode <= 2, "dsv4_indexer_topk_noalloc: mode %d unknown (0, 1 or 2)", p->mode);
  DSV4_CHECK_ARG((p->key_image == nullptr) == (p->key_inv == nullptr) &&
                     (p->key_image == nullptr) == (p->key_norm_max == nullptr),
                 "dsv4_indexer_topk_noalloc: key_image, key_inv and key_norm_max go together");
  DSV4_CHECK_ARG(p->heads == idx::HI, "dsv4_indexer_topk_noalloc: %d heads unsupported (64 only)", p->heads);
  DSV4_CHECK_ARG((reinterpret_cast<uintptr_t>(p->q) | reinterpret_cast<uintptr_t>(p->w) |
                  reinterpret_cast<uintptr_t>(p->k)) % 16 == 0,
                 "dsv4_indexer_topk_noalloc: q, w and k must be 16-byte aligned");
  DSV4_CHECK_ARG(p->batch > 0 && p->s > 0 && p->n_keys > 0 && p->top_k > 0,
                 "dsv4_indexer_topk_noalloc: bad sizes");
  DSV4_CHECK_ARG(p->n_keys <= idx::SEL_MAX_KEYS, "dsv4_indexer_topk_noalloc: n_keys %d above %d", p->n_keys,
                 idx::SEL_MAX_KEYS);
  DSV4_CHECK_ARG(p->positions == nullptr || p->ratio > 0, "dsv4_indexer_topk_noalloc: ratio must be > 0");
  DSV4_CHECK_ARG(p->out_col >= 0 && p->out_col + p->top_k <= p->out_stride,
                 "dsv4_indexer_topk_noalloc: out_col + top_k exceeds out_stride");
  DSV4_CHECK_ARG(p->block_table == nullptr || (p->page > 0 && p->table_stride > 0),
                 "dsv4_indexer_topk_noalloc: block table needs page and table_stride");
  DSV4_CHECK_ARG(p->k_batch_stride >= p->n_keys || p->batch == 1,
                 "dsv4_indexer_topk_noalloc: k_batch_stride smaller than n_keys");
  DSV4_CHECK_ARG(p->win_base == nullptr || (p->positions != nullptr && p->window > 0 &&
                                            p->out_col >= p->window),
                 "dsv4_indexer_topk_noalloc: window columns need positions and out_col >= window");
  const int64_t rows = static_cast<int64_t>(p->batch) * p->s;
  const int n_pad = (p->n_keys + 3) / 4 * 4;
  if (rows * n_pad > DSV4_INDEXER_NOALLOC_MAX_SCORES) {
    set_error("dsv4_indexer_topk_noalloc: batch*s*n_keys (padded) = %lld scores exceeds the built-in "
              "scratch of %d; use dsv4_indexer_topk with a caller-provided workspace",
              static_cast<long long>(rows * n_pad), DSV4_INDEXER_NOALLOC_MAX_SCORES);
    return DSV4_ERR_WORKSPACE;
  }
  float* scores = nullptr;
  const int st = noalloc_scratch(&scores);
  if (st != DSV4_OK) return st;

  // The scores are written for every visible key before the selection reads them, and entries past
  // a query's visible range are never read, so nothing in the scratch needs clearing between calls.
  idx::ScoreParams S = {};
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
  static PerDeviceOnce score_attr;
  DSV4_CUDA_CHECK(set_smem_once(score_attr, idx::score_kernel, static_cast<int>(sizeof(idx::ScoreSmem))));
  dim3 g1(static_cast<unsigned>(rows), (p->n_keys + idx::KT - 1) / idx::KT);
  idx::score_kernel<<<g1, idx::THREADS, sizeof(idx::ScoreSmem), as_stream(stream)>>>(S);
  DSV4_LAUNCH_CHECK("indexer score_kernel (noalloc)");

  idx::SelectParams L = {};
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
  L.win_base = p->win_base;
  L.window = p->window;
  L.window_linear = p->window_linear;
  DSV4_CUDA_CHECK(idx::launch_select(L, static_cast<unsigned>(rows), as_stream(stream)));
  return DSV4_OK;
}
