// Approximate lightning-indexer scores on the 5th-generation tensor cores (the filter stage of the
// bit-exact top-k; the error bound and the exact rescoring live with the selection in indexer.cu).
//
// Operands are split into two fp16 terms after an exact power-of-two scaling of every row (a key,
// or one head of a query) that brings its largest element into [2^14, 2^15):
//   x * 2^s = xh + xl + d,  xh = rn16(x * 2^s),  xl = rn16(x * 2^s - xh),  |d| <= 2^-22 |x * 2^s|
// and q.k is taken as (qh.kh + qh.kl + ql.kh) * 2^-(s_q + s_k), three fp16 MMAs with fp32
// accumulation; the dropped terms are below 3.01 * 2^-22 * sum_i |q_i k_i|.
//
// key_image_kernel: every key row -> its scaled fp16 hi / lo terms written as the shared-memory image
//   of its 128-key tile: two slab groups (dims 0-63, 64-127), each [hi slab 16 KB | lo slab 16 KB]
//   128-byte swizzled, so that one 32 KB bulk copy lands a slab group ready for the MMA; the key's
//   inverse scale 2^-s_k; and the maximum key norm per batch entry (for the error bound).
// approx_score_kernel: one CTA per 4 consecutive queries (N = 4 x 64 heads = 256 columns), looping
//   over the key tiles visible to the last of them. Per tile and slab group g, on M = 128 keys:
//     S^T[key, (q,h)] += kl_g.qh_g + kh_g.qh_g + kh_g.ql_g   (12 MMAs of K = 16)
//   into one of two 256-column TMEM buffers. Warp 4 (one elected lane) issues the bulk copies and the
//   MMAs; slab groups stream through a ring of three 32 KB slots, so every copy has the MMA time of the
//   two groups before it to land. Warps 0-7 (thread = key; warp w reads lane quadrant w % 4 for
//   queries 2 (w / 4) and 2 (w / 4) + 1) read the finished buffer, fold
//   sum_h (w[q,h] 2^-s_qh) relu(s) per query, scale by 2^-s_k and store the scores.
// All waits are bounded (1 s); a timeout raises DSV4_ERR_WAIT_TIMEOUT and the CTA winds down.
#include <cuda_fp16.h>

#include "common.cuh"
#include "indexer_tc.cuh"
#include "key_image.cuh"
#include "tcgen05.cuh"

namespace dsv4 {
namespace itc {

using namespace tc5;

constexpr int DI = 128, HI = 64, QG = 4, NQ = QG * HI;
constexpr int EPI_WARPS = 8;           // two per TMEM lane quadrant, two queries each
constexpr int THREADS = (EPI_WARPS + 1) * 32;  // + the producer warp
constexpr int SLAB_Q = NQ * 128;        // 32 KB: 256 (query, head) rows x 64 fp16 dims
constexpr int SLAB_K = BM * 128;        // 16 KB: 128 keys x 64 fp16 dims
constexpr int GROUP = 2 * SLAB_K;       // 32 KB: hi + lo slab of one dim group of a tile
static_assert(TILE_BYTES == 2 * GROUP && GROUP == IMG_GROUP && SLAB_K == IMG_SLAB_K, "tile image");
constexpr int TMEM_COLS = 512;
constexpr int NSLOT = 3;                // slab-group copies in flight: 3 x 32 KB next to the 128 KB of Q

struct Smem {
  alignas(1024) uint8_t qh[2 * SLAB_Q];
  alignas(1024) uint8_t ql[2 * SLAB_Q];
  alignas(1024) uint8_t kbuf[NSLOT][GROUP];  // ring of slab groups: group n in slot n % NSLOT
  float w[QG][HI];                           // w[q,h] * 2^-s_qh
  uint64_t bar_full[NSLOT], bar_empty[NSLOT];  // slab group landed / its MMAs done
  uint64_t bar_done[2], bar_free[2];     // TMEM buffer written / read by the epilogue
  uint32_t tmem_base;
  int abort;
};

static_assert(sizeof(Smem) + 1024 <= 232448, "shared memory above the 227 KB a CTA may opt into");

// max over the CTA's threads (all of them call it), one atomicMax per CTA into *dst (the values
// are non-negative floats, which order like their bit patterns)
__device__ __forceinline__ void cta_atomic_max(float v, float* dst) {
  __shared__ float wmax[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (lane == 0) wmax[warp] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = 0.f;
    for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) m = fmaxf(m, wmax[i]);
    atomicMax(reinterpret_cast<unsigned int*>(dst), __float_as_uint(m));
  }
}

// grid (tiles, batch), 128 threads: thread = key row of the tile
__global__ void __launch_bounds__(BM) key_image_kernel(ApproxArgs P) {
  const int t = blockIdx.x, b = blockIdx.y, r = threadIdx.x;
  const int j = t * BM + r;
  const int tiles = P.img_tiles;
  uint8_t* img = P.kimg + (static_cast<int64_t>(b) * tiles + t) * TILE_BYTES;
  const float4* kr = reinterpret_cast<const float4*>(P.k + (static_cast<int64_t>(b) * P.k_batch_stride + j) * DI);
  const bool valid = j < P.n_keys;
  float ss = 0.f, mx = 0.f;
  if (valid) {
#pragma unroll 8
    for (int f = 0; f < DI / 4; ++f) {
      const float4 v = __ldg(kr + f);
      ss = fmaf(v.x, v.x, ss);
      ss = fmaf(v.y, v.y, ss);
      ss = fmaf(v.z, v.z, ss);
      ss = fmaf(v.w, v.w, ss);
      mx = fmaxf(mx, amax4(v));
    }
  }
  const int sh = row_shift(mx);
  const float up = pow2(sh);
#pragma unroll 4
  for (int f = 0; f < DI / 4; ++f) {
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (valid) v = scale4(__ldg(kr + f), up);
    uint2 hi, lo;
    split4(v, &hi, &lo);
    const uint32_t off = key_off(r, f);
    *reinterpret_cast<uint2*>(img + off) = hi;
    *reinterpret_cast<uint2*>(img + off + SLAB_K) = lo;
  }
  P.kinv[static_cast<int64_t>(b) * tiles * BM + j] = pow2(-sh);
  cta_atomic_max(valid ? sqrtf(ss) : 0.f, P.kmax + b);
}

__device__ __forceinline__ int visible(const ApproxArgs& P, int64_t row) {
  if (P.positions == nullptr) return P.n_keys;
  const int nv = (P.positions[row] + 1) / P.ratio;
  return nv < 0 ? 0 : (nv < P.n_keys ? nv : P.n_keys);
}

__device__ __forceinline__ void set_abort(Smem& sm) {
  if (!*reinterpret_cast<volatile int*>(&sm.abort)) {
    *reinterpret_cast<volatile int*>(&sm.abort) = 1;
    raise_device_error(DSV4_ERR_WAIT_TIMEOUT);
  }
}

// 12 MMAs of slab group g into TMEM column base d; the first of a tile overwrites
__device__ __forceinline__ void issue_group(uint32_t d, uint32_t kb, uint32_t qh, uint32_t ql, int g, bool first) {
  constexpr uint32_t id = idesc_f16<128, NQ>(false, false);
  const uint32_t qhg = qh + g * SLAB_Q, qlg = ql + g * SLAB_Q;
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
    mma16(d, sdesc(kb + SLAB_K + kk * 32, 16, 1024), sdesc(qhg + kk * 32, 16, 1024), id, (first && kk == 0) ? 0u : 1u);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
    mma16(d, sdesc(kb + kk * 32, 16, 1024), sdesc(qhg + kk * 32, 16, 1024), id, 1u);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
    mma16(d, sdesc(kb + kk * 32, 16, 1024), sdesc(qlg + kk * 32, 16, 1024), id, 1u);
}

__global__ void __launch_bounds__(THREADS, 1) approx_score_kernel(ApproxArgs P) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gpb = (P.s + QG - 1) / QG;
  // late (causally heavier) groups first
  const int64_t gidx = static_cast<int64_t>(gridDim.x) - 1 - blockIdx.x;
  const int b = static_cast<int>(gidx / gpb);
  const int s0 = static_cast<int>(gidx % gpb) * QG;
  const int nq = min(QG, P.s - s0);
  const int64_t row0 = static_cast<int64_t>(b) * P.s + s0;
  int nvis = 0;
  for (int q = 0; q < nq; ++q) nvis = max(nvis, visible(P, row0 + q));
  const int T = (nvis + BM - 1) / BM;
  if (T == 0) return;  // block-uniform

  // stage the scaled, split Q: each warp takes (query, head) rows warp, warp + 9, ..; lane = float4
  // of the row; loads are issued 8 rows ahead of their use
  constexpr int NW = THREADS / 32;
  constexpr int QB = 8;
  for (int r0 = warp; r0 < NQ; r0 += NW * QB) {
    float4 qv[QB];
#pragma unroll
    for (int k = 0; k < QB; ++k) {
      const int r = r0 + k * NW;
      qv[k] = (r < NQ && (r >> 6) < nq) ? __ldg(reinterpret_cast<const float4*>(P.q + (row0 * HI + r) * DI) + lane)
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int k = 0; k < QB; ++k) {
    const int r = r0 + k * NW;
    if (r >= NQ) break;
    const int q = r >> 6;
    const float4 v = qv[k];
    float mx = amax4(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const int sh = row_shift(mx);
    uint2 hi, lo;
    split4(scale4(v, pow2(sh)), &hi, &lo);
    const uint32_t off = static_cast<uint32_t>((lane >> 4) * SLAB_Q + r * 128 + ((((lane >> 1) & 7) ^ (r & 7)) << 4) +
                                               (lane & 1) * 8);
    *reinterpret_cast<uint2*>(sm.qh + off) = hi;
    *reinterpret_cast<uint2*>(sm.ql + off) = lo;
    if (lane == 0) sm.w[q][r & 63] = q < nq ? P.w[(row0 + q) * HI + (r & 63)] * pow2(-sh) : 0.f;
    }
  }
  if (warp == 0) tmem_alloc<TMEM_COLS>(&sm.tmem_base);
  if (tid == 0) {
    for (int i = 0; i < NSLOT; ++i) {
      bar_init(&sm.bar_full[i], 1);
      bar_init(&sm.bar_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      bar_init(&sm.bar_done[i], 1);
      bar_init(&sm.bar_free[i], EPI_WARPS);
    }
    sm.abort = 0;
    bar_init_fence();
  }
  fence_async_smem();  // the Q slabs, written by threads, are read by the tensor cores
  before_sync();
  __syncthreads();
  after_sync();
  const uint32_t tmem = sm.tmem_base;
  const volatile int* abort = &sm.abort;
  const int tiles = P.img_tiles;  // image stride per batch entry

  if (warp == EPI_WARPS) {
    if (lane == 0) {
      const uint8_t* img = P.kimg + static_cast<int64_t>(b) * tiles * TILE_BYTES;
      const uint32_t qh = smem_u32(sm.qh), ql = smem_u32(sm.ql);
      bool ok = true;
      const int ngroups = 2 * T;  // group n = slab group (n & 1) of tile n >> 1
      int pending[NSLOT];         // group whose copy into slot k is issued and not yet waited for
      for (int k = 0; k < NSLOT; ++k) pending[k] = -1;
      int committed = -1;         // the last group whose MMAs were committed
      auto load = [&](int n) {
        const int k = n % NSLOT;
        bar_expect_tx(&sm.bar_full[k], GROUP);
        bulk_g2s(sm.kbuf[k], img + static_cast<int64_t>(n >> 1) * TILE_BYTES + (n & 1) * GROUP, GROUP,
                 &sm.bar_full[k]);
        pending[k] = n;
      };
      for (int n = 0; n < NSLOT && n < ngroups; ++n) load(n);
      for (int n = 0; n < ngroups; ++n) {
        const int i = n >> 1, g = n & 1, k = n % NSLOT;
        // the first group of tile i overwrites TMEM buffer i & 1, last read by the epilogue for tile i-2
        if (g == 0 && i >= 2 && !(ok = bar_wait_or_abort(&sm.bar_free[i & 1], ((i - 2) >> 1) & 1, abort))) break;
        if (!(ok = bar_wait_or_abort(&sm.bar_full[k], (n / NSLOT) & 1, abort))) break;
        pending[k] = -1;
        after_sync();
        issue_group(tmem + (i & 1) * 256, smem_u32(sm.kbuf[k]), qh, ql, g, g == 0);
        mma_commit(&sm.bar_empty[k]);
        if (g == 1) mma_commit(&sm.bar_done[i & 1]);
        committed = n;
        // refill the slot of group n-1 (done before group n runs) with group n-1+NSLOT
        const int m = n - 1 + NSLOT;
        if (n >= 1 && m < ngroups) {
          if (!(ok = bar_wait_or_abort(&sm.bar_empty[(n - 1) % NSLOT], ((n - 1) / NSLOT) & 1, abort))) break;
          load(m);
        }
      }
      if (!ok) {
        set_abort(sm);
        // let what was issued finish before the CTA's shared and tensor memory go away
        for (int k = 0; k < NSLOT; ++k)
          if (pending[k] >= 0) bar_wait(&sm.bar_full[k], (pending[k] / NSLOT) & 1);
        if (committed >= 0) bar_wait(&sm.bar_empty[committed % NSLOT], (committed / NSLOT) & 1);
      }
    }
    __syncwarp();
  } else {
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int qb = (warp >> 2) * 2;  // this warp's two queries
    const float* kinv = P.kinv + static_cast<int64_t>(b) * tiles * BM;
    for (int i = 0; i < T; ++i) {
      const int buf = i & 1;
      const bool ok = bar_wait_or_abort(&sm.bar_done[buf], (i >> 1) & 1, abort);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) set_abort(sm);
        break;
      }
      after_sync();
      float v[2][HI];
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int c = 0; c < HI; c += 16) tmem_ld16(tmem + lane_base + buf * 256 + (qb + u) * HI + c, v[u] + c);
      tmem_wait_ld();
      before_sync();
      __syncwarp();
      if (lane == 0) bar_arrive(&sm.bar_free[buf]);
      float acc[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
        for (int h = 0; h < HI; h += 4) {
          const float4 wv = *reinterpret_cast<const float4*>(&sm.w[qb + u][h]);
          a0 = fmaf(wv.x, fmaxf(v[u][h], 0.f), a0);
          a1 = fmaf(wv.y, fmaxf(v[u][h + 1], 0.f), a1);
          a2 = fmaf(wv.z, fmaxf(v[u][h + 2], 0.f), a2);
          a3 = fmaf(wv.w, fmaxf(v[u][h + 3], 0.f), a3);
        }
        acc[u] = (a0 + a1) + (a2 + a3);
      }
      const int key = i * BM + (warp & 3) * 32 + lane;
      if (key < P.n_keys) {
        const float ks = kinv[key];
#pragma unroll
        for (int u = 0; u < 2; ++u)
          if (qb + u < nq) P.scores[(row0 + qb + u) * P.n_pad + key] = acc[u] * ks;
      }
    }
  }
  before_sync();
  __syncthreads();
  after_sync();
  if (warp == 0) tmem_dealloc<TMEM_COLS>(tmem);
}

// ---- one query per CTA (decode batches): grid (key tiles, queries), no key image ----------------
// The CTA scales and splits its query (64 heads x 128) and its 128-key tile (fp32 rows read once)
// into fp16 hi / lo slabs itself, runs the 24 MMAs (M = 128 keys, N = 64 heads) into 64 TMEM
// columns, and folds the scores; the maximum key norm of the batch entry is accumulated as in
// key_image_kernel. About 97 KB of shared memory: two CTAs per SM.
constexpr int RT_THREADS = 128;
constexpr int RSLAB_Q = HI * 128;   // 8 KB
constexpr int RSLAB_K = BM * 128;   // 16 KB

struct RowSmem {
  alignas(1024) uint8_t qh[2 * RSLAB_Q];
  alignas(1024) uint8_t ql[2 * RSLAB_Q];
  alignas(1024) uint8_t kh[2 * RSLAB_K];
  alignas(1024) uint8_t kl[2 * RSLAB_K];
  float w[HI];                      // w[h] * 2^-s_qh
  uint64_t bar;
  uint32_t tmem_base;
};

__global__ void __launch_bounds__(RT_THREADS) approx_score_row_kernel(ApproxArgs P) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  RowSmem& sm = *reinterpret_cast<RowSmem*>(smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t = blockIdx.x;
  const int64_t row = blockIdx.y;
  const int b = static_cast<int>(row / P.s);
  const int nvis = visible(P, row);
  if (t * BM >= nvis) return;  // block-uniform

  // issue every global load first (the key row of this thread, then the query rows of this warp),
  // so that the two round trips overlap
  const int j = t * BM + tid;
  const bool valid = j < P.n_keys;
  float4 v[DI / 4];
  {
    const float4* kr = reinterpret_cast<const float4*>(P.k + (static_cast<int64_t>(b) * P.k_batch_stride + j) * DI);
#pragma unroll
    for (int f = 0; f < DI / 4; ++f) v[f] = valid ? __ldg(kr + f) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  // the query: warp w scales and splits heads w, w+4, ..; lane = float4 of the head's 128 dims
  constexpr int QH = HI / (RT_THREADS / 32);
  float4 qv[QH];
#pragma unroll
  for (int k = 0; k < QH; ++k)
    qv[k] = __ldg(reinterpret_cast<const float4*>(P.q + (row * HI + warp + k * (RT_THREADS / 32)) * DI) + lane);
#pragma unroll
  for (int k = 0; k < QH; ++k) {
    const int h = warp + k * (RT_THREADS / 32);
    float mx = amax4(qv[k]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const int sh = row_shift(mx);
    uint2 hi, lo;
    split4(scale4(qv[k], pow2(sh)), &hi, &lo);
    const uint32_t off = static_cast<uint32_t>((lane >> 4) * RSLAB_Q + h * 128 + ((((lane >> 1) & 7) ^ (h & 7)) << 4) +
                                               (lane & 1) * 8);
    *reinterpret_cast<uint2*>(sm.qh + off) = hi;
    *reinterpret_cast<uint2*>(sm.ql + off) = lo;
    if (lane == 0) sm.w[h] = P.w[row * HI + h] * pow2(-sh);
  }
  // the key tile: thread = key
  float kinv = 1.f;
  {
    float ss = 0.f, mx = 0.f;
#pragma unroll
    for (int f = 0; f < DI / 4; ++f) {
      ss = fmaf(v[f].x, v[f].x, ss);
      ss = fmaf(v[f].y, v[f].y, ss);
      ss = fmaf(v[f].z, v[f].z, ss);
      ss = fmaf(v[f].w, v[f].w, ss);
      mx = fmaxf(mx, amax4(v[f]));
    }
    const int sh = row_shift(mx);
    const float up = pow2(sh);
    kinv = pow2(-sh);
#pragma unroll
    for (int f = 0; f < DI / 4; ++f) {
      uint2 hi, lo;
      split4(scale4(v[f], up), &hi, &lo);
      const uint32_t off = static_cast<uint32_t>((f >> 4) * RSLAB_K + tid * 128 + ((((f >> 1) & 7) ^ (tid & 7)) << 4) +
                                                 (f & 1) * 8);
      *reinterpret_cast<uint2*>(sm.kh + off) = hi;
      *reinterpret_cast<uint2*>(sm.kl + off) = lo;
    }
    cta_atomic_max(valid ? sqrtf(ss) : 0.f, P.kmax + b);
  }
  if (warp == 0) tmem_alloc<64>(&sm.tmem_base);
  if (tid == 0) {
    bar_init(&sm.bar, 1);
    bar_init_fence();
  }
  fence_async_smem();
  before_sync();
  __syncthreads();
  after_sync();
  const uint32_t tmem = sm.tmem_base;
  if (tid == 0) {
    constexpr uint32_t id = idesc_f16<128, HI>(false, false);
    const uint32_t qh = smem_u32(sm.qh), ql = smem_u32(sm.ql), kh = smem_u32(sm.kh), kl = smem_u32(sm.kl);
#pragma unroll
    for (int g = 0; g < 2; ++g) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma16(tmem, sdesc(kl + g * RSLAB_K + kk * 32, 16, 1024), sdesc(qh + g * RSLAB_Q + kk * 32, 16, 1024), id,
              (g | kk) ? 1u : 0u);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma16(tmem, sdesc(kh + g * RSLAB_K + kk * 32, 16, 1024), sdesc(qh + g * RSLAB_Q + kk * 32, 16, 1024), id, 1u);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma16(tmem, sdesc(kh + g * RSLAB_K + kk * 32, 16, 1024), sdesc(ql + g * RSLAB_Q + kk * 32, 16, 1024), id, 1u);
    }
    mma_commit(&sm.bar);
  }
  const bool ok = __syncthreads_and(bar_wait(&sm.bar, 0));
  if (ok) {
    after_sync();
    float v[HI];
    const uint32_t lq = static_cast<uint32_t>(warp * 32) << 16;
#pragma unroll
    for (int c = 0; c < HI; c += 16) tmem_ld16(tmem + lq + c, v + c);
    tmem_wait_ld();
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
    for (int h = 0; h < HI; h += 4) {
      const float4 wv = *reinterpret_cast<const float4*>(&sm.w[h]);
      a0 = fmaf(wv.x, fmaxf(v[h], 0.f), a0);
      a1 = fmaf(wv.y, fmaxf(v[h + 1], 0.f), a1);
      a2 = fmaf(wv.z, fmaxf(v[h + 2], 0.f), a2);
      a3 = fmaf(wv.w, fmaxf(v[h + 3], 0.f), a3);
    }
    if (valid) P.scores[row * P.n_pad + j] = ((a0 + a1) + (a2 + a3)) * kinv;
  } else if (tid == 0) {
    raise_device_error(DSV4_ERR_WAIT_TIMEOUT);
  }
  before_sync();
  __syncthreads();
  after_sync();
  if (warp == 0) tmem_dealloc<64>(tmem);
}

// ---- decode batches, pipelined: a persistent CTA per SM walks a contiguous run of (query, key
// tile) items. The query (64 heads x 128) is scaled and split once per query it meets; each 128-key
// tile arrives as one 64 KB bulk copy of the stored fp32 rows (two tiles in flight) and is scaled
// and split by four threads per key (a quarter of its dims each; the 16-byte chunks are visited in
// an order rotated by key and quarter so that the eight threads of a shared-memory phase hit
// distinct banks), then 24 MMAs (M = 128 keys, N = 64 heads) and the fold as in
// approx_score_row_kernel, by warps 0-3 (one TMEM lane quadrant each) while the other warps
// already split the next tile. About 226 KB of shared memory: one CTA per SM.
constexpr int SQ_THREADS = 512;
constexpr int RAW_TILE = BM * DI * 4;  // 64 KB

struct SeqSmem {  // dynamic shared memory (1024-byte aligned slabs)
  alignas(1024) uint8_t raw[2][RAW_TILE];
  alignas(1024) uint8_t kh[2 * RSLAB_K];
  alignas(1024) uint8_t kl[2 * RSLAB_K];
  alignas(1024) uint8_t qh[2 * RSLAB_Q];
  alignas(1024) uint8_t ql[2 * RSLAB_Q];
};
struct SeqSmall {  // static shared memory
  float w[HI];
  float kinv[2][BM];
  uint64_t full[2], mma;
  uint32_t tmem_base;
};
static_assert(sizeof(SeqSmem) + 1024 + sizeof(SeqSmall) + 256 <= 232448,
              "shared memory above the 227 KB a CTA may opt into");

// scale and split query `row` into the Q slabs (warp w: heads w, w + NW, ..; lane = float4 of a head)
template <int NT>
__device__ __forceinline__ void split_query(const ApproxArgs& P, int64_t row, uint8_t* qh, uint8_t* ql, float* w) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int NW = NT / 32, QH = HI / NW;
  static_assert(QH <= 32, "one head weight per lane");
  float4 qv[QH];
#pragma unroll
  for (int k = 0; k < QH; ++k)
    qv[k] = __ldg(reinterpret_cast<const float4*>(P.q + (row * HI + warp + k * NW) * DI) + lane);
  // the warp's head weights with the rows (lane k: head warp + k NW), not one dependent load per head
  const float wl = lane < QH ? __ldg(P.w + row * HI + warp + lane * NW) : 0.f;
#pragma unroll
  for (int k = 0; k < QH; ++k) {
    const int h = warp + k * NW;
    float mx = amax4(qv[k]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const int sh = row_shift(mx);
    uint2 hi, lo;
    split4(scale4(qv[k], pow2(sh)), &hi, &lo);
    const uint32_t off = static_cast<uint32_t>((lane >> 4) * RSLAB_Q + h * 128 + ((((lane >> 1) & 7) ^ (h & 7)) << 4) +
                                               (lane & 1) * 8);
    *reinterpret_cast<uint2*>(qh + off) = hi;
    *reinterpret_cast<uint2*>(ql + off) = lo;
    const float wk = __shfl_sync(0xffffffffu, wl, k);
    if (lane == 0) w[h] = wk * pow2(-sh);
  }
}

struct SeqWalk {  // the CTA's items [begin, end): item = query row * tiles + key tile
  int64_t end;
  int tiles;
  int64_t vrow = -1;  // the last query row whose visible count was read (one global load per row)
  int vis = 0;
  __device__ __forceinline__ int64_t next_valid(const ApproxArgs& P, int64_t i) {
    for (; i < end; ++i) {
      const int64_t row = i / tiles;
      const int t = static_cast<int>(i % tiles);
      if (row != vrow) {
        vrow = row;
        vis = visible(P, row);
      }
      if (t * BM < vis) return i;
      i = (row + 1) * tiles - 1;  // the rest of this row's tiles are not visible either
    }
    return end;
  }
};

__device__ __forceinline__ void seq_issue(const ApproxArgs& P, SeqSmem& sm, SeqSmall& ss, int slot, int64_t item,
                                          int tiles) {
  const int64_t row = item / tiles;
  const int t = static_cast<int>(item % tiles);
  const int b = static_cast<int>(row / P.s);
  const int rows = min(BM, P.n_keys - t * BM);
  const uint32_t bytes = static_cast<uint32_t>(rows) * DI * 4;
  bar_expect_tx(&ss.full[slot], bytes);
  bulk_g2s(sm.raw[slot], P.k + (static_cast<int64_t>(b) * P.k_batch_stride + static_cast<int64_t>(t) * BM) * DI, bytes,
           &ss.full[slot]);
}

__global__ void __launch_bounds__(SQ_THREADS) approx_score_seq_kernel(ApproxArgs P, int64_t per) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  SeqSmem& sm = *reinterpret_cast<SeqSmem*>(smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023));
  __shared__ SeqSmall sx;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tiles = key_tiles(P.n_keys);
  const int64_t items = static_cast<int64_t>(P.batch) * P.s * tiles;
  const int64_t begin = static_cast<int64_t>(blockIdx.x) * per;
  SeqWalk walk{begin + per < items ? begin + per : items, tiles};
  SeqWalk pwalk = walk;  // the producer's own cursor state
  if (warp == 0) tmem_alloc<64>(&sx.tmem_base);
  if (tid == 0) {
    bar_init(&sx.full[0], 1);
    bar_init(&sx.full[1], 1);
    bar_init(&sx.mma, 1);
    bar_init_fence();
  }
  before_sync();
  __syncthreads();
  after_sync();
  const uint32_t tmem = sx.tmem_base;
  // producer cursor (thread 0): the next valid item to copy; copies issued
  int64_t pnext = 0;
  int issued = 0;
  if (tid == 0) {
    pnext = pwalk.next_valid(P, begin);
    for (int k = 0; k < 2 && pnext < walk.end; ++k) {
      seq_issue(P, sm, sx, k, pnext, tiles);
      ++issued;
      pnext = pwalk.next_valid(P, pnext + 1);
    }
  }
  const int kr = tid >> 2, part = tid & 3;  // splitting: key row, quarter of its 128 dims
  int64_t cur_row = -1;
  int k = 0;
  bool ok = true, mma_pending = false;
  for (int64_t i = walk.next_valid(P, begin); i < walk.end; ++k) {
    const int64_t row = i / tiles;
    const int t = static_cast<int>(i % tiles);
    const int b = static_cast<int>(row / P.s);
    const int slot = k & 1;
    if (row != cur_row) {
      // every thread is past the previous item's epilogue (it reads sx.w) and its MMAs are done
      __syncthreads();
      split_query<SQ_THREADS>(P, row, sm.qh, sm.ql, sx.w);
      cur_row = row;
    }
    ok = __syncthreads_and(bar_wait(&sx.full[slot], (k >> 1) & 1));
    if (!ok) break;
    // the key tile: this thread's 8 chunks c = 8 part + ((f + 2 part + kr) % 8) of key row kr
    const int j = t * BM + kr;
    const bool valid = j < P.n_keys;
    const uint32_t rowaddr = smem_u32(sm.raw[slot]) + static_cast<uint32_t>(kr) * (DI * 4);
    float4 v[8];
#pragma unroll
    for (int f = 0; f < 8; ++f) {
      const uint32_t c = static_cast<uint32_t>(8 * part + ((f + 2 * part + kr) & 7));
      asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];\n"
                   : "=f"(v[f].x), "=f"(v[f].y), "=f"(v[f].z), "=f"(v[f].w)
                   : "r"(rowaddr + c * 16));
    }
    float ss = 0.f, mx = 0.f;
#pragma unroll
    for (int f = 0; f < 8; ++f) {
      ss = fmaf(v[f].x, v[f].x, ss);
      ss = fmaf(v[f].y, v[f].y, ss);
      ss = fmaf(v[f].z, v[f].z, ss);
      ss = fmaf(v[f].w, v[f].w, ss);
      mx = fmaxf(mx, amax4(v[f]));
    }
    // the four quarters of a key are lanes 4r'..4r'+3 of one warp
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
    const int sh = valid ? row_shift(mx) : 0;
    const float up = pow2(sh);
#pragma unroll
    for (int f = 0; f < 8; ++f) {
      const int c = 8 * part + ((f + 2 * part + kr) & 7);
      uint2 hi, lo;
      split4(scale4(v[f], up), &hi, &lo);
      const uint32_t off = static_cast<uint32_t>((c >> 4) * RSLAB_K + kr * 128 + ((((c >> 1) & 7) ^ (kr & 7)) << 4) +
                                                 (c & 1) * 8);
      *reinterpret_cast<uint2*>(sm.kh + off) = hi;
      *reinterpret_cast<uint2*>(sm.kl + off) = lo;
    }
    if (part == 0) sx.kinv[slot][kr] = pow2(-sh);
    cta_atomic_max((valid && part == 0) ? sqrtf(ss) : 0.f, P.kmax + b);  // its barrier: raw[slot] consumed
    fence_async_smem();
    before_sync();
    __syncthreads();
    after_sync();
    if (tid == 0) {
      if (pnext < walk.end) {  // refill the slot just consumed
        seq_issue(P, sm, sx, slot, pnext, tiles);
        ++issued;
        pnext = pwalk.next_valid(P, pnext + 1);
      }
      constexpr uint32_t id = idesc_f16<128, HI>(false, false);
      const uint32_t qh = smem_u32(sm.qh), ql = smem_u32(sm.ql), kh = smem_u32(sm.kh), kl = smem_u32(sm.kl);
#pragma unroll
      for (int g = 0; g < 2; ++g) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma16(tmem, sdesc(kl + g * RSLAB_K + kk * 32, 16, 1024), sdesc(qh + g * RSLAB_Q + kk * 32, 16, 1024), id,
                (g | kk) ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma16(tmem, sdesc(kh + g * RSLAB_K + kk * 32, 16, 1024), sdesc(qh + g * RSLAB_Q + kk * 32, 16, 1024), id, 1u);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma16(tmem, sdesc(kh + g * RSLAB_K + kk * 32, 16, 1024), sdesc(ql + g * RSLAB_Q + kk * 32, 16, 1024), id, 1u);
      }
      mma_commit(&sx.mma);
    }
    // every thread waits for the MMAs: then the K slabs are free for the next tile's split
    ok = __syncthreads_and(bar_wait(&sx.mma, k & 1));
    if (!ok) {
      mma_pending = true;
      ++k;  // this item's copy has landed
      break;
    }
    after_sync();
    if (warp < 4) {  // the fold: thread = key (TMEM lane)
      const int key = warp * 32 + lane;
      const uint32_t lq = static_cast<uint32_t>(warp * 32) << 16;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
      for (int c = 0; c < HI; c += 16) {
        float sc[16];
        tmem_ld16(tmem + lq + c, sc);
        tmem_wait_ld();
#pragma unroll
        for (int h = 0; h < 16; h += 4) {
          const float4 wv = *reinterpret_cast<const float4*>(&sx.w[c + h]);
          a0 = fmaf(wv.x, fmaxf(sc[h], 0.f), a0);
          a1 = fmaf(wv.y, fmaxf(sc[h + 1], 0.f), a1);
          a2 = fmaf(wv.z, fmaxf(sc[h + 2], 0.f), a2);
          a3 = fmaf(wv.w, fmaxf(sc[h + 3], 0.f), a3);
        }
      }
      const int jj = t * BM + key;
      if (jj < P.n_keys) P.scores[row * P.n_pad + jj] = ((a0 + a1) + (a2 + a3)) * sx.kinv[slot][key];
      before_sync();  // these TMEM reads precede the next item's MMAs (issued after its barrier)
    }
    i = walk.next_valid(P, i + 1);
  }
  if (!ok) {
    if (tid == 0) {
      raise_device_error(DSV4_ERR_WAIT_TIMEOUT);
      // let the copies still in flight land before the CTA's shared memory goes away (bounded)
      for (int kk = k; kk < issued; ++kk) bar_wait(&sx.full[kk & 1], (kk >> 1) & 1);
      if (mma_pending) bar_wait(&sx.mma, (k - 1) & 1);
    }
  }
  before_sync();
  __syncthreads();
  after_sync();
  if (warp == 0) tmem_dealloc<64>(tmem);
}

// ---- decode batches over a cache-kept key image: a persistent CTA per SM walks a contiguous run of
// (query, key tile) items, warp-specialised. Warp 4 (one lane) streams each visible 128-key tile's
// 64 KB image by one bulk copy into a ring of three slots and issues the item's 24 MMAs (M = 128
// keys, N = 64 heads) into one of two 64-column TMEM accumulators; warps 0-3 (thread = key = TMEM
// lane) fold item k - 1 while the MMAs of item k run, and scale and split every query they meet into
// the Q slabs. The next query's loads are issued one item ahead, and the first query's before the
// first image copies (behind 28 MB of image copies they waited ~5 us). About 225 KB of shared
// memory: one CTA per SM.
constexpr int IM_FOLD = 128;              // fold warps 0-3
constexpr int IM_MMA_WARP = IM_FOLD / 32;  // warp 4: MMAs
constexpr int IM_COPY_WARP = IM_MMA_WARP + 1;  // warp 5: image copies (a copy's issue may wait for the
                                               // bulk-copy unit, which must not hold up the MMAs)
constexpr int IM_THREADS = IM_FOLD + 64;
constexpr int IM_SLOTS = 3;
constexpr int IM_QH = HI / (IM_FOLD / 32);  // heads per fold warp in the query split

struct ImgSmem {  // dynamic shared memory
  alignas(1024) uint8_t img[IM_SLOTS][TILE_BYTES];
  alignas(1024) uint8_t qh[2 * RSLAB_Q];
  alignas(1024) uint8_t ql[2 * RSLAB_Q];
};
struct ImgSmall {  // static shared memory
  float w[HI];
  uint64_t full[IM_SLOTS], slot_free[IM_SLOTS];  // tile landed / its MMAs done
  uint64_t acc_full[2], acc_free[2];            // accumulator written / folded
  uint64_t q_ready, fin;                        // Q slabs of the next query split / every MMA done
  uint32_t tmem_base;
  int abort;
};
static_assert(sizeof(ImgSmem) + 1024 + sizeof(ImgSmall) + 256 <= 232448,
              "shared memory above the 227 KB a CTA may opt into");

__device__ __forceinline__ void img_issue(const ApproxArgs& P, ImgSmem& sm, ImgSmall& sx, int slot, int64_t item,
                                          int tiles) {
  const int64_t row = item / tiles;
  const int t = static_cast<int>(item % tiles);
  const int b = static_cast<int>(row / P.s);
  bar_expect_tx(&sx.full[slot], TILE_BYTES);
  bulk_g2s(sm.img[slot], P.kimg + (static_cast<int64_t>(b) * P.img_tiles + t) * TILE_BYTES, TILE_BYTES, &sx.full[slot]);
}

__device__ __forceinline__ void img_set_abort(ImgSmall& sx) {
  if (!*reinterpret_cast<volatile int*>(&sx.abort)) {
    *reinterpret_cast<volatile int*>(&sx.abort) = 1;
    raise_device_error(DSV4_ERR_WAIT_TIMEOUT);
  }
}

// the fold warps' own barrier; returns true when every fold thread passed true
__device__ __forceinline__ bool fold_bar_and(bool v) {
  uint32_t r;
  asm volatile(
      "{\n.reg .pred p, q;\nsetp.ne.u32 p, %1, 0;\nbar.red.and.pred q, 1, %2, p;\nselp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "n"(IM_FOLD)
      : "memory");
  return r != 0;
}

// query `row` (64 heads x 128 fp32) into registers: fold warp w holds heads w, w + 4, .., and lane k
// the weight of head w + 4 k
__device__ __forceinline__ void img_query_load(const ApproxArgs& P, int64_t row, float4 (&qv)[IM_QH], float& wl) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < IM_QH; ++k)
    qv[k] = __ldg(reinterpret_cast<const float4*>(P.q + (row * HI + warp + k * (IM_FOLD / 32)) * DI) + lane);
  wl = lane < IM_QH ? __ldg(P.w + row * HI + warp + lane * (IM_FOLD / 32)) : 0.f;
}
// scale and split the loaded query into the Q slabs and the scaled head weights (as split_query)
__device__ __forceinline__ void img_query_store(const float4 (&qv)[IM_QH], float wl, uint8_t* qh, uint8_t* ql,
                                                float* w) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < IM_QH; ++k) {
    const int h = warp + k * (IM_FOLD / 32);
    float mx = amax4(qv[k]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const int sh = row_shift(mx);
    uint2 hi, lo;
    split4(scale4(qv[k], pow2(sh)), &hi, &lo);
    const uint32_t off = static_cast<uint32_t>((lane >> 4) * RSLAB_Q + h * 128 + ((((lane >> 1) & 7) ^ (h & 7)) << 4) +
                                               (lane & 1) * 8);
    *reinterpret_cast<uint2*>(qh + off) = hi;
    *reinterpret_cast<uint2*>(ql + off) = lo;
    const float wk = __shfl_sync(0xffffffffu, wl, k);
    if (lane == 0) w[h] = wk * pow2(-sh);
  }
}

__global__ void __launch_bounds__(IM_THREADS, 1) approx_score_img_kernel(ApproxArgs P, int64_t per) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  ImgSmem& sm = *reinterpret_cast<ImgSmem*>(smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023));
  __shared__ ImgSmall sx;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tiles = key_tiles(P.n_keys);
  const int64_t items = static_cast<int64_t>(P.batch) * P.s * tiles;
  const int64_t begin = static_cast<int64_t>(blockIdx.x) * per;
  const int64_t end = begin + per < items ? begin + per : items;
  if (warp == 0) tmem_alloc<128>(&sx.tmem_base);
  if (tid == 0) {
    for (int k = 0; k < IM_SLOTS; ++k) {
      bar_init(&sx.full[k], 1);
      bar_init(&sx.slot_free[k], 1);
    }
    for (int a = 0; a < 2; ++a) {
      bar_init(&sx.acc_full[a], 1);
      bar_init(&sx.acc_free[a], IM_FOLD / 32);
    }
    bar_init(&sx.q_ready, 1);
    bar_init(&sx.fin, 1);
    sx.abort = 0;
    bar_init_fence();
  }
  SeqWalk walk{end, tiles};
  const int64_t i0 = walk.next_valid(P, begin);
  float4 qv[IM_QH];
  float wl = 0.f;
  if (warp < IM_FOLD / 32 && i0 < end) img_query_load(P, i0 / tiles, qv, wl);  // ahead of the image copies
  before_sync();
  __syncthreads();
  after_sync();
  const uint32_t tmem = sx.tmem_base;
  const volatile int* abort = &sx.abort;

  if (warp == IM_COPY_WARP) {
    // ---------------------------------------------------------------- image copies (one lane)
    if (lane == 0) {
      SeqWalk pw{end, tiles};
      int issued = 0;
      bool ok = true;
      for (int64_t p = i0; p < end; p = pw.next_valid(P, p + 1), ++issued) {
        const int slot = issued % IM_SLOTS;
        // the slot's previous tile (item issued - IM_SLOTS) has been read by its MMAs
        if (issued >= IM_SLOTS &&
            !(ok = bar_wait_or_abort(&sx.slot_free[slot], ((issued - IM_SLOTS) / IM_SLOTS) & 1, abort)))
          break;
        img_issue(P, sm, sx, slot, p, tiles);
      }
      if (!ok) img_set_abort(sx);
      // the copies issued land before the CTA's shared memory goes away (bounded; immediate when
      // the MMAs consumed them)
      for (int kk = issued - IM_SLOTS > 0 ? issued - IM_SLOTS : 0; kk < issued; ++kk)
        bar_wait(&sx.full[kk % IM_SLOTS], (kk / IM_SLOTS) & 1);
    }
  } else if (warp == IM_MMA_WARP) {
    // ---------------------------------------------------------------- MMAs (one lane)
    if (lane == 0) {
      int k = 0, rc = 0;
      bool ok = true;
      int64_t prev_row = -1;
      for (int64_t i = i0; i < end; i = walk.next_valid(P, i + 1), ++k) {
        const int64_t row = i / tiles;
        const int slot = k % IM_SLOTS, a = k & 1;
        if (row != prev_row) {  // the fold warps have split this query into the Q slabs
          if (!(ok = bar_wait_or_abort(&sx.q_ready, rc & 1, abort))) break;
          ++rc;
          prev_row = row;
        }
        if (!(ok = bar_wait_or_abort(&sx.acc_free[a], ((k >> 1) & 1) ^ 1, abort))) break;
        if (!(ok = bar_wait_or_abort(&sx.full[slot], (k / IM_SLOTS) & 1, abort))) break;
        after_sync();
        constexpr uint32_t id = idesc_f16<128, HI>(false, false);
        const uint32_t d = tmem + a * HI;
        const uint32_t qh = smem_u32(sm.qh), ql = smem_u32(sm.ql), kb = smem_u32(sm.img[slot]);
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          const uint32_t kh = kb + g * GROUP, kl = kh + SLAB_K;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma16(d, sdesc(kl + kk * 32, 16, 1024), sdesc(qh + g * RSLAB_Q + kk * 32, 16, 1024), id, (g | kk) ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma16(d, sdesc(kh + kk * 32, 16, 1024), sdesc(qh + g * RSLAB_Q + kk * 32, 16, 1024), id, 1u);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma16(d, sdesc(kh + kk * 32, 16, 1024), sdesc(ql + g * RSLAB_Q + kk * 32, 16, 1024), id, 1u);
        }
        mma_commit(&sx.acc_full[a]);
        mma_commit(&sx.slot_free[slot]);
      }
      mma_commit(&sx.fin);  // every MMA issued (also on abort) is done before the CTA winds down
      bar_wait(&sx.fin, 0);
      if (!ok) img_set_abort(sx);
    }
  } else {
    // ---------------------------------------------------------------- fold warps 0-3 (thread = key)
    const uint32_t lq = static_cast<uint32_t>(warp * 32) << 16;
    int64_t prev_row = -1;
    int k = 0;
    for (int64_t i = i0; i < end; ++k) {
      const int64_t row = i / tiles;
      const int t = static_cast<int>(i % tiles);
      const int b = static_cast<int>(row / P.s);
      const int a = k & 1;
      const int64_t inext = walk.next_valid(P, i + 1);
      if (row != prev_row) {
        // item k - 1 (the previous query's last) is folded by every fold warp and its MMAs are done:
        // the Q slabs and the head weights are free
        if (prev_row >= 0) fold_bar_and(true);
        img_query_store(qv, wl, sm.qh, sm.ql, sx.w);
        fence_async_smem();
        fold_bar_and(true);
        if (tid == 0) bar_arrive(&sx.q_ready);
        prev_row = row;
        if (inext < end && inext / tiles != row) img_query_load(P, inext / tiles, qv, wl);
      } else if (inext < end && inext / tiles != row) {
        img_query_load(P, inext / tiles, qv, wl);  // the next query's loads, one item ahead
      }
      const int j = t * BM + tid;
      const float ki = j < P.n_keys ? __ldg(P.kinv + static_cast<int64_t>(b) * P.img_tiles * BM + j) : 0.f;
      const bool ok = fold_bar_and(bar_wait_or_abort(&sx.acc_full[a], (k >> 1) & 1, abort));
      if (!ok) {
        if (tid == 0) img_set_abort(sx);
        break;
      }
      after_sync();
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
      for (int c = 0; c < HI; c += 16) {
        float sc[16];
        tmem_ld16(tmem + lq + a * HI + c, sc);
        tmem_wait_ld();
#pragma unroll
        for (int h = 0; h < 16; h += 4) {
          const float4 wv = *reinterpret_cast<const float4*>(&sx.w[c + h]);
          a0 = fmaf(wv.x, fmaxf(sc[h], 0.f), a0);
          a1 = fmaf(wv.y, fmaxf(sc[h + 1], 0.f), a1);
          a2 = fmaf(wv.z, fmaxf(sc[h + 2], 0.f), a2);
          a3 = fmaf(wv.w, fmaxf(sc[h + 3], 0.f), a3);
        }
      }
      if (j < P.n_keys) P.scores[row * P.n_pad + j] = ((a0 + a1) + (a2 + a3)) * ki;
      before_sync();
      __syncwarp();
      if (lane == 0) bar_arrive(&sx.acc_free[a]);
      i = inext;
    }
  }
  before_sync();
  __syncthreads();
  after_sync();
  if (warp == 0) tmem_dealloc<128>(tmem);
}

DSV4_ERROR_READER(indexer_tc)

cudaError_t launch_key_image(const ApproxArgs& a, cudaStream_t stream) {
  cudaError_t e = cudaMemsetAsync(a.kmax, 0, sizeof(float) * a.batch, stream);
  if (e != cudaSuccess) return e;
  key_image_kernel<<<dim3(key_tiles(a.n_keys), a.batch), BM, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_approx_scores(const ApproxArgs& a, cudaStream_t stream) {
  cudaError_t e = cudaSuccess;
  if (a.img_ready && row_kernel(a.s)) {  // decode over a cache-kept image: the walk without the split
    const int smem = static_cast<int>(sizeof(ImgSmem)) + 1024;
    static PerDeviceOnce iattr;
    e = set_smem_once(iattr, approx_score_img_kernel, smem);
    if (e != cudaSuccess) return e;
    const int64_t items = static_cast<int64_t>(a.batch) * a.s * key_tiles(a.n_keys);
    const int64_t ctas = num_sms();
    const int64_t per = (items + ctas - 1) / ctas;
    approx_score_img_kernel<<<static_cast<unsigned>((items + per - 1) / per), IM_THREADS, smem, stream>>>(a, per);
    return cudaGetLastError();
  }
  if (!a.img_ready) {
    e = cudaMemsetAsync(a.kmax, 0, sizeof(float) * a.batch, stream);
    if (e != cudaSuccess) return e;
  }
  if (row_kernel(a.s)) {
    const int64_t items = static_cast<int64_t>(a.batch) * a.s * key_tiles(a.n_keys);
    if (items >= 2 * static_cast<int64_t>(num_sms())) {  // at least two items per CTA: the pipelined walk
      const int smem = static_cast<int>(sizeof(SeqSmem)) + 1024;
      static PerDeviceOnce sattr;
      e = set_smem_once(sattr, approx_score_seq_kernel, smem);
      if (e != cudaSuccess) return e;
      const int64_t ctas = num_sms();
      const int64_t per = (items + ctas - 1) / ctas;
      approx_score_seq_kernel<<<static_cast<unsigned>((items + per - 1) / per), SQ_THREADS, smem, stream>>>(a, per);
      return cudaGetLastError();
    }
    const int smem = static_cast<int>(sizeof(RowSmem)) + 1024;
    static PerDeviceOnce rattr;
    e = set_smem_once(rattr, approx_score_row_kernel, smem);
    if (e != cudaSuccess) return e;
    approx_score_row_kernel<<<dim3(key_tiles(a.n_keys), static_cast<unsigned>(static_cast<int64_t>(a.batch) * a.s)),
                              RT_THREADS, smem, stream>>>(a);
    return cudaGetLastError();
  }
  if (!a.img_ready) {
    key_image_kernel<<<dim3(key_tiles(a.n_keys), a.batch), BM, 0, stream>>>(a);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  const int smem = static_cast<int>(sizeof(Smem)) + 1024;
  static PerDeviceOnce attr;
  e = set_smem_once(attr, approx_score_kernel, smem);
  if (e != cudaSuccess) return e;
  const int64_t groups = static_cast<int64_t>(a.batch) * ((a.s + QG - 1) / QG);
  approx_score_kernel<<<static_cast<unsigned>(groups), THREADS, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace itc
}  // namespace dsv4
