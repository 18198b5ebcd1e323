// Approximate lightning-indexer scores on the 5th-generation tensor cores (the filter stage of the
// bit-exact top-k; the error bound and the exact rescoring live with the selection in indexer.cu).
//
// key_image_kernel: every key row (fp32) -> bf16 hi = rn(k), lo = rn(k - hi), written as the shared
//   memory image of its 128-key tile ([hi slab 0 | hi slab 1 | lo slab 0 | lo slab 1], 128-byte
//   swizzled, 16 KB each) so that one bulk copy per half lands a tile ready for the MMA; and the
//   maximum key norm per batch entry (an upper bound for the error term).
// approx_score_kernel: one CTA per 4 consecutive queries (N = 4 x 64 heads = 256 columns), looping
//   over the key tiles visible to the last of them. Per tile, on M = 128 keys, K = 128 dims:
//     S^T[key, (q,h)] = kl.qh  (pass A, reads the lo half)  + kh.qh + kh.ql  (passes B, C)
//   into one of two 256-column TMEM buffers. Warp 4 (one elected lane) streams the tile halves with
//   bulk copies and issues the MMAs: the lo half of tile i+1 is fetched while passes B, C of tile i
//   run, the hi half while pass A of tile i+1 runs. Warps 0-3 (thread = key) read the finished
//   buffer, fold sum_h w[q,h] * relu(s) for the 4 queries and store 4 scores per key.
// All waits are bounded (1 s); a timeout raises DSV4_ERR_WAIT_TIMEOUT and the CTA winds down.
#include "common.cuh"
#include "indexer_tc.cuh"
#include "tcgen05.cuh"

namespace dsv4 {
namespace itc {

using namespace tc5;

constexpr int DI = 128, HI = 64, QG = 4, NQ = QG * HI;
constexpr int THREADS = 160;            // warps 0-3 epilogue, warp 4 producer
constexpr int SLAB_Q = NQ * 128;        // 32 KB: 256 (query, head) rows x 64 bf16 dims
constexpr int SLAB_K = BM * 128;        // 16 KB: 128 keys x 64 bf16 dims
constexpr int HALF = 2 * SLAB_K;        // 32 KB: hi or lo of one tile
static_assert(TILE_BYTES == 2 * HALF, "tile image");
constexpr int TMEM_COLS = 512;

struct Smem {
  alignas(1024) uint8_t qh[2 * SLAB_Q];
  alignas(1024) uint8_t ql[2 * SLAB_Q];
  alignas(1024) uint8_t kh[HALF];
  alignas(1024) uint8_t kl[HALF];
  float w[QG][HI];
  uint64_t bar_kh, bar_kl, bar_lo_done;
  uint64_t bar_hi_done[2], bar_free[2];
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ uint32_t pack2(__nv_bfloat16 a, __nv_bfloat16 b) {
  return static_cast<uint32_t>(__bfloat16_as_ushort(a)) | (static_cast<uint32_t>(__bfloat16_as_ushort(b)) << 16);
}
// 4 fp32 -> (hi, lo) as two 8-byte groups of 4 bf16
__device__ __forceinline__ void split4(float4 v, uint2* hi, uint2* lo) {
  const __nv_bfloat16 h0 = __float2bfloat16_rn(v.x), h1 = __float2bfloat16_rn(v.y);
  const __nv_bfloat16 h2 = __float2bfloat16_rn(v.z), h3 = __float2bfloat16_rn(v.w);
  const __nv_bfloat16 l0 = __float2bfloat16_rn(v.x - __bfloat162float(h0));
  const __nv_bfloat16 l1 = __float2bfloat16_rn(v.y - __bfloat162float(h1));
  const __nv_bfloat16 l2 = __float2bfloat16_rn(v.z - __bfloat162float(h2));
  const __nv_bfloat16 l3 = __float2bfloat16_rn(v.w - __bfloat162float(h3));
  *hi = make_uint2(pack2(h0, h1), pack2(h2, h3));
  *lo = make_uint2(pack2(l0, l1), pack2(l2, l3));
}

// grid (tiles, batch), 128 threads: thread = key row of the tile
__global__ void __launch_bounds__(BM) key_image_kernel(ApproxArgs P) {
  const int t = blockIdx.x, b = blockIdx.y, r = threadIdx.x;
  const int j = t * BM + r;
  const int tiles = key_tiles(P.n_keys);
  uint8_t* img = P.kimg + (static_cast<int64_t>(b) * tiles + t) * TILE_BYTES;
  const float* kr = P.k + (static_cast<int64_t>(b) * P.k_batch_stride + j) * DI;
  float ss = 0.f;
#pragma unroll 4
  for (int f = 0; f < DI / 4; ++f) {
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (j < P.n_keys) v = __ldg(reinterpret_cast<const float4*>(kr) + f);
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    ss = fmaf(v.w, v.w, ss);
    uint2 hi, lo;
    split4(v, &hi, &lo);
    const uint32_t off = slab_off(r, f >> 1, SLAB_K) + (f & 1) * 8;
    *reinterpret_cast<uint2*>(img + off) = hi;
    *reinterpret_cast<uint2*>(img + HALF + off) = lo;
  }
  // non-negative floats order like their bit patterns
  if (j < P.n_keys) atomicMax(reinterpret_cast<unsigned int*>(P.kmax + b), __float_as_uint(sqrtf(ss)));
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

  // stage w and the split Q (rows r = q*64 + h)
  for (int i = tid; i < QG * HI; i += THREADS) {
    const int q = i / HI;
    sm.w[q][i % HI] = q < nq ? P.w[(row0 + q) * HI + i % HI] : 0.f;
  }
  for (int i = tid; i < NQ * DI / 4; i += THREADS) {
    const int r = i >> 5, f = i & 31;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if ((r >> 6) < nq) v = __ldg(reinterpret_cast<const float4*>(P.q + (row0 * HI + r) * DI) + f);
    uint2 hi, lo;
    split4(v, &hi, &lo);
    const uint32_t off = slab_off(r, f >> 1, SLAB_Q) + (f & 1) * 8;
    *reinterpret_cast<uint2*>(sm.qh + off) = hi;
    *reinterpret_cast<uint2*>(sm.ql + off) = lo;
  }
  if (warp == 0) tmem_alloc<TMEM_COLS>(&sm.tmem_base);
  if (tid == 0) {
    bar_init(&sm.bar_kh, 1);
    bar_init(&sm.bar_kl, 1);
    bar_init(&sm.bar_lo_done, 1);
    for (int i = 0; i < 2; ++i) {
      bar_init(&sm.bar_hi_done[i], 1);
      bar_init(&sm.bar_free[i], 4);
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

  if (warp == 4) {
    if (lane == 0) {
      const int tiles = key_tiles(P.n_keys);
      const uint8_t* img = P.kimg + static_cast<int64_t>(b) * tiles * TILE_BYTES;
      constexpr uint32_t id = idesc_bf16<128, NQ>(false, false);
      const uint32_t qh = smem_u32(sm.qh), ql = smem_u32(sm.ql), kh = smem_u32(sm.kh), kl = smem_u32(sm.kl);
      bool ok = true;
      bool kl_pending = false, kh_pending = false;  // a bulk copy issued and not yet waited for
      uint32_t k_par = 0;                           // its phase parity (tile index & 1)
      uint64_t* last_bar = nullptr;                 // the last commit and its phase parity
      uint32_t last_par = 0;
      for (int i = 0; i < T && ok; ++i) {
        const int buf = i & 1;
        const uint32_t d = tmem + static_cast<uint32_t>(buf * 256);
        // the lo half is free once pass A of tile i-1 is done
        if (i > 0 && !(ok = bar_wait_or_abort(&sm.bar_lo_done, (i - 1) & 1, abort))) break;
        bar_expect_tx(&sm.bar_kl, HALF);
        bulk_g2s(sm.kl, img + static_cast<int64_t>(i) * TILE_BYTES + HALF, HALF, &sm.bar_kl);
        kl_pending = true;
        k_par = i & 1;
        // TMEM buffer `buf` is free once the epilogue has read tile i-2
        if (i >= 2 && !(ok = bar_wait_or_abort(&sm.bar_free[buf], ((i - 2) >> 1) & 1, abort))) break;
        if (!(ok = bar_wait_or_abort(&sm.bar_kl, i & 1, abort))) break;
        kl_pending = false;
        after_sync();
#pragma unroll
        for (int k8 = 0; k8 < 8; ++k8)
          mma_bf16(d, sdesc(kl + (k8 >> 2) * SLAB_K + (k8 & 3) * 32, 16, 1024),
                   sdesc(qh + (k8 >> 2) * SLAB_Q + (k8 & 3) * 32, 16, 1024), id, k8 > 0 ? 1u : 0u);
        mma_commit(&sm.bar_lo_done);
        last_bar = &sm.bar_lo_done;
        last_par = i & 1;
        // the hi half is free once passes B, C of tile i-1 are done
        if (i > 0 && !(ok = bar_wait_or_abort(&sm.bar_hi_done[buf ^ 1], ((i - 1) >> 1) & 1, abort))) break;
        bar_expect_tx(&sm.bar_kh, HALF);
        bulk_g2s(sm.kh, img + static_cast<int64_t>(i) * TILE_BYTES, HALF, &sm.bar_kh);
        kh_pending = true;
        k_par = i & 1;
        if (!(ok = bar_wait_or_abort(&sm.bar_kh, i & 1, abort))) break;
        kh_pending = false;
        after_sync();
#pragma unroll
        for (int k8 = 0; k8 < 8; ++k8)
          mma_bf16(d, sdesc(kh + (k8 >> 2) * SLAB_K + (k8 & 3) * 32, 16, 1024),
                   sdesc(qh + (k8 >> 2) * SLAB_Q + (k8 & 3) * 32, 16, 1024), id, 1u);
#pragma unroll
        for (int k8 = 0; k8 < 8; ++k8)
          mma_bf16(d, sdesc(kh + (k8 >> 2) * SLAB_K + (k8 & 3) * 32, 16, 1024),
                   sdesc(ql + (k8 >> 2) * SLAB_Q + (k8 & 3) * 32, 16, 1024), id, 1u);
        mma_commit(&sm.bar_hi_done[buf]);
        last_bar = &sm.bar_hi_done[buf];
        last_par = (i >> 1) & 1;
      }
      if (!ok) {
        set_abort(sm);
        // let what was issued land before the CTA's shared and tensor memory go away
        if (kl_pending) bar_wait(&sm.bar_kl, k_par);
        if (kh_pending) bar_wait(&sm.bar_kh, k_par);
        if (last_bar) bar_wait(last_bar, last_par);
      }
    }
    __syncwarp();
  } else {
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    for (int i = 0; i < T; ++i) {
      const int buf = i & 1;
      const bool ok = bar_wait_or_abort(&sm.bar_hi_done[buf], (i >> 1) & 1, abort);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) set_abort(sm);
        break;
      }
      after_sync();
      float acc[QG];
#pragma unroll
      for (int q = 0; q < QG; ++q) {
        float v[HI];
#pragma unroll
        for (int c = 0; c < HI; c += 16) tmem_ld16(tmem + lane_base + buf * 256 + q * HI + c, v + c);
        tmem_wait_ld();
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
        for (int h = 0; h < HI; h += 4) {
          const float4 wv = *reinterpret_cast<const float4*>(&sm.w[q][h]);
          a0 = fmaf(wv.x, fmaxf(v[h], 0.f), a0);
          a1 = fmaf(wv.y, fmaxf(v[h + 1], 0.f), a1);
          a2 = fmaf(wv.z, fmaxf(v[h + 2], 0.f), a2);
          a3 = fmaf(wv.w, fmaxf(v[h + 3], 0.f), a3);
        }
        acc[q] = (a0 + a1) + (a2 + a3);
      }
      before_sync();
      __syncwarp();
      if (lane == 0) bar_arrive(&sm.bar_free[buf]);
      const int key = i * BM + warp * 32 + lane;
      if (key < P.n_keys)
#pragma unroll
        for (int q = 0; q < QG; ++q)
          if (q < nq) P.scores[(row0 + q) * P.n_pad + key] = acc[q];
    }
  }
  before_sync();
  __syncthreads();
  after_sync();
  if (warp == 0) tmem_dealloc<TMEM_COLS>(tmem);
}

DSV4_ERROR_READER(indexer_tc)

cudaError_t launch_approx_scores(const ApproxArgs& a, cudaStream_t stream) {
  cudaError_t e = cudaMemsetAsync(a.kmax, 0, sizeof(float) * a.batch, stream);
  if (e != cudaSuccess) return e;
  key_image_kernel<<<dim3(key_tiles(a.n_keys), a.batch), BM, 0, stream>>>(a);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  const int smem = static_cast<int>(sizeof(Smem)) + 1024;
  static bool attr = false;
  if (!attr) {
    e = cudaFuncSetAttribute(approx_score_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const int64_t groups = static_cast<int64_t>(a.batch) * ((a.s + QG - 1) / QG);
  approx_score_kernel<<<static_cast<unsigned>(groups), THREADS, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace itc
}  // namespace dsv4
