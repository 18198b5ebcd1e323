// Projection GEMM y = x W^T on the 5th-generation tensor cores, for prefill-shaped calls with bf16
// weights: the compressor's two projections (ref_torch/compressor.py:27-28, 62-63) and the MLA
// projections of a prefill (v4mlx/mla.py:16-56).
//
// x [m, groups*k] bf16 and W [rows, k] bf16, both K-major, are brought in by TMA (2-D tiled
// `cp.async.bulk.tensor`, 128-byte swizzle, out-of-range rows filled with zeros) through a 4-stage
// ring of mbarrier-tracked stages; one thread issues `tcgen05.mma` (M = 128 tokens, N = 256 weight
// rows, K = 16 per instruction) into an fp32 accumulator in tensor memory; four epilogue warps read
// the accumulator back with `tcgen05.ld` (warp w owns TMEM lanes 32 (w % 4) ..), convert and store.
// Two accumulators (512 TMEM columns) let the epilogue of one tile run under the next tile's MMAs.
// The grid is persistent (one CTA per SM, tiles strided by the grid size); consecutive tiles walk
// the weight-row tiles of one token tile first, so the CTAs running at the same time share the
// token tile through L2 and x streams from HBM about once.
//
// Each output element is the sum over k in the same order for any m or tile position (64-wide k
// steps in order, the MMA's fixed order inside a step), so a row's result does not depend on which
// rows are computed with it.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "tcgen05.cuh"

namespace dsv4 {
namespace gtc {
using namespace tc5;

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int THREADS = 192;  // warp 0: TMA producer; warp 1: MMA issuer; warps 2-5: epilogue
constexpr int EPI_WARPS = 4;
constexpr uint32_t A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2;
constexpr int TMEM_COLS = 2 * BN;
constexpr int MAXP = DSV4_LINEAR_MULTI_MAX;

struct Params {
  CUtensorMap tx;        // x: inner groups*k, outer m; box 64 x 128
  CUtensorMap tw[MAXP];  // W_p: inner k, outer rows; box 64 x 256
  void* y[MAXP];
  int n[MAXP], y_dtype[MAXP];
  int tile0[MAXP + 1];   // projection p owns the weight-row tiles [tile0[p], tile0[p + 1])
  int nprob;
  int64_t m;
  int k, groups;
  int64_t ldy;           // groups * n when nprob == 1 and groups > 1, else unused (n_p)
};

struct Smem {
  uint8_t a[STAGES][A_BYTES];  // 1024-byte aligned: the swizzle pattern repeats every 8 rows
  uint8_t b[STAGES][B_BYTES];
  uint64_t full[STAGES], empty[STAGES], acc_full[2], acc_empty[2], fin;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void set_abort(Smem& sm) {
  if (!*reinterpret_cast<volatile int*>(&sm.abort)) {
    *reinterpret_cast<volatile int*>(&sm.abort) = 1;
    raise_device_error(DSV4_ERR_WAIT_TIMEOUT);
  }
}

struct Tile {
  int64_t m0;
  int g, p, n0;
};
__device__ __forceinline__ Tile tile_at(const Params& P, int64_t t) {
  const int ntn = P.tile0[P.nprob];
  Tile T;
  const int nt = static_cast<int>(t % ntn);
  const int64_t rest = t / ntn;
  T.g = static_cast<int>(rest % P.groups);
  T.m0 = (rest / P.groups) * BM;
  int p = 0;
  while (p + 1 < P.nprob && nt >= P.tile0[p + 1]) ++p;
  T.p = p;
  T.n0 = (nt - P.tile0[p]) * BN;
  return T;
}

// 32 consecutive output columns of one row from fp32 registers
__device__ __forceinline__ void store_row32(void* y, int dtype, int64_t off, const float* v, int cols, bool vec) {
  if (dtype == DSV4_F32) {
    float* d = reinterpret_cast<float*>(y) + off;
    if (vec && cols == 32) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        reinterpret_cast<float4*>(d)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < cols) d[i] = v[i];
    }
  } else {
    __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(y) + off;
    if (vec && cols == 32) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 o;
        o.x = pack_bf16x2(v[8 * i], v[8 * i + 1]);
        o.y = pack_bf16x2(v[8 * i + 2], v[8 * i + 3]);
        o.z = pack_bf16x2(v[8 * i + 4], v[8 * i + 5]);
        o.w = pack_bf16x2(v[8 * i + 6], v[8 * i + 7]);
        reinterpret_cast<uint4*>(d)[i] = o;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < cols) d[i] = __float2bfloat16_rn(v[i]);
    }
  }
}

__global__ void __launch_bounds__(THREADS, 1) gemm_tc_kernel(const __grid_constant__ Params P) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t tiles = ((P.m + BM - 1) / BM) * P.groups * P.tile0[P.nprob];
  const int KT = P.k / BK;

  if (warp == 1) tmem_alloc<TMEM_COLS>(&sm.tmem_base);
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      bar_init(&sm.full[s], 1);
      bar_init(&sm.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      bar_init(&sm.acc_full[a], 1);
      bar_init(&sm.acc_empty[a], EPI_WARPS);
    }
    bar_init(&sm.fin, 1);
    sm.abort = 0;
    bar_init_fence();
    tma_prefetch_map(&P.tx);
    for (int p = 0; p < P.nprob; ++p) tma_prefetch_map(&P.tw[p]);
  }
  before_sync();
  __syncthreads();
  after_sync();
  const uint32_t tmem = sm.tmem_base;
  const volatile int* abort = &sm.abort;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      uint32_t armed = 0;  // stages whose last copy pair was issued (bit s), for the drain on abort
      uint32_t armed_ph = 0;
      for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const Tile T = tile_at(P, t);
        const int xcol0 = T.g * P.k;
        const int wrow0 = (P.nprob == 1 ? T.g * P.n[0] : 0) + T.n0;
        const int m0 = static_cast<int>(T.m0);
        for (int kt = 0; kt < KT; ++kt, ++it) {
          const int s = static_cast<int>(it % STAGES);
          const uint32_t ph = (it / STAGES) & 1;
          if (!(ok = bar_wait_or_abort(&sm.empty[s], ph ^ 1, abort))) break;
          bar_expect_tx(&sm.full[s], A_BYTES + B_BYTES);
          tma_load_2d(sm.a[s], &P.tx, xcol0 + kt * BK, m0, &sm.full[s]);
          tma_load_2d(sm.b[s], &P.tw[T.p], kt * BK, wrow0, &sm.full[s]);
          armed |= 1u << s;
          armed_ph = (armed_ph & ~(1u << s)) | (ph << s);
        }
      }
      if (!ok) {
        set_abort(sm);
        // the copies already issued must land before the CTA's shared memory goes away
        for (int s = 0; s < STAGES; ++s)
          if (armed & (1u << s)) bar_wait(&sm.full[s], (armed_ph >> s) & 1);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t id = idesc_bf16<BM, BN>(false, false);
      uint32_t it = 0, tl = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++tl) {
        const int a = tl & 1;
        const uint32_t aph = (tl >> 1) & 1;
        if (!(ok = bar_wait_or_abort(&sm.acc_empty[a], aph ^ 1, abort))) break;
        after_sync();
        const uint32_t d = tmem + a * BN;
        for (int kt = 0; kt < KT; ++kt, ++it) {
          const int s = static_cast<int>(it % STAGES);
          const uint32_t ph = (it / STAGES) & 1;
          if (!(ok = bar_wait_or_abort(&sm.full[s], ph, abort))) break;
          after_sync();
          const uint32_t as = smem_u32(sm.a[s]), bs = smem_u32(sm.b[s]);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma16(d, sdesc(as + kk * 32, 16, 1024), sdesc(bs + kk * 32, 16, 1024), id, (kt | kk) ? 1u : 0u);
          mma_commit(&sm.empty[s]);  // the stage is free once these MMAs have read it
        }
        if (!ok) break;
        mma_commit(&sm.acc_full[a]);
      }
      // every MMA issued (also on abort) has completed before the CTA may leave
      mma_commit(&sm.fin);
      bar_wait(&sm.fin, 0);
      if (!ok) set_abort(sm);
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2-5)
    const int e = warp & 3;  // TMEM lanes [32 e, 32 e + 32): the tile's rows 32 e ..
    uint32_t tl = 0;
    for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x, ++tl) {
      const int a = tl & 1;
      const uint32_t aph = (tl >> 1) & 1;
      const bool ok = __all_sync(0xffffffffu, bar_wait_or_abort(&sm.acc_full[a], aph, abort));
      if (!ok) {
        if (lane == 0) set_abort(sm);
        break;
      }
      after_sync();
      const Tile T = tile_at(P, t);
      const int np = P.n[T.p], dt = P.y_dtype[T.p];
      void* y = P.y[T.p];
      const int64_t ldy = P.nprob == 1 ? P.ldy : np;
      const int64_t row = T.m0 + 32 * e + lane;
      const int64_t col0 = static_cast<int64_t>(T.g) * np + T.n0;
      const bool vec = (reinterpret_cast<uintptr_t>(y) & 15) == 0 && ldy % (dt == DSV4_F32 ? 4 : 8) == 0 &&
                       col0 % (dt == DSV4_F32 ? 4 : 8) == 0;
      const uint32_t tb = tmem + (static_cast<uint32_t>(32 * e) << 16) + a * BN;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        float v[32];
        tmem_ld16(tb + c, v);
        tmem_ld16(tb + c + 16, v + 16);
        tmem_wait_ld();
        const int cols = min(32, np - T.n0 - c);
        if (row < P.m && cols > 0) store_row32(y, dt, row * ldy + col0 + c, v, cols, vec);
      }
      before_sync();
      __syncwarp();
      if (lane == 0) bar_arrive(&sm.acc_empty[a]);
    }
  }
  before_sync();
  __syncthreads();
  after_sync();
  if (warp == 1) tmem_dealloc<TMEM_COLS>(tmem);
}

DSV4_ERROR_READER(gemm_tc)

// ---------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::atomic<void*> fn{nullptr};
  void* f = fn.load(std::memory_order_acquire);
  if (!f) {
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    if (f) fn.store(f, std::memory_order_release);
  }
  return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
}

// bf16 [rows, inner] row-major (row stride `ld` elements), box (64 inner) x box_rows, 128-byte swizzle
static int encode_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t ld,
                       uint32_t box_rows) {
  auto enc = encode_fn();
  if (!enc) {
    set_error("dsv4_linear: cuTensorMapEncodeTiled is not available from the driver");
    return DSV4_ERR_CUDA;
  }
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {ld * 2};
  const cuuint32_t box[2] = {BK, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("dsv4_linear: cuTensorMapEncodeTiled failed (%d) for a [%llu, %llu] operand", static_cast<int>(r),
              static_cast<unsigned long long>(rows), static_cast<unsigned long long>(inner));
    return DSV4_ERR_CUDA;
  }
  return DSV4_OK;
}

}  // namespace gtc

// Output tiles of a tcgen05 GEMM over these problems (weight-row tiles of 256, token tiles of 128).
int64_t gemm_tc_tiles(int64_t m, int groups, const int* n, int nprob) {
  int64_t nt = 0;
  for (int p = 0; p < nprob; ++p) nt += (n[p] + gtc::BN - 1) / gtc::BN;
  return ((m + gtc::BM - 1) / gtc::BM) * groups * nt;
}

// y_p[m, groups * n_p] = x[m, groups * k] . W_p^T, bf16 x and W (16-byte aligned), k % 64 == 0;
// nprob == 1 with any groups, or up to DSV4_LINEAR_MULTI_MAX problems with groups == 1
int gemm_tc_launch(const void* x, int64_t m, int k, int groups, const void* const* w, void* const* y, const int* n,
                   const int* y_dtype, int nprob, void* stream) {
  DSV4_CHECK_ARG(nprob >= 1 && nprob <= gtc::MAXP && (nprob == 1 || groups == 1), "dsv4_linear: bad problem count");
  DSV4_CHECK_ARG(k % gtc::BK == 0 && m > 0 && m <= (int64_t{1} << 31) - 1, "dsv4_linear: bad sizes for tcgen05");
  DSV4_CHECK_ARG(static_cast<int64_t>(groups) * k <= (int64_t{1} << 31) - 1, "dsv4_linear: groups * k too large");
  gtc::Params P = {};
  int rc = gtc::encode_bf16(&P.tx, x, static_cast<uint64_t>(groups) * k, static_cast<uint64_t>(m),
                            static_cast<uint64_t>(groups) * k, gtc::BM);
  if (rc != DSV4_OK) return rc;
  int tiles_n = 0;
  for (int p = 0; p < nprob; ++p) {
    DSV4_CHECK_ARG(n[p] > 0 && static_cast<int64_t>(groups) * n[p] <= (int64_t{1} << 31) - 1, "dsv4_linear: bad n");
    rc = gtc::encode_bf16(&P.tw[p], w[p], static_cast<uint64_t>(k), static_cast<uint64_t>(groups) * n[p],
                          static_cast<uint64_t>(k), gtc::BN);
    if (rc != DSV4_OK) return rc;
    P.y[p] = y[p];
    P.n[p] = n[p];
    P.y_dtype[p] = y_dtype[p];
    P.tile0[p] = tiles_n;
    tiles_n += (n[p] + gtc::BN - 1) / gtc::BN;
  }
  P.tile0[nprob] = tiles_n;
  P.nprob = nprob;
  P.m = m;
  P.k = k;
  P.groups = groups;
  P.ldy = static_cast<int64_t>(groups) * n[0];
  const int64_t tiles = gemm_tc_tiles(m, groups, n, nprob);
  static PerDeviceOnce set;
  const int smem = static_cast<int>(sizeof(gtc::Smem)) + 1024;
  DSV4_CUDA_CHECK(set_smem_once(set, gtc::gemm_tc_kernel, smem));
  const int grid = static_cast<int>(std::min<int64_t>(tiles, num_sms()));
  gtc::gemm_tc_kernel<<<grid, gtc::THREADS, smem, as_stream(stream)>>>(P);
  DSV4_LAUNCH_CHECK("gemm_tc_kernel");
  return DSV4_OK;
}

}  // namespace dsv4
