// Projection GEMM y = x W^T for the MLA projections (v4mlx/mla.py:16-56) and the compressor's
// two projections (ref_torch/compressor.py:62-63).
//
// x [m, k] bf16 (K-major), W [n, k] (K-major) as bf16, or int8 with one bf16 scale per
// (row, 64-wide group of k) — the 8-bit grouped weights of the fast decode block
// (oracle/v4_fast.py:31-34, symmetric here). The int8 tile is widened to bf16 in shared memory
// (exact: |q| <= 127), each 64-wide k group is accumulated separately in fp32 and folded into the
// output with its scale, so the dequantised product is computed without rounding the weights.
// CTA tile 128 x 128 x 64, 8 warps (2 x 4), warp tile 64 x 32, bf16 mma.sync, 3-stage cp.async.
#include <algorithm>
#include <cstddef>
#include "common.cuh"

namespace dsv4 {
namespace gm {

constexpr int BM = 128, BN = 128, BK = 64, STAGES = 3, THREADS = 256;

__device__ __forceinline__ uint32_t swz128(int r, int c) {  // 128-byte rows, 8 chunks
  return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}
__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g, bool valid) {
  int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(saddr), "l"(g), "r"(sz));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// d = A.B (no accumulator input)
__device__ __forceinline__ void mma_bf16_z(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  const float z = 0.f;
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%10,%10,%10};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(z));
}
__device__ __forceinline__ void mma_bf16(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

struct Params {
  const __nv_bfloat16* x;   // [m, groups*k]
  const void* w;            // [groups*n, k]
  const __nv_bfloat16* ws;  // [groups*n, k/64] when int8
  void* y;                  // [m, groups*n]
  int64_t m;
  int n, k, groups;
  int y_dtype;
  int ksplit;               // CTAs along k; > 1: fp32 partials [ksplit][m][groups*n] into part
  float* part;
  // nprob > 0 (decode-shaped kernel, groups == 1): several projections of the same x in one launch;
  // projection p owns the 128-row tiles [tile0, tile0 + ceil(n / 128)) of grid.x, and w, ws, y, n,
  // y_dtype above are replaced by its own
  int nprob;
  struct Prob {
    const void* w;
    const __nv_bfloat16* ws;
    void* y;
    int n, y_dtype, tile0;
  } prob[DSV4_LINEAR_MULTI_MAX];
};

template <bool I8>
struct Smem {
  alignas(128) uint8_t a[STAGES][BM * BK * 2];
  alignas(128) uint8_t b[STAGES][BN * BK * (I8 ? 1 : 2)];
  alignas(128) uint8_t bw[I8 ? BN * BK * 2 : 16];  // widened int8 tile
};

template <bool I8>
__device__ __forceinline__ void load_stage(const Params& P, Smem<I8>& sm, int st, int64_t m0, int n0,
                                           int kt, int g) {
  const int tid = threadIdx.x;
  const int64_t lda = static_cast<int64_t>(P.groups) * P.k;
  const __nv_bfloat16* xa = P.x + static_cast<int64_t>(g) * P.k + kt * BK;
  const uint32_t as = static_cast<uint32_t>(__cvta_generic_to_shared(sm.a[st]));
#pragma unroll
  for (int i = 0; i < (BM * BK / 8) / THREADS; ++i) {  // 1024 chunks
    int c = tid + i * THREADS;
    int r = c >> 3, ch = c & 7;
    bool v = (m0 + r) < P.m;
    const __nv_bfloat16* src = xa + (v ? (m0 + r) : 0) * lda + ch * 8;
    cp_async16(as + swz128(r, ch), src, v);
  }
  const uint32_t bs = static_cast<uint32_t>(__cvta_generic_to_shared(sm.b[st]));
  const int64_t wrow0 = static_cast<int64_t>(g) * P.n + n0;
  if constexpr (I8) {
    const int8_t* wb = reinterpret_cast<const int8_t*>(P.w);
#pragma unroll
    for (int i = 0; i < (BN * BK / 16) / THREADS; ++i) {  // 512 chunks, 4 per 64-byte row
      int c = tid + i * THREADS;
      int r = c >> 2, ch = c & 3;
      bool v = (n0 + r) < P.n;
      const int8_t* src = wb + (wrow0 + (v ? r : 0)) * P.k + kt * BK + ch * 16;
      cp_async16(bs + r * 64 + ch * 16, src, v);
    }
  } else {
    const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(P.w);
#pragma unroll
    for (int i = 0; i < (BN * BK / 8) / THREADS; ++i) {
      int c = tid + i * THREADS;
      int r = c >> 3, ch = c & 7;
      bool v = (n0 + r) < P.n;
      const __nv_bfloat16* src = wb + (wrow0 + (v ? r : 0)) * P.k + kt * BK + ch * 8;
      cp_async16(bs + swz128(r, ch), src, v);
    }
  }
}

template <bool I8>
__global__ void __launch_bounds__(THREADS) gemm_kernel(Params P) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Smem<I8>& sm = *reinterpret_cast<Smem<I8>*>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int wm = warp >> 2, wn = warp & 3;  // 2 x 4 warps
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * BM;
  const int n0 = blockIdx.x * BN;
  const int g = blockIdx.z / P.ksplit;
  const int split = blockIdx.z % P.ksplit;
  const int KT = P.k / BK;
  const int per = (KT + P.ksplit - 1) / P.ksplit;
  const int kt0 = split * per;
  const int nkt = max(0, min(per, KT - kt0));  // k tiles [kt0, kt0 + nkt) of this CTA

  float acc[4][4][4];
  float gacc[4][4][4];  // per-group partial (int8 weights only)
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[a][b][c] = 0.f;

#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < nkt) load_stage<I8>(P, sm, s, m0, n0, kt0 + s, g);
    asm volatile("cp.async.commit_group;\n" ::);
  }

  for (int it = 0; it < nkt; ++it) {
    const int kt = kt0 + it;
    const int st = it % STAGES;
    asm volatile("cp.async.wait_group %0;\n" ::"n"(STAGES - 2));
    __syncthreads();
    {
      int nk = it + STAGES - 1;
      if (nk < nkt) load_stage<I8>(P, sm, nk % STAGES, m0, n0, kt0 + nk, g);
      asm volatile("cp.async.commit_group;\n" ::);
    }
    uint32_t bsm;
    if constexpr (I8) {
      // widen the int8 tile to bf16 (swizzled like a bf16 tile)
      const int8_t* src = reinterpret_cast<const int8_t*>(sm.b[st]);
      for (int c = tid; c < BN * BK / 8; c += THREADS) {
        int r = c >> 3, ch = c & 7;
        uint2 raw = *reinterpret_cast<const uint2*>(src + r * 64 + ch * 8);
        const int8_t* q8 = reinterpret_cast<const int8_t*>(&raw);
        uint4 o;
        o.x = pack_bf16x2(static_cast<float>(q8[0]), static_cast<float>(q8[1]));
        o.y = pack_bf16x2(static_cast<float>(q8[2]), static_cast<float>(q8[3]));
        o.z = pack_bf16x2(static_cast<float>(q8[4]), static_cast<float>(q8[5]));
        o.w = pack_bf16x2(static_cast<float>(q8[6]), static_cast<float>(q8[7]));
        *reinterpret_cast<uint4*>(sm.bw + swz128(r, ch)) = o;
      }
      __syncthreads();
      bsm = static_cast<uint32_t>(__cvta_generic_to_shared(sm.bw));
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b)
#pragma unroll
          for (int c = 0; c < 4; ++c) gacc[a][b][c] = 0.f;
    } else {
      bsm = static_cast<uint32_t>(__cvta_generic_to_shared(sm.b[st]));
    }
    const uint32_t asm_ = static_cast<uint32_t>(__cvta_generic_to_shared(sm.a[st]));
#pragma unroll
    for (int kk = 0; kk < BK / 16; ++kk) {
      uint32_t af[4][4], bf[4][2];
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        int r = wm * 64 + mt * 16 + (lane & 15);
        ldsm_x4(asm_ + swz128(r, kk * 2 + (lane >> 4)), af[mt][0], af[mt][1], af[mt][2], af[mt][3]);
      }
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        int r = wn * 32 + np * 16 + (lane & 7) + ((lane >> 4) << 3);
        ldsm_x4(bsm + swz128(r, kk * 2 + ((lane >> 3) & 1)), bf[np * 2][0], bf[np * 2][1],
                bf[np * 2 + 1][0], bf[np * 2 + 1][1]);
      }
#pragma unroll
      for (int mt = 0; mt < 4; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          if constexpr (I8)
            mma_bf16(gacc[mt][nt], af[mt], bf[nt][0], bf[nt][1]);
          else
            mma_bf16(acc[mt][nt], af[mt], bf[nt][0], bf[nt][1]);
        }
    }
    if constexpr (I8) {
      // fold the 64-wide group with its per-row scale
      const int kg = kt;  // BK == group
      const int64_t nrow0 = static_cast<int64_t>(g) * P.n + n0 + wn * 32;
      const int ngroups = P.k / 64;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        int nl = nt * 8 + (lane & 3) * 2;
        float s0 = 0.f, s1 = 0.f;
        if (n0 + wn * 32 + nl < P.n) s0 = __bfloat162float(P.ws[(nrow0 + nl) * ngroups + kg]);
        if (n0 + wn * 32 + nl + 1 < P.n) s1 = __bfloat162float(P.ws[(nrow0 + nl + 1) * ngroups + kg]);
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
          acc[mt][nt][0] = fmaf(gacc[mt][nt][0], s0, acc[mt][nt][0]);
          acc[mt][nt][1] = fmaf(gacc[mt][nt][1], s1, acc[mt][nt][1]);
          acc[mt][nt][2] = fmaf(gacc[mt][nt][2], s0, acc[mt][nt][2]);
          acc[mt][nt][3] = fmaf(gacc[mt][nt][3], s1, acc[mt][nt][3]);
        }
      }
      __syncthreads();  // bw is rewritten next step
    }
  }
  asm volatile("cp.async.wait_group 0;\n" ::);

  // epilogue
  const int64_t ldy = static_cast<int64_t>(P.groups) * P.n;
#pragma unroll
  for (int mt = 0; mt < 4; ++mt)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int64_t row = m0 + wm * 64 + mt * 16 + hf * 8 + (lane >> 2);
      if (row >= P.m) continue;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int col = n0 + wn * 32 + nt * 8 + (lane & 3) * 2;
        if (col >= P.n) continue;
        const int64_t off = row * ldy + static_cast<int64_t>(g) * P.n + col;
        float v0 = acc[mt][nt][hf * 2], v1 = acc[mt][nt][hf * 2 + 1];
        if (P.ksplit > 1) {
          // fp32 partial of this k range (col is even, n is even: 8-byte aligned pairs)
          *reinterpret_cast<float2*>(P.part + static_cast<int64_t>(split) * P.m * ldy + off) = make_float2(v0, v1);
        } else if (P.y_dtype == DSV4_BF16) {
          if (col + 1 < P.n)
            *reinterpret_cast<uint32_t*>(reinterpret_cast<__nv_bfloat16*>(P.y) + off) = pack_bf16x2(v0, v1);
          else
            reinterpret_cast<__nv_bfloat16*>(P.y)[off] = __float2bfloat16_rn(v0);
        } else {
          float* y = reinterpret_cast<float*>(P.y) + off;
          if (col + 1 < P.n && (off & 1) == 0) {
            *reinterpret_cast<float2*>(y) = make_float2(v0, v1);
          } else {
            y[0] = v0;
            if (col + 1 < P.n) y[1] = v1;
          }
        }
      }
    }
}

// ---------------------------------------------------------------------------------------------
// Decode-shaped projections (m <= 64 tokens): the weights are the only traffic that matters, so the
// CTA streams 128 weight rows x its k range through a cp.async ring and the tokens ride along as
// the small operand. Swapped roles: the MMA's A (16 rows) is a slice of W, its B (8 columns) eight
// tokens, D = W x^T. Every lane reads 16 contiguous k of one row and its tokens at the same
// positions, so the k order inside a 64-wide group is permuted identically in both operands (slot
// 2q+e / 2q+8+e of k-step j is element 16q + 4j + e / 16q + 4j + 2 + e); the sum is unchanged.
// int8 weights are widened in registers exactly (|q| <= 128 fits the 8 significant bits of bf16),
// each group accumulates in fp32 and folds with its scale, as in the tiled kernel.
namespace sk {

// RW m16 row tiles per warp: the CTA's 128 weight rows are 8 warps x 16 rows (RW = 1) or 4 warps x
// 32 rows (RW = 2, the tokens' fragments then serve two row tiles)
constexpr int ROWS = 128, BK = 64;
template <int RW>
constexpr int threads_for() {
  return (ROWS / (16 * RW)) * 32;
}

template <bool I8>
struct Cfg {
  // ring depth: 4 stages (32 KB of int8 weights) leave room for three CTAs per SM, whose warps hide
  // each other's latency better than deeper rings at two CTAs (config 5 step: 180 us against 192 us
  // with 8 stages, 182 with 5)
  static constexpr int NST = 4;
  static constexpr int ROW_BYTES = BK * (I8 ? 1 : 2);
};

template <bool I8, int MT>
struct Smem {
  alignas(128) uint8_t w[Cfg<I8>::NST][ROWS * Cfg<I8>::ROW_BYTES];
  alignas(128) uint8_t x[Cfg<I8>::NST][MT * 8 * 128];  // 8*MT tokens x 64 bf16, chunk c at c ^ (t % 8)
  float scale[I8 ? Cfg<I8>::NST : 1][ROWS];
};

__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}

// two signed bytes of w (bytes 2h, 2h+1) -> bf16x2, exact: 2^23 + (b ^ 0x80) as an fp32 bit pattern,
// minus 2^23 + 128, is b (both subtractions in one packed f32x2 add); an integer of magnitude
// <= 128 is its own bf16 (the fp32's upper half)
__device__ __forceinline__ uint32_t s8x2_bf16x2(uint32_t u, int h) {  // u = w ^ 0x80808080
  const uint32_t f0 = __byte_perm(u, 0x4B000000u, h ? 0x7442 : 0x7440);
  const uint32_t f1 = __byte_perm(u, 0x4B000000u, h ? 0x7443 : 0x7441);
  const uint64_t m = 0xCB000080CB000080ull;  // (-(2^23 + 128), -(2^23 + 128))
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;\n" : "=l"(d) : "l"((static_cast<uint64_t>(f1) << 32) | f0), "l"(m));
  return __byte_perm(static_cast<uint32_t>(d), static_cast<uint32_t>(d >> 32), 0x7632);
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
// fp32 at shared address `a` of the CTA with rank `rank` in this cluster
__device__ __forceinline__ float ld_dsmem_f32(uint32_t a, int rank) {
  uint32_t ra;
  float v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(ra) : "r"(a), "r"(rank));
  asm volatile("ld.shared::cluster.f32 %0, [%1];\n" : "=f"(v) : "r"(ra) : "memory");
  return v;
}
__device__ __forceinline__ void store_y(const Params& P, int64_t off, float v) {
  if (P.y_dtype == DSV4_BF16)
    reinterpret_cast<__nv_bfloat16*>(P.y)[off] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<float*>(P.y)[off] = v;
}

template <bool I8, int MT, int NT>
__device__ __forceinline__ void load_w(const Params& P, Smem<I8, MT>& sm, int st, int n0, int kg, int g) {
  const int tid = threadIdx.x;
  constexpr int CH = Cfg<I8>::ROW_BYTES / 16;  // 16-byte chunks per weight row
  const uint8_t* wb = reinterpret_cast<const uint8_t*>(P.w) +
                      (static_cast<int64_t>(g) * P.n * P.k + static_cast<int64_t>(kg) * BK) * (I8 ? 1 : 2);
  const uint32_t ws = static_cast<uint32_t>(__cvta_generic_to_shared(sm.w[st]));
#pragma unroll
  for (int i = 0; i < ROWS * CH / NT; ++i) {
    const int c = tid + i * NT;
    const int r = c / CH, ch = c % CH;
    const bool v = n0 + r < P.n;
    const uint8_t* src = wb + static_cast<int64_t>(v ? n0 + r : 0) * P.k * (I8 ? 1 : 2) + ch * 16;
    cp_async16(ws + r * Cfg<I8>::ROW_BYTES + ((I8 ? ch : (ch ^ (r & 7))) << 4), src, v);
  }
}

template <bool I8, int MT, int NT>
__device__ __forceinline__ void load_x(const Params& P, Smem<I8, MT>& sm, int st, int kg, int g) {
  const int tid = threadIdx.x;
  const int64_t ldx = static_cast<int64_t>(P.groups) * P.k;
  const __nv_bfloat16* xb = P.x + static_cast<int64_t>(g) * P.k + static_cast<int64_t>(kg) * BK;
  const uint32_t xs = static_cast<uint32_t>(__cvta_generic_to_shared(sm.x[st]));
  for (int c = tid; c < MT * 8 * 8; c += NT) {
    const int t = c >> 3, ch = c & 7;
    const bool v = t < P.m;
    cp_async16(xs + t * 128 + ((ch ^ (t & 7)) << 4), xb + (v ? t : 0) * ldx + ch * 8, v);
  }
}

__device__ __forceinline__ float load_scale(const Params& P, int n0, int kg, int g) {
  const int r = n0 + static_cast<int>(threadIdx.x);
  if (threadIdx.x >= ROWS || r >= P.n) return 0.f;
  return __bfloat162float(__ldg(P.ws + (static_cast<int64_t>(g) * P.n + r) * (P.k / BK) + kg));
}

template <bool I8, int MT, int RW>
__global__ void __launch_bounds__(threads_for<RW>()) skinny_kernel(const __grid_constant__ Params P0) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Smem<I8, MT>& sm = *reinterpret_cast<Smem<I8, MT>*>(smem_raw);
  constexpr int NST = Cfg<I8>::NST;
  constexpr int NT = threads_for<RW>();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r = lane >> 2, q = lane & 3;
  Params P = P0;
  int n0 = blockIdx.x * ROWS;
  if (P0.nprob > 0) {
    int pi = 0;
    while (pi + 1 < P0.nprob && static_cast<int>(blockIdx.x) >= P0.prob[pi + 1].tile0) ++pi;
    P.w = P0.prob[pi].w;
    P.ws = P0.prob[pi].ws;
    P.y = P0.prob[pi].y;
    P.n = P0.prob[pi].n;
    P.y_dtype = P0.prob[pi].y_dtype;
    n0 = (static_cast<int>(blockIdx.x) - P0.prob[pi].tile0) * ROWS;
  }
  const int g = blockIdx.z / P.ksplit;
  const int split = blockIdx.z % P.ksplit;
  const int KT = P.k / BK;
  const int per = (KT + P.ksplit - 1) / P.ksplit;
  const int kt0 = split * per;
  const int nkt = max(0, min(per, KT - kt0));

  float acc[RW][MT][4], gacc[RW][MT][4];
#pragma unroll
  for (int i = 0; i < RW; ++i)
#pragma unroll
    for (int a = 0; a < MT; ++a)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[i][a][c] = 0.f;

  // the weights and their scales do not depend on the kernel before this one: their first stages
  // load while it finishes (programmatic dependent launch); the tokens load after pdl_wait()
  float sc0[NST - 1];  // the prologue's scales: all loads in flight at once
#pragma unroll
  for (int s = 0; s < NST - 1; ++s) sc0[s] = (I8 && s < nkt) ? load_scale(P, n0, kt0 + s, g) : 0.f;
#pragma unroll
  for (int s = 0; s < NST - 1; ++s)
    if (s < nkt) load_w<I8, MT, NT>(P, sm, s, n0, kt0 + s, g);
  pdl_wait();
#pragma unroll
  for (int s = 0; s < NST - 1; ++s) {
    if (s < nkt) load_x<I8, MT, NT>(P, sm, s, kt0 + s, g);
    asm volatile("cp.async.commit_group;\n" ::);
  }
  // the scales are parked only now, so that their loads overlap the tokens' (the first step's
  // barrier orders these stores before any read)
  if constexpr (I8) {
#pragma unroll
    for (int s = 0; s < NST - 1; ++s)
      if (s < nkt && tid < ROWS) sm.scale[s][tid] = sc0[s];
  }

  const int wrow = warp * 16 * RW + r;  // this lane's weight rows: wrow + 16 i + {0, 8}
  // a stage's scale is loaded with its tiles (NST - 1 steps ahead) but parked in shared memory two
  // steps later, so that no step waits on the load: sc_1, sc_2 are the loads of the last two steps
  float sc_1 = 0.f, sc_2 = 0.f;
  static_assert(!I8 || NST >= 4, "the delayed scale store needs four stages");
  for (int it = 0; it < nkt; ++it) {
    const int st = it % NST;
    asm volatile("cp.async.wait_group %0;\n" ::"n"(NST - 2));
    __syncthreads();
    const int nk = it + NST - 1;
    float sc_next = 0.f;
    if (nk < nkt) {
      load_w<I8, MT, NT>(P, sm, nk % NST, n0, kt0 + nk, g);
      load_x<I8, MT, NT>(P, sm, nk % NST, kt0 + nk, g);
      if constexpr (I8) sc_next = load_scale(P, n0, kt0 + nk, g);
    }
    asm volatile("cp.async.commit_group;\n" ::);

    const uint32_t wsm = static_cast<uint32_t>(__cvta_generic_to_shared(sm.w[st]));
    const uint32_t xsm = static_cast<uint32_t>(__cvta_generic_to_shared(sm.x[st]));
    // the tokens' operands: 16 k of each of this lane's tokens
    uint32_t xw[MT][8];
#pragma unroll
    for (int nt = 0; nt < MT; ++nt) {
      const int t = nt * 8 + r;
      const uint4 a = lds128(xsm + t * 128 + (((2 * q) ^ (t & 7)) << 4));
      const uint4 b = lds128(xsm + t * 128 + (((2 * q + 1) ^ (t & 7)) << 4));
      xw[nt][0] = a.x; xw[nt][1] = a.y; xw[nt][2] = a.z; xw[nt][3] = a.w;
      xw[nt][4] = b.x; xw[nt][5] = b.y; xw[nt][6] = b.z; xw[nt][7] = b.w;
    }
#pragma unroll
    for (int i = 0; i < RW; ++i) {
      // 16 k of rows wrow + 16 i and wrow + 16 i + 8
      const int r0 = wrow + 16 * i, r1 = r0 + 8;
      uint32_t w0[8], w1[8];  // I8: words 0..3 (4 bytes each, biased by 0x80); bf16: 8 words of k pairs
      if constexpr (I8) {
        const uint4 a = lds128(wsm + r0 * 64 + q * 16), b = lds128(wsm + r1 * 64 + q * 16);
        w0[0] = a.x ^ 0x80808080u; w0[1] = a.y ^ 0x80808080u; w0[2] = a.z ^ 0x80808080u; w0[3] = a.w ^ 0x80808080u;
        w1[0] = b.x ^ 0x80808080u; w1[1] = b.y ^ 0x80808080u; w1[2] = b.z ^ 0x80808080u; w1[3] = b.w ^ 0x80808080u;
      } else {
        const uint4 a0 = lds128(wsm + r0 * 128 + (((2 * q) ^ (r0 & 7)) << 4));
        const uint4 a1 = lds128(wsm + r0 * 128 + (((2 * q + 1) ^ (r0 & 7)) << 4));
        const uint4 b0 = lds128(wsm + r1 * 128 + (((2 * q) ^ (r1 & 7)) << 4));
        const uint4 b1 = lds128(wsm + r1 * 128 + (((2 * q + 1) ^ (r1 & 7)) << 4));
        w0[0] = a0.x; w0[1] = a0.y; w0[2] = a0.z; w0[3] = a0.w; w0[4] = a1.x; w0[5] = a1.y; w0[6] = a1.z; w0[7] = a1.w;
        w1[0] = b0.x; w1[1] = b0.y; w1[2] = b0.z; w1[3] = b0.w; w1[4] = b1.x; w1[5] = b1.y; w1[6] = b1.z; w1[7] = b1.w;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t af[4];
        if constexpr (I8) {
          af[0] = s8x2_bf16x2(w0[j], 0);
          af[1] = s8x2_bf16x2(w1[j], 0);
          af[2] = s8x2_bf16x2(w0[j], 1);
          af[3] = s8x2_bf16x2(w1[j], 1);
        } else {
          af[0] = w0[2 * j];
          af[1] = w1[2 * j];
          af[2] = w0[2 * j + 1];
          af[3] = w1[2 * j + 1];
        }
#pragma unroll
        for (int nt = 0; nt < MT; ++nt) {
          if constexpr (I8) {
            if (j == 0)  // the group's first k step starts its partial from zero
              mma_bf16_z(gacc[i][nt], af, xw[nt][0], xw[nt][1]);
            else
              mma_bf16(gacc[i][nt], af, xw[nt][2 * j], xw[nt][2 * j + 1]);
          } else {
            mma_bf16(acc[i][nt], af, xw[nt][2 * j], xw[nt][2 * j + 1]);
          }
        }
      }
      if constexpr (I8) {
        const float s0 = sm.scale[st][r0], s1 = sm.scale[st][r1];
#pragma unroll
        for (int nt = 0; nt < MT; ++nt) {
          acc[i][nt][0] = fmaf(gacc[i][nt][0], s0, acc[i][nt][0]);
          acc[i][nt][1] = fmaf(gacc[i][nt][1], s0, acc[i][nt][1]);
          acc[i][nt][2] = fmaf(gacc[i][nt][2], s1, acc[i][nt][2]);
          acc[i][nt][3] = fmaf(gacc[i][nt][3], s1, acc[i][nt][3]);
        }
      }
    }
    if constexpr (I8) {
      // the scale loaded two steps ago, for stage it + NST - 3 (read at step it + NST - 3 >= it + 1,
      // after the next barrier; its slot was last read at step it - 3)
      if (it >= 2 && it + NST - 3 < nkt && tid < ROWS) sm.scale[(it + NST - 3) % NST][tid] = sc_2;
      sc_2 = sc_1;
      sc_1 = sc_next;
    }
  }
  asm volatile("cp.async.wait_group 0;\n" ::);
  pdl_trigger();

  // D fragment: c0, c1 = (row wrow + 16 i, tokens 2q, 2q+1 of the tile), c2, c3 = row + 8
  const int64_t ldy = static_cast<int64_t>(P.groups) * P.n;
  if (P.ksplit == 1) {
#pragma unroll
    for (int i = 0; i < RW; ++i)
#pragma unroll
      for (int nt = 0; nt < MT; ++nt)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int f = n0 + wrow + 16 * i + hf * 8;
          if (f >= P.n) continue;
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int64_t t = nt * 8 + 2 * q + e;
            if (t >= P.m) continue;
            store_y(P, t * ldy + static_cast<int64_t>(g) * P.n + f, acc[i][nt][hf * 2 + e]);
          }
        }
    return;
  }
  // k split over the CTAs of this cluster: each parks its partial tile in shared memory, then CTA
  // `split` sums rows [split, split + 1) * ROWS / ksplit of all partials in split order (the same
  // order whichever CTA finishes first) and stores them
  constexpr int LD = MT * 8 + 1;
  using SmT = Smem<I8, MT>;
  static_assert(ROWS * LD * 4 <= sizeof(sm.w) + sizeof(sm.x), "partial tile fits the two rings");
  static_assert(offsetof(SmT, x) == sizeof(sm.w), "the token ring follows the weight ring");
  float* red = reinterpret_cast<float*>(sm.w);  // spans the weight and token rings, both idle here
  __syncthreads();  // every warp is done with the ring
#pragma unroll
  for (int i = 0; i < RW; ++i)
#pragma unroll
    for (int nt = 0; nt < MT; ++nt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf)
#pragma unroll
        for (int e = 0; e < 2; ++e)
          red[(wrow + 16 * i + hf * 8) * LD + nt * 8 + 2 * q + e] = acc[i][nt][hf * 2 + e];
  cluster_sync();
  const int rows_per = ROWS / P.ksplit;
  const uint32_t red_s = static_cast<uint32_t>(__cvta_generic_to_shared(red));
  for (int i = tid; i < rows_per * MT * 8; i += NT) {
    const int row = split * rows_per + i / (MT * 8), t = i % (MT * 8);  // a warp reads 128 B of a peer
    const uint32_t off = static_cast<uint32_t>((row * LD + t) * 4);
    float v = 0.f;
    for (int r2 = 0; r2 < P.ksplit; ++r2) v += ld_dsmem_f32(red_s + off, r2);
    const int f = n0 + row;
    if (f < P.n && t < P.m) store_y(P, static_cast<int64_t>(t) * ldy + static_cast<int64_t>(g) * P.n + f, v);
  }
  cluster_sync();  // peers keep their partials until every CTA has read them
}

}  // namespace sk

// y = sum over the k splits of the partials, in split order (deterministic), converted to y's dtype
__global__ void __launch_bounds__(256) splitk_reduce_kernel(Params P) {
  const int64_t total = P.m * static_cast<int64_t>(P.groups) * P.n;
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x) * 2;
  if (i >= total) return;
  float2 a = *reinterpret_cast<const float2*>(P.part + i);
  for (int s = 1; s < P.ksplit; ++s) {
    const float2 b = *reinterpret_cast<const float2*>(P.part + static_cast<int64_t>(s) * total + i);
    a.x += b.x;
    a.y += b.y;
  }
  if (P.y_dtype == DSV4_BF16)
    *reinterpret_cast<uint32_t*>(reinterpret_cast<__nv_bfloat16*>(P.y) + i) = pack_bf16x2(a.x, a.y);
  else
    *reinterpret_cast<float2*>(reinterpret_cast<float*>(P.y) + i) = a;
}

// k splits for a call whose output tiles alone leave the GPU idle (decode batches: small m, with
// n in the hundreds or thousands and k in the thousands): about two CTAs per SM, two k tiles each
// at least
// at least, and partials of at most half the weight bytes (w_bytes: 1 for int8, 2 for bf16)
inline int choose_ksplit(int64_t m, int n, int k, int groups, int w_bytes) {
  const int64_t tiles = ((n + BN - 1) / BN) * ((m + BM - 1) / BM) * static_cast<int64_t>(groups);
  const int KT = k / BK;
  const int64_t want = 2 * static_cast<int64_t>(num_sms());
  if (tiles >= want || KT < 4) return 1;
  int64_t sp = (want + tiles - 1) / tiles;
  sp = std::min<int64_t>(sp, KT / 2);
  sp = std::min<int64_t>(sp, (static_cast<int64_t>(k) * w_bytes) / (8 * std::max<int64_t>(m, 1)));
  sp = std::min<int64_t>(sp, 64);
  if (sp <= 1) return 1;
  const int per = (KT + static_cast<int>(sp) - 1) / static_cast<int>(sp);
  return (KT + per - 1) / per;  // no split without k tiles
}

// token tiles of the decode-shaped kernel: m <= 8 * MT, MT in {1, 2, 4, 8}
constexpr int SKINNY_MAX_M = 64;

struct Plan {
  bool skinny;
  int mt;      // 8-token tiles (skinny kernel)
  int ksplit;  // CTAs along k
};

// the decode-shaped kernel splits k over a thread-block cluster (partials summed through distributed
// shared memory) only when its 128-row tiles leave SMs idle: about two CTAs per SM, a power of two
// up to 8 CTAs, two k groups per CTA at least
constexpr int MAX_CLUSTER = 8;
inline int skinny_ksplit_tiles(int64_t tiles, int k) {
  const int KT = k / BK;
  const int64_t sms = num_sms();
  if (tiles >= sms || KT < 4) return 1;
  const int64_t want = std::min<int64_t>((2 * sms + tiles - 1) / tiles, KT / 2);
  int sp = 1;
  while (sp * 2 <= want && sp * 2 <= MAX_CLUSTER) sp *= 2;
  return sp;
}
inline int skinny_ksplit(int n, int k, int groups) {
  return skinny_ksplit_tiles(((n + sk::ROWS - 1) / sk::ROWS) * static_cast<int64_t>(groups), k);
}

inline Plan plan(int64_t m, int n, int k, int groups, bool i8) {
  Plan pl;
  const int wb = i8 ? 1 : 2;
  pl.skinny = m <= SKINNY_MAX_M;
  pl.mt = m <= 8 ? 1 : m <= 16 ? 2 : m <= 32 ? 4 : 8;
  pl.ksplit = pl.skinny ? skinny_ksplit(n, k, groups) : choose_ksplit(m, n, k, groups, wb);
  return pl;
}

}  // namespace gm
}  // namespace dsv4

using namespace dsv4;

namespace dsv4 {
int gemm_tc_launch(const void* x, int64_t m, int k, int groups, const void* const* w, void* const* y, const int* n,
                   const int* y_dtype, int nprob, void* stream);
}  // namespace dsv4

// The tcgen05 kernel for kernel == 2, and for kernel == 0 with bf16 weights and m above the
// weight-streaming range. The choice depends on m only through that bound, so the rows of a
// prefill computed in slices (one per rank) are bit-identical to the same rows computed whole.
static bool use_tcgen05(int kernel, bool i8, int64_t m) {
  if (kernel == 2) return true;
  return kernel == 0 && !i8 && m > gm::SKINNY_MAX_M;
}

template <bool I8, int MT>
static int launch_skinny_mt(const gm::Params& P, void* stream) {
  // int8 weights: 32 rows per warp (the tokens' fragments serve two row tiles); bf16: 16
  constexpr int RW = I8 ? 2 : 1;
  const auto kern = gm::sk::skinny_kernel<I8, MT, RW>;
  static PerDeviceOnce set;
  const int smem = sizeof(gm::sk::Smem<I8, MT>);
  DSV4_CUDA_CHECK(set_smem_once(set, kern, smem));
  cudaLaunchConfig_t cfg = {};
  const int tiles = P.nprob > 0 ? P.prob[P.nprob - 1].tile0 + (P.prob[P.nprob - 1].n + gm::sk::ROWS - 1) / gm::sk::ROWS
                                : (P.n + gm::sk::ROWS - 1) / gm::sk::ROWS;
  cfg.gridDim = dim3(tiles, 1, P.groups * P.ksplit);
  cfg.blockDim = dim3(gm::sk::threads_for<RW>());
  cfg.dynamicSmemBytes = smem;
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;  // the CTAs of one output tile's k split
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = P.ksplit;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  DSV4_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, P));
  DSV4_LAUNCH_CHECK("skinny_kernel");
  return DSV4_OK;
}

template <bool I8>
static int launch_skinny(const gm::Params& P, int mt, void* stream) {
  switch (mt) {
    case 1: return launch_skinny_mt<I8, 1>(P, stream);
    case 2: return launch_skinny_mt<I8, 2>(P, stream);
    case 4: return launch_skinny_mt<I8, 4>(P, stream);
    default: return launch_skinny_mt<I8, 8>(P, stream);
  }
}

template <bool I8>
static int launch_tiled(const gm::Params& P, void* stream) {
  const int64_t mt = (P.m + gm::BM - 1) / gm::BM;
  DSV4_CHECK_ARG(mt <= 65535, "dsv4_linear: m too large");
  static PerDeviceOnce set;
  const int smem = sizeof(gm::Smem<I8>);
  DSV4_CUDA_CHECK(set_smem_once(set, gm::gemm_kernel<I8>, smem));
  dim3 grid((P.n + gm::BN - 1) / gm::BN, static_cast<unsigned>(mt), P.groups * P.ksplit);
  gm::gemm_kernel<I8><<<grid, gm::THREADS, smem, as_stream(stream)>>>(P);
  DSV4_LAUNCH_CHECK("gemm_kernel");
  return DSV4_OK;
}

extern "C" size_t dsv4_linear_workspace_size(const dsv4_linear_params* p) {
  if (!p || p->m <= 0 || p->n <= 0 || p->k <= 0 || p->groups < 1) return 0;
  if (use_tcgen05(p->kernel, p->w_dtype == DSV4_I8, p->m)) return 0;
  const gm::Plan pl = gm::plan(p->m, p->n, p->k, p->groups, p->w_dtype == DSV4_I8);
  const int sp = pl.ksplit;
  if (pl.skinny || sp <= 1) return 0;  // the decode-shaped kernel reduces inside its cluster
  return static_cast<size_t>(sp) * static_cast<size_t>(p->m) * static_cast<size_t>(p->groups) *
         static_cast<size_t>(p->n) * sizeof(float);
}

extern "C" int dsv4_linear(const dsv4_linear_params* p, void* stream) {
  DSV4_CHECK_ARG(p && p->x && p->w && p->y, "dsv4_linear: NULL tensor");
  DSV4_CHECK_ARG(p->m >= 0 && p->n > 0 && p->k > 0 && p->groups >= 1, "dsv4_linear: bad sizes");
  DSV4_CHECK_ARG(p->k % gm::BK == 0, "dsv4_linear: k=%d must be a multiple of 64", p->k);
  DSV4_CHECK_ARG(p->n % 2 == 0, "dsv4_linear: n=%d must be even", p->n);
  DSV4_CHECK_DTYPE(p->x_dtype == DSV4_BF16, "dsv4_linear: x must be BF16");
  DSV4_CHECK_DTYPE(p->w_dtype == DSV4_BF16 || p->w_dtype == DSV4_I8, "dsv4_linear: W must be BF16 or I8");
  DSV4_CHECK_DTYPE(p->y_dtype == DSV4_F32 || p->y_dtype == DSV4_BF16, "dsv4_linear: y must be F32 or BF16");
  const bool i8 = p->w_dtype == DSV4_I8;
  DSV4_CHECK_ARG(!i8 || (p->w_scale != nullptr && p->group == 64),
                 "dsv4_linear: int8 weights need bf16 scales with group 64");
  DSV4_CHECK_ARG(p->kernel >= 0 && p->kernel <= 2, "dsv4_linear: kernel=%d must be 0, 1 or 2", p->kernel);
  DSV4_CHECK_ARG(p->kernel != 2 || !i8, "dsv4_linear: the tcgen05 kernel (2) takes bf16 weights");
  if (p->m == 0) return DSV4_OK;
  DSV4_CHECK_ARG(reinterpret_cast<uintptr_t>(p->x) % 16 == 0 && reinterpret_cast<uintptr_t>(p->w) % 16 == 0,
                 "dsv4_linear: x and W must be 16-byte aligned");
  if (use_tcgen05(p->kernel, i8, p->m)) {
    const void* w = p->w;
    void* y = p->y;
    return gemm_tc_launch(p->x, p->m, p->k, p->groups, &w, &y, &p->n, &p->y_dtype, 1, stream);
  }
  gm::Params P;
  P.x = reinterpret_cast<const __nv_bfloat16*>(p->x);
  P.w = p->w;
  P.ws = reinterpret_cast<const __nv_bfloat16*>(p->w_scale);
  P.y = p->y;
  P.m = p->m;
  P.n = p->n;
  P.k = p->k;
  P.groups = p->groups;
  P.y_dtype = p->y_dtype;
  P.nprob = 0;
  const gm::Plan pl = gm::plan(p->m, p->n, p->k, p->groups, i8);
  P.ksplit = pl.skinny ? pl.ksplit : 1;
  P.part = nullptr;
  if (!pl.skinny && (p->workspace_bytes > 0 || p->workspace)) {
    const size_t need = dsv4_linear_workspace_size(p);
    if (p->workspace_bytes < need || (need > 0 && p->workspace == nullptr)) {
      set_error("dsv4_linear: workspace of %zu bytes needed, %zu given", need, p->workspace_bytes);
      return DSV4_ERR_WORKSPACE;
    }
    if (need > 0) {
      DSV4_CHECK_ARG(reinterpret_cast<uintptr_t>(p->workspace) % 16 == 0, "dsv4_linear: workspace not 16-byte aligned");
      P.ksplit = pl.ksplit;
      P.part = reinterpret_cast<float*>(p->workspace);
    }
  }
  DSV4_CHECK_ARG(static_cast<int64_t>(p->groups) * P.ksplit <= 65535, "dsv4_linear: too many groups");
  int rc;
  if (pl.skinny)
    rc = i8 ? launch_skinny<true>(P, pl.mt, stream) : launch_skinny<false>(P, pl.mt, stream);
  else
    rc = i8 ? launch_tiled<true>(P, stream) : launch_tiled<false>(P, stream);
  if (rc != DSV4_OK) return rc;
  if (!pl.skinny && P.ksplit > 1) {
    const int64_t pairs = (P.m * static_cast<int64_t>(P.groups) * P.n) / 2;
    const int64_t blocks = (pairs + 255) / 256;
    gm::splitk_reduce_kernel<<<static_cast<unsigned>(blocks), 256, 0, as_stream(stream)>>>(P);
    DSV4_LAUNCH_CHECK("splitk_reduce_kernel");
  }
  return DSV4_OK;
}

extern "C" int dsv4_linear_multi(const dsv4_linear_multi_params* p, void* stream) {
  DSV4_CHECK_ARG(p && p->x && p->count >= 1 && p->count <= DSV4_LINEAR_MULTI_MAX, "dsv4_linear_multi: bad arguments");
  DSV4_CHECK_ARG(p->m >= 0 && p->k > 0 && p->k % gm::BK == 0, "dsv4_linear_multi: k=%d must be a multiple of 64", p->k);
  DSV4_CHECK_DTYPE(p->x_dtype == DSV4_BF16, "dsv4_linear_multi: x must be BF16");
  DSV4_CHECK_DTYPE(p->w_dtype == DSV4_BF16 || p->w_dtype == DSV4_I8, "dsv4_linear_multi: W must be BF16 or I8");
  const bool i8 = p->w_dtype == DSV4_I8;
  for (int i = 0; i < p->count; ++i) {
    const dsv4_linear_out& o = p->outs[i];
    DSV4_CHECK_ARG(o.w && o.y && o.n > 0 && o.n % 2 == 0, "dsv4_linear_multi: output %d: bad W / y / n", i);
    DSV4_CHECK_DTYPE(o.y_dtype == DSV4_F32 || o.y_dtype == DSV4_BF16, "dsv4_linear_multi: y must be F32 or BF16");
    DSV4_CHECK_ARG(!i8 || (o.w_scale != nullptr && p->group == 64),
                   "dsv4_linear_multi: int8 weights need bf16 scales with group 64");
    DSV4_CHECK_ARG(reinterpret_cast<uintptr_t>(o.w) % 16 == 0, "dsv4_linear_multi: W must be 16-byte aligned");
  }
  DSV4_CHECK_ARG(p->kernel >= 0 && p->kernel <= 2, "dsv4_linear_multi: kernel=%d must be 0, 1 or 2", p->kernel);
  DSV4_CHECK_ARG(p->kernel != 2 || !i8, "dsv4_linear_multi: the tcgen05 kernel (2) takes bf16 weights");
  if (p->m == 0) return DSV4_OK;
  DSV4_CHECK_ARG(reinterpret_cast<uintptr_t>(p->x) % 16 == 0, "dsv4_linear_multi: x must be 16-byte aligned");
  {
    int n[DSV4_LINEAR_MULTI_MAX], yd[DSV4_LINEAR_MULTI_MAX];
    const void* w[DSV4_LINEAR_MULTI_MAX];
    void* y[DSV4_LINEAR_MULTI_MAX];
    for (int i = 0; i < p->count; ++i) {
      n[i] = p->outs[i].n;
      yd[i] = p->outs[i].y_dtype;
      w[i] = p->outs[i].w;
      y[i] = p->outs[i].y;
    }
    if (use_tcgen05(p->kernel, i8, p->m))  // all projections in one launch
      return gemm_tc_launch(p->x, p->m, p->k, 1, w, y, n, yd, p->count, stream);
  }
  if (p->m > gm::SKINNY_MAX_M) {  // prefill-sized: one tiled launch per projection
    for (int i = 0; i < p->count; ++i) {
      dsv4_linear_params lp = {};
      lp.x = p->x;
      lp.w = p->outs[i].w;
      lp.w_scale = p->outs[i].w_scale;
      lp.y = p->outs[i].y;
      lp.m = p->m;
      lp.n = p->outs[i].n;
      lp.k = p->k;
      lp.groups = 1;
      lp.group = p->group;
      lp.x_dtype = p->x_dtype;
      lp.w_dtype = p->w_dtype;
      lp.y_dtype = p->outs[i].y_dtype;
      lp.kernel = 1;
      const int rc = dsv4_linear(&lp, stream);
      if (rc != DSV4_OK) return rc;
    }
    return DSV4_OK;
  }
  gm::Params P = {};
  P.x = reinterpret_cast<const __nv_bfloat16*>(p->x);
  P.m = p->m;
  P.k = p->k;
  P.groups = 1;
  P.nprob = p->count;
  int tiles = 0;
  for (int i = 0; i < p->count; ++i) {
    P.prob[i].w = p->outs[i].w;
    P.prob[i].ws = reinterpret_cast<const __nv_bfloat16*>(p->outs[i].w_scale);
    P.prob[i].y = p->outs[i].y;
    P.prob[i].n = p->outs[i].n;
    P.prob[i].y_dtype = p->outs[i].y_dtype;
    P.prob[i].tile0 = tiles;
    tiles += (p->outs[i].n + gm::sk::ROWS - 1) / gm::sk::ROWS;
  }
  // the first projection's fields stand in until the kernel resolves its own
  P.w = P.prob[0].w;
  P.ws = P.prob[0].ws;
  P.y = P.prob[0].y;
  P.n = P.prob[0].n;
  P.y_dtype = P.prob[0].y_dtype;
  P.ksplit = gm::skinny_ksplit_tiles(tiles, p->k);
  P.part = nullptr;
  const int mt = p->m <= 8 ? 1 : p->m <= 16 ? 2 : p->m <= 32 ? 4 : 8;
  return i8 ? launch_skinny<true>(P, mt, stream) : launch_skinny<false>(P, mt, stream);
}
