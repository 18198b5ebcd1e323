// Projection GEMM y = x W^T for the MLA projections (v4mlx/mla.py:16-56) and the compressor's
// two projections (ref_torch/compressor.py:62-63).
//
// x [m, k] bf16 (K-major), W [n, k] (K-major) as bf16, or int8 with one bf16 scale per
// (row, 64-wide group of k) — the 8-bit grouped weights of the fast decode block
// (oracle/v4_fast.py:31-34, symmetric here). The int8 tile is widened to bf16 in shared memory
// (exact: |q| <= 127), each 64-wide k group is accumulated separately in fp32 and folded into the
// output with its scale, so the dequantised product is computed without rounding the weights.
// CTA tile 128 x 128 x 64, 8 warps (2 x 4), warp tile 64 x 32, bf16 mma.sync, 3-stage cp.async.
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
  const int g = blockIdx.z;
  const int KT = P.k / BK;

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
    if (s < KT) load_stage<I8>(P, sm, s, m0, n0, s, g);
    asm volatile("cp.async.commit_group;\n" ::);
  }

  for (int kt = 0; kt < KT; ++kt) {
    const int st = kt % STAGES;
    asm volatile("cp.async.wait_group %0;\n" ::"n"(STAGES - 2));
    __syncthreads();
    {
      int nk = kt + STAGES - 1;
      if (nk < KT) load_stage<I8>(P, sm, nk % STAGES, m0, n0, nk, g);
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
        if (P.y_dtype == DSV4_BF16) {
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

}  // namespace gm
}  // namespace dsv4

using namespace dsv4;

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
  if (p->m == 0) return DSV4_OK;
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
  const int64_t mt = (p->m + gm::BM - 1) / gm::BM;
  DSV4_CHECK_ARG(mt <= 65535 && p->groups <= 65535, "dsv4_linear: m too large");
  dim3 grid((p->n + gm::BN - 1) / gm::BN, static_cast<unsigned>(mt), p->groups);
  if (i8) {
    static bool set = false;
    const int smem = sizeof(gm::Smem<true>);
    if (!set) {
      DSV4_CUDA_CHECK(cudaFuncSetAttribute(gm::gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      set = true;
    }
    gm::gemm_kernel<true><<<grid, gm::THREADS, smem, as_stream(stream)>>>(P);
  } else {
    static bool set = false;
    const int smem = sizeof(gm::Smem<false>);
    if (!set) {
      DSV4_CUDA_CHECK(cudaFuncSetAttribute(gm::gemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      set = true;
    }
    gm::gemm_kernel<false><<<grid, gm::THREADS, smem, as_stream(stream)>>>(P);
  }
  DSV4_LAUNCH_CHECK("gemm_kernel");
  return DSV4_OK;
}
