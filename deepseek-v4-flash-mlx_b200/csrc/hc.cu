// Hyper-connections around the attention block (ref_torch/hc.py:18-80; official Block.hc_pre /
// hc_post and ParallelHead.hc_head): the residual stream holds hc = 4 copies of the hidden state.
//
// hc_pre, chained by programmatic dependent launch:
//   hc_mix_kernel: the 24 (hc_head: 4) dot products of each token's hc*dim values with the rows of
//     fn, plus the sum of squares, as a split-K CUDA-core product: a CTA takes 128 tokens (32 for
//     batches of at most 256) and one column range, staging both the weights and the tokens
//     through shared memory (cp.async, double buffered); each lane holds 8 (2) tokens x 4 columns
//     per stage and their accumulators, so one weight float4 feeds 32 (8) FMAs; the 8 column-group
//     lanes of a token meet once, through shared memory, at the end. Partials go to the workspace,
//     [split][row][nmix + 1].
//   large batches: hc_sinkhorn_kernel (one warp per token: the partials summed in split order,
//     r = rsqrt(mean(x^2) + norm_eps), mixes * r, pre = sigmoid(m*s0 + b) + eps, post =
//     2 sigmoid(m*s1 + b), comb = 4x4 Sinkhorn: row softmax + eps, column normalise, then iters-1
//     rounds of row and column normalisation, each by the sum + eps, on 16 lanes), then hc_y_kernel
//     (one CTA per token: y[d] = sum_k pre[k] x[k, d] and optionally the block's RMSNorm of y, the
//     projections' bf16 input, streaming x once more);
//   small batches: hc_fused_kernel, the split and y of one token in one CTA.
//   hc_head is the same with hc mixes and pre only.
// hc_post: y[j, d] = post[j] x[d] + sum_i comb[i, j] residual[i, d], elementwise.
#include <algorithm>

#include "common.cuh"

namespace dsv4 {
namespace hcn {

constexpr int HC = 4;
constexpr int NMIX = (2 + HC) * HC;  // 24
constexpr int MIX_THREADS = 128, MIX_BK = 32;  // columns per stage: one 32-column step
constexpr int MIX_MIN_STAGES = 4;              // columns per split >= 4 stages
constexpr int SK_THREADS = 256;                // Sinkhorn: one warp per token
constexpr int Y_THREADS = 256, MAXJ = 4;       // dim <= MAXJ * 1024
constexpr int MAXDIM = MAXJ * 1024;

__device__ __forceinline__ float sigmoidf(float v) { return 1.f / (1.f + expf(-v)); }

__device__ __forceinline__ void cp_async16(float* dst, const float* src, bool valid) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src), "r"(valid ? 16 : 0));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

__device__ __forceinline__ float dot4(const float4& a, const float4& b, float acc) {
  acc = fmaf(a.x, b.x, acc);
  acc = fmaf(a.y, b.y, acc);
  acc = fmaf(a.z, b.z, acc);
  return fmaf(a.w, b.w, acc);
}

// tokens per CTA: 4 warps x 4 token groups x TPL tokens per lane
template <int TPL>
constexpr int mix_tok() { return 16 * TPL; }

template <int NM, int TPL>
struct MixSmem {
  float w[2][NM][MIX_BK];                  // weight stages
  float x[2][mix_tok<TPL>()][MIX_BK];      // token stages
};

// Partial mixes over columns [split * kc, min(L, (split + 1) * kc)) for the CTA's 16 * TPL tokens.
// Lane (tg = lane / 8, cg = lane % 8) of warp w holds tokens 4 TPL w + TPL tg + {0..TPL-1} and
// columns 4cg..4cg+3 of each 32-column stage, so one weight float4 read from shared memory feeds
// 4 TPL FMAs (shared memory delivers one float per lane per cycle and the FMA pipes take four
// warp instructions per cycle: TPL = 8 keeps the pipes fed; TPL = 2 serves small batches).
template <int NM, int TPL>
__global__ void __launch_bounds__(MIX_THREADS) hc_mix_kernel(const float* __restrict__ x, const float* __restrict__ fn,
                                                             float* __restrict__ part, int64_t rows, int L, int kc) {
  constexpr int TOK = mix_tok<TPL>();
  __shared__ __align__(16) MixSmem<NM, TPL> sm;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int tg = lane >> 3, cg = lane & 7;
  const int split = blockIdx.y;
  const int64_t tok0 = static_cast<int64_t>(blockIdx.x) * TOK;
  const int c0 = split * kc, c1 = min(L, c0 + kc);
  const int nq = (c1 - c0 + MIX_BK - 1) / MIX_BK;
  auto stage_w = [&](int q, int buf) {
    for (int i = tid; i < NM * (MIX_BK / 4); i += MIX_THREADS) {
      const int m = i / (MIX_BK / 4), f = i % (MIX_BK / 4);
      const int col = c0 + q * MIX_BK + 4 * f;
      const bool ok = col < c1;
      cp_async16(&sm.w[buf][m][4 * f], ok ? fn + static_cast<int64_t>(m) * L + col : fn, ok);
    }
  };
  auto stage_x = [&](int q, int buf) {
    for (int i = tid; i < TOK * (MIX_BK / 4); i += MIX_THREADS) {
      const int j = i / (MIX_BK / 4), f = i % (MIX_BK / 4);
      const int col = c0 + q * MIX_BK + 4 * f;
      const bool ok = col < c1 && tok0 + j < rows;
      cp_async16(&sm.x[buf][j][4 * f], ok ? x + (tok0 + j) * L + col : x, ok);
    }
  };
  // the weights do not depend on the previous kernel: the first stage is fetched before the wait
  stage_w(0, 0);
  pdl_wait();  // programmatic dependent launch: the previous kernel is complete from here
  pdl_trigger();
  stage_x(0, 0);
  cp_async_commit();
  float acc[NM][TPL], ss[TPL];
#pragma unroll
  for (int t = 0; t < TPL; ++t) {
    ss[t] = 0.f;
#pragma unroll
    for (int m = 0; m < NM; ++m) acc[m][t] = 0.f;
  }
  const int jrow = warp * 4 * TPL + tg * TPL;
  for (int q = 0; q < nq; ++q) {
    const int buf = q & 1;
    if (q + 1 < nq) {
      stage_w(q + 1, buf ^ 1);
      stage_x(q + 1, buf ^ 1);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const int c = 4 * cg;
    float4 xv[TPL];
#pragma unroll
    for (int t = 0; t < TPL; ++t) {
      xv[t] = *reinterpret_cast<const float4*>(&sm.x[buf][jrow + t][c]);
      ss[t] = dot4(xv[t], xv[t], ss[t]);
    }
#pragma unroll
    for (int m = 0; m < NM; ++m) {
      const float4 w = *reinterpret_cast<const float4*>(&sm.w[buf][m][c]);
#pragma unroll
      for (int t = 0; t < TPL; ++t) acc[m][t] = dot4(xv[t], w, acc[m][t]);
    }
    __syncthreads();  // the buffer is refilled by the next iteration's stage
  }
  cp_async_wait<0>();
  // output (token j of the CTA, value v): the 8 column-group lanes summed in order, one token slot
  // t (j % TPL) at a time, through the (now idle) stages
  float (*red)[NM + 1] = reinterpret_cast<float (*)[NM + 1]>(&sm);
  static_assert(sizeof(float) * MIX_THREADS * (NM + 1) <= sizeof(MixSmem<NM, TPL>), "partials fit the stages");
#pragma unroll
  for (int t = 0; t < TPL; ++t) {
    __syncthreads();
#pragma unroll
    for (int m = 0; m < NM; ++m) red[tid][m] = acc[m][t];
    red[tid][NM] = ss[t];
    __syncthreads();
    for (int o = tid; o < (TOK / TPL) * (NM + 1); o += MIX_THREADS) {
      const int j = TPL * (o / (NM + 1)) + t, v = o % (NM + 1);
      const int64_t row = tok0 + j;
      if (row >= rows) continue;
      const int src = (j / (4 * TPL)) * 32 + ((j % (4 * TPL)) / TPL) * 8;
      float u = 0.f;
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) u += red[src + cc][v];
      part[(static_cast<int64_t>(split) * rows + row) * (NM + 1) + v] = u;
    }
  }
}

// The split of one token, by one warp: lane v (v <= nm) holds the token's total of value v (the
// nm mixes, then the sum of squares). r = rsqrt(mean(x^2) + norm_eps); lanes 0..3 return pre
// (pre = sigmoid(m*s0 + b) + eps); post = 2 sigmoid(m*s1 + b) and comb (16 lanes: row softmax +
// eps, column normalise, then iters-1 rounds of row and column normalisation, each by the sum +
// eps) are written to the outputs.
__device__ __forceinline__ float split_token(const dsv4_hc_params& p, int64_t row, float u) {
  const int lane = threadIdx.x & 31;
  const int L = HC * p.dim;
  const int nm = p.head ? HC : NMIX;
  const float r = rsqrtf(__shfl_sync(0xffffffffu, u, nm) / static_cast<float>(L) + p.norm_eps);
  const float mpre = __shfl_sync(0xffffffffu, u, lane & 3) * r;  // lanes 0..3: the pre mixes
  const float pre = sigmoidf(mpre * p.scale[0] + p.base[lane & 3]) + p.hc_eps;
  if (p.head) return pre;
  const float mpost = __shfl_sync(0xffffffffu, u, HC + (lane & 3)) * r;
  const float mcomb = __shfl_sync(0xffffffffu, u, 2 * HC + (lane & 15)) * r;
  // lanes 0..15: comb[i][j] with i = lane / 4, j = lane % 4
  float c = lane < 16 ? mcomb * p.scale[2] + p.base[2 * HC + lane] : -INFINITY;
  float mx = fmaxf(c, __shfl_xor_sync(0xffffffffu, c, 1));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
  const float e = lane < 16 ? expf(c - mx) : 0.f;
  float se = e + __shfl_xor_sync(0xffffffffu, e, 1);
  se += __shfl_xor_sync(0xffffffffu, se, 2);
  c = lane < 16 ? e / se + p.hc_eps : 0.f;
  float cs = c + __shfl_xor_sync(0xffffffffu, c, 4);
  cs += __shfl_xor_sync(0xffffffffu, cs, 8);
  c = lane < 16 ? c / (cs + p.hc_eps) : 0.f;
  for (int it = 1; it < p.sinkhorn_iters; ++it) {
    float rs = c + __shfl_xor_sync(0xffffffffu, c, 1);
    rs += __shfl_xor_sync(0xffffffffu, rs, 2);
    c = lane < 16 ? c / (rs + p.hc_eps) : 0.f;
    cs = c + __shfl_xor_sync(0xffffffffu, c, 4);
    cs += __shfl_xor_sync(0xffffffffu, cs, 8);
    c = lane < 16 ? c / (cs + p.hc_eps) : 0.f;
  }
  if (lane < 16) p.comb[row * HC * HC + lane] = c;
  if (lane < HC) p.post[row * HC + lane] = 2.f * sigmoidf(mpost * p.scale[1] + p.base[HC + lane]);
  return pre;
}

// Large batches: one warp per token, lane v summing value v over the splits in order; pre goes to
// the workspace for hc_y_kernel.
__global__ void __launch_bounds__(SK_THREADS) hc_sinkhorn_kernel(dsv4_hc_params p, const float* __restrict__ part,
                                                                 int splits, float* __restrict__ pre_out) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (SK_THREADS / 32) + (threadIdx.x >> 5);
  if (row >= p.rows) return;  // warp-uniform; no block barrier in this kernel
  const int nm = p.head ? HC : NMIX;
  float u = 0.f;
  if (lane <= nm) {
    const float* src = part + row * (nm + 1) + lane;
    const int64_t stride = p.rows * (nm + 1);
    int s = 0;
    for (; s + 8 <= splits; s += 8) {
      float t[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) t[i] = src[(s + i) * stride];
#pragma unroll
      for (int i = 0; i < 8; ++i) u += t[i];
    }
    for (; s < splits; ++s) u += src[s * stride];
  }
  const float pre = split_token(p, row, u);
  if (lane < HC) pre_out[row * HC + lane] = pre;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  // sum over the CTA, returned to every thread (two barriers)
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < Y_THREADS / 32; ++w) t += red[w];
  return t;
}

// y[d] = sum_k pre[k] x[k, d] for this thread's columns, the row's y written and the block's
// RMSNorm of y (fp32 math, one rounding to y_norm's dtype); every thread of the CTA calls it
template <int NJ>
__device__ __forceinline__ void y_and_norm(const dsv4_hc_params& p, int64_t row, const float4 (&v)[HC][NJ],
                                           const float4 pr, float* red) {
  const int tid = threadIdx.x;
  const int dim = p.dim;
  float4 y[NJ];
  float ys = 0.f;
#pragma unroll
  for (int jj = 0; jj < NJ; ++jj) {
    y[jj].x = pr.x * v[0][jj].x + pr.y * v[1][jj].x + pr.z * v[2][jj].x + pr.w * v[3][jj].x;
    y[jj].y = pr.x * v[0][jj].y + pr.y * v[1][jj].y + pr.z * v[2][jj].y + pr.w * v[3][jj].y;
    y[jj].z = pr.x * v[0][jj].z + pr.y * v[1][jj].z + pr.z * v[2][jj].z + pr.w * v[3][jj].z;
    y[jj].w = pr.x * v[0][jj].w + pr.y * v[1][jj].w + pr.z * v[2][jj].w + pr.w * v[3][jj].w;
    const int d = 4 * tid + 1024 * jj;
    if (d < dim) {
      if (p.y) *reinterpret_cast<float4*>(p.y + row * dim + d) = y[jj];
      ys = dot4(y[jj], y[jj], ys);
    }
  }
  if (p.y_norm == nullptr) return;  // uniform over the grid
  const float rn = rsqrtf(block_sum(ys, red) / static_cast<float>(dim) + p.y_norm_eps);
#pragma unroll
  for (int jj = 0; jj < NJ; ++jj) {
    const int d = 4 * tid + 1024 * jj;
    if (d >= dim) continue;
    float o[4] = {y[jj].x * rn, y[jj].y * rn, y[jj].z * rn, y[jj].w * rn};
    if (p.norm_w) {
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] = load_as_float(p.norm_w, d + e, p.norm_dtype) * o[e];
    }
    if (p.y_norm_dtype == DSV4_BF16) {
      uint2 pk;
      pk.x = pack_bf16x2(o[0], o[1]);
      pk.y = pack_bf16x2(o[2], o[3]);
      *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.y_norm) + row * dim + d) = pk;
    } else {
      *reinterpret_cast<float4*>(static_cast<float*>(p.y_norm) + row * dim + d) = make_float4(o[0], o[1], o[2], o[3]);
    }
  }
}

template <int NJ>
__device__ __forceinline__ void load_row(const dsv4_hc_params& p, int64_t row, float4 (&v)[HC][NJ], bool stream) {
  const float* x = p.x + row * HC * p.dim;
#pragma unroll
  for (int k = 0; k < HC; ++k)
#pragma unroll
    for (int jj = 0; jj < NJ; ++jj) {
      const int d = 4 * threadIdx.x + 1024 * jj;
      const float4* src = reinterpret_cast<const float4*>(x + k * p.dim + d);
      v[k][jj] = d >= p.dim ? make_float4(0.f, 0.f, 0.f, 0.f) : (stream ? __ldcs(src) : *src);
    }
}

// Large batches, after hc_sinkhorn_kernel: one CTA per token streams x once more.
template <int NJ>
__global__ void __launch_bounds__(Y_THREADS) hc_y_kernel(dsv4_hc_params p, const float* __restrict__ pre_in) {
  __shared__ float red[Y_THREADS / 32];
  pdl_wait();
  pdl_trigger();
  const int64_t row = blockIdx.x;
  float4 v[HC][NJ];
  load_row<NJ>(p, row, v, true);
  y_and_norm<NJ>(p, row, v, *reinterpret_cast<const float4*>(pre_in + row * HC), red);
}

// Small batches: one CTA per token does all of it. x is loaded first; the 8 warps sum the split
// partials (warp g: splits g, g + 8, ...), warp 0 adds the group sums in order and runs the split.
template <int NJ>
__global__ void __launch_bounds__(Y_THREADS) hc_fused_kernel(dsv4_hc_params p, const float* __restrict__ part,
                                                             int splits) {
  __shared__ float red[Y_THREADS / 32];
  __shared__ float msum[Y_THREADS / 32][32];
  __shared__ __align__(16) float pre_s[HC];
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31, g = threadIdx.x >> 5;
  const int64_t row = blockIdx.x;
  const int nm = p.head ? HC : NMIX;
  float4 v[HC][NJ];
  load_row<NJ>(p, row, v, false);
  {
    float u = 0.f;
    if (lane <= nm) {
      const float* src = part + row * (nm + 1) + lane;
      const int64_t stride = p.rows * (nm + 1);
#pragma unroll 4
      for (int s = g; s < splits; s += Y_THREADS / 32) u += src[s * stride];
    }
    msum[g][lane] = u;
  }
  __syncthreads();
  if (g == 0) {
    float u = 0.f;
#pragma unroll
    for (int q = 0; q < Y_THREADS / 32; ++q) u += msum[q][lane];
    const float pre = split_token(p, row, u);
    if (lane < HC) pre_s[lane] = pre;
  }
  __syncthreads();
  y_and_norm<NJ>(p, row, v, *reinterpret_cast<const float4*>(pre_s), red);
}

struct MixPlan {
  int tpl, splits, kc;
  bool fused;  // one kernel for the split and y (small batches)
};
// Small batches (<= 256 tokens): 2 tokens per lane, column splits for about four CTAs per SM, and
// the split and y in one kernel per token. Large batches: 8 tokens per lane, about two CTAs per
// SM (their residency), and a Sinkhorn warp per token before the y kernel. Every split covers at
// least MIX_MIN_STAGES stages.
inline MixPlan mix_plan(int64_t rows, int L) {
  const bool small = rows <= 256;
  const int tpl = small ? 2 : 8;
  const int64_t target = (small ? 4ll : 2ll) * num_sms();
  const int64_t groups = (rows + 16 * tpl - 1) / (16 * tpl);
  const int stages = (L + MIX_BK - 1) / MIX_BK;
  int splits = 1;
  while (splits * 2 * MIX_MIN_STAGES <= stages && groups * splits * 2 <= target) splits *= 2;
  const int per = (stages + splits - 1) / splits;
  splits = (stages + per - 1) / per;
  return {tpl, splits, per * MIX_BK, small};
}

// the partials' bytes, rounded up to 16 so that the pre gates after them are float4-aligned
inline size_t part_bytes(const MixPlan& mp, int64_t rows, int head) {
  const size_t b = static_cast<size_t>(mp.splits) * static_cast<size_t>(rows) * ((head ? HC : NMIX) + 1) * sizeof(float);
  return (b + 15) & ~static_cast<size_t>(15);
}

// y[row, j, d] = post[row, j] x[row, d] + sum_i comb[row, i, j] residual[row, i, d]
__global__ void __launch_bounds__(256) hc_post_kernel(const float* x, const float* res, const float* post,
                                                      const float* comb, float* out, int64_t rows, int dim) {
  pdl_wait();
  pdl_trigger();
  const int64_t n4 = rows * (dim / 4);
  for (int64_t i = blockIdx.x * 256ll + threadIdx.x; i < n4; i += static_cast<int64_t>(gridDim.x) * 256) {
    const int64_t row = i / (dim / 4);
    const int d = static_cast<int>(i % (dim / 4)) * 4;
    const float4 xv = *reinterpret_cast<const float4*>(x + row * dim + d);
    float4 r[HC];
#pragma unroll
    for (int k = 0; k < HC; ++k) r[k] = *reinterpret_cast<const float4*>(res + (row * HC + k) * dim + d);
#pragma unroll
    for (int j = 0; j < HC; ++j) {
      const float pj = post[row * HC + j];
      float4 o = make_float4(pj * xv.x, pj * xv.y, pj * xv.z, pj * xv.w);
#pragma unroll
      for (int k = 0; k < HC; ++k) {
        const float c = comb[(row * HC + k) * HC + j];
        o.x = fmaf(c, r[k].x, o.x);
        o.y = fmaf(c, r[k].y, o.y);
        o.z = fmaf(c, r[k].z, o.z);
        o.w = fmaf(c, r[k].w, o.w);
      }
      *reinterpret_cast<float4*>(out + (row * HC + j) * dim + d) = o;
    }
  }
}

}  // namespace hcn
}  // namespace dsv4

using namespace dsv4;

extern "C" size_t dsv4_hc_workspace_size(int64_t rows, int32_t hc, int32_t dim, int32_t head) {
  if (rows <= 0 || hc != hcn::HC || dim <= 0) return 0;
  const hcn::MixPlan mp = hcn::mix_plan(rows, hc * dim);
  // [split][row][nmix + 1] partial mixes, then [row][hc] pre gates
  return hcn::part_bytes(mp, rows, head) + static_cast<size_t>(rows) * hcn::HC * sizeof(float);
}

extern "C" int dsv4_hc_pre(const dsv4_hc_params* p, void* stream) {
  DSV4_CHECK_ARG(p && p->x && p->fn && p->scale && p->base, "dsv4_hc_pre: NULL tensor");
  DSV4_CHECK_ARG(p->hc == hcn::HC, "dsv4_hc_pre: hc %d unsupported (4 only)", p->hc);
  DSV4_CHECK_ARG(p->rows >= 0 && p->dim > 0 && p->dim % 4 == 0 && p->dim <= hcn::MAXDIM,
                 "dsv4_hc_pre: dim %d must be a multiple of 4 and at most 4096", p->dim);
  DSV4_CHECK_ARG(p->head || (p->sinkhorn_iters >= 1 && p->post && p->comb),
                 "dsv4_hc_pre: post, comb and sinkhorn_iters >= 1 are needed (head == 0)");
  DSV4_CHECK_ARG(p->y || p->y_norm, "dsv4_hc_pre: no output");
  DSV4_CHECK_DTYPE(p->y_norm == nullptr || p->y_norm_dtype == DSV4_F32 || p->y_norm_dtype == DSV4_BF16,
                   "dsv4_hc_pre: y_norm dtype");
  if (p->rows == 0) return DSV4_OK;
  const size_t need = dsv4_hc_workspace_size(p->rows, p->hc, p->dim, p->head);
  if (p->workspace == nullptr || p->workspace_bytes < need || reinterpret_cast<uintptr_t>(p->workspace) % 16) {
    set_error("dsv4_hc_pre: a 16-byte aligned workspace of %zu bytes is needed", need);
    return DSV4_ERR_WORKSPACE;
  }
  const int L = hcn::HC * p->dim;
  const hcn::MixPlan mp = hcn::mix_plan(p->rows, L);
  float* part = static_cast<float*>(p->workspace);
  float* pre = reinterpret_cast<float*>(static_cast<char*>(p->workspace) + hcn::part_bytes(mp, p->rows, p->head));
  const dim3 mgrid(static_cast<unsigned>((p->rows + 16 * mp.tpl - 1) / (16 * mp.tpl)), static_cast<unsigned>(mp.splits));
  cudaStream_t st = as_stream(stream);
  const dim3 mblock(hcn::MIX_THREADS);
  if (p->head && mp.tpl == 8)
    DSV4_CUDA_CHECK(launch_pdl(hcn::hc_mix_kernel<hcn::HC, 8>, mgrid, mblock, 0, st, p->x, p->fn, part, p->rows, L, mp.kc));
  else if (p->head)
    DSV4_CUDA_CHECK(launch_pdl(hcn::hc_mix_kernel<hcn::HC, 2>, mgrid, mblock, 0, st, p->x, p->fn, part, p->rows, L, mp.kc));
  else if (mp.tpl == 8)
    DSV4_CUDA_CHECK(
        launch_pdl(hcn::hc_mix_kernel<hcn::NMIX, 8>, mgrid, mblock, 0, st, p->x, p->fn, part, p->rows, L, mp.kc));
  else
    DSV4_CUDA_CHECK(
        launch_pdl(hcn::hc_mix_kernel<hcn::NMIX, 2>, mgrid, mblock, 0, st, p->x, p->fn, part, p->rows, L, mp.kc));
  const int nj = (p->dim + 1023) / 1024;
  const dim3 grid(static_cast<unsigned>(p->rows)), yblock(hcn::Y_THREADS);
  const float* partc = part;
  if (mp.fused) {
    if (nj <= 1)
      DSV4_CUDA_CHECK(launch_pdl(hcn::hc_fused_kernel<1>, grid, yblock, 0, st, *p, partc, mp.splits));
    else if (nj <= 2)
      DSV4_CUDA_CHECK(launch_pdl(hcn::hc_fused_kernel<2>, grid, yblock, 0, st, *p, partc, mp.splits));
    else
      DSV4_CUDA_CHECK(launch_pdl(hcn::hc_fused_kernel<4>, grid, yblock, 0, st, *p, partc, mp.splits));
    return DSV4_OK;
  }
  const dim3 sgrid(static_cast<unsigned>((p->rows + hcn::SK_THREADS / 32 - 1) / (hcn::SK_THREADS / 32)));
  DSV4_CUDA_CHECK(launch_pdl(hcn::hc_sinkhorn_kernel, sgrid, dim3(hcn::SK_THREADS), 0, st, *p, partc, mp.splits, pre));
  const float* prec = pre;
  if (nj <= 1)
    DSV4_CUDA_CHECK(launch_pdl(hcn::hc_y_kernel<1>, grid, yblock, 0, st, *p, prec));
  else if (nj <= 2)
    DSV4_CUDA_CHECK(launch_pdl(hcn::hc_y_kernel<2>, grid, yblock, 0, st, *p, prec));
  else
    DSV4_CUDA_CHECK(launch_pdl(hcn::hc_y_kernel<4>, grid, yblock, 0, st, *p, prec));
  return DSV4_OK;
}

extern "C" int dsv4_hc_post(const float* x, const float* residual, const float* post, const float* comb, float* out,
                            int64_t rows, int32_t hc, int32_t dim, void* stream) {
  DSV4_CHECK_ARG(x && residual && post && comb && out, "dsv4_hc_post: NULL tensor");
  DSV4_CHECK_ARG(hc == hcn::HC, "dsv4_hc_post: hc %d unsupported (4 only)", hc);
  DSV4_CHECK_ARG(rows >= 0 && dim > 0 && dim % 4 == 0, "dsv4_hc_post: dim %d must be a multiple of 4", dim);
  if (rows == 0) return DSV4_OK;
  const int64_t n4 = rows * (dim / 4);
  const int64_t blocks = std::min<int64_t>((n4 + 255) / 256, 16ll * num_sms());
  DSV4_CUDA_CHECK(launch_pdl(hcn::hc_post_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, as_stream(stream),
                             x, residual, post, comb, out, rows, static_cast<int>(dim)));
  return DSV4_OK;
}
