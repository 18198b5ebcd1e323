// KV block compressor (ref_torch/compressor.py:21-50; decode ring oracle/decode_engine.py:96-105).
//
// Input: the two projections kv = x wkv^T and score = x wgate^T (fp32, [b, s, 2d]) from the
// projection GEMM. For compressed row g of a sequence, dim c in [0, d):
//   slots 0..3: kv[4g-4+r, c],      score[4g-4+r, c]   + ape[r, c]      (group 0: 0 / -inf)
//   slots 4..7: kv[4g+r,   d + c],  score[4g+r,   d + c] + ape[r, d + c]
//   pooled[c] = sum_slot softmax_slot(score) * kv
// then RMSNorm(norm_w), RoPE of the last rope_dim dims at position ratio*g (+pos0), and one
// 128-bit vectorised store per thread into the cache (bf16) or a plain fp32 output; rows can be
// scattered into a paged pool through out_rows. One CTA per compressed row, one thread per two
// dims (up to 256 threads, whole warps). The decode kernel keeps the per-sequence ring [2*ratio, 2d] on the device.
#include <algorithm>

#include "common.cuh"
#include "key_image.cuh"

namespace dsv4 {
namespace cmp {

constexpr int THREADS = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x < 32) {
    t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[32] = t;
  }
  __syncthreads();
  return red[32];
}

__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_max(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x < 32) {
    t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_max(t);
    if (threadIdx.x == 0) red[32] = t;
  }
  __syncthreads();
  return red[32];
}

__device__ __forceinline__ void store_pair(float v0, float v1, int c, int d, void* out, int64_t orow, int out_dtype) {
  const int64_t off = orow * d + c;
  if (out_dtype == DSV4_BF16)
    *reinterpret_cast<uint32_t*>(reinterpret_cast<__nv_bfloat16*>(out) + off) = pack_bf16x2(v0, v1);
  else
    *reinterpret_cast<float2*>(reinterpret_cast<float*>(out) + off) = make_float2(v0, v1);
}

// The indexer compressor's key simulation (act_quant mode 2; v4mlx/compressor.py:57-59 with
// v4mlx/qat.py:8-31) on a 128-dim row held as pairs (2 tid, 2 tid + 1) by threads 0..63: the
// normalised Walsh-Hadamard transform (width-1 butterflies in the thread, widths 2..32 across lanes,
// width 64 across the two warps through `xch`, then float32(128^-0.5)), and the fp4-e2m1 round
// trip per 32-dim block (16 lanes). Every thread of the CTA calls it (one barrier).
__device__ __forceinline__ void hadamard_fp4_128(float& v0, float& v1, float* xch) {
  const int tid = threadIdx.x, lane = tid & 31;
  const bool mine = tid < 64;
  const float a = v0 + v1, b = v0 - v1;
  v0 = a;
  v1 = b;
#pragma unroll
  for (int o = 1; o <= 16; o <<= 1) {
    const float p0 = __shfl_xor_sync(0xffffffffu, v0, o), p1 = __shfl_xor_sync(0xffffffffu, v1, o);
    if (lane & o) {
      v0 = p0 - v0;
      v1 = p1 - v1;
    } else {
      v0 = v0 + p0;
      v1 = v1 + p1;
    }
  }
  if (mine) {
    xch[2 * tid] = v0;
    xch[2 * tid + 1] = v1;
  }
  __syncthreads();
  if (mine) {
    const float p0 = xch[2 * (tid ^ 32)], p1 = xch[2 * (tid ^ 32) + 1];
    if (tid & 32) {
      v0 = p0 - v0;
      v1 = p1 - v1;
    } else {
      v0 = v0 + p0;
      v1 = v1 + p1;
    }
    v0 *= 0.08838834764831845f;  // float32(128^-0.5)
    v1 *= 0.08838834764831845f;
  }
  float m = fmaxf(fabsf(v0), fabsf(v1));
#pragma unroll
  for (int o = 1; o <= 8; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (mine) {
    const int e = fp4_exp(m);
    const float dn = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);
    const float up = __uint_as_float(static_cast<uint32_t>(127 + e) << 23);
    v0 = e2m1_round(fminf(fmaxf(v0 * dn, -6.f), 6.f)) * up;
    v1 = e2m1_round(fminf(fmaxf(v1 * dn, -6.f), 6.f)) * up;
  }
}

// normalise, rope and store two adjacent dims (c, c+1) of one compressed row; the stored values
// (before the cast) are left in v0, v1. In act_quant mode 2 the pair is left unstored for
// hadamard_fp4_128 and store_pair.
__device__ __forceinline__ void finish_pair(float& v0, float& v1, int c, int d, int rope_dim,
                                            const void* norm_w, int norm_dtype, float rinv,
                                            const float* freqs, int pos, void* out, int64_t orow,
                                            int out_dtype, int act_quant) {
  v0 = v0 * rinv;
  v1 = v1 * rinv;
  if (norm_w) {
    v0 = load_as_float(norm_w, c, norm_dtype) * v0;
    v1 = load_as_float(norm_w, c + 1, norm_dtype) * v1;
  }
  if (c >= d - rope_dim) {
    float cs, sn;
    rope_cos_sin(pos, freqs[(c - (d - rope_dim)) >> 1], &cs, &sn);
    rotate_pair(v0, v1, cs, sn, false, &v0, &v1);
  }
  // fp8 act-quant simulation of the nope dims: a 64-dim block is the 32 pairs of one warp (the
  // condition is warp-uniform)
  if (act_quant == 1 && c < d - rope_dim) {
    const int ex = act_quant_exp(warp_max(fmaxf(fabsf(v0), fabsf(v1))));
    v0 = fp8_round_pow2(v0, ex);
    v1 = fp8_round_pow2(v1, ex);
  }
  if (act_quant == 2) return;
  store_pair(v0, v1, c, d, out, orow, out_dtype);
}

// softmax over 8 slots (max-subtracted, as torch.softmax) and the weighted sum
__device__ __forceinline__ float pool8(const float* kv8, const float* sc8) {
  float m = sc8[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) m = fmaxf(m, sc8[i]);
  float den = 0.f, num = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float e = expf(sc8[i] - m);
    den += e;
    num = fmaf(e, kv8[i], num);
  }
  return num / den;
}

// One CTA per compressed row; blockDim = the row's pairs of dims rounded up to whole warps (at
// most THREADS), so a 128-dim row (the indexer compressor) runs 64 threads, none idle.
__global__ void __launch_bounds__(THREADS) pool_kernel(dsv4_compressor_params p) {
  pdl_wait();  // programmatic dependent launch: the previous kernel is complete from here
  pdl_trigger();
  __shared__ float red[33];
  const int groups = p.s / p.ratio;
  const int64_t rowid = blockIdx.x;  // b * groups + g
  const int b = static_cast<int>(rowid / groups);
  const int g = static_cast<int>(rowid % groups);
  const int d = p.head_dim, d2 = 2 * d;
  const int R = p.ratio;
  const float* kvb = p.kv + static_cast<int64_t>(b) * p.s * d2;
  const float* scb = p.score + static_cast<int64_t>(b) * p.s * d2;
  float vals[2][2];  // up to 2 pairs per thread (d <= 1024)
  float ss = 0.f;
  int npairs = 0;
  for (int c = threadIdx.x * 2; c < d; c += blockDim.x * 2, ++npairs) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float kv8[16], sc8[16];
      const int cc = c + e;
      for (int r = 0; r < R; ++r) {
        if (g > 0) {
          const int64_t t = static_cast<int64_t>(g - 1) * R + r;
          kv8[r] = kvb[t * d2 + cc];
          sc8[r] = scb[t * d2 + cc] + p.ape[r * d2 + cc];
        } else {
          kv8[r] = 0.f;
          sc8[r] = -INFINITY;
        }
        const int64_t t2 = static_cast<int64_t>(g) * R + r;
        kv8[R + r] = kvb[t2 * d2 + d + cc];
        sc8[R + r] = scb[t2 * d2 + d + cc] + p.ape[r * d2 + d + cc];
      }
      float v;
      if (R == 4) {
        v = pool8(kv8, sc8);
      } else {
        float m = sc8[0];
        for (int i = 1; i < 2 * R; ++i) m = fmaxf(m, sc8[i]);
        float den = 0.f, num = 0.f;
        for (int i = 0; i < 2 * R; ++i) {
          float ex = expf(sc8[i] - m);
          den += ex;
          num = fmaf(ex, kv8[i], num);
        }
        v = num / den;
      }
      vals[npairs][e] = v;
      ss = fmaf(v, v, ss);
    }
  }
  ss = block_sum(ss, red);
  const float rinv = rsqrtf(ss / static_cast<float>(d) + p.eps);
  const int64_t orow = p.out_rows ? p.out_rows[rowid] : rowid;
  npairs = 0;
  for (int c = threadIdx.x * 2; c < d; c += blockDim.x * 2, ++npairs)
    finish_pair(vals[npairs][0], vals[npairs][1], c, d, p.rope_dim, p.norm_w, p.norm_dtype, rinv,
                p.freqs, p.pos0 + R * g, p.out, orow, p.out_dtype, p.act_quant);
  if (p.act_quant == 2) {  // head_dim 128: threads 0..63 hold the row (uniform over the CTA)
    __shared__ float xch[128];
    hadamard_fp4_128(vals[0][0], vals[0][1], xch);
    if (threadIdx.x < 64) store_pair(vals[0][0], vals[0][1], 2 * threadIdx.x, d, p.out, orow, p.out_dtype);
  }
}

// decode hand-off ring (ref_torch/compressor.py:67-74; seeding as oracle/decode_engine.py:91-95):
// rows [0, R) = last full block (kv, score+ape), rows [R, R+rem) = remainder, rest 0 / -inf.
__global__ void ring_seed_kernel(dsv4_compressor_params p) {
  pdl_wait();  // programmatic dependent launch: the previous kernel is complete from here
  pdl_trigger();
  const int b = blockIdx.y;
  const int slot = blockIdx.x;  // 0 .. 2R-1
  const int R = p.ratio, d2 = 2 * p.head_dim;
  const int cutoff = p.s - p.s % R;
  const int rem = p.s % R;
  int64_t t = -1;
  int ape_r = 0;
  if (slot < R) {
    if (cutoff >= R) {
      t = cutoff - R + slot;
      ape_r = slot;
    }
  } else if (slot - R < rem) {
    t = cutoff + (slot - R);
    ape_r = slot - R;
  }
  float* rk = p.ring_kv + (static_cast<int64_t>(b) * 2 * R + slot) * d2;
  float* rs = p.ring_score + (static_cast<int64_t>(b) * 2 * R + slot) * d2;
  const float* kvb = p.kv + static_cast<int64_t>(b) * p.s * d2;
  const float* scb = p.score + static_cast<int64_t>(b) * p.s * d2;
  for (int c = threadIdx.x; c < d2; c += blockDim.x) {
    if (t >= 0) {
      rk[c] = kvb[t * d2 + c];
      rs[c] = scb[t * d2 + c] + p.ape[ape_r * d2 + c];
    } else {
      rk[c] = 0.f;
      rs[c] = -INFINITY;
    }
  }
}

// one decode token per sequence: ring row R + p%R <- (kv, score + ape[p%R]); when (p+1)%R == 0
// emit the pooled row at position p+1-R and shift rows [R,2R) to [0,R).
// ratio 4 (the model's): the same step with every thread owning column pairs (c, c+1) of both
// halves. The ring rows it reads were written by earlier steps and the current token's row stays
// in registers, so all of a thread's loads go out at once and the only barrier is the norm's
// reduction (the generic kernel below re-reads the ring it just wrote, behind a barrier, with
// runtime-sized loops). Same operations in the same order: identical results.
__device__ __forceinline__ float2 ld2(const float* p) { return *reinterpret_cast<const float2*>(p); }
__device__ __forceinline__ void st2(float* p, float2 v) { *reinterpret_cast<float2*>(p) = v; }

// the emitted row (indexer key, head_dim 128 = 64 pairs held by threads 0..63, fp32 values as
// stored) added to the key image: scaled and split as dsv4_indexer_key_image does it, its inverse
// scale, and the entry's norm maximum raised
template <int NP>
__device__ __forceinline__ void append_key_image(const dsv4_compressor_decode_params& p, const float (&vals)[NP][2],
                                                 float* red) {
  const int tid = threadIdx.x;
  const bool mine = 2 * tid < p.head_dim;
  const float v0 = mine ? vals[0][0] : 0.f, v1 = mine ? vals[0][1] : 0.f;
  const float mx = block_max(fmaxf(fabsf(v0), fabsf(v1)), red);
  const float ss = block_sum(fmaf(v1, v1, v0 * v0), red);
  const int64_t orow = p.out_rows[blockIdx.x];
  const int64_t seq = orow / p.image_stride, j = orow % p.image_stride;
  const int64_t tiles = (p.image_stride + 127) / 128;
  const int sh = itc::row_shift(mx);
  if (mine) {
    uint32_t hi, lo;
    const float up = itc::pow2(sh);
    itc::split2(v0 * up, v1 * up, &hi, &lo);
    const int c = 2 * tid;
    uint8_t* img = p.key_image + (seq * tiles + j / 128) * itc::IMG_TILE_BYTES;
    const uint32_t off = itc::key_off(static_cast<int>(j % 128), c >> 2) + ((c >> 1) & 1) * 4;
    *reinterpret_cast<uint32_t*>(img + off) = hi;
    *reinterpret_cast<uint32_t*>(img + off + itc::IMG_SLAB_K) = lo;
  }
  if (tid == 0) {
    p.key_inv[seq * tiles * 128 + j] = itc::pow2(-sh);
    atomicMax(reinterpret_cast<unsigned int*>(p.key_norm_max + seq), __float_as_uint(sqrtf(ss)));
  }
}

// the ratio-4 step of sequence blockIdx.x for one compressor (the body of decode_r4_kernel)
template <int NP>
__device__ __forceinline__ void decode_r4_row(const dsv4_compressor_decode_params& p) {
  constexpr int R = 4;
  __shared__ float red[33];
  const int b = blockIdx.x, tid = threadIdx.x;
  const int d = p.head_dim, d2 = 2 * d;
  const int pos = p.positions[b];
  const int slot = R + pos % R;
  float* rk = p.ring_kv + static_cast<int64_t>(b) * 2 * R * d2;
  float* rs = p.ring_score + static_cast<int64_t>(b) * 2 * R * d2;
  const float* kin = p.kv + static_cast<int64_t>(b) * d2;
  const float* sin_ = p.score + static_cast<int64_t>(b) * d2;
  const float* ape = p.ape + (pos % R) * d2;
  const bool emit = (pos + 1) % R == 0;
  float2 nk[NP][2], ns[NP][2];  // this token's kv and score + ape, columns c and d + c
  float2 K[NP][8], S[NP][8], F[NP][3], G[NP][3];  // pooled inputs; rows 4..6 of the first half (shift)
#pragma unroll
  for (int np = 0; np < NP; ++np) {
    const int c = 2 * (tid + np * THREADS);
    if (c >= d) continue;
    nk[np][0] = ld2(kin + c);
    nk[np][1] = ld2(kin + d + c);
    const float2 s0 = ld2(sin_ + c), s1 = ld2(sin_ + d + c), a0 = ld2(ape + c), a1 = ld2(ape + d + c);
    ns[np][0] = make_float2(s0.x + a0.x, s0.y + a0.y);
    ns[np][1] = make_float2(s1.x + a1.x, s1.y + a1.y);
    if (emit) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        K[np][r] = ld2(rk + r * d2 + c);
        S[np][r] = ld2(rs + r * d2 + c);
      }
#pragma unroll
      for (int r = 0; r < R - 1; ++r) {
        K[np][R + r] = ld2(rk + (R + r) * d2 + d + c);
        S[np][R + r] = ld2(rs + (R + r) * d2 + d + c);
        F[np][r] = ld2(rk + (R + r) * d2 + c);
        G[np][r] = ld2(rs + (R + r) * d2 + c);
      }
      K[np][2 * R - 1] = nk[np][1];  // row 2R - 1 is this token's slot
      S[np][2 * R - 1] = ns[np][1];
    }
    // the slot is written in every case (after an emission the ring holds what the generic kernel
    // leaves: this token's row both in its slot and, shifted, in row R - 1)
    st2(rk + slot * d2 + c, nk[np][0]);
    st2(rk + slot * d2 + d + c, nk[np][1]);
    st2(rs + slot * d2 + c, ns[np][0]);
    st2(rs + slot * d2 + d + c, ns[np][1]);
  }
  if (!emit) return;  // uniform over the CTA
  float vals[NP][2];
  float ss = 0.f;
#pragma unroll
  for (int np = 0; np < NP; ++np) {
    const int c = 2 * (tid + np * THREADS);
    if (c >= d) continue;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float m = e ? S[np][0].y : S[np][0].x;
#pragma unroll
      for (int i = 1; i < 2 * R; ++i) m = fmaxf(m, e ? S[np][i].y : S[np][i].x);
      float den = 0.f, num = 0.f;
#pragma unroll
      for (int i = 0; i < 2 * R; ++i) {
        const float ex = expf((e ? S[np][i].y : S[np][i].x) - m);
        den += ex;
        num = fmaf(ex, e ? K[np][i].y : K[np][i].x, num);
      }
      vals[np][e] = num / den;
      ss = fmaf(vals[np][e], vals[np][e], ss);
    }
  }
  ss = block_sum(ss, red);
  const float rinv = rsqrtf(ss / static_cast<float>(d) + p.eps);
#pragma unroll
  for (int np = 0; np < NP; ++np) {
    const int c = 2 * (tid + np * THREADS);
    if (c >= d) continue;
    finish_pair(vals[np][0], vals[np][1], c, d, p.rope_dim, p.norm_w, p.norm_dtype, rinv, p.freqs, pos + 1 - R,
                p.out, p.out_rows[b], p.out_dtype, p.act_quant);
    // the block's rows become the previous block (rows 0..R-1); this token's row is the last
#pragma unroll
    for (int r = 0; r < R - 1; ++r) {
      st2(rk + r * d2 + c, F[np][r]);
      st2(rs + r * d2 + c, G[np][r]);
      st2(rk + r * d2 + d + c, K[np][R + r]);
      st2(rs + r * d2 + d + c, S[np][R + r]);
    }
    st2(rk + (R - 1) * d2 + c, nk[np][0]);
    st2(rs + (R - 1) * d2 + c, ns[np][0]);
    st2(rk + (R - 1) * d2 + d + c, nk[np][1]);
    st2(rs + (R - 1) * d2 + d + c, ns[np][1]);
  }
  if (p.act_quant == 2) {  // head_dim 128: threads 0..63 hold the row (uniform over the CTA)
    __shared__ float xch[128];
    hadamard_fp4_128(vals[0][0], vals[0][1], xch);
    if (tid < 64) store_pair(vals[0][0], vals[0][1], 2 * tid, d, p.out, p.out_rows[b], p.out_dtype);
  }
  if (p.key_image) append_key_image<NP>(p, vals, red);
}

template <int NP>
__global__ void __launch_bounds__(THREADS) decode_r4_kernel(dsv4_compressor_decode_params p) {
  pdl_wait();  // programmatic dependent launch: the previous kernel is complete from here
  pdl_trigger();
  decode_r4_row<NP>(p);
}

// two compressors' steps in one launch (grid.y = 2; the same batch): a decode block's main and
// indexer compressors, which read the same token's projections and write disjoint rings and rows
template <int NP>
__global__ void __launch_bounds__(THREADS) decode_r4_pair_kernel(dsv4_compressor_decode_params p0,
                                                                 dsv4_compressor_decode_params p1) {
  pdl_wait();
  pdl_trigger();
  const dsv4_compressor_decode_params& p = blockIdx.y ? p1 : p0;
  decode_r4_row<NP>(p);
}

__global__ void __launch_bounds__(THREADS) decode_kernel(dsv4_compressor_decode_params p) {
  pdl_wait();  // programmatic dependent launch: the previous kernel is complete from here
  pdl_trigger();
  __shared__ float red[33];
  const int b = blockIdx.x;
  const int R = p.ratio, d = p.head_dim, d2 = 2 * d;
  const int pos = p.positions[b];
  const int slot = R + pos % R;
  float* rk = p.ring_kv + static_cast<int64_t>(b) * 2 * R * d2;
  float* rs = p.ring_score + static_cast<int64_t>(b) * 2 * R * d2;
  const float* kin = p.kv + static_cast<int64_t>(b) * d2;
  const float* sin_ = p.score + static_cast<int64_t>(b) * d2;
  for (int c = threadIdx.x; c < d; c += blockDim.x) {
    rk[slot * d2 + c] = kin[c];
    rk[slot * d2 + d + c] = kin[d + c];
    rs[slot * d2 + c] = sin_[c] + p.ape[(pos % R) * d2 + c];
    rs[slot * d2 + d + c] = sin_[d + c] + p.ape[(pos % R) * d2 + d + c];
  }
  if ((pos + 1) % R != 0) return;
  __syncthreads();  // the pooled read below covers dims written by other threads
  float vals[2][2];
  float ss = 0.f;
  int np = 0;
  for (int c = threadIdx.x * 2; c < d; c += THREADS * 2, ++np) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int cc = c + e;
      float kv8[16], sc8[16];
      for (int r = 0; r < R; ++r) {
        kv8[r] = rk[r * d2 + cc];
        sc8[r] = rs[r * d2 + cc];
        kv8[R + r] = rk[(R + r) * d2 + d + cc];
        sc8[R + r] = rs[(R + r) * d2 + d + cc];
      }
      float m = sc8[0];
      for (int i = 1; i < 2 * R; ++i) m = fmaxf(m, sc8[i]);
      float den = 0.f, num = 0.f;
      for (int i = 0; i < 2 * R; ++i) {
        float ex = expf(sc8[i] - m);
        den += ex;
        num = fmaf(ex, kv8[i], num);
      }
      vals[np][e] = num / den;
      ss = fmaf(vals[np][e], vals[np][e], ss);
    }
  }
  ss = block_sum(ss, red);  // its barrier also orders the pooled reads before the shift below
  const float rinv = rsqrtf(ss / static_cast<float>(d) + p.eps);
  np = 0;
  for (int c = threadIdx.x * 2; c < d; c += THREADS * 2, ++np)
    finish_pair(vals[np][0], vals[np][1], c, d, p.rope_dim, p.norm_w, p.norm_dtype, rinv, p.freqs,
                pos + 1 - R, p.out, p.out_rows[b], p.out_dtype, p.act_quant);
  if (p.act_quant == 2) {  // head_dim 128: threads 0..63 hold the row (uniform over the CTA)
    __shared__ float xch[128];
    hadamard_fp4_128(vals[0][0], vals[0][1], xch);
    if (threadIdx.x < 64)
      store_pair(vals[0][0], vals[0][1], 2 * threadIdx.x, d, p.out, p.out_rows[b], p.out_dtype);
  }
  for (int c = threadIdx.x; c < d2; c += blockDim.x)
    for (int r = 0; r < R; ++r) {
      rk[r * d2 + c] = rk[(R + r) * d2 + c];
      rs[r * d2 + c] = rs[(R + r) * d2 + c];
    }
}

}  // namespace cmp
}  // namespace dsv4

using namespace dsv4;

extern "C" int dsv4_compressor_pool(const dsv4_compressor_params* p, void* stream) {
  DSV4_CHECK_ARG(p == nullptr || p->act_quant == 0 ||
                     (p->act_quant == 1 && p->head_dim % 64 == 0 && (p->head_dim - p->rope_dim) % 64 == 0) ||
                     (p->act_quant == 2 && p->head_dim == 128),
                 "dsv4_compressor_pool: act_quant 1 needs head_dim and head_dim - rope_dim multiples of 64, "
                 "act_quant 2 (Hadamard + fp4) head_dim 128");
  DSV4_CHECK_ARG(p && p->kv && p->score && p->ape && p->out && p->freqs, "dsv4_compressor_pool: NULL tensor");
  DSV4_CHECK_ARG(p->b > 0 && p->s >= 0 && p->ratio > 0 && p->ratio <= 8, "dsv4_compressor_pool: bad sizes");
  DSV4_CHECK_ARG(p->head_dim % 2 == 0 && p->head_dim <= 4 * cmp::THREADS && p->head_dim >= p->rope_dim &&
                     p->rope_dim % 2 == 0,
                 "dsv4_compressor_pool: head_dim %d unsupported", p->head_dim);
  DSV4_CHECK_DTYPE(p->out_dtype == DSV4_F32 || p->out_dtype == DSV4_BF16, "dsv4_compressor_pool: out dtype");
  DSV4_CHECK_DTYPE(p->norm_w == nullptr || p->norm_dtype == DSV4_F32 || p->norm_dtype == DSV4_BF16,
                   "dsv4_compressor_pool: norm dtype");
  const int groups = p->s / p->ratio;
  if (groups > 0) {
    // one thread per pair of dims, whole warps, at most THREADS (2 pairs a thread above 512 dims)
    const int threads = std::min(cmp::THREADS, (p->head_dim / 2 + 31) / 32 * 32);
    const dim3 grid(static_cast<unsigned>(static_cast<int64_t>(p->b) * groups));
    DSV4_CUDA_CHECK(launch_pdl(cmp::pool_kernel, grid, dim3(threads), 0, as_stream(stream), *p));
    DSV4_LAUNCH_CHECK("compressor pool_kernel");
  }
  if (p->ring_kv && p->ring_score) {
    dim3 g(2 * p->ratio, p->b);
    DSV4_CUDA_CHECK(launch_pdl(cmp::ring_seed_kernel, dim3(g), dim3(256), 0, as_stream(stream), *p));
    DSV4_LAUNCH_CHECK("compressor ring_seed_kernel");
  }
  return DSV4_OK;
}

static int check_decode_params(const dsv4_compressor_decode_params* p) {
  DSV4_CHECK_ARG(p == nullptr || p->act_quant == 0 ||
                     (p->act_quant == 1 && p->head_dim % 64 == 0 && (p->head_dim - p->rope_dim) % 64 == 0) ||
                     (p->act_quant == 2 && p->head_dim == 128),
                 "dsv4_compressor_decode: act_quant 1 needs head_dim and head_dim - rope_dim multiples of 64, "
                 "act_quant 2 (Hadamard + fp4) head_dim 128");
  DSV4_CHECK_ARG(p && p->kv && p->score && p->ape && p->ring_kv && p->ring_score && p->positions &&
                     p->out && p->out_rows && p->freqs,
                 "dsv4_compressor_decode: NULL tensor");
  DSV4_CHECK_ARG(p->b > 0 && p->ratio > 0 && p->ratio <= 8 && p->head_dim % 2 == 0 &&
                     p->head_dim <= 4 * cmp::THREADS && p->rope_dim % 2 == 0 && p->rope_dim <= p->head_dim,
                 "dsv4_compressor_decode: bad sizes");
  DSV4_CHECK_DTYPE(p->out_dtype == DSV4_F32 || p->out_dtype == DSV4_BF16, "dsv4_compressor_decode: out dtype");
  DSV4_CHECK_ARG(p->key_image == nullptr || (p->key_inv && p->key_norm_max && p->image_stride > 0 && p->ratio == 4 &&
                                              p->head_dim == 128 && p->out_dtype == DSV4_F32 &&
                                              reinterpret_cast<uintptr_t>(p->key_image) % 16 == 0),
                 "dsv4_compressor_decode: a key image needs ratio 4, head_dim 128, fp32 out, inv, norm_max, "
                 "image_stride and a 16-byte aligned image");
  return DSV4_OK;
}

extern "C" int dsv4_compressor_decode(const dsv4_compressor_decode_params* p, void* stream) {
  const int rc = check_decode_params(p);
  if (rc != DSV4_OK) return rc;
  if (p->ratio == 4 && p->head_dim <= 2 * cmp::THREADS)
    DSV4_CUDA_CHECK(launch_pdl(cmp::decode_r4_kernel<1>, dim3(p->b), dim3(cmp::THREADS), 0, as_stream(stream), *p));
  else if (p->ratio == 4)
    DSV4_CUDA_CHECK(launch_pdl(cmp::decode_r4_kernel<2>, dim3(p->b), dim3(cmp::THREADS), 0, as_stream(stream), *p));
  else
    DSV4_CUDA_CHECK(launch_pdl(cmp::decode_kernel, dim3(p->b), dim3(cmp::THREADS), 0, as_stream(stream), *p));
  DSV4_LAUNCH_CHECK("compressor decode_kernel");
  return DSV4_OK;
}

extern "C" int dsv4_compressor_decode_pair(const dsv4_compressor_decode_params* a,
                                           const dsv4_compressor_decode_params* b, void* stream) {
  int rc = check_decode_params(a);
  if (rc != DSV4_OK) return rc;
  rc = check_decode_params(b);
  if (rc != DSV4_OK) return rc;
  const bool one = a->b == b->b && a->ratio == 4 && b->ratio == 4 && a->head_dim <= 2 * cmp::THREADS &&
                   b->head_dim <= 2 * cmp::THREADS;
  if (!one) {
    rc = dsv4_compressor_decode(a, stream);
    return rc != DSV4_OK ? rc : dsv4_compressor_decode(b, stream);
  }
  DSV4_CUDA_CHECK(launch_pdl(cmp::decode_r4_pair_kernel<1>, dim3(a->b, 2), dim3(cmp::THREADS), 0, as_stream(stream),
                             *a, *b));
  DSV4_LAUNCH_CHECK("compressor decode_r4_pair_kernel");
  return DSV4_OK;
}
