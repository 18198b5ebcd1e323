// Gathered sparse MLA attention on the 5th-generation tensor cores (tcgen05 + TMEM), for prefill:
// one CTA per query, all 64 heads, the query's index list in tiles of 128 gathered rows.
//
// Per tile, in the transposed form that keeps every accumulator in tensor memory:
//   S^T[row, head] = KV_tile[row, :] . Q[head, :]         M=128 rows, N=64 heads, K=512
//   softmax over rows per head (online, exp2 domain), P^T[row, head] -> shared memory (bf16)
//   O^T[dim, head] += V_tile^T[dim, row] . P^T[row, head]  4 MMAs of M=128 dims, N=64, K=128 rows
// S^T lives in TMEM columns [256, 320), O^T in [0, 256) (lane = row for S^T, lane = dim for O^T).
// Shared memory holds Q and the gathered tile as 128-byte-swizzled K-major slabs of 64 dims
// ([rows x 128 B] each); the same tile is read as V^T through an MN-major descriptor, so V is
// never copied. One elected thread issues the MMAs; completion is tracked by mbarriers whose waits
// are bounded: on a timeout the kernel records DSV4_ERR_WAIT_TIMEOUT, stops issuing work, waits
// (bounded) for what it issued, frees its tensor memory and returns.
// The sink enters only the denominator, as in ref_torch/sparse_attn.py:33.
#include "common.cuh"
#include "tcgen05.cuh"

namespace dsv4 {
namespace tc {

constexpr int D = 512, HB = 64, BN = 128, THREADS = 128;
constexpr int SLAB_Q = HB * 128;     // bytes of one 64-dim slab of Q (64 rows x 128 B)
constexpr int SLAB_KV = BN * 128;    // bytes of one 64-dim slab of the tile (128 rows x 128 B)
constexpr int TMEM_COLS = 512;
constexpr int COL_O = 0, COL_S = 256;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float RESCALE_THRESHOLD = 8.0f;   // log2 units: p may reach 2^8 before O is rescaled

struct Smem {
  alignas(1024) uint8_t q[8 * SLAB_Q];     // 64 KB
  alignas(1024) uint8_t kv[8 * SLAB_KV];   // 128 KB
  alignas(1024) uint8_t p[BN * 128];       // 16 KB: P^T rows (64 heads x bf16)
  float red[4][HB];
  float m_run[HB];
  float l_run[HB];
  float alpha[HB];
  int32_t rows[BN];
  uint64_t bar_s, bar_o;
  uint32_t tmem_base;
  int flags;  // bit 0: rescale needed this tile; bit 1: abort
};

struct Params {
  const __nv_bfloat16* q;
  const __nv_bfloat16* kv;
  const float* sink;
  const void* idx;
  void* out;
  int64_t s, n;
  int h, t;
  int idx_dtype, out_dtype;
  float scale_log2;
  const float* rope_freqs;
  const int32_t* positions;
  int rope_dim;
  const int64_t* win_base;
  int win_stride, window, window_linear;
};

using namespace tc5;

// pool row of logical list entry u of query qi ([implicit window | idx]); -1 = masked
__device__ __forceinline__ int64_t list_row(const Params& P, int64_t qi, int u) {
  if (P.win_base != nullptr) {
    if (u < P.window) {
      const int p = P.positions[qi];
      const int W = P.window;
      int slot;
      if (P.window_linear) {
        const int lo = p - W + 1 > 0 ? p - W + 1 : 0;
        slot = (lo + u <= p) ? lo + u : -1;
      } else if (p >= W - 1) {
        const int sp = p % W;
        slot = (u < W - sp - 1) ? (sp + 1 + u) : (u - (W - sp - 1));
      } else {
        slot = (u <= p) ? u : -1;
      }
      return slot < 0 ? -1 : P.win_base[qi * P.win_stride] + slot;
    }
    u -= P.window;
  }
  if (P.idx_dtype == DSV4_I64) return __ldg(reinterpret_cast<const long long*>(P.idx) + qi * P.t + u);
  return __ldg(reinterpret_cast<const int32_t*>(P.idx) + qi * P.t + u);
}

// Column reduction of 64 per-lane values over the warp's 32 lanes ("transpose-reduce"): after
// five halving rounds lane l holds the result for heads 2l and 2l+1.
template <bool MAX>
__device__ __forceinline__ void warp_col_reduce(const float* v, float* out2) {
  const int lane = threadIdx.x & 31;
  float a[32];
  {
    const bool b = lane & 16;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float keep = b ? v[i + 32] : v[i];
      const float send = b ? v[i] : v[i + 32];
      const float got = __shfl_xor_sync(0xffffffffu, send, 16);
      a[i] = MAX ? fmaxf(keep, got) : keep + got;
    }
  }
#pragma unroll
  for (int c = 16, o = 8; c >= 2; c >>= 1, o >>= 1) {
    const bool b = lane & o;
#pragma unroll
    for (int i = 0; i < c; ++i) {
      const float keep = b ? a[i + c] : a[i];
      const float send = b ? a[i] : a[i + c];
      const float got = __shfl_xor_sync(0xffffffffu, send, o);
      a[i] = MAX ? fmaxf(keep, got) : keep + got;
    }
  }
  out2[0] = a[0];
  out2[1] = a[1];
}

__global__ void __launch_bounds__(THREADS, 1) attn_tc_kernel(Params P) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // the 128-byte swizzle pattern is anchored to 1024-byte boundaries
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t qi = blockIdx.x;
  const int L = (P.win_base ? P.window : 0) + P.t;
  const int ntiles = (L + BN - 1) / BN;

  if (warp == 0) tmem_alloc<TMEM_COLS>(&sm.tmem_base);
  if (tid == 0) {
    bar_init(&sm.bar_s, 1);
    bar_init(&sm.bar_o, 1);
    sm.flags = 0;
    bar_init_fence();
  }
  if (tid < HB) {
    sm.m_run[tid] = -INFINITY;
    sm.l_run[tid] = 0.f;
  }
  // Q -> 8 swizzled slabs (64 heads x 128 B)
  {
    const uint32_t qs = smem_u32(sm.q);
    const __nv_bfloat16* qg = P.q + qi * HB * D;
    for (int c = tid; c < HB * 64; c += THREADS) {
      const int hh = c >> 6, ch = c & 63;
      cp_async16(qs + slab_off(hh, ch, SLAB_Q), qg + hh * D + ch * 8, true);
    }
    asm volatile("cp.async.commit_group;\n" ::);
  }
  before_sync();
  __syncthreads();
  after_sync();
  const uint32_t tmem = sm.tmem_base;
  const uint32_t t_lane = static_cast<uint32_t>(warp * 32) << 16;  // this warp's TMEM lane quadrant

  const uint32_t id_s = idesc_bf16<128, HB>(false, false);
  const uint32_t id_o = idesc_bf16<128, HB>(true, true);
  uint32_t phase = 0;
  bool abort = false;

  for (int tile = 0; tile < ntiles && !abort; ++tile) {
    // (a) the previous O^T MMAs read the tile and P: wait for them before overwriting
    // every abort decision is block-uniform (__syncthreads_or), so no thread is left at a barrier
    if (tile > 0) {
      const bool ok = bar_wait(&sm.bar_o, phase ^ 1);
      if (__syncthreads_or(!ok)) {
        abort = true;
        break;
      }
    }
    // (b) gather the tile's rows into the swizzled slabs
    {
      const int u = tile * BN + tid;
      int64_t v = -1;
      if (u < L) v = list_row(P, qi, u);
      if (v >= P.n) {
        raise_device_error(DSV4_ERR_INDEX_OUT_OF_RANGE);
        v = -1;
      }
      sm.rows[tid] = static_cast<int32_t>(v);
    }
    __syncthreads();
    {
      const uint32_t ks = smem_u32(sm.kv);
      for (int c = tid; c < BN * 64; c += THREADS) {
        const int r = c >> 6, ch = c & 63;
        const int32_t row = sm.rows[r];
        cp_async16(ks + slab_off(r, ch, SLAB_KV), P.kv + static_cast<int64_t>(row < 0 ? 0 : row) * D + ch * 8,
                   row >= 0);
      }
      asm volatile("cp.async.commit_group;\n" ::);
      asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    }
    fence_async_smem();
    before_sync();
    __syncthreads();
    after_sync();
    // (c) S^T = KV . Q^T over K = 512 (8 slabs x 4 steps of 16 dims)
    if (tid == 0) {
      const uint32_t ks = smem_u32(sm.kv), qs = smem_u32(sm.q);
#pragma unroll 1
      for (int sl = 0; sl < 8; ++sl)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma16(tmem + COL_S, sdesc(ks + sl * SLAB_KV + kk * 32, 16, 1024),
                  sdesc(qs + sl * SLAB_Q + kk * 32, 16, 1024), id_s, (sl | kk) ? 1u : 0u);
      mma_commit(&sm.bar_s);
    }
    {
      const bool ok = bar_wait(&sm.bar_s, phase);
      if (__syncthreads_or(!ok)) {
        abort = true;
        break;
      }
    }
    after_sync();
    // (d) this thread's row of S^T: 64 heads
    float s[HB];
#pragma unroll
    for (int c = 0; c < HB; c += 16) tmem_ld16(tmem + t_lane + COL_S + c, s + c);
    tmem_wait_ld();
    const bool valid = sm.rows[tid] >= 0;
#pragma unroll
    for (int i = 0; i < HB; ++i) s[i] = valid ? s[i] * P.scale_log2 : -INFINITY;
    // (e) per-head maximum over the tile's 128 rows
    float r2[2];
    warp_col_reduce<true>(s, r2);
    sm.red[warp][2 * lane] = r2[0];
    sm.red[warp][2 * lane + 1] = r2[1];
    __syncthreads();
    if (tid < HB) {
      const float tmax = fmaxf(fmaxf(sm.red[0][tid], sm.red[1][tid]), fmaxf(sm.red[2][tid], sm.red[3][tid]));
      const float mr = sm.m_run[tid];
      const float mc = fmaxf(mr, tmax);
      // rescale only when the running maximum is -inf (nothing accumulated yet: adopt the new
      // one, O is overwritten by the first MMA) or grows by more than the threshold
      if (mr == -INFINITY) {
        sm.m_run[tid] = mc;
        sm.alpha[tid] = 0.f;
      } else if (mc - mr > RESCALE_THRESHOLD) {
        sm.m_run[tid] = mc;
        sm.alpha[tid] = exp2f(mr - mc);
        atomicOr(&sm.flags, 1);
      } else {
        sm.alpha[tid] = 1.f;
      }
    }
    __syncthreads();
    const bool rescale = (sm.flags & 1) != 0;
    // (f) p = exp2(s - m); column sums; P^T row -> shared memory (bf16, swizzled)
#pragma unroll
    for (int i = 0; i < HB; ++i) {
      const float m = sm.m_run[i];
      s[i] = (m == -INFINITY) ? 0.f : exp2f(s[i] - m);
    }
    {
      uint8_t* prow = sm.p + tid * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 u = make_uint4(pack_bf16x2(s[c * 8 + 0], s[c * 8 + 1]), pack_bf16x2(s[c * 8 + 2], s[c * 8 + 3]),
                             pack_bf16x2(s[c * 8 + 4], s[c * 8 + 5]), pack_bf16x2(s[c * 8 + 6], s[c * 8 + 7]));
        *reinterpret_cast<uint4*>(prow + ((c ^ (tid & 7)) << 4)) = u;
      }
    }
    warp_col_reduce<false>(s, r2);
    __syncthreads();  // red[] reuse
    sm.red[warp][2 * lane] = r2[0];
    sm.red[warp][2 * lane + 1] = r2[1];
    __syncthreads();
    if (tid < HB) {
      const float ts = (sm.red[0][tid] + sm.red[1][tid]) + (sm.red[2][tid] + sm.red[3][tid]);
      const float a = sm.alpha[tid];
      sm.l_run[tid] = (a == 0.f ? 0.f : sm.l_run[tid] * a) + ts;
    }
    // O^T *= alpha per head (column) when some maximum grew past the threshold
    if (rescale && tile > 0) {
      float al[HB];
#pragma unroll
      for (int i = 0; i < HB; ++i) al[i] = sm.alpha[i] == 0.f ? 1.f : sm.alpha[i];
#pragma unroll 1
      for (int mt = 0; mt < 4; ++mt) {
#pragma unroll
        for (int c = 0; c < HB; c += 16) {
          float v[16];
          tmem_ld16(tmem + t_lane + COL_O + mt * HB + c, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] *= al[c + i];
          tmem_st16(tmem + t_lane + COL_O + mt * HB + c, v);
        }
      }
      tmem_wait_st();
    }
    fence_async_smem();
    before_sync();
    __syncthreads();
    after_sync();
    if (tid == 0) sm.flags &= ~1;
    // (g) O^T += V^T . P^T : 4 M-tiles of 128 dims, K = 128 rows in 8 steps of 16
    if (tid == 0) {
      const uint32_t ks = smem_u32(sm.kv), ps = smem_u32(sm.p);
#pragma unroll 1
      for (int mt = 0; mt < 4; ++mt)
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma16(tmem + COL_O + mt * HB, sdesc(ks + 2 * mt * SLAB_KV + kk * 2048, SLAB_KV, 1024),
                  sdesc(ps + kk * 2048, 16384, 1024), id_o, (tile > 0 || kk > 0) ? 1u : 0u);
      mma_commit(&sm.bar_o);
    }
    phase ^= 1;
  }
  bool ok = !abort;
  if (ok && ntiles > 0) ok = !__syncthreads_or(!bar_wait(&sm.bar_o, phase ^ 1));
  if (!ok) {
    // let whatever was issued drain (bounded waits) before the tensor memory is freed
    if (tid == 0) raise_device_error(DSV4_ERR_WAIT_TIMEOUT);
    bar_wait(&sm.bar_s, phase);
    bar_wait(&sm.bar_o, phase ^ 1);
  }
  after_sync();
  if (ok) {
    // epilogue: lane = dim (within the M-tile), 64 heads per thread; normalise, inverse rope, store
    const bool rope = P.rope_freqs != nullptr;
    const int pos = rope ? P.positions[qi] : 0;
    float inv[HB];
#pragma unroll
    for (int i = 0; i < HB; ++i) {
      const float m = sm.m_run[i];
      inv[i] = (m == -INFINITY) ? __int_as_float(0x7fc00000)
                                : 1.f / (sm.l_run[i] + exp2f(P.sink[i] * LOG2E - m));
    }
#pragma unroll 1
    for (int mt = 0; mt < 4; ++mt) {
      const int d = mt * 128 + tid;
      const bool do_rope = rope && d >= D - P.rope_dim;
      float c = 1.f, sn = 0.f;
      if (do_rope) rope_cos_sin(pos, P.rope_freqs[(d - (D - P.rope_dim)) >> 1], &c, &sn);
#pragma unroll
      for (int cc = 0; cc < HB; cc += 16) {
        float v[16];
        tmem_ld16(tmem + t_lane + COL_O + mt * HB + cc, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float x = v[i] * inv[cc + i];
          if (do_rope) {
            // the pair (d, d+1) sits in lanes (even, odd)
            const float other = __shfl_xor_sync(0xffffffffu, x, 1);
            float y0, y1;
            if ((d & 1) == 0) {
              rotate_pair(x, other, c, sn, true, &y0, &y1);
              x = y0;
            } else {
              rotate_pair(other, x, c, sn, true, &y0, &y1);
              x = y1;
            }
          }
          const int64_t off = (qi * P.h + cc + i) * D + d;
          if (P.out_dtype == DSV4_BF16)
            reinterpret_cast<__nv_bfloat16*>(P.out)[off] = __float2bfloat16_rn(x);
          else
            reinterpret_cast<float*>(P.out)[off] = x;
        }
      }
    }
  }
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");  // Q copies, when the list was empty
  before_sync();
  __syncthreads();
  if (warp == 0) tmem_dealloc<TMEM_COLS>(tmem);
}

DSV4_ERROR_READER(attn_tc)

}  // namespace tc
}  // namespace dsv4

using namespace dsv4;

// Internal entry used by dsv4_sparse_attn for prefill shapes (64 heads, bf16 q, no split).
int dsv4_sparse_attn_tc(const dsv4_sparse_attn_params* p, void* stream) {
  tc::Params P;
  P.q = reinterpret_cast<const __nv_bfloat16*>(p->q);
  P.kv = reinterpret_cast<const __nv_bfloat16*>(p->kv);
  P.sink = p->sink;
  P.idx = p->idx;
  P.out = p->out;
  P.s = p->s;
  P.n = p->n;
  P.h = p->h;
  P.t = p->t;
  P.idx_dtype = p->idx_dtype;
  P.out_dtype = p->out_dtype;
  P.scale_log2 = p->scale * tc::LOG2E;
  P.rope_freqs = p->rope_freqs;
  P.positions = p->positions;
  P.rope_dim = p->rope_dim;
  P.win_base = p->win_base;
  P.win_stride = p->win_stride;
  P.window = p->win_base ? p->window : 0;
  P.window_linear = p->window_linear;
  const int smem = static_cast<int>(sizeof(tc::Smem)) + 1024;
  static bool attr = false;
  if (!attr) {
    DSV4_CUDA_CHECK(cudaFuncSetAttribute(tc::attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr = true;
  }
  tc::attn_tc_kernel<<<static_cast<unsigned>(p->s), tc::THREADS, smem, as_stream(stream)>>>(P);
  DSV4_LAUNCH_CHECK("attn_tc_kernel");
  return DSV4_OK;
}
