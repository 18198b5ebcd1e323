// Gathered sparse MLA attention on the 5th-generation tensor cores (tcgen05 + TMEM), for prefill:
// one CTA per query, all 64 heads, the query's index list in tiles of 128 gathered rows.
//
// Per tile, in the transposed form that keeps every accumulator in tensor memory:
//   S^T[row, head] = KV_tile[row, :] . Q[head, :]          M=128 rows, N=64 heads, K=512
//   P^T[row, head] = exp2(S^T * scale * log2e - m[head])   (bf16, shared memory)
//   O^T[dim, head] += V_tile^T[dim, row] . P^T[row, head]  4 MMAs of M=128 dims, N=64, K=128 rows
//   L[*, head]     += ones[*, row] . P^T[row, head]        the softmax denominators (A in TMEM)
// TMEM columns: O^T [0, 256), S^T [256, 320), L [320, 384), the ones operand [384, 400).
// Shared memory holds Q and the gathered tile as 128-byte-swizzled K-major slabs of 64 dims; the
// tile is read again as V^T through an MN-major descriptor, so V is never copied. (An N=64 MMA
// reads 6 KB of shared memory per K=16 step and takes ~48 cycles on B200 whatever its M, so the
// 128-row tile keeps every row of the S^T MMA useful; the single tile buffer is pipelined by slab
// pairs instead of double-buffered.)
//
// Warp roles (12 warps):
//  - warps 1-11 gather: each thread owns the same 5-6 (row, 16-byte chunk) positions of every slab
//    pair and fetches them with cp.async (completion counted on the pair's mbarrier), slab pair
//    2mt, 2mt+1 of tile i as soon as the O^T MMAs of M-tile mt of tile i-1 have released it; the row
//    indices of tile i+1 are loaded while tile i is processed;
//  - warp 0, one lane, issues the MMAs: S^T pair by pair as the pairs land, then, once P^T is
//    published, the O^T M-tiles (each committed to its pair's barrier) and L;
//  - warps 4-11 also run the softmax (warp w reads TMEM lane quadrant w % 4, heads 32 * ((w-4)/4)..)
//    and the epilogue. The running maximum m is lazy: it is recomputed (exact tile maximum per head)
//    only when some score exceeds m + 8 (log2 units) or on the first tile, in which case O^T and L
//    are rescaled in TMEM; otherwise p may reach 2^8, which bf16 P and the fp32 sums absorb.
// The sink enters only the denominator, as in ref_torch/sparse_attn.py:33. All waits are bounded
// (1 s); a timeout raises DSV4_ERR_WAIT_TIMEOUT, the roles stop, and the CTA drains what it issued.
#include "common.cuh"
#include "tcgen05.cuh"

namespace dsv4 {
namespace tc {

using namespace tc5;

constexpr int D = 512, HB = 64, BN = 128;
constexpr int THREADS = 384;               // 12 warps (3 per SM sub-partition: 168 registers each)
constexpr int SM_WARP0 = 4;                 // first softmax warp
constexpr int SM_THREADS = 256;             // softmax warps 4-11 (warp w: lane quadrant w % 4)
constexpr int W_WARP0 = 1, W_THREADS = 352;  // gather workers: warps 1-11
constexpr int W_CHUNKS = 6;                 // ceil(128 rows x 16 chunks per slab pair / 352)
constexpr int SLAB_Q = HB * 128;            // 8 KB: one 64-dim slab of Q (64 rows x 128 B)
constexpr int SLAB_KV = BN * 128;           // 16 KB: one 64-dim slab of the tile (128 rows x 128 B)
constexpr int TMEM_COLS = 512;
constexpr int COL_O = 0, COL_S = 256, COL_L = 320, COL_ONES = 384;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float RESCALE_THRESHOLD = 8.0f;   // log2 units: p may reach 2^8 before m is raised

struct Smem {
  alignas(1024) uint8_t q[8 * SLAB_Q];      // 64 KB
  alignas(1024) uint8_t kv[8 * SLAB_KV];    // 128 KB
  alignas(1024) uint8_t p[BN * 128];        // 16 KB: P^T rows (64 heads x bf16)
  float red[4][HB];                         // per-quadrant column maxima
  float alpha[HB];                          // rescale factors of a tile that raised m
  float rope_c[32], rope_s[32];             // the query position's RoPE angles (rope_dim <= 64)
  uint64_t bar_full[4];                     // slab pair mt of the current tile landed (one arrival per worker)
  uint64_t bar_empty[4];                    // O^T M-tile mt done: slab pair mt free
  uint64_t bar_s, bar_p, bar_fin;           // S^T done / P^T published / everything issued done
  uint32_t tmem_base;
  int abort;
};
static_assert(sizeof(Smem) + 1024 <= 232448, "shared memory above the 227 KB a CTA may opt into");

struct Params {
  int splits;             // CTAs per query; > 1: partials into part (the split-K layout of sparse_attn.cu)
  float* part;
  const __nv_bfloat16* q;
  const __nv_bfloat16* kv;
  const void* idx;
  const float* sink;
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

__device__ __forceinline__ bool row_valid(const Params& P, int64_t qi, int u, int L) {
  if (u >= L) return false;
  const int64_t v = list_row(P, qi, u);
  return v >= 0 && v < P.n;
}

// D (+)= A . B with A in tensor memory (K-major, 16-bit), B from shared memory
__device__ __forceinline__ void mma16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(id), "r"(acc));
}

// 2^x on the SFU (ex2.approx.ftz: relative error ~2^-22, 2^-inf = +0), for the bf16 probabilities
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void sm_bar() { asm volatile("bar.sync 1, %0;\n" ::"n"(SM_THREADS) : "memory"); }
__device__ __forceinline__ bool sm_bar_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n.reg .pred p, q;\nsetp.ne.u32 p, %1, 0;\nbar.red.or.pred q, 1, %2, p;\nselp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "n"(SM_THREADS)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void set_abort(Smem& sm) {
  if (!*reinterpret_cast<volatile int*>(&sm.abort)) {
    *reinterpret_cast<volatile int*>(&sm.abort) = 1;
    raise_device_error(DSV4_ERR_WAIT_TIMEOUT);
  }
}

// Column reduction (max) of 32 per-lane values over the warp's 32 lanes: lane l ends with column l.
__device__ __forceinline__ float warp_col_max32(const float* v) {
  const int lane = threadIdx.x & 31;
  float a[16];
  {
    const bool b = lane & 16;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float keep = b ? v[i + 16] : v[i];
      const float send = b ? v[i] : v[i + 16];
      a[i] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, 16));
    }
  }
#pragma unroll
  for (int c = 8, o = 8; c >= 1; c >>= 1, o >>= 1) {
    const bool b = lane & o;
#pragma unroll
    for (int i = 0; i < c; ++i) {
      const float keep = b ? a[i + c] : a[i];
      const float send = b ? a[i] : a[i + c];
      a[i] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, o));
    }
  }
  return a[0];
}

__global__ void __launch_bounds__(THREADS, 1) attn_tc_kernel(Params P) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // the 128-byte swizzle pattern is anchored to 1024-byte boundaries
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // CTA = (query, split): tiles [tbase, tbase + ntiles) of the query's list
  const int64_t qi = blockIdx.x / P.splits;
  const int split = static_cast<int>(blockIdx.x % P.splits);
  const int L = (P.win_base ? P.window : 0) + P.t;
  const int tiles_all = (L + BN - 1) / BN;
  const int per = (tiles_all + P.splits - 1) / P.splits;
  const int tbase = split * per;
  const int ntiles = max(0, min(per, tiles_all - tbase));

  if (warp == 0) tmem_alloc<TMEM_COLS>(&sm.tmem_base);
  if (tid == 0) {
    for (int i = 0; i < 4; ++i) {
      bar_init(&sm.bar_full[i], W_THREADS);
      bar_init(&sm.bar_empty[i], 1);
    }
    bar_init(&sm.bar_s, 1);
    bar_init(&sm.bar_p, SM_THREADS);
    bar_init(&sm.bar_fin, 1);
    sm.abort = 0;
    bar_init_fence();
  }
  // gather workers (warps 1-11): this worker's (row, chunk) positions within a slab pair: c = wt + 352 k
  // < 2048; row c / 16, chunk c % 16 (slab 2mt + chunk / 8, 16-byte chunk chunk % 8 of the row's 128 B)
  const int wt = tid - W_WARP0 * 32;
  int nown = 0;
#pragma unroll
  for (int k = 0; k < W_CHUNKS; ++k) nown += (wt + W_THREADS * k < BN * 16);
  auto load_rows = [&](int i, int* rr) {
#pragma unroll
    for (int k = 0; k < W_CHUNKS; ++k) {
      const int c = wt + W_THREADS * k;
      int32_t v = 0;
      if (k < nown) {
        const int u = (tbase + i) * BN + (c >> 4);
        int64_t r = u < L ? list_row(P, qi, u) : -1;
        if (r >= P.n) {
          raise_device_error(DSV4_ERR_INDEX_OUT_OF_RANGE);
          r = -1;
        }
        v = static_cast<int32_t>(r < 0 ? 0 : r);  // masked rows fetch row 0; their p is 0
      }
      rr[k] = v;
    }
  };
  // Q -> 8 swizzled slabs (64 heads x 128 B); the first tile's row numbers and the softmax rows'
  // validity (dependent index loads) are fetched while Q lands
  int rr[W_CHUNKS];
  bool valid0 = false;
  {
    const uint32_t qs = smem_u32(sm.q);
    const __nv_bfloat16* qg = P.q + qi * HB * D;
    for (int c = tid; c < HB * 64; c += THREADS) {
      const int hh = c >> 6, ch = c & 63;
      cp_async16(qs + slab_off(hh, ch, SLAB_Q), qg + hh * D + ch * 8, true);
    }
    asm volatile("cp.async.commit_group;\n" ::);
    if (warp >= W_WARP0 && ntiles > 0) load_rows(0, rr);
    if (warp >= SM_WARP0) valid0 = row_valid(P, qi, tbase * BN + (warp & 3) * 32 + lane, L);
    // the RoPE angles of the query's position, once per CTA (one sincosf per lane of warp 0, which
    // is idle here): the epilogue's inverse rotation reads them from shared memory
    if (warp == 0 && P.rope_freqs != nullptr && P.rope_dim <= 64 && lane < P.rope_dim / 2)
      rope_cos_sin(P.positions[qi], P.rope_freqs[lane], &sm.rope_c[lane], &sm.rope_s[lane]);
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
  }
  fence_async_smem();
  before_sync();
  __syncthreads();
  after_sync();
  const uint32_t tmem = sm.tmem_base;
  const volatile int* abort = &sm.abort;

  if (warp == 0) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_bf16<128, HB>(false, false);
      constexpr uint32_t id_o = idesc_bf16<128, HB>(true, true);
      constexpr uint32_t id_l = idesc_bf16<128, HB>(false, true);
      const uint32_t ks = smem_u32(sm.kv), qs = smem_u32(sm.q), ps = smem_u32(sm.p);
      bool ok = true;
      for (int i = 0; i < ntiles && ok; ++i) {
        for (int mt = 0; mt < 4; ++mt) {
          if (!(ok = bar_wait_or_abort(&sm.bar_full[mt], i & 1, abort))) break;
          fence_async_smem();  // the cp.async writes (generic proxy) are read by the tensor cores
          after_sync();
#pragma unroll
          for (int sl = 2 * mt; sl < 2 * mt + 2; ++sl)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma16(tmem + COL_S, sdesc(ks + sl * SLAB_KV + kk * 32, 16, 1024),
                    sdesc(qs + sl * SLAB_Q + kk * 32, 16, 1024), id_s, (sl | kk) ? 1u : 0u);
        }
        if (!ok) break;
        mma_commit(&sm.bar_s);
        if (!(ok = bar_wait_or_abort(&sm.bar_p, i & 1, abort))) break;
        after_sync();
        for (int mt = 0; mt < 4; ++mt) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma16(tmem + COL_O + mt * HB, sdesc(ks + 2 * mt * SLAB_KV + kk * 2048, SLAB_KV, 1024),
                  sdesc(ps + kk * 2048, 1024, 1024), id_o, (i > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&sm.bar_empty[mt]);
        }
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma16_ta(tmem + COL_L, tmem + COL_ONES, sdesc(ps + kk * 2048, 1024, 1024), id_l, (i > 0 || kk > 0) ? 1u : 0u);
      }
      mma_commit(&sm.bar_fin);  // also on abort, so that the drain below can wait for everything issued
      if (!ok) set_abort(sm);
    }
  } else {
    // ---------------------------------------------------------------- gather workers (warps 1-11)
    const bool smx = warp >= SM_WARP0;
    const uint32_t ks = smem_u32(sm.kv);

    // softmax state (warps 4-11)
    const int qd = warp & 3;                    // TMEM lane quadrant: rows / dims qd*32 + lane
    const int half = (warp - SM_WARP0) >> 2;    // heads half*32 .. half*32+31
    const uint32_t lq = static_cast<uint32_t>(qd * 32) << 16;
    const int row = qd * 32 + lane;
    float m[32];
#pragma unroll
    for (int c = 0; c < 32; ++c) m[c] = -INFINITY;
    bool valid = false;
    if (smx) {
      {  // the ones operand (bf16 pairs) of the L MMA
        float ones[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) ones[c] = __uint_as_float(0x3F803F80u);
        if (half == 0) {
          tmem_st16(tmem + lq + COL_ONES, ones);
          tmem_wait_st();
        }
      }
      before_sync();
      sm_bar();
      valid = valid0;
    }
    bool ok = true;
    for (int i = 0; i < ntiles; ++i) {
      // gather tile i, pair by pair
      for (int mt = 0; mt < 4 && ok; ++mt) {
        if (i > 0) ok = __all_sync(0xffffffffu, bar_wait_or_abort(&sm.bar_empty[mt], (i - 1) & 1, abort));
        if (!ok) break;
#pragma unroll
        for (int k = 0; k < W_CHUNKS; ++k) {
          if (k < nown) {
            const int c = wt + W_THREADS * k;
            const int r = c >> 4, j = c & 15;
            const int sl = 2 * mt + (j >> 3), ch = j & 7;
            cp_async16(ks + static_cast<uint32_t>(sl * SLAB_KV + r * 128 + ((ch ^ (r & 7)) << 4)),
                       P.kv + static_cast<int64_t>(rr[k]) * D + sl * 64 + ch * 8, true);
          }
        }
        asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n" ::"r"(smem_u32(&sm.bar_full[mt]))
                     : "memory");
      }
      if (!ok) {
        if (lane == 0) set_abort(sm);
        if (!smx) break;
      }
      if (i + 1 < ntiles) load_rows(i + 1, rr);
      if (!smx) continue;

      // ---------------------------------------------------------- softmax of tile i (warps 4-11)
      if (ok) ok = __all_sync(0xffffffffu, bar_wait_or_abort(&sm.bar_s, i & 1, abort));
      float x[32];
      bool grow = false;
      if (ok) {
        after_sync();
        tmem_ld16(tmem + lq + COL_S + half * 32, x);
        tmem_ld16(tmem + lq + COL_S + half * 32 + 16, x + 16);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          x[c] = valid ? x[c] * P.scale_log2 : -INFINITY;
          grow |= x[c] > m[c] + RESCALE_THRESHOLD;
        }
      }
      // one block reduction in the common case; a second only when something is off
      if (sm_bar_or(grow || !ok)) {
        if (sm_bar_or(!ok)) {
          ok = false;
          if (lane == 0) set_abort(sm);
          break;
        }
        grow = true;
      }
      if (grow) {
        bool grow_any = false;
        // exact tile maximum per head, then m = max(m, tile max); O^T and L rescaled by 2^(m_old - m)
        sm.red[qd][half * 32 + lane] = warp_col_max32(x);
        sm_bar();
        // the rescale factors go to shared memory (every warp of a half writes the same values); m is
        // the same in every lane, so lane c updates head half * 32 + c and the warp shares the result
        float mo = 0.f;
#pragma unroll
        for (int c = 0; c < 32; ++c)
          if (c == lane) mo = m[c];
        {
          const int hh = half * 32 + lane;
          const float tm = fmaxf(fmaxf(sm.red[0][hh], sm.red[1][hh]), fmaxf(sm.red[2][hh], sm.red[3][hh]));
          const float mn = fmaxf(mo, tm);
          sm.alpha[hh] = (mo == -INFINITY) ? 0.f : exp2f(mo - mn);
          const bool any = __any_sync(0xffffffffu, (mn != mo) && (mo != -INFINITY));
#pragma unroll
          for (int c = 0; c < 32; ++c) m[c] = __shfl_sync(0xffffffffu, mn, c);
          grow_any = any;
        }
        sm_bar();  // red[] reuse; alpha[] written
        if (i > 0 && grow_any) {
          // the previous tile's O^T and L MMAs completed before this tile's S^T (one commit covers all)
#pragma unroll 1
          for (int mt = 0; mt < 4; ++mt) {
            float v[32];
            tmem_ld16(tmem + lq + COL_O + mt * HB + half * 32, v);
            tmem_ld16(tmem + lq + COL_O + mt * HB + half * 32 + 16, v + 16);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) v[c] *= sm.alpha[half * 32 + c];
            tmem_st16(tmem + lq + COL_O + mt * HB + half * 32, v);
            tmem_st16(tmem + lq + COL_O + mt * HB + half * 32 + 16, v + 16);
          }
          float v[32];
          tmem_ld16(tmem + lq + COL_L + half * 32, v);
          tmem_ld16(tmem + lq + COL_L + half * 32 + 16, v + 16);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) v[c] *= sm.alpha[half * 32 + c];
          tmem_st16(tmem + lq + COL_L + half * 32, v);
          tmem_st16(tmem + lq + COL_L + half * 32 + 16, v + 16);
          tmem_wait_st();
        }
      }
      // p = 2^(x - m) -> P^T row (bf16, swizzled), this thread's 32 heads = 4 chunks of 16 B
      {
        uint8_t* prow = sm.p + row * 128;
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          float pv[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int c = c4 * 8 + e;
            pv[e] = (m[c] == -INFINITY) ? 0.f : ex2_approx(x[c] - m[c]);
          }
          const uint4 u = make_uint4(pack_bf16x2(pv[0], pv[1]), pack_bf16x2(pv[2], pv[3]), pack_bf16x2(pv[4], pv[5]),
                                     pack_bf16x2(pv[6], pv[7]));
          *reinterpret_cast<uint4*>(prow + (((half * 4 + c4) ^ (row & 7)) << 4)) = u;
        }
      }
      fence_async_smem();
      before_sync();
      bar_arrive(&sm.bar_p);
      valid = row_valid(P, qi, (tbase + i + 1) * BN + row, L);
    }

    if (smx) {
      if (ok) {
        ok = __all_sync(0xffffffffu, bar_wait_or_abort(&sm.bar_fin, 0, abort));
        if (!ok && lane == 0) set_abort(sm);
      }
      ok = ok && !*abort;
      if (ok && P.splits > 1) {
        after_sync();
        // split partial: O unnormalised (relative to m), m and l per head, for the combine kernel;
        // part [s][splits][64][512] then [s][splits][64][2]
        const int64_t unit = qi * P.splits + split;
        float* po = P.part + unit * (HB * D);
        float* pml = P.part + P.s * P.splits * static_cast<int64_t>(HB * D) + unit * (HB * 2);
        if (ntiles > 0) {
#pragma unroll 1
          for (int mt = 0; mt < 4; ++mt) {
            const int d = mt * 128 + qd * 32 + lane;
            float v[32];
            tmem_ld16(tmem + lq + COL_O + mt * HB + half * 32, v);
            tmem_ld16(tmem + lq + COL_O + mt * HB + half * 32 + 16, v + 16);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) po[(half * 32 + c) * D + d] = v[c];
          }
          if (qd == 0) {
            // m and l of this half's 32 heads through shared memory (red[0], red[1]: free here)
            float l[32];
            tmem_ld16(tmem + lq + COL_L + half * 32, l);
            tmem_ld16(tmem + lq + COL_L + half * 32 + 16, l + 16);
            tmem_wait_ld();
            if (lane == 0) {
#pragma unroll
              for (int c = 0; c < 32; ++c) {
                sm.red[0][half * 32 + c] = m[c];
                sm.red[1][half * 32 + c] = l[c];
              }
            }
            __syncwarp();
            pml[(half * 32 + lane) * 2 + 0] = sm.red[0][half * 32 + lane];
            pml[(half * 32 + lane) * 2 + 1] = sm.red[1][half * 32 + lane];
          }
        } else {
          for (int c = 0; c < 32; ++c)
#pragma unroll 1
            for (int mt = 0; mt < 4; ++mt) po[(half * 32 + c) * D + mt * 128 + qd * 32 + lane] = 0.f;
          if (qd == 0) {
            pml[(half * 32 + lane) * 2 + 0] = -INFINITY;
            pml[(half * 32 + lane) * 2 + 1] = 0.f;
          }
        }
      } else if (ok) {
        after_sync();
        // epilogue: lane = dim (within the M-tile quadrant), 32 heads per thread. m and l are the
        // same in every lane, so lane c computes the normaliser of head half * 32 + c once and the
        // warp shares it (the exp and the division per head per lane took ~4.6 us)
        float inv[32];
        {
          float l[32];
          tmem_ld16(tmem + lq + COL_L + half * 32, l);
          tmem_ld16(tmem + lq + COL_L + half * 32 + 16, l + 16);
          tmem_wait_ld();
          float mm = 0.f, ll = 0.f;
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if (c == lane) {
              mm = m[c];
              ll = l[c];
            }
          const float mine = (mm == -INFINITY) ? __int_as_float(0x7fc00000)
                                               : 1.f / (ll + exp2f(P.sink[half * 32 + lane] * LOG2E - mm));
#pragma unroll
          for (int c = 0; c < 32; ++c) inv[c] = __shfl_sync(0xffffffffu, mine, c);
        }
        const bool rope = P.rope_freqs != nullptr;
        const int pos = rope ? P.positions[qi] : 0;
        const bool bf = P.out_dtype == DSV4_BF16;
#pragma unroll 1
        for (int mt = 0; mt < 4; ++mt) {
          const int d = mt * 128 + qd * 32 + lane;
          const bool do_rope = rope && d >= D - P.rope_dim;
          float cs = 1.f, sn = 0.f;
          if (do_rope) {
            const int f = (d - (D - P.rope_dim)) >> 1;
            if (P.rope_dim <= 64) {
              cs = sm.rope_c[f];
              sn = sm.rope_s[f];
            } else {
              rope_cos_sin(pos, P.rope_freqs[f], &cs, &sn);
            }
          }
          float v[32];
          tmem_ld16(tmem + lq + COL_O + mt * HB + half * 32, v);
          tmem_ld16(tmem + lq + COL_O + mt * HB + half * 32 + 16, v + 16);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            float xo = v[c] * inv[c];
            if (do_rope) {
              // the pair (d, d+1) sits in lanes (even, odd)
              const float other = __shfl_xor_sync(0xffffffffu, xo, 1);
              float y0, y1;
              if ((d & 1) == 0) {
                rotate_pair(xo, other, cs, sn, true, &y0, &y1);
                xo = y0;
              } else {
                rotate_pair(other, xo, cs, sn, true, &y0, &y1);
                xo = y1;
              }
            }
            const int64_t off = (qi * P.h + half * 32 + c) * D + d;
            if (bf)
              reinterpret_cast<__nv_bfloat16*>(P.out)[off] = __float2bfloat16_rn(xo);
            else
              reinterpret_cast<float*>(P.out)[off] = xo;
          }
        }
      }
    }
  }
  __syncthreads();
  if (*abort) {
    // drain (bounded): the MMA thread's last commit covers every MMA it issued; this thread's copies
    if (tid == 0) bar_wait(&sm.bar_fin, 0);
    asm volatile("cp.async.wait_all;\n" ::: "memory");
  }
  before_sync();
  __syncthreads();
  after_sync();
  if (warp == 0) tmem_dealloc<TMEM_COLS>(tmem);
}

DSV4_ERROR_READER(attn_tc)

}  // namespace tc
}  // namespace dsv4

using namespace dsv4;

// Internal entry used by dsv4_sparse_attn (64 heads, bf16 q); splits > 1 writes the partials that
// sparse_attn.cu's combine kernel merges.
int dsv4_sparse_attn_tc(const dsv4_sparse_attn_params* p, int splits, float* part, void* stream) {
  tc::Params P;
  P.splits = splits;
  P.part = part;
  P.q = reinterpret_cast<const __nv_bfloat16*>(p->q);
  P.idx = p->idx;
  P.sink = p->sink;
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
  DSV4_CHECK_ARG(p->n <= 0x7fffffffLL, "dsv4_sparse_attn: the tcgen05 kernel addresses at most 2^31 kv rows");
  DSV4_CHECK_ARG((reinterpret_cast<uintptr_t>(p->kv) & 15) == 0, "dsv4_sparse_attn: kv must be 16-byte aligned");
  P.kv = reinterpret_cast<const __nv_bfloat16*>(p->kv);
  const int smem = static_cast<int>(sizeof(tc::Smem)) + 1024;
  static PerDeviceOnce attr;
  DSV4_CUDA_CHECK(set_smem_once(attr, tc::attn_tc_kernel, smem));
  DSV4_CHECK_ARG(splits >= 1 && (splits == 1 || part != nullptr), "dsv4_sparse_attn: split partials need a workspace");
  tc::attn_tc_kernel<<<static_cast<unsigned>(p->s * splits), tc::THREADS, smem, as_stream(stream)>>>(P);
  DSV4_LAUNCH_CHECK("attn_tc_kernel");
  return DSV4_OK;
}
