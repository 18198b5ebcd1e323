// Gathered sparse MLA attention (ref_torch/sparse_attn.py:23-34) for B200.
//
// One CTA owns one query, a block of 64 heads and a contiguous range of its index list (a
// "split"). All heads share the gathered latent rows (MLA: K and V are the same 512-wide row),
// so the heads are the MMA M dimension. Per tile of 64 gathered rows:
//   gather   : cp.async 16-byte copies of the rows named by idx into a swizzled smem tile
//              (double buffered: the next tile's gather overlaps this tile's math)
//   S = Q K^T: bf16 mma.sync m16n8k16, fp32 accumulate (64 heads x 64 rows, K = 512)
//   softmax  : online (running max / sum per head, exp2 domain), masked rows are -inf
//   O += P V : P in bf16, V = the same smem tile read transposed (64 heads x 512 dims)
// A query whose list spans several CTAs writes an unnormalised partial (O, m, l) to the
// workspace and a combine kernel merges the partials; the sink enters only the denominator,
// exactly as the reference: o = sum p v / (sum p + exp(sink - m)).
#include <cstdlib>

#include "common.cuh"

namespace dsv4 {
namespace sa {

constexpr int D = 512;          // latent row (K and V)
constexpr int HB = 64;          // heads per CTA
constexpr int BN = 64;          // gathered rows per tile
constexpr int THREADS = 256;
constexpr int ROW_BYTES = D * 2;               // 1024
constexpr int Q_BYTES = HB * ROW_BYTES;        // 64 KB
constexpr int KV_BYTES = BN * ROW_BYTES;       // 64 KB
constexpr int P_BYTES = HB * BN * 2;           // 8 KB
constexpr float LOG2E = 1.4426950408889634f;
constexpr int IDX_CAP = 2048;                  // rows of a CTA's range preloaded into shared memory

struct Smem {
  alignas(128) uint8_t q[Q_BYTES];
  alignas(128) uint8_t kv[2][KV_BYTES];
  alignas(128) uint8_t p[P_BYTES];
  float red_max[4][HB];
  float red_sum[4][HB];
  float m_run[2][HB];
  float l_run[HB];
  float alpha[HB];
  int32_t rowidx[2][BN];
  int32_t rows[IDX_CAP];  // pool rows of this CTA's whole index range (loaded once)
};

// swizzled byte offset of 16-byte chunk `c` of row `r` in a tile whose rows are `row_chunks`
// chunks long (XOR of the low three chunk bits with the row keeps ldmatrix conflict-free).
__device__ __forceinline__ uint32_t swz(int r, int c, int row_bytes) {
  return static_cast<uint32_t>(r * row_bytes + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g, bool valid) {
  int sz = valid ? 16 : 0;  // 0 source bytes: the 16 destination bytes are zero-filled
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(saddr), "l"(g), "r"(sz));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float* c, uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

struct Params {
  const void* q;
  const __nv_bfloat16* kv;
  const float* sink;
  const void* idx;
  void* out;
  float* part;  // workspace partials [s][hblocks][splits][HB][D] then m,l [s][hblocks][splits][HB][2]
  int64_t s, n;
  int h, t, splits, hblocks;
  int q_dtype, idx_dtype, out_dtype;
  float scale_log2;  // scale * log2(e)
  const float* rope_freqs;
  const int32_t* positions;
  int rope_dim;
  const int64_t* win_base;  // implicit window (NULL: the list is idx alone)
  int win_stride, window, window_linear;
  int cluster;  // 1: the splits of a query are one thread-block cluster and merge through DSMEM
};

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
__device__ __forceinline__ uint32_t dsmem_addr(uint32_t a, int rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(a), "r"(rank));
  return r;
}
__device__ __forceinline__ float dsmem_f32(uint32_t a, int rank) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];\n" : "=f"(v) : "r"(dsmem_addr(a, rank)) : "memory");
  return v;
}
__device__ __forceinline__ float4 dsmem_f32x4(uint32_t a, int rank) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];\n"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(dsmem_addr(a, rank))
               : "memory");
  return v;
}

// logical list length of a query: implicit window rows followed by the explicit indices
__device__ __forceinline__ int list_len(const Params& P) { return (P.win_base ? P.window : 0) + P.t; }

// pool row of logical entry u of query qi (-1 = masked)
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

// whether tile `tile` reads explicit indices (written by the kernel launched before this one)
__device__ __forceinline__ bool tile_needs_idx(const Params& P, int tile) {
  return P.win_base == nullptr || (tile + 1) * 64 > P.window;
}

__device__ __forceinline__ int64_t load_idx(const void* idx, int64_t off, int dtype) {
  if (dtype == DSV4_I64) return __ldg(reinterpret_cast<const long long*>(idx) + off);
  return __ldg(reinterpret_cast<const int32_t*>(idx) + off);
}

// Issue the gather of tile rows [t0, t0+BN) of this query into kv buffer `buf`: every thread first
// loads the indices of the 16 rows it copies (independent loads, one round trip), then issues its
// 16-byte cp.async copies; rows past the list or masked (-1) are zero-filled and marked invalid.
__device__ __forceinline__ void gather_tile(const Params& P, Smem& sm, int buf, int64_t qi, int t0,
                                            int t_end, int range0, bool preloaded) {
  const int tid = threadIdx.x;
  constexpr int ROWS_PER_THREAD = BN / (THREADS / 64);  // 16
  const int chunk = tid & 63;                            // 64 chunks of 16 B per row
  const int r0 = tid >> 6;
  int32_t rows[ROWS_PER_THREAD];
#pragma unroll
  for (int i = 0; i < ROWS_PER_THREAD; ++i) {
    const int t = t0 + r0 + i * (THREADS / 64);
    if (preloaded) {
      const int32_t v = t < t_end ? sm.rows[t - range0] : -1;
      rows[i] = (v >= 0 && v < P.n) ? v : -1;  // every entry was checked at preload; kept as a guard
    } else {
      int64_t v = -1;
      if (t < t_end) v = list_row(P, qi, t);
      if (v >= P.n) {
        if (chunk == 0) raise_device_error(DSV4_ERR_INDEX_OUT_OF_RANGE);
        v = -1;
      }
      rows[i] = static_cast<int32_t>(v < 0 ? -1 : v);
    }
  }
  const uint32_t base = static_cast<uint32_t>(__cvta_generic_to_shared(sm.kv[buf]));
#pragma unroll
  for (int i = 0; i < ROWS_PER_THREAD; ++i) {
    const int rr = r0 + i * (THREADS / 64);
    const bool valid = rows[i] >= 0;
    const __nv_bfloat16* src = P.kv + static_cast<int64_t>(valid ? rows[i] : 0) * D + chunk * 8;
    cp_async16(base + swz(rr, chunk, ROW_BYTES), src, valid);
    if (chunk == 0) sm.rowidx[buf][rr] = rows[i];
  }
  cp_async_commit();
}

// Load the pool rows of logical entries [a, b) into sm.rows[u - base] (the CTA's range starts at
// `base`, a >= base, b - base <= IDX_CAP); out-of-range rows are recorded in the device error word
// and masked.
__device__ __forceinline__ void preload_rows(const Params& P, Smem& sm, int64_t qi, int base, int a, int b) {
  for (int u = a + threadIdx.x; u < b; u += THREADS) {
    int64_t v = list_row(P, qi, u);
    if (v >= P.n) {
      raise_device_error(DSV4_ERR_INDEX_OUT_OF_RANGE);
      v = -1;
    }
    sm.rows[u - base] = static_cast<int32_t>(v < 0 ? -1 : v);
  }
}

__global__ void __launch_bounds__(THREADS, 1) sparse_attn_kernel(Params P) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t qi = blockIdx.x / P.splits;
  const int split = static_cast<int>(blockIdx.x % P.splits), hblk = blockIdx.y;
  const int h0 = hblk * HB;
  const int heads_here = min(HB, P.h - h0);

  // index range of this split (in whole tiles) over the logical list [implicit window | idx]
  const int t_end = list_len(P);
  const int ntiles_all = (t_end + BN - 1) / BN;
  const int per = (ntiles_all + P.splits - 1) / P.splits;
  const int tile_begin = split * per;
  const int tile_end = min(ntiles_all, tile_begin + per);

  pdl_trigger();
  // Programmatic dependent launch: nothing before pdl_wait() writes global memory, and it reads only
  // q, the pool rows of the implicit window and positions, which no kernel in flight writes. Tiles
  // that read explicit indices (the previous kernel's output) wait first.
  bool waited = false;
  if (P.win_base == nullptr) {
    pdl_wait();
    waited = true;
  }
  // ---- stage Q (64 heads x 512) as bf16, swizzled ----
  const uint32_t qbase = static_cast<uint32_t>(__cvta_generic_to_shared(sm.q));
  if (P.q_dtype == DSV4_BF16) {
    const __nv_bfloat16* qg = reinterpret_cast<const __nv_bfloat16*>(P.q) + ((qi * P.h) + h0) * D;
#pragma unroll 4
    for (int c = tid; c < HB * 64; c += THREADS) {
      const int hh = c >> 6, ch = c & 63;
      const bool ok = hh < heads_here;
      cp_async16(qbase + swz(hh, ch, ROW_BYTES), qg + (ok ? hh * D + ch * 8 : 0), ok);
    }
    cp_async_commit();
  } else {
#pragma unroll 4
    for (int c = tid; c < HB * 64; c += THREADS) {
      const int hh = c >> 6, ch = c & 63;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (hh < heads_here) {
        const float4* f = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(P.q) +
                                                          ((qi * P.h) + h0 + hh) * D + ch * 8);
        const float4 x = __ldg(f), y = __ldg(f + 1);
        v = make_uint4(pack_bf16x2(x.x, x.y), pack_bf16x2(x.z, x.w), pack_bf16x2(y.x, y.y), pack_bf16x2(y.z, y.w));
      }
      asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};\n" ::"r"(qbase + swz(hh, ch, ROW_BYTES)), "r"(v.x),
                   "r"(v.y), "r"(v.z), "r"(v.w));
    }
  }
  if (tid < HB) {
    sm.m_run[0][tid] = -INFINITY;
    sm.m_run[1][tid] = -INFINITY;
    sm.l_run[tid] = 0.f;
  }

  float o[4][8][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 8; ++b)
#pragma unroll
      for (int c = 0; c < 4; ++c) o[a][b][c] = 0.f;

  // preload the pool rows of this CTA's whole range into shared memory (one round trip) so that
  // issuing a tile's gather never waits on global loads; window rows first (no dependency), the
  // explicit indices after the programmatic-dependency wait
  const int range0 = tile_begin * BN, range1 = min(t_end, tile_end * BN);
  const bool preloaded = range1 - range0 <= IDX_CAP;
  if (preloaded && range0 < range1) {
    const int wend = P.win_base ? min(range1, P.window) : range0;
    if (wend > range0) preload_rows(P, sm, qi, range0, range0, wend);
    if (range1 > wend) {
      if (!waited) {
        pdl_wait();
        waited = true;
      }
      preload_rows(P, sm, qi, range0, max(range0, wend), range1);
    }
    __syncthreads();
  }
  if (tile_begin < tile_end) {
    if (!waited && tile_needs_idx(P, tile_begin)) {
      pdl_wait();
      waited = true;
    }
    gather_tile(P, sm, 0, qi, tile_begin * BN, t_end, range0, preloaded);
  }

  const uint32_t q_s = static_cast<uint32_t>(__cvta_generic_to_shared(sm.q));
  const uint32_t p_s = static_cast<uint32_t>(__cvta_generic_to_shared(sm.p));
  // QK warp layout: heads [wm*32, +32), rows [wn*16, +16)
  const int wm = warp & 1, wn = warp >> 1;
  int cur = 0;

  for (int tile = tile_begin; tile < tile_end; ++tile) {
    const int buf = (tile - tile_begin) & 1;
    cp_async_wait<0>();
    __syncthreads();  // S1: tile `buf` landed; previous PV finished
    if (tile + 1 < tile_end) {
      if (!waited && tile_needs_idx(P, tile + 1)) {
        pdl_wait();
        waited = true;
      }
      gather_tile(P, sm, buf ^ 1, qi, (tile + 1) * BN, t_end, range0, preloaded);
    }
    const uint32_t kv_s = static_cast<uint32_t>(__cvta_generic_to_shared(sm.kv[buf]));

    // ---- S = Q K^T ----
    float s[2][2][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int c = 0; c < 4; ++c) s[a][b][c] = 0.f;
#pragma unroll 2
    for (int kc = 0; kc < D / 16; ++kc) {
      uint32_t a[2][4], b[4];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        int r = wm * 32 + mt * 16 + (lane & 15);
        int c = kc * 2 + (lane >> 4);
        ldsm_x4(q_s + swz(r, c, ROW_BYTES), a[mt][0], a[mt][1], a[mt][2], a[mt][3]);
      }
      {
        int r = wn * 16 + (lane & 7) + ((lane >> 4) << 3);
        int c = kc * 2 + ((lane >> 3) & 1);
        ldsm_x4(kv_s + swz(r, c, ROW_BYTES), b[0], b[1], b[2], b[3]);
      }
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        mma_bf16(s[mt][0], a[mt][0], a[mt][1], a[mt][2], a[mt][3], b[0], b[1]);
        mma_bf16(s[mt][1], a[mt][0], a[mt][1], a[mt][2], a[mt][3], b[2], b[3]);
      }
    }
    // scale to log2 domain, mask invalid rows, partial row max over this warp's 16 rows
    float pmax[2][2];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) pmax[mt][hf] = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        int row = wn * 16 + nt * 8 + (lane & 3) * 2 + j;
        bool valid = sm.rowidx[buf][row] >= 0;
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            float v = valid ? s[mt][nt][hf * 2 + j] * P.scale_log2 : -INFINITY;
            s[mt][nt][hf * 2 + j] = v;
            pmax[mt][hf] = fmaxf(pmax[mt][hf], v);
          }
        }
      }
    }
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        float v = pmax[mt][hf];
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
        if ((lane & 3) == 0) sm.red_max[wn][wm * 32 + mt * 16 + hf * 8 + (lane >> 2)] = v;
      }
    __syncthreads();  // S2

    // ---- p = exp2(s - m_new), partial sums, P -> smem (bf16) ----
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int hh = wm * 32 + mt * 16 + hf * 8 + (lane >> 2);
        float mnew = fmaxf(fmaxf(sm.red_max[0][hh], sm.red_max[1][hh]),
                           fmaxf(sm.red_max[2][hh], sm.red_max[3][hh]));
        mnew = fmaxf(mnew, sm.m_run[cur][hh]);
        const float msub = (mnew == -INFINITY) ? 0.f : mnew;
        float psum = 0.f;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          float p0 = exp2f(s[mt][nt][hf * 2 + 0] - msub);
          float p1 = exp2f(s[mt][nt][hf * 2 + 1] - msub);
          psum += p0 + p1;
          int row = wn * 16 + nt * 8 + (lane & 3) * 2;
          uint32_t addr = p_s + swz(hh, row >> 3, BN * 2) + (row & 7) * 2;
          asm volatile("st.shared.u32 [%0], %1;\n" ::"r"(addr), "r"(pack_bf16x2(p0, p1)));
        }
        psum += __shfl_xor_sync(0xffffffffu, psum, 1);
        psum += __shfl_xor_sync(0xffffffffu, psum, 2);
        if ((lane & 3) == 0) sm.red_sum[wn][hh] = psum;
      }
    }
    if (tid < HB) {
      float mold = sm.m_run[cur][tid];
      float mnew = fmaxf(fmaxf(sm.red_max[0][tid], sm.red_max[1][tid]),
                         fmaxf(sm.red_max[2][tid], sm.red_max[3][tid]));
      mnew = fmaxf(mnew, mold);
      sm.alpha[tid] = (mold == -INFINITY) ? 0.f : exp2f(mold - mnew);
      sm.m_run[cur ^ 1][tid] = mnew;
    }
    __syncthreads();  // S3
    if (tid < HB)
      sm.l_run[tid] = sm.l_run[tid] * sm.alpha[tid] +
                      ((sm.red_sum[0][tid] + sm.red_sum[1][tid]) + (sm.red_sum[2][tid] + sm.red_sum[3][tid]));

    // ---- O = O * alpha + P V  (warp owns dims [warp*64, +64), all 64 heads) ----
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
      float a0 = sm.alpha[mt * 16 + (lane >> 2)];
      float a1 = sm.alpha[mt * 16 + 8 + (lane >> 2)];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        o[mt][nt][0] *= a0;
        o[mt][nt][1] *= a0;
        o[mt][nt][2] *= a1;
        o[mt][nt][3] *= a1;
      }
    }
#pragma unroll 1
    for (int kc = 0; kc < BN / 16; ++kc) {
      uint32_t a[4][4];
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        int r = mt * 16 + (lane & 15);
        int c = kc * 2 + (lane >> 4);
        ldsm_x4(p_s + swz(r, c, BN * 2), a[mt][0], a[mt][1], a[mt][2], a[mt][3]);
      }
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // pairs of n8 tiles
        uint32_t b[4];
        int r = kc * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        int c = warp * 8 + np * 2 + (lane >> 4);
        ldsm_x4_t(kv_s + swz(r, c, ROW_BYTES), b[0], b[1], b[2], b[3]);
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
          mma_bf16(o[mt][np * 2 + 0], a[mt][0], a[mt][1], a[mt][2], a[mt][3], b[0], b[1]);
          mma_bf16(o[mt][np * 2 + 1], a[mt][0], a[mt][1], a[mt][2], a[mt][3], b[2], b[3]);
        }
      }
    }
    cur ^= 1;
  }
  __syncthreads();

  if (!waited) pdl_wait();  // global writes only after the previous kernel has completed
  // ---- epilogue: O (scaled for the final output) -> smem fp32 [64][OSTRIDE] over the kv buffers,
  // then one rolled, coalesced pass writes it out (inverse rope applied there)
  constexpr int OSTRIDE = D + 8;
  float* os = reinterpret_cast<float*>(sm.kv[0]);
  const bool final_out = P.splits == 1;
#pragma unroll
  for (int mt = 0; mt < 4; ++mt)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int hh = mt * 16 + hf * 8 + (lane >> 2);
      float inv = 1.f;
      if (final_out) {
        const float m = sm.m_run[cur][hh];
        inv = (m == -INFINITY) ? __int_as_float(0x7fc00000)  // no valid index: NaN like the reference
                               : 1.f / (sm.l_run[hh] + exp2f(P.sink[min(h0 + hh, P.h - 1)] * LOG2E - m));
      }
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int d = warp * 64 + nt * 8 + (lane & 3) * 2;
        *reinterpret_cast<float2*>(os + hh * OSTRIDE + d) =
            make_float2(o[mt][nt][hf * 2 + 0] * inv, o[mt][nt][hf * 2 + 1] * inv);
      }
    }
  __syncthreads();
  if (P.cluster) {
    // The query's splits are this cluster: each CTA parks (m, l) beside its unnormalised O, then
    // CTA `split` merges heads [split * nh, +nh) over all splits exactly as combine_kernel does
    // (weights by a warp with lane = split, the dims in split order) and writes them out.
    if (tid < HB) {
      sm.red_max[0][tid] = sm.m_run[cur][tid];
      sm.red_sum[0][tid] = sm.l_run[tid];
    }
    cluster_sync_all();
    const int nh = (HB + P.splits - 1) / P.splits;
    const int hb0 = split * nh, hb1 = min(min(HB, heads_here), hb0 + nh);
    float* wbuf = &sm.red_max[1][0];  // [nh][splits], at most 64 + splits floats
    const uint32_t m_s = static_cast<uint32_t>(__cvta_generic_to_shared(&sm.red_max[0][0]));
    const uint32_t l_s = static_cast<uint32_t>(__cvta_generic_to_shared(&sm.red_sum[0][0]));
    for (int j = warp; j < hb1 - hb0; j += THREADS / 32) {
      const int hh = hb0 + j;
      float m = -INFINITY, l = 0.f;
      if (lane < P.splits) {
        m = dsmem_f32(m_s + hh * 4, lane);
        l = dsmem_f32(l_s + hh * 4, lane);
      }
      const float M = warp_max(m);
      const float w = (m == -INFINITY) ? 0.f : exp2f(m - M);
      if (lane < P.splits) wbuf[j * P.splits + lane] = w;
      const float L = warp_sum(w * l);
      if (lane == 0)
        sm.alpha[hh] = (M == -INFINITY) ? __int_as_float(0x7fc00000) : 1.f / (L + exp2f(P.sink[h0 + hh] * LOG2E - M));
    }
    __syncthreads();
    const bool rope = P.rope_freqs != nullptr;
    const int pos = rope ? P.positions[qi] : 0;
    const uint32_t os_s = static_cast<uint32_t>(__cvta_generic_to_shared(os));
#pragma unroll 1
    for (int c = tid; c < (hb1 - hb0) * (D / 4); c += THREADS) {
      const int j = c / (D / 4), hh = hb0 + j, d = (c % (D / 4)) * 4;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int sp = 0; sp < P.splits; ++sp) {
        const float4 v = dsmem_f32x4(os_s + (hh * OSTRIDE + d) * 4, sp);
        const float w = wbuf[j * P.splits + sp];
        acc.x = fmaf(w, v.x, acc.x);
        acc.y = fmaf(w, v.y, acc.y);
        acc.z = fmaf(w, v.z, acc.z);
        acc.w = fmaf(w, v.w, acc.w);
      }
      const float inv = sm.alpha[hh];
      float4 v = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
      if (rope && d >= D - P.rope_dim) {
        const int f0 = (d - (D - P.rope_dim)) >> 1;
        float c0, s0, c1, s1;
        rope_cos_sin(pos, P.rope_freqs[f0], &c0, &s0);
        rope_cos_sin(pos, P.rope_freqs[f0 + 1], &c1, &s1);
        rotate_pair(v.x, v.y, c0, s0, true, &v.x, &v.y);
        rotate_pair(v.z, v.w, c1, s1, true, &v.z, &v.w);
      }
      const int64_t off = ((qi * P.h) + h0 + hh) * D + d;
      if (P.out_dtype == DSV4_BF16)
        *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(P.out) + off) =
            make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
      else
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(P.out) + off) = v;
    }
    cluster_sync_all();  // the peers keep their partials until every CTA of the cluster has read them
    return;
  }
  if (final_out) {
    const bool rope = P.rope_freqs != nullptr;
    const int pos = rope ? P.positions[qi] : 0;
#pragma unroll 1
    for (int c = tid; c < HB * (D / 4); c += THREADS) {
      const int hh = c / (D / 4), d = (c % (D / 4)) * 4;
      if (hh >= heads_here) continue;
      float4 v = *reinterpret_cast<const float4*>(os + hh * OSTRIDE + d);
      if (rope && d >= D - P.rope_dim) {
        const int f0 = (d - (D - P.rope_dim)) >> 1;
        float c0, s0, c1, s1;
        rope_cos_sin(pos, P.rope_freqs[f0], &c0, &s0);
        rope_cos_sin(pos, P.rope_freqs[f0 + 1], &c1, &s1);
        rotate_pair(v.x, v.y, c0, s0, true, &v.x, &v.y);
        rotate_pair(v.z, v.w, c1, s1, true, &v.z, &v.w);
      }
      const int64_t off = ((qi * P.h) + h0 + hh) * D + d;
      if (P.out_dtype == DSV4_BF16)
        *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(P.out) + off) =
            make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
      else
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(P.out) + off) = v;
    }
  } else {
    const int64_t unit = (qi * P.hblocks + hblk) * P.splits + split;
    float* po = P.part + unit * (HB * D);
    float* pml = P.part + (P.s * P.hblocks * P.splits) * (int64_t)(HB * D) + unit * (HB * 2);
#pragma unroll 1
    for (int c = tid; c < HB * (D / 4); c += THREADS) {
      const int hh = c / (D / 4), d = (c % (D / 4)) * 4;
      *reinterpret_cast<float4*>(po + hh * D + d) = *reinterpret_cast<const float4*>(os + hh * OSTRIDE + d);
    }
    if (tid < HB) {
      pml[tid * 2 + 0] = sm.m_run[cur][tid];
      pml[tid * 2 + 1] = sm.l_run[tid];
    }
  }
}

// Merge split partials: o = sum_s e^{m_s-M} O_s / (sum_s e^{m_s-M} l_s + e^{sink-M}).
// One CTA of 128 threads per (query, head): each thread merges 4 consecutive dims over all splits,
// with the split loop unrolled so the partial loads of different splits are in flight together.
__global__ void __launch_bounds__(128) combine_kernel(Params P) {
  pdl_trigger();
  pdl_wait();
  const int64_t unitq = blockIdx.x;             // qi * hblocks + hblk
  const int hh = blockIdx.y;
  const int64_t qi = unitq / P.hblocks;
  const int hblk = static_cast<int>(unitq % P.hblocks);
  const int h0 = hblk * HB;
  if (h0 + hh >= P.h) return;
  const int64_t unit0 = unitq * P.splits;
  const float* pml = P.part + (P.s * P.hblocks * P.splits) * (int64_t)(HB * D);
  __shared__ float s_w[64];
  __shared__ float s_inv;
  // the first splits' partials load while warp 0 works out the weights (the loads do not depend on
  // them); the sums below keep split order
  const int d = threadIdx.x * 4;
  const float* src = P.part + unit0 * (HB * D) + hh * D + d;
  const int npre = P.splits < 4 ? P.splits : 4;
  float4 pre[4];
#pragma unroll
  for (int u = 0; u < 4; ++u)  // (a repeat of the last split past npre: loaded, never used)
    pre[u] = *reinterpret_cast<const float4*>(src + static_cast<int64_t>(u < npre ? u : npre - 1) * (HB * D));
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    if (lane < P.splits) {
      m0 = pml[(unit0 + lane) * (HB * 2) + hh * 2];
      l0 = pml[(unit0 + lane) * (HB * 2) + hh * 2 + 1];
    }
    if (lane + 32 < P.splits) {
      m1 = pml[(unit0 + lane + 32) * (HB * 2) + hh * 2];
      l1 = pml[(unit0 + lane + 32) * (HB * 2) + hh * 2 + 1];
    }
    const float M = warp_max(fmaxf(m0, m1));
    const float w0 = (m0 == -INFINITY) ? 0.f : exp2f(m0 - M);
    const float w1 = (m1 == -INFINITY) ? 0.f : exp2f(m1 - M);
    if (lane < P.splits) s_w[lane] = w0;
    if (lane + 32 < P.splits) s_w[lane + 32] = w1;
    const float L = warp_sum(w0 * l0 + w1 * l1);
    if (lane == 0)
      s_inv = (M == -INFINITY) ? __int_as_float(0x7fc00000)
                               : 1.f / (L + exp2f(P.sink[h0 + hh] * LOG2E - M));
  }
  __syncthreads();
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int u = 0; u < 4; ++u)
    if (u < npre) {
      const float w = s_w[u];
      acc.x = fmaf(w, pre[u].x, acc.x);
      acc.y = fmaf(w, pre[u].y, acc.y);
      acc.z = fmaf(w, pre[u].z, acc.z);
      acc.w = fmaf(w, pre[u].w, acc.w);
    }
  int sp = npre;
  for (; sp + 4 <= P.splits; sp += 4) {
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = *reinterpret_cast<const float4*>(src + (int64_t)(sp + u) * (HB * D));
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float w = s_w[sp + u];
      acc.x = fmaf(w, v[u].x, acc.x);
      acc.y = fmaf(w, v[u].y, acc.y);
      acc.z = fmaf(w, v[u].z, acc.z);
      acc.w = fmaf(w, v[u].w, acc.w);
    }
  }
  for (; sp < P.splits; ++sp) {
    const float4 v = *reinterpret_cast<const float4*>(src + (int64_t)sp * (HB * D));
    const float w = s_w[sp];
    acc.x = fmaf(w, v.x, acc.x);
    acc.y = fmaf(w, v.y, acc.y);
    acc.z = fmaf(w, v.z, acc.z);
    acc.w = fmaf(w, v.w, acc.w);
  }
  const float inv = s_inv;
  float o[4] = {acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv};
  if (P.rope_freqs != nullptr && d >= D - P.rope_dim) {
    const int pos = P.positions[qi];
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      float c, sn;
      rope_cos_sin(pos, P.rope_freqs[(d + e - (D - P.rope_dim)) >> 1], &c, &sn);
      rotate_pair(o[e], o[e + 1], c, sn, true, &o[e], &o[e + 1]);
    }
  }
  const int64_t off = ((qi * P.h) + h0 + hh) * D + d;
  if (P.out_dtype == DSV4_BF16) {
    *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(P.out) + off) =
        make_uint2(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]));
  } else {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(P.out) + off) = make_float4(o[0], o[1], o[2], o[3]);
  }
}

static int choose_splits(const dsv4_sparse_attn_params* p) {
  if (p->num_splits > 0) return p->num_splits;
  const int hblocks = (p->h + HB - 1) / HB;
  const int len = (p->win_base ? p->window : 0) + p->t;
  const int ntiles = (len + BN - 1) / BN;
  const int64_t units = p->s * hblocks;
  const int sms = num_sms();
  if (units >= sms || ntiles <= 1) return 1;
  // one CTA per SM (the kernel's shared memory allows no more): as many splits as fit in one wave
  int want = static_cast<int>(sms / units);
  if (want < 1) want = 1;
  if (want > ntiles) want = ntiles;
  if (want > 64) want = 64;
  int per = (ntiles + want - 1) / want;
  return (ntiles + per - 1) / per;
}

}  // namespace sa
DSV4_ERROR_READER(sparse_attn)

}  // namespace dsv4

using namespace dsv4;

int dsv4_sparse_attn_tc(const dsv4_sparse_attn_params* p, int splits, float* part, void* stream);
int dsv4_sparse_attn_hg(const dsv4_sparse_attn_params* p, int splits, void* stream);
int dsv4_hg_splits(const dsv4_sparse_attn_params* p);
bool dsv4_hg_cluster_fits(int splits);

// tcgen05 kernel: 64 heads, bf16 q (or the fused prologue, which writes bf16 q), 128-row tiles,
// one CTA per (query, split). The plan (kernel and split count) is made in one place, for the
// workspace size and for the launch.
static bool tc_shape_ok(const dsv4_sparse_attn_params* p) {
  return p->h == sa::HB && (p->q_dtype == DSV4_BF16 || p->q_norm_rope);
}
struct AttnPlan {
  bool tc;
  int splits;
  bool cluster;  // mma.sync kernel: the splits of a query merge inside a cluster (no partials in HBM)
  bool hg;       // the head-group decode kernel (16 heads per CTA, row splits merged in a cluster)
};

// whether `splits` CTAs of the mma.sync kernel (one per SM by shared memory) can run as one cluster
// on this GPU; asked once per size
static bool cluster_fits(int splits) {
  // per device ordinal (the attributes set here are per device): 0 unknown, 1 yes, -1 no
  static std::atomic<int> known[64][17];
  if (splits < 2 || splits > 16) return false;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    (void)cudaGetLastError();
    return false;
  }
  const int k = known[dev][splits].load(std::memory_order_relaxed);
  if (k != 0) return k > 0;
  const int smem = static_cast<int>(sizeof(sa::Smem));
  bool ok = cudaFuncSetAttribute(sa::sparse_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) ==
            cudaSuccess;
  if (ok && splits > 8)
    ok = cudaFuncSetAttribute(sa::sparse_attn_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
         cudaSuccess;
  int nclusters = 0;
  if (ok) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(splits, 1, 1);
    cfg.blockDim = dim3(sa::THREADS);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ok = cudaOccupancyMaxActiveClusters(&nclusters, sa::sparse_attn_kernel, &cfg) == cudaSuccess && nclusters > 0;
  }
  (void)cudaGetLastError();  // a refused query leaves no sticky error
  known[dev][splits].store(ok ? 1 : -1, std::memory_order_relaxed);
  return ok;
}
static int tc_splits(const dsv4_sparse_attn_params* p) {
  const int len = (p->win_base ? p->window : 0) + p->t;
  const int tiles = (len + 127) / 128;
  if (tiles <= 1) return 1;
  int want;
  if (p->num_splits > 0) {
    want = p->num_splits;
  } else {
    const int sms = num_sms();
    if (p->s >= sms) return 1;
    want = static_cast<int>(sms / p->s);  // one CTA per SM: as many splits as fit in one wave
  }
  if (want > tiles) want = tiles;
  if (want > 64) want = 64;
  if (want < 1) want = 1;
  const int per = (tiles + want - 1) / want;
  return (tiles + per - 1) / per;
}
// Automatic: tcgen05 from 16 queries per call (measured on B200: config 3, 64 decode queries, 39 us
// against 45 us for the mma.sync kernel; config 2, one query, 18 us against 14 us).
constexpr int64_t TC_MIN_QUERIES = 16;
static AttnPlan plan_attention(const dsv4_sparse_attn_params* p) {
  const bool tc = p->kernel == 2 || (p->kernel == 0 && tc_shape_ok(p) && p->s >= TC_MIN_QUERIES);
  if (tc && tc_shape_ok(p)) return {true, tc_splits(p), false, false};
  // decode-sized calls: the head-group kernel, when its row splits fit in one cluster
  if (p->kernel == 3 || (p->kernel == 0 && p->s < TC_MIN_QUERIES)) {
    const int sp = dsv4_hg_splits(p);
    if (dsv4_hg_cluster_fits(sp)) return {false, sp, sp > 1, true};
  }
  const int sp = sa::choose_splits(p);
  return {false, sp, sp > 1 && cluster_fits(sp), false};
}

// workspace: [split partials (O, m, l)] [bf16 q after the fused norm/rope pre-pass]
static size_t partial_bytes(const dsv4_sparse_attn_params* p) {
  const AttnPlan pl = plan_attention(p);
  const int splits = pl.splits;
  if (splits <= 1 || pl.cluster || pl.hg) return 0;
  const int hblocks = (p->h + sa::HB - 1) / sa::HB;
  const int64_t units = p->s * hblocks * splits;
  return static_cast<size_t>(units) * (sa::HB * sa::D + sa::HB * 2) * sizeof(float);
}

extern "C" size_t dsv4_sparse_attn_workspace_size(const dsv4_sparse_attn_params* p) {
  if (!p || p->s <= 0 || p->h <= 0 || (p->t <= 0 && p->win_base == nullptr)) return 0;
  size_t bytes = (partial_bytes(p) + 255) / 256 * 256;
  if (p->q_norm_rope && !plan_attention(p).hg) bytes += static_cast<size_t>(p->s) * p->h * p->d * 2;
  return bytes;
}

extern "C" int dsv4_sparse_attn(const dsv4_sparse_attn_params* p, void* stream) {
  DSV4_CHECK_ARG(p != nullptr, "dsv4_sparse_attn: params is NULL");
  DSV4_CHECK_ARG(p->q && p->kv && p->sink && p->idx && p->out, "dsv4_sparse_attn: NULL tensor");
  DSV4_CHECK_ARG(p->d == sa::D, "dsv4_sparse_attn: head dim %d unsupported (512 only)", p->d);
  DSV4_CHECK_ARG(p->h > 0 && p->h % 16 == 0, "dsv4_sparse_attn: heads %d must be a positive multiple of 16", p->h);
  DSV4_CHECK_ARG(p->s >= 0 && (p->t > 0 || p->win_base != nullptr) && p->t >= 0 && p->n > 0,
                 "dsv4_sparse_attn: bad sizes s=%lld t=%d n=%lld",
                 (long long)p->s, p->t, (long long)p->n);
  DSV4_CHECK_DTYPE(p->q_dtype == DSV4_F32 || p->q_dtype == DSV4_BF16, "dsv4_sparse_attn: q dtype");
  DSV4_CHECK_DTYPE(p->idx_dtype == DSV4_I32 || p->idx_dtype == DSV4_I64, "dsv4_sparse_attn: idx dtype");
  DSV4_CHECK_DTYPE(p->out_dtype == DSV4_F32 || p->out_dtype == DSV4_BF16, "dsv4_sparse_attn: out dtype");
  DSV4_CHECK_ARG(p->rope_freqs == nullptr || (p->positions != nullptr && p->rope_dim > 0 &&
                                               p->rope_dim <= 64 && p->rope_dim % 2 == 0),
                 "dsv4_sparse_attn: inverse rope needs positions and 0 < rope_dim <= 64");
  DSV4_CHECK_ARG(p->win_base == nullptr || (p->positions != nullptr && p->window > 0 && p->window % sa::BN == 0),
                 "dsv4_sparse_attn: the implicit window needs positions and a window that is a multiple of 64");
  DSV4_CHECK_ARG(!p->q_norm_rope || p->rope_freqs != nullptr,
                 "dsv4_sparse_attn: the fused q norm/rope needs rope_freqs, positions and rope_dim");
  DSV4_CHECK_ARG(p->s * 64 < (int64_t)INT32_MAX, "dsv4_sparse_attn: too many queries per call");
  DSV4_CHECK_ARG(p->kernel >= 0 && p->kernel <= 3 && (p->kernel != 2 || tc_shape_ok(p)),
                 "dsv4_sparse_attn: kernel %d unavailable for h=%d q_dtype=%d", p->kernel, p->h, p->q_dtype);
  if (p->s == 0) return DSV4_OK;
  sa::Params P;
  P.q = p->q;
  P.kv = reinterpret_cast<const __nv_bfloat16*>(p->kv);
  P.sink = p->sink;
  P.idx = p->idx;
  P.out = p->out;
  P.s = p->s;
  P.n = p->n;
  P.h = p->h;
  P.t = p->t;
  P.hblocks = (p->h + sa::HB - 1) / sa::HB;
  const AttnPlan plan = plan_attention(p);
  P.splits = plan.splits;
  P.cluster = plan.cluster ? 1 : 0;
  P.q_dtype = p->q_dtype;
  P.idx_dtype = p->idx_dtype;
  P.out_dtype = p->out_dtype;
  P.scale_log2 = p->scale * sa::LOG2E;
  P.rope_freqs = p->rope_freqs;
  P.positions = p->positions;
  P.rope_dim = p->rope_dim;
  P.win_base = p->win_base;
  P.win_stride = p->win_stride;
  P.window = p->win_base ? p->window : 0;
  P.window_linear = p->window_linear;
  P.part = nullptr;
  const size_t need = dsv4_sparse_attn_workspace_size(p);
  if (need > 0 && (p->workspace == nullptr || p->workspace_bytes < need)) {
    set_error("dsv4_sparse_attn: workspace of %zu bytes needed, %zu given", need, p->workspace_bytes);
    return DSV4_ERR_WORKSPACE;
  }
  if (plan.hg) return dsv4_sparse_attn_hg(p, plan.splits, stream);  // q prologue fused in the kernel
  if (P.splits > 1 && !P.cluster) P.part = reinterpret_cast<float*>(p->workspace);
  if (p->q_norm_rope) {
    // weightless per-head norm + rope of q into bf16 scratch, then attention reads it
    void* qn = static_cast<char*>(p->workspace) + (partial_bytes(p) + 255) / 256 * 256;
    dsv4_norm_rope_params n = {};
    n.x = p->q;
    n.weight = nullptr;
    n.out = qn;
    n.rows = p->s;
    n.heads = p->h;
    n.dim = p->d;
    n.rope_dim = p->rope_dim;
    n.x_dtype = p->q_dtype;
    n.w_dtype = DSV4_F32;
    n.out_dtype = DSV4_BF16;
    n.eps = p->q_eps;
    n.freqs = p->rope_freqs;
    n.positions = p->positions;
    const int st = dsv4_norm_rope(&n, stream);
    if (st != DSV4_OK) return st;
    P.q = qn;
    P.q_dtype = DSV4_BF16;
  }
  if (plan.tc) {
    dsv4_sparse_attn_params pt = *p;
    pt.q = P.q;
    pt.q_dtype = DSV4_BF16;
    const int st = dsv4_sparse_attn_tc(&pt, P.splits, P.part, stream);
    if (st != DSV4_OK || P.splits == 1) return st;
    dim3 g2(static_cast<unsigned>(P.s * P.hblocks), sa::HB);
    DSV4_CUDA_CHECK(launch_pdl(sa::combine_kernel, g2, dim3(128), 0, as_stream(stream), P));
    return DSV4_OK;
  }
  static PerDeviceOnce attr_set;
  const int smem = static_cast<int>(sizeof(sa::Smem));
  DSV4_CUDA_CHECK(set_smem_once(attr_set, sa::sparse_attn_kernel, smem));
  dim3 grid(static_cast<unsigned>(P.s * P.splits), P.hblocks);
  if (P.cluster) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(sa::THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = as_stream(stream);
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;  // the splits of one query
    attr[1].val.clusterDim.x = P.splits;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    DSV4_CUDA_CHECK(cudaLaunchKernelEx(&cfg, sa::sparse_attn_kernel, P));
    return DSV4_OK;
  }
  DSV4_CUDA_CHECK(launch_pdl(sa::sparse_attn_kernel, grid, dim3(sa::THREADS), smem, as_stream(stream), P));
  if (P.splits > 1) {
    dim3 g2(static_cast<unsigned>(P.s * P.hblocks), sa::HB);
    DSV4_CUDA_CHECK(launch_pdl(sa::combine_kernel, g2, dim3(128), 0, as_stream(stream), P));
  }
  return DSV4_OK;
}
