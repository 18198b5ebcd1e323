// Small-batch decode attention (ref_torch/sparse_attn.py:23-34 with the decode q chain of
// oracle/v4_fast.py:88-89, 118-119) for B200: head groups x row splits, merged in a cluster.
//
// A decode call has few queries (batch 1 in the latency-bound case), so the work of one query is
// spread over many SMs two ways at once:
//   * heads: 16 per CTA (the MMA M dimension), h / 16 head groups;
//   * rows: the query's list [window | selected] in 64-row tiles, split over up to 16 CTAs.
// The row splits of one (query, head group) run as one thread-block cluster and merge their
// unnormalised partials (O, m, l) through distributed shared memory: each split finalises a slice of
// the 16 x 512 outputs, reading every split's partial of it (and their m, l) in one round of peer loads.
//
// Per CTA: q of its 16 heads is staged as bf16 (with the fused prologue: the weightless per-head
// RMS norm and the RoPE of the last rope_dim dims, in the arithmetic of the norm_rope kernel), the
// gathered rows arrive by 16-byte cp.async (double-buffered tiles), S = Q K^T and O += P V run on
// bf16 mma.sync m16n8k16 with fp32 accumulation, the softmax is online in the exp2 domain. The
// sink enters only the denominator and an all-masked query yields NaN, as in the reference.
//
// Programmatic dependent launch: by default the kernel waits for the previous kernel before it
// reads any global memory. With pre_wait (the decode step: scores, selection, attention, where the
// score kernel waits for all earlier work before the other two launch) it stages q and computes the
// window tiles while the selection runs, and waits only before it reads the selected indices.
#include "common.cuh"

namespace dsv4 {
namespace hg {

constexpr int D = 512;
constexpr int HG = 16;          // heads per CTA
constexpr int BN = 64;          // gathered rows per tile
constexpr int THREADS = 256;    // 8 warps
constexpr int ROW_BYTES = D * 2;
constexpr int MAX_SPLITS = 16;
constexpr int OSTRIDE = D + 4;  // fp32 partial O row stride in shared memory
constexpr float LOG2E = 1.4426950408889634f;

struct Smem {
  alignas(128) uint8_t q[HG * ROW_BYTES];         // 16 KB, swizzled
  alignas(128) uint8_t kv[2][BN * ROW_BYTES];     // 2 x 64 KB, swizzled; reused for the partial O
  alignas(128) uint8_t p[HG * BN * 2];            // 2 KB
  float red_max[THREADS / 32][HG];
  float red_sum[THREADS / 32][HG];
  float m_run[HG];
  float l_run[HG];
  float alpha[HG];
  float inv[HG];
  float rope_c[32], rope_s[32];  // cos / sin of the query position times each rope pair's frequency
  int32_t rowidx[2][BN];
  float2 ml[HG];                 // (m, l) per head, read by the cluster merge
};
static_assert(sizeof(float) * HG * OSTRIDE <= 2 * BN * ROW_BYTES, "partial O fits in the kv buffers");

struct Params {
  const void* q;
  const __nv_bfloat16* kv;
  const float* sink;
  const void* idx;
  void* out;
  int64_t s, n;
  int h, t, splits;
  int q_dtype, idx_dtype, out_dtype;
  float scale_log2;
  const float* rope_freqs;
  const int32_t* positions;
  int rope_dim;
  int q_norm_rope;
  float q_eps;
  const int64_t* win_base;
  int win_stride, window, window_linear;
  int pre_wait;
};

__device__ __forceinline__ uint32_t swz(int r, int c, int row_bytes) {
  return static_cast<uint32_t>(r * row_bytes + ((c ^ (r & 7)) << 4));
}
__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g, bool valid) {
  const int sz = valid ? 16 : 0;  // 0 source bytes: the 16 destination bytes are zero-filled
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(saddr), "l"(g), "r"(sz));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
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
__device__ __forceinline__ float2 dsmem_f32x2(uint32_t a, int rank) {
  float2 v;
  asm volatile("ld.shared::cluster.v2.f32 {%0,%1}, [%2];\n" : "=f"(v.x), "=f"(v.y) : "r"(dsmem_addr(a, rank)) : "memory");
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

__device__ __forceinline__ int list_len(const Params& P) { return (P.win_base ? P.window : 0) + P.t; }

// whether tile `tile` holds explicit indices (written by the kernel launched before this one)
__device__ __forceinline__ bool tile_needs_idx(const Params& P, int tile) {
  return P.win_base == nullptr || (tile + 1) * BN > P.window;
}

// pool row of logical entry u of query qi (-1 = masked): implicit window rows, then idx
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

// pool rows of list entries [t0, t0 + BN) into sm.rowidx[buf]: thread r < 64 takes entry t0 + r
// (-1 masked; an index past the pool is recorded in the device error word and masked)
__device__ __forceinline__ void load_rows(const Params& P, Smem& sm, int buf, int64_t qi, int t0, int t_end) {
  const int r = threadIdx.x;
  if (r < BN) {
    const int t = t0 + r;
    int64_t v = t < t_end ? list_row(P, qi, t) : -1;
    if (v >= P.n) {
      raise_device_error(DSV4_ERR_INDEX_OUT_OF_RANGE);
      v = -1;
    }
    sm.rowidx[buf][r] = static_cast<int32_t>(v < 0 ? -1 : v);
  }
}

// the gather of buffer `buf` (its rows in sm.rowidx[buf], after a barrier): thread = (16-byte chunk,
// 16 rows); masked rows are zero-filled
__device__ __forceinline__ void issue_tile(const Params& P, Smem& sm, int buf) {
  const int tid = threadIdx.x;
  const int chunk = tid & 63, r0 = tid >> 6;
  const uint32_t base = static_cast<uint32_t>(__cvta_generic_to_shared(sm.kv[buf]));
#pragma unroll
  for (int i = 0; i < BN / (THREADS / 64); ++i) {
    const int rr = r0 + i * (THREADS / 64);
    const int32_t row = sm.rowidx[buf][rr];
    const bool valid = row >= 0;
    cp_async16(base + swz(rr, chunk, ROW_BYTES), P.kv + static_cast<int64_t>(valid ? row : 0) * D + chunk * 8,
               valid);
  }
  cp_async_commit();
}

constexpr int QPER = D / 32;               // q dims per lane
constexpr int QHPW = HG / (THREADS / 32);  // q heads per warp

// q of heads [h0, h0 + 16) of query qi. bf16 q goes straight to sm.q by cp.async (its own commit
// group), each warp copying the two heads it later finishes; fp32 q is loaded into registers.
__device__ __forceinline__ void load_q(const Params& P, Smem& sm, int64_t qi, int h0, float (&v)[QHPW][QPER]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (P.q_dtype == DSV4_BF16) {
    const uint32_t qbase = static_cast<uint32_t>(__cvta_generic_to_shared(sm.q));
#pragma unroll
    for (int j = 0; j < QHPW; ++j) {
      const int hh = warp * QHPW + j;
      const __nv_bfloat16* qg = reinterpret_cast<const __nv_bfloat16*>(P.q) + (qi * P.h + h0 + hh) * D;
#pragma unroll
      for (int c = lane; c < 64; c += 32) cp_async16(qbase + swz(hh, c, ROW_BYTES), qg + c * 8, true);
    }
    cp_async_commit();
    return;
  }
#pragma unroll
  for (int j = 0; j < QHPW; ++j) {
    const float* x = reinterpret_cast<const float*>(P.q) + (qi * P.h + h0 + warp * QHPW + j) * D + lane * QPER;
#pragma unroll
    for (int e = 0; e < QPER; e += 4) {
      const float4 f = *reinterpret_cast<const float4*>(x + e);
      v[j][e] = f.x;
      v[j][e + 1] = f.y;
      v[j][e + 2] = f.z;
      v[j][e + 3] = f.w;
    }
  }
}

// the rest of q's staging (after the barrier that publishes the RoPE table, with the bf16 copy's
// group complete): with the fused prologue the weightless per-head RMS norm (lane-sequential fmaf
// sum of squares, the warp butterfly, x * rsqrt(ss / 512 + eps)) and the RoPE of the last rope_dim
// dims, in the norm_rope kernel's arithmetic, so both give the same bf16 q; the bf16 rows then
// (over)write sm.q, each warp its own two heads
__device__ __forceinline__ void finish_q(const Params& P, Smem& sm, float (&v)[QHPW][QPER]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (!P.q_norm_rope && P.q_dtype == DSV4_BF16) return;  // staged as it is
  const uint32_t qbase = static_cast<uint32_t>(__cvta_generic_to_shared(sm.q));
  if (P.q_dtype == DSV4_BF16) {  // this warp's copies have landed (wait_group + syncwarp by the caller)
#pragma unroll
    for (int j = 0; j < QHPW; ++j) {
      const int hh = warp * QHPW + j;
#pragma unroll
      for (int e = 0; e < QPER; e += 8) {
        uint32_t r0, r1, r2, r3;
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                     : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                     : "r"(qbase + swz(hh, (lane * QPER + e) >> 3, ROW_BYTES)));
        const uint32_t w[4] = {r0, r1, r2, r3};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          v[j][e + 2 * k] = __uint_as_float(w[k] << 16);
          v[j][e + 2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
        }
      }
    }
    __syncwarp();  // every lane has read its chunks before any lane overwrites them
  }
  const int rope_lo = D - P.rope_dim;
#pragma unroll
  for (int j = 0; j < QHPW; ++j) {
    if (P.q_norm_rope) {
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < QPER; ++e) ss = fmaf(v[j][e], v[j][e], ss);
      ss = warp_sum(ss);
      const float r = rsqrtf(ss / static_cast<float>(D) + P.q_eps);
#pragma unroll
      for (int e = 0; e < QPER; ++e) v[j][e] = v[j][e] * r;
      if (lane * QPER + QPER > rope_lo) {
#pragma unroll
        for (int e = 0; e < QPER; e += 2) {
          const int d = lane * QPER + e;
          if (d >= rope_lo) {
            const int f = (d - rope_lo) >> 1;
            rotate_pair(v[j][e], v[j][e + 1], sm.rope_c[f], sm.rope_s[f], false, &v[j][e], &v[j][e + 1]);
          }
        }
      }
    }
    const int hh = warp * QHPW + j;
#pragma unroll
    for (int e = 0; e < QPER; e += 8) {
      const int ch = (lane * QPER + e) >> 3;
      asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};\n" ::"r"(qbase + swz(hh, ch, ROW_BYTES)),
                   "r"(pack_bf16x2(v[j][e], v[j][e + 1])), "r"(pack_bf16x2(v[j][e + 2], v[j][e + 3])),
                   "r"(pack_bf16x2(v[j][e + 4], v[j][e + 5])), "r"(pack_bf16x2(v[j][e + 6], v[j][e + 7])));
    }
  }
}

// final value of output element (head hh, dims d..d+3), after the normalisation: inverse RoPE on
// the rope dims (angles from the shared table), then the store. Warp-collective (every lane calls
// it; `valid` marks the lanes that hold an element): for a bf16 output the even lane of a pair
// holding dims d and d + 4 of one head (d a multiple of 8) stores both as one 16-byte write, which
// halves the writes that cross the bus when the output is pinned host memory.
__device__ __forceinline__ void write_out(const Params& P, const Smem& sm, int64_t qi, int h0, int hh, int d,
                                          float4 v, bool valid) {
  if (valid && P.rope_freqs != nullptr && d >= D - P.rope_dim) {
    const int f0 = (d - (D - P.rope_dim)) >> 1;
    rotate_pair(v.x, v.y, sm.rope_c[f0], sm.rope_s[f0], true, &v.x, &v.y);
    rotate_pair(v.z, v.w, sm.rope_c[f0 + 1], sm.rope_s[f0 + 1], true, &v.z, &v.w);
  }
  const int64_t off = (qi * P.h + h0 + hh) * D + d;
  if (P.out_dtype == DSV4_BF16) {
    const uint32_t a = pack_bf16x2(v.x, v.y), b = pack_bf16x2(v.z, v.w);
    const uint32_t pa = __shfl_xor_sync(0xffffffffu, a, 1), pb = __shfl_xor_sync(0xffffffffu, b, 1);
    const bool pv = __shfl_xor_sync(0xffffffffu, valid ? 1 : 0, 1) != 0;
    const bool even = (threadIdx.x & 1) == 0;
    const bool pair = valid && pv && (d & 7) == (even ? 0 : 4) && (reinterpret_cast<uintptr_t>(P.out) & 15) == 0;
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(P.out) + off;
    if (pair) {
      if (even) *reinterpret_cast<uint4*>(o) = make_uint4(a, b, pa, pb);
    } else if (valid) {
      *reinterpret_cast<uint2*>(o) = make_uint2(a, b);
    }
  } else if (valid) {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(P.out) + off) = v;
  }
}

// grid (splits, h / 16, s); cluster (splits, 1, 1) when splits > 1
__global__ void __launch_bounds__(THREADS, 1) decode_attn_kernel(Params P) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int split = blockIdx.x;
  const int h0 = blockIdx.y * HG;
  const int64_t qi = blockIdx.z;

  const int t_end = list_len(P);
  const int ntiles = (t_end + BN - 1) / BN;
  const int per = (ntiles + P.splits - 1) / P.splits;
  const int tile_begin = min(ntiles, split * per);
  const int tile_end = min(ntiles, tile_begin + per);

  pdl_trigger();
  // Without pre_wait every read follows the wait. With it (the caller's guarantee that only idx can
  // still be in flight), q, the RoPE angles and the window rows are read while the kernel before this
  // one finishes, and a CTA whose tiles are all window rows computes them too; reading idx waits first.
  bool waited = false;
  if (!P.pre_wait) {
    pdl_wait();
    waited = true;
  }
  float qv[QHPW][QPER];
  load_q(P, sm, qi, h0, qv);
  if (warp == 2 && P.rope_freqs != nullptr && lane < P.rope_dim / 2)  // angles of the rope pairs
    rope_cos_sin(P.positions[qi], P.rope_freqs[lane], &sm.rope_c[lane], &sm.rope_s[lane]);
  const bool first_idx = tile_begin < tile_end && tile_needs_idx(P, tile_begin);
  if (tile_begin < tile_end && !first_idx) load_rows(P, sm, 0, qi, tile_begin * BN, t_end);  // window rows
  if (tid < HG) {
    sm.m_run[tid] = -INFINITY;
    sm.l_run[tid] = 0.f;
  }
  __syncthreads();  // the RoPE table (and a window tile's rows) are in shared memory
  // q's norm and RoPE before the tile's copies are issued: shared-memory accesses queued behind a
  // tile's worth of copies would wait for them
  cp_async_wait<0>();  // the bf16 q copies (this warp's heads)
  __syncwarp();
  finish_q(P, sm, qv);
  if (first_idx) {  // rows from idx: after the dependency wait
    if (!waited) {
      pdl_wait();
      waited = true;
    }
    load_rows(P, sm, 0, qi, tile_begin * BN, t_end);
    __syncthreads();
  }
  if (tile_begin < tile_end) issue_tile(P, sm, 0);
  float o[8][4];
#pragma unroll
  for (int a = 0; a < 8; ++a)
#pragma unroll
    for (int c = 0; c < 4; ++c) o[a][c] = 0.f;

  const uint32_t q_s = static_cast<uint32_t>(__cvta_generic_to_shared(sm.q));
  const uint32_t p_s = static_cast<uint32_t>(__cvta_generic_to_shared(sm.p));
  const int hA = lane >> 2, hB = hA + 8;
  for (int tile = tile_begin; tile < tile_end; ++tile) {
    const int buf = (tile - tile_begin) & 1;
    cp_async_wait<0>();
    __syncthreads();  // tile `buf` (and q) landed; the previous tile's PV is done with buffer buf ^ 1
    const bool has_next = tile + 1 < tile_end;
    if (has_next) {  // the next tile's rows now; its copies after the next barrier
      if (!waited && tile_needs_idx(P, tile + 1)) {
        pdl_wait();
        waited = true;
      }
      load_rows(P, sm, buf ^ 1, qi, (tile + 1) * BN, t_end);
    }
    const uint32_t kv_s = static_cast<uint32_t>(__cvta_generic_to_shared(sm.kv[buf]));

    // ---- S = Q K^T: warp w takes gathered rows [8w, 8w + 8), all 16 heads, K = 512; four
    // accumulators (k steps mod 4) keep four independent MMA chains in flight ----
    float sacc[4][4] = {};
#pragma unroll 2
    for (int kc = 0; kc < D / 16; kc += 4) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int k0 = kc + 2 * half;
        uint32_t b[4], a0[4], a1[4];
        ldsm_x4(kv_s + swz(warp * 8 + (lane & 7), k0 * 2 + (lane >> 3), ROW_BYTES), b[0], b[1], b[2], b[3]);
        ldsm_x4(q_s + swz(lane & 15, k0 * 2 + (lane >> 4), ROW_BYTES), a0[0], a0[1], a0[2], a0[3]);
        ldsm_x4(q_s + swz(lane & 15, k0 * 2 + 2 + (lane >> 4), ROW_BYTES), a1[0], a1[1], a1[2], a1[3]);
        mma_bf16(sacc[2 * half], a0[0], a0[1], a0[2], a0[3], b[0], b[1]);
        mma_bf16(sacc[2 * half + 1], a1[0], a1[1], a1[2], a1[3], b[2], b[3]);
      }
    }
    float s[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) s[c] = (sacc[0][c] + sacc[1][c]) + (sacc[2][c] + sacc[3][c]);
    // s[0..1]: head lane/4, rows 8w + 2(lane%4) + {0,1}; s[2..3]: head lane/4 + 8
    const int rbase = warp * 8 + (lane & 3) * 2;
    const bool v0 = sm.rowidx[buf][rbase] >= 0, v1 = sm.rowidx[buf][rbase + 1] >= 0;
    s[0] = v0 ? s[0] * P.scale_log2 : -INFINITY;
    s[1] = v1 ? s[1] * P.scale_log2 : -INFINITY;
    s[2] = v0 ? s[2] * P.scale_log2 : -INFINITY;
    s[3] = v1 ? s[3] * P.scale_log2 : -INFINITY;
    float mx0 = fmaxf(s[0], s[1]), mx1 = fmaxf(s[2], s[3]);
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    if ((lane & 3) == 0) {
      sm.red_max[warp][hA] = mx0;
      sm.red_max[warp][hB] = mx1;
    }
    __syncthreads();
    if (has_next) issue_tile(P, sm, buf ^ 1);
    float mA = sm.m_run[hA], mB = sm.m_run[hB];
#pragma unroll
    for (int w = 0; w < THREADS / 32; ++w) {
      mA = fmaxf(mA, sm.red_max[w][hA]);
      mB = fmaxf(mB, sm.red_max[w][hB]);
    }
    const float subA = mA == -INFINITY ? 0.f : mA, subB = mB == -INFINITY ? 0.f : mB;
    const float p0 = exp2f(s[0] - subA), p1 = exp2f(s[1] - subA);
    const float p2 = exp2f(s[2] - subB), p3 = exp2f(s[3] - subB);
    asm volatile("st.shared.u32 [%0], %1;\n" ::"r"(p_s + swz(hA, rbase >> 3, BN * 2) + (rbase & 7) * 2),
                 "r"(pack_bf16x2(p0, p1)));
    asm volatile("st.shared.u32 [%0], %1;\n" ::"r"(p_s + swz(hB, rbase >> 3, BN * 2) + (rbase & 7) * 2),
                 "r"(pack_bf16x2(p2, p3)));
    float sA = p0 + p1, sB = p2 + p3;
    sA += __shfl_xor_sync(0xffffffffu, sA, 1);
    sA += __shfl_xor_sync(0xffffffffu, sA, 2);
    sB += __shfl_xor_sync(0xffffffffu, sB, 1);
    sB += __shfl_xor_sync(0xffffffffu, sB, 2);
    if ((lane & 3) == 0) {
      sm.red_sum[warp][hA] = sA;
      sm.red_sum[warp][hB] = sB;
    }
    __syncthreads();  // P and the partial sums are in shared memory; every thread has read m_run
    if (tid < HG) {
      const float mold = sm.m_run[tid];
      float mnew = mold;
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < THREADS / 32; ++w) {
        mnew = fmaxf(mnew, sm.red_max[w][tid]);
        sum += sm.red_sum[w][tid];
      }
      const float alpha = mold == -INFINITY ? 0.f : exp2f(mold - mnew);
      sm.alpha[tid] = alpha;
      sm.l_run[tid] = sm.l_run[tid] * alpha + sum;
      sm.m_run[tid] = mnew;
    }
    __syncthreads();
    // ---- O = O * alpha + P V: warp w owns dims [64w, 64w + 64), all 16 heads, K = 64 rows ----
    const float aA = sm.alpha[hA], aB = sm.alpha[hB];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      o[nt][0] *= aA;
      o[nt][1] *= aA;
      o[nt][2] *= aB;
      o[nt][3] *= aB;
    }
#pragma unroll
    for (int kc = 0; kc < BN / 16; ++kc) {
      uint32_t a[4];
      ldsm_x4(p_s + swz(lane & 15, kc * 2 + (lane >> 4), BN * 2), a[0], a[1], a[2], a[3]);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b[4];
        ldsm_x4_t(kv_s + swz(kc * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), warp * 8 + np * 2 + (lane >> 4),
                             ROW_BYTES),
                  b[0], b[1], b[2], b[3]);
        mma_bf16(o[np * 2 + 0], a[0], a[1], a[2], a[3], b[0], b[1]);
        mma_bf16(o[np * 2 + 1], a[0], a[1], a[2], a[3], b[2], b[3]);
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();  // every warp is done with the kv buffers: they hold the partial O from here
  if (!waited) pdl_wait();  // global writes only once the kernel before has completed

  // ---- partial O (unnormalised) -> shared memory fp32 [16][OSTRIDE], (m, l) per head ----
  float* os = reinterpret_cast<float*>(sm.kv[0]);
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    const int d = warp * 64 + nt * 8 + (lane & 3) * 2;
    *reinterpret_cast<float2*>(os + hA * OSTRIDE + d) = make_float2(o[nt][0], o[nt][1]);
    *reinterpret_cast<float2*>(os + hB * OSTRIDE + d) = make_float2(o[nt][2], o[nt][3]);
  }
  if (tid < HG) sm.ml[tid] = make_float2(sm.m_run[tid], sm.l_run[tid]);
  const int S = P.splits;
  if (S == 1) {
    if (tid < HG) {
      const float m = sm.m_run[tid];
      sm.inv[tid] = m == -INFINITY ? __int_as_float(0x7fc00000)  // no valid row: NaN, as the reference
                                   : 1.f / (sm.l_run[tid] + exp2f(P.sink[h0 + tid] * LOG2E - m));
    }
    __syncthreads();
#pragma unroll 2
    for (int c = tid; c < HG * (D / 4); c += THREADS) {
      const int hh = c / (D / 4), d = (c % (D / 4)) * 4;
      const float4 a = *reinterpret_cast<const float4*>(os + hh * OSTRIDE + d);
      const float iv = sm.inv[hh];
      write_out(P, sm, qi, h0, hh, d, make_float4(a.x * iv, a.y * iv, a.z * iv, a.w * iv), true);
    }
    return;
  }
  // ---- cluster merge: this CTA's slice of the 16 x 512 outputs; the weights of the slice's heads
  // (w_s = e^(m_s - M), 1 / (sum_s w_s l_s + e^(sink - M))) first, then every thread requests, in one
  // round of peer loads, the splits' partials of its four outputs and weighs them ----
  cluster_sync_all();  // every split's partial O, m and l are in its shared memory
  const uint32_t os_s = static_cast<uint32_t>(__cvta_generic_to_shared(os));
  const uint32_t ml_s = static_cast<uint32_t>(__cvta_generic_to_shared(&sm.ml[0]));
  constexpr int NF4 = HG * (D / 4);  // 2048 float4 outputs per (query, head group)
  const int chunk = ((NF4 + S - 1) / S + 1) & ~1;  // even: a slice starts on a 16-byte store pair
  const int f0 = min(NF4, split * chunk), f1 = min(NF4, f0 + chunk);
  // the splits' weights w_s = e^(m_s - M) and the normaliser of each head of this slice, once per
  // (head, split) (a half-warp per head, lane = split) instead of per output; the products are summed
  // in split order as before. The P buffer is free from here.
  constexpr int MAXH = 12;  // heads a slice touches: chunk / 128 + 2 <= 10
  float* wbuf = reinterpret_cast<float*>(sm.p);  // [MAXH][MAX_SPLITS]
  float* ivbuf = wbuf + MAXH * MAX_SPLITS;
  static_assert((MAXH * MAX_SPLITS + MAXH) * 4 <= sizeof(sm.p), "merge weights fit the P buffer");
  const int hlo = f0 / (D / 4);
  const int nhs = f1 > f0 ? (f1 - 1) / (D / 4) - hlo + 1 : 0;
  if (tid < (nhs * MAX_SPLITS + 31) / 32 * 32) {  // whole warps
    const int hl = tid / MAX_SPLITS, sp = tid % MAX_SPLITS;
    float2 ml = make_float2(-INFINITY, 0.f);
    if (hl < nhs && sp < S) ml = dsmem_f32x2(ml_s + (hlo + hl) * 8, sp);
    float M = ml.x;
#pragma unroll
    for (int o = MAX_SPLITS / 2; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o, MAX_SPLITS));
    const float w = ml.x == -INFINITY ? 0.f : exp2f(ml.x - M);
    float L = 0.f;
#pragma unroll
    for (int s2 = 0; s2 < MAX_SPLITS; ++s2) {
      const float ws = __shfl_sync(0xffffffffu, w, s2, MAX_SPLITS);
      const float ls = __shfl_sync(0xffffffffu, ml.y, s2, MAX_SPLITS);
      if (s2 < S) L = fmaf(ws, ls, L);
    }
    if (hl < nhs) {
      if (sp < S) wbuf[hl * MAX_SPLITS + sp] = w;
      if (sp == 0)
        ivbuf[hl] = M == -INFINITY ? __int_as_float(0x7fc00000)
                                   : 1.f / (L + exp2f(P.sink[h0 + hlo + hl] * LOG2E - M));
    }
  }
  __syncthreads();
  for (int fb = f0 + warp * 32; fb < f1; fb += THREADS) {  // warp-uniform: write_out is collective
    const int f = fb + lane;
    const bool valid = f < f1;
    const int hh = valid ? f / (D / 4) : hlo, d = valid ? (f % (D / 4)) * 4 : 0;
    const float* wh = wbuf + (hh - hlo) * MAX_SPLITS;
    float4 v[MAX_SPLITS];
#pragma unroll
    for (int sp = 0; sp < MAX_SPLITS; ++sp)
      if (sp < S) v[sp] = valid ? dsmem_f32x4(os_s + (hh * OSTRIDE + d) * 4, sp) : make_float4(0.f, 0.f, 0.f, 0.f);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int sp = 0; sp < MAX_SPLITS; ++sp)
      if (sp < S) {
        const float w = wh[sp];
        acc.x = fmaf(w, v[sp].x, acc.x);
        acc.y = fmaf(w, v[sp].y, acc.y);
        acc.z = fmaf(w, v[sp].z, acc.z);
        acc.w = fmaf(w, v[sp].w, acc.w);
      }
    const float iv = ivbuf[hh - hlo];
    write_out(P, sm, qi, h0, hh, d, make_float4(acc.x * iv, acc.y * iv, acc.z * iv, acc.w * iv), valid);
  }
  cluster_sync_all();  // the peers keep their partials until every CTA of the cluster has read them
}

}  // namespace hg
DSV4_ERROR_READER(decode_attn)
}  // namespace dsv4

using namespace dsv4;

// whether `splits` CTAs of the kernel (one per SM by shared memory) can run as one cluster on the
// current device; asked once per (device, size)
bool dsv4_hg_cluster_fits(int splits) {
  static std::atomic<int> known[64][hg::MAX_SPLITS + 1];
  if (splits < 2) return true;
  if (splits > hg::MAX_SPLITS) return false;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    (void)cudaGetLastError();
    return false;
  }
  const int k = known[dev][splits].load(std::memory_order_relaxed);
  if (k != 0) return k > 0;
  const int smem = static_cast<int>(sizeof(hg::Smem));
  bool ok = cudaFuncSetAttribute(hg::decode_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) ==
            cudaSuccess;
  if (ok && splits > 8)
    ok = cudaFuncSetAttribute(hg::decode_attn_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
         cudaSuccess;
  int nclusters = 0;
  if (ok) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(splits, 1, 1);
    cfg.blockDim = dim3(hg::THREADS);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ok = cudaOccupancyMaxActiveClusters(&nclusters, hg::decode_attn_kernel, &cfg) == cudaSuccess && nclusters > 0;
  }
  (void)cudaGetLastError();
  known[dev][splits].store(ok ? 1 : -1, std::memory_order_relaxed);
  return ok;
}

// row splits of the kernel: 64-row tiles per split rounded so that no split is empty
int dsv4_hg_splits(const dsv4_sparse_attn_params* p) {
  const int len = (p->win_base ? p->window : 0) + p->t;
  const int tiles = (len + hg::BN - 1) / hg::BN;
  if (tiles <= 1) return 1;
  int want = p->num_splits;
  if (want <= 0) {
    const int64_t units = p->s * (p->h / hg::HG);
    want = units >= num_sms() ? 1 : static_cast<int>(num_sms() / units);
  }
  if (want > tiles) want = tiles;
  if (want > hg::MAX_SPLITS) want = hg::MAX_SPLITS;
  if (want < 1) want = 1;
  const int per = (tiles + want - 1) / want;
  return (tiles + per - 1) / per;
}

// launch of the head-group kernel; the caller (dsv4_sparse_attn) has validated the parameters
int dsv4_sparse_attn_hg(const dsv4_sparse_attn_params* p, int splits, void* stream) {
  hg::Params P;
  P.q = p->q;
  P.kv = reinterpret_cast<const __nv_bfloat16*>(p->kv);
  P.sink = p->sink;
  P.idx = p->idx;
  P.out = p->out;
  P.s = p->s;
  P.n = p->n;
  P.h = p->h;
  P.t = p->t;
  P.splits = splits;
  P.q_dtype = p->q_dtype;
  P.idx_dtype = p->idx_dtype;
  P.out_dtype = p->out_dtype;
  P.scale_log2 = p->scale * hg::LOG2E;
  P.rope_freqs = p->rope_freqs;
  P.positions = p->positions;
  P.rope_dim = p->rope_dim;
  P.q_norm_rope = p->q_norm_rope;
  P.q_eps = p->q_eps;
  P.win_base = p->win_base;
  P.win_stride = p->win_stride;
  P.window = p->win_base ? p->window : 0;
  P.window_linear = p->window_linear;
  P.pre_wait = p->pre_wait;
  static PerDeviceOnce attr;
  const int smem = static_cast<int>(sizeof(hg::Smem));
  DSV4_CUDA_CHECK(set_smem_once(attr, hg::decode_attn_kernel, smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(splits, p->h / hg::HG, static_cast<unsigned>(p->s));
  cfg.blockDim = dim3(hg::THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[0].val.programmaticStreamSerializationAllowed = 1;
  attrs[1].id = cudaLaunchAttributeClusterDimension;
  attrs[1].val.clusterDim.x = splits;
  attrs[1].val.clusterDim.y = 1;
  attrs[1].val.clusterDim.z = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = splits > 1 ? 2 : 1;
  DSV4_CUDA_CHECK(cudaLaunchKernelEx(&cfg, hg::decode_attn_kernel, P));
  return DSV4_OK;
}
