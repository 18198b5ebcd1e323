// Inline-PTX helpers for the 5th-generation tensor cores (tcgen05 + tensor memory), mbarriers and
// bulk copies, shared by the tcgen05 kernels of this library.
//
// Shared-memory operands are 128-byte-swizzled slabs: rows of 128 bytes, 16-byte chunk c of row r
// stored at chunk position c ^ (r % 8), slabs 1024-byte aligned. K-major operands advance their
// start address by 32 bytes per 16-element k-step inside a slab; MN-major operands use the leading
// byte offset as the stride between 64-element MN blocks and the stride byte offset (1024) between
// groups of 8 K rows.
#pragma once
#include <cstdint>

namespace dsv4 {
namespace tc5 {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 64-bit shared-memory matrix descriptor: start, leading / stride byte offsets, version 1 (sm_100),
// layout 2 = 128-byte swizzle
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFF) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | (2ull << 61);
}

// instruction descriptor, kind::f16: fp32 accumulate, bf16 A and B, shape M x N
template <int M, int N>
__host__ __device__ constexpr uint32_t idesc_bf16(bool a_mn_major, bool b_mn_major) {
  static_assert(M == 64 || M == 128, "M");
  static_assert(N % 16 == 0 && N >= 16 && N <= 256, "N");
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         ((static_cast<uint32_t>(N) >> 3) << 17) | ((static_cast<uint32_t>(M) >> 4) << 24);
}

// instruction descriptor, kind::f16: fp32 accumulate, fp16 A and B, shape M x N
template <int M, int N>
__host__ __device__ constexpr uint32_t idesc_f16(bool a_mn_major, bool b_mn_major) {
  static_assert(M == 64 || M == 128, "M");
  static_assert(N % 16 == 0 && N >= 16 && N <= 256, "N");
  return (1u << 4) | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         ((static_cast<uint32_t>(N) >> 3) << 17) | ((static_cast<uint32_t>(M) >> 4) << 24);
}

// D (fp32, tensor memory) (+)= A . B^T for 16-bit A, B of the kind given by the descriptor
__device__ __forceinline__ void mma16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(id), "r"(acc));
}
// arrive on `bar` once every tcgen05 operation this thread issued before has completed
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void bar_init(uint64_t* bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void bar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }
__device__ __forceinline__ void bar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void bar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}
constexpr uint64_t WAIT_NS = 1000000000ull;  // 1 s: a wait longer than this is an error

__device__ __forceinline__ bool bar_try(uint32_t a, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(a), "r"(parity)
      : "memory");
  return done != 0;
}
// wait for the phase with the given parity, bounded by WAIT_NS of wall time; false on timeout
__device__ __forceinline__ bool bar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  if (bar_try(a, parity)) return true;
  const uint64_t t0 = global_ns();
  while (true) {
    if (bar_try(a, parity)) return true;
    if (global_ns() - t0 > WAIT_NS) return false;
  }
}
// as bar_wait, but also gives up as soon as *abort (set by another thread) is nonzero
__device__ __forceinline__ bool bar_wait_or_abort(uint64_t* bar, uint32_t parity, const volatile int* abort) {
  const uint32_t a = smem_u32(bar);
  if (bar_try(a, parity)) return true;
  const uint64_t t0 = global_ns();
  while (true) {
    if (bar_try(a, parity)) return true;
    if (*abort) return false;
    if (global_ns() - t0 > WAIT_NS) return false;
  }
}

// bulk copy global -> this CTA's shared memory only, completion counted in bytes on `bar`;
// both addresses 16-byte aligned, bytes a multiple of 16
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 2-D tiled tensor copy (TMA) of the box at element coordinates (x inner, y outer) of the tensor map
// into this CTA's shared memory, completion counted in bytes on `bar`; x * element size must be a
// multiple of 16 bytes, and `tmap` the generic address of a __grid_constant__ CUtensorMap
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_map(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
__device__ __forceinline__ void before_sync() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void after_sync() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

template <int COLS>
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(dst_smem)),
               "r"(COLS)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
template <int COLS>
__device__ __forceinline__ void tmem_dealloc(uint32_t base) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(base), "r"(COLS) : "memory");
}

// 16 consecutive fp32 columns of this thread's lane
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g, bool valid) {
  int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(saddr), "l"(g), "r"(sz));
}

// byte offset of 16-byte chunk c of row r in a slab-major, 128-byte-swizzled tile: slab = c / 8
// (64 bf16 or 32 fp32 elements), row r at 128 B, chunk (c % 8) XOR (r % 8)
__device__ __forceinline__ uint32_t slab_off(int r, int c, int slab_bytes) {
  return static_cast<uint32_t>((c >> 3) * slab_bytes + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

}  // namespace tc5
}  // namespace dsv4
