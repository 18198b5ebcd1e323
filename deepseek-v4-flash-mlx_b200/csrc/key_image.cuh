// The scaled two-term fp16 split of indexer keys and queries, and the 64 KB shared-memory image of
// a 128-key tile that the tcgen05 filter reads (shared by the filter kernels, the image builders and
// the compressor decode step that appends keys to a decode cache's image).
//
// A row (a key, or one head of a query) is scaled by the power of two 2^s that brings its largest
// element into [2^14, 2^15), then x * 2^s = xh + xl + d with xh = rn16(x * 2^s),
// xl = rn16(x * 2^s - xh), |d| <= 2^-22 |x * 2^s|.
// Tile image: two slab groups (dims 0-63, 64-127), each [hi slab 16 KB | lo slab 16 KB], rows of
// 128 bytes (64 fp16), 16-byte chunk c of row r at chunk position c ^ (r % 8) (the 128-byte swizzle
// of a K-major tcgen05 operand).
#pragma once
#include <cuda_fp16.h>

#include <cstdint>

namespace dsv4 {
namespace itc {

constexpr int IMG_SLAB_K = 128 * 128;       // 16 KB: 128 keys x 64 fp16 dims
constexpr int IMG_GROUP = 2 * IMG_SLAB_K;   // 32 KB: hi + lo slab of one dim group
constexpr int IMG_TILE_BYTES = 2 * IMG_GROUP;  // 64 KB: one 128-key tile

// exponent s (|s| <= 100) with max_abs * 2^s in [2^14, 2^15); 0 for a zero row
__device__ __forceinline__ int row_shift(float max_abs) {
  if (!(max_abs > 0.f)) return 0;
  int adj = 0;
  if (max_abs < 0x1p-100f) {
    max_abs *= 0x1p64f;
    adj = 64;
  }
  const int e = static_cast<int>((__float_as_uint(max_abs) >> 23) & 0xff) - 127 - adj;  // floor(log2)
  const int s = 14 - e;
  return s < -100 ? -100 : (s > 100 ? 100 : s);
}
__device__ __forceinline__ float pow2(int s) { return __uint_as_float(static_cast<uint32_t>(s + 127) << 23); }

__device__ __forceinline__ uint32_t pack2h(__half a, __half b) {
  return static_cast<uint32_t>(__half_as_ushort(a)) | (static_cast<uint32_t>(__half_as_ushort(b)) << 16);
}
// 4 fp32 (already scaled) -> (hi, lo) as two 8-byte groups of 4 fp16
__device__ __forceinline__ void split4(float4 v, uint2* hi, uint2* lo) {
  const __half h0 = __float2half_rn(v.x), h1 = __float2half_rn(v.y);
  const __half h2 = __float2half_rn(v.z), h3 = __float2half_rn(v.w);
  const __half l0 = __float2half_rn(v.x - __half2float(h0));
  const __half l1 = __float2half_rn(v.y - __half2float(h1));
  const __half l2 = __float2half_rn(v.z - __half2float(h2));
  const __half l3 = __float2half_rn(v.w - __half2float(h3));
  *hi = make_uint2(pack2h(h0, h1), pack2h(h2, h3));
  *lo = make_uint2(pack2h(l0, l1), pack2h(l2, l3));
}
// 2 fp32 (already scaled) -> (hi, lo) as two 4-byte pairs of fp16, the same values split4 gives
__device__ __forceinline__ void split2(float x, float y, uint32_t* hi, uint32_t* lo) {
  const __half h0 = __float2half_rn(x), h1 = __float2half_rn(y);
  const __half l0 = __float2half_rn(x - __half2float(h0));
  const __half l1 = __float2half_rn(y - __half2float(h1));
  *hi = pack2h(h0, h1);
  *lo = pack2h(l0, l1);
}
__device__ __forceinline__ float4 scale4(float4 v, float f) {
  return make_float4(v.x * f, v.y * f, v.z * f, v.w * f);
}
__device__ __forceinline__ float amax4(float4 v) {
  return fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
}
// byte offset of float4 f (dims 4f..4f+3) of row r inside a tile image's slab group layout
__device__ __forceinline__ uint32_t key_off(int r, int f) {
  const int g = f >> 4, c = (f >> 1) & 7;
  return static_cast<uint32_t>(g * IMG_GROUP + r * 128 + ((c ^ (r & 7)) << 4) + (f & 1) * 8);
}

}  // namespace itc
}  // namespace dsv4
