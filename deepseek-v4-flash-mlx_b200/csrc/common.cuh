// Shared helpers for the dsv4 sm_100a kernels: status plumbing, dtype access, bf16 packing.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <string>
#include <utility>

#include "dsv4.h"

namespace dsv4 {

// Thread-local message behind dsv4_last_error().
void set_error(const char* fmt, ...);
void clear_error();

// Device error word: kernels record the first failure here (index out of range, wait timeout);
// dsv4_device_error() reads and clears it. Each translation unit has its own word (no
// relocatable device code); DSV4_ERROR_READER registers a reader of that word with the library.
static __device__ int g_device_error = 0;

__device__ __forceinline__ void raise_device_error(int code) { atomicCAS(&g_device_error, 0, code); }

typedef cudaError_t (*error_reader_fn)(int*);
int register_error_reader(error_reader_fn fn);
cudaError_t read_all_error_words(int* first);

#define DSV4_ERROR_READER(tag)                                                       \
  static cudaError_t dsv4_read_error_##tag(int* out) {                               \
    int v = 0, z = 0;                                                                \
    cudaError_t e = cudaMemcpyFromSymbol(&v, ::dsv4::g_device_error, sizeof(int));   \
    if (e != cudaSuccess) return e;                                                  \
    e = cudaMemcpyToSymbol(::dsv4::g_device_error, &z, sizeof(int));                 \
    *out = v;                                                                        \
    return e;                                                                        \
  }                                                                                  \
  static int dsv4_error_reader_reg_##tag = ::dsv4::register_error_reader(dsv4_read_error_##tag);

#define DSV4_CHECK_ARG(cond, ...)                 \
  do {                                            \
    if (!(cond)) {                                \
      ::dsv4::set_error(__VA_ARGS__);             \
      return DSV4_ERR_INVALID_ARGUMENT;           \
    }                                             \
  } while (0)

#define DSV4_CHECK_DTYPE(cond, ...)               \
  do {                                            \
    if (!(cond)) {                                \
      ::dsv4::set_error(__VA_ARGS__);             \
      return DSV4_ERR_UNSUPPORTED_DTYPE;          \
    }                                             \
  } while (0)

// After a launch: turn a launch failure into DSV4_ERR_CUDA with the kernel name.
#define DSV4_LAUNCH_CHECK(name)                                                     \
  do {                                                                              \
    cudaError_t e_ = cudaGetLastError();                                            \
    if (e_ != cudaSuccess) {                                                        \
      ::dsv4::set_error("%s: launch failed: %s", name, cudaGetErrorString(e_));     \
      return DSV4_ERR_CUDA;                                                         \
    }                                                                               \
  } while (0)

#define DSV4_CUDA_CHECK(expr)                                                            \
  do {                                                                                   \
    cudaError_t e_ = (expr);                                                             \
    if (e_ != cudaSuccess) {                                                             \
      ::dsv4::set_error("%s: %s (%s:%d)", #expr, cudaGetErrorString(e_), __FILE__, __LINE__); \
      return DSV4_ERR_CUDA;                                                              \
    }                                                                                    \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// SM count of the current device (looked up once per device ordinal below 64)
inline int num_sms() {
  static std::atomic<int> cached[64];
  int dev = 0;
  cudaGetDevice(&dev);
  const bool slot = dev >= 0 && dev < 64;
  int n = slot ? cached[dev].load(std::memory_order_relaxed) : 0;
  if (n <= 0) {
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
    if (slot) cached[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// Kernel attributes set with cudaFuncSetAttribute belong to the current device, so a process that
// drives several GPUs must set them on each one. A `PerDeviceOnce` runs its setter once per device
// ordinal (below 64; other ordinals on every call) and remembers only a success.
class PerDeviceOnce {
 public:
  template <typename F>
  cudaError_t operator()(F&& set) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = (dev >= 0 && dev < 64) ? (uint64_t{1} << dev) : 0;
    if (bit != 0 && (done_.load(std::memory_order_acquire) & bit) != 0) return cudaSuccess;
    e = set();
    if (e == cudaSuccess && bit != 0) done_.fetch_or(bit, std::memory_order_acq_rel);
    return e;
  }

 private:
  std::atomic<uint64_t> done_{0};
};

// a kernel's dynamic shared-memory limit, set once per device through `once`
template <typename K>
inline cudaError_t set_smem_once(PerDeviceOnce& once, K kernel, int bytes) {
  return once([&] { return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes); });
}

// a kernel's preferred shared-memory carveout (percent of the unified L1 / shared array), once per
// device through `once`
template <typename K>
inline cudaError_t set_carveout_once(PerDeviceOnce& once, K kernel, int percent) {
  return once([&] { return cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, percent); });
}

// ---- element access by runtime dtype ------------------------------------------------------
__device__ __forceinline__ float load_as_float(const void* p, int64_t i, int dtype) {
  if (dtype == DSV4_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}
__device__ __forceinline__ void store_from_float(void* p, int64_t i, int dtype, float v) {
  if (dtype == DSV4_BF16)
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<float*>(p)[i] = v;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Programmatic dependent launch: every kernel of the path is launched with the PDL attribute and
// calls pdl_wait() before touching global memory, so stream order is kept while the launch and
// prologue of a kernel overlap the tail of the one before it; pdl_trigger() lets the next kernel
// be scheduled as soon as this grid's CTAs are all running.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// fp8-e4m3 round trip of y = x * 2^-e (nearest even, saturating at 448), times 2^e: exact in fp32
// and in bf16, since e4m3 keeps 4 significant bits
__device__ __forceinline__ float fp8_round_pow2(float x, int e) {
  const float y = fminf(fmaxf(x * __uint_as_float(static_cast<uint32_t>(127 - e) << 23), -448.f), 448.f);
  const __half_raw h = __nv_cvt_fp8_to_halfraw(__nv_cvt_float_to_fp8(y, __NV_SATFINITE, __NV_E4M3), __NV_E4M3);
  return __half2float(__half(h)) * __uint_as_float(static_cast<uint32_t>(127 + e) << 23);
}
// the act-quant block scale exponent: ceil(log2(max(amax, 1e-4) / 448)), from the bits of the
// (correctly rounded) fp32 quotient
__device__ __forceinline__ int act_quant_exp(float amax) {
  const uint32_t b = __float_as_uint(fmaxf(amax, 1e-4f) / 448.f);
  return static_cast<int>((b >> 23) & 0xff) - 127 + ((b & 0x7fffff) != 0 ? 1 : 0);
}

// nearest fp4-e2m1 value (ties to the even mantissa) of y, |y| <= 6: the format holds 0, 0.5, 1,
// 1.5, 2, 3, 4, 6, i.e. spacing 0.5 below 2, 1 in [2, 4) and 2 in [4, 6]; every step is exact
__device__ __forceinline__ float e2m1_round(float y) {
  const float a = fabsf(y);
  const float q = a < 2.f ? rintf(2.f * a) * 0.5f : (a < 4.f ? rintf(a) : 2.f * rintf(0.5f * a));
  return copysignf(q, y);
}
// the fp4 block scale exponent: ceil(log2(max(amax, 6 * 2^-126) / 6)), from the bits of the
// (correctly rounded) fp32 quotient; in [-126, 126] for finite amax
__device__ __forceinline__ int fp4_exp(float amax) {
  const uint32_t b = __float_as_uint(fmaxf(amax, __uint_as_float(0x01C00000u)) / 6.f);
  return static_cast<int>((b >> 23) & 0xff) - 127 + ((b & 0x7fffff) != 0 ? 1 : 0);
}

// rope angle as the reference forms it: fp32 product of the position and the frequency
// (torch.outer in fp32, ref_torch/norm_rope.py:48-50), then cos/sin of that fp32 angle.
__device__ __forceinline__ void rope_cos_sin(int pos, float freq, float* c, float* s) {
  float ang = __fmul_rn(static_cast<float>(pos), freq);
  sincosf(ang, s, c);
}

// interleaved-pair complex rotation (x0 + i x1) * (c + i s), conj for the inverse.
__device__ __forceinline__ void rotate_pair(float x0, float x1, float c, float s, bool inverse,
                                            float* y0, float* y1) {
  if (inverse) s = -s;
  *y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
  *y1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
}

}  // namespace dsv4
