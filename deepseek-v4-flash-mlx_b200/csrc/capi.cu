// Status plumbing, the device error word, host-side YaRN table, window indices and casts.
#include <cmath>
#include <vector>

#include "common.cuh"

namespace dsv4 {

static thread_local std::string t_last_error;

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
}
void clear_error() { t_last_error.clear(); }

static error_reader_fn g_readers[32];
static int g_nreaders = 0;

int register_error_reader(error_reader_fn fn) {
  if (g_nreaders < 32) g_readers[g_nreaders++] = fn;
  return g_nreaders;
}

cudaError_t read_all_error_words(int* first) {
  *first = 0;
  for (int i = 0; i < g_nreaders; ++i) {
    int v = 0;
    cudaError_t e = g_readers[i](&v);
    if (e != cudaSuccess) return e;
    if (*first == 0) *first = v;
  }
  return cudaSuccess;
}

// ref_torch/sparse_attn.py:9-20, all three branches; int32 out [bsz, seqlen, cols].
__global__ void window_idx_kernel(int32_t window, int32_t bsz, int32_t seqlen, int32_t start_pos,
                                  int32_t cols, int32_t* out) {
  int64_t total = static_cast<int64_t>(bsz) * seqlen * cols;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    int c = static_cast<int>(e % cols);
    int i = static_cast<int>((e / cols) % seqlen);
    int v;
    if (start_pos >= window - 1) {
      int sp = start_pos % window;
      // cat(arange(sp+1, window), arange(0, sp+1))
      v = (c < window - sp - 1) ? (sp + 1 + c) : (c - (window - sp - 1));
    } else if (start_pos > 0) {
      v = (c <= start_pos) ? c : -1;
    } else {
      int base = i - window + 1;
      if (base < 0) base = 0;
      v = base + c;
      if (v > i) v = -1;
    }
    out[e] = v;
  }
}

__global__ void cast_kernel(const void* x, int32_t xd, void* y, int32_t yd, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    store_from_float(y, i, yd, load_as_float(x, i, xd));
}

// 16-byte copy by the SMs (either side may be pinned host memory, reached over the bus through its
// unified address); under programmatic dependent launch it waits for the previous kernel first
constexpr int COPY_THREADS = 64;
// The copies ask for the largest shared-memory carveout although they use none: an SM changes its
// L1 / shared split only when it is empty, so copy blocks resident under a small carveout would
// keep a following large-shared-memory kernel (launched early by programmatic dependent launch, or
// beside on another stream) off that SM until they leave.
constexpr int COPY_CARVEOUT = 100;

__global__ void copy16_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, int64_t n16) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = src[i];
}

// The copy of dsv4_copy_beside: it runs while the kernel launched before it finishes (no wait
// first), makes its stores visible device-wide and only then lets the next kernel launch, and waits
// for the kernel before it at the end, so that the next kernel's wait covers both.
__global__ void copy16_beside_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, int64_t n16) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = src[i];
  __threadfence();
  pdl_trigger();
  pdl_wait();
}

}  // namespace dsv4

using namespace dsv4;

extern "C" {

const char* dsv4_last_error(void) { return t_last_error.c_str(); }

int dsv4_abi_version(void) { return DSV4_ABI_VERSION; }

int dsv4_device_error(int* code, void* stream) {
  DSV4_CHECK_ARG(code != nullptr, "dsv4_device_error: code is NULL");
  DSV4_CUDA_CHECK(cudaStreamSynchronize(as_stream(stream)));
  int v = 0;
  DSV4_CUDA_CHECK(read_all_error_words(&v));
  *code = v;
  return DSV4_OK;
}

// ref_torch/norm_rope.py:19-43 precompute_freqs. The reference computes the base table in fp32
// (base ** (arange/dim) on a float32 tensor) and the ramp in fp32; this follows the same order.
int dsv4_yarn_freqs(int32_t dim, int64_t original_seq_len, double base, double factor,
                    double beta_fast, double beta_slow, float* out_host) {
  DSV4_CHECK_ARG(out_host != nullptr && dim > 0 && dim % 2 == 0, "dsv4_yarn_freqs: bad arguments");
  const int half = dim / 2;
  const float fdim = static_cast<float>(dim);
  const float fbase = static_cast<float>(base);
  for (int i = 0; i < half; ++i) {
    float e = static_cast<float>(2 * i) / fdim;
    out_host[i] = 1.0f / powf(fbase, e);
  }
  if (original_seq_len > 0) {
    auto corr_dim = [&](double rot) {
      return dim * std::log(static_cast<double>(original_seq_len) / (rot * 2 * M_PI)) /
             (2 * std::log(base));
    };
    double low = std::floor(corr_dim(beta_fast));
    double high = std::ceil(corr_dim(beta_slow));
    if (low < 0) low = 0;
    if (high > dim - 1) high = dim - 1;
    float mn = static_cast<float>(low), mx = static_cast<float>(high);
    if (mn == mx) mx += 0.001f;
    const float ffactor = static_cast<float>(factor);
    for (int i = 0; i < half; ++i) {
      float lin = (static_cast<float>(i) - mn) / (mx - mn);
      lin = fminf(fmaxf(lin, 0.0f), 1.0f);
      float smooth = 1.0f - lin;
      float f = out_host[i];
      out_host[i] = f / ffactor * (1.0f - smooth) + f * smooth;
    }
  }
  return DSV4_OK;
}

int dsv4_window_topk_idxs(int32_t window, int32_t bsz, int32_t seqlen, int32_t start_pos,
                          int32_t* out, void* stream) {
  DSV4_CHECK_ARG(out != nullptr && window > 0 && bsz > 0 && seqlen > 0 && start_pos >= 0,
                 "dsv4_window_topk_idxs: bad arguments");
  int32_t cols = (start_pos > 0) ? window : (seqlen < window ? seqlen : window);
  int64_t total = static_cast<int64_t>(bsz) * seqlen * cols;
  int blocks = static_cast<int>((total + 255) / 256);
  if (blocks > 4096) blocks = 4096;
  window_idx_kernel<<<blocks, 256, 0, as_stream(stream)>>>(window, bsz, seqlen, start_pos, cols, out);
  DSV4_LAUNCH_CHECK("window_idx_kernel");
  return DSV4_OK;
}

int dsv4_copy(void* dst, const void* src, size_t bytes, void* stream) {
  DSV4_CHECK_ARG(dst && src, "dsv4_copy: NULL pointer");
  DSV4_CHECK_ARG(reinterpret_cast<uintptr_t>(dst) % 16 == 0 && reinterpret_cast<uintptr_t>(src) % 16 == 0 &&
                     bytes % 16 == 0,
                 "dsv4_copy: addresses and size must be multiples of 16 bytes");
  if (bytes == 0) return DSV4_OK;
  const int64_t n16 = static_cast<int64_t>(bytes / 16);
  // small blocks spread the 16-byte loads over more SMs: more reads of pinned memory in flight at
  // once (a 33 KB step input: 9 blocks of 256 threads -> 33 of 64, ~0.4 us less per decode step)
  int blocks = static_cast<int>((n16 + COPY_THREADS - 1) / COPY_THREADS);
  if (blocks > 8 * num_sms()) blocks = 8 * num_sms();
  static PerDeviceOnce carve;
  DSV4_CUDA_CHECK(set_carveout_once(carve, copy16_kernel, COPY_CARVEOUT));
  DSV4_CUDA_CHECK(launch_pdl(copy16_kernel, dim3(blocks), dim3(COPY_THREADS), 0, as_stream(stream),
                             reinterpret_cast<const uint4*>(src), reinterpret_cast<uint4*>(dst), n16));
  return DSV4_OK;
}

int dsv4_copy_beside(void* dst, const void* src, size_t bytes, void* stream) {
  DSV4_CHECK_ARG(dst && src, "dsv4_copy_beside: NULL pointer");
  DSV4_CHECK_ARG(reinterpret_cast<uintptr_t>(dst) % 16 == 0 && reinterpret_cast<uintptr_t>(src) % 16 == 0 &&
                     bytes % 16 == 0,
                 "dsv4_copy_beside: addresses and size must be multiples of 16 bytes");
  if (bytes == 0) return DSV4_OK;
  const int64_t n16 = static_cast<int64_t>(bytes / 16);
  // small blocks spread the 16-byte loads over more SMs: more reads of pinned memory in flight at
  // once (a 33 KB step input: 9 blocks of 256 threads -> 33 of 64, ~0.4 us less per decode step)
  int blocks = static_cast<int>((n16 + COPY_THREADS - 1) / COPY_THREADS);
  if (blocks > 8 * num_sms()) blocks = 8 * num_sms();
  static PerDeviceOnce carve;
  DSV4_CUDA_CHECK(set_carveout_once(carve, copy16_beside_kernel, COPY_CARVEOUT));
  DSV4_CUDA_CHECK(launch_pdl(copy16_beside_kernel, dim3(blocks), dim3(COPY_THREADS), 0, as_stream(stream),
                             reinterpret_cast<const uint4*>(src), reinterpret_cast<uint4*>(dst), n16));
  return DSV4_OK;
}

int dsv4_cast(const void* x, int32_t x_dtype, void* y, int32_t y_dtype, int64_t numel, void* stream) {
  DSV4_CHECK_ARG(x && y && numel >= 0, "dsv4_cast: bad arguments");
  DSV4_CHECK_DTYPE((x_dtype == DSV4_F32 || x_dtype == DSV4_BF16) &&
                       (y_dtype == DSV4_F32 || y_dtype == DSV4_BF16),
                   "dsv4_cast: only F32/BF16");
  if (numel == 0) return DSV4_OK;
  int blocks = static_cast<int>((numel + 255) / 256);
  if (blocks > 8 * num_sms()) blocks = 8 * num_sms();
  cast_kernel<<<blocks, 256, 0, as_stream(stream)>>>(x, x_dtype, y, y_dtype, numel);
  DSV4_LAUNCH_CHECK("cast_kernel");
  return DSV4_OK;
}

}  // extern "C"
