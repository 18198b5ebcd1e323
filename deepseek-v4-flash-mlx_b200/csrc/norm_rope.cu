// RMSNorm / per-head norm / interleaved RoPE (ref_torch/norm_rope.py:10-62, v4mlx/mla.py:26-28).
//
// All math in fp32: var = mean(x^2), x * rsqrt(var + eps) [* weight], then the rope rotation of
// the last rope_dim dims as interleaved complex pairs, then one cast to the output dtype.
// One warp per row; the row lives in registers between the reduction and the write.
#include "common.cuh"

namespace dsv4 {
namespace nr {

// four consecutive elements as fp32 (16-byte fp32 or 8-byte bf16 access)
__device__ __forceinline__ float4 load4(const void* p, int64_t i, int dtype) {
  if (dtype == DSV4_BF16) {
    const uint2 r = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(p) + i);
    return make_float4(__uint_as_float(r.x << 16), __uint_as_float(r.x & 0xFFFF0000u), __uint_as_float(r.y << 16),
                       __uint_as_float(r.y & 0xFFFF0000u));
  }
  return *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i);
}
__device__ __forceinline__ void store4(void* p, int64_t i, int dtype, float4 v) {
  if (dtype == DSV4_BF16)
    *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p) + i) = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
  else
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(p) + i) = v;
}

// RMSNorm for few rows (decode batches): one CTA per row, the row in registers (VPT groups of 4
// elements per thread), one block reduction; the CTAs of a handful of rows still fill the GPU's
// memory pipes, where one warp per row would serialise the row's loads on a few SMs
template <int VPT>
__global__ void __launch_bounds__(256) rmsnorm_row_kernel(dsv4_rmsnorm_params p) {
  pdl_wait();  // programmatic dependent launch: the previous kernel is complete from here
  pdl_trigger();
  __shared__ float part[8];
  const int tid = threadIdx.x, nt = blockDim.x;
  const int64_t base = static_cast<int64_t>(blockIdx.x) * p.dim;
  float4 v[VPT];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int i = (j * nt + tid) * 4;
    v[j] = i < p.dim ? load4(p.x, base + i, p.x_dtype) : make_float4(0.f, 0.f, 0.f, 0.f);
    ss = fmaf(v[j].x, v[j].x, ss);
    ss = fmaf(v[j].y, v[j].y, ss);
    ss = fmaf(v[j].z, v[j].z, ss);
    ss = fmaf(v[j].w, v[j].w, ss);
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) part[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int w = 0; w < (nt >> 5); ++w) tot += part[w];
  const float r = rsqrtf(tot / static_cast<float>(p.dim) + p.eps);
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int i = (j * nt + tid) * 4;
    if (i >= p.dim) continue;
    float4 o = make_float4(v[j].x * r, v[j].y * r, v[j].z * r, v[j].w * r);
    if (p.weight) {
      const float4 w = load4(p.weight, i, p.w_dtype);
      o = make_float4(w.x * o.x, w.y * o.y, w.z * o.z, w.w * o.w);
    }
    store4(p.out, base + i, p.out_dtype, o);
  }
}

// generic RMSNorm, any dim (multiple of 2), one warp per row, two passes over L1-resident data
__global__ void rmsnorm_kernel(dsv4_rmsnorm_params p) {
  pdl_wait();  // programmatic dependent launch: the previous kernel is complete from here
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int64_t row = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= p.rows) return;
  const int64_t base = row * p.dim;
  float ss = 0.f;
  for (int i = lane; i < p.dim; i += 32) {
    float v = load_as_float(p.x, base + i, p.x_dtype);
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / static_cast<float>(p.dim) + p.eps);
  for (int i = lane; i < p.dim; i += 32) {
    float v = load_as_float(p.x, base + i, p.x_dtype) * r;
    if (p.weight) v = load_as_float(p.weight, i, p.w_dtype) * v;
    store_from_float(p.out, base + i, p.out_dtype, v);
  }
}

// copy_rest: out != x, and the non-rope part of every row is copied by the same launch (elements
// [0, s * heads * (dim - rope_dim)) of the loop; the rope pairs follow)
__global__ void rope_kernel(dsv4_rope_params p, int copy_rest) {
  pdl_wait();  // programmatic dependent launch: the previous kernel is complete from here
  pdl_trigger();
  const int half = p.rope_dim / 2;
  const int keep = p.dim - p.rope_dim;
  const int64_t ncopy = copy_rest ? p.s * p.heads * keep : 0;
  const int64_t total = ncopy + p.s * p.heads * half;
  for (int64_t e0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e0 < total;
       e0 += (int64_t)gridDim.x * blockDim.x) {
    if (e0 < ncopy) {
      const int64_t rowh = e0 / keep;
      const int i = static_cast<int>(e0 % keep);
      store_from_float(p.out, rowh * p.dim + i, p.out_dtype, load_as_float(p.x, rowh * p.dim + i, p.x_dtype));
      continue;
    }
    const int64_t e = e0 - ncopy;
    const int i = static_cast<int>(e % half);
    const int64_t rowh = e / half;           // (position, head)
    const int64_t pos_row = rowh / p.heads;
    float c, s;
    if (p.cis) {
      const int64_t tr = pos_row % p.cis_rows;
      c = p.cis[(tr * half + i) * 2 + 0];
      s = p.cis[(tr * half + i) * 2 + 1];
    } else {
      int pos = p.positions ? p.positions[pos_row] : static_cast<int>(p.pos_offset + pos_row);
      rope_cos_sin(pos, p.freqs[i], &c, &s);
    }
    const int64_t off = rowh * p.dim + (p.dim - p.rope_dim) + 2 * i;
    float x0 = load_as_float(p.x, off, p.x_dtype), x1 = load_as_float(p.x, off + 1, p.x_dtype);
    float y0, y1;
    rotate_pair(x0, x1, c, s, p.inverse != 0, &y0, &y1);
    store_from_float(p.out, off, p.out_dtype, y0);
    store_from_float(p.out, off + 1, p.out_dtype, y1);
  }
}

// fused norm + rope + cast for rows of DIM (compile-time) elements: one warp per (row, head).
template <int DIM>
__global__ void norm_rope_kernel(dsv4_norm_rope_params p) {
  pdl_wait();  // programmatic dependent launch: the previous kernel is complete from here
  pdl_trigger();
  constexpr int PER = DIM / 32;  // contiguous elements per lane
  const int lane = threadIdx.x & 31;
  const int64_t unit = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (unit >= p.rows * p.heads) return;
  const int64_t row = unit / p.heads;
  const int head = static_cast<int>(unit % p.heads);
  const int64_t src = unit * DIM + lane * PER;
  float v[PER];
  if (p.x_dtype == DSV4_BF16) {
    const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(p.x) + src;
#pragma unroll
    for (int e = 0; e < PER; e += 8) {
      uint4 u = *reinterpret_cast<const uint4*>(x + e);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float2 f = __bfloat1622float2(h2[q]);
        v[e + 2 * q] = f.x;
        v[e + 2 * q + 1] = f.y;
      }
    }
  } else {
    const float* x = reinterpret_cast<const float*>(p.x) + src;
#pragma unroll
    for (int e = 0; e < PER; e += 4) {
      float4 f = *reinterpret_cast<const float4*>(x + e);
      v[e] = f.x;
      v[e + 1] = f.y;
      v[e + 2] = f.z;
      v[e + 3] = f.w;
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < PER; ++e) ss = fmaf(v[e], v[e], ss);
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / static_cast<float>(DIM) + p.eps);
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    float t = v[e] * r;
    if (p.weight) t = load_as_float(p.weight, lane * PER + e, p.w_dtype) * t;
    v[e] = t;
  }
  const int rope_lo = DIM - p.rope_dim;
  if (lane * PER + PER > rope_lo) {
    const int pos = p.positions[row];
#pragma unroll
    for (int e = 0; e < PER; e += 2) {
      const int d = lane * PER + e;
      if (d >= rope_lo) {
        float c, s;
        rope_cos_sin(pos, p.freqs[(d - rope_lo) >> 1], &c, &s);
        rotate_pair(v[e], v[e + 1], c, s, false, &v[e], &v[e + 1]);
      }
    }
  }
  if (p.act_quant) {  // fp8 act-quant simulation of the nope dims in blocks of 64 (64 / PER lanes)
    constexpr int LPB = 64 / PER;
    static_assert(64 % PER == 0, "a block spans whole lanes");
    float amax = 0.f;
#pragma unroll
    for (int e = 0; e < PER; ++e) amax = fmaxf(amax, fabsf(v[e]));
#pragma unroll
    for (int o = 1; o < LPB; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane * PER < DIM - p.rope_dim) {
      const int ex = act_quant_exp(amax);
#pragma unroll
      for (int e = 0; e < PER; ++e) v[e] = fp8_round_pow2(v[e], ex);
    }
  }
  int64_t dst;
  if (p.out_rows) {
    dst = (p.out_rows[row] * p.heads + head) * DIM + lane * PER;
  } else {
    dst = unit * DIM + lane * PER;
  }
  if (p.out_dtype == DSV4_BF16) {
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + dst;
#pragma unroll
    for (int e = 0; e < PER; e += 8) {
      uint4 u = make_uint4(pack_bf16x2(v[e], v[e + 1]), pack_bf16x2(v[e + 2], v[e + 3]),
                           pack_bf16x2(v[e + 4], v[e + 5]), pack_bf16x2(v[e + 6], v[e + 7]));
      *reinterpret_cast<uint4*>(o + e) = u;
    }
  } else {
    float* o = reinterpret_cast<float*>(p.out) + dst;
#pragma unroll
    for (int e = 0; e < PER; e += 4) *reinterpret_cast<float4*>(o + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
  }
}

}  // namespace nr
}  // namespace dsv4

using namespace dsv4;

static bool is_float_dtype(int d) { return d == DSV4_F32 || d == DSV4_BF16; }

extern "C" int dsv4_rmsnorm(const dsv4_rmsnorm_params* p, void* stream) {
  DSV4_CHECK_ARG(p && p->x && p->out && p->rows >= 0 && p->dim > 0, "dsv4_rmsnorm: bad arguments");
  DSV4_CHECK_DTYPE(is_float_dtype(p->x_dtype) && is_float_dtype(p->out_dtype) &&
                       (p->weight == nullptr || is_float_dtype(p->w_dtype)),
                   "dsv4_rmsnorm: F32/BF16 only");
  if (p->rows == 0) return DSV4_OK;
  const auto al = [](const void* q, int dt) { return reinterpret_cast<uintptr_t>(q) % (dt == DSV4_BF16 ? 8 : 16) == 0; };
  if (p->rows <= 4 * num_sms() && p->dim % 4 == 0 && p->dim >= 128 && p->dim <= 8192 && al(p->x, p->x_dtype) &&
      al(p->out, p->out_dtype) && (p->weight == nullptr || al(p->weight, p->w_dtype))) {
    const int threads = p->dim >= 1024 ? 256 : 128;
    const int vpt = (p->dim / 4 + threads - 1) / threads;  // <= 8
    const dim3 grid(static_cast<unsigned>(p->rows));
    if (vpt <= 1)
      DSV4_CUDA_CHECK(launch_pdl(nr::rmsnorm_row_kernel<1>, dim3(grid), dim3(threads), 0, as_stream(stream), *p));
    else if (vpt <= 2)
      DSV4_CUDA_CHECK(launch_pdl(nr::rmsnorm_row_kernel<2>, dim3(grid), dim3(threads), 0, as_stream(stream), *p));
    else if (vpt <= 4)
      DSV4_CUDA_CHECK(launch_pdl(nr::rmsnorm_row_kernel<4>, dim3(grid), dim3(threads), 0, as_stream(stream), *p));
    else
      DSV4_CUDA_CHECK(launch_pdl(nr::rmsnorm_row_kernel<8>, dim3(grid), dim3(threads), 0, as_stream(stream), *p));
    DSV4_LAUNCH_CHECK("rmsnorm_row_kernel");
    return DSV4_OK;
  }
  const int warps = 8;
  int64_t blocks = (p->rows + warps - 1) / warps;
  DSV4_CUDA_CHECK(launch_pdl(nr::rmsnorm_kernel, dim3(static_cast<unsigned>(blocks)), dim3(warps * 32), 0, as_stream(stream), *p));
  DSV4_LAUNCH_CHECK("rmsnorm_kernel");
  return DSV4_OK;
}

extern "C" int dsv4_rope(const dsv4_rope_params* p, void* stream) {
  DSV4_CHECK_ARG(p && p->x && p->out && p->s >= 0 && p->heads > 0 && p->rope_dim > 0 &&
                     p->rope_dim % 2 == 0 && p->rope_dim <= p->dim,
                 "dsv4_rope: bad arguments");
  DSV4_CHECK_ARG((p->cis != nullptr) != (p->freqs != nullptr), "dsv4_rope: give exactly one of cis / freqs");
  DSV4_CHECK_ARG(p->cis == nullptr || p->cis_rows > 0, "dsv4_rope: cis_rows must be > 0");
  DSV4_CHECK_DTYPE(is_float_dtype(p->x_dtype) && is_float_dtype(p->out_dtype), "dsv4_rope: F32/BF16 only");
  if (p->s == 0) return DSV4_OK;
  const int copy_rest = (p->out != p->x && p->dim > p->rope_dim) ? 1 : 0;
  const int64_t total = p->s * p->heads * ((p->rope_dim / 2) + (copy_rest ? p->dim - p->rope_dim : 0));
  int blocks = static_cast<int>((total + 255) / 256);
  if (blocks > 16 * num_sms()) blocks = 16 * num_sms();
  DSV4_CUDA_CHECK(launch_pdl(nr::rope_kernel, dim3(blocks), dim3(256), 0, as_stream(stream), *p, copy_rest));
  DSV4_LAUNCH_CHECK("rope_kernel");
  return DSV4_OK;
}

extern "C" int dsv4_norm_rope(const dsv4_norm_rope_params* p, void* stream) {
  DSV4_CHECK_ARG(p == nullptr || p->act_quant == 0 ||
                     (p->act_quant == 1 && p->dim >= 128 && (p->dim - p->rope_dim) % 64 == 0),
                 "dsv4_norm_rope: act_quant needs (dim - rope_dim) a multiple of 64");
  DSV4_CHECK_ARG(p && p->x && p->out && p->freqs && p->positions && p->rows >= 0 && p->heads > 0,
                 "dsv4_norm_rope: bad arguments");
  DSV4_CHECK_ARG(p->rope_dim > 0 && p->rope_dim % 2 == 0 && p->rope_dim <= p->dim,
                 "dsv4_norm_rope: bad rope_dim");
  DSV4_CHECK_DTYPE(is_float_dtype(p->x_dtype) && is_float_dtype(p->out_dtype) &&
                       (p->weight == nullptr || is_float_dtype(p->w_dtype)),
                   "dsv4_norm_rope: F32/BF16 only");
  if (p->rows == 0) return DSV4_OK;
  const int warps = 8;
  const int64_t units = p->rows * p->heads;
  const unsigned blocks = static_cast<unsigned>((units + warps - 1) / warps);
  switch (p->dim) {
    case 512:
      DSV4_CUDA_CHECK(launch_pdl(nr::norm_rope_kernel<512>, dim3(blocks), dim3(warps * 32), 0, as_stream(stream), *p));
      break;
    case 256:
      DSV4_CUDA_CHECK(launch_pdl(nr::norm_rope_kernel<256>, dim3(blocks), dim3(warps * 32), 0, as_stream(stream), *p));
      break;
    case 128:
      DSV4_CUDA_CHECK(launch_pdl(nr::norm_rope_kernel<128>, dim3(blocks), dim3(warps * 32), 0, as_stream(stream), *p));
      break;
    default:
      set_error("dsv4_norm_rope: dim %d unsupported (128/256/512)", p->dim);
      return DSV4_ERR_INVALID_ARGUMENT;
  }
  DSV4_LAUNCH_CHECK("norm_rope_kernel");
  return DSV4_OK;
}
