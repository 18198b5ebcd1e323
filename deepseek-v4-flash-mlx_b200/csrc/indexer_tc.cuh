// Tensor-core filter of the lightning indexer (internal interface between indexer.cu and
// indexer_tc.cu).
//
// approx score A[i, j] = sum_h w[i,h] * relu(q[i,h,:] . k[j,:]) with every dot product taken on
// tcgen05 from a two-term fp16 split of both operands after an exact power-of-two scaling of each row
// (q = qh + ql, k = kh + kl; qh.kh + qh.kl + ql.kh, fp32 accumulate). The select kernel then bounds
// |A - E| (E: the canonical fp32 score) by eps_i = C * sum_h |w[i,h]| * ||q[i,h,:]|| * max_j ||k[j,:]||,
// keeps the keys that are certainly in the top-k, drops those certainly out, and rescores only the
// keys in between in the canonical order.
#pragma once
#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

namespace dsv4 {
namespace itc {

constexpr int BM = 128;                 // keys per tile
constexpr int TILE_BYTES = 64 * 1024;   // one tile's bf16 hi and lo image (2 x 2 swizzled slabs)

struct ApproxArgs {
  const float* q;       // [batch*s, 64, 128]
  const float* w;       // [batch*s, 64]
  const float* k;       // [batch, n_keys, 128] (batch stride k_batch_stride rows)
  float* scores;        // [batch*s, n_pad] approximate scores
  int32_t batch, s, n_keys, n_pad;
  int64_t k_batch_stride;
  const int32_t* positions;
  int32_t ratio;
  uint8_t* kimg;        // [batch][img_tiles][TILE_BYTES]: workspace, or a decode cache's image
  float* kinv;          // [batch][img_tiles * BM] inverse power-of-two scale of each key row
  float* kmax;          // [batch] max key norm (zeroed by the launcher unless img_ready)
  int32_t img_tiles;    // tiles per batch entry in kimg / kinv
  int32_t img_ready;    // kimg / kinv / kmax already hold every visible key (a decode cache's image)
};

__host__ __device__ inline int key_tiles(int n_keys) { return (n_keys + BM - 1) / BM; }
inline size_t kimg_bytes(int batch, int n_keys) {
  return static_cast<size_t>(batch) * key_tiles(n_keys) * TILE_BYTES;
}
// fewer than 4 queries per batch entry (decode): one query per CTA, keys split in tiles across CTAs,
// no key image (kimg / kinv unused)
inline bool row_kernel(int s) { return s < 4; }
inline size_t kinv_bytes(int batch, int n_keys) {
  return static_cast<size_t>(batch) * key_tiles(n_keys) * BM * sizeof(float);
}

// key image + norms (unless img_ready), then the approximate scores
cudaError_t launch_approx_scores(const ApproxArgs& a, cudaStream_t stream);
// key image + norms of keys [0, n_keys) of every batch entry into kimg / kinv / kmax (kmax zeroed)
cudaError_t launch_key_image(const ApproxArgs& a, cudaStream_t stream);

}  // namespace itc
}  // namespace dsv4
