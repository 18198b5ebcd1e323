// Row bookkeeping of one decode step over the device-resident sparse-MLA state, in one launch:
// where this token's window row, its compressed row and its indexer key go. The reference keeps
// this state on the host (oracle/v4_fast.py:93-118, oracle/step12_glue.py:142-173); here it is a
// pool of rows in HBM addressed through a block table, and the addresses are computed on the
// device so that a whole decode step stays inside one CUDA graph.
//
// For sequence i at position p: win_rows[i] = win_base[i] + p % window;
// entry = max((p + 1) / ratio - 1, 0), the compressed entry that the step emits (or, when
// (p + 1) % ratio != 0, the one it would overwrite last: the compressor writes it only on emission);
// comp_rows[i] = comp_base + block_table[i * bt_stride + entry / page] * page + entry % page;
// key_rows[i] = i * max_comp + entry. An entry at or past max_comp raises
// DSV4_ERR_INDEX_OUT_OF_RANGE on the device error word and is clamped to the last entry.
// A cache with max_comp == 0 holds no compressed rows: the window-only layers (ratio 0 and the
// ratio-128 layers, which the reference runs without a compressor, oracle/v4_fast.py:42-43, 114);
// then comp_rows and key_rows are -1, ratio is ignored and the block table is not read.
#include "common.cuh"

namespace dsv4 {
namespace dr {

__global__ void decode_rows_kernel(dsv4_decode_rows_params p) {
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < p.b) {
    const int64_t pos = p.positions[i];
    const int64_t wpos = pos < 0 ? 0 : pos;
    p.win_rows[i] = p.win_base[i] + wpos % p.window;
    if (p.max_comp == 0) {
      p.comp_rows[i] = -1;
      p.key_rows[i] = -1;
    } else {
      int64_t entry = (pos + 1) / p.ratio - 1;
      if (entry < 0) entry = 0;
      if (entry >= p.max_comp) {
        raise_device_error(DSV4_ERR_INDEX_OUT_OF_RANGE);
        entry = p.max_comp - 1;
      }
      const int64_t blk = p.block_table[static_cast<int64_t>(i) * p.bt_stride + entry / p.page];
      p.comp_rows[i] = p.comp_base + blk * p.page + entry % p.page;
      p.key_rows[i] = static_cast<int64_t>(i) * p.max_comp + entry;
    }
  }
  pdl_trigger();
}

}  // namespace dr
}  // namespace dsv4

using namespace dsv4;

DSV4_ERROR_READER(decode_rows)

extern "C" int dsv4_decode_rows(const dsv4_decode_rows_params* p, void* stream) {
  DSV4_CHECK_ARG(p && p->positions && p->win_base && p->win_rows && p->comp_rows && p->key_rows &&
                     (p->block_table || p->max_comp == 0),
                 "dsv4_decode_rows: NULL pointer");
  DSV4_CHECK_ARG(p->b >= 0 && p->window > 0 && p->max_comp >= 0 &&
                     (p->max_comp == 0 || (p->ratio > 0 && p->page > 0 &&
                                           p->bt_stride * static_cast<int64_t>(p->page) >= p->max_comp)),
                 "dsv4_decode_rows: bad sizes");
  if (p->b == 0) return DSV4_OK;
  const int threads = 128;
  DSV4_CUDA_CHECK(launch_pdl(dr::decode_rows_kernel, dim3((p->b + threads - 1) / threads), dim3(threads), 0,
                             as_stream(stream), *p));
  return DSV4_OK;
}
