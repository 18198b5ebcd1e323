/*
 * Oracle (test infrastructure only): lightning-indexer scores and top-k selection on the CPU, in
 * exactly the fp32 operation order of the library's score kernel, so that scores match bit for bit.
 *
 *   dot[h]   = fmaf chain over d = 0..127 (ascending), starting from +0
 *   r[h]     = dot[h] > 0 ? dot[h] : +0
 *   P[m]     = fmaf chain over h = 4m..4m+3 (ascending) of w[h] * r[h], starting from +0
 *   score    = balanced binary tree over P[0..15] (pairs (2t, 2t+1) at every level)
 *
 * The reference has no indexer (it attends to every visible compressed row,
 * oracle/decode_engine.py:112-114); this is the selection rule the library defines: keys ordered by
 * (score desc, index asc), score compared through its order-preserving 32-bit image; the chosen
 * keys are returned in ascending order, padded with -1.
 *
 * Build: gcc -O2 -ffp-contract=off -fno-fast-math -fopenmp -shared -fPIC (oracle/indexer_ref.py).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define HI 64
#define DI 128

static float score_one(const float* q, const float* w, const float* k) {
  float part[16];
  for (int m = 0; m < 16; ++m) {
    float p = 0.0f;
    for (int a = 0; a < 4; ++a) {
      const int h = 4 * m + a;
      const float* qh = q + h * DI;
      float d = 0.0f;
      for (int i = 0; i < DI; ++i) d = fmaf(qh[i], k[i], d);
      const float r = d > 0.0f ? d : 0.0f;
      p = fmaf(w[h], r, p);
    }
    part[m] = p;
  }
  for (int width = 16; width > 1; width >>= 1)
    for (int t = 0; t < width / 2; ++t) part[t] = part[2 * t] + part[2 * t + 1];
  return part[0];
}

/* scores[n] for one query over keys[n][128] */
void dsv4_oracle_scores(const float* q, const float* w, const float* keys, int64_t n, float* scores) {
#pragma omp parallel for schedule(static)
  for (int64_t j = 0; j < n; ++j) scores[j] = score_one(q, w, keys + j * DI);
}

static uint32_t ordered_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

static int cmp_desc_u64(const void* a, const void* b) {
  uint64_t x = *(const uint64_t*)a, y = *(const uint64_t*)b;
  return x < y ? 1 : (x > y ? -1 : 0);
}
static int cmp_asc_i32(const void* a, const void* b) {
  int32_t x = *(const int32_t*)a, y = *(const int32_t*)b;
  return x < y ? -1 : (x > y ? 1 : 0);
}

/* top_k of n scores by (score desc, index asc); out[top_k] ascending key indices, -1 padded */
void dsv4_oracle_select(const float* scores, int64_t n, int32_t top_k, int32_t* out) {
  if (n <= top_k) {
    for (int32_t r = 0; r < top_k; ++r) out[r] = r < n ? r : -1;
    return;
  }
  uint64_t* keys = (uint64_t*)malloc(sizeof(uint64_t) * n);
  for (int64_t j = 0; j < n; ++j)
    keys[j] = ((uint64_t)ordered_bits(scores[j]) << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)j);
  qsort(keys, n, sizeof(uint64_t), cmp_desc_u64);
  for (int32_t r = 0; r < top_k; ++r) out[r] = (int32_t)(0xFFFFFFFFu - (uint32_t)(keys[r] & 0xFFFFFFFFu));
  qsort(out, top_k, sizeof(int32_t), cmp_asc_i32);
  free(keys);
}

/* batched: q [rows][64][128], w [rows][64], keys [batch][n_keys][128]; query row r belongs to
 * batch r / s and sees keys j < nvis[r]. out [rows][top_k]. */
void dsv4_oracle_indexer_topk(const float* q, const float* w, const float* keys, int32_t batch, int32_t s,
                              int32_t n_keys, const int32_t* nvis, int32_t top_k, int32_t* out) {
  const int64_t rows = (int64_t)batch * s;
  float* sc = (float*)malloc(sizeof(float) * (size_t)n_keys);
  for (int64_t r = 0; r < rows; ++r) {
    const int64_t b = r / s;
    int64_t nv = nvis ? nvis[r] : n_keys;
    if (nv > n_keys) nv = n_keys;
    if (nv < 0) nv = 0;
    dsv4_oracle_scores(q + r * HI * DI, w + r * HI, keys + b * (int64_t)n_keys * DI, nv, sc);
    dsv4_oracle_select(sc, nv, top_k, out + r * top_k);
  }
  free(sc);
}
