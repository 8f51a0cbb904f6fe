/*
 * CPU oracle of the index-build steps.  TEST INFRASTRUCTURE ONLY: the checker
 * the CUDA kernels of csrc/index.cu are compared against; nothing in the
 * product path links or calls it.
 *
 * Restates (f32, in the reference's loop order, built with -ffp-contract=off):
 *   - matmul_argmax_batched   src/lib.rs:187-208: sim = X C^T, argmax per row.
 *     The reference's default build multiplies with candle's f32 matmul; here
 *     each dot product is one fused multiply-add chain over the dimensions in
 *     order (fmaf), and argmax keeps the first maximum.  Candle's summation
 *     order is not reproduced bit for bit (its gemm crate is absent here).
 *   - the k-means update      src/lib.rs:238-274: per-cluster sums in data
 *     order, each cluster divided by its L2 norm (sum of squares in dimension
 *     order); empty clusters take a given data row (the reference draws one
 *     at random).
 *   - residual codes          src/lib.rs:1376: (x - center), mu-law compand
 *     (src/packops.rs:136-142: s = 4x, sign(s) ln(1 + 255 |s|) / ln(256)),
 *     quantize(4) (round(y 7.5 + 7.5) clamped to [0, 15], :156-162), two
 *     4-bit codes per byte, the first in the high nibble (to_q4_bytes, :440-462).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* idx[i] = argmax_c sum_d x[i][d] c[c][d] */
void oracle_assign(const float* x, int64_t m, const float* c, int64_t k, int dim, uint32_t* idx) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < m; ++i) {
    const float* xi = x + i * dim;
    float best = -INFINITY;
    uint32_t bi = 0;
    for (int64_t j = 0; j < k; ++j) {
      const float* cj = c + j * dim;
      float acc = 0.0f;
      for (int d = 0; d < dim; ++d) acc = fmaf(xi[d], cj[d], acc);
      if (acc > best || j == 0) {
        best = acc;
        bi = (uint32_t)j;
      }
    }
    idx[i] = bi;
  }
}

/* centers_out[c] = normalised sum of the rows assigned to c, in row order;
 * empty clusters use row empty_src[c].  counts[c] = members. */
void oracle_kmeans_update(const float* x, int64_t m, int dim, const uint32_t* idx, int64_t k,
                          const int64_t* empty_src, float* centers_out, uint32_t* counts) {
  float* sums = calloc((size_t)(k * dim), sizeof(float));
  memset(counts, 0, sizeof(uint32_t) * (size_t)k);
  for (int64_t j = 0; j < m; ++j) {
    const uint32_t cl = idx[j];
    counts[cl]++;
    for (int d = 0; d < dim; ++d) sums[(int64_t)cl * dim + d] += x[j * dim + d];
  }
  for (int64_t i = 0; i < k; ++i) {
    const float* e = counts[i] > 0 ? sums + i * dim : x + empty_src[i] * dim;
    float ss = 0.0f;
    for (int d = 0; d < dim; ++d) ss += e[d] * e[d];
    const float norm = sqrtf(ss);
    for (int d = 0; d < dim; ++d) centers_out[i * dim + d] = norm > 0.0f ? e[d] / norm : e[d];
  }
  free(sums);
}

static float compand_q4(float r) {
  const float s = r * 4.0f;
  const float inv_den = (float)(1.0 / log(256.0));
  const float a = fabsf(s);
  const float y = logf(a * 255.0f + 1.0f) * inv_den;
  const float v = s > 0.0f ? y : (s < 0.0f ? -y : 0.0f);
  float q = roundf(v * 7.5f + 7.5f);
  if (q < 0.0f) q = 0.0f;
  if (q > 15.0f) q = 15.0f;
  return q;
}

/* out[i][dim / 2]: 4-bit codes of x[i] - centers[idx[i]] (dim even). */
void oracle_residual_q4(const float* x, int64_t m, int dim, const uint32_t* idx, const float* centers, uint8_t* out) {
  for (int64_t i = 0; i < m; ++i) {
    const float* xi = x + i * dim;
    const float* ci = centers + (int64_t)idx[i] * dim;
    for (int d = 0; d < dim; d += 2) {
      const uint8_t hi = (uint8_t)compand_q4(xi[d] - ci[d]) & 0x0F;
      const uint8_t lo = (uint8_t)compand_q4(xi[d + 1] - ci[d + 1]) & 0x0F;
      out[i * (dim / 2) + d / 2] = (uint8_t)((hi << 4) | lo);
    }
  }
}
