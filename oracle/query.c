/*
 * CPU oracle of the query-side candidate scoring.  TEST INFRASTRUCTURE ONLY:
 * the checker csrc/query.cu is compared against; nothing in the product path
 * links or calls it.
 *
 * Restates match_centroids' scoring (src/lib.rs:715-808) over a prepared
 * candidate set: each indexed row's similarity to query token t is
 * <q_t, table[codes]> + centroid_score[t][cluster] (the residual decoded with
 * the q4 table, src/packops.rs:14-24, 491-514), an unindexed row's is <q_t, e>;
 * rows are grouped by (document, sub-chunk) in sorted order; within a
 * document the per-token running maximum starts at `missing` and carries over
 * from one sub-chunk to the next (vmax_inplace, doc_scores / sub_scores);
 * each sub-chunk's score is (1 / m) * sum over tokens (in token order).
 * Dot products are fmaf chains over the dimensions in order, as in the CUDA
 * kernel; the reference's candle matmul order is not reproduced bit for bit.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* table[16] = inv_compand(dequantize(q, 4)) (make_q4_dequant_table,
 * src/packops.rs:14-24, 144-154, 164-170); candle's Tensor::pow(b, e) is
 * exp(e * ln(b)). */
void oracle_q4_table(float* table) {
  for (int q = 0; q < 16; ++q) {
    const float x = ((float)q - 7.5f) * (float)(2.0 / 15.0); /* dequantize(4): (x - zp) * (2 / qmax) */
    const float a = fabsf(x);
    const float sign = x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f);
    const float p = expf(a * logf(256.0f));
    const float scaled = sign * ((p - 1.0f) * (float)(1.0 / 255.0));
    table[q] = scaled * 0.25f;
  }
}

/* rows: n_idx indexed rows (codes [n_idx][dim/2], cluster [n_idx]) followed by
 * n_raw unindexed rows (raw [n_raw][dim]); a row id r < n_idx is indexed.
 * Groups: group g covers group_rows[group_start[g], group_start[g+1]);
 * documents: doc d covers groups [doc_start[d], doc_start[d+1]).  out[g]. */
void oracle_score_candidates(const float* q, int m, int dim, const uint8_t* codes, const uint32_t* cluster,
                             const float* cscores, int n_cent, const float* table, int64_t n_idx, const float* raw,
                             const int64_t* group_rows, const int64_t* group_start, const int64_t* doc_start,
                             int64_t n_docs, const float* missing, float* out) {
  float* s = malloc(sizeof(float) * (size_t)m);
  float* e = malloc(sizeof(float) * (size_t)dim);
  const float scaler = 1.0f / (float)m;
  for (int64_t d = 0; d < n_docs; ++d) {
    memcpy(s, missing, sizeof(float) * (size_t)m);
    for (int64_t g = doc_start[d]; g < doc_start[d + 1]; ++g) {
      for (int64_t p = group_start[g]; p < group_start[g + 1]; ++p) {
        const int64_t r = group_rows[p];
        const float* v;
        if (r < n_idx) {
          for (int k = 0; k < dim; k += 2) {
            const uint8_t b = codes[r * (dim / 2) + k / 2];
            e[k] = table[b >> 4];
            e[k + 1] = table[b & 15];
          }
          v = e;
        } else {
          v = raw + (r - n_idx) * dim;
        }
        for (int t = 0; t < m; ++t) {
          float acc = 0.0f;
          for (int k = 0; k < dim; ++k) acc = fmaf(q[t * dim + k], v[k], acc);
          if (r < n_idx) acc = acc + cscores[(int64_t)t * n_cent + cluster[r]];
          s[t] = fmaxf(s[t], acc);
        }
      }
      float sum = 0.0f;
      for (int t = 0; t < m; ++t) sum += s[t];
      out[g] = scaler * sum;
    }
  }
  free(s);
  free(e);
}

/* out[t][j] = <q_t, c_j>, one fmaf chain over the dimensions in order. */
void oracle_similarities(const float* q, int m, const float* c, int64_t k, int dim, float* out) {
  for (int t = 0; t < m; ++t)
    for (int64_t j = 0; j < k; ++j) {
      float acc = 0.0f;
      for (int d = 0; d < dim; ++d) acc = fmaf(q[t * dim + d], c[j * dim + d], acc);
      out[t * k + j] = acc;
    }
}
