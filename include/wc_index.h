/*
 * Index-build steps of witchcraft on a B200 (src/lib.rs:187-274, 1376):
 * nearest-center assignment (matmul_argmax_batched), the k-means center
 * update, and the 4-bit mu-law residual codes the index stores per
 * embedding.  Device pointers; stream is a cudaStream_t (may be 0).  Return
 * codes are those of wc_t5cuda.h; wc_index_last_error() gives the calling
 * thread's last message.
 */
#ifndef WC_INDEX_H
#define WC_INDEX_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* idx[i] = argmax_c <x_i, c_c> (first maximum) for x [m][dim], centers
 * [k][dim] f32, 1 <= dim <= 128, dim % 4 == 0 (matmul_argmax_batched,
 * src/lib.rs:187-208).  Each similarity is one fused multiply-add chain over
 * the dimensions in order. */
int wc_assign_centers(const float* d_x, int64_t m, const float* d_centers, int64_t k, int dim, uint32_t* d_idx,
                      void* stream);

/* One k-means center update (src/lib.rs:238-274): centers_out[c] = sum of
 * the rows assigned to c (in row order) divided by its L2 norm; a center
 * with no rows takes row empty_src[c] (normalised) instead of the
 * reference's random row.  counts[c] = rows assigned.  Asynchronous on
 * stream. */
int wc_kmeans_update(const float* d_x, int64_t m, int dim, const uint32_t* d_idx, int64_t k,
                     const int64_t* d_empty_src, float* d_centers_out, uint32_t* d_counts, void* stream);

/* out[i][dim / 2] = 4-bit codes of compand(x_i - centers[idx_i]), two per
 * byte, the first in the high nibble (src/lib.rs:1376; src/packops.rs:136-162,
 * 440-462). */
int wc_residual_q4(const float* d_x, int64_t m, int dim, const uint32_t* d_idx, const float* d_centers,
                   uint8_t* d_out, void* stream);

const char* wc_index_last_error(void);

#ifdef __cplusplus
}
#endif

#endif
