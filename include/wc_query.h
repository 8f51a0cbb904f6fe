/*
 * Query-side scoring of witchcraft's match_centroids (src/lib.rs:600-887) on
 * a B200: the similarities of a query's tokens to the candidate embeddings
 * and the per-sub-chunk max-sum scores.  The caller selects the clusters and
 * gathers the candidates (witchcraft_b200/query.py shows the whole search).
 * Device pointers; stream is a cudaStream_t (may be 0).  Return codes are
 * those of wc_t5cuda.h; wc_query_last_error() gives the thread's last message.
 */
#ifndef WC_QUERY_H
#define WC_QUERY_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* q [m][dim] query tokens (1 <= m <= 128, even dim <= 128).  Rows 0..n_idx-1
 * are indexed candidates: codes [n_idx][dim/2] (4-bit residual codes, high
 * nibble first), cluster [n_idx], whose similarity to token t is
 * <q_t, table[codes]> + cscores[t][cluster]; rows n_idx.. are unindexed,
 * raw [.][dim] f32, similarity <q_t, e>.  table[16] is the q4 decoding table
 * (make_q4_dequant_table).  group g (a document's sub-chunk) covers
 * group_rows[group_start[g] .. group_start[g+1]); document d covers groups
 * doc_start[d] .. doc_start[d+1] in sub-chunk order.  out[g] = (1/m) sum_t
 * max(missing[t], similarities of token t to the rows of the document's
 * groups up to g) (src/lib.rs:715-808). */
int wc_score_candidates(const float* d_q, int m, int dim, const uint8_t* d_codes, const uint32_t* d_cluster,
                        const float* d_cscores, int n_cent, const float* d_table, int64_t n_idx, const float* d_raw,
                        const int64_t* d_group_rows, const int64_t* d_group_start, const int64_t* d_doc_start,
                        int64_t n_docs, const float* d_missing, float* d_out, void* stream);

/* out[16] = the q4 residual decoding table inv_compand(dequantize(q, 4))
 * (make_q4_dequant_table, src/packops.rs:14-24), computed on the host with
 * the C library's expf / logf (candle's pow is exp(e ln b)). */
int wc_q4_table(float* out);

/* out[t][j] = <q_t, c_j> for q [m][dim], c [k][dim] f32 (the query-centroid
 * similarities, src/lib.rs:637-640); one fused multiply-add chain each. */
int wc_similarities(const float* d_q, int m, const float* d_c, int64_t k, int dim, float* d_out, void* stream);

const char* wc_query_last_error(void);

#ifdef __cplusplus
}
#endif

#endif
