/*
 * Packed-embedding codec of witchcraft on a B200: the reference's
 * TensorPackOps::embeddings_to_packed / embeddings_from_packed
 * (src/packops.rs:172-301, 303-438; Haar src/haarops.rs, rANS64
 * src/rans64.rs), for many documents per call.  The packed bytes of each
 * document are identical to the reference's (the blob `embed_chunks` stores
 * with add_chunk, src/lib.rs:1091, and the query side reads back,
 * src/lib.rs:712, 1178, 1296).
 *
 * Documents are given as one row-major f32 matrix [total_rows][cols] of
 * L2-normalised embeddings plus a host prefix array doc_rows[n_docs + 1]
 * (doc_rows[0] = 0); every document has at least one row.  The packed output
 * is one byte buffer with per-document offsets out_offsets[n_docs + 1].
 * Return codes are those of wc_t5cuda.h (0 = success); wc_codec_last_error()
 * gives the calling thread's last message.  One call at a time per device
 * (the device scratch is shared); calls allocate device scratch on demand.
 */
#ifndef WC_CODEC_H
#define WC_CODEC_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Upper bound of the packed size of the given documents (bytes), or -1. */
int64_t wc_packed_bound(const int64_t* doc_rows, int n_docs, int cols);

/* embeddings_to_packed of every document; d_emb / d_out device pointers,
 * doc_rows / out_offsets host arrays, stream a cudaStream_t (may be 0).
 * Returns when the output is complete.  cols in [1, 255]. */
int wc_pack_embeddings_device(const float* d_emb, const int64_t* doc_rows, int n_docs, int cols, uint8_t* d_out,
                              int64_t out_cap, int64_t* out_offsets, void* stream);

/* The same from and to host memory, on CUDA device `device`. */
int wc_pack_embeddings(const float* emb, const int64_t* doc_rows, int n_docs, int cols, uint8_t* out,
                       int64_t out_cap, int64_t* out_offsets, int device);

/* embeddings_from_packed of every document: the packed bytes in device
 * memory (d_in) and the same bytes in host memory (in, read for the window
 * headers), in_offsets[n_docs + 1]; writes L2-normalised rows to d_out
 * [rows][cols] and row_offsets[n_docs + 1] (host).  Malformed input returns
 * WC_E_INVALID_ARG (the reference returns an error). */
int wc_unpack_embeddings_device(const uint8_t* d_in, const uint8_t* in, const int64_t* in_offsets, int n_docs,
                                int cols, float* d_out, int64_t out_rows_cap, int64_t* row_offsets, void* stream);

/* The same from and to host memory, on CUDA device `device`. */
int wc_unpack_embeddings(const uint8_t* in, const int64_t* in_offsets, int n_docs, int cols, float* out,
                         int64_t out_rows_cap, int64_t* row_offsets, int device);

const char* wc_codec_last_error(void);

#ifdef __cplusplus
}
#endif

#endif
