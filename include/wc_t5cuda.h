/*
 * wc_t5cuda.h — C ABI of the B200 (sm_100a) XTR-base T5 encoder backend.
 *
 * This is the boundary a `t5-cuda` feature of dropbox/witchcraft binds over
 * FFI.  It replaces, behind the unchanged Embedder API, the encoder backend
 * contract of the reference:
 *   T5ModelBuilder::build_encoder   src/quantized_t5.rs:731-749
 *   T5EncoderModel::load            src/quantized_t5.rs:680-696
 *   T5EncoderModel::forward         src/quantized_t5.rs:698-701
 *   T5EncoderModel::device          src/quantized_t5.rs:703-705
 * (the OpenVINO backend implements the same surface, src/openvino_t5.rs:151-245).
 *
 * Conventions
 *   - Every function returns 0 (WC_OK) on success or a negative WC_E* code;
 *     the forward calls may also return the positive warning
 *     WC_W_F16_CLIPPED (results delivered, see below).  Nothing aborts,
 *     throws or exits across this boundary.
 *   - The caller owns all host buffers.  A handle owns its device memory,
 *     stream and workspaces; wc_t5_destroy frees them.
 *   - One handle drives one GPU.  A handle is not re-entrant (wrap it in a
 *     mutex); different handles may be used from different threads at once.
 *   - Kernels never trap: a failed in-kernel wait sets a device status word
 *     that the forward call turns into WC_E_TIMEOUT.
 *   - Numerics: the residual stream, RMSNorm statistics, every accumulation
 *     and all outputs are f32; tensor-core operands (normalised activations,
 *     dequantised weights, Q/K/V, softmax weights, gated-GELU output) are f16
 *     (11-bit significand), saturated to the finite f16 range.  A forward in
 *     which any such value was clipped (|x| >= 65520, or NaN) returns
 *     WC_W_F16_CLIPPED instead of WC_OK: the outputs are written, but they
 *     may deviate from the reference's f32 computation beyond the stated
 *     tolerance.  (The f32 reference has no such limit; a checkpoint whose
 *     activations leave the f16 range needs a wider operand type.)
 *   - Functions taking `void* stream` accept a cudaStream_t (NULL = legacy
 *     default stream) and device pointers; they return once the work is
 *     enqueued.
 */
#ifndef WC_T5CUDA_H
#define WC_T5CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  WC_W_F16_CLIPPED = 1,    /* success, but an f16 activation was clipped (see Numerics) */
  WC_OK = 0,
  WC_E_INVALID_ARG = -1,   /* null pointer, bad size, token id >= vocab, ... */
  WC_E_GGUF = -2,          /* malformed or truncated GGUF, missing tensor */
  WC_E_UNSUPPORTED = -3,   /* tensor dtype/shape or config this backend does not run */
  WC_E_CUDA = -4,          /* CUDA runtime error (no device, out of memory, launch failure) */
  WC_E_TIMEOUT = -5,       /* an in-kernel wait hit its time limit */
  WC_E_CONFIG = -6         /* config.json missing a field or unparsable */
};

typedef struct wc_t5 wc_t5;

/* Number of CUDA devices visible to this process (0 when none; never fails). */
int wc_t5_device_count(void);

/* Page-locked host memory (cudaHostAlloc, portable across devices) for the
 * ids / outputs of wc_t5_forward_many, whose copies overlap the compute only
 * from page-locked buffers.  Returns NULL on failure.  No reference
 * counterpart (the reference keeps results in candle host tensors). */
void* wc_host_alloc(size_t bytes);
void wc_host_free(void* p);

/* Build an encoder on device `device_ordinal` from the bytes of xtr.gguf and
 * the text of config.json (T5ModelBuilder::load + build_encoder,
 * src/quantized_t5.rs:713-749).  Q4_K tensors are uploaded unchanged (raw
 * super-blocks); F32/F16 tensors are uploaded as f32.  The layer matrices are
 * also dequantised once to resident f16 copies (170 MB for XTR-base) that the
 * GEMMs of batches of 512 tokens and more read; with the environment variable
 * WC_F16_WEIGHTS=0 set at create time the handle keeps only the Q4_K bytes
 * and those GEMMs dequantise the super-blocks in the kernel instead (same
 * operand bits, same results).  On failure *out is set to NULL and the reason
 * is available from wc_t5_last_error(NULL). */
int wc_t5_create(int device_ordinal, const uint8_t* gguf, size_t gguf_len, const char* config_json,
                 wc_t5** out);

/* Free everything the handle owns.  NULL is accepted. */
int wc_t5_destroy(wc_t5* h);

/* Last error message of the handle (or of the last failed wc_t5_create when
 * h is NULL).  The string lives until the next call on the same handle. */
const char* wc_t5_last_error(const wc_t5* h);

/* Encode a padded batch (T5EncoderModel::forward, src/quantized_t5.rs:698-701,
 * generalised from batch 1 to B rows with a key padding mask).
 *   ids      host u32 [B][L], row-major; positions >= lengths[b] are ignored
 *   lengths  host i32 [B], 1 <= lengths[b] <= L (NULL = every row has length L)
 *   L        1..2048 (the Embedder's window, src/embedder.rs:27)
 *   out      host f32 [B][L][128]: the raw 768->128 projection (what the
 *            reference forward returns; rows past lengths[b] are 0)
 *   norms    host f32 [B][L] L2 norm of each raw row, or NULL
 *   out_normalised host f32 [B][L][128] rows divided by their norm, or NULL
 * Each row b equals the reference's batch-1 forward of ids[b][0:lengths[b]].
 * Blocks until the results are in host memory. */
int wc_t5_forward(wc_t5* h, const uint32_t* ids, const int32_t* lengths, int B, int L, float* out, float* norms,
                  float* out_normalised);

/* Same as wc_t5_forward with device buffers, enqueued on `stream`; returns
 * without synchronising (the status word is checked by the next blocking
 * call, or by wc_t5_sync). */
int wc_t5_forward_device(wc_t5* h, const uint32_t* d_ids, const int32_t* d_lengths, int B, int L, float* d_out,
                         float* d_norms, float* d_out_normalised, void* stream);

/* n batches through the same forward as wc_t5_forward, pipelined: while
 * batch i runs, batch i's predecessor's results are copied out and batch
 * i + 2's inputs copied in (a second stream and two device I/O buffer sets),
 * so with page-locked host buffers the copies hide behind the compute.
 * ids[i] / lengths[i] (lengths may be NULL, or lengths[i] NULL for full
 * rows) / B[i] / L[i] / out[i] / norms[i] (norms may be NULL) as in
 * wc_t5_forward; every result is the same as that batch's wc_t5_forward.
 * Returns when all results are in host memory.  No reference counterpart:
 * the reference embeds one document per call (src/embedder.rs:22-102); this
 * is the entry for a batched caller. */
int wc_t5_forward_many(wc_t5* h, int n, const uint32_t* const* ids, const int32_t* const* lengths, const int* B,
                       const int* L, float* const* out, float* const* norms);

/* n device-resident batches (d_ids[i], d_lengths[i], B[i], L[i], d_out[i],
 * d_norms[i] as in wc_t5_forward_device; d_norms may be NULL) enqueued in one
 * call, ordered after the caller's earlier work on `stream`.  With several
 * batches past the captured-graph size the odd batches run on the handle's
 * second compute lane (its own stream and activation buffers), and `stream`
 * waits for that lane before this call returns, so work the caller enqueues
 * on `stream` afterwards (an event, a copy) sees every result.  Returns
 * without synchronising; check with wc_t5_sync.  No reference counterpart:
 * the entry for a caller whose batches are already on the device (a
 * multi-GPU worker, or a pipeline that tokenises on the GPU). */
int wc_t5_forward_many_device(wc_t5* h, int n, const uint32_t* const* d_ids, const int32_t* const* d_lengths,
                              const int* B, const int* L, float* const* d_out, float* const* d_norms,
                              void* stream);

/* Same computation as wc_t5_forward_device, for callers that must not
 * allocate GPU memory during a call: a real-time query path that cannot
 * afford cudaMalloc's implicit device synchronisation, or a host that owns
 * and pre-reserves all device memory itself.  (No counterpart in the
 * reference, whose CPU path has no device memory.)  The activations live in
 * one fixed 8 MiB array that every GPU loading this library holds until the
 * process exits, instead of the handle's workspace; B*L is limited to what
 * fits (about 560 tokens at XTR-base dimensions) and larger calls return
 * WC_E_INVALID_ARG with the limit in the message.  The first call on a device
 * looks up the array's device address (and loads the module there), so make
 * it before any stream capture.  All calls on a device share the array and
 * the handle's status word: calls that overlap on the GPU race, so serialise
 * them (one stream, or wait between calls).  If the device is reset
 * (cudaDeviceReset) the handle is gone with it; the array's address is looked
 * up again in the new context by the next call.  Errors are reported like
 * wc_t5_forward_device (check with wc_t5_sync). */
int wc_t5_forward_device_noalloc(wc_t5* h, const uint32_t* d_ids, const int32_t* d_lengths, int B, int L,
                                 float* d_out, float* d_norms, float* d_out_normalised, void* stream);

/* Wait for the handle's work on `stream` and report any in-kernel failure. */
int wc_t5_sync(wc_t5* h, void* stream);

/* Model dimensions of a handle: d_model, number of layers, output dim, vocab. */
int wc_t5_dims(const wc_t5* h, int* d_model, int* n_layers, int* d_proj, int* vocab);

/* ---- kernel-level entry points (device pointers), used by the parity tests
 *      and the microbenchmarks ---- */

/* Q4_K super-blocks -> f32, bit-exact with the reference dequant (candle
 * k_quants BlockQ4K as used at src/quantized_t5.rs:44). */
int wc_q4k_dequant(const void* d_blocks, int64_t nblocks, float* d_out, void* stream);

/* The same values rounded to f16 (nearest even): the resident weight copies
 * that the large-M GEMMs of wc_t5_forward read (the reference dequantises at
 * load too, src/quantized_t5.rs:44). */
int wc_q4k_dequant_f16(const void* d_blocks, int64_t nblocks, void* d_out_f16, void* stream);

/* Y = X . W^T with X f16 [M][K] and W Q4_K [N][K/256 blocks]
 * (QMatMul::forward, src/quantized_t5.rs:39-49; QTiledOp, src/fused_matmul.rs:46-59).
 * epilogue: 0 = f16 out [M][N]; 1 = gated GELU: gelu_tanh(X.W^T) * (X.W_up^T)
 *           as f16 [M][N] (T5DenseGatedActDense, src/quantized_t5.rs:231-252;
 *           QGatedMatMul, src/fused_matmul.rs:138-177), d_w_up required;
 *           2 = f32 residual: out[M][N] += X.W^T (src/fast_ops.rs:42-48);
 *           3 = f32 out [M][N].
 * K % 256 == 0, N % 128 == 0, M >= 1. */
int wc_gemm_q4k(const void* d_x, int M, int K, const void* d_w, const void* d_w_up, int N, int epilogue,
                void* d_out, void* stream);

/* The same GEMM and epilogues with W already dequantised to f16 [N][K]
 * (wc_q4k_dequant_f16): the kernel wc_t5_forward runs for batches of 512
 * rows and more (the 2-SM persistent GEMM).  K % 256 == 0, N % 256 == 0
 * (N % 128 == 0 for the gated GELU), M >= 1. */
int wc_gemm_f16(const void* d_x, int M, int K, const void* d_w_f16, const void* d_w_up_f16, int N, int epilogue,
                void* d_out, void* stream);

/* Encoder self-attention (src/quantized_t5.rs:426-500) over a padded batch.
 * d_qkv f16 [B*L][3*H*64] (q | k | v), d_out f16 [B*L][H*64], d_lengths
 * i32 [B], d_bias_table f32 [num_buckets][H] (relative_attention_bias),
 * 2 <= num_buckets <= 32 (T5 uses 32).
 * No 1/sqrt(d) scaling; keys >= lengths[b] are masked. */
int wc_attention(const void* d_qkv, int B, int L, int H, const int32_t* d_lengths, const float* d_bias_table,
                 int num_buckets, int max_distance, void* d_out, void* stream);

/* T5 bidirectional relative-position bucket of (query, key) as this backend
 * computes it (host side; src/quantized_t5.rs:447-483).  Returns the bucket
 * or WC_E_INVALID_ARG. */
int wc_t5_relative_bucket(int query, int key, int num_buckets, int max_distance);

/* Failure-detection self-test (no counterpart in the reference, which has no
 * device code): launches one warp whose mbarrier wait can never complete,
 * bounded by limit_ns (1e6 .. 1e10).  Returns WC_E_TIMEOUT when the kernel
 * gave up, reported it through the device status word and the CUDA context
 * stayed usable afterwards; WC_E_CUDA otherwise.  Blocks until done. */
int wc_selftest_wait_timeout(uint64_t limit_ns);

#ifdef __cplusplus
}
#endif

#endif /* WC_T5CUDA_H */
