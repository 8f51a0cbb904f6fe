// Encoder self-attention for short padded batches (L <= 64: the query path),
// the same computation as attention_tc.cu (src/quantized_t5.rs:426-500:
// scores without 1/sqrt(d), + relative-position bias, key padding mask,
// softmax, P.V) with warp-level mma.sync instead of the tcgen05 pipeline.
// At L <= 64 a 128-query tcgen05 tile is mostly padding and the kernel is
// bound by its per-step handshake latency; here one CTA owns one (sequence,
// head), each warp takes 16 queries, and everything after the loads stays in
// registers.  The padded tile is KL = 32 or 64 rows (L <= 32 takes the
// smaller one: half the shared memory and warps per CTA, so twice as many
// CTAs keep their loads in flight on an SM).
//
// Per CTA: Q, K, V of the head (rows past L zero) in padded shared memory
// (144-byte rows: conflict-free ldmatrix), the head's bias for every
// key - query offset (|delta| <= 63), pre-scaled by log2(e).  Per warp: S =
// Q K^T (m16n8k16, f16 in, f32 out) over all 64 keys, v = S log2(e) + bias,
// keys past the sequence at -inf, row max / sum across the quad, P = 2^(v -
// max) rounded to f16 straight into the A fragments of O = P V (V through
// ldmatrix.trans), O / sum to f16.  A sequence of length 0 gets zero rows.
#include "attention_small.cuh"

namespace wc {

namespace {

constexpr int kL = 64;  // max padded length handled here

template <int KL>
__global__ void __launch_bounds__(KL * 2)
    attention_small_kernel(const __half* __restrict__ qkv, __half* __restrict__ out,
                           const int32_t* __restrict__ lengths, int L, int H, const float* __restrict__ bias_tab,
                           BucketThresholds bt) {
  __shared__ __align__(16) uint8_t smem[attn_small::smem_bytes(KL)];
  // the item waits for the previous kernel once its bias row is built
  attn_small::item<KL>(qkv, out, lengths, L, H, bias_tab, bt, blockIdx.y, blockIdx.x, smem, true);
}

}  // namespace

bool attention_small_supports(int L) { return L >= 1 && L <= kL; }

cudaError_t attention_small_launch(const __half* qkv, __half* out, const int32_t* lengths, int B, int L, int H,
                                   const float* bias_tab, const BucketThresholds& bt, cudaStream_t st) {
  if (B <= 0) return cudaSuccess;
  if (!attention_small_supports(L) || H <= 0 || H > 65535 || B > 65535) return cudaErrorInvalidValue;
  if (L <= 32)
    return launch_pdl(attention_small_kernel<32>, dim3(H, B), dim3(64), 0, st, nullptr, 0, qkv, out, lengths, L, H,
                      bias_tab, bt);
  return launch_pdl(attention_small_kernel<64>, dim3(H, B), dim3(128), 0, st, nullptr, 0, qkv, out, lengths, L, H,
                    bias_tab, bt);
}

}  // namespace wc
