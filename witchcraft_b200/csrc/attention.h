// Host-visible declarations of the encoder attention kernel (attention_tc.cu).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace wc {

// The T5 bidirectional bucket function of |key - query| is monotone, so it is
// carried to the device as thresholds: bucket_half(d) = #{v in [1, half) :
// thr[v] <= d}, plus `half` when the key comes after the query.  The host
// derives thr[] from the reference's own f32 formula (t5_bucket_thresholds in t5_host.h), so no
// device logarithm ever decides a bucket.
struct BucketThresholds {
  int half;      // num_buckets / 2
  int thr[32];   // thr[v] = smallest distance d with bucket_half(d) >= v
};

// tcgen05 attention: tm_qkv is the TMA descriptor of the QKV projection
// [B*L][3*H*64] f16 (box 64 x 64, 128-byte swizzle); L <= 2048.
cudaError_t attention_tc_launch(const CUtensorMap& tm_qkv, __half* out, const int32_t* lengths, int B, int L, int H,
                                const float* bias_tab, const BucketThresholds& bt, uint32_t* status, cudaStream_t st);

// Short padded batches (1 <= L <= 64, the query path): mma.sync kernel over
// the raw QKV pointer, one CTA per (sequence, head).
bool attention_small_supports(int L);
cudaError_t attention_small_launch(const __half* qkv, __half* out, const int32_t* lengths, int B, int L, int H,
                                   const float* bias_tab, const BucketThresholds& bt, cudaStream_t st);

}  // namespace wc
