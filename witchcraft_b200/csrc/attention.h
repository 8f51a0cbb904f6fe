// Host-visible declarations of the encoder attention kernel.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace wc {

// The T5 bidirectional bucket function of |key - query| is monotone, so it is
// carried to the device as thresholds: bucket_half(d) = #{v in [1, half) :
// thr[v] <= d}, plus `half` when the key comes after the query.  The host
// derives thr[] from the reference's own f32 formula (see t5_buckets.h), so no
// device logarithm ever decides a bucket.
struct BucketThresholds {
  int half;      // num_buckets / 2
  int thr[32];   // thr[v] = smallest distance d with bucket_half(d) >= v
};

// qkv: [B*L][3*H*64] f16 (q | k | v); out: [B*L][H*64] f16;
// lengths: device [B]; bias_tab: device f32 [num_buckets][H].
cudaError_t attention_launch(const __half* qkv, __half* out, const int32_t* lengths, int B, int L,
                             int H, const float* bias_tab, const BucketThresholds& bt, cudaStream_t st);

}  // namespace wc
