// Host-visible declarations of the memory-bound kernels: Q4_K dequant,
// embedding gather (+ the first RMSNorm) and RMSNorm.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace wc {

// nblocks Q4_K super-blocks -> 256 * nblocks f32, bit-exact with the reference.
cudaError_t q4k_dequant_launch(const uint8_t* blocks, int64_t nblocks, float* out, cudaStream_t st);
// Same, rounded to f16 (round to nearest even).
cudaError_t q4k_dequant_f16_launch(const uint8_t* blocks, int64_t nblocks, __half* out, cudaStream_t st);

// x[m] = dequant(table row ids[m]) (id 0 for positions past a sequence's
// valid length), xn[m] = f16(RMSNorm(x[m]) * w).  table: Q4_K [vocab][D/256].
cudaError_t embed_rmsnorm_launch(const uint8_t* table, const uint32_t* ids, const int32_t* lengths, int L, int M,
                                 int D, const float* w, float eps, float* x, __half* xn, uint32_t* status,
                                 cudaStream_t st);

// With delta != null first x[m] += delta[m] (the residual add, written back);
// then y[m] = f16(x[m] / sqrt(mean(x[m]^2) + eps) * w), D % 128 == 0.
// Both norms set kStatusF16Clipped in *status (may be null) when an output
// value was clipped to the f16 range.
cudaError_t rmsnorm_launch(float* x, const float* delta, const float* w, __half* y, int M, int D, float eps,
                           uint32_t* status, cudaStream_t st);

// One warp waits on an mbarrier nobody arrives on, for at most limit_ns; the
// timeout sets kStatusWaitTimeout in *status.
cudaError_t wait_timeout_selftest_launch(uint32_t* status, uint64_t limit_ns, cudaStream_t st);

}  // namespace wc
