// Host-visible declarations of the small-M (<= 32 tokens) Q4_K GEMM.
#pragma once
#include <cuda_fp16.h>

#include "gemm_q4k.h"

namespace wc {

constexpr int kGemvMaxRows = 32;

// kEpiF16 / kEpiF32 / kEpiGeGLU, 1 <= M <= 32, N % 16 == 0 (N = output
// features; for kEpiGeGLU W0 = wi_0 and W1 = wi_1, each N rows), K % 256 == 0,
// K <= 2048.
bool gemv_q4k_supports(int epi, int M, int N, int K);

// X f16 [M][K] (row stride K); W raw Q4_K rows; out [M][ldo].  f16 outputs
// clipped to the f16 range set kStatusF16Clipped in *status (may be null).
cudaError_t gemv_q4k_launch(int epi, const __half* X, int M, int K, const uint8_t* W0, const uint8_t* W1, int N,
                            void* out, int ldo, uint32_t* status, cudaStream_t st);

}  // namespace wc
