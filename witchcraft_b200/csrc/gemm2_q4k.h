// Host-visible declarations of the 2-SM (cta_group::2) persistent Q4_K GEMM.
#pragma once
#include "gemm_q4k.h"

namespace wc {

// Rows of W one TMA box covers in the 2-SM kernel (each CTA's half of a
// 256-column tile); its raw-weight tensor maps are encoded with this height.
constexpr int kGemm2WBoxRows = 128;

// True when the 2-SM kernel handles this epilogue and shape (N % 256 == 0,
// K % 256 == 0; N is tile-space: 2 x features for kEpiGeGLU).
bool gemm2_q4k_supports(int epi, int M, int N, int K);

// Persistent launch over min(tiles, num_sms / 2) clusters of 2 CTAs.  `out`
// is the TMA descriptor of the output matrix p.out ([M][ldo]; box 64 x 32
// for f16 outputs, 32 x 32 for the f32 kEpiF32 / kEpiResid, 128-byte
// swizzle); kEpiResid adds into the residual x through it (TMA reduce-add).  w0 / w1
// describe raw Q4_K rows (box kGemm2WBoxRows rows of super-blocks), or with
// w_f16 the same weights dequantised to f16 [N][K] (box 64 x kGemm2WBoxRows,
// 128-byte swizzle, like an activation map).
// bn = 128 (kEpiResid / kEpiF32 on f16 weights only; weight maps with a 64-row box)
// halves the tile width, for batches whose 256-column tiles would leave
// clusters idle (N = 768 at a few thousand rows).
// Tile width for the f32 epilogues on f16 weights: 128 only when every
// 128-column tile fits in one round of clusters (N = 768 up to 2,368 rows).
// Past that, half-width tiles load 1.5x the operand bytes per MMA cycle, and
// the operand feed from L2 already bounds these GEMMs: measured at M = 4096,
// O took 12.9 us with 128-column tiles against 11.1 us with 256.
int gemm2_resid_bn(int M, int N, int num_sms);

cudaError_t gemm2_q4k_launch(int epi, const CUtensorMap& a, const CUtensorMap& w0, const CUtensorMap& w1,
                             const CUtensorMap& out, const GemmParams& p, int num_sms, cudaStream_t st,
                             bool w_f16 = false, int bn = 256);

}  // namespace wc
