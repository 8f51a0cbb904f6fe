// Host-visible declarations of the Q4_K x f16 tcgen05 GEMM.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace wc {

enum GemmEpilogue : int { kEpiF16 = 0, kEpiGeGLU = 1, kEpiResid = 2, kEpiF32 = 3, kEpiProj = 4 };

struct GemmParams {
  int M;                    // rows of X / Y
  int N;                    // tile-space columns (for kEpiGeGLU: 2 x output features)
  int K;                    // multiple of 256
  void* out;                // f16 or f32 [M, ldo]; for kEpiResid the f32 residual stream (read + written)
  int ldo;                  // elements
  float* norms;             // kEpiProj: [M] L2 norm of each raw row (may be null)
  float* out_normalised;    // kEpiProj: [M, ldo] normalised rows (may be null)
  const int32_t* lengths;   // kEpiProj: per-sequence valid lengths (null = all rows valid)
  int L;                    // kEpiProj: padded sequence length (rows per sequence)
  uint32_t* status;         // device status word (wait timeouts)
};

// BN (128 or 256) the launcher uses for an epilogue and tile-space width N,
// or -1 when N is unsupported.
int gemm_q4k_bn_for(int epi, int N);

// Rows of W one TMA box covers for (epi, bn): the raw-weight tensor maps must
// be encoded with this box height.
inline int gemm_q4k_w_box_rows(int epi, int bn) { return epi == kEpiGeGLU ? bn / 2 : bn; }

// a: X map (f16 [M][K], box 64 x 128, 128-B swizzle); w0 (and w1 for
// kEpiGeGLU): raw Q4_K maps (uint8 [rows][K/256*144], box 144 x box_rows).
cudaError_t gemm_q4k_launch(int epi, int bn, const CUtensorMap& a, const CUtensorMap& w0, const CUtensorMap& w1,
                            const GemmParams& p, cudaStream_t st);

}  // namespace wc
