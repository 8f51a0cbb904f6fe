// Small-M Q4_K GEMM (M <= 32 tokens: queries, short documents).
//
// With few tokens the layer GEMMs are weight-streaming problems: every weight
// is used M times, so the work is spread over as many SMs as possible and each
// weight is dequantised exactly once.  One CTA owns 16 weight rows (output
// features) -- for the gated GELU 16 wi_0 rows and the same 16 wi_1 rows --
// and all M tokens; its 4 warps split K by Q4_K super-block.  A warp copies
// (cp.async, all at once) the raw super-blocks of its rows to shared memory,
// dequantises them straight
// into the A-operand registers of mma.sync m16n8k16 (weights x tokens, f16 in,
// f32 accumulate; the activations, staged once per CTA in shared memory, are
// the B operand), and the 4 warps' partial sums are added in shared memory
// before the epilogue.  Dequant arithmetic is the exact reference formula
// (see q4k.cuh) rounded to f16, as in the large-M kernels.
#include "gemv_q4k.h"
#include "gemv_tile.cuh"

namespace wc {

namespace {

constexpr int kWarps = kGemvWarps;
constexpr int kRows = kGemvRows;

// MT: 8-token column tiles (M <= 8 * MT).  One CTA per 16-row tile.
template <int EPI, int MT>
__global__ void __launch_bounds__(kWarps * 32) gemv_q4k_kernel(const __half* __restrict__ X, int M, int K,
                                                               const uint8_t* __restrict__ W0,
                                                               const uint8_t* __restrict__ W1, void* __restrict__ out,
                                                               int ldo, uint32_t* __restrict__ status) {
  constexpr int NMAT = EPI == kEpiGeGLU ? 2 : 1;
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* sX = smem;
  uint8_t* sW = smem + gemv_sx_bytes(MT * 8, K);
  float* sRed = reinterpret_cast<float*>(sW + gemv_sw_bytes(NMAT, K));
  const int row0 = blockIdx.x * kRows;
  // Everything this CTA reads is requested up front with cp.async and waited
  // for once; the raw weights are constant, so they are requested before
  // waiting for the previous kernel, the activations after.
  gemv_issue_weights<NMAT>(W0, W1, K, row0, sW);
  pdl_wait();
  pdl_launch_next();  // after the wait: at most one grid waits ahead
  gemv_issue_x<MT>(X, M, K, sX);
  gv_cp_async_wait_all();
  __syncthreads();
  gemv_tile_compute<EPI, MT>(sX, M, K, sW, sRed, out, ldo, row0, status);
}

template <int EPI, int MT>
cudaError_t launch(const __half* X, int M, int K, const uint8_t* W0, const uint8_t* W1, int N, void* out, int ldo,
                   uint32_t* status, cudaStream_t st) {
  constexpr int NMAT = EPI == kEpiGeGLU ? 2 : 1;
  const size_t smem = gemv_sx_bytes(MT * 8, K) + gemv_sw_bytes(NMAT, K) + gemv_red_bytes(NMAT, MT * 8);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(gemv_q4k_kernel<EPI, MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  return launch_pdl(gemv_q4k_kernel<EPI, MT>, dim3(N / kRows), dim3(kWarps * 32), smem, st, nullptr, 0, X, M, K, W0,
                    W1, out, ldo, status);
}

template <int EPI>
cudaError_t launch_mt(const __half* X, int M, int K, const uint8_t* W0, const uint8_t* W1, int N, void* out, int ldo,
                      uint32_t* status, cudaStream_t st) {
  if (M <= 8) return launch<EPI, 1>(X, M, K, W0, W1, N, out, ldo, status, st);
  if (M <= 16) return launch<EPI, 2>(X, M, K, W0, W1, N, out, ldo, status, st);
  return launch<EPI, 4>(X, M, K, W0, W1, N, out, ldo, status, st);
}

}  // namespace

bool gemv_q4k_supports(int epi, int M, int N, int K) {
  return (epi == kEpiF16 || epi == kEpiF32 || epi == kEpiGeGLU) && M >= 1 && M <= kGemvMaxRows && N % kRows == 0 &&
         K % 256 == 0 && K <= 2048;
}

cudaError_t gemv_q4k_launch(int epi, const __half* X, int M, int K, const uint8_t* W0, const uint8_t* W1, int N,
                            void* out, int ldo, uint32_t* status, cudaStream_t st) {
  switch (epi) {
    case kEpiF16: return launch_mt<kEpiF16>(X, M, K, W0, W1, N, out, ldo, status, st);
    case kEpiF32: return launch_mt<kEpiF32>(X, M, K, W0, W1, N, out, ldo, status, st);
    case kEpiGeGLU: return launch_mt<kEpiGeGLU>(X, M, K, W0, W1, N, out, ldo, status, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace wc
