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
#include "common.cuh"
#include "gemv_q4k.h"
#include "q4k.cuh"

namespace wc {

namespace {

constexpr int kWarps = 4;
constexpr int kRows = 16;  // weight rows per CTA (per matrix)

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(pred ? 16 : 0)
               : "memory");
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Two consecutive weights of one row as f16x2: the nibbles (4*hs) of bytes
// p[0], p[1] of the qs run, value d1*q - m1 rounded once.
__device__ __forceinline__ uint32_t dq2(const uint8_t* p, int hs, float d1, float m1) {
  const uint32_t b = *reinterpret_cast<const uint16_t*>(p);
  const uint32_t x = (b >> (4 * hs)) & 0x0F0Fu;
  return pack_f16x2(fmaf(d1, nib_to_float(x, 0), -m1), fmaf(d1, nib_to_float(x, 1), -m1));
}

// MT: 8-token column tiles (M <= 8 * MT); NMAT: 1, or 2 for the gated GELU.
template <int EPI, int MT>
__global__ void __launch_bounds__(kWarps * 32) gemv_q4k_kernel(const __half* __restrict__ X, int M, int K,
                                                               const uint8_t* __restrict__ W0,
                                                               const uint8_t* __restrict__ W1, void* __restrict__ out,
                                                               int ldo) {
  constexpr int NMAT = EPI == kEpiGeGLU ? 2 : 1;
  constexpr int TOK = MT * 8;
  extern __shared__ __align__(16) uint8_t smem[];
  const int xstride = K * 2 + 16;  // bytes per token row (padded: conflict-free ldmatrix)
  uint8_t* sX = smem;
  uint8_t* sW = smem + TOK * xstride;  // [warp][its super-blocks][NMAT*16 rows][144]
  float* sRed = reinterpret_cast<float*>(sW + ((K / 256 + kWarps - 1) / kWarps) * kWarps * NMAT * kRows * 144);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row0 = blockIdx.x * kRows;
  const int kblocks = K / 256;
  const size_t wrow_bytes = static_cast<size_t>(kblocks) * 144;

  // Everything this CTA reads is requested up front with cp.async (the
  // activations, TOK rows with rows >= M zero-filled, and every raw
  // super-block of this warp's rows), then waited for once.
  const int kb_per_warp = (kblocks + kWarps - 1) / kWarps;
  uint8_t* myW = sW + warp * kb_per_warp * NMAT * kRows * 144;
  // the raw weights are constant: request them before waiting for the
  // previous kernel, the activations after
  for (int s = 0; s < kb_per_warp; ++s) {
    const int kb = warp + s * kWarps;
    if (kb >= kblocks) break;
    for (int i = lane; i < NMAT * kRows * 9; i += 32) {
      const int rr = i / 9, c = i % 9;
      const uint8_t* src = (rr < kRows ? W0 : W1) + (row0 + (rr % kRows)) * wrow_bytes + kb * 144 + c * 16;
      cp_async16(myW + (s * NMAT * kRows + rr) * 144 + c * 16, src, true);
    }
  }
  pdl_wait();
  pdl_launch_next();  // after the wait: at most one grid waits ahead
  for (int i = tid; i < TOK * (K / 8); i += blockDim.x) {
    const int r = i / (K / 8), c = i % (K / 8);
    cp_async16(sX + r * xstride + c * 16, X + static_cast<size_t>(r < M ? r : 0) * K + c * 8, r < M);
  }
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
  __syncthreads();

  float acc[NMAT][MT][4];
#pragma unroll
  for (int m = 0; m < NMAT; ++m)
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[m][t][0] = acc[m][t][1] = acc[m][t][2] = acc[m][t][3] = 0.f;

  const int g = lane >> 2, tq = lane & 3;
  for (int s = 0; s < kb_per_warp; ++s) {
    const int kb = warp + s * kWarps;
    if (kb >= kblocks) break;
    const uint8_t* wblk = myW + s * NMAT * kRows * 144;
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
      const uint8_t* blkA = wblk + (m * kRows + g) * 144;      // row g
      const uint8_t* blkB = wblk + (m * kRows + g + 8) * 144;  // row g + 8
      const Q4KScales sa = q4k_load_scales(blkA);
      const Q4KScales sb = q4k_load_scales(blkB);
#pragma unroll
      for (int j = 0; j < 16; ++j) {  // 16-wide K steps of the super-block
        const int c = j >> 2, hs = (j >> 1) & 1, lb = 16 * (j & 1) + 2 * tq;
        float dA, mA, dB, mB;
        q4k_sub_scale(sa, 2 * c + hs, dA, mA);
        q4k_sub_scale(sb, 2 * c + hs, dB, mB);
        uint32_t a[4];
        a[0] = dq2(blkA + 16 + 32 * c + lb, hs, dA, mA);
        a[1] = dq2(blkB + 16 + 32 * c + lb, hs, dB, mB);
        a[2] = dq2(blkA + 16 + 32 * c + lb + 8, hs, dA, mA);
        a[3] = dq2(blkB + 16 + 32 * c + lb + 8, hs, dB, mB);
        const int k0 = kb * 256 + 16 * j;
#pragma unroll
        for (int tp = 0; tp < MT; tp += 2) {
          const int tok = tp * 8 + (lane & 7) + ((lane >> 4) << 3);
          const int kk = k0 + (((lane >> 3) & 1) << 3);
          uint32_t b0, b1, b2, b3;
          if (MT == 1) {
            // one 8-token tile: lanes 16-31 repeat lanes 0-15's addresses
            const int tok1 = lane & 7;
            ldmatrix_x4(smem_u32(sX + tok1 * xstride + kk * 2), b0, b1, b2, b3);
            mma16816(acc[m][0], a, b0, b1);
          } else {
            ldmatrix_x4(smem_u32(sX + tok * xstride + kk * 2), b0, b1, b2, b3);
            mma16816(acc[m][tp], a, b0, b1);
            mma16816(acc[m][tp + 1], a, b2, b3);
          }
        }
      }
    }
  }

  // partial sums of the 4 warps -> smem, then reduce + epilogue
#pragma unroll
  for (int m = 0; m < NMAT; ++m)
#pragma unroll
    for (int t = 0; t < MT; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int f = g + ((e >> 1) << 3);
        const int tok = t * 8 + 2 * tq + (e & 1);
        sRed[((warp * NMAT + m) * kRows + f) * TOK + tok] = acc[m][t][e];
      }
  __syncthreads();
  for (int i = tid; i < kRows * M; i += blockDim.x) {
    const int f = i % kRows, tok = i / kRows;
    float v[NMAT];
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) s += sRed[((w * NMAT + m) * kRows + f) * TOK + tok];
      v[m] = s;
    }
    const size_t o = static_cast<size_t>(tok) * ldo + row0 + f;
    if (EPI == kEpiGeGLU) {
      const float h = gelu_tanh_fast(v[0]) * v[NMAT - 1];
      reinterpret_cast<__half*>(out)[o] = __float2half_rn(fminf(fmaxf(h, -65504.f), 65504.f));
    } else if (EPI == kEpiF16) {
      reinterpret_cast<__half*>(out)[o] = __float2half_rn(fminf(fmaxf(v[0], -65504.f), 65504.f));
    } else {
      reinterpret_cast<float*>(out)[o] = v[0];
    }
  }
}

template <int EPI, int MT>
cudaError_t launch(const __half* X, int M, int K, const uint8_t* W0, const uint8_t* W1, int N, void* out, int ldo,
                   cudaStream_t st) {
  constexpr int NMAT = EPI == kEpiGeGLU ? 2 : 1;
  const int kb_per_warp = (K / 256 + kWarps - 1) / kWarps;
  const size_t smem = static_cast<size_t>(MT * 8) * (K * 2 + 16) + kb_per_warp * kWarps * NMAT * kRows * 144 +
                      kWarps * NMAT * kRows * MT * 8 * 4;
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
                    W1, out, ldo);
}

template <int EPI>
cudaError_t launch_mt(const __half* X, int M, int K, const uint8_t* W0, const uint8_t* W1, int N, void* out, int ldo,
                      cudaStream_t st) {
  if (M <= 8) return launch<EPI, 1>(X, M, K, W0, W1, N, out, ldo, st);
  if (M <= 16) return launch<EPI, 2>(X, M, K, W0, W1, N, out, ldo, st);
  return launch<EPI, 4>(X, M, K, W0, W1, N, out, ldo, st);
}

}  // namespace

bool gemv_q4k_supports(int epi, int M, int N, int K) {
  return (epi == kEpiF16 || epi == kEpiF32 || epi == kEpiGeGLU) && M >= 1 && M <= kGemvMaxRows && N % kRows == 0 &&
         K % 256 == 0 && K <= 2048;
}

cudaError_t gemv_q4k_launch(int epi, const __half* X, int M, int K, const uint8_t* W0, const uint8_t* W1, int N,
                            void* out, int ldo, cudaStream_t st) {
  switch (epi) {
    case kEpiF16: return launch_mt<kEpiF16>(X, M, K, W0, W1, N, out, ldo, st);
    case kEpiF32: return launch_mt<kEpiF32>(X, M, K, W0, W1, N, out, ldo, st);
    case kEpiGeGLU: return launch_mt<kEpiGeGLU>(X, M, K, W0, W1, N, out, ldo, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace wc
