// Device-side pieces of the small-M Q4_K GEMM (gemv_q4k.cu), as device
// functions a kernel can call per 16-row tile.
//
// One tile = 16 weight rows (output features; for the gated GELU 16 wi_0 rows
// and the same 16 wi_1 rows) x all M <= 8 MT tokens.  The CTA's 4 warps split
// K by Q4_K super-block: a warp copies (cp.async) the raw super-blocks of its
// rows to shared memory, dequantises them straight into the A-operand
// registers of mma.sync m16n8k16 (weights x tokens, f16 in, f32 accumulate;
// the activations, staged once per CTA in shared memory, are the B operand),
// and the 4 warps' partial sums are added in shared memory before the
// epilogue.  Dequant arithmetic is the exact reference formula (q4k.cuh)
// rounded to f16, as in the large-M kernels.
//
// Shared memory of a tile: [sX: 8 MT token rows of K f16 + 16 B padding]
// [sW: the warps' raw super-blocks] [sRed: the warps' partial sums].
#pragma once
#include "common.cuh"
#include "gemm_q4k.h"
#include "q4k.cuh"

namespace wc {

constexpr int kGemvWarps = 4;
constexpr int kGemvRows = 16;  // weight rows per tile (per matrix)

__host__ __device__ constexpr int gemv_xstride(int K) { return K * 2 + 16; }  // conflict-free ldmatrix rows
__host__ __device__ constexpr int gemv_kb_per_warp(int K) { return (K / 256 + kGemvWarps - 1) / kGemvWarps; }
__host__ __device__ constexpr size_t gemv_sx_bytes(int tok, int K) { return static_cast<size_t>(tok) * gemv_xstride(K); }
__host__ __device__ constexpr size_t gemv_sw_bytes(int nmat, int K) {
  return static_cast<size_t>(gemv_kb_per_warp(K)) * kGemvWarps * nmat * kGemvRows * 144;
}
__host__ __device__ constexpr size_t gemv_red_bytes(int nmat, int tok) {
  return static_cast<size_t>(kGemvWarps) * nmat * kGemvRows * tok * 4;
}

__device__ __forceinline__ void gv_ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                               uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void gv_cp_async16(void* dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(pred ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void gv_cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void gv_mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Two consecutive weights of one row as f16x2: the nibbles (4*hs) of bytes
// p[0], p[1] of the qs run, value d1*q - m1 rounded once.
__device__ __forceinline__ uint32_t gv_dq2(const uint8_t* p, int hs, float d1, float m1) {
  const uint32_t b = *reinterpret_cast<const uint16_t*>(p);
  const uint32_t x = (b >> (4 * hs)) & 0x0F0Fu;
  return pack_f16x2(fmaf(d1, nib_to_float(x, 0), -m1), fmaf(d1, nib_to_float(x, 1), -m1));
}

// cp.async (not waited) of the raw super-blocks this warp owns: rows
// [row0, row0 + 16) of W0 (and W1), K blocks warp, warp + 4, ...
template <int NMAT>
__device__ __forceinline__ void gemv_issue_weights(const uint8_t* __restrict__ W0, const uint8_t* __restrict__ W1,
                                                   int K, int row0, uint8_t* sW) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kblocks = K / 256, kbpw = gemv_kb_per_warp(K);
  const size_t wrow_bytes = static_cast<size_t>(kblocks) * 144;
  uint8_t* myW = sW + warp * kbpw * NMAT * kGemvRows * 144;
  for (int s = 0; s < kbpw; ++s) {
    const int kb = warp + s * kGemvWarps;
    if (kb >= kblocks) break;
    for (int i = lane; i < NMAT * kGemvRows * 9; i += 32) {
      const int rr = i / 9, c = i % 9;
      const uint8_t* src =
          (rr < kGemvRows ? W0 : W1) + (row0 + (rr % kGemvRows)) * wrow_bytes + kb * 144 + c * 16;
      gv_cp_async16(myW + (s * NMAT * kGemvRows + rr) * 144 + c * 16, src, true);
    }
  }
}

// cp.async (not waited) of the activations: 8 MT token rows of X [M][K] f16,
// rows >= M zero-filled.
template <int MT>
__device__ __forceinline__ void gemv_issue_x(const __half* __restrict__ X, int M, int K, uint8_t* sX) {
  const int xstride = gemv_xstride(K);
  for (int i = threadIdx.x; i < MT * 8 * (K / 8); i += blockDim.x) {
    const int r = i / (K / 8), c = i % (K / 8);
    gv_cp_async16(sX + r * xstride + c * 16, X + static_cast<size_t>(r < M ? r : 0) * K + c * 8, r < M);
  }
}

// The tile's MMAs, the reduction of the 4 warps' partial sums and the
// epilogue, once sX and sW hold their data (the caller waits for its
// cp.async groups and syncs the CTA first).  Ends with every thread done
// with sX, sW and sRed.
template <int EPI, int MT>
__device__ __forceinline__ void gemv_tile_compute(const uint8_t* sX, int M, int K, const uint8_t* sW, float* sRed,
                                                  void* __restrict__ out, int ldo, int row0,
                                                  uint32_t* __restrict__ status) {
  constexpr int NMAT = EPI == kEpiGeGLU ? 2 : 1;
  constexpr int TOK = MT * 8;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int xstride = gemv_xstride(K);
  const int kblocks = K / 256, kbpw = gemv_kb_per_warp(K);
  const uint8_t* myW = sW + warp * kbpw * NMAT * kGemvRows * 144;

  float acc[NMAT][MT][4];
#pragma unroll
  for (int m = 0; m < NMAT; ++m)
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[m][t][0] = acc[m][t][1] = acc[m][t][2] = acc[m][t][3] = 0.f;

  const int g = lane >> 2, tq = lane & 3;
  for (int s = 0; s < kbpw; ++s) {
    const int kb = warp + s * kGemvWarps;
    if (kb >= kblocks) break;
    const uint8_t* wblk = myW + s * NMAT * kGemvRows * 144;
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
      const uint8_t* blkA = wblk + (m * kGemvRows + g) * 144;      // row g
      const uint8_t* blkB = wblk + (m * kGemvRows + g + 8) * 144;  // row g + 8
      const Q4KScales sa = q4k_load_scales(blkA);
      const Q4KScales sb = q4k_load_scales(blkB);
#pragma unroll
      for (int j = 0; j < 16; ++j) {  // 16-wide K steps of the super-block
        const int c = j >> 2, hs = (j >> 1) & 1, lb = 16 * (j & 1) + 2 * tq;
        float dA, mA, dB, mB;
        q4k_sub_scale(sa, 2 * c + hs, dA, mA);
        q4k_sub_scale(sb, 2 * c + hs, dB, mB);
        uint32_t a[4];
        a[0] = gv_dq2(blkA + 16 + 32 * c + lb, hs, dA, mA);
        a[1] = gv_dq2(blkB + 16 + 32 * c + lb, hs, dB, mB);
        a[2] = gv_dq2(blkA + 16 + 32 * c + lb + 8, hs, dA, mA);
        a[3] = gv_dq2(blkB + 16 + 32 * c + lb + 8, hs, dB, mB);
        const int k0 = kb * 256 + 16 * j;
#pragma unroll
        for (int tp = 0; tp < MT; tp += 2) {
          const int tok = tp * 8 + (lane & 7) + ((lane >> 4) << 3);
          const int kk = k0 + (((lane >> 3) & 1) << 3);
          uint32_t b0, b1, b2, b3;
          if (MT == 1) {
            // one 8-token tile: lanes 16-31 repeat lanes 0-15's addresses
            const int tok1 = lane & 7;
            gv_ldmatrix_x4(smem_u32(sX + tok1 * xstride + kk * 2), b0, b1, b2, b3);
            gv_mma16816(acc[m][0], a, b0, b1);
          } else {
            gv_ldmatrix_x4(smem_u32(sX + tok * xstride + kk * 2), b0, b1, b2, b3);
            gv_mma16816(acc[m][tp], a, b0, b1);
            gv_mma16816(acc[m][tp + 1], a, b2, b3);
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
        sRed[((warp * NMAT + m) * kGemvRows + f) * TOK + tok] = acc[m][t][e];
      }
  __syncthreads();
  bool clip = false;  // an f16 output value was clipped
  for (int i = tid; i < kGemvRows * M; i += blockDim.x) {
    const int f = i % kGemvRows, tok = i / kGemvRows;
    float v[NMAT];
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kGemvWarps; ++w) s += sRed[((w * NMAT + m) * kGemvRows + f) * TOK + tok];
      v[m] = s;
    }
    const size_t o = static_cast<size_t>(tok) * ldo + row0 + f;
    if (EPI == kEpiGeGLU) {
      const float h = gelu_tanh_fast(v[0]) * v[NMAT - 1];
      clip |= f16_clips(h);
      reinterpret_cast<__half*>(out)[o] = __float2half_rn(fminf(fmaxf(h, -65504.f), 65504.f));
    } else if (EPI == kEpiF16) {
      clip |= f16_clips(v[0]);
      reinterpret_cast<__half*>(out)[o] = __float2half_rn(fminf(fmaxf(v[0], -65504.f), 65504.f));
    } else {
      reinterpret_cast<float*>(out)[o] = v[0];
    }
  }
  report_f16_clip(clip, status);
  __syncthreads();
}

}  // namespace wc
