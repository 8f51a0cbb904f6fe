// Q4_K x f16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
//
//   Y[M, N] = X[M, K] . W[N, K]^T      X: f16 row-major, W: Q4_K rows
//
// replaces the reference's QMatMul::forward (candle, dequantised to f32 at
// load on CPU, src/quantized_t5.rs:39-49) and the hybrid path's
// QTiledOp / QGatedMatMul (src/fused_matmul.rs:46-59,138-177).
//
// One CTA computes a 128 x BN output tile.  Warp roles (320 threads):
//   warp 0      TMA producer: X tiles (128 x 64 f16, 128-B swizzle) and raw
//               Q4_K super-block tiles (BN rows x 144 B) into smem rings
//   warp 1      TMEM allocation + the single MMA-issuing thread
//   warps 2-9   dequant: raw Q4_K (smem) -> f16 B tiles (BN x 64, 128-B
//               swizzled, K-major) in a third ring; then the epilogue
//               (tcgen05.ld TMEM -> registers -> global)
// The f32 accumulator (128 lanes x BN columns) lives in TMEM.
//
// Epilogues:
//   kEpiF16    store f16                                 (Q/K/V projection)
//   kEpiGeGLU  gelu_tanh(gate) * up -> f16, the tile's first BN/2 columns
//              are wi_0 rows and the last BN/2 are wi_1 rows of the same
//              output features (src/quantized_t5.rs:231-252)
//   kEpiResid  x[m, n] += acc in f32 (O and wo with the residual add of
//              src/quantized_t5.rs:291,533)
//   kEpiF32    store f32 (microbench / tests)
//   kEpiProj   final 768->128 projection: raw f32 rows, their L2 norms and
//              the L2-normalised rows (src/quantized_t5.rs:700 and
//              src/embedder.rs:79-94); rows past a sequence's length are 0.
#include "common.cuh"
#include "gemm_q4k.h"
#include "q4k.cuh"

namespace wc {

template <int BN>
struct GemmCfg {
  static constexpr int BM = 128;
  static constexpr int BK = 64;
  static constexpr int SA = BN == 256 ? 3 : 4;  // X ring depth (64-wide K steps)
  static constexpr int SW = 2;                  // raw Q4_K ring depth (256-wide super-blocks)
  static constexpr int SB = BN == 256 ? 3 : 4;  // dequantised B ring depth
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int W_BYTES = BN * 144;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_W = OFF_A + SA * A_BYTES;
  static constexpr int OFF_B = OFF_W + SW * W_BYTES;
  static constexpr int OFF_BAR = OFF_B + SB * B_BYTES;
  static constexpr int SMEM = 1024 /*align slack*/ + OFF_BAR + 256;
  static constexpr int THREADS = 320;
  static_assert(W_BYTES % 1024 == 0, "raw stage must keep 1024-B alignment");
};

template <int BN, int EPI>
__global__ void __launch_bounds__(320, 1)
    gemm_q4k_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW0,
                    const __grid_constant__ CUtensorMap tmW1, GemmParams p) {
  using C = GemmCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem + C::OFF_A;
  uint8_t* sW = smem + C::OFF_W;
  uint8_t* sB = smem + C::OFF_B;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* full_a = bars;
  uint64_t* empty_a = full_a + C::SA;
  uint64_t* full_w = empty_a + C::SA;
  uint64_t* empty_w = full_w + C::SW;
  uint64_t* full_b = empty_w + C::SW;
  uint64_t* empty_b = full_b + C::SB;
  uint64_t* acc_full = empty_b + C::SB;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x;
  const int m0 = blockIdx.y * C::BM;
  const int ksteps = p.K / C::BK;
  const int kblocks = p.K / 256;

  if (warp == 0 && lane == 0) {
    for (int i = 0; i < C::SA; ++i) {
      mbar_init(&full_a[i], 1);
      mbar_init(&empty_a[i], 1);
    }
    for (int i = 0; i < C::SW; ++i) {
      mbar_init(&full_w[i], 1);
      mbar_init(&empty_w[i], 8);
    }
    for (int i = 0; i < C::SB; ++i) {
      mbar_init(&full_b[i], 8);
      mbar_init(&empty_b[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_fence_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW0);
    if (EPI == kEpiGeGLU) tma_prefetch_desc(&tmW1);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_acc = *tmem_slot;
  pdl_wait();  // every role touches activations only after this
  pdl_launch_next();  // after the wait: at most one grid waits ahead

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const int w_row0 = EPI == kEpiGeGLU ? n_tile * (BN / 2) : n_tile * BN;
      for (int t = 0; t < ksteps; ++t) {
        if ((t & 3) == 0) {
          const int kb = t >> 2;
          const int sw = kb % C::SW;
          if (!mbar_wait(&empty_w[sw], ((kb / C::SW) & 1) ^ 1, p.status)) break;
          mbar_arrive_expect_tx(&full_w[sw], C::W_BYTES);
          if (EPI == kEpiGeGLU) {
            tma_load_2d(sW + sw * C::W_BYTES, &tmW0, &full_w[sw], kb * 144, w_row0);
            tma_load_2d(sW + sw * C::W_BYTES + (BN / 2) * 144, &tmW1, &full_w[sw], kb * 144, w_row0);
          } else {
            tma_load_2d(sW + sw * C::W_BYTES, &tmW0, &full_w[sw], kb * 144, w_row0);
          }
        }
        const int sa = t % C::SA;
        if (!mbar_wait(&empty_a[sa], ((t / C::SA) & 1) ^ 1, p.status)) break;
        mbar_arrive_expect_tx(&full_a[sa], C::A_BYTES);
        tma_load_2d(sA + sa * C::A_BYTES, &tmA, &full_a[sa], t * C::BK, m0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(128, BN);
      bool ok = true;
      for (int t = 0; t < ksteps && ok; ++t) {
        const int sa = t % C::SA;
        const int sb = t % C::SB;
        ok = mbar_wait(&full_a[sa], (t / C::SA) & 1, p.status) &&
             mbar_wait(&full_b[sb], (t / C::SB) & 1, p.status);
        if (!ok) break;
        tc_fence_after();
        const uint64_t adesc = sw128_kmajor_desc(smem_u32(sA + sa * C::A_BYTES));
        const uint64_t bdesc = sw128_kmajor_desc(smem_u32(sB + sb * C::B_BYTES));
#pragma unroll
        for (int k = 0; k < C::BK / 16; ++k) {
          // advance 16 f16 (32 B) along K inside the swizzle atom
          tc_mma_f16(tmem_acc, adesc + 2 * k, bdesc + 2 * k, idesc, (t > 0 || k > 0) ? 1u : 0u);
        }
        tc_commit(&empty_a[sa]);
        tc_commit(&empty_b[sb]);
      }
      tc_commit(acc_full);
    }
  } else {
    // ------------------------------------------------------------ dequant
    const int td = threadIdx.x - 64;  // 0..255
    constexpr int ROWS_SPLIT = BN == 256 ? 1 : 2;  // threads per B row
    const int r = BN == 256 ? td : (td & (BN - 1));
    const int hsel = BN == 256 ? 0 : (td / BN);      // which nibble half this thread writes
    const int dwarp_lane0 = (lane == 0);
    bool ok = true;
    for (int kb = 0; kb < kblocks && ok; ++kb) {
      const int sw = kb % C::SW;
      ok = mbar_wait(&full_w[sw], (kb / C::SW) & 1, p.status);
      if (!ok) break;
      const uint8_t* blk = sW + sw * C::W_BYTES + r * 144;
      const Q4KScales sc = q4k_load_scales(blk);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const int t = kb * 4 + ks;
        const int sb = t % C::SB;
        ok = mbar_wait(&empty_b[sb], ((t / C::SB) & 1) ^ 1, p.status);
        if (!ok) break;
        const uint4* qp = reinterpret_cast<const uint4*>(blk + 16 + 32 * ks);
        const uint4 q0 = qp[0], q1 = qp[1];
        const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        uint8_t* bt = sB + sb * C::B_BYTES;
#pragma unroll
        for (int hh = 0; hh < 2 / ROWS_SPLIT; ++hh) {
          const int hs = ROWS_SPLIT == 1 ? hh : hsel;
          float d1, m1;
          q4k_sub_scale(sc, 2 * ks + hs, d1, m1);
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            uint32_t x0 = qw[2 * cc], x1 = qw[2 * cc + 1];
            if (hs) {
              x0 >>= 4;
              x1 >>= 4;
            }
            x0 &= 0x0F0F0F0Fu;
            x1 &= 0x0F0F0F0Fu;
            float v[8];
            q4k_dequant8(x0, x1, d1, m1, v);
            uint4 o;
            o.x = pack_f16x2(v[0], v[1]);
            o.y = pack_f16x2(v[2], v[3]);
            o.z = pack_f16x2(v[4], v[5]);
            o.w = pack_f16x2(v[6], v[7]);
            *reinterpret_cast<uint4*>(bt + sw128_offset(r, hs * 4 + cc)) = o;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (dwarp_lane0) mbar_arrive(&full_b[sb]);
      }
      __syncwarp();
      if (ok && dwarp_lane0) mbar_arrive(&empty_w[sw]);
    }

    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;                 // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;       // 0 or 1: which column half
    const int row = q * 32 + lane;
    const int m = m0 + row;
    const bool acc_ok = __all_sync(0xFFFFFFFFu, mbar_wait(acc_full, 0, p.status));
    tc_fence_after();
    bool clip = false;  // an f16 output value was clipped
    if (acc_ok) {
      const uint32_t tbase = tmem_acc + (static_cast<uint32_t>(q * 32) << 16);
      if (EPI == kEpiF16 || EPI == kEpiF32 || EPI == kEpiResid) {
        const int n_base = n_tile * BN;
#pragma unroll 1
        for (int c = half * (BN / 2); c < (half + 1) * (BN / 2); c += 32) {
          float v[32];
          tmem_ld_32x32b_x32(tbase + c, v);
          if (m < p.M) {
            if (EPI == kEpiF16) {
              __half* out = reinterpret_cast<__half*>(p.out) + static_cast<size_t>(m) * p.ldo + n_base + c;
#pragma unroll
              for (int i = 0; i < 32; i += 8) {
                uint4 o;
                o.x = pack_f16x2_sat(v[i], v[i + 1], clip);
                o.y = pack_f16x2_sat(v[i + 2], v[i + 3], clip);
                o.z = pack_f16x2_sat(v[i + 4], v[i + 5], clip);
                o.w = pack_f16x2_sat(v[i + 6], v[i + 7], clip);
                *reinterpret_cast<uint4*>(out + i) = o;
              }
            } else if (EPI == kEpiF32) {
              float* out = reinterpret_cast<float*>(p.out) + static_cast<size_t>(m) * p.ldo + n_base + c;
#pragma unroll
              for (int i = 0; i < 32; i += 4)
                *reinterpret_cast<float4*>(out + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
            } else {
              float* out = reinterpret_cast<float*>(p.out) + static_cast<size_t>(m) * p.ldo + n_base + c;
#pragma unroll
              for (int i = 0; i < 32; i += 4) {
                float4 x = *reinterpret_cast<const float4*>(out + i);
                x.x += v[i];
                x.y += v[i + 1];
                x.z += v[i + 2];
                x.w += v[i + 3];
                *reinterpret_cast<float4*>(out + i) = x;
              }
            }
          }
        }
      } else if (EPI == kEpiGeGLU) {
        const int out_base = n_tile * (BN / 2);
#pragma unroll 1
        for (int c = half * (BN / 4); c < (half + 1) * (BN / 4); c += 32) {
          float g[32], u[32];
          tmem_ld_32x32b_x32(tbase + c, g);
          tmem_ld_32x32b_x32(tbase + BN / 2 + c, u);
          if (m < p.M) {
            __half* out = reinterpret_cast<__half*>(p.out) + static_cast<size_t>(m) * p.ldo + out_base + c;
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              uint4 o;
              o.x = pack_f16x2_sat(gelu_tanh_fast(g[i]) * u[i], gelu_tanh_fast(g[i + 1]) * u[i + 1], clip);
              o.y = pack_f16x2_sat(gelu_tanh_fast(g[i + 2]) * u[i + 2], gelu_tanh_fast(g[i + 3]) * u[i + 3], clip);
              o.z = pack_f16x2_sat(gelu_tanh_fast(g[i + 4]) * u[i + 4], gelu_tanh_fast(g[i + 5]) * u[i + 5], clip);
              o.w = pack_f16x2_sat(gelu_tanh_fast(g[i + 6]) * u[i + 6], gelu_tanh_fast(g[i + 7]) * u[i + 7], clip);
              *reinterpret_cast<uint4*>(out + i) = o;
            }
          }
        }
      } else if (EPI == kEpiProj) {
        // BN == N == 128: warps of the first column half own whole rows.
        if (half == 0) {
          float v[BN];
#pragma unroll
          for (int c = 0; c < BN; c += 32) {
            float t32[32];
            tmem_ld_32x32b_x32(tbase + c, t32);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[c + i] = t32[i];
          }
          if (m < p.M) {
            bool valid = true;
            if (p.lengths != nullptr) {
              const int b = m / p.L, i = m - b * p.L;
              valid = i < p.lengths[b];
            }
            float ss = 0.f;
#pragma unroll
            for (int i = 0; i < BN; ++i) ss += v[i] * v[i];
            const float nrm = valid ? sqrtf(ss) : 0.f;
            const float inv = nrm > 0.f ? 1.0f / nrm : 0.f;
            float* out = reinterpret_cast<float*>(p.out) + static_cast<size_t>(m) * p.ldo;
            float* outn = p.out_normalised ? p.out_normalised + static_cast<size_t>(m) * p.ldo : nullptr;
#pragma unroll
            for (int i = 0; i < BN; i += 4) {
              const float4 x = valid ? make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]) : make_float4(0.f, 0.f, 0.f, 0.f);
              *reinterpret_cast<float4*>(out + i) = x;
              if (outn) *reinterpret_cast<float4*>(outn + i) = make_float4(x.x * inv, x.y * inv, x.z * inv, x.w * inv);
            }
            if (p.norms) p.norms[m] = nrm;
          }
        }
      }
    }
    report_f16_clip(clip, p.status);
  }

  // ------------------------------------------------------------ teardown
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_acc, BN);
  }
}

// ---------------------------------------------------------------- host side

template <int BN, int EPI>
static cudaError_t launch_one(const CUtensorMap& a, const CUtensorMap& w0, const CUtensorMap& w1,
                              const GemmParams& p, cudaStream_t st) {
  using C = GemmCfg<BN>;
  static bool attr_set[64] = {};  // the attribute lives in each device's context
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_q4k_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const int n_tiles = p.N / BN;
  dim3 grid(n_tiles, (p.M + C::BM - 1) / C::BM);
  return launch_pdl(gemm_q4k_kernel<BN, EPI>, grid, dim3(C::THREADS), C::SMEM, st, nullptr, 0, a, w0, w1, p);
}

int gemm_q4k_bn_for(int epi, int N) {
  if (epi == kEpiProj) return N == 128 ? 128 : -1;
  if (epi == kEpiGeGLU) return (N % 256 == 0 && N >= 1024) ? 256 : (N % 128 == 0 ? 128 : -1);
  if (epi == kEpiResid) return N % 128 == 0 ? 128 : -1;
  return (N % 256 == 0 && N >= 1536) ? 256 : (N % 128 == 0 ? 128 : -1);
}

cudaError_t gemm_q4k_launch(int epi, int bn, const CUtensorMap& a, const CUtensorMap& w0, const CUtensorMap& w1,
                            const GemmParams& p, cudaStream_t st) {
  if (bn == 256) {
    switch (epi) {
      case kEpiF16: return launch_one<256, kEpiF16>(a, w0, w1, p, st);
      case kEpiGeGLU: return launch_one<256, kEpiGeGLU>(a, w0, w1, p, st);
      case kEpiResid: return launch_one<256, kEpiResid>(a, w0, w1, p, st);
      case kEpiF32: return launch_one<256, kEpiF32>(a, w0, w1, p, st);
      default: return cudaErrorInvalidValue;
    }
  } else if (bn == 128) {
    switch (epi) {
      case kEpiF16: return launch_one<128, kEpiF16>(a, w0, w1, p, st);
      case kEpiGeGLU: return launch_one<128, kEpiGeGLU>(a, w0, w1, p, st);
      case kEpiResid: return launch_one<128, kEpiResid>(a, w0, w1, p, st);
      case kEpiF32: return launch_one<128, kEpiF32>(a, w0, w1, p, st);
      case kEpiProj: return launch_one<128, kEpiProj>(a, w0, w1, p, st);
      default: return cudaErrorInvalidValue;
    }
  }
  return cudaErrorInvalidValue;
}

}  // namespace wc
