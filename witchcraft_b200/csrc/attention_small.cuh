// Device body of the short-sequence encoder attention (attention_small.cu):
// one (sequence, head) item for padded L <= KL rows, KL = 32 or 64, by a CTA
// of at least 2 KL threads (one warp per 16 queries; extra warps only help
// with the loads), as a device function; the stand-alone kernel runs one
// item per CTA.
#pragma once
#include "attention.h"
#include "common.cuh"

namespace wc {
namespace attn_small {


constexpr int kDh = 64;
constexpr int kRowB = kDh * 2 + 16;  // padded row bytes

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ float ex2s(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void cp16s(uint32_t dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(pred ? 16 : 0)
               : "memory");
}

__device__ __forceinline__ int bucket_of(const BucketThresholds& bt, int delta) {
  const int d = delta < 0 ? -delta : delta;
  int f = 0;
  for (int v = 1; v < 32 && v < bt.half; ++v) f += d >= bt.thr[v] ? 1 : 0;
  return f + (delta > 0 ? bt.half : 0);
}


// Shared memory of one item: Q, K, V rows (144-byte padded rows), the bias by
// key - query offset, the head's bias-table column.
__host__ __device__ constexpr int smem_bytes(int KL) { return 3 * KL * kRowB + (2 * KL + 64) * 4; }

template <int KL>
__device__ __forceinline__ void item(const __half* __restrict__ qkv, __half* __restrict__ out,
                                     const int32_t* __restrict__ lengths, int L, int H,
                                     const float* __restrict__ bias_tab, const BucketThresholds& bt, int b, int h,
                                     uint8_t* smem, bool pdl) {
  uint8_t* sQ = smem;
  uint8_t* sK = smem + KL * kRowB;
  uint8_t* sV = smem + 2 * KL * kRowB;
  float* sBias = reinterpret_cast<float*>(smem + 3 * KL * kRowB);  // bias(key - query = delta) at delta + KL - 1, * log2(e)
  float* sCol = sBias + 2 * KL;                                    // this head's column of the bias table
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, kT = blockDim.x;
  const int len = min(max(lengths[b], 0), L);
  const int inner = H * kDh;
  const size_t row0 = static_cast<size_t>(b) * L;
  // the bias row reads only weights and the launch's thresholds: with pdl it
  // is built before the wait for the previous kernel (which writes qkv)
  if (tid < 2 * bt.half) sCol[tid] = bias_tab[tid * H + h] * 1.4426950408889634f;
  __syncthreads();
  for (int i = tid; i < 2 * KL - 1; i += kT) sBias[i] = sCol[bucket_of(bt, i - (KL - 1))];
  if (pdl) {
    pdl_wait();
    pdl_launch_next();  // after the wait: at most one grid waits ahead
  }
  if (len == 0) {
    for (int i = tid; i < L * (kDh / 8); i += kT) {
      const int r = i >> 3, c = i & 7;
      *reinterpret_cast<uint4*>(out + (row0 + r) * inner + h * kDh + c * 8) = make_uint4(0, 0, 0, 0);
    }
    return;
  }
  // all loads in flight at once: Q, K, V rows (past L zero-filled) by cp.async
  for (int i = tid; i < 3 * KL * 8; i += kT) {
    const int mat = i / (KL * 8), rem = i % (KL * 8), r = rem >> 3, c = rem & 7;
    const uint32_t dst = smem_u32(mat == 0 ? sQ : mat == 1 ? sK : sV) + r * kRowB + c * 16;
    cp16s(dst, qkv + (row0 + (r < L ? r : 0)) * (3 * inner) + mat * inner + h * kDh + c * 8, r < L);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  const int q0 = warp * 16;
  if (q0 < L) {
    const int g = lane >> 2, t4 = lane & 3;
    // ---- S = Q K^T over KL keys (KL / 8 n-blocks of 8, 4 k-steps of 16)
    constexpr int NB = KL / 8;
    float s[NB][4];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int i = 0; i < 4; ++i) s[nb][i] = 0.0f;
    const uint32_t qa = smem_u32(sQ) + (q0 + (lane & 15)) * kRowB + (lane >> 4) * 16;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4(qa + ks * 32, a0, a1, a2, a3);
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        uint32_t b0, b1;
        ldsm_x2(smem_u32(sK) + (nb * 8 + (lane & 7)) * kRowB + ks * 32 + ((lane >> 3) & 1) * 16, b0, b1);
        mma16816(s[nb], a0, a1, a2, a3, b0, b1);
      }
    }
    // ---- v = S log2(e) + bias, mask, row max / sum (rows g and g + 8 of the block)
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = q0 + g + 8 * (i >> 1), key = nb * 8 + 2 * t4 + (i & 1);
        const float v = key < len ? fmaf(s[nb][i], 1.4426950408889634f, sBias[key - row + KL - 1]) : -INFINITY;
        s[nb][i] = v;
        mx[i >> 1] = fmaxf(mx[i >> 1], v);
      }
#pragma unroll
    for (int hlf = 0; hlf < 2; ++hlf) {
      mx[hlf] = fmaxf(mx[hlf], __shfl_xor_sync(0xFFFFFFFFu, mx[hlf], 1));
      mx[hlf] = fmaxf(mx[hlf], __shfl_xor_sync(0xFFFFFFFFu, mx[hlf], 2));
    }
    float sum[2] = {0.0f, 0.0f};
    uint32_t pa[KL / 16][4];  // A fragments of P for the KL / 16 key steps
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      const float p0 = ex2s(s[nb][0] - mx[0]), p1 = ex2s(s[nb][1] - mx[0]);
      const float p2 = ex2s(s[nb][2] - mx[1]), p3 = ex2s(s[nb][3] - mx[1]);
      sum[0] += p0 + p1;
      sum[1] += p2 + p3;
      pa[nb >> 1][(nb & 1) * 2] = pack_f16x2(p0, p1);
      pa[nb >> 1][(nb & 1) * 2 + 1] = pack_f16x2(p2, p3);
    }
#pragma unroll
    for (int hlf = 0; hlf < 2; ++hlf) {
      sum[hlf] += __shfl_xor_sync(0xFFFFFFFFu, sum[hlf], 1);
      sum[hlf] += __shfl_xor_sync(0xFFFFFFFFu, sum[hlf], 2);
    }
    // ---- O = P V (V [keys][d] through ldmatrix.trans)
    float o[8][4];
#pragma unroll
    for (int nb = 0; nb < 8; ++nb)
#pragma unroll
      for (int i = 0; i < 4; ++i) o[nb][i] = 0.0f;
#pragma unroll
    for (int ks = 0; ks < KL / 16; ++ks) {
#pragma unroll
      for (int nb = 0; nb < 8; ++nb) {
        uint32_t b0, b1;
        ldsm_x2_t(smem_u32(sV) + (ks * 16 + (lane & 15)) * kRowB + nb * 16, b0, b1);
        // A fragment order: (row g, k 0-7), (row g+8, k 0-7), (row g, k 8-15), (row g+8, k 8-15)
        mma16816(o[nb], pa[ks][0], pa[ks][1], pa[ks][2], pa[ks][3], b0, b1);
      }
    }
    const float inv0 = 1.0f / sum[0], inv1 = 1.0f / sum[1];
#pragma unroll
    for (int hlf = 0; hlf < 2; ++hlf) {
      const int row = q0 + g + 8 * hlf;
      if (row >= L) continue;
      const float inv = hlf ? inv1 : inv0;
      __half* dst = out + (row0 + row) * inner + h * kDh + 2 * t4;
#pragma unroll
      for (int nb = 0; nb < 8; ++nb)
        *reinterpret_cast<uint32_t*>(dst + nb * 8) = pack_f16x2_sat(o[nb][2 * hlf] * inv, o[nb][2 * hlf + 1] * inv);
    }
  }
  __syncthreads();  // shared memory free for the caller's next use
}

}  // namespace attn_small
}  // namespace wc
