// Bidirectional T5 encoder self-attention, flash-style (one pass over keys
// with an online softmax), with the T5 relative-position bias and a key
// padding mask.  Replaces src/quantized_t5.rs:426-500 (scores without 1/sqrt(d)
// scaling, + position bias, softmax_last_dim, P.V, transpose back to tokens).
//
// Input: the token-major QKV projection [B*L][3*inner] (q | k | v, each
// H heads x 64), f16.  Output: [B*L][inner] f16, token-major, which is the
// layout the O projection reads.  Query rows past a sequence's valid length
// that fall in an all-padding 64-row tile are written as zeros; keys past the
// valid length never contribute.
//
// Tiling: one CTA per (64 queries, head, sequence), 4 warps x 16 query rows;
// 64-key K/V tiles double-buffered in shared memory by cp.async; QK^T and PV
// on the f16 tensor cores (m16n8k16, f32 accumulate); softmax in f32 with
// exp2 and a running max/sum per row kept by the 4 lanes that share it.
#include "attention.h"
#include "common.cuh"

namespace wc {

namespace {

constexpr int kTile = 64;  // queries per CTA and keys per K/V tile
constexpr int kDh = 64;    // head dimension (fixed by the kernel)

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  const int n = pred ? 16 : 0;  // 0 source bytes -> 16 zero bytes
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// 64 rows x 128 B tile, 16-B chunks XOR-swizzled by row to keep ldmatrix
// conflict-free.
__device__ __forceinline__ uint32_t tile_off(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                  uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_f16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Relative-position bucket of key - query = delta from the monotone
// thresholds: f(d) = #{v : thr[v] <= d} for d = |delta|; keys after the
// query add num_buckets/2 (src/quantized_t5.rs:447-483).
__device__ __forceinline__ int rel_bucket(const BucketThresholds& bt, int delta) {
  const int d = delta < 0 ? -delta : delta;
  int f = 0;
#pragma unroll 1
  for (int v = 1; v < bt.half; ++v) f += (d >= bt.thr[v]) ? 1 : 0;
  return f + (delta > 0 ? bt.half : 0);
}

__global__ void __launch_bounds__(128) attention_kernel(const __half* __restrict__ qkv,
                                                        __half* __restrict__ out,
                                                        const int32_t* __restrict__ lengths, int L, int H,
                                                        const float* __restrict__ bias_tab, BucketThresholds bt) {
  __shared__ __align__(1024) uint8_t sQ[kTile * 128];
  __shared__ __align__(1024) uint8_t sK[2][kTile * 128];
  __shared__ __align__(1024) uint8_t sV[2][kTile * 128];
  __shared__ float sBias[2 * kTile];

  const int q_tile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int inner = H * kDh;
  const int ld = 3 * inner;
  const int len = min(lengths[b], L);
  const int q0 = q_tile * kTile;
  const size_t seq_row0 = static_cast<size_t>(b) * L;

  if (q0 >= len) {
    // all-padding query tile: zero output rows so later layers stay finite
    for (int idx = tid; idx < kTile * (kDh / 8); idx += blockDim.x) {
      const int r = idx >> 3, c = idx & 7;
      if (q0 + r < L)
        *reinterpret_cast<uint4*>(out + (seq_row0 + q0 + r) * inner + h * kDh + c * 8) = make_uint4(0, 0, 0, 0);
    }
    return;
  }

  const __half* qbase = qkv + seq_row0 * ld + h * kDh;
  const __half* kbase = qbase + inner;
  const __half* vbase = qbase + 2 * inner;

  auto load_tile = [&](uint8_t* dst, const __half* base, int row0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = tid + i * 128;
      const int r = idx >> 3, c = idx & 7;
      const bool ok = row0 + r < L;
      const __half* src = base + static_cast<size_t>(ok ? row0 + r : 0) * ld + c * 8;
      cp_async16(smem_u32(dst + tile_off(r, c)), src, ok);
    }
  };

  const int n_kt = (len + kTile - 1) / kTile;
  load_tile(sQ, qbase, q0);
  load_tile(sK[0], kbase, 0);
  load_tile(sV[0], vbase, 0);
  cp_async_commit();

  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float row_max[2] = {-INFINITY, -INFINITY};
  float row_sum[2] = {0.f, 0.f};
  uint32_t qf[4][4];
  constexpr float kLog2e = 1.4426950408889634f;

  const int r_lo = warp * 16 + (lane >> 2);  // this thread's rows within the tile: r_lo, r_lo + 8
  const float* bias_h = bias_tab;            // [num_buckets][H]

  for (int kt = 0; kt < n_kt; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < n_kt) {
      load_tile(sK[buf ^ 1], kbase, (kt + 1) * kTile);
      load_tile(sV[buf ^ 1], vbase, (kt + 1) * kTile);
    }
    cp_async_commit();
    // bias for delta = key - query over this (query tile, key tile) pair:
    // delta in [k0 - q0 - 63, k0 - q0 + 63]
    const int k0 = kt * kTile;
    const int dmin = k0 - q0 - (kTile - 1);
    if (tid < 2 * kTile - 1) sBias[tid] = bias_h[rel_bucket(bt, dmin + tid) * H + h];
    cp_async_wait<1>();
    __syncthreads();

    if (kt == 0) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int row = warp * 16 + (lane & 15);
        const int chunk = 2 * kk + (lane >> 4);
        ldmatrix_x4(smem_u32(sQ + tile_off(row, chunk)), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }

    // S = Q K^T  (16 x 64 per warp)
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // pairs of 8-key n-tiles
        const int key = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int chunk = 2 * kk + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(smem_u32(sK[buf] + tile_off(key, chunk)), b0, b1, b2, b3);
        mma_f16_16816(s[2 * np], qf[kk], b0, b1);
        mma_f16_16816(s[2 * np + 1], qf[kk], b2, b3);
      }
    }

    // bias, mask, online softmax
    float tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = r_lo + ((e >> 1) << 3);
        const int kc = nt * 8 + 2 * (lane & 3) + (e & 1);
        const int key = k0 + kc;
        float v = s[nt][e] + sBias[kc - r + (kTile - 1)];
        v = key < len ? v : -INFINITY;
        s[nt][e] = v;
        tmax[e >> 1] = fmaxf(tmax[e >> 1], v);
      }
    }
    float corr[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      tmax[hr] = fmaxf(tmax[hr], __shfl_xor_sync(0xFFFFFFFFu, tmax[hr], 1));
      tmax[hr] = fmaxf(tmax[hr], __shfl_xor_sync(0xFFFFFFFFu, tmax[hr], 2));
      const float nm = fmaxf(row_max[hr], tmax[hr]);
      corr[hr] = exp2f((row_max[hr] - nm) * kLog2e);
      row_max[hr] = nm;
      row_sum[hr] *= corr[hr];
    }
    float psum[2] = {0.f, 0.f};
    uint32_t pf[4][4];  // P as the A operand of P.V, per 16-key step
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      float pv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        pv[e] = exp2f((s[nt][e] - row_max[e >> 1]) * kLog2e);
        psum[e >> 1] += pv[e];
      }
      pf[nt >> 1][(nt & 1) * 2 + 0] = pack_f16x2(pv[0], pv[1]);
      pf[nt >> 1][(nt & 1) * 2 + 1] = pack_f16x2(pv[2], pv[3]);
    }
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) row_sum[hr] += psum[hr];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      o[nt][0] *= corr[0];
      o[nt][1] *= corr[0];
      o[nt][2] *= corr[1];
      o[nt][3] *= corr[1];
    }

    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t a[4] = {pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3]};
#pragma unroll
      for (int dp = 0; dp < 4; ++dp) {  // pairs of 8-wide d tiles
        const int key = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int chunk = 2 * dp + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(smem_u32(sV[buf] + tile_off(key, chunk)), b0, b1, b2, b3);
        mma_f16_16816(o[2 * dp], a, b0, b1);
        mma_f16_16816(o[2 * dp + 1], a, b2, b3);
      }
    }
    __syncthreads();  // buffers of this tile are refilled next iteration
  }
  cp_async_wait<0>();

  // finalise: quad-reduce the row sums, normalise, store f16
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    row_sum[hr] += __shfl_xor_sync(0xFFFFFFFFu, row_sum[hr], 1);
    row_sum[hr] += __shfl_xor_sync(0xFFFFFFFFu, row_sum[hr], 2);
  }
  const float inv0 = 1.0f / row_sum[0], inv1 = 1.0f / row_sum[1];
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int qi = q0 + r_lo + hr * 8;
    if (qi < L) {
      __half* dst = out + (seq_row0 + qi) * inner + h * kDh;
      const float inv = hr ? inv1 : inv0;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int d = nt * 8 + 2 * (lane & 3);
        *reinterpret_cast<uint32_t*>(dst + d) = pack_f16x2_sat(o[nt][2 * hr] * inv, o[nt][2 * hr + 1] * inv);
      }
    }
  }
}

}  // namespace

cudaError_t attention_launch(const __half* qkv, __half* out, const int32_t* lengths, int B, int L,
                             int H, const float* bias_tab, const BucketThresholds& bt, cudaStream_t st) {
  if (B <= 0 || L <= 0) return cudaSuccess;
  dim3 grid((L + kTile - 1) / kTile, H, B);
  attention_kernel<<<grid, 128, 0, st>>>(qkv, out, lengths, L, H, bias_tab, bt);
  return cudaGetLastError();
}

}  // namespace wc
