// Memory-bound kernels of the encoder: Q4_K dequant, embedding gather fused
// with the first RMSNorm, and RMSNorm (T5LayerNorm, src/quantized_t5.rs:162-173:
// f32 statistics, no mean subtraction, no bias, x / sqrt(var + eps) * w).
// One warp per row, 16-byte vector accesses, the row kept in registers.
#include "common.cuh"
#include "rownorm.cuh"
#include "elementwise.h"
#include "q4k.cuh"

namespace wc {

namespace {

constexpr int kMaxD = 1024;           // d_model supported by the row kernels
constexpr int kPerLane = kMaxD / 32;  // floats per lane at kMaxD

__global__ void q4k_dequant_kernel(const uint8_t* __restrict__ blocks, int64_t nblocks, float* __restrict__ out) {
  // one thread per 8 outputs; 32 threads per super-block
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t blk = gid >> 5;
  if (blk >= nblocks) return;
  const int e = static_cast<int>(gid & 31) * 8;
  const uint8_t* p = blocks + blk * 144;
  const Q4KScales s = q4k_load_scales(p);
  float v[8];
  q4k_block_elems8(p, s, e, v);
  float4* o = reinterpret_cast<float4*>(out + blk * 256 + e);
  o[0] = make_float4(v[0], v[1], v[2], v[3]);
  o[1] = make_float4(v[4], v[5], v[6], v[7]);
}

// The same elements rounded to f16 (round to nearest even): the operand
// values the fused-dequant GEMMs feed the tensor cores.
__global__ void q4k_dequant_f16_kernel(const uint8_t* __restrict__ blocks, int64_t nblocks, __half* __restrict__ out) {
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t blk = gid >> 5;
  if (blk >= nblocks) return;
  const int e = static_cast<int>(gid & 31) * 8;
  const uint8_t* p = blocks + blk * 144;
  const Q4KScales s = q4k_load_scales(p);
  float v[8];
  q4k_block_elems8(p, s, e, v);
  *reinterpret_cast<uint4*>(out + blk * 256 + e) =
      make_uint4(pack_f16x2(v[0], v[1]), pack_f16x2(v[2], v[3]), pack_f16x2(v[4], v[5]), pack_f16x2(v[6], v[7]));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// lane owns elements [8*(lane + 32*i), +8) for i < D/256
__global__ void embed_rmsnorm_kernel(const uint8_t* __restrict__ table, const uint32_t* __restrict__ ids,
                                     const int32_t* __restrict__ lengths, int L, int M, int D,
                                     const float* __restrict__ w, float eps, float* __restrict__ x,
                                     __half* __restrict__ xn, uint32_t* __restrict__ status) {
  pdl_wait();
  pdl_launch_next();  // after the wait: at most one grid waits ahead
  const int m = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (m >= M) return;
  const int b = m / L, i = m - b * L;
  const uint32_t id = i < lengths[b] ? ids[m] : 0u;
  const int nb = D / 256;
  const uint8_t* row = table + static_cast<size_t>(id) * nb * 144;
  float v[kMaxD / 256][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kMaxD / 256; ++c) {
    if (c < nb) {
      const uint8_t* blk = row + c * 144;
      const Q4KScales s = q4k_load_scales(blk);
      q4k_block_elems8(blk, s, lane * 8, v[c]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[c][j] * v[c][j];
    }
  }
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / static_cast<float>(D) + eps);
  bool clip = false;
#pragma unroll
  for (int c = 0; c < kMaxD / 256; ++c) {
    if (c < nb) {
      const int e = c * 256 + lane * 8;
      float* xo = x + static_cast<size_t>(m) * D + e;
      reinterpret_cast<float4*>(xo)[0] = make_float4(v[c][0], v[c][1], v[c][2], v[c][3]);
      reinterpret_cast<float4*>(xo)[1] = make_float4(v[c][4], v[c][5], v[c][6], v[c][7]);
      const float4 w0 = reinterpret_cast<const float4*>(w + e)[0];
      const float4 w1 = reinterpret_cast<const float4*>(w + e)[1];
      uint4 o;
      o.x = pack_f16x2_sat(v[c][0] * inv * w0.x, v[c][1] * inv * w0.y, clip);
      o.y = pack_f16x2_sat(v[c][2] * inv * w0.z, v[c][3] * inv * w0.w, clip);
      o.z = pack_f16x2_sat(v[c][4] * inv * w1.x, v[c][5] * inv * w1.y, clip);
      o.w = pack_f16x2_sat(v[c][6] * inv * w1.z, v[c][7] * inv * w1.w, clip);
      *reinterpret_cast<uint4*>(xn + static_cast<size_t>(m) * D + e) = o;
    }
  }
  report_f16_clip(clip, status);
}

// One warp per row (rownorm.cuh).  With delta != null the residual add of the
// preceding sub-layer happens here first: x += delta (written back), then the
// norm of the updated row.
__global__ void rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ delta, const float* __restrict__ w,
                               __half* __restrict__ y, int M, int D, float eps, uint32_t* __restrict__ status) {
  const int m = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  // the norm weights are not written by the previous kernel: load them
  // before waiting for it
  const RowNormW ww = rownorm_load_w(w, D, lane);
  pdl_wait();
  pdl_launch_next();  // after the wait: at most one grid waits ahead
  if (m >= M) return;
  const bool clip = rownorm_row(x + static_cast<size_t>(m) * D, delta ? delta + static_cast<size_t>(m) * D : nullptr,
                                true, ww, y + static_cast<size_t>(m) * D, D, eps, lane);
  report_f16_clip(clip, status);
}

// The same normalisation for D = 768 without a residual add (the large-M
// forward, whose GEMMs already added it): each warp normalises two rows and
// issues all twelve 16-byte loads of a lane before any arithmetic, so their
// latencies overlap.  Per row the arithmetic is rownorm_row's, in the same
// order, so the results are the same bits.
__global__ void rmsnorm768x2_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                    __half* __restrict__ y, int M, float eps, uint32_t* __restrict__ status) {
  constexpr int D = 768, G = D / 128;
  const int m0 = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 2;
  const int lane = threadIdx.x & 31;
  // the norm weights are not written by the previous kernel: load them
  // before waiting for it
  const float4* wr = reinterpret_cast<const float4*>(w);
  float4 ww[G];
#pragma unroll
  for (int g = 0; g < G; ++g) ww[g] = wr[lane + 32 * g];
  pdl_wait();
  pdl_launch_next();
  if (m0 >= M) return;
  const bool two = m0 + 1 < M;
  float4 v[2][G];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(two ? m0 + r : m0) * D);
#pragma unroll
    for (int g = 0; g < G; ++g) v[r][g] = xr[lane + 32 * g];
  }
  float ss[2] = {0.f, 0.f};
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int g = 0; g < G; ++g)
      ss[r] += v[r][g].x * v[r][g].x + v[r][g].y * v[r][g].y + v[r][g].z * v[r][g].z + v[r][g].w * v[r][g].w;
#pragma unroll
  for (int r = 0; r < 2; ++r) ss[r] = rownorm_warp_sum(ss[r]);
  bool clip = false;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    if (r == 1 && !two) break;
    const float inv = 1.0f / sqrtf(ss[r] / static_cast<float>(D) + eps);
    uint2* yr = reinterpret_cast<uint2*>(y + static_cast<size_t>(m0 + r) * D);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      uint2 o;
      o.x = pack_f16x2_sat(v[r][g].x * inv * ww[g].x, v[r][g].y * inv * ww[g].y, clip);
      o.y = pack_f16x2_sat(v[r][g].z * inv * ww[g].z, v[r][g].w * inv * ww[g].w, clip);
      yr[lane + 32 * g] = o;
    }
  }
  report_f16_clip(clip, status);
}

// A wait on an mbarrier that nothing ever arrives on, bounded by limit_ns:
// exercises the timeout path every pipelined kernel uses.
__global__ void wait_timeout_selftest_kernel(uint32_t* status, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  mbar_wait_limit(&bar, 0, status, limit_ns);
}

}  // namespace

cudaError_t wait_timeout_selftest_launch(uint32_t* status, uint64_t limit_ns, cudaStream_t st) {
  wait_timeout_selftest_kernel<<<1, 32, 0, st>>>(status, limit_ns);
  return cudaGetLastError();
}

cudaError_t q4k_dequant_launch(const uint8_t* blocks, int64_t nblocks, float* out, cudaStream_t st) {
  if (nblocks <= 0) return cudaSuccess;
  const int64_t threads = nblocks * 32;
  const int bs = 256;
  q4k_dequant_kernel<<<static_cast<unsigned>((threads + bs - 1) / bs), bs, 0, st>>>(blocks, nblocks, out);
  return cudaGetLastError();
}

cudaError_t q4k_dequant_f16_launch(const uint8_t* blocks, int64_t nblocks, __half* out, cudaStream_t st) {
  if (nblocks <= 0) return cudaSuccess;
  const int64_t threads = nblocks * 32;
  const int bs = 256;
  q4k_dequant_f16_kernel<<<static_cast<unsigned>((threads + bs - 1) / bs), bs, 0, st>>>(blocks, nblocks, out);
  return cudaGetLastError();
}

cudaError_t embed_rmsnorm_launch(const uint8_t* table, const uint32_t* ids, const int32_t* lengths, int L, int M,
                                 int D, const float* w, float eps, float* x, __half* xn, uint32_t* status,
                                 cudaStream_t st) {
  if (M <= 0) return cudaSuccess;
  if (D % 256 != 0 || D > kMaxD) return cudaErrorInvalidValue;
  return launch_pdl(embed_rmsnorm_kernel, dim3((M + 7) / 8), dim3(256), 0, st, nullptr, 0, table, ids, lengths, L, M, D,
                    w, eps, x, xn, status);
}

cudaError_t rmsnorm_launch(float* x, const float* delta, const float* w, __half* y, int M, int D, float eps,
                           uint32_t* status, cudaStream_t st) {
  if (M <= 0) return cudaSuccess;
  if (D % 128 != 0 || D > kMaxD) return cudaErrorInvalidValue;
  if (D == 768 && delta == nullptr)
    return launch_pdl(rmsnorm768x2_kernel, dim3((M + 15) / 16), dim3(256), 0, st, nullptr, 0,
                      static_cast<const float*>(x), w, y, M, eps, status);
  return launch_pdl(rmsnorm_kernel, dim3((M + 7) / 8), dim3(256), 0, st, nullptr, 0, x, delta, w, y, M, D, eps, status);
}

}  // namespace wc
