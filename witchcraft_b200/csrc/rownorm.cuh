// One T5 RMSNorm row by one warp (src/quantized_t5.rs:162-173): the body of
// the RMSNorm kernel (elementwise.cu), as a device function other kernels can
// call and get the same bits.
#pragma once
#include "common.cuh"

namespace wc {

constexpr int kRowNormMaxD = 1024;  // d_model supported (D % 128 == 0)

__device__ __forceinline__ float rownorm_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// Lane owns float4 groups lane + 32 g, g < D / 128.  v = x (+ delta), written
// back to x when write_x; y = f16(v * (1 / sqrt(mean(v^2) + eps)) * w).  y may
// point to global or shared memory (8-byte aligned row).
// The lane's norm weights (float4 groups lane + 32 g), loaded ahead of the
// row so a kernel can issue them before it waits for its predecessor.
struct RowNormW {
  float4 v[kRowNormMaxD / 128];
};
__device__ __forceinline__ RowNormW rownorm_load_w(const float* __restrict__ w, int D, int lane) {
  RowNormW r;
  const float4* wr = reinterpret_cast<const float4*>(w);
#pragma unroll
  for (int g = 0; g < kRowNormMaxD / 128; ++g)
    r.v[g] = g < D / 128 ? wr[lane + 32 * g] : make_float4(0.f, 0.f, 0.f, 0.f);
  return r;
}

__device__ __forceinline__ bool rownorm_row(float* __restrict__ x, const float* __restrict__ delta, bool write_x,
                                            const RowNormW& ww, __half* __restrict__ y, int D, float eps,
                                            int lane) {
  const int ng = D / 128;
  float4* xr = reinterpret_cast<float4*>(x);
  const float4* dr = reinterpret_cast<const float4*>(delta);
  float4 v[kRowNormMaxD / 128];
  float ss = 0.f;
#pragma unroll
  for (int g = 0; g < kRowNormMaxD / 128; ++g) {
    if (g < ng) {
      v[g] = xr[lane + 32 * g];
      if (dr) {
        const float4 d = dr[lane + 32 * g];
        v[g].x += d.x;
        v[g].y += d.y;
        v[g].z += d.z;
        v[g].w += d.w;
        if (write_x) xr[lane + 32 * g] = v[g];
      }
      ss += v[g].x * v[g].x + v[g].y * v[g].y + v[g].z * v[g].z + v[g].w * v[g].w;
    }
  }
  ss = rownorm_warp_sum(ss);
  // x / den as x * (1 / den): one division per row instead of one per
  // element (the product differs from the quotient by at most one f32 ulp)
  const float inv = 1.0f / sqrtf(ss / static_cast<float>(D) + eps);
  uint2* yr = reinterpret_cast<uint2*>(y);
  bool clip = false;
#pragma unroll
  for (int g = 0; g < kRowNormMaxD / 128; ++g) {
    if (g < ng) {
      const float4 wg = ww.v[g];
      uint2 o;
      o.x = pack_f16x2_sat(v[g].x * inv * wg.x, v[g].y * inv * wg.y, clip);
      o.y = pack_f16x2_sat(v[g].z * inv * wg.z, v[g].w * inv * wg.w, clip);
      yr[lane + 32 * g] = o;
    }
  }
  return clip;  // whether an output value was clipped to the f16 range
}
__device__ __forceinline__ bool rownorm_row(float* __restrict__ x, const float* __restrict__ delta, bool write_x,
                                            const float* __restrict__ w, __half* __restrict__ y, int D, float eps,
                                            int lane) {
  return rownorm_row(x, delta, write_x, rownorm_load_w(w, D, lane), y, D, eps, lane);
}

}  // namespace wc
