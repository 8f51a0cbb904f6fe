// Q4_K super-block decoding shared by the dequant kernel, the embedding
// gather and the GEMM's dequant warps.
//
// Layout (GGML Q4_K, 144 bytes per 256 weights; the format candle's
// k_quants::BlockQ4K reads for src/quantized_t5.rs:44): f16 d, f16 dmin,
// 12 bytes of packed 6-bit scale/min for 8 sub-blocks of 32, 128 bytes of
// nibbles.  Byte l of 32-byte chunk c holds element l of sub-block 2c (low
// nibble) and element l of sub-block 2c+1 (high nibble).
//
// Value of element e of sub-block j:  (d*sc_j) * q_e - (dmin*m_j), where the
// reference rounds each product to f32 and then the difference.  d and dmin
// are f16 (11 significant bits) and sc_j, m_j < 64 (6 bits), so both products
// are exact in f32; (d*sc_j)*q_e has at most 21 significant bits and is exact
// too.  Therefore the reference value equals fmaf(d*sc_j, q_e, -(dmin*m_j))
// with its single rounding, which is what the code below computes: bit-exact.
#pragma once
#include "common.cuh"

namespace wc {

struct Q4KScales {
  uint32_t sc_lo, sc_hi, m_lo, m_hi;  // 4 six-bit values per word, one per byte
  float d, dmin;
};

// Decode the super-block header at p (16-byte aligned).
__device__ __forceinline__ Q4KScales q4k_load_scales(const uint8_t* p) {
  const uint4 h = *reinterpret_cast<const uint4*>(p);
  Q4KScales s;
  s.d = __half2float(__ushort_as_half(static_cast<unsigned short>(h.x & 0xFFFFu)));
  s.dmin = __half2float(__ushort_as_half(static_cast<unsigned short>(h.x >> 16)));
  const uint32_t s0 = h.y, s1 = h.z, s2 = h.w;  // packed scale bytes 0-3, 4-7, 8-11
  s.sc_lo = s0 & 0x3F3F3F3Fu;
  s.m_lo = s1 & 0x3F3F3F3Fu;
  s.sc_hi = (s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u);
  s.m_hi = ((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u);
  return s;
}

// (d*sc_j, dmin*m_j) of sub-block j (0..7).
__device__ __forceinline__ void q4k_sub_scale(const Q4KScales& s, int j, float& d1, float& m1) {
  const uint32_t scw = j < 4 ? s.sc_lo : s.sc_hi;
  const uint32_t mw = j < 4 ? s.m_lo : s.m_hi;
  const int sh = (j & 3) * 8;
  d1 = s.d * static_cast<float>((scw >> sh) & 0xFFu);
  m1 = s.dmin * static_cast<float>((mw >> sh) & 0xFFu);
}

// Exact float of the 4-bit value in byte b (0..3) of x (each byte holds 0..15):
// 0x4B0000qq is the float 2^23 + q, so subtracting 2^23 gives q exactly.
__device__ __forceinline__ float nib_to_float(uint32_t x, int b) {
  return __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7440u | static_cast<uint32_t>(b))) - 8388608.0f;
}

// Dequantise the 8 consecutive elements whose 4-bit values sit in the bytes of
// (w0, w1) (nibbles already isolated to 0..15 per byte).
__device__ __forceinline__ void q4k_dequant8(uint32_t x0, uint32_t x1, float d1, float m1, float (&v)[8]) {
#pragma unroll
  for (int b = 0; b < 4; ++b) v[b] = fmaf(d1, nib_to_float(x0, b), -m1);
#pragma unroll
  for (int b = 0; b < 4; ++b) v[4 + b] = fmaf(d1, nib_to_float(x1, b), -m1);
}

// Elements [e, e+8) (e % 8 == 0, e < 256) of the super-block at blk.
__device__ __forceinline__ void q4k_block_elems8(const uint8_t* blk, const Q4KScales& s, int e, float (&v)[8]) {
  const int c = e >> 6;          // 32-byte chunk
  const int hs = (e >> 5) & 1;   // low (0) or high (1) nibble
  const int l0 = e & 31;         // first byte in the chunk
  const uint2 w = *reinterpret_cast<const uint2*>(blk + 16 + 32 * c + l0);
  uint32_t x0 = w.x, x1 = w.y;
  if (hs) {
    x0 >>= 4;
    x1 >>= 4;
  }
  x0 &= 0x0F0F0F0Fu;
  x1 &= 0x0F0F0F0Fu;
  float d1, m1;
  q4k_sub_scale(s, 2 * c + hs, d1, m1);
  q4k_dequant8(x0, x1, d1, m1, v);
}

}  // namespace wc
