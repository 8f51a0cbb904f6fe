// Packed-embedding codec on the GPU: embeddings_to_packed /
// embeddings_from_packed (src/packops.rs:172-438) for many documents per
// call, byte-identical to the reference's stream:
//   u32 rows; per window of <= 1024 rows: cols bytes (inverse column
//   permutation), u16 symbol count, (u16 symbol, u16 frequency) pairs in
//   symbol order, u16 rANS byte count (wrapping like the reference's
//   `as u16`), the rANS64 bytes.
//
// Encode, per window:
//   pack_transform   one CTA: column sums (each column summed over its rows in
//                    row order, as the reference does), the stable ascending
//                    column order, the permuted copy, the mirror-edge Haar on
//                    every row and then every column (src/haarops.rs:4-30),
//                    warp-parallel inside each level but with every value
//                    computed exactly as the serial loop computes it, the
//                    largest |x| below 1, the symbols, their histogram, the
//                    symbol list and its frequencies normalised to 2^12
//                    (scale_histogram, src/packops.rs:31-103: the largest-
//                    remainder step ranks the remainders in parallel, a
//                    stable descending order), and the rANS encoder table;
//                    symbols are rewritten as indices into that table.
//   pack_encode      one thread per window: the rANS64 encode
//                    (src/rans64.rs:88-166), serial by construction, from the
//                    window's table of encoder constants; all windows of a
//                    chunk encode at once.
//   pack_assemble    one CTA per window copies header and stream into place.
// Decode mirrors it: unpack_decode (one CTA per window: the cumulative-
// frequency tables in shared memory, one thread runs the serial rANS decode)
// then unpack_inverse (inverse Haar on rows then columns, src/haarops.rs:
// 32-70, un-permute, L2-normalise each row in column order).
//
// Every float operation is a separate IEEE f32 operation in the reference's
// order (__fadd_rn / __fmul_rn where the compiler could otherwise contract),
// so the symbols, and with them the bytes, match the reference exactly.
#include "codec.h"
#include "common.cuh"

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

namespace wc {

namespace {

constexpr int kWinRows = 1024;  // MAX_WINDOW_ROWS, src/packops.rs:8
constexpr int kRansBits = 12;   // RANS_BITS
constexpr int kMaxSyms = 1 << kRansBits;
constexpr uint64_t kRansL = 1ull << 31;
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxCols = 255;
constexpr float kInvSqrt2 = 0.7071067811865475f;
constexpr float kRange = 29.0f;

// Status bits (per call, device word)
enum : uint32_t { kErrTooManySymbols = 1, kErrEncodeOverflow = 2, kErrBadStream = 4 };

struct WinDesc {
  int64_t row0;    // first global row (rows of all documents concatenated)
  int rows;        // <= kWinRows
  int doc;
};

// Per-window outputs of pack_transform.
struct WinOut {
  int m;           // distinct symbols
  int enc_len;     // rANS bytes
  int enc_start;   // first byte in the window's encoder scratch
  int pad;
};

// Encoder constants of one symbol (RansEncSymbol, src/rans64.rs:28-82);
// x_max = freq << 51 and cmpl_freq = 4096 - freq are derived from freq.
struct alignas(16) EncSym {
  uint64_t rcp_freq;
  uint32_t bias;       // cum, or cum + 4095 for freq 1
  uint16_t freq;
  uint16_t rcp_shift;
};

__device__ __forceinline__ EncSym enc_symbol(uint32_t cum, uint32_t freq) {
  EncSym s;
  s.freq = static_cast<uint16_t>(freq);
  if (freq < 2) {
    s.rcp_freq = ~0ull;
    s.rcp_shift = 0;
    s.bias = cum + ((1u << kRansBits) - 1);
  } else {
    uint32_t shift = 0;
    while (freq > (1u << shift)) ++shift;
    // ceil(2^(shift + 63) / freq) without 128-bit arithmetic: with
    // 2^63 = a freq + b, 2^(shift+63) = a 2^shift freq + b 2^shift, and
    // b 2^shift < 2^24; the quotient fits 64 bits because freq > 2^(shift-1).
    const uint64_t two63 = 1ull << 63;
    const uint64_t a = two63 / freq, b = two63 % freq;
    const uint64_t t = b << shift;
    const uint64_t q = (a << shift) + t / freq;
    s.rcp_freq = q + ((t % freq) != 0 ? 1 : 0);
    s.rcp_shift = static_cast<uint16_t>(shift - 1);
    s.bias = cum;
  }
  return s;
}

__device__ __forceinline__ uint16_t coef_symbol(float x) {
  const float q = roundf(__fmul_rn(kRange, x));
  const float sf = __fadd_rn(__fmul_rn(2.0f, fabsf(q)), q < 0.0f ? 1.0f : 0.0f);
  const uint64_t s = sf >= 18446744073709551615.0f ? ~0ull : static_cast<uint64_t>(sf);  // `as usize` saturates
  return static_cast<uint16_t>(s > 0 ? s - 1 : 0);
}

// One level-sweep of the forward mirror-edge Haar over x[0, n0) by one warp;
// x and tmp are this warp's shared buffers (values end in x).
__device__ void warp_haar_forward(float* x, float* tmp, int n0, int lane) {
  int n = n0;
  while (n > 1) {
    const int pairs = n / 2, odd = n & 1, nc = pairs + odd;
    for (int i = lane; i < pairs; i += 32) {
      const float a = x[2 * i], b = x[2 * i + 1];
      tmp[i] = __fmul_rn(__fadd_rn(a, b), kInvSqrt2);
      tmp[nc + i] = __fmul_rn(__fsub_rn(a, b), kInvSqrt2);
    }
    if (odd && lane == 0) {
      const float a = x[n - 1];
      tmp[pairs] = __fmul_rn(__fadd_rn(a, a), kInvSqrt2);
    }
    __syncwarp();
    for (int i = lane; i < n; i += 32) x[i] = tmp[i];
    __syncwarp();
    n = nc;
  }
}

__device__ void warp_haar_inverse(float* x, float* tmp, int n0, int lane) {
  int levels[12];
  int nl = 0, n = n0;
  levels[nl++] = n;
  while (n > 1) {
    n = n / 2 + (n & 1);
    levels[nl++] = n;
  }
  for (int w = nl - 1; w >= 1; --w) {
    const int n_prev = levels[w - 1];
    const int odd = n_prev & 1, pairs = n_prev / 2, nc = pairs + odd;
    for (int i = lane; i < pairs; i += 32) {
      const float s = x[i], d = x[nc + i];
      tmp[2 * i] = __fmul_rn(__fadd_rn(s, d), kInvSqrt2);
      tmp[2 * i + 1] = __fmul_rn(__fsub_rn(s, d), kInvSqrt2);
    }
    if (odd && lane == 0) tmp[n_prev - 1] = __fmul_rn(x[nc - 1], kInvSqrt2);
    __syncwarp();
    for (int i = lane; i < n_prev; i += 32) x[i] = tmp[i];
    __syncwarp();
  }
}

// Shared memory of pack_transform / unpack_inverse: a union of the Haar
// buffers (per warp: 2 x kWinRows floats) and the histogram-scaling arrays
// (remainders u64, counts, frequencies).
constexpr int kHaarFloats = kWarps * 2 * kWinRows;
constexpr size_t kTransformSmem =
    std::max<size_t>(kHaarFloats * sizeof(float), kMaxSyms * (sizeof(uint64_t) + 2 * sizeof(uint32_t)));
constexpr int kChunkWins = 4096;  // windows per transform + encode round (encoder tables: 64 KB each)

__device__ __forceinline__ float block_max(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
  for (int i = 1; i < kWarps; ++i) r = fmaxf(r, red[i]);
  return r;
}

template <typename T>
__device__ __forceinline__ T block_sum(T v, T* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  T r = 0;
  for (int i = 0; i < kWarps; ++i) r += red[i];
  return r;
}

// Exclusive prefix over the block of one int per thread; returns the total.
__device__ __forceinline__ int block_scan(int v, int* red, int* excl) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xFFFFFFFFu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) red[warp] = x;
  __syncthreads();
  int base = 0, total = 0;
  for (int i = 0; i < kWarps; ++i) {
    if (i < warp) base += red[i];
    total += red[i];
  }
  *excl = base + x - v;
  return total;
}

// hdr layout per window: the inverse permutation in bytes [0, cols), the m
// (sym, freq) u16 pairs from byte kPairsOff (aligned whatever cols is).
constexpr int kPairsOff = 256;
constexpr size_t kHdrStride = kPairsOff + 4 * kMaxSyms;

__global__ void __launch_bounds__(kThreads)
    pack_transform(const float* __restrict__ emb, int cols, const WinDesc* __restrict__ wins, int w_begin,
                   int w_end, float* __restrict__ S, uint16_t* __restrict__ Q, uint32_t* __restrict__ hist_pool,
                   uint8_t* __restrict__ hdr, EncSym* __restrict__ esyms, WinOut* __restrict__ wout,
                   uint32_t* __restrict__ status) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float s_sum[kMaxCols + 1];
  __shared__ int s_perm[kMaxCols + 1];
  __shared__ float s_redf[kWarps];
  __shared__ int s_redi[kWarps];
  __shared__ uint64_t s_redu[kWarps];
  __shared__ int s_m, s_maxsym, s_fail;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t* hist = hist_pool + static_cast<size_t>(blockIdx.x) * 65536;

  for (int w = w_begin + blockIdx.x; w < w_end; w += gridDim.x) {
    const WinDesc wd = wins[w];
    const int R = wd.rows;
    const float* E = emb + wd.row0 * cols;
    float* W = S + wd.row0 * cols;
    uint16_t* Qw = Q + wd.row0 * cols;
    uint8_t* H = hdr + static_cast<size_t>(w) * kHdrStride;
    // -------- column sums (row order) and the stable ascending order
    if (tid < cols) {
      float s = 0.0f;
      for (int r = 0; r < R; ++r) s = __fadd_rn(s, E[static_cast<size_t>(r) * cols + tid]);
      s_sum[tid] = s;
    }
    __syncthreads();
    if (tid < cols) {
      const float v = s_sum[tid];
      int rank = 0;
      for (int c = 0; c < cols; ++c) {
        const float u = s_sum[c];
        rank += (u < v || (u == v && c < tid)) ? 1 : 0;
      }
      s_perm[rank] = tid;
      H[tid] = static_cast<uint8_t>(rank);  // inverse permutation: original column -> position
    }
    __syncthreads();
    // -------- permuted rows, forward Haar along each row
    float* bx = reinterpret_cast<float*>(smem) + warp * 2 * kWinRows;
    float* bt = bx + kWinRows;
    for (int r = warp; r < R; r += kWarps) {
      const float* er = E + static_cast<size_t>(r) * cols;
      for (int c = lane; c < cols; c += 32) bx[c] = er[s_perm[c]];
      __syncwarp();
      warp_haar_forward(bx, bt, cols, lane);
      float* wr = W + static_cast<size_t>(r) * cols;
      for (int c = lane; c < cols; c += 32) wr[c] = bx[c];
      __syncwarp();
    }
    __syncthreads();
    // -------- forward Haar along each column, largest |x| below 1
    float amax = 0.00001f;
    for (int c = warp; c < cols; c += kWarps) {
      for (int r = lane; r < R; r += 32) bx[r] = W[static_cast<size_t>(r) * cols + c];
      __syncwarp();
      warp_haar_forward(bx, bt, R, lane);
      for (int r = lane; r < R; r += 32) {
        const float v = bx[r];
        W[static_cast<size_t>(r) * cols + c] = v;
        const float a = fabsf(v);
        if (a < 1.0f && a > amax) amax = a;
      }
      __syncwarp();
    }
    __syncthreads();  // W complete (global writes of other warps)
    const float abs_max = block_max(amax, s_redf);
    const float inv_max = __fdiv_rn(1.0f, abs_max);
    // -------- symbols and their largest value
    const int n = R * cols;
    int mx = 0;
    for (int i = tid; i < n; i += kThreads) {
      const uint16_t s = coef_symbol(__fmul_rn(W[i], inv_max));
      Qw[i] = s;
      mx = max(mx, static_cast<int>(s));
    }
    for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    __syncthreads();
    if (lane == 0) s_redi[warp] = mx;
    __syncthreads();
    if (tid == 0) {
      int v = 0;
      for (int i = 0; i < kWarps; ++i) v = max(v, s_redi[i]);
      s_maxsym = v;
      s_fail = 0;
    }
    __syncthreads();
    const int max_symbol = s_maxsym;
    for (int s = tid; s <= max_symbol; s += kThreads) hist[s] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += kThreads) atomicAdd(&hist[Qw[i]], 1u);
    __syncthreads();
    // -------- compact (symbol, count) list in symbol order; hist[s] := index
    uint32_t* cnt = reinterpret_cast<uint32_t*>(smem + kMaxSyms * sizeof(uint64_t));
    uint32_t* freq = cnt + kMaxSyms;
    uint64_t* rem = reinterpret_cast<uint64_t*>(smem);  // reuses the Haar buffers
    uint16_t* pairs = reinterpret_cast<uint16_t*>(H + kPairsOff);
    int m_base = 0;
    for (int s0 = 0; s0 <= max_symbol; s0 += kThreads) {
      const int s = s0 + tid;
      const uint32_t c = s <= max_symbol ? hist[s] : 0u;
      int pos;
      const int tot = block_scan(c > 0 ? 1 : 0, s_redi, &pos);
      pos += m_base;
      if (c > 0) {
        if (pos < kMaxSyms) {
          cnt[pos] = c;
          pairs[2 * pos] = static_cast<uint16_t>(s);
          hist[s] = static_cast<uint32_t>(pos);
        } else {
          s_fail = 1;
        }
      }
      m_base += tot;
    }
    __syncthreads();
    const int m = m_base;
    if (m > kMaxSyms || s_fail) {
      if (tid == 0) {
        atomicOr(status, kErrTooManySymbols);
        wout[w].m = -1;
      }
      __syncthreads();
      continue;
    }
    // -------- scale_histogram: 1 + floor(count * (4096 - m) / sum) each, the
    // deficit to the largest remainders (stable), then the max fixup
    uint64_t ls = 0;
    for (int i = tid; i < m; i += kThreads) ls += cnt[i];
    const uint64_t sum = block_sum<uint64_t>(ls, s_redu);
    const uint32_t remaining = kMaxSyms - m;
    uint64_t lacc = 0;
    for (int i = tid; i < m; i += kThreads) {
      const uint64_t num = static_cast<uint64_t>(cnt[i]) * remaining;
      const uint64_t q = num / sum;
      rem[i] = num - q * sum;
      freq[i] = 1 + static_cast<uint32_t>(q);
      lacc += q;
    }
    const uint64_t acc = block_sum<uint64_t>(lacc, s_redu);
    const uint32_t deficit = remaining - static_cast<uint32_t>(acc);
    if (deficit > 0) {
      for (int i = tid; i < m; i += kThreads) {
        const uint64_t ri = rem[i];
        int rank = 0;
        for (int j = 0; j < m; ++j) {
          const uint64_t rj = rem[j];
          rank += (rj > ri || (rj == ri && j < i)) ? 1 : 0;
        }
        if (static_cast<uint32_t>(rank) < deficit) freq[i] += 1;
      }
    }
    __syncthreads();
    if (tid == 0) {
      int64_t total = 0;
      for (int i = 0; i < m; ++i) total += freq[i];
      if (total != kMaxSyms) {
        int mi = 0;
        for (int i = 1; i < m; ++i)
          if (freq[i] >= freq[mi]) mi = i;  // Iterator::max_by_key: the last maximum
        while (total < kMaxSyms) {
          freq[mi] += 1;
          ++total;
        }
        while (total > kMaxSyms && freq[mi] > 1) {
          freq[mi] -= 1;
          --total;
        }
      }
      s_m = m;
    }
    __syncthreads();
    // -------- frequencies into the header, cumulative starts, encoder table
    EncSym* es = esyms + static_cast<size_t>(w - w_begin) * kMaxSyms;
    int cbase = 0;
    for (int i0 = 0; i0 < m; i0 += kThreads) {
      const int i = i0 + tid;
      const int f = i < m ? static_cast<int>(freq[i]) : 0;
      int cum;
      const int tot = block_scan(f, s_redi, &cum);
      if (i < m) {
        pairs[2 * i + 1] = static_cast<uint16_t>(f);
        es[i] = enc_symbol(static_cast<uint32_t>(cbase + cum), static_cast<uint32_t>(f));
      }
      cbase += tot;
    }
    // -------- symbols -> table indices for the encoder
    for (int i = tid; i < n; i += kThreads) Qw[i] = static_cast<uint16_t>(hist[Qw[i]]);
    if (tid == 0) wout[w].m = m;
    __syncthreads();
  }
}

// One thread per window of [w_begin, w_end): rANS64 encode of its n symbols
// in order into enc[2 row0 cols, + 2 n) from the back (src/rans64.rs:88-166).
__global__ void pack_encode(int cols, const WinDesc* __restrict__ wins, int w_begin, int w_end,
                            const uint16_t* __restrict__ Q, const EncSym* __restrict__ esyms,
                            uint8_t* __restrict__ enc, WinOut* __restrict__ wout, uint32_t* __restrict__ status) {
  const int w = w_begin + static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x);
  if (w >= w_end || wout[w].m < 0) return;
  const WinDesc wd = wins[w];
  const int64_t n = static_cast<int64_t>(wd.rows) * cols;
  const uint16_t* q = Q + wd.row0 * cols;
  const EncSym* es = esyms + static_cast<size_t>(w - w_begin) * kMaxSyms;
  uint8_t* buf = enc + 2 * wd.row0 * cols;
  const int64_t cap = 2 * n;
  int64_t idx = cap;
  uint64_t x = kRansL;
  for (int64_t k = 0; k < n; ++k) {
    const EncSym e = es[q[k]];
    const uint64_t x_max = static_cast<uint64_t>(e.freq) << 51;  // ((2^31 >> 12) << 32) * freq
    while (x >= x_max) {
      if (idx < 4) {
        atomicOr(status, kErrEncodeOverflow);
        wout[w].m = -1;
        return;
      }
      idx -= 4;
      const uint32_t v = static_cast<uint32_t>(x);
      buf[idx] = static_cast<uint8_t>(v);
      buf[idx + 1] = static_cast<uint8_t>(v >> 8);
      buf[idx + 2] = static_cast<uint8_t>(v >> 16);
      buf[idx + 3] = static_cast<uint8_t>(v >> 24);
      x >>= 32;
    }
    const uint64_t qq = __umul64hi(x, e.rcp_freq) >> e.rcp_shift;
    x = x + e.bias + qq * ((1u << kRansBits) - e.freq);
  }
  if (idx < 8) {
    atomicOr(status, kErrEncodeOverflow);
    wout[w].m = -1;
    return;
  }
  idx -= 8;
  for (int i = 0; i < 8; ++i) buf[idx + i] = static_cast<uint8_t>(x >> (8 * i));
  wout[w].enc_start = static_cast<int>(idx);
  wout[w].enc_len = static_cast<int>(cap - idx);
}

// One CTA per window: header and rANS bytes into the output stream at
// win_off[w]; the first window of each document also writes its u32 rows.
__global__ void pack_assemble(int cols, const WinDesc* __restrict__ wins, int n_wins, const uint8_t* __restrict__ hdr,
                              const uint8_t* __restrict__ enc, const WinOut* __restrict__ wout,
                              const int64_t* __restrict__ win_off, const int64_t* __restrict__ doc_rows_first,
                              uint8_t* __restrict__ out) {
  const int w = blockIdx.x;
  if (w >= n_wins) return;
  const WinDesc wd = wins[w];
  const WinOut wo = wout[w];
  uint8_t* o = out + win_off[w];
  const uint8_t* H = hdr + static_cast<size_t>(w) * kHdrStride;
  if (threadIdx.x == 0 && wd.row0 == doc_rows_first[wd.doc]) {
    const int64_t rows = doc_rows_first[wd.doc + 1] - doc_rows_first[wd.doc];
    uint8_t* p = o - 4;
    p[0] = static_cast<uint8_t>(rows);
    p[1] = static_cast<uint8_t>(rows >> 8);
    p[2] = static_cast<uint8_t>(rows >> 16);
    p[3] = static_cast<uint8_t>(rows >> 24);
  }
  for (int i = threadIdx.x; i < cols; i += blockDim.x) o[i] = H[i];
  o += cols;
  if (threadIdx.x == 0) {
    o[0] = static_cast<uint8_t>(wo.m);
    o[1] = static_cast<uint8_t>(wo.m >> 8);
  }
  o += 2;
  for (int i = threadIdx.x; i < 4 * wo.m; i += blockDim.x) o[i] = H[kPairsOff + i];
  o += 4 * wo.m;
  if (threadIdx.x == 0) {
    o[0] = static_cast<uint8_t>(wo.enc_len);
    o[1] = static_cast<uint8_t>(wo.enc_len >> 8);
  }
  o += 2;
  const uint8_t* e = enc + 2 * wd.row0 * cols + wo.enc_start;
  for (int i = threadIdx.x; i < wo.enc_len; i += blockDim.x) o[i] = e[i];
}

// ---------------------------------------------------------------- decode

struct DecWin {
  int64_t row0;      // first output row
  int64_t hdr_off;   // byte offset of the window's permutation bytes in the input
  int rows;
  int n_sym;
  int64_t data_off;  // byte offset of the rANS bytes
  int data_len;
  int pad;
};

// One CTA per window: the symbol tables of the window in shared memory, one
// thread runs the serial rANS decode into T (src/packops.rs:318-390).
__global__ void unpack_decode(const uint8_t* __restrict__ in, int cols, const DecWin* __restrict__ wins, int n_wins,
                              float* __restrict__ T, uint32_t* __restrict__ status) {
  __shared__ float s_val[kMaxSyms];
  __shared__ uint16_t s_start[kMaxSyms];
  __shared__ uint16_t s_freq[kMaxSyms];  // 4096 does not fit: stored as freq - 1
  __shared__ int s_bad;
  const int w = blockIdx.x;
  if (w >= n_wins) return;
  const DecWin d = wins[w];
  const uint8_t* pairs = in + d.hdr_off + cols + 2;
  const float scale = __fdiv_rn(1.0f, kRange);
  if (threadIdx.x == 0) s_bad = 0;
  for (int c = threadIdx.x; c < kMaxSyms; c += blockDim.x) {
    s_val[c] = 0.0f;
    s_start[c] = 0;
    s_freq[c] = 0;  // the reference's default symbol (start 0, freq 1)
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // cumulative starts (serial: n_sym <= 4096 additions)
    uint32_t cum = 0;
    for (int i = 0; i < d.n_sym && !s_bad; ++i) {
      const uint16_t q = static_cast<uint16_t>(pairs[4 * i] | (pairs[4 * i + 1] << 8));
      const uint32_t f = static_cast<uint32_t>(pairs[4 * i + 2] | (pairs[4 * i + 3] << 8));
      if (cum + f > kMaxSyms) {
        s_bad = 1;
        break;
      }
      float v = 0.0f;
      if (q != 0) {
        const uint16_t q1 = static_cast<uint16_t>(q + 1);
        const float sign = (q1 & 1) ? -1.0f : 1.0f;
        v = __fmul_rn(__fmul_rn(scale, sign), static_cast<float>(q1 >> 1));
      }
      for (uint32_t c = cum; c < cum + f; ++c) {
        s_val[c] = v;
        s_start[c] = static_cast<uint16_t>(cum);
        s_freq[c] = static_cast<uint16_t>(f - 1);
      }
      cum += f;
    }
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  if (s_bad || d.data_len < 8) {
    atomicOr(status, kErrBadStream);
    return;
  }
  const uint8_t* p = in + d.data_off;
  uint64_t x = 0;
  for (int i = 0; i < 8; ++i) x |= static_cast<uint64_t>(p[i]) << (8 * i);
  int di = 8;
  float* t = T + d.row0 * cols;
  const uint64_t mask = (1ull << kRansBits) - 1;
  for (int64_t i = static_cast<int64_t>(d.rows) * cols - 1; i >= 0; --i) {
    const uint32_t c = static_cast<uint32_t>(x & mask);
    t[i] = s_val[c];
    x = (static_cast<uint64_t>(s_freq[c]) + 1) * (x >> kRansBits) + (x & mask) - s_start[c];
    if (x < kRansL) {
      if (di + 4 > d.data_len) {
        atomicOr(status, kErrBadStream);
        return;
      }
      const uint64_t v = static_cast<uint64_t>(p[di]) | (static_cast<uint64_t>(p[di + 1]) << 8) |
                         (static_cast<uint64_t>(p[di + 2]) << 16) | (static_cast<uint64_t>(p[di + 3]) << 24);
      di += 4;
      x = (x << 32) | v;
      if (x < kRansL) {
        atomicOr(status, kErrBadStream);
        return;
      }
    }
  }
}

// One CTA per window: inverse Haar on rows then columns, the column order
// restored, then each row L2-normalised (sum of squares in column order).
__global__ void __launch_bounds__(kThreads)
    unpack_inverse(const uint8_t* __restrict__ in, int cols, const DecWin* __restrict__ wins, int n_wins,
                   float* __restrict__ T, float* __restrict__ out) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ int s_idx[kMaxCols + 1];
  const int w = blockIdx.x;
  if (w >= n_wins) return;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const DecWin d = wins[w];
  const int R = d.rows;
  float* t = T + d.row0 * cols;
  float* bx = reinterpret_cast<float*>(smem) + warp * 2 * kWinRows;
  float* bt = bx + kWinRows;
  if (tid < cols) s_idx[tid] = in[d.hdr_off + tid];
  for (int r = warp; r < R; r += kWarps) {
    float* tr = t + static_cast<size_t>(r) * cols;
    for (int c = lane; c < cols; c += 32) bx[c] = tr[c];
    __syncwarp();
    warp_haar_inverse(bx, bt, cols, lane);
    for (int c = lane; c < cols; c += 32) tr[c] = bx[c];
    __syncwarp();
  }
  __syncthreads();
  for (int c = warp; c < cols; c += kWarps) {
    for (int r = lane; r < R; r += 32) bx[r] = t[static_cast<size_t>(r) * cols + c];
    __syncwarp();
    warp_haar_inverse(bx, bt, R, lane);
    for (int r = lane; r < R; r += 32) t[static_cast<size_t>(r) * cols + c] = bx[r];
    __syncwarp();
  }
  __syncthreads();
  float* o = out + d.row0 * cols;
  for (int r = warp; r < R; r += kWarps) {
    const float* tr = t + static_cast<size_t>(r) * cols;
    for (int c = lane; c < cols; c += 32) bx[c] = tr[s_idx[c]];
    __syncwarp();
    if (lane == 0) {
      float ss = 0.0f;
      for (int c = 0; c < cols; ++c) ss = __fadd_rn(ss, __fmul_rn(bx[c], bx[c]));
      bt[0] = __fdiv_rn(1.0f, __fsqrt_rn(ss));
    }
    __syncwarp();
    const float inv = bt[0];
    float* orow = o + static_cast<size_t>(r) * cols;
    for (int c = lane; c < cols; c += 32) orow[c] = __fmul_rn(bx[c], inv);
    __syncwarp();
  }
}

// ---------------------------------------------------------------- host side

thread_local std::string g_codec_error;

int codec_fail(int code, const std::string& msg) {
  g_codec_error = msg;
  return code;
}

// Device scratch of one device, grown on demand (one call at a time per device).
struct Scratch {
  std::mutex mu;
  void* p[10] = {};
  size_t cap[10] = {};
};
Scratch g_scratch[64];

template <typename T>
int grow(Scratch& s, int slot, size_t count, T** out) {
  const size_t bytes = std::max<size_t>(count * sizeof(T), 256);
  if (s.cap[slot] < bytes) {
    if (s.p[slot]) cudaFree(s.p[slot]);
    s.p[slot] = nullptr;
    s.cap[slot] = 0;
    const size_t want = bytes + bytes / 4;
    if (cudaMalloc(&s.p[slot], want) != cudaSuccess) return WC_E_CUDA;
    s.cap[slot] = want;
  }
  *out = static_cast<T*>(s.p[slot]);
  return WC_OK;
}

int device_sms(int dev) {
  static int counts[64] = {};
  if (!counts[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    counts[dev] = n > 0 ? n : 148;
  }
  return counts[dev];
}

int64_t window_bytes_bound(int rows, int cols) { return cols + 2 + 4ll * kMaxSyms + 2 + 2ll * rows * cols; }

}  // namespace

}  // namespace wc

using namespace wc;

extern "C" const char* wc_codec_last_error(void) { return g_codec_error.c_str(); }

extern "C" int64_t wc_packed_bound(const int64_t* doc_rows, int n_docs, int cols) {
  if (!doc_rows || n_docs < 0 || cols < 1 || cols > kMaxCols) return -1;
  int64_t b = 0;
  for (int d = 0; d < n_docs; ++d) {
    const int64_t rows = doc_rows[d + 1] - doc_rows[d];
    b += 4;
    for (int64_t r = 0; r < rows; r += kWinRows) b += window_bytes_bound(static_cast<int>(std::min<int64_t>(kWinRows, rows - r)), cols);
  }
  return b;
}

extern "C" int wc_pack_embeddings_device(const float* d_emb, const int64_t* doc_rows, int n_docs, int cols,
                                         uint8_t* d_out, int64_t out_cap, int64_t* out_offsets, void* stream) {
  if (!doc_rows || !out_offsets || n_docs < 0 || cols < 1 || cols > kMaxCols)
    return codec_fail(WC_E_INVALID_ARG, "invalid arguments (1 <= cols <= 255, doc_rows and out_offsets required)");
  out_offsets[0] = 0;
  if (n_docs == 0) return WC_OK;
  if (!d_emb || !d_out) return codec_fail(WC_E_INVALID_ARG, "null device buffer");
  std::vector<WinDesc> wins;
  for (int d = 0; d < n_docs; ++d) {
    const int64_t rows = doc_rows[d + 1] - doc_rows[d];
    if (rows < 1 || rows > 0xFFFFFFFFll)
      return codec_fail(WC_E_INVALID_ARG, "every document needs 1 <= rows < 2^32 (the reference's u32 header)");
    for (int64_t r = 0; r < rows; r += kWinRows)
      wins.push_back(WinDesc{doc_rows[d] + r, static_cast<int>(std::min<int64_t>(kWinRows, rows - r)), d});
  }
  const int n_wins = static_cast<int>(wins.size());
  const int64_t total_rows = doc_rows[n_docs] - doc_rows[0];
  if (doc_rows[0] != 0) return codec_fail(WC_E_INVALID_ARG, "doc_rows[0] must be 0");
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return codec_fail(WC_E_CUDA, "device ordinal out of range");
  Scratch& sc = g_scratch[dev];
  std::lock_guard<std::mutex> lk(sc.mu);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = std::min(std::min(n_wins, kChunkWins), 3 * device_sms(dev));
  const int chunk = std::min(n_wins, kChunkWins);
  float* S;
  uint16_t* Q;
  uint32_t* hist;
  uint8_t *hdr, *enc;
  EncSym* es;
  WinOut* wout;
  WinDesc* dwins;
  int64_t *dwoff, *ddoc;
  if (grow(sc, 0, static_cast<size_t>(total_rows) * cols, &S) || grow(sc, 1, static_cast<size_t>(total_rows) * cols, &Q) ||
      grow(sc, 2, static_cast<size_t>(grid) * 65536, &hist) || grow(sc, 3, static_cast<size_t>(n_wins) * kHdrStride, &hdr) ||
      grow(sc, 4, static_cast<size_t>(2 * total_rows * cols), &enc) || grow(sc, 5, static_cast<size_t>(chunk) * kMaxSyms, &es) ||
      grow(sc, 6, static_cast<size_t>(n_wins) + 1, &wout) || grow(sc, 7, static_cast<size_t>(n_wins), &dwins) ||
      grow(sc, 8, static_cast<size_t>(n_wins) + 1, &dwoff) || grow(sc, 9, static_cast<size_t>(n_docs) + 2, &ddoc))
    return codec_fail(WC_E_CUDA, "codec scratch allocation failed");
  uint32_t* status = reinterpret_cast<uint32_t*>(wout + n_wins);
  cudaError_t e;
  static bool attr[64] = {};
  if (!attr[dev]) {
    if ((e = cudaFuncSetAttribute(pack_transform, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(kTransformSmem))) != cudaSuccess ||
        (e = cudaFuncSetAttribute(unpack_inverse, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(kHaarFloats * sizeof(float)))) != cudaSuccess)
      return codec_fail(WC_E_CUDA, std::string("codec kernel attributes: ") + cudaGetErrorString(e));
    attr[dev] = true;
  }
  if ((e = cudaMemcpyAsync(dwins, wins.data(), sizeof(WinDesc) * n_wins, cudaMemcpyHostToDevice, st)) ||
      (e = cudaMemcpyAsync(ddoc, doc_rows, sizeof(int64_t) * (n_docs + 1), cudaMemcpyHostToDevice, st)) ||
      (e = cudaMemsetAsync(status, 0, sizeof(uint32_t), st)))
    return codec_fail(WC_E_CUDA, std::string("codec setup copies: ") + cudaGetErrorString(e));
  for (int w0 = 0; w0 < n_wins; w0 += kChunkWins) {
    const int w1 = std::min(n_wins, w0 + kChunkWins);
    pack_transform<<<std::min(grid, w1 - w0), kThreads, kTransformSmem, st>>>(d_emb, cols, dwins, w0, w1, S, Q, hist,
                                                                                hdr, es, wout, status);
    pack_encode<<<(w1 - w0 + 31) / 32, 32, 0, st>>>(cols, dwins, w0, w1, Q, es, enc, wout, status);
  }
  if ((e = cudaGetLastError()) != cudaSuccess)
    return codec_fail(WC_E_CUDA, std::string("codec launch: ") + cudaGetErrorString(e));
  std::vector<WinOut> wo(n_wins + 1);
  if ((e = cudaMemcpyAsync(wo.data(), wout, sizeof(WinOut) * (n_wins + 1), cudaMemcpyDeviceToHost, st)) ||
      (e = cudaStreamSynchronize(st)))
    return codec_fail(WC_E_CUDA, std::string("codec sizes: ") + cudaGetErrorString(e));
  uint32_t stat = 0;
  std::memcpy(&stat, &wo[n_wins], sizeof(uint32_t));
  if (stat & kErrTooManySymbols)
    return codec_fail(WC_E_UNSUPPORTED, "a window has more than 4096 distinct symbols (the reference asserts)");
  if (stat) return codec_fail(WC_E_CUDA, "rANS encoder overflow");
  // offsets: per document u32 rows, then its windows back to back
  std::vector<int64_t> woff(n_wins);
  int64_t pos = 0;
  int wi = 0;
  for (int d = 0; d < n_docs; ++d) {
    out_offsets[d] = pos;
    pos += 4;
    for (; wi < n_wins && wins[wi].doc == d; ++wi) {
      woff[wi] = pos;
      pos += cols + 2 + 4ll * wo[wi].m + 2 + wo[wi].enc_len;
    }
  }
  out_offsets[n_docs] = pos;
  if (pos > out_cap) return codec_fail(WC_E_INVALID_ARG, "output buffer too small (wc_packed_bound gives a bound)");
  if ((e = cudaMemcpyAsync(dwoff, woff.data(), sizeof(int64_t) * n_wins, cudaMemcpyHostToDevice, st)))
    return codec_fail(WC_E_CUDA, std::string("codec offsets: ") + cudaGetErrorString(e));
  pack_assemble<<<n_wins, 256, 0, st>>>(cols, dwins, n_wins, hdr, enc, wout, dwoff, ddoc, d_out);
  if ((e = cudaGetLastError()) != cudaSuccess || (e = cudaStreamSynchronize(st)) != cudaSuccess)
    return codec_fail(WC_E_CUDA, std::string("codec assemble: ") + cudaGetErrorString(e));
  return WC_OK;
}

extern "C" int wc_pack_embeddings(const float* emb, const int64_t* doc_rows, int n_docs, int cols, uint8_t* out,
                                  int64_t out_cap, int64_t* out_offsets, int device) {
  if (!doc_rows || !out_offsets || n_docs < 0 || cols < 1 || cols > kMaxCols || (n_docs > 0 && (!emb || !out)))
    return codec_fail(WC_E_INVALID_ARG, "invalid arguments");
  out_offsets[0] = 0;
  if (n_docs == 0) return WC_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  if (cudaSetDevice(device) != cudaSuccess) return codec_fail(WC_E_CUDA, "cudaSetDevice failed");
  const int64_t total = doc_rows[n_docs];
  const int64_t bound = std::min(out_cap, wc_packed_bound(doc_rows, n_docs, cols));
  float* d_emb = nullptr;
  uint8_t* d_out = nullptr;
  int rc = WC_OK;
  cudaStream_t st = nullptr;
  if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&d_emb, sizeof(float) * total * cols) != cudaSuccess || cudaMalloc(&d_out, bound) != cudaSuccess) {
    rc = codec_fail(WC_E_CUDA, "device buffers for the packed codec");
  } else if (cudaMemcpyAsync(d_emb, emb, sizeof(float) * total * cols, cudaMemcpyHostToDevice, st) != cudaSuccess) {
    rc = codec_fail(WC_E_CUDA, "copy of the embeddings");
  } else if ((rc = wc_pack_embeddings_device(d_emb, doc_rows, n_docs, cols, d_out, bound, out_offsets, st)) == WC_OK) {
    if (cudaMemcpyAsync(out, d_out, out_offsets[n_docs], cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
      rc = codec_fail(WC_E_CUDA, "copy of the packed bytes");
  }
  if (d_emb) cudaFree(d_emb);
  if (d_out) cudaFree(d_out);
  if (st) cudaStreamDestroy(st);
  cudaSetDevice(prev);
  return rc;
}

extern "C" int wc_unpack_embeddings_device(const uint8_t* d_in, const uint8_t* in, const int64_t* in_offsets,
                                           int n_docs, int cols, float* d_out, int64_t out_rows_cap,
                                           int64_t* row_offsets, void* stream) {
  if (!in || !in_offsets || !row_offsets || n_docs < 0 || cols < 1 || cols > kMaxCols)
    return codec_fail(WC_E_INVALID_ARG, "invalid arguments");
  row_offsets[0] = 0;
  if (n_docs == 0) return WC_OK;
  if (!d_in || !d_out) return codec_fail(WC_E_INVALID_ARG, "null device buffer");
  // walk the headers on the host: window boundaries and symbol counts
  std::vector<DecWin> wins;
  int64_t row = 0;
  auto get16 = [&](int64_t p) { return static_cast<int>(in[p] | (in[p + 1] << 8)); };
  for (int d = 0; d < n_docs; ++d) {
    int64_t p = in_offsets[d];
    const int64_t end = in_offsets[d + 1];
    if (end - p < 4) return codec_fail(WC_E_INVALID_ARG, "document " + std::to_string(d) + ": truncated header");
    const int64_t rows = static_cast<int64_t>(in[p]) | (static_cast<int64_t>(in[p + 1]) << 8) |
                         (static_cast<int64_t>(in[p + 2]) << 16) | (static_cast<int64_t>(in[p + 3]) << 24);
    p += 4;
    row_offsets[d] = row;
    for (int64_t r = 0; r < rows; r += kWinRows) {
      DecWin wd{};
      wd.row0 = row + r;
      wd.rows = static_cast<int>(std::min<int64_t>(kWinRows, rows - r));
      wd.hdr_off = p;
      if (p + cols + 2 > end) return codec_fail(WC_E_INVALID_ARG, "document " + std::to_string(d) + ": truncated");
      for (int c = 0; c < cols; ++c)
        if (in[p + c] >= cols) return codec_fail(WC_E_INVALID_ARG, "document " + std::to_string(d) + ": bad permutation");
      wd.n_sym = get16(p + cols);
      p += cols + 2 + 4ll * wd.n_sym;
      if (p + 2 > end) return codec_fail(WC_E_INVALID_ARG, "document " + std::to_string(d) + ": truncated");
      wd.data_len = get16(p);
      wd.data_off = p + 2;
      p += 2 + wd.data_len;
      if (p > end) return codec_fail(WC_E_INVALID_ARG, "document " + std::to_string(d) + ": truncated stream");
      wins.push_back(wd);
    }
    if (p != end)
      return codec_fail(WC_E_INVALID_ARG, "document " + std::to_string(d) + ": leftover bytes after its windows");
    row += rows;
  }
  row_offsets[n_docs] = row;
  if (row > out_rows_cap) return codec_fail(WC_E_INVALID_ARG, "output buffer too small");
  const int n_wins = static_cast<int>(wins.size());
  if (n_wins == 0) return WC_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  Scratch& sc = g_scratch[dev];
  std::lock_guard<std::mutex> lk(sc.mu);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* T;
  DecWin* dw;
  WinOut* stat_buf;
  if (grow(sc, 0, static_cast<size_t>(row) * cols, &T) || grow(sc, 7, sizeof(DecWin) * n_wins, reinterpret_cast<uint8_t**>(&dw)) ||
      grow(sc, 6, 1, &stat_buf))
    return codec_fail(WC_E_CUDA, "codec scratch allocation failed");
  uint32_t* status = reinterpret_cast<uint32_t*>(stat_buf);
  static bool attr[64] = {};
  cudaError_t e;
  if (!attr[dev]) {
    if ((e = cudaFuncSetAttribute(unpack_inverse, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(kHaarFloats * sizeof(float)))) != cudaSuccess)
      return codec_fail(WC_E_CUDA, std::string("codec kernel attributes: ") + cudaGetErrorString(e));
    attr[dev] = true;
  }
  if ((e = cudaMemcpyAsync(dw, wins.data(), sizeof(DecWin) * n_wins, cudaMemcpyHostToDevice, st)) ||
      (e = cudaMemsetAsync(status, 0, sizeof(uint32_t), st)))
    return codec_fail(WC_E_CUDA, std::string("codec setup copies: ") + cudaGetErrorString(e));
  unpack_decode<<<n_wins, 128, 0, st>>>(d_in, cols, dw, n_wins, T, status);
  unpack_inverse<<<n_wins, kThreads, kHaarFloats * sizeof(float), st>>>(d_in, cols, dw, n_wins, T, d_out);
  uint32_t hs = 0;
  if ((e = cudaGetLastError()) || (e = cudaMemcpyAsync(&hs, status, 4, cudaMemcpyDeviceToHost, st)) ||
      (e = cudaStreamSynchronize(st)))
    return codec_fail(WC_E_CUDA, std::string("codec decode: ") + cudaGetErrorString(e));
  if (hs) return codec_fail(WC_E_INVALID_ARG, "malformed rANS stream");
  return WC_OK;
}

extern "C" int wc_unpack_embeddings(const uint8_t* in, const int64_t* in_offsets, int n_docs, int cols, float* out,
                                    int64_t out_rows_cap, int64_t* row_offsets, int device) {
  if (!in || !in_offsets || !row_offsets || n_docs < 0 || cols < 1 || cols > kMaxCols || (n_docs > 0 && !out))
    return codec_fail(WC_E_INVALID_ARG, "invalid arguments");
  row_offsets[0] = 0;
  if (n_docs == 0) return WC_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  if (cudaSetDevice(device) != cudaSuccess) return codec_fail(WC_E_CUDA, "cudaSetDevice failed");
  const int64_t nbytes = in_offsets[n_docs];
  uint8_t* d_in = nullptr;
  float* d_out = nullptr;
  cudaStream_t st = nullptr;
  int rc = WC_OK;
  if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&d_in, std::max<int64_t>(nbytes, 1)) != cudaSuccess ||
      cudaMalloc(&d_out, sizeof(float) * std::max<int64_t>(out_rows_cap, 1) * cols) != cudaSuccess) {
    rc = codec_fail(WC_E_CUDA, "device buffers for the packed codec");
  } else if (cudaMemcpyAsync(d_in, in, nbytes, cudaMemcpyHostToDevice, st) != cudaSuccess) {
    rc = codec_fail(WC_E_CUDA, "copy of the packed bytes");
  } else if ((rc = wc_unpack_embeddings_device(d_in, in, in_offsets, n_docs, cols, d_out, out_rows_cap, row_offsets,
                                               st)) == WC_OK) {
    if (cudaMemcpyAsync(out, d_out, sizeof(float) * row_offsets[n_docs] * cols, cudaMemcpyDeviceToHost, st) !=
            cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
      rc = codec_fail(WC_E_CUDA, "copy of the embeddings");
  }
  if (d_in) cudaFree(d_in);
  if (d_out) cudaFree(d_out);
  if (st) cudaStreamDestroy(st);
  cudaSetDevice(prev);
  return rc;
}
