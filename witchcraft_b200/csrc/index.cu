// Index-build steps on the GPU (src/lib.rs:187-274, 1376): nearest-center
// assignment (matmul_argmax_batched), the k-means center update, and the
// 4-bit mu-law residual codes.
//
// assign_kernel: X [m][dim] f32 against C [k][dim] f32, dim <= 128.  One CTA
//   owns 128 rows, keeps them transposed in shared memory and streams the
//   centers through in tiles of 256; each thread holds an 8 x 16 block of dot
//   products, each one fused-multiply-add chain over the dimensions in order
//   (so every similarity is the same f32 number a serial fmaf loop gives), and
//   folds each tile into its rows' running (best value, first index).  This is
//   FP32 CUDA-core work on purpose: tensor-core formats round the operands
//   (tf32: 10-bit mantissa), which flips near-tie assignments among tens of
//   thousands of centers.
// kmeans_update: the rows stably sorted by center (CUB radix sort, so each
//   center's rows stay in row order), then one warp per center sums its rows
//   dimension by dimension in that order and divides by the L2 norm, exactly
//   the reference's loop (src/lib.rs:238-274).
// residual_q4: (x - center) -> mu-law compand -> quantize(4) -> nibbles.
#include "common.cuh"
#include "index_ops.h"

#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>

#include <mutex>
#include <string>

namespace wc {

namespace {

constexpr int kTile = 128;   // rows per CTA
constexpr int kCTile = 256;  // centers per streamed tile
constexpr int kMaxDim = 128;

// 256 threads: thread (ty = tid / 16, tx = tid % 16) owns rows 8 ty .. 8 ty + 7
// and centers 64 q + 4 tx + (0..3), q = 0..3, of each tile: 128 dot products
// per thread.  Shared-memory loads cost one wavefront per float a thread
// reads per dimension, so the 8 x 16 block needs 24 wavefronts per 128 FMAs
// of a warp and the FMA pipes, not the shared-memory pipe, set the pace.
__global__ void __launch_bounds__(256, 1)
    assign_kernel(const float* __restrict__ X, int64_t m, const float* __restrict__ C, int64_t k, int dim,
                  uint32_t* __restrict__ idx) {
  extern __shared__ __align__(16) float smem[];
  float* Xs = smem;                    // [dim][kTile] rows transposed
  float* Cs = smem + kMaxDim * kTile;  // [dim][kCTile] centers transposed
  __shared__ float s_best[kTile];
  __shared__ uint32_t s_bidx[kTile];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kTile;
  // transposed fills: consecutive threads take consecutive rows (conflict-
  // free shared stores), each reading 4 dimensions at once
  const int d4n = dim / 4;
  for (int i = tid; i < kTile * d4n; i += 256) {
    const int r = i % kTile, d4 = i / kTile;
    const float4 v = row0 + r < m ? *reinterpret_cast<const float4*>(X + (row0 + r) * dim + 4 * d4)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
    Xs[(4 * d4) * kTile + r] = v.x;
    Xs[(4 * d4 + 1) * kTile + r] = v.y;
    Xs[(4 * d4 + 2) * kTile + r] = v.z;
    Xs[(4 * d4 + 3) * kTile + r] = v.w;
  }
  if (tid < kTile) {
    s_best[tid] = -INFINITY;
    s_bidx[tid] = 0;
  }
  for (int64_t c0 = 0; c0 < k; c0 += kCTile) {
    __syncthreads();  // previous tile consumed
    for (int i = tid; i < kCTile * d4n; i += 256) {
      const int r = i % kCTile, d4 = i / kCTile;
      const float4 v = c0 + r < k ? *reinterpret_cast<const float4*>(C + (c0 + r) * dim + 4 * d4)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
      Cs[(4 * d4) * kCTile + r] = v.x;
      Cs[(4 * d4 + 1) * kCTile + r] = v.y;
      Cs[(4 * d4 + 2) * kCTile + r] = v.z;
      Cs[(4 * d4 + 3) * kCTile + r] = v.w;
    }
    __syncthreads();
    float acc[8][16];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 16; ++j) acc[i][j] = 0.0f;
#pragma unroll 2
    for (int d = 0; d < dim; ++d) {
      // rows: 2 distinct addresses per warp (broadcast); centers: each
      // quarter of a warp reads one contiguous 128-byte span per load
      const float4 xa = *reinterpret_cast<const float4*>(Xs + d * kTile + 8 * ty);
      const float4 xb = *reinterpret_cast<const float4*>(Xs + d * kTile + 8 * ty + 4);
      float cv[16];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 c4 = *reinterpret_cast<const float4*>(Cs + d * kCTile + 64 * q + 4 * tx);
        cv[4 * q] = c4.x;
        cv[4 * q + 1] = c4.y;
        cv[4 * q + 2] = c4.z;
        cv[4 * q + 3] = c4.w;
      }
      const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[i][j] = __fmaf_rn(xv[i], cv[j], acc[i][j]);
    }
    // per row: first maximum over this thread's 16 centers, then over the 16
    // threads of the row group (lanes with the same ty), then fold into the
    // running best (earlier tiles win ties)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float bv = -INFINITY;
      uint32_t bj = 0xFFFFFFFFu;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int64_t c = c0 + 64 * (j >> 2) + 4 * tx + (j & 3);  // increasing in j
        if (c < k && (acc[i][j] > bv || bj == 0xFFFFFFFFu)) {
          bv = acc[i][j];
          bj = static_cast<uint32_t>(c);
        }
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
        const uint32_t oj = __shfl_xor_sync(0xFFFFFFFFu, bj, o);
        if (oj != 0xFFFFFFFFu && (bj == 0xFFFFFFFFu || ov > bv || (ov == bv && oj < bj))) {
          bv = ov;
          bj = oj;
        }
      }
      if (tx == 0) {
        const int r = 8 * ty + i;
        if (bj != 0xFFFFFFFFu && (c0 == 0 || bv > s_best[r])) {
          s_best[r] = bv;
          s_bidx[r] = bj;
        }
      }
    }
  }
  __syncthreads();
  if (tid < kTile && row0 + tid < m) idx[row0 + tid] = s_bidx[tid];
}

// One warp per center: sum its rows (sorted order = row order) per dimension,
// then divide by the L2 norm (sum of squares in dimension order).
__global__ void kmeans_update_kernel(const float* __restrict__ X, int dim, const uint32_t* __restrict__ sorted_rows,
                                     const uint32_t* __restrict__ seg_start, const uint32_t* __restrict__ counts,
                                     int64_t k, const int64_t* __restrict__ empty_src, float* __restrict__ out) {
  const int64_t c = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (c >= k) return;
  float s[kMaxDim / 32];
#pragma unroll
  for (int q = 0; q < kMaxDim / 32; ++q) s[q] = 0.0f;
  const uint32_t n = counts[c], beg = seg_start[c];
  if (n > 0) {
    for (uint32_t t = 0; t < n; ++t) {
      const float* xr = X + static_cast<int64_t>(sorted_rows[beg + t]) * dim;
#pragma unroll
      for (int q = 0; q < kMaxDim / 32; ++q)
        if (lane + 32 * q < dim) s[q] = __fadd_rn(s[q], xr[lane + 32 * q]);
    }
  } else {
    const float* xr = X + empty_src[c] * dim;
#pragma unroll
    for (int q = 0; q < kMaxDim / 32; ++q)
      if (lane + 32 * q < dim) s[q] = xr[lane + 32 * q];
  }
  // sum of squares in dimension order: gather to lane 0 through shared memory
  __shared__ float s_row[8][kMaxDim];
  float* row = s_row[threadIdx.x >> 5];
#pragma unroll
  for (int q = 0; q < kMaxDim / 32; ++q)
    if (lane + 32 * q < dim) row[lane + 32 * q] = s[q];
  __syncwarp();
  float norm = 0.0f;
  if (lane == 0) {
    float ss = 0.0f;
    for (int d = 0; d < dim; ++d) ss = __fadd_rn(ss, __fmul_rn(row[d], row[d]));
    norm = __fsqrt_rn(ss);
  }
  norm = __shfl_sync(0xFFFFFFFFu, norm, 0);
#pragma unroll
  for (int q = 0; q < kMaxDim / 32; ++q)
    if (lane + 32 * q < dim) out[c * dim + lane + 32 * q] = norm > 0.0f ? __fdiv_rn(s[q], norm) : s[q];
}

__global__ void count_kernel(const uint32_t* __restrict__ idx, int64_t m, uint32_t* __restrict__ counts) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < m) atomicAdd(&counts[idx[i]], 1u);
}

__global__ void iota_kernel(uint32_t* __restrict__ v, int64_t m) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < m) v[i] = static_cast<uint32_t>(i);
}

__device__ __forceinline__ uint32_t compand_q4(float r) {
  const float s = __fmul_rn(r, 4.0f);
  const float inv_den = static_cast<float>(1.0 / 5.5451774444795623);  // (1 / ln 256) rounded to f32
  const float y = __fmul_rn(logf(__fadd_rn(__fmul_rn(fabsf(s), 255.0f), 1.0f)), inv_den);
  const float v = s > 0.0f ? y : (s < 0.0f ? -y : 0.0f);
  float q = roundf(__fadd_rn(__fmul_rn(v, 7.5f), 7.5f));
  q = fminf(fmaxf(q, 0.0f), 15.0f);
  return static_cast<uint32_t>(q) & 0x0Fu;
}

__global__ void residual_q4_kernel(const float* __restrict__ X, int64_t m, int dim, const uint32_t* __restrict__ idx,
                                   const float* __restrict__ C, uint8_t* __restrict__ out) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int half = dim / 2;
  if (t >= m * half) return;
  const int64_t i = t / half;
  const int d = 2 * static_cast<int>(t % half);
  const float* xi = X + i * dim;
  const float* ci = C + static_cast<int64_t>(idx[i]) * dim;
  const uint32_t hi = compand_q4(__fsub_rn(xi[d], ci[d]));
  const uint32_t lo = compand_q4(__fsub_rn(xi[d + 1], ci[d + 1]));
  out[t] = static_cast<uint8_t>((hi << 4) | lo);
}

thread_local std::string g_index_error;
int ifail(int code, const std::string& m) {
  g_index_error = m;
  return code;
}

}  // namespace

}  // namespace wc

using namespace wc;

extern "C" const char* wc_index_last_error(void) { return g_index_error.c_str(); }

extern "C" int wc_assign_centers(const float* d_x, int64_t m, const float* d_centers, int64_t k, int dim,
                                 uint32_t* d_idx, void* stream) {
  if (m < 0 || k < 1 || dim < 1 || dim > kMaxDim || dim % 4 || k > 0xFFFFFFFFll || (m > 0 && (!d_x || !d_idx)) ||
      !d_centers)
    return ifail(WC_E_INVALID_ARG, "invalid arguments (1 <= dim <= 128, dim % 4 == 0, k >= 1)");
  if (m == 0) return WC_OK;
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int smem = kMaxDim * (kTile + kCTile) * sizeof(float);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    if (cudaFuncSetAttribute(assign_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return ifail(WC_E_CUDA, "assign kernel attribute");
    attr[dev] = true;
  }
  assign_kernel<<<static_cast<unsigned>((m + kTile - 1) / kTile), 256, smem, static_cast<cudaStream_t>(stream)>>>(
      d_x, m, d_centers, k, dim, d_idx);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? WC_OK : ifail(WC_E_CUDA, std::string("assign launch: ") + cudaGetErrorString(e));
}

extern "C" int wc_kmeans_update(const float* d_x, int64_t m, int dim, const uint32_t* d_idx, int64_t k,
                                const int64_t* d_empty_src, float* d_centers_out, uint32_t* d_counts, void* stream) {
  if (m < 1 || m > 0xFFFFFFFFll || k < 1 || dim < 1 || dim > kMaxDim || !d_x || !d_idx || !d_empty_src ||
      !d_centers_out || !d_counts)
    return ifail(WC_E_INVALID_ARG, "invalid arguments (1 <= dim <= 128, m, k >= 1)");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // scratch: sorted keys/values, row ids, segment starts, CUB temp
  uint32_t *keys_out = nullptr, *rows_in = nullptr, *rows_out = nullptr, *seg = nullptr;
  void* tmp = nullptr;
  size_t tmp_bytes = 0;
  int end_bit = 1;
  while (end_bit < 32 && (1ll << end_bit) < k) ++end_bit;
  cub::DeviceRadixSort::SortPairs(nullptr, tmp_bytes, d_idx, keys_out, rows_in, rows_out, static_cast<int>(m), 0,
                                  end_bit, st);
  int rc = WC_OK;
  if (cudaMallocAsync(&keys_out, m * 4, st) || cudaMallocAsync(&rows_in, m * 4, st) ||
      cudaMallocAsync(&rows_out, m * 4, st) || cudaMallocAsync(&seg, k * 4, st) ||
      cudaMallocAsync(&tmp, tmp_bytes, st)) {
    rc = ifail(WC_E_CUDA, "k-means scratch allocation");
  } else {
    cudaMemsetAsync(d_counts, 0, k * 4, st);
    iota_kernel<<<static_cast<unsigned>((m + 255) / 256), 256, 0, st>>>(rows_in, m);
    count_kernel<<<static_cast<unsigned>((m + 255) / 256), 256, 0, st>>>(d_idx, m, d_counts);
    cub::DeviceRadixSort::SortPairs(tmp, tmp_bytes, d_idx, keys_out, rows_in, rows_out, static_cast<int>(m), 0,
                                    end_bit, st);
    size_t scan_bytes = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, scan_bytes, d_counts, seg, static_cast<int>(k), st);
    void* scan_tmp = nullptr;
    if (cudaMallocAsync(&scan_tmp, scan_bytes, st)) {
      rc = ifail(WC_E_CUDA, "k-means scan scratch");
    } else {
      cub::DeviceScan::ExclusiveSum(scan_tmp, scan_bytes, d_counts, seg, static_cast<int>(k), st);
      kmeans_update_kernel<<<static_cast<unsigned>((k + 7) / 8), 256, 0, st>>>(d_x, dim, rows_out, seg, d_counts, k,
                                                                               d_empty_src, d_centers_out);
      cudaFreeAsync(scan_tmp, st);
    }
  }
  if (keys_out) cudaFreeAsync(keys_out, st);
  if (rows_in) cudaFreeAsync(rows_in, st);
  if (rows_out) cudaFreeAsync(rows_out, st);
  if (seg) cudaFreeAsync(seg, st);
  if (tmp) cudaFreeAsync(tmp, st);
  const cudaError_t e = cudaGetLastError();
  if (rc == WC_OK && e != cudaSuccess) rc = ifail(WC_E_CUDA, std::string("k-means update: ") + cudaGetErrorString(e));
  return rc;
}

extern "C" int wc_residual_q4(const float* d_x, int64_t m, int dim, const uint32_t* d_idx, const float* d_centers,
                              uint8_t* d_out, void* stream) {
  if (m < 0 || dim < 2 || dim % 2 || (m > 0 && (!d_x || !d_idx || !d_centers || !d_out)))
    return ifail(WC_E_INVALID_ARG, "invalid arguments (dim even)");
  if (m == 0) return WC_OK;
  const int64_t n = m * (dim / 2);
  residual_q4_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      d_x, m, dim, d_idx, d_centers, d_out);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? WC_OK : ifail(WC_E_CUDA, std::string("residual launch: ") + cudaGetErrorString(e));
}
