// Query-side candidate scoring of match_centroids (src/lib.rs:715-808) on the
// GPU.  The host picks the clusters and gathers the candidates (indexed rows
// as 4-bit residual codes with their cluster, unindexed rows as f32) and
// their (document, sub-chunk) grouping in sorted order; this kernel scores
// every sub-chunk.
//
// One warp per document walks its groups in order; lane t keeps query token
// t's running maximum (starting at `missing`, carried across the document's
// sub-chunks as the reference's doc_scores / sub_scores do).  Each row is
// decoded once into the warp's shared buffer (two table lookups per byte),
// then every lane takes its token's dot product as one fmaf chain over the
// dimensions in order, adds the centroid score for indexed rows and folds it
// into the maximum.  A sub-chunk's score is (1/m) * the sum over tokens in
// token order (lane 0, from shared memory).  Queries longer than 32 tokens
// give each lane ceil(m / 32) tokens.
#include "common.cuh"
#include "query_ops.h"

#include <cmath>
#include <string>

namespace wc {

namespace {

constexpr int kMaxDim = 128;
constexpr int kMaxTokens = 128;
constexpr int kWarpsPerBlock = 4;

__global__ void __launch_bounds__(32 * kWarpsPerBlock)
    score_kernel(const float* __restrict__ q, int m, int dim, const uint8_t* __restrict__ codes,
                 const uint32_t* __restrict__ cluster, const float* __restrict__ cscores, int n_cent,
                 const float* __restrict__ table, int64_t n_idx, const float* __restrict__ raw,
                 const int64_t* __restrict__ group_rows, const int64_t* __restrict__ group_start,
                 const int64_t* __restrict__ doc_start, int64_t n_docs, const float* __restrict__ missing,
                 float* __restrict__ out) {
  __shared__ float s_row[kWarpsPerBlock][kMaxDim];
  __shared__ float s_tok[kWarpsPerBlock][kMaxTokens];
  __shared__ float s_tab[16];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  if (threadIdx.x < 16) s_tab[threadIdx.x] = table[threadIdx.x];
  __syncthreads();
  const int64_t d = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + wib;
  if (d >= n_docs) return;
  float* row = s_row[wib];
  float* tok = s_tok[wib];
  constexpr int kPer = kMaxTokens / 32;
  float smax[kPer];
#pragma unroll
  for (int u = 0; u < kPer; ++u) {
    const int t = lane + 32 * u;
    smax[u] = t < m ? missing[t] : 0.0f;
  }
  for (int64_t g = doc_start[d]; g < doc_start[d + 1]; ++g) {
    for (int64_t p = group_start[g]; p < group_start[g + 1]; ++p) {
      const int64_t r = group_rows[p];
      const bool indexed = r < n_idx;
      __syncwarp();
      if (indexed) {
        const uint8_t* cr = codes + r * (dim / 2);
        for (int k = lane; k < dim / 2; k += 32) {
          const uint8_t b = cr[k];
          row[2 * k] = s_tab[b >> 4];
          row[2 * k + 1] = s_tab[b & 15];
        }
      } else {
        const float* er = raw + (r - n_idx) * dim;
        for (int k = lane; k < dim; k += 32) row[k] = er[k];
      }
      __syncwarp();
      const uint32_t cl = indexed ? cluster[r] : 0u;
#pragma unroll
      for (int u = 0; u < kPer; ++u) {
        const int t = lane + 32 * u;
        if (t < m) {
          const float* qt = q + static_cast<int64_t>(t) * dim;
          float acc = 0.0f;
          for (int k = 0; k < dim; ++k) acc = __fmaf_rn(qt[k], row[k], acc);
          if (indexed) acc = __fadd_rn(acc, cscores[static_cast<int64_t>(t) * n_cent + cl]);
          smax[u] = fmaxf(smax[u], acc);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int t = lane + 32 * u;
      if (t < m) tok[t] = smax[u];
    }
    __syncwarp();
    if (lane == 0) {
      float sum = 0.0f;
      for (int t = 0; t < m; ++t) sum = __fadd_rn(sum, tok[t]);
      out[g] = __fmul_rn(__fdiv_rn(1.0f, static_cast<float>(m)), sum);
    }
    __syncwarp();
  }
}

// The same scoring for the common shape (m <= 32 query tokens, dim = 128):
// lane t holds query token t in registers, and the warp decodes R rows of a
// sub-chunk at a time into shared memory, so each lane runs R independent
// fmaf chains (each still over the dimensions in order, so every dot product
// is the same bits as the general kernel's) and reads each row value once per
// four dimensions (float4 broadcast loads).
template <int R>
__global__ void __launch_bounds__(32 * kWarpsPerBlock)
    score_kernel_q128(const float* __restrict__ q, int m, const uint8_t* __restrict__ codes,
                      const uint32_t* __restrict__ cluster, const float* __restrict__ cscores, int n_cent,
                      const float* __restrict__ table, int64_t n_idx, const float* __restrict__ raw,
                      const int64_t* __restrict__ group_rows, const int64_t* __restrict__ group_start,
                      const int64_t* __restrict__ doc_start, int64_t n_docs, const float* __restrict__ missing,
                      float* __restrict__ out) {
  constexpr int D = 128;
  __shared__ __align__(16) float s_row[kWarpsPerBlock][R][D];
  __shared__ float s_tok[kWarpsPerBlock][32];
  __shared__ float s_tab[16];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  if (threadIdx.x < 16) s_tab[threadIdx.x] = table[threadIdx.x];
  __syncthreads();
  const int64_t d = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + wib;
  if (d >= n_docs) return;
  const bool active = lane < m;
  float qv[D];
#pragma unroll
  for (int k = 0; k < D; k += 4) {
    const float4 v = active ? *reinterpret_cast<const float4*>(q + static_cast<int64_t>(lane) * D + k)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
    qv[k] = v.x;
    qv[k + 1] = v.y;
    qv[k + 2] = v.z;
    qv[k + 3] = v.w;
  }
  float smax = active ? missing[lane] : 0.0f;
  const float* cs_t = cscores + static_cast<int64_t>(active ? lane : 0) * n_cent;
  // The codes and centroid scores of the next R rows are fetched (into
  // registers) while the current R rows are scored, so their global-memory
  // latency overlaps the fmaf chains.  Raw (unindexed) rows are read when
  // their turn comes.
  const int64_t g0 = doc_start[d], g1 = doc_start[d + 1];
  int64_t g = g0, p = g0 < g1 ? group_start[g0] : 0;
  auto next_rows = [&](int64_t& gg, int64_t& pp, int64_t (&rid)[R], uchar2 (&cb)[R], float (&cv)[R], int& nr,
                       int64_t& grp) {
    // the rows [pp, pp + nr) of group gg (nr = 0 past the document)
    while (gg < g1 && pp >= group_start[gg + 1]) {
      ++gg;
      if (gg < g1) pp = group_start[gg];
    }
    grp = gg;
    nr = 0;
    if (gg >= g1) return;
    const int64_t ge = group_start[gg + 1];
    nr = static_cast<int>(ge - pp < R ? ge - pp : R);
#pragma unroll
    for (int rr = 0; rr < R; ++rr) {
      rid[rr] = rr < nr ? group_rows[pp + rr] : -1;
      cb[rr] = (rr < nr && rid[rr] < n_idx) ? *reinterpret_cast<const uchar2*>(codes + rid[rr] * (D / 2) + 2 * lane)
                                            : make_uchar2(0, 0);
    }
    // the centroid score of each indexed row for this lane's token
#pragma unroll
    for (int rr = 0; rr < R; ++rr) cv[rr] = (rr < nr && rid[rr] < n_idx) ? cs_t[cluster[rid[rr]]] : 0.0f;
    pp += nr;
  };
  // score of groups [ga, gb) given the running maxima (one sum, written to
  // each: groups without rows keep the maxima of the groups before them)
  auto emit = [&](int64_t ga, int64_t gb) {
    if (ga >= gb) return;
    if (active) s_tok[wib][lane] = smax;
    __syncwarp();
    if (lane == 0) {
      float sum = 0.0f;
      for (int t = 0; t < m; ++t) sum = __fadd_rn(sum, s_tok[wib][t]);
      const float sc = __fmul_rn(__fdiv_rn(1.0f, static_cast<float>(m)), sum);
      for (int64_t gg = ga; gg < gb; ++gg) out[gg] = sc;
    }
    __syncwarp();
  };
  int64_t rid[R], grp;
  uchar2 cb[R];
  float cv[R];
  int nr;
  next_rows(g, p, rid, cb, cv, nr, grp);
  emit(g0, nr > 0 ? grp : g1);  // leading groups without rows
  while (nr > 0) {
    __syncwarp();
#pragma unroll
    for (int rr = 0; rr < R; ++rr) {
      if (rr >= nr) continue;
      float* row = s_row[wib][rr];
      if (rid[rr] < n_idx)
        *reinterpret_cast<float4*>(row + 4 * lane) =
            make_float4(s_tab[cb[rr].x >> 4], s_tab[cb[rr].x & 15], s_tab[cb[rr].y >> 4], s_tab[cb[rr].y & 15]);
      else
        *reinterpret_cast<float4*>(row + 4 * lane) =
            *reinterpret_cast<const float4*>(raw + (rid[rr] - n_idx) * D + 4 * lane);
    }
    __syncwarp();
    const int cur_nr = nr;
    const int64_t cur_grp = grp;
    int64_t cur_rid[R];
    float cur_cv[R];
#pragma unroll
    for (int rr = 0; rr < R; ++rr) {
      cur_rid[rr] = rid[rr];
      cur_cv[rr] = cv[rr];
    }
    next_rows(g, p, rid, cb, cv, nr, grp);  // prefetch
    float acc[R];
#pragma unroll
    for (int rr = 0; rr < R; ++rr) acc[rr] = 0.0f;
#pragma unroll
    for (int k = 0; k < D; k += 4) {
#pragma unroll
      for (int rr = 0; rr < R; ++rr) {
        const float4 x = *reinterpret_cast<const float4*>(&s_row[wib][rr][k]);
        acc[rr] = __fmaf_rn(qv[k], x.x, acc[rr]);
        acc[rr] = __fmaf_rn(qv[k + 1], x.y, acc[rr]);
        acc[rr] = __fmaf_rn(qv[k + 2], x.z, acc[rr]);
        acc[rr] = __fmaf_rn(qv[k + 3], x.w, acc[rr]);
      }
    }
#pragma unroll
    for (int rr = 0; rr < R; ++rr) {
      if (rr < cur_nr && active) {
        float a = acc[rr];
        if (cur_rid[rr] < n_idx) a = __fadd_rn(a, cur_cv[rr]);
        smax = fmaxf(smax, a);
      }
    }
    // the sub-chunk ends when the next rows belong to another group (or none)
    // (and groups without rows before the next one get the same score)
    if (nr == 0 || grp != cur_grp) emit(cur_grp, nr > 0 ? grp : g1);
  }
}

// out[t][j] = <q_t, c_j>, one fmaf chain over the dimensions per output.
__global__ void similarities_kernel(const float* __restrict__ q, int m, const float* __restrict__ c, int64_t k, int dim,
                                    float* __restrict__ out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= m * k) return;
  const int64_t t = i / k, j = i % k;
  const float* qt = q + t * dim;
  const float* cj = c + j * dim;
  float acc = 0.0f;
  for (int d = 0; d < dim; ++d) acc = __fmaf_rn(qt[d], cj[d], acc);
  out[i] = acc;
}

thread_local std::string g_query_error;

}  // namespace

}  // namespace wc

using namespace wc;

extern "C" const char* wc_query_last_error(void) { return g_query_error.c_str(); }

// Host code: libm's expf / logf, the functions Rust's f32 exp / ln call.
extern "C" int wc_q4_table(float* out) {
  if (!out) return WC_E_INVALID_ARG;
  for (int q = 0; q < 16; ++q) {
    const float x = (static_cast<float>(q) - 7.5f) * static_cast<float>(2.0 / 15.0);
    const float a = fabsf(x);
    const float sign = x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f);
    volatile float l = logf(256.0f);  // keep the library call (no constant folding)
    const float p = expf(a * l);
    const float scaled = sign * ((p - 1.0f) * static_cast<float>(1.0 / 255.0));
    out[q] = scaled * 0.25f;
  }
  return WC_OK;
}

extern "C" int wc_similarities(const float* d_q, int m, const float* d_c, int64_t k, int dim, float* d_out,
                               void* stream) {
  if (m < 1 || k < 1 || dim < 1 || !d_q || !d_c || !d_out) {
    g_query_error = "invalid arguments";
    return WC_E_INVALID_ARG;
  }
  const int64_t n = static_cast<int64_t>(m) * k;
  similarities_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      d_q, m, d_c, k, dim, d_out);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    g_query_error = std::string("similarities launch: ") + cudaGetErrorString(e);
    return WC_E_CUDA;
  }
  return WC_OK;
}

extern "C" int wc_score_candidates(const float* d_q, int m, int dim, const uint8_t* d_codes, const uint32_t* d_cluster,
                                   const float* d_cscores, int n_cent, const float* d_table, int64_t n_idx,
                                   const float* d_raw, const int64_t* d_group_rows, const int64_t* d_group_start,
                                   const int64_t* d_doc_start, int64_t n_docs, const float* d_missing, float* d_out,
                                   void* stream) {
  if (m < 1 || m > kMaxTokens || dim < 2 || dim > kMaxDim || dim % 2 || n_docs < 0 || n_idx < 0 || !d_q ||
      !d_table || !d_missing || (n_docs > 0 && (!d_group_rows || !d_group_start || !d_doc_start || !d_out)) ||
      (n_idx > 0 && (!d_codes || !d_cluster || !d_cscores || n_cent < 1))) {
    g_query_error = "invalid arguments (1 <= m <= 128 query tokens, even dim <= 128)";
    return WC_E_INVALID_ARG;
  }
  if (n_docs == 0) return WC_OK;
  if (m <= 32 && dim == 128 && (reinterpret_cast<uintptr_t>(d_q) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(d_raw) & 15) == 0 && (reinterpret_cast<uintptr_t>(d_codes) & 1) == 0) {
    score_kernel_q128<4><<<static_cast<unsigned>((n_docs + kWarpsPerBlock - 1) / kWarpsPerBlock),
                           32 * kWarpsPerBlock, 0, static_cast<cudaStream_t>(stream)>>>(
        d_q, m, d_codes, d_cluster, d_cscores, n_cent, d_table, n_idx, d_raw, d_group_rows, d_group_start,
        d_doc_start, n_docs, d_missing, d_out);
  } else {
  score_kernel<<<static_cast<unsigned>((n_docs + kWarpsPerBlock - 1) / kWarpsPerBlock), 32 * kWarpsPerBlock, 0,
                 static_cast<cudaStream_t>(stream)>>>(d_q, m, dim, d_codes, d_cluster, d_cscores, n_cent, d_table,
                                                      n_idx, d_raw, d_group_rows, d_group_start, d_doc_start, n_docs,
                                                      d_missing, d_out);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    g_query_error = std::string("score launch: ") + cudaGetErrorString(e);
    return WC_E_CUDA;
  }
  return WC_OK;
}
