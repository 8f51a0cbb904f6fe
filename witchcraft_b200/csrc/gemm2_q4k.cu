// Q4_K x f16 GEMM on pairs of SMs (tcgen05 cta_group::2), persistent, with a
// double-buffered TMEM accumulator so the epilogue of one tile overlaps the
// main loop of the next.  Same contract as gemm_q4k.cu
// (Y[M, N] = X[M, K] . W[N, K]^T, W in Q4_K rows) and the same epilogues; used
// for the large-M encoder GEMMs (QKV, O, wi_0|wi_1 + gated GELU, wo).
//
// A cluster of two CTAs (one per SM) owns a 256 x 256 output tile:
//   - each CTA TMA-loads its own 128 rows of X per 64-wide K step;
//   - each CTA dequantises its own half of the B tile (128 weight rows) from
//     raw Q4_K super-blocks into f16, so the per-SM dequant work is half of
//     what a 1-SM 128 x 256 tile needs for the same tensor-core work;
//   - the even CTA's single MMA thread issues tcgen05.mma.cta_group::2
//     (M = 256, N = 256) reading A and B from both CTAs' shared memory;
//   - each CTA's TMEM holds the f32 accumulator of its 128 rows x 256 columns,
//     twice (512 columns), and its epilogue warps drain one buffer while the
//     MMAs fill the other.
// For the gated GELU the even CTA's B half is wi_0 rows and the odd CTA's is
// the wi_1 rows of the same 128 features, so accumulator columns [0, 128) are
// gate and [128, 256) are up for every row.
//
// Warp roles (448 threads per CTA):
//   warp 0      TMA producer (X stages; raw Q4_K stages)
//   warp 1      TMEM allocation; MMA issue (even CTA, one thread)
//   warps 2-9   dequant: raw Q4_K -> f16 K-major 128-B-swizzled B stages
//   warps 10-13 epilogue: tcgen05.ld -> registers -> swizzled smem staging ->
//               TMA tensor store (kEpiResid: TMA reduce-add into x)
// With WF16 the weights are already f16 ([N][K], dequantised once from the
// same Q4_K bytes with the same arithmetic, so the operands are bit-identical):
// the producer TMA-loads each CTA's 128-row B half into the stage of its X
// rows, both completing on the same barrier, and the dequant warps idle.
// Cross-CTA signalling: X loads of both CTAs complete on the even CTA's
// barrier; dequant and epilogue warps arrive on the even CTA's barriers
// through shared::cluster addresses; MMA completion is committed to both
// CTAs' barriers (tcgen05.commit multicast).  No TMA load is multicast.
#include "common.cuh"
#include "gemm2_q4k.h"
#include "q4k.cuh"

#include <algorithm>
#include <cstdlib>

namespace wc {

namespace {

constexpr int kBM = 256;          // rows per cluster tile (128 per CTA)
constexpr int kBN = 256;          // columns per tile (128 weight rows per CTA)
constexpr int kBK = 64;
constexpr int kHalfN = kBN / 2;   // weight rows dequantised by one CTA
constexpr int kSA = 4;            // X ring depth
constexpr int kSW = 3;            // raw Q4_K ring depth (super-blocks)
constexpr int kSB = 4;            // dequantised B ring depth
constexpr int kABytes = 128 * kBK * 2;
constexpr int kWBytes = kHalfN * 144;
constexpr int kBBytes = kHalfN * kBK * 2;
constexpr int kOffA = 0;
constexpr int kOffW = kOffA + kSA * kABytes;
constexpr int kOffB = kOffW + kSW * kWBytes;
constexpr int kOutBytes = 32 * 128;  // one staged 32-row x 128-byte output chunk
constexpr int kOffOut = kOffB + kSB * kBBytes;  // [epilogue warp][2] staged chunks (Q4_K variant)
// Shared-memory plan per variant.  With f16 weights there is no raw Q4_K
// ring, and its space buys a deeper X / B ring: stage i holds X and the
// weight rows of the same K step.  (Four staged output chunks per epilogue
// warp instead of two, at the cost of one stage, made the f32 epilogues no
// faster.)
template <int EPI, bool WF16, int BN = kBN>
struct Plan {
  static constexpr int kStages = WF16 ? 6 : kSA;
  static constexpr int kNOut = 2;  // staged output chunks per epilogue warp
  static constexpr int kBBytesT = (BN / 2) * kBK * 2;  // one CTA's weight rows of a K step
  static constexpr int kOffA_ = 0;
  static constexpr int kOffB_ = WF16 ? kStages * kABytes : kOffB;
  static constexpr int kOffOut_ = WF16 ? kOffB_ + kStages * kBBytesT : kOffOut;
  static constexpr int kOffBar_ = kOffOut_ + 4 * kNOut * kOutBytes;
  static constexpr int kSmem_ = 1024 + kOffBar_ + 512;
  static_assert(kSmem_ <= 232448, "dynamic shared memory per block");
};
constexpr int kEpiWarps = 4;  // one per TMEM lane quarter
constexpr int kThreads = 64 + 256 + 32 * kEpiWarps;
constexpr int kDequantWarps = 8;
constexpr uint32_t kTmemCols = 512;  // two 256-column accumulators

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t num_clusters() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// shared::cluster address of the same-offset object in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on a barrier given by its shared::cluster address (default .release
// semantics; the arriving thread has already fenced its smem writes to the
// async proxy, which is what the consuming tcgen05.mma reads through).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait (cluster-scope acquire) for barriers other CTAs arrive on.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, uint32_t* status) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((it & 255u) == 255u && global_timer_ns() - t0 > kWaitLimitNs) {
      if (status) atomicOr(status, kStatusWaitTimeout);
      return false;
    }
  }
}
// 2-D TMA load into this CTA's smem whose completion is counted on the
// barrier at cluster address `bar_cluster` (the even CTA's barrier).
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_mma_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the same-offset barrier of both CTAs when this thread's
// previously issued MMAs complete.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 8 weights from the nibbles in the bytes of x0, x1 (0..15 each):
// d1*q - m1 exactly as the reference (see q4k.cuh), then f16.
__device__ __forceinline__ uint4 dequant8_f16(uint32_t x0, uint32_t x1, uint64_t d1, uint64_t negm1) {
  const uint64_t kNeg223 = f2(-8388608.0f, -8388608.0f);
  uint32_t o[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint32_t x = p < 2 ? x0 : x1;
    const uint32_t b = (p & 1) * 2;
    const uint64_t magic = (static_cast<uint64_t>(__byte_perm(x, 0x4B000000u, 0x7440u | (b + 1))) << 32) |
                           __byte_perm(x, 0x4B000000u, 0x7440u | b);
    const uint64_t q = f2_add(magic, kNeg223);
    o[p] = f2_to_h2(f2_fma(d1, q, negm1));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Optional wait accounting for pipeline analysis (off in the library build):
// per CTA, cycles the MMA thread waited for accumulators / operand stages and
// its loop total, the producer's waits for free stages, the first epilogue
// warp's waits for accumulators, and the global timer at entry and exit.
#ifdef WC_GEMM_TRACE
__device__ unsigned long long g_gemm_trace[512][8];
#define GT_NOW() static_cast<unsigned long long>(clock64())
#endif

// BN: output columns per cluster tile, 256 or (f16 weights only) 128; each
// CTA holds BN / 2 weight rows of a tile.
template <int EPI, bool WF16, int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm2_q4k_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW0,
                     const __grid_constant__ CUtensorMap tmW1, const __grid_constant__ CUtensorMap tmOut,
                     GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  static_assert(BN == 256 || (BN == 128 && WF16 && EPI != kEpiGeGLU), "128-column tiles: f16 weights only");
  using PL = Plan<EPI, WF16, BN>;
  constexpr int kHalfNT = BN / 2;
  constexpr int kBBytesT = PL::kBBytesT;
  constexpr int SA = PL::kStages;  // X (and f16 B) ring depth
  uint8_t* sA = smem + PL::kOffA_;
  uint8_t* sW = smem + kOffW;
  uint8_t* sB = smem + PL::kOffB_;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + PL::kOffBar_);
  uint64_t* full_a = bars;                 // [SA]   even CTA: X bytes of both CTAs
  uint64_t* empty_a = full_a + SA;         // [SA]   each CTA: MMA done with the stage
  uint64_t* full_w = empty_a + SA;         // [kSW]  local raw Q4_K landed
  uint64_t* empty_w = full_w + kSW;        // [kSW]  local dequant warps done with it
  uint64_t* full_b = empty_w + kSW;        // [kSB]  even CTA: the owning warp pair of both CTAs
  uint64_t* empty_b = full_b + kSB;        // [kSB]  each CTA: MMA done with the stage
  uint64_t* acc_full = empty_b + kSB;      // [2]    each CTA: accumulator ready
  uint64_t* acc_empty = acc_full + 2;      // [2]    even CTA: 16 epilogue warps drained it
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
#ifdef WC_GEMM_TRACE
  if (threadIdx.x == 0) g_gemm_trace[blockIdx.x][5] = global_timer_ns();
#endif
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int ksteps = p.K / kBK;
  const int kblocks = p.K / 256;
  const int m_tiles = (p.M + kBM - 1) / kBM;
  const int n_tiles = p.N / BN;
  const int n_total = m_tiles * n_tiles;
  const int cid = static_cast<int>(cluster_id());
  const int ncl = static_cast<int>(num_clusters());

  if (threadIdx.x == 0) {
    for (int i = 0; i < SA; ++i) {
      mbar_init(&full_a[i], 1);
      mbar_init(&empty_a[i], 1);
    }
    for (int i = 0; i < kSW; ++i) {
      mbar_init(&full_w[i], 1);
      mbar_init(&empty_w[i], kDequantWarps);
    }
    for (int i = 0; i < kSB; ++i) {
      mbar_init(&full_b[i], 4);  // 2 warps of the owning pair x 2 CTAs
      mbar_init(&empty_b[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 2 * kEpiWarps);
    }
    mbar_fence_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW0);
    tma_prefetch_desc(&tmW1);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // every role touches activations only after this
  pdl_launch_next();  // after the wait: at most one grid waits ahead

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const CUtensorMap* wmap = (EPI == kEpiGeGLU && rank == 1) ? &tmW1 : &tmW0;
      uint32_t ia = 0, iw = 0;
      bool ok = true;
      for (int tile = cid; tile < n_total && ok; tile += ncl) {
        const int m0 = (tile / n_tiles) * kBM + static_cast<int>(rank) * 128;
        const int nt = tile % n_tiles;
        const int w_row0 = EPI == kEpiGeGLU ? nt * kHalfN : nt * BN + static_cast<int>(rank) * kHalfNT;
        for (int t = 0; t < ksteps; ++t) {
          if (!WF16 && (t & 3) == 0) {
            const uint32_t sw = iw % kSW;
            if (!(ok = mbar_wait(&empty_w[sw], ((iw / kSW) & 1) ^ 1, p.status))) break;
            mbar_arrive_expect_tx(&full_w[sw], kWBytes);
            tma_load_2d(sW + sw * kWBytes, wmap, &full_w[sw], (t >> 2) * 144, w_row0);
            ++iw;
          }
          const uint32_t sa = ia % SA;
#ifdef WC_GEMM_TRACE
          const unsigned long long w0_ = GT_NOW();
#endif
          if (!(ok = mbar_wait(&empty_a[sa], ((ia / SA) & 1) ^ 1, p.status))) break;
#ifdef WC_GEMM_TRACE
          g_gemm_trace[blockIdx.x][4] += GT_NOW() - w0_;
#endif
          if (leader) mbar_arrive_expect_tx(&full_a[sa], WF16 ? 2 * (kABytes + kBBytesT) : 2 * kABytes);
          tma_load_2d_pair(sA + sa * kABytes, &tmA, map_to_rank(&full_a[sa], 0), t * kBK, m0);
          if (WF16)  // B stage sa holds this CTA's weight rows of the same K step
            tma_load_2d_pair(sB + sa * kBBytesT, wmap, map_to_rank(&full_a[sa], 0), t * kBK, w_row0);
          ++ia;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(kBM, BN);
      uint32_t ia = 0, ib = 0, it = 0;
      bool ok = true;
#ifdef WC_GEMM_TRACE
      const unsigned long long t0_ = GT_NOW();
      unsigned long long wacc_ = 0, wfull_ = 0, nk_ = 0;
#endif
      for (int tile = cid; tile < n_total && ok; tile += ncl, ++it) {
        const uint32_t buf = it & 1;
#ifdef WC_GEMM_TRACE
        const unsigned long long w0_ = GT_NOW();
#endif
        if (!(ok = mbar_wait_cluster(&acc_empty[buf], ((it >> 1) & 1) ^ 1, p.status))) break;
#ifdef WC_GEMM_TRACE
        wacc_ += GT_NOW() - w0_;
#endif
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int t = 0; t < ksteps; ++t, ++ia, ++ib) {
          const uint32_t sa = ia % SA, sb = ib % kSB;
#ifdef WC_GEMM_TRACE
          const unsigned long long w1_ = GT_NOW();
#endif
          ok = mbar_wait_cluster(&full_a[sa], (ia / SA) & 1, p.status) &&
               (WF16 || mbar_wait_cluster(&full_b[sb], (ib / kSB) & 1, p.status));
          if (!ok) break;
#ifdef WC_GEMM_TRACE
          wfull_ += GT_NOW() - w1_;
          ++nk_;
#endif
          tc_fence_after();
          const uint64_t adesc = sw128_kmajor_desc(smem_u32(sA + sa * kABytes));
          const uint64_t bdesc = sw128_kmajor_desc(smem_u32(sB + (WF16 ? sa * kBBytesT : sb * kBBytes)));
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            tc_mma_pair(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (t > 0 || k > 0) ? 1u : 0u);
          tc_commit_pair(&empty_a[sa]);
          if (!WF16) tc_commit_pair(&empty_b[sb]);
        }
        if (ok) tc_commit_pair(&acc_full[buf]);
      }
#ifdef WC_GEMM_TRACE
      g_gemm_trace[blockIdx.x][0] = wacc_;
      g_gemm_trace[blockIdx.x][1] = wfull_;
      g_gemm_trace[blockIdx.x][2] = GT_NOW() - t0_;
      g_gemm_trace[blockIdx.x][3] = nk_;
#endif
    }
  } else if (warp < 2 + kDequantWarps) {
    if (WF16) {
      // no dequant work: the weights arrive by TMA
    } else {
    // ------------------------------------------------------------ dequant
    // The 4 B stages rotate over 4 pairs of warps: pair g dequantises every
    // K step with (step % 4) == g, i.e. the 64-wide slice g of each Q4_K
    // super-block, for all 128 weight rows of this CTA.  While one pair
    // fences and signals its stage the other pairs keep converting.
    static_assert(kSB == 4, "one B stage per dequant warp pair");
    const int g = (warp - 2) >> 1;        // 0..3: slice of the super-block
    const int gt = threadIdx.x - 64 - 64 * g;  // 0..63 within the pair
    const uint32_t full_b_leader = map_to_rank(&full_b[g], 0);
    uint8_t* bt = sB + g * kBBytes;
    uint32_t iw = 0;
    bool ok = true;
    for (int tile = cid; tile < n_total && ok; tile += ncl) {
      for (int kb = 0; kb < kblocks && ok; ++kb, ++iw) {
        const uint32_t sw = iw % kSW;
        if (!(ok = mbar_wait(&full_w[sw], (iw / kSW) & 1, p.status))) break;
        if (!(ok = mbar_wait(&empty_b[g], (iw & 1) ^ 1, p.status))) break;
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          const int r = gt + 64 * rr;
          const uint8_t* blk = sW + sw * kWBytes + r * 144;
          const Q4KScales sc = q4k_load_scales(blk);
          const uint4* qp = reinterpret_cast<const uint4*>(blk + 16 + 32 * g);
          const uint4 q0 = qp[0], q1 = qp[1];
          const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
          for (int hs = 0; hs < 2; ++hs) {
            float d1f, m1f;
            q4k_sub_scale(sc, 2 * g + hs, d1f, m1f);
            const uint64_t d1 = f2(d1f, d1f), negm1 = f2(-m1f, -m1f);
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
              const uint32_t x0 = (qw[2 * cc] >> (4 * hs)) & 0x0F0F0F0Fu;
              const uint32_t x1 = (qw[2 * cc + 1] >> (4 * hs)) & 0x0F0F0F0Fu;
              *reinterpret_cast<uint4*>(bt + sw128_offset(r, hs * 4 + cc)) = dequant8_f16(x0, x1, d1, negm1);
            }
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&empty_w[sw]);
          mbar_arrive_remote(full_b_leader);
        }
      }
    }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    constexpr int NOUT = PL::kNOut;
    uint8_t* sOutW = smem + PL::kOffOut_ + (warp - 10) * NOUT * kOutBytes;
    uint32_t ostage = 0;
    const uint32_t acc_empty_leader0 = map_to_rank(&acc_empty[0], 0);
    uint32_t it = 0;
    bool clip = false;  // an f16 output value was clipped
    for (int tile = cid; tile < n_total; tile += ncl, ++it) {
      const uint32_t buf = it & 1;
#ifdef WC_GEMM_TRACE
      const unsigned long long w0_ = GT_NOW();
#endif
      const bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(&acc_full[buf], (it >> 1) & 1, p.status));
      if (!ok) break;
#ifdef WC_GEMM_TRACE
      if (warp == 10 && lane == 0) g_gemm_trace[blockIdx.x][6] += GT_NOW() - w0_;
#endif
      tc_fence_after();
      const int nt = tile % n_tiles;
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * BN;
      {
        // Each 128-byte-wide chunk of this warp's 32 rows is converted into
        // a swizzled staging buffer and written by one TMA tensor store
        // (rows past M are clipped by the tensor map), so global writes are
        // whole lines instead of one 16-byte piece per row per instruction.
        // kEpiResid (x += acc) stages the f32 accumulator the same way and
        // issues a TMA reduce-add instead of the store: L2 adds it into x,
        // one add per element, so nothing is loaded first.
        constexpr bool kF32Out = EPI == kEpiF32 || EPI == kEpiResid;
        constexpr int kCW = kF32Out ? 32 : 64;                // output columns per chunk
        constexpr int kOutCols = EPI == kEpiGeGLU ? kHalfN : BN;
        const int col_base = nt * kOutCols;
        const int y0 = (tile / n_tiles) * kBM + static_cast<int>(rank) * 128 + q * 32;
#pragma unroll 1
        for (int c = 0; c < kOutCols; c += kCW, ++ostage) {
          uint8_t* sbuf = sOutW + (ostage % NOUT) * kOutBytes;
          if (lane == 0) asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(NOUT - 1) : "memory");
          __syncwarp();
          uint8_t* srow = sbuf + lane * 128;
          if (kF32Out) {
            float v[32];
            tmem_ld_32x32b_x32(tb + c, v);
#pragma unroll
            for (int k = 0; k < 8; ++k)
              *reinterpret_cast<float4*>(srow + ((k ^ (lane & 7)) << 4)) =
                  make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
          } else {
#pragma unroll
            for (int hc = 0; hc < 2; ++hc) {  // two 32-column halves of the 64-column chunk
              float v[32];
              tmem_ld_32x32b_x32(tb + c + 32 * hc, v);
              if (EPI == kEpiGeGLU) {
                float u[32];
                tmem_ld_32x32b_x32(tb + kHalfN + c + 32 * hc, u);
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = gelu_tanh_fast(v[i]) * u[i];
              }
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                uint4 o;
                o.x = pack_f16x2_sat(v[8 * k], v[8 * k + 1], clip);
                o.y = pack_f16x2_sat(v[8 * k + 2], v[8 * k + 3], clip);
                o.z = pack_f16x2_sat(v[8 * k + 4], v[8 * k + 5], clip);
                o.w = pack_f16x2_sat(v[8 * k + 6], v[8 * k + 7], clip);
                *reinterpret_cast<uint4*>(srow + (((4 * hc + k) ^ (lane & 7)) << 4)) = o;
              }
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (EPI == kEpiResid)
              asm volatile(
                  "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                      reinterpret_cast<uint64_t>(&tmOut)),
                  "r"(smem_u32(sbuf)), "r"(col_base + c), "r"(y0)
                  : "memory");
            else
              asm volatile(
                  "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                      reinterpret_cast<uint64_t>(&tmOut)),
                  "r"(smem_u32(sbuf)), "r"(col_base + c), "r"(y0)
                  : "memory");
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(acc_empty_leader0 + buf * 8);
    }
    report_f16_clip(clip, p.status);
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  }

  // ------------------------------------------------------------ teardown
  __syncwarp();
  tc_fence_before();
  cluster_sync();
#ifdef WC_GEMM_TRACE
  if (threadIdx.x == 0) g_gemm_trace[blockIdx.x][7] = global_timer_ns();
#endif
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

template <int EPI, bool WF16, int BN = kBN>
cudaError_t launch(const CUtensorMap& a, const CUtensorMap& w0, const CUtensorMap& w1, const CUtensorMap& out,
                   const GemmParams& p, int num_sms, cudaStream_t st) {
  constexpr int smem_bytes = Plan<EPI, WF16, BN>::kSmem_;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(gemm2_q4k_kernel<EPI, WF16, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const int tiles = ((p.M + kBM - 1) / kBM) * (p.N / BN);
  const int clusters = std::max(1, std::min(tiles, num_sms / 2));
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  return launch_pdl(gemm2_q4k_kernel<EPI, WF16, BN>, dim3(2 * clusters), dim3(kThreads), smem_bytes, st, attr, 1, a, w0, w1, out, p);
}

}  // namespace

#ifdef WC_GEMM_TRACE
extern "C" int wc_gemm_trace(unsigned long long* host, int reset) {
  if (reset) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_gemm_trace);
    if (e == cudaSuccess) e = cudaMemset(p, 0, sizeof(g_gemm_trace));
    return static_cast<int>(e);
  }
  return static_cast<int>(cudaMemcpyFromSymbol(host, g_gemm_trace, sizeof(g_gemm_trace)));
}
#endif

int gemm2_resid_bn(int M, int N, int num_sms) {
  // WC_RESID_BN=128 / 256 forces the width (A/B runs)
  static const int forced = [] {
    const char* e = std::getenv("WC_RESID_BN");
    return e ? std::atoi(e) : 0;
  }();
  if ((forced == 128 && N % 128 == 0) || (forced == 256 && N % kBN == 0)) return forced;
  if (N % kBN != 0) return 128;
  const int64_t clusters = std::max(1, num_sms / 2);
  const int64_t t128 = static_cast<int64_t>((M + kBM - 1) / kBM) * (N / 128);
  return t128 <= clusters ? 128 : kBN;
}

bool gemm2_q4k_supports(int epi, int M, int N, int K) {
  return (epi == kEpiF16 || epi == kEpiGeGLU || epi == kEpiResid || epi == kEpiF32) && M >= 1 && N % kBN == 0 &&
         K % 256 == 0 && K >= 256;
}

cudaError_t gemm2_q4k_launch(int epi, const CUtensorMap& a, const CUtensorMap& w0, const CUtensorMap& w1,
                             const CUtensorMap& out, const GemmParams& p, int num_sms, cudaStream_t st, bool w_f16,
                             int bn) {
  if (bn == 128) {
    if (!w_f16 || p.N % 128) return cudaErrorInvalidValue;
    if (epi == kEpiResid) return launch<kEpiResid, true, 128>(a, w0, w1, out, p, num_sms, st);
    if (epi == kEpiF32) return launch<kEpiF32, true, 128>(a, w0, w1, out, p, num_sms, st);
    return cudaErrorInvalidValue;
  }
  if (bn != kBN) return cudaErrorInvalidValue;
  if (w_f16) {
    switch (epi) {
      case kEpiF16: return launch<kEpiF16, true>(a, w0, w1, out, p, num_sms, st);
      case kEpiGeGLU: return launch<kEpiGeGLU, true>(a, w0, w1, out, p, num_sms, st);
      case kEpiResid: return launch<kEpiResid, true>(a, w0, w1, out, p, num_sms, st);
      case kEpiF32: return launch<kEpiF32, true>(a, w0, w1, out, p, num_sms, st);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (epi) {
    case kEpiF16: return launch<kEpiF16, false>(a, w0, w1, out, p, num_sms, st);
    case kEpiGeGLU: return launch<kEpiGeGLU, false>(a, w0, w1, out, p, num_sms, st);
    case kEpiResid: return launch<kEpiResid, false>(a, w0, w1, out, p, num_sms, st);
    case kEpiF32: return launch<kEpiF32, false>(a, w0, w1, out, p, num_sms, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace wc
