// Bidirectional T5 encoder self-attention on the 5th-generation tensor cores
// (tcgen05 + TMEM), flash-style with an online softmax, the T5 relative-
// position bias and a key padding mask.  Replaces src/quantized_t5.rs:426-500:
// scores without 1/sqrt(d) scaling, + position bias, softmax_last_dim, P.V,
// transpose back to tokens.
//
// One CTA owns 128 queries of one sequence for a group of heads and walks the
// flattened sequence of steps (head, 64-key tile) as one pipeline, so the
// TMA loads and S MMAs of the next step -- also across a head boundary --
// overlap the softmax of the current one:
//   warp 0      TMA: the Q tile of each head (one shared-memory buffer),
//               its K and V tiles (two 3-stage rings; a K stage is freed as
//               soon as its S is done)
//   warp 1      TMEM allocation and the single MMA-issuing thread
//   warps 2-5   Q staging, softmax and epilogue (thread = query row = TMEM lane)
// Shared-memory bandwidth bounds this kernel at d = 64, so both A operands
// live in tensor memory: the softmax warps copy each head's Q tile into one
// of two TMEM Q buffers (one head ahead), and write P as f16 over the S
// buffer it came from.  Step t (head h, key tile j): S(t) = Q_h K_j^T (M=128,
// N=64, K=64, A from TMEM, f32 in TMEM buffer t % 2, computed ahead); the
// softmax warps add the relative-position bias (a per-tile window of 191
// biases they build), mask keys past the sequence, update the running max /
// sum, rescale the O row in TMEM when the max moved and store P = 2^(S - max)
// into the first 32 columns of S buffer t % 2; then O += P V_j (M=128, N=64,
// K=64, A = P from TMEM, V read MN-major from its TMA tile).  S(t + 2) reuses
// that buffer only after P(t) V(t), in MMA issue order.  One O buffer
// suffices: the same warps read it out before they release the next P.
// Input: the token-major QKV projection [B*L][3*H*64] f16 through one TMA
// descriptor (box 64 x 64); output [B*L][H*64] f16.  Query rows of an
// all-padding tile are written as zeros.
#include "attention.h"
#include "common.cuh"

#include <algorithm>

namespace wc {

namespace {

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 columns of raw 32-bit words; returns once the store is done.
__device__ __forceinline__ void tmem_st_u32_x32(uint32_t taddr, const uint32_t (&v)[32]) {
  tmem_st_32x32b_x32(taddr, reinterpret_cast<const float(&)[32]>(v));
}

// 32 lanes x 32 columns without waiting; tmem_wait_ld() completes them.
__device__ __forceinline__ void tmem_ld_32x32b_x32_nowait(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Shared-memory descriptor of an MN-major operand with the 128-byte swizzle:
// rows of 64 f16 along N (128 B) for consecutive K, 8-row groups 1024 B apart
// (stride byte offset); the leading byte offset (stride between 64-wide N
// atoms) is unused for N = 64.
__device__ __forceinline__ uint64_t sw128_mnmajor_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(8192u >> 4) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Bucket of key - query = delta from the monotone thresholds in shared
// memory (thr[v] = smallest distance in bucket >= v): a binary search for
// the largest v < half with thr[v] <= |delta|.
__device__ __forceinline__ int rel_bucket_tc(const int* thr, int half, int delta) {
  const int d = delta < 0 ? -delta : delta;
  int f = 0;
#pragma unroll
  for (int step = 16; step > 0; step >>= 1)
    if (f + step < half && thr[f + step] <= d) f += step;
  return f + (delta > 0 ? half : 0);
}


#ifdef WC_ATTN_TRACE
// Development instrumentation: per-CTA clock64 stamps of softmax thread 0.
constexpr int kTraceCtas = 8192, kTraceSlots = 12;
__device__ unsigned long long g_attn_trace[kTraceCtas][kTraceSlots];
#define ATTN_TRACE(slot, val) \
  if (threadIdx.x == 64 && trace_id < kTraceCtas) g_attn_trace[trace_id][slot] = (val)
#define ATTN_TRACE_ADD(slot, val) tr_acc[slot] += (val)
#else
#define ATTN_TRACE(slot, val)
#define ATTN_TRACE_ADD(slot, val)
#endif

constexpr int kQ = 128;       // queries per CTA
constexpr int kKeys = 64;     // keys per tile
constexpr int kDh = 64;
constexpr int kQBytes = kQ * 128;      // 128 x 64 f16
constexpr int kKVBytes = kKeys * 128;  // 64 x 64 f16
constexpr int kWin = kQ + kKeys - 1;   // distinct key - query offsets of one tile pair
constexpr int kMaxHeads = 16;          // heads of one CTA's group
constexpr int kKVStages = 3;
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kQBytes;                // kKVStages stages
constexpr int kOffV = kOffK + kKVStages * kKVBytes;   // kKVStages stages
// Bias window of one step in two copies, the second shifted by one entry, so
// that every thread reads its biases as 8-byte aligned pairs.
constexpr int kWinPad = kWin + 1;
constexpr int kOffWin = kOffV + kKVStages * kKVBytes;  // f32 [2 steps][2 copies][kWinPad]
constexpr int kOffTab = kOffWin + 2 * 2 * kWinPad * 4;  // f32 [kMaxHeads][64]
constexpr int kMaxL = 2048;
constexpr int kOffThr = kOffTab + kMaxHeads * 64 * 4;  // int [32]
// u8 bucket of key - query = x - q0 - (kQ - 1) at index x
constexpr int kOffBkt = kOffThr + 32 * 4;
constexpr int kOffBar = kOffBkt + ((kMaxL + kWin + 127) / 128) * 128;
constexpr int kSmem = 1024 + kOffBar + 256;
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 256;
// S (and P) buffers at 0 / 64, O at 128, Q buffers at 192 / 224
constexpr uint32_t kColS = 0, kColO = 128, kColQ = 192;

__global__ void __launch_bounds__(kThreads)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQKV, __half* __restrict__ out,
                        const int32_t* __restrict__ lengths, int L, int H, int heads_per_cta,
                        const float* __restrict__ bias_tab, BucketThresholds bt, uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + kOffQ;
  uint8_t* sK = smem + kOffK;
  uint8_t* sV = smem + kOffV;
  float* sWin = reinterpret_cast<float*>(smem + kOffWin);
  float* sTab = reinterpret_cast<float*>(smem + kOffTab);  // [head in group][bucket] * log2(e)
  uint8_t* sBkt = smem + kOffBkt;
  int* sThr = reinterpret_cast<int*>(smem + kOffThr);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars;          // [1]
  uint64_t* q_empty = bars + 1;     // [1] (4 softmax warps arrive once Q is in TMEM)
  uint64_t* k_full = bars + 2;      // [kKVStages]
  uint64_t* k_empty = bars + 5;     // [kKVStages]  freed when S(t) is done
  uint64_t* v_full = bars + 8;      // [kKVStages]
  uint64_t* v_empty = bars + 11;    // [kKVStages]  freed when P(t) V(t) is done
  uint64_t* s_full = bars + 14;     // [2] per S buffer
  uint64_t* p_full = bars + 16;     // [1] (4 softmax warps arrive)
  uint64_t* o_done = bars + 17;     // [1] one phase per step
  uint64_t* q_tm = bars + 18;       // [2] per TMEM Q buffer (4 softmax warps arrive)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 20);

#ifdef WC_ATTN_TRACE
  const int trace_id = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  const unsigned long long tr0 = clock64();
  unsigned long long tr_acc[kTraceSlots] = {};
  if (threadIdx.x == 64 && trace_id < kTraceCtas)
    for (int i = 0; i < kTraceSlots; ++i) g_attn_trace[trace_id][i] = 0;
  ATTN_TRACE(0, tr0);
  {
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    ATTN_TRACE(8, smid);
  }
#endif
  pdl_wait();  // before lengths and any activation (see pdl_wait)
  pdl_launch_next();  // after the wait: at most one grid waits ahead
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z;
  const int h0 = blockIdx.y * heads_per_cta;
  const int nh = min(heads_per_cta, H - h0);
  const int q0 = blockIdx.x * kQ;
  const int len = min(lengths[b], L);
  const int inner = H * kDh;
  const size_t row0 = static_cast<size_t>(b) * L;
  const int n_kt = (len + kKeys - 1) / kKeys;
  const int n_steps = nh * n_kt;

  if (q0 >= len || nh <= 0) {
    // every query row of this CTA is padding: zero output rows, no MMA work
    for (int i = threadIdx.x; i < kQ * nh * (kDh / 8); i += blockDim.x) {
      const int r = i / (nh * 8), rest = i % (nh * 8), hh = rest >> 3, c = rest & 7;
      if (q0 + r < L)
        *reinterpret_cast<uint4*>(out + (row0 + q0 + r) * inner + (h0 + hh) * kDh + c * 8) = make_uint4(0, 0, 0, 0);
    }
    return;
  }

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 4);
    for (int i = 0; i < kKVStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&q_tm[i], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(o_done, 1);
    mbar_fence_init();
    tma_prefetch_desc(&tmQKV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (threadIdx.x < 32) sThr[threadIdx.x] = bt.thr[threadIdx.x];
  __syncthreads();
  // bucket of every key - query offset this CTA meets, once
  for (int x = threadIdx.x; x < n_kt * kKeys + kWin; x += blockDim.x)
    sBkt[x] = static_cast<uint8_t>(rel_bucket_tc(sThr, bt.half, x - q0 - (kQ - 1)));
  for (int i = threadIdx.x; i < nh * 2 * bt.half; i += blockDim.x) {
    const int hh = i / (2 * bt.half), bk = i % (2 * bt.half);
    sTab[hh * 64 + bk] = bias_tab[bk * H + h0 + hh] * 1.4426950408889634f;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  ATTN_TRACE(1, clock64());
  ATTN_TRACE(7, n_steps);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      // Q of head hq (single buffer, free once the previous head's Q is in TMEM)
      auto load_q = [&](int hq) -> bool {
        if (!mbar_wait(q_empty, (hq & 1) ^ 1, status)) return false;
        mbar_arrive_expect_tx(q_full, kQBytes);
        tma_load_2d(sQ, &tmQKV, q_full, (h0 + hq) * kDh, static_cast<int>(row0) + q0);  // box: 64 rows
        tma_load_2d(sQ + kQBytes / 2, &tmQKV, q_full, (h0 + hq) * kDh, static_cast<int>(row0) + q0 + 64);
        return true;
      };
      bool ok = load_q(0);
      for (int t = 0; t < n_steps && ok; ++t) {
        const int hh = t / n_kt, j = t % n_kt, h = h0 + hh;
        if (j == 0 && hh + 1 < nh && !(ok = load_q(hh + 1))) break;
        const int s = t % kKVStages;
        const uint32_t par = ((t / kKVStages) & 1) ^ 1;
        if (!(ok = mbar_wait(&k_empty[s], par, status))) break;
        mbar_arrive_expect_tx(&k_full[s], kKVBytes);
        tma_load_2d(sK + s * kKVBytes, &tmQKV, &k_full[s], inner + h * kDh, static_cast<int>(row0) + j * kKeys);
        if (!(ok = mbar_wait(&v_empty[s], par, status))) break;
        mbar_arrive_expect_tx(&v_full[s], kKVBytes);
        tma_load_2d(sV + s * kKVBytes, &tmQKV, &v_full[s], 2 * inner + h * kDh, static_cast<int>(row0) + j * kKeys);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_f16_f32(kQ, kKeys);
      constexpr uint32_t idesc_pv = idesc_f16_f32(kQ, kDh) | (1u << 16);  // B (V) MN-major
      bool ok = true;
      // S(t) = Q_h K_j^T into S buffer t % 2 (needs its Q and K/V stage)
      auto issue_s = [&](int t) -> bool {
        const int hh = t / n_kt, j = t % n_kt, s = t % kKVStages;
        if (j == 0 && !mbar_wait(&q_tm[hh & 1], (hh >> 1) & 1, status)) return false;
        if (!mbar_wait(&k_full[s], (t / kKVStages) & 1, status)) return false;
        tc_fence_after();
        const uint32_t qa = tmem + kColQ + 32 * (hh & 1);
        const uint64_t bk = sw128_kmajor_desc(smem_u32(sK + s * kKVBytes));
#pragma unroll
        for (int k = 0; k < kDh / 16; ++k)
          tc_mma_f16_ts(tmem + kColS + 64 * (t & 1), qa + 8 * k, bk + 2 * k, idesc_qk, k > 0);
        tc_commit(&s_full[t & 1]);
        tc_commit(&k_empty[s]);
        return true;
      };
      for (int t = 0; t < 2 && t < n_steps && ok; ++t) ok = issue_s(t);
      for (int t = 0; t < n_steps && ok; ++t) {
        const int j = t % n_kt, s = t % kKVStages;
        // P(t) also means the epilogue of the previous head has read O
        if (!(ok = mbar_wait(p_full, t & 1, status))) break;
        if (!(ok = mbar_wait(&v_full[s], (t / kKVStages) & 1, status))) break;
        tc_fence_after();
        const uint64_t v = sw128_mnmajor_desc(smem_u32(sV + s * kKVBytes));
        const uint32_t pa = tmem + kColS + 64 * (t & 1);
#pragma unroll
        for (int k = 0; k < kKeys / 16; ++k)
          tc_mma_f16_ts(tmem + kColO, pa + 8 * k, v + 128 * k, idesc_pv, (j > 0 || k > 0) ? 1u : 0u);
        tc_commit(o_done);
        tc_commit(&v_empty[s]);
        if (t + 2 < n_steps) ok = issue_s(t + 2);  // S buffer t % 2 is free again
      }
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int st = threadIdx.x - 64;  // 0..127
    const int qd = warp & 3;          // TMEM lane quarter
    const int r = qd * 32 + lane;     // query row within the tile
    const int qi = q0 + r;
    const uint32_t trow = tmem + (static_cast<uint32_t>(qd * 32) << 16);
    float m_run = -INFINITY, l_run = 0.f;
    // Q of head hq: shared memory (TMA, 128-B swizzle) -> this thread's row
    // of TMEM Q buffer hq % 2, then release the shared buffer.
    auto stage_q = [&](int hq) -> bool {
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(q_full, hq & 1, status))) return false;
      uint32_t qr[32];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 w = *reinterpret_cast<const uint4*>(sQ + sw128_offset(r, c));
        qr[4 * c] = w.x;
        qr[4 * c + 1] = w.y;
        qr[4 * c + 2] = w.z;
        qr[4 * c + 3] = w.w;
      }
      tmem_st_u32_x32(trow + kColQ + 32 * (hq & 1), qr);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(q_empty);
        mbar_arrive(&q_tm[hq & 1]);
      }
      return true;
    };
    bool ok = stage_q(0);
    // Every step passes the named barrier, even after a failed wait, so a
    // timed-out warp can never strand the other softmax warps there.
    for (int t = 0; t < n_steps; ++t) {
      const int hh = t / n_kt, j = t % n_kt;
      const int k0 = j * kKeys;
      if (j == 0) {
        m_run = -INFINITY;
        l_run = 0.f;
        // one head ahead: Q buffer (hh + 1) % 2 last served head hh - 1,
        // whose S tiles this thread has all consumed
        if (ok && hh + 1 < nh) ok = stage_q(hh + 1);
      }
      // bias window of this step: win[e] for key - query = k0 - q0 - (kQ - 1) + e
      // and win1[e] = win[e + 1]
      float* win = sWin + (t & 1) * 2 * kWinPad;
      float* win1 = win + kWinPad;
      const float* tab = sTab + hh * 64;
#ifdef WC_ATTN_TRACE
      const unsigned long long ta = clock64();
#endif
      for (int e = st; e < kWin; e += 128) {
        const float w = tab[sBkt[k0 + e]];
        win[e] = w;
        if (e > 0) win1[e - 1] = w;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      // bias of key k0 + c at brow[c], brow 8-byte aligned
      const float* brow = ((kQ - 1 - r) & 1) ? win1 + (kQ - 2 - r) : win + (kQ - 1 - r);
#ifdef WC_ATTN_TRACE
      const unsigned long long tb = clock64();
      ATTN_TRACE_ADD(5, tb - ta);
#endif
      if (ok) ok = __all_sync(0xFFFFFFFFu, mbar_wait(&s_full[t & 1], (t >> 1) & 1, status));
#ifdef WC_ATTN_TRACE
      const unsigned long long tc = clock64();
      ATTN_TRACE_ADD(4, tc - tb);
      if (t == 0) ATTN_TRACE(2, tc);
#endif
      if (ok) {
        tc_fence_after();
        float v[kKeys];
        tmem_ld_32x32b_x32_nowait(trow + kColS + 64 * (t & 1), &v[0]);
        tmem_ld_32x32b_x32_nowait(trow + kColS + 64 * (t & 1) + 32, &v[32]);
        tmem_wait_ld();
        // v = S log2(e) + bias, two lanes per instruction; 4 max chains
        const uint64_t kLog2e2 = f2(1.4426950408889634f, 1.4426950408889634f);
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int i = 0; i < kKeys; i += 2) {
          const float2 bb = *reinterpret_cast<const float2*>(brow + i);
          const uint64_t x = f2_fma(f2(v[i], v[i + 1]), kLog2e2, f2(bb.x, bb.y));
          v[i] = f2_lo(x);
          v[i + 1] = f2_hi(x);
        }
        if (k0 + kKeys > len) {
#pragma unroll
          for (int i = 0; i < kKeys; ++i)
            if (k0 + i >= len) v[i] = -INFINITY;
        }
#pragma unroll
        for (int i = 0; i < kKeys; i += 2) mx[(i >> 1) & 3] = fmax3(mx[(i >> 1) & 3], v[i], v[i + 1]);
        const float tmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
        // Lazy rescale: keep the running max unless this tile raises it by
        // more than 8 (log2 units), so P stays <= 2^8 and O is rescaled
        // rarely; the final division by the matching sum makes it exact.
        const float m_new = (tmax > m_run + 8.0f) ? tmax : m_run;
        const float corr = ex2(m_run - m_new);  // 1 when kept, 0 on the head's first tile
        // p = 2^(t - max) -> f16 P row over the first 32 columns of S buffer
        // t % 2 (S(t) is in registers), row sum in f32
        const uint64_t negm = f2(-m_new, -m_new);
        uint64_t ps[4] = {0, 0, 0, 0};  // (+0, +0) pairs
        uint32_t pk[kKeys / 2];
#pragma unroll
        for (int i = 0; i < kKeys; i += 2) {
          const uint64_t x = f2_add(f2(v[i], v[i + 1]), negm);
          const uint64_t p = f2(ex2(f2_lo(x)), ex2(f2_hi(x)));
          ps[(i >> 1) & 3] = f2_add(ps[(i >> 1) & 3], p);
          pk[i >> 1] = f2_to_h2(p);
        }
        tmem_st_u32_x32(trow + kColS + 64 * (t & 1), pk);
        const uint64_t ps2 = f2_add(f2_add(ps[0], ps[1]), f2_add(ps[2], ps[3]));
        const float psum = f2_lo(ps2) + f2_hi(ps2);
        l_run = l_run * corr + psum;
        m_run = m_new;
        if (j > 0 && __any_sync(0xFFFFFFFFu, corr != 1.0f)) {
          // O holds P(t-1) V(t-1) of this head once o_done says so; rescale it
          // to the new max (rare with the lazy rule above)
          ok = __all_sync(0xFFFFFFFFu, mbar_wait(o_done, (t - 1) & 1, status));
          if (ok) {
            tc_fence_after();
            const uint32_t ocol = trow + kColO;
#pragma unroll 1
            for (int c = 0; c < kDh; c += 32) {
              float o[32];
              tmem_ld_32x32b_x32(ocol + c, o);
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] *= corr;
              tmem_st_32x32b_x32(ocol + c, o);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
#ifdef WC_ATTN_TRACE
      const unsigned long long td = clock64();
      ATTN_TRACE_ADD(9, td - tc);
#endif
      if (j == n_kt - 1) {
        // epilogue of head h: O / l -> f16, then release the O buffer
        if (ok) ok = __all_sync(0xFFFFFFFFu, mbar_wait(o_done, t & 1, status));
#ifdef WC_ATTN_TRACE
        ATTN_TRACE_ADD(6, clock64() - td);
#endif
        if (ok) {
          tc_fence_after();
          const float inv = 1.0f / l_run;
          const uint32_t ocol = trow + kColO;
#pragma unroll 1
          for (int c = 0; c < kDh; c += 32) {
            float o[32];
            tmem_ld_32x32b_x32(ocol + c, o);
            if (qi < L) {
              __half* dst = out + (row0 + qi) * inner + (h0 + hh) * kDh + c;
#pragma unroll
              for (int i = 0; i < 32; i += 8) {
                uint4 w;
                w.x = pack_f16x2_sat(o[i] * inv, o[i + 1] * inv);
                w.y = pack_f16x2_sat(o[i + 2] * inv, o[i + 3] * inv);
                w.z = pack_f16x2_sat(o[i + 4] * inv, o[i + 5] * inv);
                w.w = pack_f16x2_sat(o[i + 6] * inv, o[i + 7] * inv);
                *reinterpret_cast<uint4*>(dst + i) = w;
              }
            }
          }
        }
      }
    }
  }

  ATTN_TRACE(3, clock64());
#ifdef WC_ATTN_TRACE
  ATTN_TRACE(4, tr_acc[4]);
  ATTN_TRACE(5, tr_acc[5]);
  ATTN_TRACE(6, tr_acc[6]);
  ATTN_TRACE(9, tr_acc[9]);
#endif
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

#ifdef WC_ATTN_TRACE
extern "C" int wc_debug_attn_trace(unsigned long long* host, int n_ctas) {
  return cudaMemcpyFromSymbol(host, g_attn_trace, sizeof(unsigned long long) * kTraceSlots *
                                                      (n_ctas < kTraceCtas ? n_ctas : kTraceCtas)) == cudaSuccess ? 0 : -4;
}
#endif

cudaError_t attention_tc_launch(const CUtensorMap& tm_qkv, __half* out, const int32_t* lengths, int B, int L, int H,
                                const float* bias_tab, const BucketThresholds& bt, uint32_t* status,
                                cudaStream_t st) {
  if (B <= 0 || L <= 0) return cudaSuccess;
  if (L > kMaxL || 2 * bt.half > 64) return cudaErrorInvalidValue;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  // Heads per CTA: a CTA walks (head, key tile) steps as one pipeline, so
  // short sequences take several heads per CTA to amortise its set-up, long
  // ones one head (more, shorter CTAs balance the waves better); measured on
  // B200 at L = 32, 182 and 512.
  const int q_tiles = (L + kQ - 1) / kQ;
  int hpc = std::min(std::min(H, kMaxHeads), std::max(1, (256 + L - 1) / L));
  // ... but never fewer than about two CTAs per SM while heads can be split
  while (hpc > 1 && static_cast<int64_t>(q_tiles) * B * ((H + hpc - 1) / hpc) < 2 * 148) --hpc;
  const int groups = (H + hpc - 1) / hpc;
  hpc = (H + groups - 1) / groups;  // balance the groups
  dim3 grid(q_tiles, groups, B);
  return launch_pdl(attention_tc_kernel, grid, dim3(kThreads), kSmem, st, nullptr, 0, tm_qkv, out, lengths, L, H, hpc,
                    bias_tab, bt, status);
}

}  // namespace wc
