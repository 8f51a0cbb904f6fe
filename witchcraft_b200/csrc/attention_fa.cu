// Bidirectional T5 encoder self-attention on tcgen05, two query tiles per
// CTA in ping-pong (padded lengths 65..1024, an even head count).  Same
// mathematics as attention_tc.cu (src/quantized_t5.rs:426-500: scores without
// 1/sqrt(d) scaling + relative-position bias, key padding mask, softmax, P V),
// restructured so that the tensor cores and the exponential units overlap:
//
//   * One CTA per SM walks "pairs" of 128-query tiles of one sequence: the
//     tiles 2p and 2p+1 of one head (they share every K and V tile), or,
//     for the last tile of a sequence with an odd tile count, that tile of
//     heads 2k and 2k+1.  Both tiles of a pair have the same key tiles, so
//     the two softmax warpgroups step in lockstep.
//   * Key tiles of 128 (S = Q K^T is M=128 x N=128 x K=64; P V is M=128 x
//     N=64 x K=128), half as many pipeline steps as 64-key tiles.
//   * Warpgroup A (warps 0-3) and B (warps 4-7) own one S buffer each in
//     TMEM.  The MMA thread issues P_A V, then S_A of the next step, then
//     P_B V and S_B of the next step, so while one warpgroup computes its
//     exponentials the tensor cores run the other's products.
//   * TMEM (512 columns): S_A 0-127, S_B 128-255, O_A in 256/320 and O_B in
//     384/448 (two buffers each, by pair parity, so a pair's epilogue runs
//     after the next pair's first step instead of waiting for its last P V).
//   * K and V arrive through 3-stage TMA rings in consumption order (one
//     tile per step when the pair shares its head, two otherwise).
//   * warp 8: TMA producer; warp 9: TMEM allocation and the MMA thread.
// Rows of query tiles that lie wholly past a sequence's length (up to the
// padded length L) are written as zeros.  Every wait is bounded; a timeout
// sets kStatusWaitTimeout and the kernel runs to its end.
#include "attention.h"
#include "attn_common.cuh"
#include "common.cuh"

#include <algorithm>

namespace wc {

namespace {

constexpr int kQ = 128;        // queries per tile
constexpr int kKeys = 128;     // keys per step
constexpr int kDh = 64;
constexpr int kTileBytes = 128 * 128;  // 128 rows x 64 f16
constexpr int kKS = 3, kVS = 3;        // K / V ring stages
constexpr int kMaxL = 1024;
constexpr int kMaxHeads = 16;
constexpr int kMaxSeqs = 1024;
constexpr int kThreads = 320;
// Bias row of a tile: bias[x] for key - query = x - q0 - (kQ - 1), x in
// [0, n_kt * kKeys + kQ - 1), in two copies, the second shifted by one entry
// (8-byte aligned pair loads for every row); 1168 = 16 (mod 32) words apart so
// neighbouring lanes reading different copies use different banks.
constexpr int kBiasPad = 1168;
static_assert(kBiasPad >= kMaxL + kQ && kBiasPad % 32 == 16, "bias row copies");
constexpr int kBktHalf = kMaxL + kQ;  // bucket LUT covers |delta| <= kBktHalf

constexpr int kOffQ = 0;                                  // [2 pair buffers][2 tiles]
constexpr int kOffK = kOffQ + 4 * kTileBytes;             // [kKS]
constexpr int kOffV = kOffK + kKS * kTileBytes;           // [kVS]
constexpr int kOffBias = kOffV + kVS * kTileBytes;        // f32 [2 tiles][2 copies][kBiasPad]
constexpr int kOffTab = kOffBias + 2 * 2 * kBiasPad * 4;  // f32 [kMaxHeads][64]
constexpr int kOffThr = kOffTab + kMaxHeads * 64 * 4;     // int [32]
constexpr int kOffOrder = kOffThr + 32 * 4;               // u32 [kMaxSeqs]: b | length << 16
constexpr int kOffPre = kOffOrder + kMaxSeqs * 4;         // int [kMaxSeqs + 1]: pairs before each
constexpr int kOffHist = kOffPre + (kMaxSeqs + 32) * 4;   // int [64]
constexpr int kOffBkt = kOffHist + 64 * 4;                // u8 [2 kBktHalf + 1]
constexpr int kOffStage = kOffBkt + ((2 * kBktHalf + 1 + 127) & ~127);  // [8 warps][32 rows][64 B]
constexpr int kOffBar = kOffStage + 8 * 32 * 64;
constexpr int kSmem = 1024 + kOffBar + 256;
static_assert(kSmem <= 232448, "shared memory");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 256;

// One pair: tile A (head hA, queries q0A..) and tile B (hB, q0B) of sequence
// b; `shared` when both are the same head (one K / V tile per step).
struct Pair {
  int id, round, b, len, n_kt, hA, q0A, hB, q0B;
  bool shared;
};

struct PairList {
  const uint32_t* order;  // sorted (b | len << 16), longest first
  const int* pre;         // pre[pos] = pairs of the sequences before pos
  int n_seq, n_pairs, H;

  __device__ __forceinline__ Pair decode(int round) const {
    const int g = static_cast<int>(gridDim.x);
    const int id = round * g + ((round & 1) ? g - 1 - static_cast<int>(blockIdx.x) : static_cast<int>(blockIdx.x));
    Pair p{id, round, 0, 0, 0, 0, 0, 0, 0, true};
    if (id >= n_pairs) return p;
    int lo = 0, hi = n_seq - 1;  // last pos with pre[pos] <= id
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (pre[mid] <= id) lo = mid;
      else hi = mid - 1;
    }
    const int k = id - pre[lo];
    const uint32_t e = order[lo];
    p.b = static_cast<int>(e & 0xFFFFu);
    p.len = static_cast<int>(e >> 16);
    const int qt = (p.len + kQ - 1) / kQ;
    p.n_kt = (p.len + kKeys - 1) / kKeys;
    const int full = qt >> 1;
    if (k < H * full) {
      p.hA = p.hB = k / full;
      p.q0A = (k % full) * 2 * kQ;
      p.q0B = p.q0A + kQ;
      p.shared = true;
    } else {
      const int k2 = k - H * full;
      p.hA = 2 * k2;
      p.hB = 2 * k2 + 1;
      p.q0A = p.q0B = (qt - 1) * kQ;
      p.shared = false;
    }
    return p;
  }
};

__device__ __forceinline__ int pairs_of(int len, int H) {
  const int qt = (len + kQ - 1) / kQ;
  return H * (qt >> 1) + (H >> 1) * (qt & 1);
}

struct Cursor {
  Pair p;
  int j, g;
  __device__ __forceinline__ bool valid(const PairList& pl) const { return p.id < pl.n_pairs; }
  __device__ __forceinline__ void advance(const PairList& pl) {
    if (++j == p.n_kt) {
      p = pl.decode(p.round + 1);
      j = 0;
      ++g;
    }
  }
};

// One warp: order[] = the sequences by descending key-tile count (a stable
// counting sort, identical in every CTA) with their clamped lengths, and
// pre[] = the exclusive prefix of their pair counts (pre[n_seq] = total).
__device__ void sort_sequences(const int32_t* lengths, int B, int L, int H, uint32_t* order, int* pre, int* hist,
                               int lane) {
  constexpr int kBins = kMaxL / kKeys + 1;
  for (int i = lane; i < 64; i += 32) hist[i] = 0;
  __syncwarp();
  auto len_of = [&](int b) { return max(0, min(lengths[b], L)); };
  for (int b0 = 0; b0 < B; b0 += 32) {
    const int b = b0 + lane;
    const int key = b < B ? (len_of(b) + kKeys - 1) / kKeys : -1;
    const unsigned same = __match_any_sync(0xFFFFFFFFu, key);
    if (key >= 0 && lane == __ffs(same) - 1) hist[key] += __popc(same);
    __syncwarp();
  }
  if (lane == 0) {
    int run = 0;
    for (int k = kBins - 1; k >= 0; --k) {
      const int c = hist[k];
      hist[k] = run;
      run += c;
    }
  }
  __syncwarp();
  for (int b0 = 0; b0 < B; b0 += 32) {
    const int b = b0 + lane;
    const int len = b < B ? len_of(b) : 0;
    const int key = b < B ? (len + kKeys - 1) / kKeys : -1;
    const unsigned same = __match_any_sync(0xFFFFFFFFu, key);
    if (key >= 0)
      order[hist[key] + __popc(same & ((1u << lane) - 1u))] =
          static_cast<uint32_t>(b) | (static_cast<uint32_t>(len) << 16);
    __syncwarp();
    if (key >= 0 && lane == __ffs(same) - 1) hist[key] += __popc(same);
    __syncwarp();
  }
  // exclusive prefix of the pair counts in sorted order
  int run = 0;
  for (int p0 = 0; p0 < B; p0 += 32) {
    const int p = p0 + lane;
    const int c = p < B ? pairs_of(static_cast<int>(order[p] >> 16), H) : 0;
    int x = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xFFFFFFFFu, x, o);
      if (lane >= o) x += y;
    }
    if (p < B) pre[p] = run + x - c;
    run += __shfl_sync(0xFFFFFFFFu, x, 31);
  }
  if (lane == 0) pre[B] = run;
  __syncwarp();
}

__global__ void __maxnreg__(200)
    attention_fa_kernel(const __grid_constant__ CUtensorMap tmQKV, __half* __restrict__ out,
                        const int32_t* __restrict__ lengths, int B, int L, int H,
                        const float* __restrict__ bias_tab, BucketThresholds bt, uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + kOffQ;
  uint8_t* sK = smem + kOffK;
  uint8_t* sV = smem + kOffV;
  float* sTab = reinterpret_cast<float*>(smem + kOffTab);  // [head][bucket] * log2(e)
  int* sThr = reinterpret_cast<int*>(smem + kOffThr);
  uint32_t* sOrder = reinterpret_cast<uint32_t*>(smem + kOffOrder);
  int* sPre = reinterpret_cast<int*>(smem + kOffPre);
  uint8_t* sBkt = smem + kOffBkt;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars;              // [2] Q of both tiles of the pair in buffer g % 2
  uint64_t* q_empty = bars + 2;         // [2] the pair's last S is done
  uint64_t* k_full = bars + 4;          // [kKS]
  uint64_t* k_empty = k_full + kKS;     // [kKS]
  uint64_t* v_full = k_empty + kKS;     // [kVS]
  uint64_t* v_empty = v_full + kVS;     // [kVS]
  uint64_t* s_full = v_empty + kVS;     // [2 tiles]
  uint64_t* p_full = s_full + 2;        // [2 tiles], 4 warps arrive
  uint64_t* o_done = p_full + 2;        // [2 tiles][2 step parities]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 4);

  pdl_wait();
  pdl_launch_next();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int inner = H * kDh;

  if (threadIdx.x == 0) {
    mbar_init(&q_full[0], 1);
    mbar_init(&q_full[1], 1);
    mbar_init(&q_empty[0], 1);
    mbar_init(&q_empty[1], 1);
    for (int i = 0; i < kKS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < kVS; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int w = 0; w < 2; ++w) {
      mbar_init(&s_full[w], 1);
      mbar_init(&p_full[w], 4);
      mbar_init(&o_done[2 * w], 1);
      mbar_init(&o_done[2 * w + 1], 1);
    }
    mbar_fence_init();
    tma_prefetch_desc(&tmQKV);
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 8) sort_sequences(lengths, B, L, H, sOrder, sPre, reinterpret_cast<int*>(smem + kOffHist), lane);
  if (threadIdx.x < 32) sThr[threadIdx.x] = bt.thr[threadIdx.x];
  for (int i = threadIdx.x; i < H * 2 * bt.half; i += blockDim.x) {
    const int h = i / (2 * bt.half), bk = i % (2 * bt.half);
    sTab[h * 64 + bk] = bias_tab[bk * H + h] * 1.4426950408889634f;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // buckets of every key - query offset a tile can meet (after sThr is set)
  for (int i = threadIdx.x; i < 2 * kBktHalf + 1; i += blockDim.x)
    sBkt[i] = static_cast<uint8_t>(rel_bucket_tc(sThr, bt.half, i - kBktHalf));
  const uint32_t tmem = *tmem_slot;
  const PairList pl{sOrder, sPre, B, sPre[B], H};
  const Cursor start{pl.decode(0), 0, 0};

  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      auto load_q = [&](const Pair& p, int g) -> bool {
        const int s = g & 1;
        if (!mbar_wait(&q_empty[s], ((g >> 1) & 1) ^ 1, status)) return false;
        uint8_t* dst = sQ + s * 2 * kTileBytes;
        mbar_arrive_expect_tx(&q_full[s], 2 * kTileBytes);
        const int ra = p.b * L + p.q0A, rb = p.b * L + p.q0B;
        tma_load_2d(dst, &tmQKV, &q_full[s], p.hA * kDh, ra);
        tma_load_2d(dst + kTileBytes / 2, &tmQKV, &q_full[s], p.hA * kDh, ra + 64);
        tma_load_2d(dst + kTileBytes, &tmQKV, &q_full[s], p.hB * kDh, rb);
        tma_load_2d(dst + kTileBytes + kTileBytes / 2, &tmQKV, &q_full[s], p.hB * kDh, rb + 64);
        return true;
      };
      auto load_kv = [&](uint8_t* ring, uint64_t* full, uint64_t* empty, int stages, int pos, int col,
                         int row) -> bool {
        const int s = pos % stages;
        if (!mbar_wait(&empty[s], ((pos / stages) & 1) ^ 1, status)) return false;
        uint8_t* dst = ring + s * kTileBytes;
        mbar_arrive_expect_tx(&full[s], kTileBytes);
        tma_load_2d(dst, &tmQKV, &full[s], col, row);
        tma_load_2d(dst + kTileBytes / 2, &tmQKV, &full[s], col, row + 64);
        return true;
      };
      Cursor c = start;
      bool ok = !c.valid(pl) || load_q(c.p, 0);
      int kp = 0, vp = 0;
      while (ok && c.valid(pl)) {
        if (c.j == 0) {
          const Pair nx = pl.decode(c.p.round + 1);
          if (nx.id < pl.n_pairs && !(ok = load_q(nx, c.g + 1))) break;
        }
        const int krow = c.p.b * L + c.j * kKeys;
        if (!(ok = load_kv(sK, k_full, k_empty, kKS, kp++, inner + c.p.hA * kDh, krow))) break;
        if (!c.p.shared && !(ok = load_kv(sK, k_full, k_empty, kKS, kp++, inner + c.p.hB * kDh, krow))) break;
        if (!(ok = load_kv(sV, v_full, v_empty, kVS, vp++, 2 * inner + c.p.hA * kDh, krow))) break;
        if (!c.p.shared && !(ok = load_kv(sV, v_full, v_empty, kVS, vp++, 2 * inner + c.p.hB * kDh, krow))) break;
        c.advance(pl);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_f16_f32(kQ, kKeys);
      constexpr uint32_t idesc_pv = idesc_f16_f32(kQ, kDh) | (1u << 16);  // B (V) MN-major
      bool ok = true;
      int kc = 0, vc = 0;  // K / V ring positions consumed
      // S_w of step c = Q_w K^T into S buffer w (K-ring position kpos)
      auto issue_s = [&](const Cursor& c, int w, int kpos) -> bool {
        const int s = kpos % kKS;
        if (!mbar_wait(&k_full[s], (kpos / kKS) & 1, status)) return false;
        tc_fence_after();
        const uint64_t qa = sw128_kmajor_desc(smem_u32(sQ + ((c.g & 1) * 2 + w) * kTileBytes));
        const uint64_t bk = sw128_kmajor_desc(smem_u32(sK + s * kTileBytes));
#pragma unroll
        for (int k = 0; k < kDh / 16; ++k) tc_mma_f16(tmem + w * 128, qa + 2 * k, bk + 2 * k, idesc_qk, k > 0);
        return true;
      };
      // both S of step c, then free their K slots (and the Q buffer after
      // the pair's last step)
      auto issue_s_pair_a = [&](const Cursor& c, int& ka) -> bool {
        if (c.j == 0 && !mbar_wait(&q_full[c.g & 1], (c.g >> 1) & 1, status)) return false;
        ka = kc++;
        return issue_s(c, 0, ka);
      };
      auto issue_s_pair_b = [&](const Cursor& c, int ka) -> bool {
        const int kb = c.p.shared ? ka : kc++;
        if (!issue_s(c, 1, kb)) return false;
        tc_commit(&k_empty[ka % kKS]);
        if (!c.p.shared) tc_commit(&k_empty[kb % kKS]);
        if (c.j == c.p.n_kt - 1) tc_commit(&q_empty[c.g & 1]);
        return true;
      };
      auto issue_pv = [&](const Cursor& c, int w, int vpos, int t) -> bool {
        const int s = vpos % kVS;
        if (!mbar_wait(&v_full[s], (vpos / kVS) & 1, status)) return false;
        tc_fence_after();
        const uint64_t v = sw128_mnmajor_desc(smem_u32(sV + s * kTileBytes));
        const uint32_t pa = tmem + w * 128;
        const uint32_t od = tmem + kColO + w * 128 + 64 * (c.g & 1);
#pragma unroll
        for (int k = 0; k < kKeys / 16; ++k)
          tc_mma_f16_ts(od, pa + 8 * k, v + 128 * k, idesc_pv, (c.j > 0 || k > 0) ? 1u : 0u);
        tc_commit(&o_done[2 * w + (t & 1)]);
        return true;
      };
      Cursor c = start;
      int ka = 0;
      if (c.valid(pl)) ok = issue_s_pair_a(c, ka) && issue_s_pair_b(c, ka);
      for (int t = 0; ok && c.valid(pl); ++t) {
        const int va = vc++;
        const int vb = c.p.shared ? va : vc++;
        Cursor n = c;
        n.advance(pl);
        if (!(ok = mbar_wait(&p_full[0], t & 1, status))) break;
        if (!(ok = issue_pv(c, 0, va, t))) break;
        int na = 0;
        if (n.valid(pl) && !(ok = issue_s_pair_a(n, na))) break;
        if (!(ok = mbar_wait(&p_full[1], t & 1, status))) break;
        if (!(ok = issue_pv(c, 1, vb, t))) break;
        tc_commit(&v_empty[va % kVS]);
        if (!c.p.shared) tc_commit(&v_empty[vb % kVS]);
        if (n.valid(pl) && !(ok = issue_s_pair_b(n, na))) break;
        c = n;
      }
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue (warpgroup w)
    const int w = warp >> 2;             // tile A or B of each pair
    const int st = threadIdx.x & 127;    // thread within the warpgroup
    const int qd = warp & 3;             // TMEM lane quarter
    const int r = qd * 32 + lane;        // query row within the tile
    const uint32_t trow = tmem + (static_cast<uint32_t>(qd * 32) << 16);
    const uint32_t scol = trow + w * 128;
    float* sBias = reinterpret_cast<float*>(smem + kOffBias) + w * 2 * kBiasPad;

    // zero rows of the query tiles that lie wholly past their sequence
    {
      const int wid = warp, nw = 8;
      for (int pos = blockIdx.x; pos < B; pos += gridDim.x) {
        const uint32_t e = sOrder[pos];
        const int b = static_cast<int>(e & 0xFFFFu), len = static_cast<int>(e >> 16);
        const int z0 = (len + kQ - 1) / kQ * kQ;
        for (int row = z0 + wid; row < L; row += nw) {
          uint4* dst = reinterpret_cast<uint4*>(out + (static_cast<size_t>(b) * L + row) * inner);
          for (int c = lane; c < inner / 8; c += 32) dst[c] = make_uint4(0, 0, 0, 0);
        }
      }
    }

    struct Pending {
      size_t row0;
      int q0, h, t_last, g;
      float inv;
    };
    auto epilogue = [&](const Pending& e) -> bool {
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(&o_done[2 * w + (e.t_last & 1)], (e.t_last >> 1) & 1, status)))
        return false;
      tc_fence_after();
      const uint32_t ocol = trow + kColO + w * 128 + 64 * (e.g & 1);
      uint8_t* stage = smem + kOffStage + warp * 2048;
      const int rq0 = e.q0 + qd * 32;
      bool clip = false;
#pragma unroll 1
      for (int c = 0; c < kDh; c += 32) {
        float o[32];
        tmem_ld_32x32b_x32(ocol + c, o);
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 v;
          v.x = pack_f16x2_sat(o[i] * e.inv, o[i + 1] * e.inv, clip);
          v.y = pack_f16x2_sat(o[i + 2] * e.inv, o[i + 3] * e.inv, clip);
          v.z = pack_f16x2_sat(o[i + 4] * e.inv, o[i + 5] * e.inv, clip);
          v.w = pack_f16x2_sat(o[i + 6] * e.inv, o[i + 7] * e.inv, clip);
          *reinterpret_cast<uint4*>(stage + lane * 64 + 16 * ((i >> 3) ^ ((lane >> 1) & 3))) = v;
        }
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int rr = k * 8 + (lane >> 2), ch = lane & 3;
          const uint4 v = *reinterpret_cast<const uint4*>(stage + rr * 64 + 16 * (ch ^ ((rr >> 1) & 3)));
          if (rq0 + rr < L)
            *reinterpret_cast<uint4*>(out + (e.row0 + rq0 + rr) * inner + e.h * kDh + c + ch * 8) = v;
        }
        __syncwarp();
      }
      report_f16_clip(clip, status);
      return true;
    };

    Pending pend{0, 0, 0, 0, 0, 0.f};
    bool has_pend = false, ok = true;
    int t = 0, g = 0;
    const uint32_t bar_id = 1 + w;
    for (int round = 0;; ++round, ++g) {
      const Pair p = pl.decode(round);
      if (p.id >= pl.n_pairs) break;
      const int h = w ? p.hB : p.hA, q0 = w ? p.q0B : p.q0A;
      const size_t row0 = static_cast<size_t>(p.b) * L;
      // bias row of this tile, after every thread of the warpgroup has
      // finished the previous tile's steps
      asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");
      {
        const float* tab = sTab + h * 64;
        const uint8_t* bk = sBkt + kBktHalf - q0 - (kQ - 1);
        for (int x = st; x < p.n_kt * kKeys + kQ - 1; x += 128) {
          const float v = tab[bk[x]];
          sBias[x] = v;
          if (x > 0) sBias[kBiasPad + x - 1] = v;
        }
      }
      asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");
      // bias of key c at brow[c], brow 8-byte aligned
      const float* brow = ((kQ - 1 - r) & 1) ? sBias + kBiasPad + (kQ - 2 - r) : sBias + (kQ - 1 - r);
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = 0; j < p.n_kt; ++j, ++t) {
        const int k0 = j * kKeys;
        if (ok) ok = __all_sync(0xFFFFFFFFu, mbar_wait(&s_full[w], t & 1, status));
        if (ok) {
          tc_fence_after();
          float v[kKeys];
#pragma unroll
          for (int c = 0; c < kKeys; c += 32) tmem_ld_32x32b_x32_nowait(scol + c, &v[c]);
          tmem_wait_ld();
          const uint64_t kLog2e2 = f2(1.4426950408889634f, 1.4426950408889634f);
#pragma unroll
          for (int i = 0; i < kKeys; i += 2) {
            const float2 bb = *reinterpret_cast<const float2*>(brow + k0 + i);
            const uint64_t x = f2_fma(f2(v[i], v[i + 1]), kLog2e2, f2(bb.x, bb.y));
            v[i] = f2_lo(x);
            v[i + 1] = f2_hi(x);
          }
          if (k0 + kKeys > p.len) {
#pragma unroll
            for (int i = 0; i < kKeys; ++i)
              if (k0 + i >= p.len) v[i] = -INFINITY;
          }
          float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int i = 0; i < kKeys; i += 2) mx[(i >> 1) & 3] = fmax3(mx[(i >> 1) & 3], v[i], v[i + 1]);
          const float tmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
          // lazy rescale: keep the running max unless this tile raises it by
          // more than 15 (log2 units), so P <= 2^15 stays in the f16 range
          const float m_new = (tmax > m_run + 15.0f) ? tmax : m_run;
          const float corr = ex2(m_run - m_new);
          const uint64_t negm = f2(-m_new, -m_new);
          uint64_t ps[4] = {0, 0, 0, 0};
          // P = 2^(v - max) as f16 pairs over the first 64 columns of the S
          // buffer, 64 keys (32 columns) at a time
#pragma unroll
          for (int hk = 0; hk < kKeys; hk += 64) {
            uint32_t pk[32];
#pragma unroll
            for (int i = 0; i < 64; i += 2) {
              const uint64_t x = f2_add(f2(v[hk + i], v[hk + i + 1]), negm);
              const uint64_t e = f2(ex2(f2_lo(x)), ex2(f2_hi(x)));
              ps[(i >> 1) & 3] = f2_add(ps[(i >> 1) & 3], e);
              pk[i >> 1] = f2_to_h2(e);
            }
            tmem_st_u32_x32(scol + hk / 2, pk);
          }
          const uint64_t ps2 = f2_add(f2_add(ps[0], ps[1]), f2_add(ps[2], ps[3]));
          l_run = l_run * corr + (f2_lo(ps2) + f2_hi(ps2));
          m_run = m_new;
          if (j > 0 && __any_sync(0xFFFFFFFFu, corr != 1.0f)) {
            // O holds P V of the previous step once o_done says so; rescale
            ok = __all_sync(0xFFFFFFFFu,
                            mbar_wait(&o_done[2 * w + ((t - 1) & 1)], ((t - 1) >> 1) & 1, status));
            if (ok) {
              tc_fence_after();
              const uint32_t ocol = trow + kColO + w * 128 + 64 * (g & 1);
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
        if (lane == 0) mbar_arrive(&p_full[w]);
        if (j == 0 && has_pend) {
          // the previous pair's last P V ran while this step was computed
          if (ok) ok = epilogue(pend);
          has_pend = false;
        }
      }
      pend = Pending{row0, q0, h, t - 1, g, 1.0f / l_run};
      has_pend = true;
    }
    if (has_pend && ok) epilogue(pend);
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

bool attention_fa_supports(int B, int L, int H, int num_buckets) {
  return L > 64 && L <= kMaxL && B >= 1 && B <= kMaxSeqs && H >= 2 && H <= kMaxHeads && H % 2 == 0 &&
         num_buckets <= 64;
}

cudaError_t attention_fa_launch(const CUtensorMap& tm_qkv, __half* out, const int32_t* lengths, int B, int L, int H,
                                const float* bias_tab, const BucketThresholds& bt, uint32_t* status,
                                cudaStream_t st) {
  if (B <= 0 || L <= 0) return cudaSuccess;
  if (!attention_fa_supports(B, L, H, 2 * bt.half)) return cudaErrorInvalidValue;
  static bool attr_set[64] = {};
  static int num_sms[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attention_fa_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&num_sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  // upper bound of the pair count: every sequence at the padded length
  const int qt = (L + kQ - 1) / kQ;
  const int64_t max_pairs = static_cast<int64_t>(B) * (H * (qt >> 1) + (H >> 1) * (qt & 1));
  const int grid = static_cast<int>(std::min<int64_t>(max_pairs, num_sms[dev]));
  return launch_pdl(attention_fa_kernel, dim3(grid), dim3(kThreads), kSmem, st, nullptr, 0, tm_qkv, out, lengths, B,
                    L, H, bias_tab, bt, status);
}

}  // namespace wc
