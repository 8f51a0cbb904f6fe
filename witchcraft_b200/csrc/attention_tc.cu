// Bidirectional T5 encoder self-attention on the 5th-generation tensor cores
// (tcgen05 + TMEM), flash-style with an online softmax, the T5 relative-
// position bias and a key padding mask.  Replaces src/quantized_t5.rs:426-500:
// scores without 1/sqrt(d) scaling, + position bias, softmax_last_dim, P.V,
// transpose back to tokens.
//
// Persistent: a grid of two CTAs per SM walks the items (sequence, 128-query
// tile, head) with a static stride, and each CTA runs the flattened sequence
// of its steps (item, 64-key tile) as one pipeline, so the TMA loads and S
// MMAs of the next step -- also across an item boundary -- overlap the
// softmax of the current one, and the set-up (barriers, TMEM, the bias
// tables of all heads) is paid once per CTA:
//   warp 0      TMA: the Q tile of each item (two shared-memory buffers,
//               one item ahead), its K and V tiles (two 2-stage rings; a K
//               stage is freed as soon as its S is done)
//   warp 1      TMEM allocation and the single MMA-issuing thread
//   warps 2-5   softmax and epilogue (thread = query row = TMEM lane)
// Step t (item g, key tile j): S(t) = Q K_j^T (M=128, N=64, K=64, Q and K
// K-major from their TMA tiles, f32 in TMEM buffer t % 2, computed two steps
// ahead); the softmax warps add the relative-position bias (a per-item bias
// row they build), mask keys past the sequence, update the running max / sum,
// rescale the O row in TMEM when the max moved and store P = 2^(S - max) as
// f16 into the first 32 columns of S buffer t % 2; then O_g += P V_j (M=128,
// N=64, K=64, A = P from TMEM, V read MN-major from its TMA tile).  S(t + 2)
// reuses that buffer only after P(t) V(t), in MMA issue order.  O has two
// TMEM buffers (item g in buffer g % 2), so the epilogue of item g (O / sum
// -> f16 -> global) runs after the first step of item g + 1, when its last
// P V has long finished, instead of waiting for it.
// Input: the token-major QKV projection [B*L][3*H*64] f16 through one TMA
// descriptor (box 64 x 64); output [B*L][H*64] f16.  Query rows of an
// all-padding tile are written as zeros.
#include "attention.h"
#include "attn_common.cuh"
#include "common.cuh"

#include <algorithm>
#include <cstdlib>

namespace wc {

namespace {

// Optional event trace for pipeline analysis (off in the library build):
// single threads of the first kTraceCtas CTAs log (event code, SM clock).
#ifdef WC_ATTN_TRACE
constexpr int kTraceCtas = 16, kTraceLen = 8192, kTraceRole = kTraceLen / 8;
__device__ unsigned long long g_attn_trace[kTraceCtas][kTraceLen];
#define ATRACE(code)                                                                                    \
  do {                                                                                                  \
    if (blockIdx.x < kTraceCtas && tr_n < kTraceRole)                                                   \
      g_attn_trace[blockIdx.x][(threadIdx.x >> 5) * kTraceRole + tr_n++] =   \
          (static_cast<unsigned long long>(code) << 56) |                                               \
          (static_cast<unsigned long long>(clock64()) & ((1ull << 56) - 1));                            \
  } while (0)
#define ATRACE_NS(code)                                                                              \
  do {                                                                                               \
    if (blockIdx.x < kTraceCtas && threadIdx.x == 0)                                                 \
      g_attn_trace[blockIdx.x][7 * kTraceRole + (code & 1)] =                                        \
          (static_cast<unsigned long long>(code) << 56) | (global_timer_ns() & ((1ull << 56) - 1));   \
  } while (0)
#else
#define ATRACE_NS(code) \
  do {                  \
  } while (0)
#define ATRACE(code) \
  do {               \
  } while (0)
#endif

constexpr int kQ = 128;       // queries per item
constexpr int kKeys = 64;     // keys per tile
constexpr int kDh = 64;
constexpr int kQBytes = kQ * 128;      // 128 x 64 f16
constexpr int kKVBytes = kKeys * 128;  // 64 x 64 f16
constexpr int kWin = kQ + kKeys - 1;   // distinct key - query offsets of one tile pair
constexpr int kMaxHeads = 32;          // bias tables of all heads stay in shared memory
// K runs three stages deep, so the load of K(t) can start once S(t - 3) is
// done, a whole softmax step before S(t - 2) would free a two-stage ring; V
// keeps two stages (it is needed a step after K)
constexpr int kKStages = 3;
constexpr int kVStages = 2;
constexpr int kOffQ = 0;                              // 2 buffers
constexpr int kOffK = kOffQ + 2 * kQBytes;            // kKStages stages
constexpr int kOffV = kOffK + kKStages * kKVBytes;    // kVStages stages
constexpr int kMaxL = 2048;
// Bias row of one item: bias[x] for key - query = x - q0 - (kQ - 1), built
// once per item, in two copies, the second shifted by one entry, so that
// every thread reads its biases as 8-byte aligned pairs; the copies are
// 2256 = 16 (mod 32) words apart, so the neighbouring lanes that read the
// same offsets from different copies fall in different banks.
constexpr int kBiasPad = 2256;
static_assert(kBiasPad >= kMaxL + kWin + 1 && kBiasPad % 32 == 16, "bias row copies");
constexpr int kOffBias = kOffV + kVStages * kKVBytes;  // f32 [2 copies][kBiasPad]
constexpr int kMaxBuckets = 32;                        // T5's relative_attention_num_buckets
constexpr int kOffTab = kOffBias + 2 * kBiasPad * 4;   // f32 [kMaxHeads][kMaxBuckets]
constexpr int kOffThr = kOffTab + kMaxHeads * kMaxBuckets * 4;  // int [32]
constexpr int kMaxSortSeqs = 1024;  // larger batches keep their own sequence order
constexpr int kOffOrder = kOffThr + 32 * 4;            // u32 [kMaxSortSeqs]: b | length << 16
constexpr int kOffHist = kOffOrder + kMaxSortSeqs * 4;                   // int [64]
// bucket of every key - query offset an item's bias row can need: index
// delta + kBktHalf, |delta| <= kMaxL + kWin
constexpr int kBktHalf = kMaxL + kWin;
constexpr int kOffBkt = kOffHist + 64 * 4;                               // u8 [2 kBktHalf + 1]
constexpr int kOffStage = kOffBkt + ((2 * kBktHalf + 1 + 127) & ~127);   // [4 warps][32 rows][64 B]
constexpr int kOffBar = kOffStage + 4 * 32 * 64;
constexpr int kSmem = 1024 + kOffBar + 256;
constexpr int kThreads = 192;
constexpr int kCtasPerSm = 2;
constexpr uint32_t kTmemCols = 256;
// S (and P) buffers at 0 / 64, O buffers at 128 / 192
constexpr uint32_t kColS = 0, kColO = 128;

// One unit of work: the kQ queries from q0 of sequence b, head h.  Items
// are numbered with the sequences in descending order of key tiles (the
// order every CTA derives identically, see sort_sequences), then query tile,
// then head; in round r a CTA takes item r * grid + its rank, its rank taken
// from the other end in odd rounds, which balances the CTAs' work like
// longest-first scheduling.  id >= n_items marks the end of a CTA's list.
struct Item {
  int id, round, b, q0, h, len, n_kt;
};

struct ItemList {
  const int32_t* lengths;
  const uint32_t* order;  // sorted (sequence | length << 16), or null: identity
  int n_items, q_tiles, H, L;

  __device__ __forceinline__ int seq_len(int b) const { return max(0, min(lengths[b], L)); }
  __device__ __forceinline__ Item decode(int round) const {
    const int g = static_cast<int>(gridDim.x);
    const int id = round * g + ((round & 1) ? g - 1 - static_cast<int>(blockIdx.x) : static_cast<int>(blockIdx.x));
    Item it{id, round, 0, 0, 0, 0, 0};
    if (id >= n_items) return it;
    it.h = id % H;
    const int rest = id / H;
    it.q0 = (rest % q_tiles) * kQ;
    const int pos = rest / q_tiles;
    if (order) {
      const uint32_t e = order[pos];
      it.b = static_cast<int>(e & 0xFFFFu);
      it.len = static_cast<int>(e >> 16);
    } else {
      it.b = pos;
      it.len = seq_len(pos);
    }
    it.n_kt = (it.len + kKeys - 1) / kKeys;
    return it;
  }
  // This CTA's next item from round `round` on with at least one valid query.
  __device__ __forceinline__ Item next_active(int round) const {
    for (;; ++round) {
      const Item it = decode(round);
      if (it.id >= n_items || it.q0 < it.len) return it;
    }
  }
};

// Walks one CTA's steps: key tile j of its g-th active item.
struct Cursor {
  Item it;
  int j, g;
  __device__ __forceinline__ bool valid(const ItemList& il) const { return it.id < il.n_items; }
  __device__ __forceinline__ void advance(const ItemList& il) {
    if (++j == it.n_kt) {
      it = il.next_active(it.round + 1);
      j = 0;
      ++g;
    }
  }
};

// One warp: order[pos] = the sequences by descending key-tile count, ties in
// index order (a stable counting sort, so every CTA gets the same order),
// each with its clamped length, so no later step reads the lengths again.
__device__ void sort_sequences(const ItemList& il, int B, uint32_t* order, int* hist, int lane) {
  constexpr int kBins = kMaxL / kKeys + 1;
  for (int i = lane; i < 64; i += 32) hist[i] = 0;
  __syncwarp();
  for (int b0 = 0; b0 < B; b0 += 32) {
    const int b = b0 + lane;
    const int key = b < B ? (il.seq_len(b) + kKeys - 1) / kKeys : -1;
    const unsigned same = __match_any_sync(0xFFFFFFFFu, key);
    if (key >= 0 && lane == __ffs(same) - 1) hist[key] += __popc(same);
    __syncwarp();
  }
  if (lane == 0) {
    int run = 0;  // exclusive prefix, largest key first
    for (int k = kBins - 1; k >= 0; --k) {
      const int c = hist[k];
      hist[k] = run;
      run += c;
    }
  }
  __syncwarp();
  for (int b0 = 0; b0 < B; b0 += 32) {
    const int b = b0 + lane;
    const int len = b < B ? il.seq_len(b) : 0;
    const int key = b < B ? (len + kKeys - 1) / kKeys : -1;
    const unsigned same = __match_any_sync(0xFFFFFFFFu, key);
    if (key >= 0)
      order[hist[key] + __popc(same & ((1u << lane) - 1u))] =
          static_cast<uint32_t>(b) | (static_cast<uint32_t>(len) << 16);
    __syncwarp();
    if (key >= 0 && lane == __ffs(same) - 1) hist[key] += __popc(same);
    __syncwarp();
  }
}

__global__ void __launch_bounds__(kThreads)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQKV, __half* __restrict__ out,
                        const int32_t* __restrict__ lengths, int B, int L, int H,
                        const float* __restrict__ bias_tab, BucketThresholds bt, uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  ATRACE_NS(30);
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + kOffQ;
  uint8_t* sK = smem + kOffK;
  uint8_t* sV = smem + kOffV;
  float* sBias = reinterpret_cast<float*>(smem + kOffBias);
  float* sTab = reinterpret_cast<float*>(smem + kOffTab);  // [head][bucket] * log2(e)
  int* sThr = reinterpret_cast<int*>(smem + kOffThr);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars;                        // [2] per Q buffer
  uint64_t* q_empty = bars + 2;                   // [2] the item's last S is done
  // K stage t % 3 is free again once S(t) is done (k_empty, committed with
  // it); V stage t % 2 once P(t) V(t) is done, which o_done of that step
  // reports
  uint64_t* k_full = bars + 4;                    // [kKStages]
  uint64_t* k_empty = k_full + kKStages;          // [kKStages]
  uint64_t* v_full = k_empty + kKStages;          // [kVStages]
  uint64_t* s_full = v_full + kVStages;           // [2] per S buffer
  // [2] by step parity (4 softmax warps arrive): the warps do not step in
  // lockstep, one may arrive for step t + 1 before another for step t, but
  // never for t + 2 (S(t + 2) is issued only after P(t))
  uint64_t* p_full = s_full + 2;
  // [2] by step parity: P(t) V(t) done.  A softmax warp waits for P V of step
  // t - 1 (rescale, epilogue) while P V(t + 1) cannot have been issued (it
  // needs this warp's P(t + 1)); one barrier per step parity keeps that wait
  // one phase deep, which a parity wait tells apart.
  uint64_t* o_done = p_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 2);

#ifdef WC_ATTN_TRACE
  int tr_n = 0;
#endif
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q_tiles = (L + kQ - 1) / kQ;
  uint32_t* sOrder = reinterpret_cast<uint32_t*>(smem + kOffOrder);
  uint8_t* sBkt = smem + kOffBkt;
  const ItemList il{lengths, B <= kMaxSortSeqs ? sOrder : nullptr, B * q_tiles * H, q_tiles, H, L};
  const int inner = H * kDh;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kKStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < kVStages; ++i) mbar_init(&v_full[i], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_done[i], 1);
    }
    mbar_fence_init();
    tma_prefetch_desc(&tmQKV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 2 && il.order) sort_sequences(il, B, sOrder, reinterpret_cast<int*>(smem + kOffHist), lane);
  if (threadIdx.x < 32) sThr[threadIdx.x] = bt.thr[threadIdx.x];
  for (int i = threadIdx.x; i < H * 2 * bt.half; i += blockDim.x) {
    const int h = i / (2 * bt.half), bk = i % (2 * bt.half);
    sTab[h * kMaxBuckets + bk] = bias_tab[bk * H + h] * 1.4426950408889634f;
  }
  // buckets of the offsets this launch can meet (|delta| < L + kWin), from
  // the thresholds once they are in shared memory
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * (L + kWin) - 1; i += kThreads) {
    const int delta = i - (L + kWin - 1);
    sBkt[delta + kBktHalf] = static_cast<uint8_t>(rel_bucket_tc(sThr, bt.half, delta));
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Everything above reads no activation: the relative-bias weights, the
  // launch's bucket thresholds, and the lengths, which every forward copies
  // in before its first kernel.  So it runs before the wait for the previous
  // kernel (the QKV GEMM) and overlaps that kernel's last round.
  pdl_wait();
  pdl_launch_next();  // after the wait: at most one grid waits ahead
  const Cursor start{il.next_active(0), 0, 0};

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      // Q of the g-th active item into buffer g % 2 (free once the last S
      // of item g - 2 is done), one item ahead.  Issuing it later (after the
      // step's K and V loads, or only once its buffer is free) measured
      // slower: the next item's first S then waits for Q.
      auto load_q = [&](const Item& it, int g) -> bool {
        if (!mbar_wait(&q_empty[g & 1], ((g >> 1) & 1) ^ 1, status)) return false;
        ATRACE(22);
        uint8_t* dst = sQ + (g & 1) * kQBytes;
        mbar_arrive_expect_tx(&q_full[g & 1], kQBytes);
        const int row = it.b * L + it.q0;
        tma_load_2d(dst, &tmQKV, &q_full[g & 1], it.h * kDh, row);  // box: 64 rows
        tma_load_2d(dst + kQBytes / 2, &tmQKV, &q_full[g & 1], it.h * kDh, row + 64);
        return true;
      };
      // V(t) waits for P(t - 2) V(t - 2), which comes a softmax step after
      // S(t - 2); loading it one iteration late, after K(t + 1), keeps that
      // wait from holding back the next K load.
      auto load_v = [&](int tv, int col, int row) -> bool {
        // V stage tv % 2 last held V(tv - 2), free once P(tv - 2) V(tv - 2) is
        // done: o_done of that step (2 stages, 2 barriers: same index and parity)
        static_assert(kVStages == 2, "V stages are freed through the per-step P V barriers");
        const int s = tv % kVStages;
        if (!mbar_wait(&o_done[s], ((tv / kVStages) & 1) ^ 1, status)) return false;
        ATRACE(21);
        mbar_arrive_expect_tx(&v_full[s], kKVBytes);
        tma_load_2d(sV + s * kKVBytes, &tmQKV, &v_full[s], col, row);
        return true;
      };
      Cursor c = start;
      bool ok = !c.valid(il) || load_q(c.it, 0);
      int v_col = 0, v_row = 0;  // V tile of the previous step
      int t = 0;
      for (; c.valid(il) && ok; ++t) {
        if (c.j == 0) {
          // one item ahead
          const Item nx = il.next_active(c.it.round + 1);
          if (nx.id < il.n_items && !(ok = load_q(nx, c.g + 1))) break;
        }
        const int s = t % kKStages;
        const int krow = c.it.b * L + c.j * kKeys;
        // stage s last held K(t - 3), free once S(t - 3) is done
        if (!(ok = mbar_wait(&k_empty[s], ((t / kKStages) & 1) ^ 1, status))) break;
        ATRACE(20);
        mbar_arrive_expect_tx(&k_full[s], kKVBytes);
        tma_load_2d(sK + s * kKVBytes, &tmQKV, &k_full[s], inner + c.it.h * kDh, krow);
        // V(t - 1) into its stage, free once P(t - 3) V(t - 3) is done
        if (t > 0 && !(ok = load_v(t - 1, v_col, v_row))) break;
        v_col = 2 * inner + c.it.h * kDh;
        v_row = krow;
        c.advance(il);
      }
      if (ok && t > 0) load_v(t - 1, v_col, v_row);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_f16_f32(kQ, kKeys);
      constexpr uint32_t idesc_pv = idesc_f16_f32(kQ, kDh) | (1u << 16);  // B (V) MN-major
      bool ok = true;
      Cursor cs = start;  // next S to issue (two steps ahead of P V)
      int ts = 0;
      // Inputs of S(ts): its Q (first key tile of an item) and K stage.
      // Waited for before the P of the step that issues it, so that only
      // the MMAs and commits follow the softmax warps' signal.
      auto wait_s_inputs = [&]() -> bool {
        const int s = ts % kKStages;
        if (cs.j == 0 && !mbar_wait(&q_full[cs.g & 1], (cs.g >> 1) & 1, status)) return false;
        if (!mbar_wait(&k_full[s], (ts / kKStages) & 1, status)) return false;
        ATRACE(15);
        return true;
      };
      // S(ts) = Q K_j^T into S buffer ts % 2
      auto issue_s = [&]() {
        const int s = ts % kKStages;
        tc_fence_after();
        const uint64_t qa = sw128_kmajor_desc(smem_u32(sQ + (cs.g & 1) * kQBytes));
        const uint64_t bk = sw128_kmajor_desc(smem_u32(sK + s * kKVBytes));
#pragma unroll
        for (int k = 0; k < kDh / 16; ++k)
          tc_mma_f16(tmem + kColS + 64 * (ts & 1), qa + 2 * k, bk + 2 * k, idesc_qk, k > 0);
        ATRACE(16);
        tc_commit(&s_full[ts & 1]);
        tc_commit(&k_empty[s]);
        ATRACE(12);
        if (cs.j == cs.it.n_kt - 1) tc_commit(&q_empty[cs.g & 1]);
      };
      for (int k = 0; k < 2 && cs.valid(il) && ok; ++k) {
        if (!(ok = wait_s_inputs())) break;
        issue_s();
        cs.advance(il);
        ++ts;
      }
      Cursor cp = start;
      for (int t = 0; cp.valid(il) && ok; ++t) {
        const int s = t % kVStages;
        // S(t + 2) goes into S buffer t % 2 right after P(t) V(t) in issue
        // order (the tensor pipe runs them in order, so P(t) is read first)
        const bool has_s = cs.valid(il);
        if (has_s && !(ok = wait_s_inputs())) break;
        if (!(ok = mbar_wait(&v_full[s], (t / kVStages) & 1, status))) break;
        ATRACE(13);
        // P(t) of item g also means the epilogue of item g - 2 has read O buffer g % 2
        if (!(ok = mbar_wait(&p_full[t & 1], (t >> 1) & 1, status))) break;
        ATRACE(10);
        tc_fence_after();
        const uint64_t v = sw128_mnmajor_desc(smem_u32(sV + s * kKVBytes));
        const uint32_t pa = tmem + kColS + 64 * (t & 1);
#pragma unroll
        for (int k = 0; k < kKeys / 16; ++k)
          tc_mma_f16_ts(tmem + kColO + 64 * (cp.g & 1), pa + 8 * k, v + 128 * k, idesc_pv,
                        (cp.j > 0 || k > 0) ? 1u : 0u);
        ATRACE(14);
        tc_commit(&o_done[t & 1]);
        ATRACE(11);
        if (has_s) issue_s();
        cp.advance(il);
        if (has_s) {
          cs.advance(il);
          ++ts;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int st = threadIdx.x - 64;  // 0..127
    const int qd = warp & 3;          // TMEM lane quarter
    const int r = qd * 32 + lane;     // query row within the tile
    const uint32_t trow = tmem + (static_cast<uint32_t>(qd * 32) << 16);
    // Epilogue of an item whose O is final once P V of its last step t_last
    // is done: O / sum -> f16 -> global.  Each 32-column half of the warp's 32
    // rows goes through a 2 KB staging tile (16-byte chunks XOR-swizzled by
    // row, conflict-free both ways), so every store instruction writes 8 rows
    // x 64 contiguous bytes.
    struct Pending {
      size_t row0;
      int q0, h, t_last, g;
      float inv;
    };
    auto epilogue = [&](const Pending& e) -> bool {
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(&o_done[e.t_last & 1], (e.t_last >> 1) & 1, status))) return false;
      tc_fence_after();
      const uint32_t ocol = trow + kColO + 64 * (e.g & 1);
      uint8_t* stage = smem + kOffStage + qd * 2048;
      const int rq0 = e.q0 + qd * 32;  // first query row of this warp
#pragma unroll 1
      for (int c = 0; c < kDh; c += 32) {
        float o[32];
        tmem_ld_32x32b_x32(ocol + c, o);
        if (lane == 0) ATRACE(8);
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 w;
          w.x = pack_f16x2_sat(o[i] * e.inv, o[i + 1] * e.inv);
          w.y = pack_f16x2_sat(o[i + 2] * e.inv, o[i + 3] * e.inv);
          w.z = pack_f16x2_sat(o[i + 4] * e.inv, o[i + 5] * e.inv);
          w.w = pack_f16x2_sat(o[i + 6] * e.inv, o[i + 7] * e.inv);
          *reinterpret_cast<uint4*>(stage + lane * 64 + 16 * ((i >> 3) ^ ((lane >> 1) & 3))) = w;
        }
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int rr = k * 8 + (lane >> 2), ch = lane & 3;
          const uint4 w = *reinterpret_cast<const uint4*>(stage + rr * 64 + 16 * (ch ^ ((rr >> 1) & 3)));
          if (rq0 + rr < L)
            *reinterpret_cast<uint4*>(out + (e.row0 + rq0 + rr) * inner + e.h * kDh + c + ch * 8) = w;
        }
        __syncwarp();
        if (lane == 0) ATRACE(9);
      }
      return true;
    };
    Pending pend{0, 0, 0, 0, 0, 0.f};
    bool has_pend = false;
    bool ok = true;
    int t = 0, g = 0;
    for (int round = 0;; ++round) {
      const Item it = il.decode(round);
      if (it.id >= il.n_items) break;
      const size_t row0 = static_cast<size_t>(it.b) * L;
      const int qi = it.q0 + r;
      // Every item passes the named barriers, even after a failed wait, so a
      // timed-out warp can never strand the other softmax warps there.
      if (it.q0 >= it.len) {
        // every query row of this item is padding: zero output rows
        if (qi < L) {
          uint4* dst = reinterpret_cast<uint4*>(out + (row0 + qi) * inner + it.h * kDh);
#pragma unroll
          for (int c = 0; c < kDh / 8; ++c) dst[c] = make_uint4(0, 0, 0, 0);
        }
        continue;
      }
      if (lane == 0) ATRACE(1);
      // bias row of this item (after every softmax thread has finished the
      // previous one's steps)
      if (lane == 0) ATRACE(2);
      asm volatile("bar.sync 1, 128;" ::: "memory");
      {
        const float* tab = sTab + it.h * kMaxBuckets;
        const uint8_t* bk = sBkt + kBktHalf - it.q0 - (kQ - 1);
        for (int x = st; x < it.n_kt * kKeys + kWin; x += 128) {
          const float w = tab[bk[x]];
          sBias[x] = w;
          if (x > 0) sBias[kBiasPad + x - 1] = w;
        }
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (lane == 0) ATRACE(3);
      // bias of key c at brow[c], brow 8-byte aligned
      const float* brow = ((kQ - 1 - r) & 1) ? sBias + kBiasPad + (kQ - 2 - r) : sBias + (kQ - 1 - r);
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = 0; j < it.n_kt; ++j, ++t) {
        const int k0 = j * kKeys;
        if (ok) ok = __all_sync(0xFFFFFFFFu, mbar_wait(&s_full[t & 1], (t >> 1) & 1, status));
        if (lane == 0) ATRACE(4);
        if (ok) {
          tc_fence_after();
          float v[kKeys];
          tmem_ld_32x32b_x32_nowait(trow + kColS + 64 * (t & 1), &v[0]);
          tmem_ld_32x32b_x32_nowait(trow + kColS + 64 * (t & 1) + 32, &v[32]);
          tmem_wait_ld();
          if (lane == 0) ATRACE(17);
          // v = S log2(e) + bias, two lanes per instruction; 4 max chains
          const uint64_t kLog2e2 = f2(1.4426950408889634f, 1.4426950408889634f);
          float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int i = 0; i < kKeys; i += 2) {
            const float2 bb = *reinterpret_cast<const float2*>(brow + k0 + i);
            const uint64_t x = f2_fma(f2(v[i], v[i + 1]), kLog2e2, f2(bb.x, bb.y));
            v[i] = f2_lo(x);
            v[i + 1] = f2_hi(x);
          }
          if (k0 + kKeys > it.len) {
#pragma unroll
            for (int i = 0; i < kKeys; ++i)
              if (k0 + i >= it.len) v[i] = -INFINITY;
          }
#pragma unroll
          for (int i = 0; i < kKeys; i += 2) mx[(i >> 1) & 3] = fmax3(mx[(i >> 1) & 3], v[i], v[i + 1]);
          const float tmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
          // Lazy rescale: keep the running max unless this tile raises it by
          // more than 15 (log2 units), so P stays <= 2^15 (f16 holds up to
          // 65504 at the same relative precision) and O, whose rescale waits
          // for the previous P V, is rescaled rarely; the final division by
          // the matching sum makes it exact.
          const float m_new = (tmax > m_run + 15.0f) ? tmax : m_run;
          const float corr = ex2(m_run - m_new);  // 1 when kept, 0 on the item's first tile
          // p = 2^(v - max) -> f16 P row over the first 32 columns of S buffer
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
          if (lane == 0) ATRACE(19);
          tmem_st_u32_x32(trow + kColS + 64 * (t & 1), pk);
          if (lane == 0) ATRACE(18);
          const uint64_t ps2 = f2_add(f2_add(ps[0], ps[1]), f2_add(ps[2], ps[3]));
          const float psum = f2_lo(ps2) + f2_hi(ps2);
          l_run = l_run * corr + psum;
          m_run = m_new;
          if (j > 0 && __any_sync(0xFFFFFFFFu, corr != 1.0f)) {
            // O holds P(t-1) V(t-1) of this item once o_done says so; rescale
            // it to the new max (rare with the lazy rule above)
            ok = __all_sync(0xFFFFFFFFu, mbar_wait(&o_done[(t - 1) & 1], ((t - 1) >> 1) & 1, status));
            if (ok) {
              tc_fence_after();
              const uint32_t ocol = trow + kColO + 64 * (g & 1);
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
        tmem_wait_st();  // P (and a rescaled O) complete before the MMA thread is told
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t & 1]);
        if (lane == 0) ATRACE(5);
        if (j == 0 && has_pend) {
          // the previous item's P V finished while this step ran; its O
          // buffer is reused by the item after this one, whose first P this
          // thread releases only after these reads
          if (ok) ok = epilogue(pend);
          has_pend = false;
          if (lane == 0) ATRACE(7);
        }
      }
      pend = Pending{row0, it.q0, it.h, t - 1, g, 1.0f / l_run};
      has_pend = true;
      ++g;
    }
    if (has_pend && ok) epilogue(pend);
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  ATRACE_NS(31);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

#ifdef WC_ATTN_TRACE
extern "C" int wc_attn_trace_reset() {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_attn_trace);
  if (e == cudaSuccess) e = cudaMemset(p, 0, sizeof(unsigned long long) * kTraceCtas * kTraceLen);
  return static_cast<int>(e);
}
extern "C" int wc_attn_trace_read(unsigned long long* events, unsigned* counts) {
  (void)counts;
  return static_cast<int>(
      cudaMemcpyFromSymbol(events, g_attn_trace, sizeof(unsigned long long) * kTraceCtas * kTraceLen));
}
#endif

cudaError_t attention_tc_launch(const CUtensorMap& tm_qkv, __half* out, const int32_t* lengths, int B, int L, int H,
                                const float* bias_tab, const BucketThresholds& bt, uint32_t* status,
                                cudaStream_t st) {
  if (B <= 0 || L <= 0) return cudaSuccess;
  if (L > kMaxL || 2 * bt.half > kMaxBuckets || H <= 0 || H > kMaxHeads) return cudaErrorInvalidValue;
  const int64_t n_items = static_cast<int64_t>((L + kQ - 1) / kQ) * B * H;
  if (n_items > INT32_MAX || static_cast<int64_t>(B) * L > INT32_MAX) return cudaErrorInvalidValue;
  static bool attr_set[64] = {};
  static int num_sms[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&num_sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const int grid = static_cast<int>(std::min<int64_t>(n_items, static_cast<int64_t>(kCtasPerSm) * num_sms[dev]));
  return launch_pdl(attention_tc_kernel, dim3(grid), dim3(kThreads), kSmem, st, nullptr, 0, tm_qkv, out, lengths, B, L,
                    H, bias_tab, bt, status);
}

}  // namespace wc
