// Shared device helpers for the sm_100a kernels: mbarriers with bounded waits,
// TMA tiled loads, tcgen05 (TMEM alloc / MMA / commit / ld) wrappers and the
// shared-memory matrix descriptors for K-major 128-byte-swizzled operands.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdlib.h>

#include <utility>

#include <mutex>
#include <set>
#include <utility>

namespace wc {

// Asks once per (device, kernel) for the largest shared-memory carveout, so
// that consecutive kernels of the forward, whatever shared memory each uses,
// run under one SM configuration and the next one can start on an SM before
// the previous one has drained (programmatic dependent launch).
// WC_DEFAULT_CARVEOUT=1 leaves the driver's choice.
inline cudaError_t ensure_max_carveout(const void* func) {
  static const bool on = [] {
    const char* e = getenv("WC_DEFAULT_CARVEOUT");
    return !(e && e[0] == '1');
  }();
  if (!on) return cudaSuccess;
  static std::mutex mu;
  static std::set<std::pair<int, const void*>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({dev, func})) return cudaSuccess;
  e = cudaFuncSetAttribute(func, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (e == cudaSuccess) done.insert({dev, func});
  return e;
}

// Launches kernel on `st` with programmatic stream serialisation (see
// pdl_wait); extra launch attributes (e.g. a cluster shape) may be appended.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              const cudaLaunchAttribute* extra, int n_extra, Args&&... args) {
  if (cudaError_t ce = ensure_max_carveout(reinterpret_cast<const void*>(kernel)); ce != cudaSuccess) return ce;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attrs[4];
  int n = 0;
  // WC_DISABLE_PDL=1 turns the overlap off (griddepcontrol.* are then no-ops).
  static const bool pdl_on = [] {
    const char* e = getenv("WC_DISABLE_PDL");
    return !(e && e[0] == '1');
  }();
  if (pdl_on) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  for (int i = 0; i < n_extra && n < 4; ++i) attrs[n++] = extra[i];
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Status bits a kernel ORs into the per-handle device status word instead of
// trapping.  The host reads the word after each forward and turns a non-zero
// value into an error return.
enum : uint32_t {
  kStatusWaitTimeout = 1u,   // an mbarrier wait ran past its time limit
  kStatusBadArgument = 2u,   // a kernel saw a shape it does not support
  kStatusF16Clipped = 4u,    // an f16 activation store clipped a value (|x| >= 65520 or NaN) to +-65504
};

// Wall-clock limit for any single spin-wait inside a kernel (ns).  A healthy
// pipeline waits microseconds; this only ends a wait that can never finish.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with the given parity.  Returns false (and sets
// kStatusWaitTimeout in *status) if the limit passes first.
__device__ __forceinline__ bool mbar_wait_limit(uint64_t* bar, uint32_t parity, uint32_t* status,
                                                uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 255u && global_timer_ns() - t0 > limit_ns) {
      if (status) atomicOr(status, kStatusWaitTimeout);
      return false;
    }
  }
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* status) {
  return mbar_wait_limit(bar, parity, status, kWaitLimitNs);
}

// ---------------------------------------------------------------- programmatic dependent launch
// Every kernel of the forward is launched with programmatic stream
// serialisation: it lets the next kernel start (pdl_launch_next) right away,
// does only work that touches no activation (barrier init, TMEM allocation,
// descriptor prefetch) and then waits (pdl_wait) for the previous kernel to
// complete and flush before it reads or writes any activation buffer.  So the
// launch latency and prologue of each kernel overlap its predecessor's tail.
__device__ __forceinline__ void pdl_launch_next() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// 2-D tiled load of one box into shared memory, completion signalled on bar.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x,
                                            int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
// Generic-proxy smem writes -> visible to the async proxy (tensor cores, TMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, 16-bit inputs, f32 accumulate, one CTA.
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Same MMA with A read from tensor memory: a_tmem addresses lane 0 of an
// M x K operand whose rows are TMEM lanes and whose 32-bit columns each hold
// two consecutive K elements (low half first).
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on bar when all previously issued tcgen05.mma of this thread finish.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
// 32 lanes x 32 consecutive f32 columns: thread t of the warp gets row (lane
// base + t), columns [col, col+32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor (tcgen05 "UMMA" descriptor) for a K-major
// operand tile stored with the 128-byte swizzle: rows of 64 f16 (128 B),
// 8-row groups 1024 B apart.  Fields: start address >> 4 in [0,14), leading
// byte offset >> 4 in [16,30) (unused for swizzled K-major), stride byte
// offset >> 4 in [32,46), descriptor version 1 in [46,48), layout type in
// [61,64) with 2 = 128-byte swizzle.  The tile base must be 1024-B aligned.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with f16 A/B, f32 D, both K-major
// (A/B format field 0 = f16, 1 = bf16; both operands must share the type).
__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n) {
  return (1u << 4)                                // D format f32
         | (0u << 7)                              // A format f16
         | (0u << 10)                             // B format f16
         | (static_cast<uint32_t>(n >> 3) << 17)  // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24); // M / 16
}

// Physical byte offset of 16-byte chunk `chunk` (0..7) of row `row` inside a
// 128-byte-swizzled K-major tile (the pattern TMA's SWIZZLE_128B writes).
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

// Hardware tanh (MUFU tanh.approx.f32, relative error about 2^-11, the size of
// one f16 rounding of the output it feeds).
__device__ __forceinline__ float tanh_fast(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// GELU, tanh form (candle's NewGelu / HF gelu_new, the XTR "gated-gelu"
// activation): 0.5 g (1 + tanh(sqrt(2/pi) (g + 0.044715 g^3))).
__device__ __forceinline__ float gelu_tanh_fast(float g) {
  return 0.5f * g * (1.0f + tanh_fast(0.7978845608f * (g + 0.044715f * g * g * g)));
}

// Two f32 -> packed f16x2, round to nearest even.
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
// Same, saturating to the finite f16 range (+-65504) so an activation that
// leaves the range stays finite instead of becoming inf (one cvt.satfinite:
// in-range values round exactly as above, larger magnitudes give +-65504).
__device__ __forceinline__ uint32_t pack_f16x2_sat(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// A value the f16 conversion cannot represent: round-to-nearest would give
// inf (|x| >= 65520) or it is NaN.  The saturating stores clip it to +-65504.
__device__ __forceinline__ bool f16_clips(float x) { return !(fabsf(x) < 65520.f); }

// pack_f16x2_sat that also records in `clip` whether either value was clipped.
__device__ __forceinline__ uint32_t pack_f16x2_sat(float lo, float hi, bool& clip) {
  clip |= f16_clips(lo) | f16_clips(hi);
  return pack_f16x2_sat(lo, hi);
}

// Sets kStatusF16Clipped in *status when this thread clipped a value.  The
// flag is read first so a kernel that clips everywhere issues few atomics.
__device__ __forceinline__ void report_f16_clip(bool clip, uint32_t* status) {
  if (clip && status && !(*reinterpret_cast<volatile uint32_t*>(status) & kStatusF16Clipped))
    atomicOr(status, kStatusF16Clipped);
}

// Packed f32x2 arithmetic (one instruction for two lanes of f32 on sm_100).
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  return (static_cast<uint64_t>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// f16x2 of the two f32 lanes, round to nearest even.
__device__ __forceinline__ uint32_t f2_to_h2(uint64_t v) {
  return pack_f16x2(__uint_as_float(static_cast<uint32_t>(v)), __uint_as_float(static_cast<uint32_t>(v >> 32)));
}

__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float f2_hi(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }
// Three-input maximum (one instruction on sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}


}  // namespace wc
