// The encoder handle behind include/wc_t5cuda.h: weight upload, workspaces,
// TMA descriptors and the per-forward launch sequence.
//
// Forward (one padded batch of B sequences x L tokens, M = B*L rows):
//   embed_rmsnorm      x = dequant(embedding rows), xn = RMSNorm_0(x)
//   per layer l:
//     gemm  kEpiF16   qkv = xn . [Wq|Wk|Wv]^T                (f16 [M][3*inner])
//     attention        att = softmax(QK^T + bias, key mask) V (f16 [M][inner])
//     gemm  kEpiResid  x += att . Wo^T  (M >= 512: TMA load-add-store epilogue)
//       (or kEpiF32    y = att . Wo^T into the dead qkv buffer, for small M)
//     rmsnorm          (x += y;) xn = RMSNorm_ff(x)
//     gemm  kEpiGeGLU  h = gelu(xn . Wi0^T) * (xn . Wi1^T)    (f16 [M][d_ff])
//     gemm  kEpiResid  x += h . Wwo^T   (or kEpiF32 + add in the RMSNorm)
//     rmsnorm          xn = RMSNorm_{next attn | final}(x)
//   gemm  kEpiProj     out = xn . Wlin^T, norms, out / norm   (f32 [M][128])
// following T5Stack::forward / T5Block::forward / T5EncoderModel::forward
// (src/quantized_t5.rs:654-670, 598-628, 698-701).  The residual stream x
// stays f32; GEMM and attention operands are f16 with f32 accumulation.
#include <cuda.h>
#include <cuda_runtime.h>
#include <string.h>

#include <map>
#include <mutex>
#include <tuple>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/wc_t5cuda.h"
#include <algorithm>

#include "attention.h"
#include "common.cuh"
#include "elementwise.h"
#include "gemm2_q4k.h"
#include "gemm_q4k.h"
#include "gemv_q4k.h"
#include "t5_host.h"

namespace wc {

namespace {

constexpr int kMaxL = 2048;  // Embedder window (src/embedder.rs:27)

thread_local std::string g_create_error;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

// The calling thread's current CUDA context (the device's primary context
// once the runtime has initialised it), or nullptr.  Per-device caches of
// device addresses key on it: after a cudaDeviceReset the primary context is
// a new one and addresses cached under the old one are stale.
CUcontext current_context() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  CUcontext c = nullptr;
  if (!fn || fn(&c) != CUDA_SUCCESS) return nullptr;
  return c;
}

// f16 activation matrix [rows][K], box 64 x box_rows, 128-byte swizzle.
bool make_act_map(CUtensorMap* m, const void* ptr, uint64_t rows, uint64_t K, uint32_t box_rows = 128) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {K, rows};
  cuuint64_t strides[1] = {K * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t es[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// GEMM output matrix [rows][cols] (f16 or f32) for TMA tensor stores: box of
// 128 bytes x 32 rows, 128-byte swizzle.
bool make_out_map(CUtensorMap* m, const void* ptr, uint64_t rows, uint64_t cols, bool f32) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  const uint64_t esz = f32 ? 4 : 2;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * esz};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / esz), 32};
  cuuint32_t es[2] = {1, 1};
  return enc(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims,
             strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// raw Q4_K matrix [rows][K/256 * 144 bytes], box 144 x box_rows, no swizzle.
bool make_q4k_map(CUtensorMap* m, const void* ptr, uint64_t rows, uint64_t K, uint32_t box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  const uint64_t row_bytes = K / 256 * 144;
  cuuint64_t dims[2] = {row_bytes, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {144, box_rows};
  cuuint32_t es[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct LayerW {
  uint8_t *qkv, *o, *wi0, *wi1, *wo;
  float *ln0, *ln1;
  CUtensorMap tm_qkv, tm_o, tm_wi0, tm_wi1, tm_wo;  // 1-SM kernel boxes
  // The same matrices dequantised once to f16 [N][K] (the large-M GEMMs)
  __half *h_qkv, *h_o, *h_wi0, *h_wi1, *h_wo;
  CUtensorMap tmh_qkv, tmh_o, tmh_wi0, tmh_wi1, tmh_wo;
  // O and wo f16 weights with a 64-row box, for 128-column residual tiles
  CUtensorMap tmh64_o, tmh64_wo;
  // Raw Q4_K rows with the 2-SM kernel's box, for its fused-dequant variant
  // (handles created with WC_F16_WEIGHTS=0)
  CUtensorMap tmq2_qkv, tmq2_o, tmq2_wi0, tmq2_wi1, tmq2_wo;
};

// Rows from which the 2-SM persistent GEMM replaces the 1-SM kernel.
constexpr int kGemm2MinRows = 512;

int device_sm_count(int dev) {
  static int counts[64] = {};
  if (dev < 0 || dev >= 64) return 148;
  if (!counts[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 2) n = 148;
    counts[dev] = n;
  }
  return counts[dev];
}

}  // namespace

}  // namespace wc

struct wc_t5 {
  int device = 0;
  cudaStream_t stream = nullptr;
  wc::T5Config cfg;
  int inner = 0, d_proj = 128;
  int bn_qkv = 0, bn_o = 0, bn_wi = 0, bn_wo = 0;
  uint8_t* arena = nullptr;  // all weights, one allocation
  __half* arena_f16 = nullptr;  // the layer matrices dequantised to f16, one allocation
  // Large-M GEMMs on the resident f16 copies (default) or, with
  // WC_F16_WEIGHTS=0 at create time, dequantising the Q4_K rows in the kernel
  bool f16_weights = true;
  uint8_t* embed = nullptr;
  uint8_t* proj = nullptr;
  float* final_ln = nullptr;
  float* rel_bias = nullptr;
  wc::BucketThresholds bt{};
  std::vector<wc::LayerW> layers;
  CUtensorMap tm_proj;
  // workspaces (capacity in rows)
  int64_t cap_rows = 0;
  int cap_b = 0;
  uint8_t* ws = nullptr;
  float* x = nullptr;
  __half *xn = nullptr, *qkv = nullptr, *att = nullptr, *hbuf = nullptr;
  CUtensorMap tm_xn, tm_att, tm_h;
  // host-API staging
  uint32_t* d_ids = nullptr;
  int32_t* d_len = nullptr;
  float *d_out = nullptr, *d_norms = nullptr, *d_outn = nullptr;
  uint32_t* d_status = nullptr;
  // wc_t5_forward_many: two I/O buffer sets (ids, lengths, out, norms), a copy
  // stream and its events, created on first use
  uint8_t* io = nullptr;
  int64_t io_rows = 0;
  int io_b = 0;
  uint32_t* io_ids[2] = {};
  int32_t* io_len[2] = {};
  float *io_out[2] = {}, *io_norms[2] = {};
  cudaStream_t copy_stream = nullptr;
  cudaEvent_t ev_in[2] = {}, ev_fwd[2] = {}, ev_out[2] = {};
  // wc_t5_forward_many's second compute lane for large batches: odd batches
  // run on their own stream with their own activation buffers, so one
  // batch's memory-bound kernels (RMSNorm, attention) share the SMs with the
  // other's GEMMs; created on first use
  cudaStream_t lane_stream = nullptr;
  cudaEvent_t ev_lane = nullptr;
  uint8_t* lane_ws = nullptr;
  int64_t lane_rows = 0;
  float* lane_x = nullptr;
  __half *lane_xn = nullptr, *lane_qkv = nullptr, *lane_att = nullptr, *lane_h = nullptr;
  CUtensorMap lane_tm_xn, lane_tm_att, lane_tm_h;
  // CUDA graphs of the kernel sequence for small batches, keyed by shape,
  // buffers and stream; an entry first records that the key was seen and is
  // captured on its second use.
  struct GraphKey {
    int B, L;
    const void *ids, *len, *out, *norms, *outn;
    cudaStream_t st;
    bool operator<(const GraphKey& o) const {
      return std::tie(B, L, ids, len, out, norms, outn, st) < std::tie(o.B, o.L, o.ids, o.len, o.out, o.norms, o.outn, o.st);
    }
  };
  std::map<GraphKey, cudaGraphExec_t> graphs;  // nullptr = seen once, not captured
  std::string err;
};

namespace wc {
namespace {

int fail(wc_t5* h, int code, const std::string& msg) {
  if (h)
    h->err = msg;
  else
    g_create_error = msg;
  return code;
}

int cuda_fail(wc_t5* h, cudaError_t e, const char* what) {
  return fail(h, WC_E_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

void clear_graphs(wc_t5* h) {
  for (auto& kv : h->graphs)
    if (kv.second) cudaGraphExecDestroy(kv.second);
  h->graphs.clear();
}

void free_workspace(wc_t5* h) {
  clear_graphs(h);  // captured graphs hold workspace pointers
  if (h->ws) cudaFree(h->ws);
  h->ws = nullptr;
  h->cap_rows = 0;
  h->cap_b = 0;
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

int ensure_workspace(wc_t5* h, int64_t rows, int B) {
  if (rows <= h->cap_rows && B <= h->cap_b) return WC_OK;
  const int64_t cap = std::max<int64_t>((rows + 127) / 128 * 128, h->cap_rows);
  // B <= rows always (L >= 1): size the lengths for `cap` rows so a batch of
  // many short rows never reallocates the workspace on its own
  const int capb = static_cast<int>(std::max<int64_t>({cap, static_cast<int64_t>(B), h->cap_b}));
  free_workspace(h);
  const int D = h->cfg.d_model, F = h->cfg.d_ff, I = h->inner, P = h->d_proj;
  size_t off = 0;
  const size_t o_x = off; off = align256(off + cap * D * 4);
  const size_t o_xn = off; off = align256(off + cap * D * 2);
  const size_t o_qkv = off; off = align256(off + cap * std::max(3 * I * 2, D * 4));  // also the f32 O / wo output
  const size_t o_att = off; off = align256(off + cap * I * 2);
  const size_t o_h = off; off = align256(off + cap * F * 2);
  const size_t o_ids = off; off = align256(off + cap * 4);
  const size_t o_len = off; off = align256(off + capb * 4);
  const size_t o_out = off; off = align256(off + cap * P * 4);
  const size_t o_norms = off; off = align256(off + cap * 4);
  const size_t o_outn = off; off = align256(off + cap * P * 4);
  cudaError_t e = cudaMalloc(&h->ws, off);
  if (e != cudaSuccess) {
    h->ws = nullptr;
    return cuda_fail(h, e, "workspace allocation");
  }
  h->x = reinterpret_cast<float*>(h->ws + o_x);
  h->xn = reinterpret_cast<__half*>(h->ws + o_xn);
  h->qkv = reinterpret_cast<__half*>(h->ws + o_qkv);
  h->att = reinterpret_cast<__half*>(h->ws + o_att);
  h->hbuf = reinterpret_cast<__half*>(h->ws + o_h);
  h->d_ids = reinterpret_cast<uint32_t*>(h->ws + o_ids);
  h->d_len = reinterpret_cast<int32_t*>(h->ws + o_len);
  h->d_out = reinterpret_cast<float*>(h->ws + o_out);
  h->d_norms = reinterpret_cast<float*>(h->ws + o_norms);
  h->d_outn = reinterpret_cast<float*>(h->ws + o_outn);
  if (!make_act_map(&h->tm_xn, h->xn, cap, D) || !make_act_map(&h->tm_att, h->att, cap, I) ||
      !make_act_map(&h->tm_h, h->hbuf, cap, F))
    return fail(h, WC_E_CUDA, "cuTensorMapEncodeTiled failed for an activation buffer");
  h->cap_rows = cap;
  h->cap_b = capb;
  return WC_OK;
}

int gemm(wc_t5* h, int epi, int bn, const CUtensorMap& a, const CUtensorMap& w0, const CUtensorMap& w1, int M,
         int N, int K, void* out, int ldo, cudaStream_t st, float* norms = nullptr, float* outn = nullptr,
         const int32_t* lengths = nullptr, int L = 0) {
  GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.out = out;
  p.ldo = ldo;
  p.norms = norms;
  p.out_normalised = outn;
  p.lengths = lengths;
  p.L = L;
  p.status = h->d_status;
  cudaError_t e = gemm_q4k_launch(epi, bn, a, w0, w1, p, st);
  return e == cudaSuccess ? WC_OK : cuda_fail(h, e, "GEMM launch");
}

// Layer GEMM: the 2-SM persistent kernel for large M (on the resident f16
// weights, w0_2 / w1_2), else the 1-SM kernel on the Q4_K rows.
// Up to kGemvMaxRows rows the small-M kernel (all SMs stream the weights once)
// runs instead; it reads the activations and the raw weights by pointer.
int layer_gemm(wc_t5* h, int epi, int bn, const CUtensorMap& a, const CUtensorMap& w0, const CUtensorMap& w1,
               const CUtensorMap& w0_2, const CUtensorMap& w1_2, int M, int N, int K, void* out, int ldo,
               cudaStream_t st, const __half* a_ptr, const uint8_t* w0_ptr, const uint8_t* w1_ptr,
               const CUtensorMap* w_narrow = nullptr) {
  const int feat = epi == kEpiGeGLU ? N / 2 : N;
  if (gemv_q4k_supports(epi, M, feat, K)) {
    cudaError_t e = gemv_q4k_launch(epi, a_ptr, M, K, w0_ptr, w1_ptr, feat, out, ldo, h->d_status, st);
    return e == cudaSuccess ? WC_OK : cuda_fail(h, e, "GEMM launch");
  }
  if (M >= kGemm2MinRows && gemm2_q4k_supports(epi, M, N, K)) {
    GemmParams p{};
    p.M = M;
    p.N = N;
    p.K = K;
    p.out = out;
    p.ldo = ldo;
    p.status = h->d_status;
    CUtensorMap tm_out;
    if (!make_out_map(&tm_out, out, M, ldo, epi == kEpiF32 || epi == kEpiResid))
      return fail(h, WC_E_CUDA, "cuTensorMapEncodeTiled failed for a GEMM output");
    // 128-column tiles for the residual GEMMs when their cluster rounds are
    // shorter in total than with 256-column tiles
    const int sms = device_sm_count(h->device);
    const bool narrow = w_narrow && h->f16_weights && epi == kEpiResid && gemm2_resid_bn(M, N, sms) == 128;
    cudaError_t e = narrow ? gemm2_q4k_launch(epi, a, *w_narrow, *w_narrow, tm_out, p, sms, st, true, 128)
                           : gemm2_q4k_launch(epi, a, w0_2, w1_2, tm_out, p, sms, st, h->f16_weights);
    return e == cudaSuccess ? WC_OK : cuda_fail(h, e, "GEMM launch");
  }
  return gemm(h, epi, bn, a, w0, w1, M, N, K, out, ldo, st);
}

int forward_on(wc_t5* h, float* x, __half* xn, __half* qkv, __half* att, __half* hbuf, const CUtensorMap& tm_xn,
               const CUtensorMap& tm_att, const CUtensorMap& tm_h, const uint32_t* ids, const int32_t* lengths,
               int B, int L, float* out, float* norms, float* outn, cudaStream_t st);

int forward_device(wc_t5* h, const uint32_t* ids, const int32_t* lengths, int B, int L, float* out, float* norms,
                   float* outn, cudaStream_t st) {
  return forward_on(h, h->x, h->xn, h->qkv, h->att, h->hbuf, h->tm_xn, h->tm_att, h->tm_h, ids, lengths, B, L, out,
                    norms, outn, st);
}

int check_status(wc_t5* h, cudaStream_t st) {
  uint32_t s = 0;
  cudaError_t e = cudaMemcpyAsync(&s, h->d_status, 4, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(h, e, "synchronising the forward");
  if (s & kStatusWaitTimeout) return fail(h, WC_E_TIMEOUT, "an in-kernel wait timed out");
  if (s & ~kStatusF16Clipped) return fail(h, WC_E_CUDA, "kernel reported status " + std::to_string(s));
  if (s & kStatusF16Clipped)
    return fail(h, WC_W_F16_CLIPPED,
                "an f16 activation exceeded the f16 range and was clipped to +-65504; the outputs may deviate "
                "from the f32 reference");
  return WC_OK;
}

// Batches up to this many rows replay a captured CUDA graph of the ~86
// launches instead of launching them one by one (launch overhead dominates a
// 32-token query).
constexpr int64_t kGraphMaxRows = 4096;

int forward_cached(wc_t5* h, const uint32_t* ids, const int32_t* lengths, int B, int L, float* out, float* norms,
                   float* outn, cudaStream_t st) {
  const int64_t M = static_cast<int64_t>(B) * L;
  if (M > kGraphMaxRows || st == nullptr || st == cudaStreamLegacy || st == cudaStreamPerThread)
    return forward_device(h, ids, lengths, B, L, out, norms, outn, st);
  const wc_t5::GraphKey key{B, L, ids, lengths, out, norms, outn, st};
  auto it = h->graphs.find(key);
  if (it != h->graphs.end() && it->second) {
    cudaError_t e = cudaGraphLaunch(it->second, st);
    return e == cudaSuccess ? WC_OK : cuda_fail(h, e, "graph launch");
  }
  if (it == h->graphs.end()) {
    if (h->graphs.size() >= 256) clear_graphs(h);
    h->graphs[key] = nullptr;  // seen once: run eagerly
    return forward_device(h, ids, lengths, B, L, out, norms, outn, st);
  }
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) return cuda_fail(h, e, "graph capture begin");
  const int rc = forward_device(h, ids, lengths, B, L, out, norms, outn, st);
  e = cudaStreamEndCapture(st, &graph);
  if (rc != WC_OK || e != cudaSuccess) {
    if (graph) cudaGraphDestroy(graph);
    h->graphs.erase(key);
    return rc != WC_OK ? rc : cuda_fail(h, e, "graph capture");
  }
  cudaGraphExec_t exec = nullptr;
  e = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) {
    h->graphs.erase(key);
    return cuda_fail(h, e, "graph instantiate");
  }
  h->graphs[key] = exec;
  e = cudaGraphLaunch(exec, st);
  return e == cudaSuccess ? WC_OK : cuda_fail(h, e, "graph launch");
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

}  // namespace
}  // namespace wc

using namespace wc;

extern "C" int wc_t5_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

extern "C" const char* wc_t5_last_error(const wc_t5* h) { return h ? h->err.c_str() : g_create_error.c_str(); }

extern "C" int wc_t5_destroy(wc_t5* h) {
  if (!h) return WC_OK;
  {
    DeviceGuard g(h->device);
    if (h->stream) cudaStreamSynchronize(h->stream);
    free_workspace(h);
    if (h->arena) cudaFree(h->arena);
    if (h->arena_f16) cudaFree(h->arena_f16);
    if (h->copy_stream) cudaStreamSynchronize(h->copy_stream);
    if (h->io) cudaFree(h->io);
    for (int i = 0; i < 2; ++i) {
      if (h->ev_in[i]) cudaEventDestroy(h->ev_in[i]);
      if (h->ev_fwd[i]) cudaEventDestroy(h->ev_fwd[i]);
      if (h->ev_out[i]) cudaEventDestroy(h->ev_out[i]);
    }
    if (h->copy_stream) cudaStreamDestroy(h->copy_stream);
    if (h->lane_stream) {
      cudaStreamSynchronize(h->lane_stream);
      cudaStreamDestroy(h->lane_stream);
    }
    if (h->ev_lane) cudaEventDestroy(h->ev_lane);
    if (h->lane_ws) cudaFree(h->lane_ws);
    if (h->d_status) cudaFree(h->d_status);
    if (h->stream) cudaStreamDestroy(h->stream);
  }
  delete h;
  return WC_OK;
}

extern "C" int wc_t5_create(int device_ordinal, const uint8_t* gguf, size_t gguf_len, const char* config_json,
                            wc_t5** out) {
  if (!out) return fail(nullptr, WC_E_INVALID_ARG, "out is NULL");
  *out = nullptr;
  T5Config cfg;
  std::string err;
  if (!config_parse(config_json, &cfg, &err)) return fail(nullptr, WC_E_CONFIG, err);
  if (!cfg.gated_gelu)
    return fail(nullptr, WC_E_UNSUPPORTED, "only the gated-gelu feed-forward (XTR / T5 v1.1) is supported");
  if (cfg.d_kv != 64) return fail(nullptr, WC_E_UNSUPPORTED, "d_kv must be 64");
  if (cfg.d_model % 256 || cfg.d_model > 1024 || cfg.d_ff % 256 || (cfg.num_heads * 64) % 256 ||
      cfg.num_layers < 1 || cfg.num_buckets < 2 || cfg.num_buckets > 32 || cfg.vocab_size < 1)
    return fail(nullptr, WC_E_UNSUPPORTED, "unsupported model dimensions in config.json");
  std::unordered_map<std::string, GgufTensor> t;
  if (!gguf_parse(gguf, gguf_len, &t, &err)) return fail(nullptr, WC_E_GGUF, err);

  const int D = cfg.d_model, F = cfg.d_ff, I = cfg.num_heads * 64;
  auto get = [&](const std::string& name, uint64_t rows, uint64_t cols, bool q4k, const GgufTensor** o) -> int {
    auto it = t.find(name);
    if (it == t.end()) return fail(nullptr, WC_E_GGUF, "GGUF has no tensor " + name);
    const GgufTensor& g = it->second;
    if (g.rows() != rows || g.cols() != cols || g.dims.size() > 2)
      return fail(nullptr, WC_E_UNSUPPORTED,
                  "tensor " + name + " has shape [" + std::to_string(g.rows()) + ", " + std::to_string(g.cols()) +
                      "], expected [" + std::to_string(rows) + ", " + std::to_string(cols) + "]");
    if (q4k && g.type != kGgmlQ4K) return fail(nullptr, WC_E_UNSUPPORTED, "tensor " + name + " is not Q4_K");
    if (!q4k && g.type != kGgmlF32 && g.type != kGgmlF16)
      return fail(nullptr, WC_E_UNSUPPORTED, "tensor " + name + " is not F32/F16");
    *o = &g;
    return WC_OK;
  };
  // the shared embedding: shared.weight, else encoder.embed_tokens.weight (src/quantized_t5.rs:682-687)
  const char* emb_name = t.count("shared.weight") ? "shared.weight" : "encoder.embed_tokens.weight";
  const GgufTensor *g_emb, *g_proj, *g_fln, *g_bias;
  int rc;
  if ((rc = get(emb_name, cfg.vocab_size, D, true, &g_emb))) return rc;
  auto it_proj = t.find("linear.weight");
  if (it_proj == t.end()) return fail(nullptr, WC_E_GGUF, "GGUF has no tensor linear.weight");
  if ((rc = get("linear.weight", 128, D, true, &g_proj))) return rc;
  if ((rc = get("encoder.final_layer_norm.weight", 1, D, false, &g_fln))) return rc;
  if ((rc = get("encoder.block.0.layer.0.SelfAttention.relative_attention_bias.weight", cfg.num_buckets,
                cfg.num_heads, false, &g_bias)))
    return rc;
  struct LT {
    const GgufTensor *q, *k, *v, *o, *wi0, *wi1, *wo, *ln0, *ln1;
  };
  std::vector<LT> lt(cfg.num_layers);
  for (int l = 0; l < cfg.num_layers; ++l) {
    const std::string p = "encoder.block." + std::to_string(l) + ".layer.";
    if ((rc = get(p + "0.SelfAttention.q.weight", I, D, true, &lt[l].q)) ||
        (rc = get(p + "0.SelfAttention.k.weight", I, D, true, &lt[l].k)) ||
        (rc = get(p + "0.SelfAttention.v.weight", I, D, true, &lt[l].v)) ||
        (rc = get(p + "0.SelfAttention.o.weight", D, I, true, &lt[l].o)) ||
        (rc = get(p + "0.layer_norm.weight", 1, D, false, &lt[l].ln0)) ||
        (rc = get(p + "1.DenseReluDense.wi_0.weight", F, D, true, &lt[l].wi0)) ||
        (rc = get(p + "1.DenseReluDense.wi_1.weight", F, D, true, &lt[l].wi1)) ||
        (rc = get(p + "1.DenseReluDense.wo.weight", D, F, true, &lt[l].wo)) ||
        (rc = get(p + "1.layer_norm.weight", 1, D, false, &lt[l].ln1)))
      return rc;
  }

  // Dequantised weights are tensor-core operands in f16: refuse checkpoints
  // whose Q4_K scales could produce values outside the f16 range.
  {
    std::vector<const GgufTensor*> gemm_w = {g_proj};
    for (auto& x : lt) gemm_w.insert(gemm_w.end(), {x.q, x.k, x.v, x.o, x.wi0, x.wi1, x.wo});
    for (const GgufTensor* g : gemm_w) {
      const double b = q4k_max_abs_bound(g->data, g->nbytes / 144);
      if (!(b <= 65504.0))
        return fail(nullptr, WC_E_UNSUPPORTED, "tensor " + g->name + " has Q4_K scales outside the f16 operand range");
    }
  }
  int ndev = wc_t5_device_count();
  if (device_ordinal < 0 || device_ordinal >= ndev)
    return fail(nullptr, WC_E_CUDA,
                "CUDA device " + std::to_string(device_ordinal) + " not available (" + std::to_string(ndev) +
                    " visible)");
  if (!get_encode_fn()) return fail(nullptr, WC_E_CUDA, "cuTensorMapEncodeTiled is not available from the driver");

  wc_t5* h = new wc_t5();
  h->device = device_ordinal;
  h->cfg = cfg;
  h->inner = I;
  DeviceGuard guard(device_ordinal);
  cudaError_t e;
  int dmaj = 0;
  cudaDeviceGetAttribute(&dmaj, cudaDevAttrComputeCapabilityMajor, device_ordinal);
  if (dmaj != 10) {
    delete h;
    return fail(nullptr, WC_E_UNSUPPORTED, "this backend is built for sm_100a (B200); device has compute capability major " + std::to_string(dmaj));
  }
  if ((e = cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking)) != cudaSuccess ||
      (e = cudaMalloc(&h->d_status, 4)) != cudaSuccess) {
    std::string m = std::string("stream/status allocation: ") + cudaGetErrorString(e);
    wc_t5_destroy(h);
    return fail(nullptr, WC_E_CUDA, m);
  }
  cudaMemset(h->d_status, 0, 4);

  // ---- weight arena layout
  const size_t row_q4k_D = D / 256 * 144, row_q4k_F = F / 256 * 144, row_q4k_I = I / 256 * 144;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  const size_t o_emb = take(g_emb->nbytes);
  const size_t o_proj = take(g_proj->nbytes);
  const size_t o_fln = take(D * 4);
  const size_t o_bias = take(cfg.num_buckets * cfg.num_heads * 4);
  struct LO {
    size_t qkv, o, wi0, wi1, wo, ln0, ln1;
  };
  std::vector<LO> lo(cfg.num_layers);
  for (int l = 0; l < cfg.num_layers; ++l) {
    lo[l].qkv = take(3 * I * row_q4k_D);
    lo[l].o = take(D * row_q4k_I);
    lo[l].wi0 = take(F * row_q4k_D);
    lo[l].wi1 = take(F * row_q4k_D);
    lo[l].wo = take(D * row_q4k_F);
    lo[l].ln0 = take(D * 4);
    lo[l].ln1 = take(D * 4);
  }
  std::vector<uint8_t> host(off, 0);
  auto put_f32 = [&](size_t o, const GgufTensor* g) {
    float* dst = reinterpret_cast<float*>(host.data() + o);
    const size_t n = g->rows() * g->cols();
    if (g->type == kGgmlF32) {
      memcpy(dst, g->data, n * 4);
    } else {  // F16 -> F32
      for (size_t i = 0; i < n; ++i) {
        uint16_t hb;
        memcpy(&hb, g->data + 2 * i, 2);
        __half_raw hr;
        hr.x = hb;
        dst[i] = __half2float(__half(hr));
      }
    }
  };
  memcpy(host.data() + o_emb, g_emb->data, g_emb->nbytes);
  memcpy(host.data() + o_proj, g_proj->data, g_proj->nbytes);
  put_f32(o_fln, g_fln);
  put_f32(o_bias, g_bias);
  for (int l = 0; l < cfg.num_layers; ++l) {
    // q | k | v rows concatenated: raw super-blocks copied unchanged
    memcpy(host.data() + lo[l].qkv, lt[l].q->data, lt[l].q->nbytes);
    memcpy(host.data() + lo[l].qkv + lt[l].q->nbytes, lt[l].k->data, lt[l].k->nbytes);
    memcpy(host.data() + lo[l].qkv + 2 * lt[l].q->nbytes, lt[l].v->data, lt[l].v->nbytes);
    memcpy(host.data() + lo[l].o, lt[l].o->data, lt[l].o->nbytes);
    memcpy(host.data() + lo[l].wi0, lt[l].wi0->data, lt[l].wi0->nbytes);
    memcpy(host.data() + lo[l].wi1, lt[l].wi1->data, lt[l].wi1->nbytes);
    memcpy(host.data() + lo[l].wo, lt[l].wo->data, lt[l].wo->nbytes);
    put_f32(lo[l].ln0, lt[l].ln0);
    put_f32(lo[l].ln1, lt[l].ln1);
  }
  if ((e = cudaMalloc(&h->arena, off)) != cudaSuccess ||
      (e = cudaMemcpy(h->arena, host.data(), off, cudaMemcpyHostToDevice)) != cudaSuccess) {
    std::string m = std::string("weight upload: ") + cudaGetErrorString(e);
    wc_t5_destroy(h);
    return fail(nullptr, WC_E_CUDA, m);
  }
  h->embed = h->arena + o_emb;
  h->proj = h->arena + o_proj;
  h->final_ln = reinterpret_cast<float*>(h->arena + o_fln);
  h->rel_bias = reinterpret_cast<float*>(h->arena + o_bias);
  h->bt = t5_bucket_thresholds(cfg.num_buckets, cfg.max_distance, kMaxL);
  h->bn_qkv = gemm_q4k_bn_for(kEpiF16, 3 * I);
  h->bn_o = gemm_q4k_bn_for(kEpiF32, D);
  h->bn_wi = gemm_q4k_bn_for(kEpiGeGLU, 2 * F);
  h->bn_wo = gemm_q4k_bn_for(kEpiF32, D);
  if (h->bn_qkv < 0 || h->bn_o < 0 || h->bn_wi < 0 || h->bn_wo < 0) {
    wc_t5_destroy(h);
    return fail(nullptr, WC_E_UNSUPPORTED, "no GEMM tiling for these model dimensions");
  }
  bool ok = make_q4k_map(&h->tm_proj, h->proj, 128, D, 128);
  h->layers.resize(cfg.num_layers);
  for (int l = 0; l < cfg.num_layers && ok; ++l) {
    LayerW& w = h->layers[l];
    w.qkv = h->arena + lo[l].qkv;
    w.o = h->arena + lo[l].o;
    w.wi0 = h->arena + lo[l].wi0;
    w.wi1 = h->arena + lo[l].wi1;
    w.wo = h->arena + lo[l].wo;
    w.ln0 = reinterpret_cast<float*>(h->arena + lo[l].ln0);
    w.ln1 = reinterpret_cast<float*>(h->arena + lo[l].ln1);
    ok = make_q4k_map(&w.tm_qkv, w.qkv, 3 * I, D, gemm_q4k_w_box_rows(kEpiF16, h->bn_qkv)) &&
         make_q4k_map(&w.tm_o, w.o, D, I, gemm_q4k_w_box_rows(kEpiF32, h->bn_o)) &&
         make_q4k_map(&w.tm_wi0, w.wi0, F, D, gemm_q4k_w_box_rows(kEpiGeGLU, h->bn_wi)) &&
         make_q4k_map(&w.tm_wi1, w.wi1, F, D, gemm_q4k_w_box_rows(kEpiGeGLU, h->bn_wi)) &&
         make_q4k_map(&w.tm_wo, w.wo, D, F, gemm_q4k_w_box_rows(kEpiF32, h->bn_wo)) &&
         make_q4k_map(&w.tmq2_qkv, w.qkv, 3 * I, D, kGemm2WBoxRows) &&
         make_q4k_map(&w.tmq2_o, w.o, D, I, kGemm2WBoxRows) &&
         make_q4k_map(&w.tmq2_wi0, w.wi0, F, D, kGemm2WBoxRows) &&
         make_q4k_map(&w.tmq2_wi1, w.wi1, F, D, kGemm2WBoxRows) &&
         make_q4k_map(&w.tmq2_wo, w.wo, D, F, kGemm2WBoxRows);
  }
  if (!ok) {
    wc_t5_destroy(h);
    return fail(nullptr, WC_E_CUDA, "cuTensorMapEncodeTiled failed for a weight tensor");
  }
  // Resident f16 copies of the layer matrices for the large-M GEMMs: the
  // reference dequantises its Q4_K weights once at load, and so does this,
  // with the rounding to f16 the fused-dequant kernels apply to their operands.
  {
    const char* fw = getenv("WC_F16_WEIGHTS");
    h->f16_weights = !(fw && fw[0] == '0' && fw[1] == 0);
  }
  if (h->f16_weights) {
    const int64_t per_layer = (3 * static_cast<int64_t>(I) * D + static_cast<int64_t>(D) * I +
                               2 * static_cast<int64_t>(F) * D + static_cast<int64_t>(D) * F);
    if ((e = cudaMalloc(&h->arena_f16, per_layer * cfg.num_layers * sizeof(__half))) != cudaSuccess) {
      std::string m = std::string("f16 weights: ") + cudaGetErrorString(e);
      wc_t5_destroy(h);
      return fail(nullptr, WC_E_CUDA, m);
    }
    __half* hp = h->arena_f16;
    auto deq = [&](const uint8_t* q4k, int64_t rows, int64_t K, __half*& dst) -> bool {
      dst = hp;
      hp += rows * K;
      return q4k_dequant_f16_launch(q4k, rows * K / 256, dst, h->stream) == cudaSuccess;
    };
    for (int l = 0; l < cfg.num_layers && ok; ++l) {
      LayerW& w = h->layers[l];
      ok = deq(w.qkv, 3 * I, D, w.h_qkv) && deq(w.o, D, I, w.h_o) && deq(w.wi0, F, D, w.h_wi0) &&
           deq(w.wi1, F, D, w.h_wi1) && deq(w.wo, D, F, w.h_wo) &&
           make_act_map(&w.tmh_qkv, w.h_qkv, 3 * I, D, kGemm2WBoxRows) &&
           make_act_map(&w.tmh_o, w.h_o, D, I, kGemm2WBoxRows) &&
           make_act_map(&w.tmh_wi0, w.h_wi0, F, D, kGemm2WBoxRows) &&
           make_act_map(&w.tmh_wi1, w.h_wi1, F, D, kGemm2WBoxRows) &&
           make_act_map(&w.tmh_wo, w.h_wo, D, F, kGemm2WBoxRows) &&
           make_act_map(&w.tmh64_o, w.h_o, D, I, 64) && make_act_map(&w.tmh64_wo, w.h_wo, D, F, 64);
    }
    if (ok) ok = cudaStreamSynchronize(h->stream) == cudaSuccess;
    if (!ok) {
      wc_t5_destroy(h);
      return fail(nullptr, WC_E_CUDA, "dequantising the f16 layer weights failed");
    }
  }
  *out = h;
  return WC_OK;
}

extern "C" int wc_t5_dims(const wc_t5* h, int* d_model, int* n_layers, int* d_proj, int* vocab) {
  if (!h) return WC_E_INVALID_ARG;
  if (d_model) *d_model = h->cfg.d_model;
  if (n_layers) *n_layers = h->cfg.num_layers;
  if (d_proj) *d_proj = h->d_proj;
  if (vocab) *vocab = h->cfg.vocab_size;
  return WC_OK;
}

extern "C" int wc_t5_forward_device(wc_t5* h, const uint32_t* d_ids, const int32_t* d_lengths, int B, int L,
                                    float* d_out, float* d_norms, float* d_outn, void* stream) {
  if (!h) return WC_E_INVALID_ARG;
  if (!d_ids || !d_lengths || !d_out || B < 1 || L < 1 || L > kMaxL || static_cast<int64_t>(B) * L > (1 << 26))
    return fail(h, WC_E_INVALID_ARG, "invalid ids/lengths/out pointer or B, L out of range (1 <= L <= 2048)");
  DeviceGuard g(h->device);
  int rc = ensure_workspace(h, static_cast<int64_t>(B) * L, B);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(h->d_status, 0, 4, st);
  if (e != cudaSuccess) return cuda_fail(h, e, "status reset");
  return forward_cached(h, d_ids, d_lengths, B, L, d_out, d_norms, d_outn, st);
}

extern "C" int wc_t5_sync(wc_t5* h, void* stream) {
  if (!h) return WC_E_INVALID_ARG;
  DeviceGuard g(h->device);
  return check_status(h, static_cast<cudaStream_t>(stream));
}

extern "C" int wc_t5_forward(wc_t5* h, const uint32_t* ids, const int32_t* lengths, int B, int L, float* out,
                             float* norms, float* out_normalised) {
  if (!h) return WC_E_INVALID_ARG;
  if (!ids || !out || B < 1 || L < 1 || L > kMaxL || static_cast<int64_t>(B) * L > (1 << 26))
    return fail(h, WC_E_INVALID_ARG, "invalid ids/out pointer or B, L out of range (1 <= L <= 2048)");
  std::vector<int32_t> len(B, L);
  if (lengths) {
    for (int b = 0; b < B; ++b) {
      if (lengths[b] < 1 || lengths[b] > L)
        return fail(h, WC_E_INVALID_ARG, "lengths[" + std::to_string(b) + "] is outside [1, L]");
      len[b] = lengths[b];
    }
  }
  for (int b = 0; b < B; ++b)
    for (int i = 0; i < len[b]; ++i)
      if (ids[static_cast<size_t>(b) * L + i] >= static_cast<uint32_t>(h->cfg.vocab_size))
        return fail(h, WC_E_INVALID_ARG, "token id " + std::to_string(ids[static_cast<size_t>(b) * L + i]) +
                                             " is not below vocab_size " + std::to_string(h->cfg.vocab_size));
  DeviceGuard g(h->device);
  const int64_t M = static_cast<int64_t>(B) * L;
  int rc = ensure_workspace(h, M, B);
  if (rc) return rc;
  cudaStream_t st = h->stream;
  cudaError_t e;
  if ((e = cudaMemsetAsync(h->d_status, 0, 4, st)) != cudaSuccess ||
      (e = cudaMemcpyAsync(h->d_ids, ids, M * 4, cudaMemcpyHostToDevice, st)) != cudaSuccess ||
      (e = cudaMemcpyAsync(h->d_len, len.data(), B * 4, cudaMemcpyHostToDevice, st)) != cudaSuccess)
    return cuda_fail(h, e, "input upload");
  rc = forward_cached(h, h->d_ids, h->d_len, B, L, h->d_out, norms ? h->d_norms : nullptr,
                      out_normalised ? h->d_outn : nullptr, st);
  if (rc) return rc;
  const size_t ob = static_cast<size_t>(M) * h->d_proj * 4;
  if ((e = cudaMemcpyAsync(out, h->d_out, ob, cudaMemcpyDeviceToHost, st)) != cudaSuccess ||
      (norms && (e = cudaMemcpyAsync(norms, h->d_norms, M * 4, cudaMemcpyDeviceToHost, st)) != cudaSuccess) ||
      (out_normalised &&
       (e = cudaMemcpyAsync(out_normalised, h->d_outn, ob, cudaMemcpyDeviceToHost, st)) != cudaSuccess))
    return cuda_fail(h, e, "output download");
  return check_status(h, st);
}

// ---------------------------------------------------------------- kernel-level entry points

namespace {
uint32_t* kernel_status_word() {
  // One status word per device for the kernel-level entry points, allocated
  // again when the device's context is not the one it was allocated in (the
  // device was reset in between).
  static uint32_t* words[64] = {};
  static CUcontext ctxs[64] = {};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  cudaFree(nullptr);  // make the device's primary context current
  const CUcontext ctx = current_context();
  std::lock_guard<std::mutex> lk(mu);
  if (!words[dev] || ctxs[dev] != ctx) {
    words[dev] = nullptr;
    if (cudaMalloc(&words[dev], 4) != cudaSuccess) return nullptr;
    cudaMemset(words[dev], 0, 4);
    ctxs[dev] = ctx;
  }
  return words[dev];
}
}  // namespace

namespace wc {
namespace {

// Validates one host batch like wc_t5_forward and fills its lengths.
int check_batch(wc_t5* h, const uint32_t* ids, const int32_t* lengths, int B, int L, const float* out,
                std::vector<int32_t>& len) {
  if (!ids || !out || B < 1 || L < 1 || L > kMaxL || static_cast<int64_t>(B) * L > (1 << 26))
    return fail(h, WC_E_INVALID_ARG, "invalid ids/out pointer or B, L out of range (1 <= L <= 2048)");
  len.assign(B, L);
  if (lengths) {
    for (int b = 0; b < B; ++b) {
      if (lengths[b] < 1 || lengths[b] > L)
        return fail(h, WC_E_INVALID_ARG, "lengths[" + std::to_string(b) + "] is outside [1, L]");
      len[b] = lengths[b];
    }
  }
  for (int b = 0; b < B; ++b)
    for (int i = 0; i < len[b]; ++i)
      if (ids[static_cast<size_t>(b) * L + i] >= static_cast<uint32_t>(h->cfg.vocab_size))
        return fail(h, WC_E_INVALID_ARG, "token id " + std::to_string(ids[static_cast<size_t>(b) * L + i]) +
                                             " is not below vocab_size " + std::to_string(h->cfg.vocab_size));
  return WC_OK;
}

int ensure_io(wc_t5* h, int64_t rows, int B) {
  if (!h->copy_stream) {
    cudaError_t e = cudaStreamCreateWithFlags(&h->copy_stream, cudaStreamNonBlocking);
    for (int i = 0; i < 2 && e == cudaSuccess; ++i) {
      if ((e = cudaEventCreateWithFlags(&h->ev_in[i], cudaEventDisableTiming)) == cudaSuccess &&
          (e = cudaEventCreateWithFlags(&h->ev_fwd[i], cudaEventDisableTiming)) == cudaSuccess)
        e = cudaEventCreateWithFlags(&h->ev_out[i], cudaEventDisableTiming);
    }
    if (e != cudaSuccess) return cuda_fail(h, e, "copy stream / events");
  }
  if (rows <= h->io_rows && B <= h->io_b) return WC_OK;
  clear_graphs(h);  // captured graphs may hold the old I/O pointers
  if (h->io) {
    cudaStreamSynchronize(h->stream);
    cudaStreamSynchronize(h->copy_stream);
    cudaFree(h->io);
    h->io = nullptr;
  }
  const int64_t cap = std::max<int64_t>((rows + 127) / 128 * 128, h->io_rows);
  const int capb = static_cast<int>(std::max<int64_t>({cap, static_cast<int64_t>(B), h->io_b}));
  const size_t P = h->d_proj;
  size_t off = 0, o_ids[2], o_len[2], o_out[2], o_norms[2];
  for (int i = 0; i < 2; ++i) {
    o_ids[i] = off; off = align256(off + cap * 4);
    o_len[i] = off; off = align256(off + capb * 4);
    o_out[i] = off; off = align256(off + cap * P * 4);
    o_norms[i] = off; off = align256(off + cap * 4);
  }
  cudaError_t e = cudaMalloc(&h->io, off);
  if (e != cudaSuccess) {
    h->io = nullptr;
    h->io_rows = 0;
    h->io_b = 0;
    return cuda_fail(h, e, "I/O buffer allocation");
  }
  for (int i = 0; i < 2; ++i) {
    h->io_ids[i] = reinterpret_cast<uint32_t*>(h->io + o_ids[i]);
    h->io_len[i] = reinterpret_cast<int32_t*>(h->io + o_len[i]);
    h->io_out[i] = reinterpret_cast<float*>(h->io + o_out[i]);
    h->io_norms[i] = reinterpret_cast<float*>(h->io + o_norms[i]);
  }
  h->io_rows = cap;
  h->io_b = capb;
  return WC_OK;
}

// Stream, event and activation buffers (x, xn, qkv, att, h) of the second
// compute lane for batches of up to `rows` tokens.
int ensure_lane(wc_t5* h, int64_t rows) {
  if (!h->lane_stream) {
    cudaError_t e = cudaStreamCreateWithFlags(&h->lane_stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h->ev_lane, cudaEventDisableTiming);
    if (e != cudaSuccess) return cuda_fail(h, e, "second compute lane stream / event");
  }
  if (rows <= h->lane_rows) return WC_OK;
  if (h->lane_ws) {
    cudaStreamSynchronize(h->lane_stream);
    cudaFree(h->lane_ws);
    h->lane_ws = nullptr;
    h->lane_rows = 0;
  }
  const int64_t cap = (rows + 127) / 128 * 128;
  const int D = h->cfg.d_model, F = h->cfg.d_ff, I = h->inner;
  size_t off = 0;
  const size_t o_x = off; off = align256(off + cap * D * 4);
  const size_t o_xn = off; off = align256(off + cap * D * 2);
  const size_t o_qkv = off; off = align256(off + cap * std::max(3 * I * 2, D * 4));
  const size_t o_att = off; off = align256(off + cap * I * 2);
  const size_t o_h = off; off = align256(off + cap * F * 2);
  cudaError_t e = cudaMalloc(&h->lane_ws, off);
  if (e != cudaSuccess) {
    h->lane_ws = nullptr;
    return cuda_fail(h, e, "second compute lane workspace");
  }
  h->lane_x = reinterpret_cast<float*>(h->lane_ws + o_x);
  h->lane_xn = reinterpret_cast<__half*>(h->lane_ws + o_xn);
  h->lane_qkv = reinterpret_cast<__half*>(h->lane_ws + o_qkv);
  h->lane_att = reinterpret_cast<__half*>(h->lane_ws + o_att);
  h->lane_h = reinterpret_cast<__half*>(h->lane_ws + o_h);
  if (!make_act_map(&h->lane_tm_xn, h->lane_xn, cap, D) || !make_act_map(&h->lane_tm_att, h->lane_att, cap, I) ||
      !make_act_map(&h->lane_tm_h, h->lane_h, cap, F))
    return fail(h, WC_E_CUDA, "cuTensorMapEncodeTiled failed for a second-lane activation buffer");
  h->lane_rows = cap;
  return WC_OK;
}

}  // namespace
}  // namespace wc

extern "C" int wc_t5_forward_many(wc_t5* h, int n, const uint32_t* const* ids, const int32_t* const* lengths,
                                  const int* B, const int* L, float* const* out, float* const* norms) {
  if (!h) return WC_E_INVALID_ARG;
  if (n < 0 || (n > 0 && (!ids || !B || !L || !out)))
    return fail(h, WC_E_INVALID_ARG, "invalid batch arrays");
  if (n == 0) return WC_OK;
  std::vector<std::vector<int32_t>> lens(n);
  int64_t max_rows = 0;
  int max_b = 0;
  for (int i = 0; i < n; ++i) {
    const int rc = check_batch(h, ids[i], lengths ? lengths[i] : nullptr, B[i], L[i], out[i], lens[i]);
    if (rc) return rc;
    max_rows = std::max<int64_t>(max_rows, static_cast<int64_t>(B[i]) * L[i]);
    max_b = std::max(max_b, B[i]);
  }
  DeviceGuard g(h->device);
  // two compute lanes when there are several batches and the largest is
  // past the captured-graph size
  // (WC_FORWARD_LANES=1 keeps every batch on the handle's stream)
  static const bool one_lane = [] {
    const char* v = getenv("WC_FORWARD_LANES");
    return v && v[0] == '1' && v[1] == 0;
  }();
  const bool two_lanes = !one_lane && n > 1 && max_rows > kGraphMaxRows;
  int rc = ensure_workspace(h, max_rows, max_b);
  if (!rc) rc = ensure_io(h, max_rows, max_b);
  if (!rc && two_lanes) rc = ensure_lane(h, max_rows);
  if (rc) return rc;
  cudaStream_t cs = h->stream, ps = h->copy_stream;
  cudaError_t e = cudaMemsetAsync(h->d_status, 0, 4, cs);
  if (two_lanes && e == cudaSuccess && (e = cudaEventRecord(h->ev_lane, cs)) == cudaSuccess)
    e = cudaStreamWaitEvent(h->lane_stream, h->ev_lane, 0);  // after the status reset
  auto upload = [&](int i) -> cudaError_t {
    const int s = i & 1;
    const int64_t M = static_cast<int64_t>(B[i]) * L[i];
    cudaError_t r = cudaMemcpyAsync(h->io_ids[s], ids[i], M * 4, cudaMemcpyHostToDevice, ps);
    if (r == cudaSuccess) r = cudaMemcpyAsync(h->io_len[s], lens[i].data(), B[i] * 4, cudaMemcpyHostToDevice, ps);
    if (r == cudaSuccess) r = cudaEventRecord(h->ev_in[s], ps);
    return r;
  };
  for (int i = 0; i < 2 && i < n && e == cudaSuccess; ++i) e = upload(i);
  for (int i = 0; i < n && e == cudaSuccess && rc == WC_OK; ++i) {
    const int s = i & 1;  // I/O set, and compute lane with two lanes
    const int64_t M = static_cast<int64_t>(B[i]) * L[i];
    float* nrm = norms ? norms[i] : nullptr;
    cudaStream_t fs = two_lanes && s ? h->lane_stream : cs;
    // compute: inputs of batch i landed; d_out of set s read out (batch i - 2)
    if ((e = cudaStreamWaitEvent(fs, h->ev_in[s], 0)) != cudaSuccess) break;
    if (i >= 2 && (e = cudaStreamWaitEvent(fs, h->ev_out[s], 0)) != cudaSuccess) break;
    // Bulk calls (two lanes) launch their small batches eagerly: a one-off
    // shape would pay a graph capture and instantiation (tens of ms when
    // another process shares the driver) and never replay it.
    if (fs == cs && !two_lanes)
      rc = forward_cached(h, h->io_ids[s], h->io_len[s], B[i], L[i], h->io_out[s], nrm ? h->io_norms[s] : nullptr,
                          nullptr, cs);
    else if (fs == cs)
      rc = forward_device(h, h->io_ids[s], h->io_len[s], B[i], L[i], h->io_out[s], nrm ? h->io_norms[s] : nullptr,
                          nullptr, cs);
    else
      rc = forward_on(h, h->lane_x, h->lane_xn, h->lane_qkv, h->lane_att, h->lane_h, h->lane_tm_xn,
                      h->lane_tm_att, h->lane_tm_h, h->io_ids[s], h->io_len[s], B[i], L[i], h->io_out[s],
                      nrm ? h->io_norms[s] : nullptr, nullptr, fs);
    if (rc) break;
    if ((e = cudaEventRecord(h->ev_fwd[s], fs)) != cudaSuccess) break;
    // copy: results of batch i out, then inputs of batch i + 2 into set s
    if ((e = cudaStreamWaitEvent(ps, h->ev_fwd[s], 0)) != cudaSuccess) break;
    if ((e = cudaMemcpyAsync(out[i], h->io_out[s], M * h->d_proj * 4, cudaMemcpyDeviceToHost, ps)) != cudaSuccess)
      break;
    if (nrm && (e = cudaMemcpyAsync(nrm, h->io_norms[s], M * 4, cudaMemcpyDeviceToHost, ps)) != cudaSuccess) break;
    if ((e = cudaEventRecord(h->ev_out[s], ps)) != cudaSuccess) break;
    if (i + 2 < n && (e = upload(i + 2)) != cudaSuccess) break;
  }
  cudaError_t es = cudaStreamSynchronize(ps);
  if (two_lanes) {
    const cudaError_t el = cudaStreamSynchronize(h->lane_stream);
    if (es == cudaSuccess) es = el;
  }
  if (rc) {
    cudaStreamSynchronize(cs);
    return rc;
  }
  if (e == cudaSuccess) e = es;
  if (e != cudaSuccess) {
    cudaStreamSynchronize(cs);
    return cuda_fail(h, e, "pipelined forward");
  }
  return check_status(h, cs);
}

extern "C" void* wc_host_alloc(size_t bytes) {
  void* p = nullptr;
  if (bytes == 0 || cudaHostAlloc(&p, bytes, cudaHostAllocPortable) != cudaSuccess) return nullptr;
  return p;
}

extern "C" void wc_host_free(void* p) {
  if (p) cudaFreeHost(p);
}

extern "C" int wc_t5_forward_many_device(wc_t5* h, int n, const uint32_t* const* d_ids,
                                         const int32_t* const* d_lengths, const int* B, const int* L,
                                         float* const* d_out, float* const* d_norms, void* stream) {
  if (!h) return WC_E_INVALID_ARG;
  if (n < 0 || (n > 0 && (!d_ids || !d_lengths || !B || !L || !d_out)))
    return fail(h, WC_E_INVALID_ARG, "invalid batch arrays");
  if (n == 0) return WC_OK;
  int64_t max_rows = 0;
  int max_b = 0;
  for (int i = 0; i < n; ++i) {
    if (!d_ids[i] || !d_lengths[i] || !d_out[i] || B[i] < 1 || L[i] < 1 || L[i] > kMaxL ||
        static_cast<int64_t>(B[i]) * L[i] > (1 << 26))
      return fail(h, WC_E_INVALID_ARG, "batch " + std::to_string(i) +
                                           ": invalid ids/lengths/out pointer or B, L out of range (1 <= L <= 2048)");
    max_rows = std::max<int64_t>(max_rows, static_cast<int64_t>(B[i]) * L[i]);
    max_b = std::max(max_b, B[i]);
  }
  DeviceGuard g(h->device);
  static const bool one_lane = [] {
    const char* v = getenv("WC_FORWARD_LANES");
    return v && v[0] == '1' && v[1] == 0;
  }();
  const bool two_lanes = !one_lane && n > 1 && max_rows > kGraphMaxRows;
  int rc = ensure_workspace(h, max_rows, max_b);
  if (!rc && two_lanes) rc = ensure_lane(h, max_rows);
  if (rc) return rc;
  cudaStream_t cs = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(h->d_status, 0, 4, cs);
  // the second lane starts after the caller's earlier work and the status reset
  if (two_lanes && e == cudaSuccess && (e = cudaEventRecord(h->ev_lane, cs)) == cudaSuccess)
    e = cudaStreamWaitEvent(h->lane_stream, h->ev_lane, 0);
  if (e != cudaSuccess) return cuda_fail(h, e, "lane fork");
  for (int i = 0; i < n && rc == WC_OK; ++i) {
    float* nrm = d_norms ? d_norms[i] : nullptr;
    if (!two_lanes)
      rc = forward_cached(h, d_ids[i], d_lengths[i], B[i], L[i], d_out[i], nrm, nullptr, cs);
    else if ((i & 1) == 0)  // bulk: no graph capture of one-off shapes
      rc = forward_device(h, d_ids[i], d_lengths[i], B[i], L[i], d_out[i], nrm, nullptr, cs);
    else
      rc = forward_on(h, h->lane_x, h->lane_xn, h->lane_qkv, h->lane_att, h->lane_h, h->lane_tm_xn,
                      h->lane_tm_att, h->lane_tm_h, d_ids[i], d_lengths[i], B[i], L[i], d_out[i], nrm, nullptr,
                      h->lane_stream);
  }
  // join: the caller's stream continues after both lanes (also on an error,
  // so no work of this call is left unordered behind the caller's stream)
  if (two_lanes && (e = cudaEventRecord(h->ev_lane, h->lane_stream)) == cudaSuccess)
    e = cudaStreamWaitEvent(cs, h->ev_lane, 0);
  if (rc) return rc;
  return e == cudaSuccess ? WC_OK : cuda_fail(h, e, "lane join");
}

extern "C" int wc_q4k_dequant_f16(const void* d_blocks, int64_t nblocks, void* d_out_f16, void* stream) {
  if (nblocks < 0 || (nblocks > 0 && (!d_blocks || !d_out_f16))) return WC_E_INVALID_ARG;
  return q4k_dequant_f16_launch(static_cast<const uint8_t*>(d_blocks), nblocks, static_cast<__half*>(d_out_f16),
                                static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? WC_OK
             : WC_E_CUDA;
}

extern "C" int wc_q4k_dequant(const void* d_blocks, int64_t nblocks, float* d_out, void* stream) {
  if (nblocks < 0 || (nblocks > 0 && (!d_blocks || !d_out))) return WC_E_INVALID_ARG;
  return q4k_dequant_launch(static_cast<const uint8_t*>(d_blocks), nblocks, d_out,
                            static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? WC_OK
             : WC_E_CUDA;
}

extern "C" int wc_gemm_f16(const void* d_x, int M, int K, const void* d_w, const void* d_w_up, int N, int epilogue,
                           void* d_out, void* stream) {
  if (!d_x || !d_w || !d_out || M < 1 || K < 256 || K % 256 || N < 128 || N % 128) return WC_E_INVALID_ARG;
  if (epilogue < 0 || epilogue > 3) return WC_E_INVALID_ARG;
  if (epilogue == kEpiGeGLU && !d_w_up) return WC_E_INVALID_ARG;
  const int tile_n = epilogue == kEpiGeGLU ? 2 * N : N;
  if (!gemm2_q4k_supports(epilogue, M, tile_n, K)) return WC_E_UNSUPPORTED;
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = device_sm_count(dev);
  // the f32 epilogues take the tile width the encoder picks for its residual GEMMs
  const int bn = (epilogue == kEpiResid || epilogue == kEpiF32) ? gemm2_resid_bn(M, N, sms) : 256;
  CUtensorMap ta, tw0, tw1, tout;
  if (!make_act_map(&ta, d_x, M, K) || !make_act_map(&tw0, d_w, N, K, bn / 2) ||
      !make_act_map(&tw1, epilogue == kEpiGeGLU ? d_w_up : d_w, N, K, bn / 2) ||
      !make_out_map(&tout, d_out, M, N, epilogue == kEpiF32 || epilogue == kEpiResid))
    return WC_E_CUDA;
  GemmParams p{};
  p.M = M;
  p.N = tile_n;
  p.K = K;
  p.out = d_out;
  p.ldo = N;
  p.status = kernel_status_word();
  if (!p.status) return WC_E_CUDA;
  return gemm2_q4k_launch(epilogue, ta, tw0, tw1, tout, p, sms, static_cast<cudaStream_t>(stream), true, bn) ==
                 cudaSuccess
             ? WC_OK
             : WC_E_CUDA;
}

extern "C" int wc_gemm_q4k(const void* d_x, int M, int K, const void* d_w, const void* d_w_up, int N, int epilogue,
                           void* d_out, void* stream) {
  if (!d_x || !d_w || !d_out || M < 1 || K < 256 || K % 256 || N < 128 || N % 128) return WC_E_INVALID_ARG;
  if (epilogue < 0 || epilogue > 3) return WC_E_INVALID_ARG;
  if (epilogue == kEpiGeGLU && !d_w_up) return WC_E_INVALID_ARG;
  const int tile_n = epilogue == kEpiGeGLU ? 2 * N : N;
  if (gemv_q4k_supports(epilogue, M, N, K))
    return gemv_q4k_launch(epilogue, static_cast<const __half*>(d_x), M, K, static_cast<const uint8_t*>(d_w),
                           static_cast<const uint8_t*>(epilogue == kEpiGeGLU ? d_w_up : d_w), N, d_out, N,
                           nullptr, static_cast<cudaStream_t>(stream)) == cudaSuccess
               ? WC_OK
               : WC_E_CUDA;
  if (M >= kGemm2MinRows && gemm2_q4k_supports(epilogue, M, tile_n, K)) {
    CUtensorMap ta, tw0, tw1;
    if (!make_act_map(&ta, d_x, M, K) || !make_q4k_map(&tw0, d_w, N, K, kGemm2WBoxRows) ||
        !make_q4k_map(&tw1, epilogue == kEpiGeGLU ? d_w_up : d_w, N, K, kGemm2WBoxRows))
      return WC_E_CUDA;
    GemmParams p{};
    p.M = M;
    p.N = tile_n;
    p.K = K;
    p.out = d_out;
    p.ldo = N;
    p.status = kernel_status_word();
    if (!p.status) return WC_E_CUDA;
    CUtensorMap tout;
    if (!make_out_map(&tout, d_out, M, N, epilogue == kEpiF32 || epilogue == kEpiResid)) return WC_E_CUDA;
    int dev = 0;
    cudaGetDevice(&dev);
    return gemm2_q4k_launch(epilogue, ta, tw0, tw1, tout, p, device_sm_count(dev), static_cast<cudaStream_t>(stream)) ==
                   cudaSuccess
               ? WC_OK
               : WC_E_CUDA;
  }
  const int bn = gemm_q4k_bn_for(epilogue, tile_n);
  if (bn < 0) return WC_E_UNSUPPORTED;
  const int box = gemm_q4k_w_box_rows(epilogue, bn);
  CUtensorMap ta, tw0, tw1;
  if (!make_act_map(&ta, d_x, M, K) || !make_q4k_map(&tw0, d_w, N, K, box) ||
      !make_q4k_map(&tw1, epilogue == kEpiGeGLU ? d_w_up : d_w, N, K, box))
    return WC_E_CUDA;
  GemmParams p{};
  p.M = M;
  p.N = tile_n;
  p.K = K;
  p.out = d_out;
  p.ldo = N;
  p.status = kernel_status_word();
  if (!p.status) return WC_E_CUDA;
  return gemm_q4k_launch(epilogue, bn, ta, tw0, tw1, p, static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? WC_OK
             : WC_E_CUDA;
}

namespace wc {
namespace {
// Thresholds of the last (num_buckets, max_distance) asked for: computing
// them takes thousands of reference bucket evaluations on the host.
BucketThresholds cached_thresholds(int num_buckets, int max_distance) {
  static std::mutex mu;
  static int key[2] = {-1, -1};
  static BucketThresholds bt{};
  std::lock_guard<std::mutex> lk(mu);
  if (key[0] != num_buckets || key[1] != max_distance) {
    bt = t5_bucket_thresholds(num_buckets, max_distance, kMaxL);
    key[0] = num_buckets;
    key[1] = max_distance;
  }
  return bt;
}
}  // namespace
}  // namespace wc

extern "C" int wc_attention(const void* d_qkv, int B, int L, int H, const int32_t* d_lengths,
                            const float* d_bias_table, int num_buckets, int max_distance, void* d_out,
                            void* stream) {
  if (!d_qkv || !d_lengths || !d_bias_table || !d_out || B < 1 || L < 1 || L > kMaxL || H < 1 ||
      num_buckets < 2 || num_buckets > 32 || max_distance < 1)
    return WC_E_INVALID_ARG;
  const BucketThresholds bt = cached_thresholds(num_buckets, max_distance);
  if (attention_small_supports(L))
    return attention_small_launch(static_cast<const __half*>(d_qkv), static_cast<__half*>(d_out), d_lengths, B, L, H,
                                  d_bias_table, bt, static_cast<cudaStream_t>(stream)) == cudaSuccess
               ? WC_OK
               : WC_E_CUDA;
  CUtensorMap tm;
  if (!make_act_map(&tm, d_qkv, static_cast<uint64_t>(B) * L, 3 * H * 64, 64)) return WC_E_CUDA;
  uint32_t* status = kernel_status_word();
  if (!status) return WC_E_CUDA;
  return attention_tc_launch(tm, static_cast<__half*>(d_out), d_lengths, B, L, H, d_bias_table, bt, status,
                             static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? WC_OK
             : WC_E_CUDA;
}

extern "C" int wc_t5_relative_bucket(int query, int key, int num_buckets, int max_distance) {
  if (num_buckets < 2 || num_buckets > 64 || max_distance < 1 || query < 0 || key < 0 || query >= kMaxL ||
      key >= kMaxL)
    return WC_E_INVALID_ARG;
  const BucketThresholds bt = cached_thresholds(num_buckets, max_distance);
  return t5_bucket_from_thresholds(bt, key - query);
}

// ---------------------------------------------------------------- no-allocation forward
//
// wc_t5_forward_device_noalloc runs the same kernels as wc_t5_forward_device
// but keeps its activations (the per-call scratch) in the fixed device array
// below instead of the handle's workspace, so a call never allocates device
// memory.  The array exists once per GPU that loads this library and is held
// until the process exits.

static constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace wc {
namespace {

struct NoAllocLayout {
  size_t x, xn, qkv, att, h, total;
};

NoAllocLayout noalloc_layout(const wc_t5* h, int64_t M) {
  const size_t D = h->cfg.d_model, F = h->cfg.d_ff, I = h->inner;
  NoAllocLayout l{};
  size_t off = 0;
  l.x = off; off = align256(off + M * D * 4);
  l.xn = off; off = align256(off + M * D * 2);
  l.qkv = off; off = align256(off + M * std::max(3 * I * 2, D * 4));  // also the f32 O / wo output
  l.att = off; off = align256(off + M * I * 2);
  l.h = off; off = align256(off + M * F * 2);
  l.total = off;
  return l;
}

// Device address of g_noalloc_scratch on the current device.  Looked up once
// per device and context (the host-side name of a __device__ array is not a
// device address); this first lookup also loads the module on that device.
// If the device was reset since, its context is a new one and the address is
// looked up again rather than reused.
uint8_t* noalloc_scratch_ptr(int dev, cudaError_t* err) {
  static uint8_t* ptrs[64] = {};
  static CUcontext ctxs[64] = {};
  static std::mutex mu;
  *err = cudaSuccess;
  if (dev < 0 || dev >= 64) {
    *err = cudaErrorInvalidDevice;
    return nullptr;
  }
  const CUcontext ctx = current_context();
  std::lock_guard<std::mutex> lk(mu);
  if (!ptrs[dev] || ctxs[dev] != ctx) {
    void* p = nullptr;
    *err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (*err != cudaSuccess) return nullptr;
    ptrs[dev] = static_cast<uint8_t*>(p);
    ctxs[dev] = ctx;
  }
  return ptrs[dev];
}

// The launch sequence of one forward over the given activation buffers
// (x, xn, qkv, att, hbuf) and their tensor maps.
// Optional per-launch event marks for timeline analysis (off in the library
// build): an event after every launch of the last forward.
#ifdef WC_FWD_EVENTS
cudaEvent_t g_fwd_ev[128];
int g_fwd_n = 0;
#define FWD_MARK()                                                          \
  do {                                                                      \
    if (g_fwd_n < 128) {                                                    \
      if (!g_fwd_ev[g_fwd_n]) cudaEventCreate(&g_fwd_ev[g_fwd_n]);          \
      cudaEventRecord(g_fwd_ev[g_fwd_n++], st);                             \
    }                                                                       \
  } while (0)
#define FWD_BEGIN() \
  do {              \
    g_fwd_n = 0;    \
    FWD_MARK();     \
  } while (0)
#else
#define FWD_MARK() \
  do {             \
  } while (0)
#define FWD_BEGIN() \
  do {              \
  } while (0)
#endif

int forward_on(wc_t5* h, float* x, __half* xn, __half* qkv, __half* att, __half* hbuf, const CUtensorMap& tm_xn,
               const CUtensorMap& tm_att, const CUtensorMap& tm_h, const uint32_t* ids, const int32_t* lengths,
               int B, int L, float* out, float* norms, float* outn, cudaStream_t st) {
  FWD_BEGIN();
  const T5Config& c = h->cfg;
  const int D = c.d_model, F = c.d_ff, I = h->inner, H = c.num_heads;
  const int M = B * L;
  CUtensorMap tm_qkv;
  if (!make_act_map(&tm_qkv, qkv, M, 3 * I, 64)) return fail(h, WC_E_CUDA, "cuTensorMapEncodeTiled failed for qkv");
  // Residual adds: for large M the O / wo GEMM epilogue adds into x itself
  // (TMA load-add-store) and the RMSNorm only normalises; otherwise the GEMM
  // writes f32 into the dead qkv buffer and the RMSNorm adds it.
  const bool fused_res = M >= kGemm2MinRows;
  const int res_epi = fused_res ? kEpiResid : kEpiF32;
  void* res_out = fused_res ? static_cast<void*>(x) : static_cast<void*>(qkv);
  const float* res_delta = fused_res ? nullptr : reinterpret_cast<const float*>(qkv);
  cudaError_t e;
  if ((e = embed_rmsnorm_launch(h->embed, ids, lengths, L, M, D, h->layers[0].ln0, c.eps, x, xn, h->d_status, st)) !=
      cudaSuccess)
    return cuda_fail(h, e, "embedding launch");
  FWD_MARK();
  int rc;
  for (int l = 0; l < c.num_layers; ++l) {
    LayerW& w = h->layers[l];
    if ((rc = layer_gemm(h, kEpiF16, h->bn_qkv, tm_xn, w.tm_qkv, w.tm_qkv, h->f16_weights ? w.tmh_qkv : w.tmq2_qkv, h->f16_weights ? w.tmh_qkv : w.tmq2_qkv, M, 3 * I, D, qkv, 3 * I, st, xn, w.qkv, w.qkv))) return rc;
    FWD_MARK();
    e = attention_small_supports(L) ? attention_small_launch(qkv, att, lengths, B, L, H, h->rel_bias, h->bt, st)
                                    : attention_tc_launch(tm_qkv, att, lengths, B, L, H, h->rel_bias, h->bt,
                                                          h->d_status, st);
    if (e != cudaSuccess) return cuda_fail(h, e, "attention launch");
    FWD_MARK();
    if ((rc = layer_gemm(h, res_epi, h->bn_o, tm_att, w.tm_o, w.tm_o, h->f16_weights ? w.tmh_o : w.tmq2_o, h->f16_weights ? w.tmh_o : w.tmq2_o, M, D, I, res_out, D, st, att, w.o, w.o, &w.tmh64_o))) return rc;
    FWD_MARK();
    if ((e = rmsnorm_launch(x, res_delta, w.ln1, xn, M, D, c.eps, h->d_status, st)) != cudaSuccess) return cuda_fail(h, e, "rmsnorm launch");
    FWD_MARK();
    if ((rc = layer_gemm(h, kEpiGeGLU, h->bn_wi, tm_xn, w.tm_wi0, w.tm_wi1, h->f16_weights ? w.tmh_wi0 : w.tmq2_wi0, h->f16_weights ? w.tmh_wi1 : w.tmq2_wi1, M, 2 * F, D, hbuf, F, st, xn, w.wi0, w.wi1))) return rc;
    FWD_MARK();
    if ((rc = layer_gemm(h, res_epi, h->bn_wo, tm_h, w.tm_wo, w.tm_wo, h->f16_weights ? w.tmh_wo : w.tmq2_wo, h->f16_weights ? w.tmh_wo : w.tmq2_wo, M, D, F, res_out, D, st, hbuf, w.wo, w.wo, &w.tmh64_wo))) return rc;
    FWD_MARK();
    const float* next_ln = l + 1 < c.num_layers ? h->layers[l + 1].ln0 : h->final_ln;
    if ((e = rmsnorm_launch(x, res_delta, next_ln, xn, M, D, c.eps, h->d_status, st)) != cudaSuccess) return cuda_fail(h, e, "rmsnorm launch");
    FWD_MARK();
  }
  return gemm(h, kEpiProj, 128, tm_xn, h->tm_proj, h->tm_proj, M, h->d_proj, D, out, h->d_proj, st, norms, outn,
              lengths, L);
}

}  // namespace
}  // namespace wc

extern "C" int wc_t5_forward_device_noalloc(wc_t5* h, const uint32_t* d_ids, const int32_t* d_lengths, int B,
                                            int L, float* d_out, float* d_norms, float* d_outn, void* stream) {
  if (!h) return WC_E_INVALID_ARG;
  if (!d_ids || !d_lengths || !d_out || B < 1 || L < 1 || L > kMaxL)
    return fail(h, WC_E_INVALID_ARG, "invalid ids/lengths/out pointer or B, L out of range (1 <= L <= 2048)");
  DeviceGuard g(h->device);
  const int64_t M = static_cast<int64_t>(B) * L;
  const NoAllocLayout lay = noalloc_layout(h, M);
  if (lay.total > kNoAllocScratchBytes) {
    const NoAllocLayout one = noalloc_layout(h, 1);
    int64_t max_tokens = static_cast<int64_t>(kNoAllocScratchBytes / one.total);
    while (max_tokens > 0 && noalloc_layout(h, max_tokens).total > kNoAllocScratchBytes) --max_tokens;
    return fail(h, WC_E_INVALID_ARG,
                "B*L = " + std::to_string(M) + " tokens needs " + std::to_string(lay.total) +
                    " bytes of scratch; the no-allocation forward has " + std::to_string(kNoAllocScratchBytes) +
                    " (at most " + std::to_string(max_tokens) + " tokens per call for this model)");
  }
  cudaError_t e;
  uint8_t* base = noalloc_scratch_ptr(h->device, &e);
  if (!base) return cuda_fail(h, e, "cudaGetSymbolAddress of the no-allocation scratch");
  float* x = reinterpret_cast<float*>(base + lay.x);
  __half* xn = reinterpret_cast<__half*>(base + lay.xn);
  __half* qkv = reinterpret_cast<__half*>(base + lay.qkv);
  __half* att = reinterpret_cast<__half*>(base + lay.att);
  __half* hb = reinterpret_cast<__half*>(base + lay.h);
  CUtensorMap tm_xn, tm_att, tm_h;
  if (!make_act_map(&tm_xn, xn, M, h->cfg.d_model) || !make_act_map(&tm_att, att, M, h->inner) ||
      !make_act_map(&tm_h, hb, M, h->cfg.d_ff))
    return fail(h, WC_E_CUDA, "cuTensorMapEncodeTiled failed for a no-allocation scratch buffer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The status word was allocated with the handle; clear it for this call.
  if ((e = cudaMemsetAsync(h->d_status, 0, 4, st)) != cudaSuccess) return cuda_fail(h, e, "status reset");
  return forward_on(h, x, xn, qkv, att, hb, tm_xn, tm_att, tm_h, d_ids, d_lengths, B, L, d_out, d_norms, d_outn, st);
}

extern "C" int wc_selftest_wait_timeout(uint64_t limit_ns) {
  if (limit_ns < 1000000ull || limit_ns > 10000000000ull) return WC_E_INVALID_ARG;
  uint32_t* status = kernel_status_word();
  if (!status) return WC_E_CUDA;
  uint32_t s = 0;
  if (cudaMemset(status, 0, 4) != cudaSuccess ||
      wait_timeout_selftest_launch(status, limit_ns, nullptr) != cudaSuccess ||
      cudaMemcpy(&s, status, 4, cudaMemcpyDeviceToHost) != cudaSuccess || cudaMemset(status, 0, 4) != cudaSuccess)
    return WC_E_CUDA;  // the context did not stay usable
  return (s & kStatusWaitTimeout) ? WC_E_TIMEOUT : WC_E_CUDA;
}

#ifdef WC_FWD_EVENTS
// Milliseconds between consecutive marks of the last forward; returns the count.
extern "C" int wc_fwd_events(float* ms, int max) {
  const int n = wc::g_fwd_n;
  if (n < 2) return 0;
  cudaEventSynchronize(wc::g_fwd_ev[n - 1]);
  for (int i = 1; i < n && i <= max; ++i) cudaEventElapsedTime(&ms[i - 1], wc::g_fwd_ev[i - 1], wc::g_fwd_ev[i]);
  return n - 1;
}
#endif
