// extern "C" entry points of libtsb_moe.so (declared in include/tsb_moe.h).
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/tsb_moe.h"
#include "qformats.cuh"
#include "tsb_internal.h"

namespace tsb {

static thread_local std::string g_last_error;

int set_error(int code, const char* msg) {
  g_last_error = msg ? msg : "";
  return code;
}

void weight_bytes_of(int fmt, int64_t rows, int64_t cols, int64_t& data, int64_t& scales) {
  const int64_t n = rows * cols;
  scales = 0;
  switch (fmt) {
    case FMT_Q8_0: data = n / 32 * 34; break;
    case FMT_Q4_K: data = n / 256 * 144; break;
    case FMT_Q5_K: data = n / 256 * 176; break;
    case FMT_Q6_K: data = n / 256 * 210; break;
    case FMT_MXFP4: data = n / 2; scales = n / 32; break;
    case TSB_FMT_F32: data = n * 4; break;
    case TSB_FMT_F16:
    case TSB_FMT_BF16: data = n * 2; break;
    default: data = 0;
  }
}

static bool known_fmt(int f) {
  return f == FMT_Q8_0 || f == FMT_Q4_K || f == FMT_Q5_K || f == FMT_Q6_K || f == FMT_MXFP4;
}

static int check_shape(int fmt, int64_t rows, int64_t cols) {
  char buf[256];
  if (!known_fmt(fmt)) {
    snprintf(buf, sizeof buf, "Unsupported ggml_type: %d. Supported: Q8_0(8), Q4_K(12), Q5_K(13), Q6_K(14), MXFP4(39)",
             fmt);
    return set_error(TSB_ERR_UNSUPPORTED, buf);
  }
  if (rows < 0 || cols <= 0 || cols % 32) {
    snprintf(buf, sizeof buf, "in_features (%lld) must be a positive multiple of 32", (long long)cols);
    return set_error(TSB_ERR_INVALID, buf);
  }
  const bool kq = fmt == FMT_Q4_K || fmt == FMT_Q5_K || fmt == FMT_Q6_K;
  if (kq && (rows * cols) % 256) {
    snprintf(buf, sizeof buf, "rows*cols (%lld) must be a multiple of 256 for K-quants", (long long)(rows * cols));
    return set_error(TSB_ERR_INVALID, buf);
  }
  return TSB_OK;
}

// Workspace layout of tsb_moe_decode (offsets in bytes).
struct WsLayout {
  size_t err, counter, logits, act, total;
};

static WsLayout ws_layout(const TsbMoeSpec& sp, int T) {
  WsLayout L;
  auto al = [](size_t v) { return (v + 255) & ~size_t(255); };
  L.err = 0;
  L.counter = 4;
  L.logits = 256;
  L.act = L.logits + al(sizeof(float) * (size_t)T * sp.n_experts);
  L.total = L.act + al(sizeof(float) * (size_t)T * sp.top_k * sp.inter);
  return L;
}

// A spec whose experts are dense float tensors (both projections dense).
static bool dense_spec(const TsbMoeSpec& sp) { return is_dense_fmt(sp.fmt_gate_up) && is_dense_fmt(sp.fmt_down); }

// Validation of a layer spec: quantised (both projections quantised, no
// transposition) or dense (both dense).
static int check_layer_spec(const TsbMoeSpec& sp) {
  if (sp.top_k < 1 || sp.top_k > 8 || sp.top_k > sp.n_experts) return set_error(TSB_ERR_INVALID, "top_k must be in [1, min(8, E)]");
  if (sp.n_experts < 1 || sp.n_experts > 1024) return set_error(TSB_ERR_INVALID, "n_experts must be in [1, 1024]");
  if (sp.hidden % 32 || sp.inter % 32 || sp.hidden <= 0 || sp.inter <= 0)
    return set_error(TSB_ERR_INVALID, "hidden and inter must be positive multiples of 32");
  if (sp.gate_up_layout < 0 || sp.gate_up_layout > 2) return set_error(TSB_ERR_INVALID, "bad gate_up_layout");
  if (sp.activation < 0 || sp.activation > 1) return set_error(TSB_ERR_INVALID, "bad activation");
  if (sp.out_f32 != 0 && sp.out_f32 != 1) return set_error(TSB_ERR_INVALID, "out_f32 must be 0 or 1");
  const bool dg = is_dense_fmt(sp.fmt_gate_up), dd = is_dense_fmt(sp.fmt_down);
  if (dg != dd) return set_error(TSB_ERR_UNSUPPORTED, "gate/up and down must both be dense or both be quantised");
  if (sp.transposed & ~(TSB_T_GATE_UP | TSB_T_DOWN)) return set_error(TSB_ERR_INVALID, "bad transposed bits");
  if (!dg && sp.transposed) return set_error(TSB_ERR_INVALID, "transposed applies to dense formats only");
  if (dg && (sp.hidden > 16384 || sp.inter > 16384))
    return set_error(TSB_ERR_UNSUPPORTED, "dense experts: hidden and inter must be <= 16384");
  return TSB_OK;
}

// Dense layers run every token of a call in one launch per projection.
static int dense_layer(const TsbMoeSpec& sp, const TsbExpert* experts, const void* x, int32_t T, const void* router_w,
                       const float* router_b, int32_t* ids, float* weights, void* out, void* workspace,
                       size_t workspace_bytes, void* stream) {
  int rc = check_layer_spec(sp);
  if (rc) return rc;
  if (router_w && sp.hidden % 8) return set_error(TSB_ERR_INVALID, "hidden must be a multiple of 8 for the router");
  if ((int64_t)T * sp.top_k > 65535) return set_error(TSB_ERR_UNSUPPORTED, "dense experts: T * top_k must be <= 65535");
  const DenseLayout L = dense_layout(sp, T);
  if (workspace_bytes < L.total) return set_error(TSB_ERR_WORKSPACE, "workspace too small");
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return set_error(TSB_ERR_INVALID, "workspace must be 256-byte aligned");
  return launch_dense_layer(sp, experts, x, T, router_w, router_b, ids, weights, out, static_cast<char*>(workspace), L,
                            static_cast<cudaStream_t>(stream));
}

}  // namespace tsb

using namespace tsb;

extern "C" {

int tsb_version(void) { return 200; }

int tsb_last_error(char* buf, size_t n) {
  const std::string& s = g_last_error;
  if (buf && n) {
    const size_t m = s.size() < n - 1 ? s.size() : n - 1;
    memcpy(buf, s.data(), m);
    buf[m] = 0;
  }
  return (int)s.size();
}

int tsb_format_info(int fmt, int32_t* be, int32_t* bb) {
  int e = 0, b = 0;
  switch (fmt) {
    case FMT_Q8_0: e = 32; b = 34; break;
    case FMT_Q4_K: e = 256; b = 144; break;
    case FMT_Q5_K: e = 256; b = 176; break;
    case FMT_Q6_K: e = 256; b = 210; break;
    case FMT_MXFP4: e = 32; b = 17; break;
    case TSB_FMT_F32: e = 1; b = 4; break;
    case TSB_FMT_F16:
    case TSB_FMT_BF16: e = 1; b = 2; break;
    default: return check_shape(fmt, 0, 32);
  }
  if (be) *be = e;
  if (bb) *bb = b;
  return TSB_OK;
}

int tsb_weight_bytes(int fmt, int64_t rows, int64_t cols, int64_t* data_bytes, int64_t* scale_bytes) {
  int rc = is_dense_fmt(fmt) ? (rows < 0 || cols <= 0 ? set_error(TSB_ERR_INVALID, "bad shape") : TSB_OK)
                             : check_shape(fmt, rows, cols);
  if (rc) return rc;
  int64_t d, s;
  weight_bytes_of(fmt, rows, cols, d, s);
  if (data_bytes) *data_bytes = d;
  if (scale_bytes) *scale_bytes = s;
  return TSB_OK;
}

int tsb_dequant(int fmt, const void* w, const void* scales, int64_t rows, int64_t cols, void* out, int out_dtype,
                void* stream) {
  int rc = check_shape(fmt, rows, cols);
  if (rc) return rc;
  if (!w || !out || (fmt == FMT_MXFP4 && !scales)) return set_error(TSB_ERR_INVALID, "null pointer");
  if (out_dtype != TSB_DT_F32 && out_dtype != TSB_DT_BF16) return set_error(TSB_ERR_INVALID, "out_dtype must be f32 or bf16");
  return launch_dequant(fmt, w, scales, rows, cols, out, out_dtype, static_cast<cudaStream_t>(stream));
}

int tsb_quant_matvec(int fmt, const void* w, const void* scales, int64_t N, int64_t K, const void* x, int x_dtype,
                     int64_t nvec, int64_t x_stride, void* y, int y_dtype, int64_t y_stride, int32_t* dev_err,
                     void* stream) {
  int rc = check_shape(fmt, N, K);
  if (rc) return rc;
  if (nvec <= 0 || N == 0) return TSB_OK;
  if (!w || !x || !y || (fmt == FMT_MXFP4 && !scales)) return set_error(TSB_ERR_INVALID, "null pointer");
  if (reinterpret_cast<uintptr_t>(w) & 15) return set_error(TSB_ERR_INVALID, "weight pointer must be 16-byte aligned");
  if (x_dtype < 0 || x_dtype > 2 || y_dtype < 0 || y_dtype > 2) return set_error(TSB_ERR_INVALID, "bad dtype");
  if (x_stride < K || y_stride < N) {
    if (nvec > 1) return set_error(TSB_ERR_INVALID, "x_stride must be >= K and y_stride >= N");
  }
  const int maxv = max_vectors_for((int)K);
  if (maxv <= 0) return set_error(TSB_ERR_UNSUPPORTED, "K too large for the activation stage");
  const size_t xes = x_dtype == TSB_DT_F32 ? 4 : 2, yes = y_dtype == TSB_DT_F32 ? 4 : 2;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int64_t v0 = 0; v0 < nvec; v0 += maxv) {
    const int nv = (int)((nvec - v0) < maxv ? (nvec - v0) : maxv);
    rc = launch_matvec(fmt, w, scales, N, K, static_cast<const char*>(x) + v0 * x_stride * xes, x_dtype, nv, x_stride,
                       static_cast<char*>(y) + v0 * y_stride * yes, y_dtype, y_stride, dev_err, st);
    if (rc) return rc;
  }
  return TSB_OK;
}

// Bytes per element of the layer output (bf16, or fp32 with spec.out_f32).
static int64_t out_elem(const TsbMoeSpec& sp) { return sp.out_f32 ? 4 : 2; }

// Validation shared by the batch-1 decode entry points.
static int check_decode_spec(const TsbMoeSpec& sp, const void* router_w) {
  if (sp.top_k < 1 || sp.top_k > 8 || sp.top_k > sp.n_experts) return set_error(TSB_ERR_INVALID, "top_k must be in [1, min(8, E)]");
  if (sp.n_experts < 1 || sp.n_experts > 1024) return set_error(TSB_ERR_INVALID, "n_experts must be in [1, 1024]");
  if (sp.hidden % 32 || sp.inter % 32 || sp.hidden <= 0 || sp.inter <= 0)
    return set_error(TSB_ERR_INVALID, "hidden and inter must be positive multiples of 32");
  if (router_w && sp.hidden % 8) return set_error(TSB_ERR_INVALID, "hidden must be a multiple of 8 for the router");
  if (sp.gate_up_layout < 0 || sp.gate_up_layout > 2) return set_error(TSB_ERR_INVALID, "bad gate_up_layout");
  if (sp.activation < 0 || sp.activation > 1) return set_error(TSB_ERR_INVALID, "bad activation");
  if (sp.out_f32 != 0 && sp.out_f32 != 1) return set_error(TSB_ERR_INVALID, "out_f32 must be 0 or 1");
  const int rc = check_shape(sp.fmt_gate_up, sp.inter, sp.hidden);
  if (rc) return rc;
  return check_shape(sp.fmt_down, sp.hidden, sp.inter);
}

// Up to this many tokens, tsb_moe_decode runs the batch-1 kernels once per
// token: each token costs one HBM pass over its 4 experts (~45-55 us on the
// GPT-OSS-20B shape), which beats the grouped GEMM path until the batch
// shares enough experts (measured crossover between 16 and 32 tokens).
constexpr int kDecodeLoopMax = 16;

size_t tsb_moe_decode_workspace(const TsbMoeSpec* spec, int32_t T) {
  if (!spec || T <= 0) return 0;
  if (dense_spec(*spec)) return dense_layout(*spec, T).total;
  if (T > kDecodeLoopMax) return prefill_layout(*spec, T).total;  // grouped GEMMs
  return ws_layout(*spec, 1).total;
}

int tsb_moe_decode(const TsbMoeSpec* spec, const TsbExpert* experts, const void* x, int32_t T, const void* router_w,
                   const float* router_b, int32_t* ids, float* weights, void* out, void* workspace,
                   size_t workspace_bytes, void* stream) {
  if (!spec || !experts || !x || !ids || !weights || !out || !workspace) return set_error(TSB_ERR_INVALID, "null pointer");
  const TsbMoeSpec& sp = *spec;
  if (T < 1) return set_error(TSB_ERR_INVALID, "T must be >= 1");
  if (is_dense_fmt(sp.fmt_gate_up) || is_dense_fmt(sp.fmt_down))
    return dense_layer(sp, experts, x, T, router_w, router_b, ids, weights, out, workspace, workspace_bytes, stream);
  if (sp.transposed) return set_error(TSB_ERR_INVALID, "transposed applies to dense formats only");
  // Larger batches (ExpertBatcher) share each expert's weight stream through
  // the grouped path; small ones run token by token (stream-ordered: the next
  // token's first kernel is launched without programmatic overlap).
  if (T > kDecodeLoopMax)
    return tsb_moe_prefill(spec, experts, x, T, router_w, router_b, ids, weights, out, workspace, workspace_bytes, stream);
  if (T > 1) {
    const int64_t H = spec->hidden, k = spec->top_k;
    for (int t = 0; t < T; ++t) {
      const int rc = tsb_moe_decode(spec, experts, static_cast<const uint16_t*>(x) + t * H, 1, router_w, router_b,
                                    ids + t * k, weights + t * k, static_cast<char*>(out) + t * H * out_elem(sp),
                                    workspace, workspace_bytes, stream);
      if (rc) return rc;
    }
    return TSB_OK;
  }
  int rc = check_decode_spec(sp, router_w);
  if (rc) return rc;
  const WsLayout L = ws_layout(sp, T);
  if (workspace_bytes < L.total) return set_error(TSB_ERR_WORKSPACE, "workspace too small");
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return set_error(TSB_ERR_INVALID, "workspace must be 256-byte aligned");
  char* ws = static_cast<char*>(workspace);
  int32_t* err = reinterpret_cast<int32_t*>(ws + L.err);
  float* act = reinterpret_cast<float*>(ws + L.act);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool routed = router_w != nullptr;
  if (routed) {
    rc = launch_router(x, router_w, router_b, sp.hidden, sp.n_experts, T, sp.top_k,
                       reinterpret_cast<float*>(ws + L.logits), ids, weights,
                       reinterpret_cast<unsigned*>(ws + L.counter), st);
    if (rc) return rc;
  }
  rc = launch_gate_up(sp, experts, ids, x, act, err, st, routed);
  if (rc) return rc;
  return launch_down(sp, experts, ids, weights, act, out, err, st, true);
}

size_t tsb_moe_packed_bytes(const TsbMoeSpec* spec) {
  if (!spec || !packable(*spec)) return 0;
  return packed_total_bytes(*spec);
}

int tsb_moe_pack(const TsbMoeSpec* spec, const TsbExpert* experts, void* packed, size_t packed_bytes, void* stream) {
  if (!spec || !experts || !packed) return set_error(TSB_ERR_INVALID, "null pointer");
  const TsbMoeSpec& sp = *spec;
  if (!packable(sp))
    return set_error(TSB_ERR_UNSUPPORTED, "no packed form: needs Q4_K or MXFP4 gate/up and down, H and I multiples of 32 up to 16384");
  int rc = check_decode_spec(sp, nullptr);
  if (rc) return rc;
  if (packed_bytes < tsb_moe_packed_bytes(spec)) return set_error(TSB_ERR_WORKSPACE, "packed buffer too small");
  if (reinterpret_cast<uintptr_t>(packed) & 255) return set_error(TSB_ERR_INVALID, "packed buffer must be 256-byte aligned");
  return launch_pack(sp, experts, packed, static_cast<cudaStream_t>(stream));
}

size_t tsb_moe_decode_packed_workspace(const TsbMoeSpec* spec, int32_t T) {
  if (!spec || T <= 0) return 0;
  if (T > kDecodeLoopMax) return prefill_layout(*spec, T).total;
  return ws_layout(*spec, 1).total + ((packed_ws_bytes(*spec) + 255) & ~size_t(255));
}

int tsb_moe_decode_packed(const TsbMoeSpec* spec, const void* packed, const TsbExpert* experts, const void* x,
                          int32_t T, const void* router_w, const float* router_b, int32_t* ids, float* weights,
                          void* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (!spec || !packed || !experts || !x || !ids || !weights || !out || !workspace)
    return set_error(TSB_ERR_INVALID, "null pointer");
  const TsbMoeSpec& sp = *spec;
  if (T < 1) return set_error(TSB_ERR_INVALID, "T must be >= 1");
  if (!packable(sp)) return set_error(TSB_ERR_UNSUPPORTED, "no packed form for this spec");
  if (T > kDecodeLoopMax)
    return tsb_moe_prefill(spec, experts, x, T, router_w, router_b, ids, weights, out, workspace, workspace_bytes, stream);
  if (T > 1) {
    const int64_t H = sp.hidden, k = sp.top_k;
    for (int t = 0; t < T; ++t) {
      const int rc = tsb_moe_decode_packed(spec, packed, experts, static_cast<const uint16_t*>(x) + t * H, 1, router_w,
                                           router_b, ids + t * k, weights + t * k,
                                           static_cast<char*>(out) + t * H * out_elem(sp), workspace,
                                           workspace_bytes, stream);
      if (rc) return rc;
    }
    return TSB_OK;
  }
  int rc = check_decode_spec(sp, router_w);
  if (rc) return rc;
  const WsLayout L = ws_layout(sp, 1);
  if (workspace_bytes < tsb_moe_decode_packed_workspace(spec, 1)) return set_error(TSB_ERR_WORKSPACE, "workspace too small");
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return set_error(TSB_ERR_INVALID, "workspace must be 256-byte aligned");
  if (reinterpret_cast<uintptr_t>(packed) & 255) return set_error(TSB_ERR_INVALID, "packed buffer must be 256-byte aligned");
  char* ws = static_cast<char*>(workspace);
  int32_t* err = reinterpret_cast<int32_t*>(ws + L.err);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // with router weights, routing runs inside the gate/up launch
  return launch_packed_decode(sp, packed, experts, x, ids, weights, out, sp.out_f32 != 0, err, ws + L.total, st,
                              router_w, router_b);
}

int tsb_read_device_error(void* workspace, int32_t* code, void* stream) {
  if (!workspace || !code) return set_error(TSB_ERR_INVALID, "null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t h = 0;
  cudaError_t e = cudaMemcpyAsync(&h, workspace, sizeof h, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && h) e = cudaMemsetAsync(workspace, 0, sizeof(int32_t), st);
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  *code = h;
  return TSB_OK;
}

int tsb_moe_route(const TsbMoeSpec* spec, const void* x, int32_t T, const void* router_w, const float* router_b,
                  int32_t* ids, float* weights, void* stream) {
  if (!spec) return set_error(TSB_ERR_INVALID, "null pointer");
  if (T < 0) return set_error(TSB_ERR_INVALID, "T must be >= 0");
  if (T == 0) return TSB_OK;
  if (!x || !router_w || !ids || !weights) return set_error(TSB_ERR_INVALID, "null pointer");
  const TsbMoeSpec& sp = *spec;
  if (sp.n_experts < 1 || sp.n_experts > 1024) return set_error(TSB_ERR_INVALID, "n_experts must be in [1, 1024]");
  if (sp.top_k < 1 || sp.top_k > 8 || sp.top_k > sp.n_experts) return set_error(TSB_ERR_INVALID, "top_k must be in [1, min(8, E)]");
  if (sp.hidden <= 0 || sp.hidden % 8) return set_error(TSB_ERR_INVALID, "hidden must be a positive multiple of 8");
  return launch_route(sp, x, T, router_w, router_b, ids, weights, static_cast<cudaStream_t>(stream));
}

size_t tsb_moe_prefill_workspace(const TsbMoeSpec* spec, int32_t T) {
  if (!spec || T < 0) return 0;
  if (dense_spec(*spec)) return T ? dense_layout(*spec, T).total : 0;
  return prefill_layout(*spec, T).total;
}

int tsb_moe_prefill(const TsbMoeSpec* spec, const TsbExpert* experts, const void* x, int32_t T, const void* router_w,
                    const float* router_b, int32_t* ids, float* weights, void* out, void* workspace,
                    size_t workspace_bytes, void* stream) {
  if (!spec) return set_error(TSB_ERR_INVALID, "null pointer");
  if (T < 0) return set_error(TSB_ERR_INVALID, "T must be >= 0");
  if (T == 0) return TSB_OK;
  if (!experts || !x || !ids || !weights || !out || !workspace) return set_error(TSB_ERR_INVALID, "null pointer");
  const TsbMoeSpec& sp = *spec;
  if (is_dense_fmt(sp.fmt_gate_up) || is_dense_fmt(sp.fmt_down))
    return dense_layer(sp, experts, x, T, router_w, router_b, ids, weights, out, workspace, workspace_bytes, stream);
  if (sp.transposed) return set_error(TSB_ERR_INVALID, "transposed applies to dense formats only");
  if (sp.n_experts < 1 || sp.n_experts > 1024) return set_error(TSB_ERR_INVALID, "n_experts must be in [1, 1024]");
  if (sp.top_k < 1 || sp.top_k > 8 || sp.top_k > sp.n_experts) return set_error(TSB_ERR_INVALID, "top_k must be in [1, min(8, E)]");
  if (sp.hidden % 32 || sp.inter % 32 || sp.hidden <= 0 || sp.inter <= 0)
    return set_error(TSB_ERR_INVALID, "hidden and inter must be positive multiples of 32");
  if (sp.gate_up_layout < 0 || sp.gate_up_layout > 2) return set_error(TSB_ERR_INVALID, "bad gate_up_layout");
  if (sp.activation < 0 || sp.activation > 1) return set_error(TSB_ERR_INVALID, "bad activation");
  if (sp.out_f32 != 0 && sp.out_f32 != 1) return set_error(TSB_ERR_INVALID, "out_f32 must be 0 or 1");
  if ((int64_t)T * sp.top_k > (int64_t)1 << 26) return set_error(TSB_ERR_UNSUPPORTED, "T * top_k too large");
  int rc = check_shape(sp.fmt_gate_up, sp.inter, sp.hidden);
  if (rc) return rc;
  rc = check_shape(sp.fmt_down, sp.hidden, sp.inter);
  if (rc) return rc;
  const PrefillLayout L = prefill_layout(sp, T);
  if (!L.nt_gu || !L.nt_dn) return set_error(TSB_ERR_UNSUPPORTED, "no tensor-core tile divides hidden / inter");
  if (workspace_bytes < L.total) return set_error(TSB_ERR_WORKSPACE, "workspace too small");
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return set_error(TSB_ERR_INVALID, "workspace must be 256-byte aligned");
  return launch_moe_prefill(sp, experts, x, T, router_w, router_b, ids, weights, out, static_cast<char*>(workspace), L,
                            static_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free variant of tsb_moe_decode.
//
// Some callers have no device scratch memory to hand over: hosts whose
// memory is planned ahead and that forbid any allocation behind their back,
// or language bindings that only ever see the tensors they pass in.  For them
// the workspace lives in this file-scope device array, sized for one layer of
// up to kNoAllocBytes of scratch; the entry point calls neither cudaMalloc
// nor cudaFree.
// ---------------------------------------------------------------------------
namespace tsb {
constexpr size_t kNoAllocBytes = size_t(1) << 20;  // 1 MiB, held on every GPU that loads the library
static __device__ __align__(256) unsigned char g_noalloc_ws[kNoAllocBytes];

static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[64];  // device address of g_noalloc_ws, per device ordinal
}  // namespace tsb

extern "C" int tsb_moe_decode_noalloc(const TsbMoeSpec* spec, const TsbExpert* experts, const void* x, int32_t T,
                                      const void* router_w, const float* router_b, int32_t* ids, float* weights,
                                      void* out, void* stream) {
  using namespace tsb;
  if (!spec) return set_error(TSB_ERR_INVALID, "null pointer");
  const size_t need = tsb_moe_decode_workspace(spec, T);
  if (need == 0) return set_error(TSB_ERR_INVALID, "T must be positive");
  if (need > kNoAllocBytes) {
    char buf[160];
    snprintf(buf, sizeof buf, "tsb_moe_decode_noalloc: this layer needs %zu bytes of scratch, more than the %zu-byte static workspace",
             need, kNoAllocBytes);
    return set_error(TSB_ERR_WORKSPACE, buf);
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_error(TSB_ERR_UNSUPPORTED, "device ordinal out of range");
  void* ws = nullptr;
  {
    // First call on a device: look up the array's device address with that
    // device current (the host-side symbol is not a device address).
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_ws);
      if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
      g_noalloc_ptr[dev] = p;
    }
    ws = g_noalloc_ptr[dev];
  }
  // The array keeps the previous call's contents: clear the error word and the
  // counters at its start, which must begin at zero.
  e = cudaMemsetAsync(ws, 0, 256, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  return tsb_moe_decode(spec, experts, x, T, router_w, router_b, ids, weights, out, ws, kNoAllocBytes, stream);
}
