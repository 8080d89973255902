// Dense (fp32 / fp16 / bf16) expert layers: the unquantised counterpart of
// the quantised decode path, for checkpoints whose experts are plain float
// tensors.
//
// Reference behaviour (tinyserve/expert_forward.py:109-194, the template
// forward tinyserve/_model_hooks.py:376-412 and the C++ loop
// tinyserve/csrc/expert_loop.cpp:41-123): gate_up = x @ W_gu^T (+ b_gu), the
// activation (SiLU over chunked halves, or the GPT-OSS clamp-SwiGLU over
// interleaved columns), down = act @ W_dn^T (+ b_dn), and the routed experts'
// outputs summed with the routing weights.  The reference accepts a weight in
// either orientation ([out, in], as nn.Linear stores it, or [in, out] with a
// transpose before F.linear, expert_forward.py:140-149); both are read in
// place here, selected per projection by TsbMoeSpec.transposed.
//
// Design: every token-slot (token t, routing slot j) is one unit u = t*k + j.
// All units of a call run in one launch per projection, fp32 accumulation.
//  * [out, in] weights: one warp per output row, 16-byte loads along the row,
//    the input vector staged once per CTA in shared memory (fp32), a warp
//    shuffle reduction.  Gate/up runs its epilogue (biases, activation) in
//    place; down writes one fp32 partial row per unit.
//  * [in, out] weights: each thread owns 16 bytes of output columns and walks
//    a slice of the input rows (coalesced 4 KB row segments per CTA); K is
//    split into S slices so the grid covers the GPU, the partials land in the
//    workspace and a small pass sums them in slice order (deterministic).
//  * combine: out[t] = sum_j w[t,j] * (sum_s P[s][u] + b_dn[e]) in slot order.
// HBM-bound: the algorithmic bytes are the routed experts' weight bytes.
#include "../../include/tsb_moe.h"
#include "moe_math.cuh"
#include "tsb_common.cuh"
#include "tsb_internal.h"

namespace tsb {

bool is_dense_fmt(int f) { return f == TSB_FMT_F32 || f == TSB_FMT_F16 || f == TSB_FMT_BF16; }

__host__ __device__ __forceinline__ int dense_elem_bytes(int f) { return f == TSB_FMT_F32 ? 4 : 2; }

namespace {

constexpr int kRowsWarps = 8;    // warps (= output rows) per CTA, row-major kernels
constexpr int kColThreads = 256;  // threads per CTA, column kernels

// 16 bytes of weights -> V floats (V = 4 for fp32, 8 for 16-bit types).
template <int FMT> struct Vec { static constexpr int V = 8; };
template <> struct Vec<TSB_FMT_F32> { static constexpr int V = 4; };

template <int FMT>
__device__ __forceinline__ void unpack16(const uint4 w, float (&f)[Vec<FMT>::V]) {
  const uint32_t q[4] = {w.x, w.y, w.z, w.w};
  if constexpr (FMT == TSB_FMT_F32) {
#pragma unroll
    for (int i = 0; i < 4; ++i) f[i] = __uint_as_float(q[i]);
  } else if constexpr (FMT == TSB_FMT_BF16) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(q[i] << 16);
      f[2 * i + 1] = __uint_as_float(q[i] & 0xFFFF0000u);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 h = __half22float2(*reinterpret_cast<const __half2*>(&q[i]));
      f[2 * i] = h.x;
      f[2 * i + 1] = h.y;
    }
  }
}

__device__ __forceinline__ bool misaligned(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) != 0; }

__device__ __forceinline__ void flag(int32_t* err, int code) {
  if (err) atomicExch(err, code);
}

struct DenseArgs {
  const TsbExpert* experts;
  const int32_t* ids;     // [T, k]
  const float* wts;       // [T, k]
  const uint16_t* x;      // bf16 [T, H]
  float* act;             // fp32 [U, I]
  float* part;            // fp32 partials [S, U, C]
  void* out;              // [T, H] bf16 or fp32
  int32_t* err;
  int H, I, E, k, U;
  int layout, activation;
  float limit, alpha;
  int out_f32;
  int S;                  // K slices of the column kernels
  int kslice;             // input rows per slice
};

// Output column c of the (virtual) gate/up matrix -> (weight base, column in it,
// row stride).  Separate gate and up form a chunked [2I] column space.
__device__ __forceinline__ int gu_gate_col(int layout, int i, int I) { return layout == TSB_GU_INTERLEAVED ? 2 * i : i; }
__device__ __forceinline__ int gu_up_col(int layout, int i, int I) { return layout == TSB_GU_INTERLEAVED ? 2 * i + 1 : I + i; }

// Expert id of unit u, or -1 for a skipped slot (and -1 with the error word set
// for an id outside [0, E)).
__device__ __forceinline__ int unit_expert(const DenseArgs& a, int u) {
  const int e = a.ids[u];
  if (e >= a.E) {
    flag(a.err, kDevBadPlan);
    return -1;
  }
  return e;
}

// Stage n floats of an input vector (bf16 or fp32) into shared memory.
__device__ __forceinline__ void stage_bf16(float* s, const uint16_t* src, int n) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) s[i] = __uint_as_float(static_cast<uint32_t>(src[i]) << 16);
}
__device__ __forceinline__ void stage_f32(float* s, const float* src, int n) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) s[i] = src[i];
}

// Dot of one weight row (n elements, 16-byte aligned) with a shared-memory vector,
// reduced across the warp (every lane gets the sum).
template <int FMT>
__device__ __forceinline__ float warp_row_dot(const void* row, const float* xs, int n) {
  constexpr int V = Vec<FMT>::V;
  const uint4* w = static_cast<const uint4*>(row);
  const int nv = n / V, lane = threadIdx.x & 31;
  float acc0 = 0.f, acc1 = 0.f;
  int c = lane;
  for (; c + 32 < nv; c += 64) {
    const uint4 w0 = __ldcs(w + c), w1 = __ldcs(w + c + 32);
    float f0[V], f1[V];
    unpack16<FMT>(w0, f0);
    unpack16<FMT>(w1, f1);
#pragma unroll
    for (int v = 0; v < V; ++v) {
      acc0 = fmaf(f0[v], xs[c * V + v], acc0);
      acc1 = fmaf(f1[v], xs[(c + 32) * V + v], acc1);
    }
  }
  if (c < nv) {
    float f0[V];
    unpack16<FMT>(__ldcs(w + c), f0);
#pragma unroll
    for (int v = 0; v < V; ++v) acc0 = fmaf(f0[v], xs[c * V + v], acc0);
  }
  float acc = acc0 + acc1;
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  return acc;
}

// ---- [out, in] weights -------------------------------------------------------

// grid (ceil(I / 8), U): warp w of block (bx, u) computes activation i = 8*bx + w of unit u.
template <int FMT>
__global__ void __launch_bounds__(kRowsWarps * 32) dense_gu_rows(DenseArgs a) {
  extern __shared__ float xs[];
  const int u = blockIdx.y, e = unit_expert(a, u);
  if (e < 0) return;
  stage_bf16(xs, a.x + (int64_t)(u / a.k) * a.H, a.H);
  __syncthreads();
  const int i = blockIdx.x * kRowsWarps + (threadIdx.x >> 5);
  if (i >= a.I) return;
  const TsbExpert ex = a.experts[e];
  const char* base = static_cast<const char*>(ex.gate);
  const int64_t rb = (int64_t)a.H * dense_elem_bytes(FMT);  // bytes per row
  const char *g, *up;
  if (a.layout == TSB_GU_SEPARATE) {
    g = base + i * rb;
    up = static_cast<const char*>(ex.up) + i * rb;
  } else {
    g = base + gu_gate_col(a.layout, i, a.I) * rb;
    up = base + gu_up_col(a.layout, i, a.I) * rb;
  }
  if (misaligned(g) || misaligned(up)) {
    if ((threadIdx.x & 31) == 0) flag(a.err, kDevMisaligned);
    return;
  }
  float gv = warp_row_dot<FMT>(g, xs, a.H);
  float uv = warp_row_dot<FMT>(up, xs, a.H);
  if ((threadIdx.x & 31) == 0) {
    if (ex.gate_bias) gv += ex.gate_bias[i];
    if (ex.up_bias) uv += ex.up_bias[i];
    a.act[(int64_t)u * a.I + i] = act_fn(a.activation, gv, uv, a.limit, a.alpha);
  }
}

// grid (ceil(H / 8), U): warp w of block (bx, u) computes down output h = 8*bx + w
// of unit u (no bias; the combine adds it) into part[u][h].
template <int FMT>
__global__ void __launch_bounds__(kRowsWarps * 32) dense_dn_rows(DenseArgs a) {
  extern __shared__ float xs[];
  const int u = blockIdx.y, e = unit_expert(a, u);
  if (e < 0) return;
  stage_f32(xs, a.act + (int64_t)u * a.I, a.I);
  __syncthreads();
  const int h = blockIdx.x * kRowsWarps + (threadIdx.x >> 5);
  if (h >= a.H) return;
  const char* row = static_cast<const char*>(a.experts[e].down) + (int64_t)h * a.I * dense_elem_bytes(FMT);
  if (misaligned(row)) {
    if ((threadIdx.x & 31) == 0) flag(a.err, kDevMisaligned);
    return;
  }
  const float y = warp_row_dot<FMT>(row, xs, a.I);
  if ((threadIdx.x & 31) == 0) a.part[(int64_t)u * a.H + h] = y;
}

// ---- [in, out] weights ---------------------------------------------------------

// Partial products of input rows [s*kslice, min(K, (s+1)*kslice)) for V output
// columns per thread: P[s][u][c..c+V) (C columns).  grid (ceil(C / (256 V)), S, U).
// GATEUP: K = H, columns are the gate/up output space (separate gate and up read as
// the two halves of a chunked space); else down: K = I, C = H.
template <int FMT, bool GATEUP>
__global__ void __launch_bounds__(kColThreads) dense_cols(DenseArgs a) {
  constexpr int V = Vec<FMT>::V;
  extern __shared__ float xs[];
  const int u = blockIdx.z, e = unit_expert(a, u);
  if (e < 0) return;
  const int K = GATEUP ? a.H : a.I, C = GATEUP ? 2 * a.I : a.H;
  const int r0 = blockIdx.y * a.kslice, r1 = min(K, r0 + a.kslice);
  if (GATEUP)
    stage_bf16(xs, a.x + (int64_t)(u / a.k) * a.H + r0, r1 - r0);
  else
    stage_f32(xs, a.act + (int64_t)u * a.I + r0, r1 - r0);
  __syncthreads();
  const int c = (blockIdx.x * kColThreads + threadIdx.x) * V;
  if (c >= C) return;
  const TsbExpert ex = a.experts[e];
  const char* base;
  int ldc, cc;  // row length (elements) and column within that matrix
  if (!GATEUP) {
    base = static_cast<const char*>(ex.down);
    ldc = a.H;
    cc = c;
  } else if (a.layout == TSB_GU_SEPARATE) {
    base = static_cast<const char*>(c < a.I ? ex.gate : ex.up);
    ldc = a.I;
    cc = c < a.I ? c : c - a.I;
  } else {
    base = static_cast<const char*>(ex.gate);
    ldc = C;
    cc = c;
  }
  const int eb = dense_elem_bytes(FMT);
  const char* p = base + ((int64_t)r0 * ldc + cc) * eb;
  if (misaligned(base)) {
    flag(a.err, kDevMisaligned);
    return;
  }
  const int64_t stride = (int64_t)ldc * eb;
  float acc[V];
#pragma unroll
  for (int v = 0; v < V; ++v) acc[v] = 0.f;
  int r = r0;
  for (; r + 4 <= r1; r += 4) {
    uint4 w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) w[j] = __ldcs(reinterpret_cast<const uint4*>(p + j * stride));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float f[V];
      unpack16<FMT>(w[j], f);
      const float xv = xs[r - r0 + j];
#pragma unroll
      for (int v = 0; v < V; ++v) acc[v] = fmaf(f[v], xv, acc[v]);
    }
    p += 4 * stride;
  }
  for (; r < r1; ++r, p += stride) {
    float f[V];
    unpack16<FMT>(__ldcs(reinterpret_cast<const uint4*>(p)), f);
    const float xv = xs[r - r0];
#pragma unroll
    for (int v = 0; v < V; ++v) acc[v] = fmaf(f[v], xv, acc[v]);
  }
  float* dst = a.part + ((int64_t)blockIdx.y * a.U + u) * C + c;
#pragma unroll
  for (int v = 0; v < V; v += 4) *reinterpret_cast<float4*>(dst + v) = make_float4(acc[v], acc[v + 1], acc[v + 2], acc[v + 3]);
}

// Sum the S gate/up partials of activation i of unit u in slice order, add the
// biases and apply the activation.  grid (ceil(I / 256), U).
__global__ void __launch_bounds__(256) dense_gu_finish(DenseArgs a) {
  const int u = blockIdx.y, i = blockIdx.x * 256 + threadIdx.x;
  if (i >= a.I) return;
  const int e = a.ids[u];
  if (e < 0 || e >= a.E) return;
  const int C = 2 * a.I, gc = gu_gate_col(a.layout, i, a.I), uc = gu_up_col(a.layout, i, a.I);
  float gv = 0.f, uv = 0.f;
  for (int s = 0; s < a.S; ++s) {
    const float* P = a.part + ((int64_t)s * a.U + u) * C;
    gv += P[gc];
    uv += P[uc];
  }
  const TsbExpert& ex = a.experts[e];
  if (ex.gate_bias) gv += ex.gate_bias[i];
  if (ex.up_bias) uv += ex.up_bias[i];
  a.act[(int64_t)u * a.I + i] = act_fn(a.activation, gv, uv, a.limit, a.alpha);
}

// out[t][h] = sum_j w[t,j] * (sum_s P[s][t*k+j][h] + b_dn[e_j][h]), slots in order,
// skipped slots (negative ids) contribute nothing.  grid (ceil(H / 256), T).
__global__ void __launch_bounds__(256) dense_combine(DenseArgs a) {
  const int t = blockIdx.y, h = blockIdx.x * 256 + threadIdx.x;
  if (h >= a.H) return;
  float y = 0.f;
  for (int j = 0; j < a.k; ++j) {
    const int u = t * a.k + j, e = a.ids[u];
    if (e < 0 || e >= a.E) continue;
    float v = 0.f;
    for (int s = 0; s < a.S; ++s) v += a.part[((int64_t)s * a.U + u) * a.H + h];
    const float* b = a.experts[e].down_bias;
    if (b) v += b[h];
    y = fmaf(a.wts[u], v, y);
  }
  if (a.out_f32)
    static_cast<float*>(a.out)[(int64_t)t * a.H + h] = y;
  else
    static_cast<uint16_t*>(a.out)[(int64_t)t * a.H + h] = f32_to_bf16_bits(y);
}

int sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// K slices for a column kernel: enough CTAs for about four per SM, at least 32
// input rows per slice.
int col_slices(int C, int K, int U, int V) {
  const int ctas = (C + kColThreads * V - 1) / (kColThreads * V) * U;
  int S = (4 * sms() + ctas - 1) / ctas;
  S = S < 1 ? 1 : S;
  const int smax = K / 32 > 0 ? K / 32 : 1;
  return S > smax ? smax : S;
}

int vec_of(int fmt) { return fmt == TSB_FMT_F32 ? 4 : 8; }

cudaError_t set_smem(const void* fn, size_t bytes) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

template <int FMT>
cudaError_t run_gate_up(const DenseArgs& a, bool transposed, int S, cudaStream_t st) {
  if (!transposed) {
    const size_t smem = sizeof(float) * a.H;
    cudaError_t e = set_smem((const void*)dense_gu_rows<FMT>, smem);
    if (e != cudaSuccess) return e;
    dense_gu_rows<FMT><<<dim3((a.I + kRowsWarps - 1) / kRowsWarps, a.U), kRowsWarps * 32, smem, st>>>(a);
    return cudaGetLastError();
  }
  DenseArgs b = a;
  b.S = S;
  b.kslice = (a.H + S - 1) / S;
  const size_t smem = sizeof(float) * b.kslice;
  cudaError_t e = set_smem((const void*)dense_cols<FMT, true>, smem);
  if (e != cudaSuccess) return e;
  const int C = 2 * a.I, V = Vec<FMT>::V;
  dense_cols<FMT, true><<<dim3((C + kColThreads * V - 1) / (kColThreads * V), S, a.U), kColThreads, smem, st>>>(b);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  dense_gu_finish<<<dim3((a.I + 255) / 256, a.U), 256, 0, st>>>(b);
  return cudaGetLastError();
}

template <int FMT>
cudaError_t run_down(const DenseArgs& a, bool transposed, int S, cudaStream_t st) {
  if (!transposed) {
    const size_t smem = sizeof(float) * a.I;
    cudaError_t e = set_smem((const void*)dense_dn_rows<FMT>, smem);
    if (e != cudaSuccess) return e;
    dense_dn_rows<FMT><<<dim3((a.H + kRowsWarps - 1) / kRowsWarps, a.U), kRowsWarps * 32, smem, st>>>(a);
    return cudaGetLastError();
  }
  DenseArgs b = a;
  b.S = S;
  b.kslice = (a.I + S - 1) / S;
  const size_t smem = sizeof(float) * b.kslice;
  cudaError_t e = set_smem((const void*)dense_cols<FMT, false>, smem);
  if (e != cudaSuccess) return e;
  const int V = Vec<FMT>::V;
  dense_cols<FMT, false><<<dim3((a.H + kColThreads * V - 1) / (kColThreads * V), S, a.U), kColThreads, smem, st>>>(b);
  return cudaGetLastError();
}

}  // namespace

DenseLayout dense_layout(const TsbMoeSpec& sp, int T) {
  auto al = [](size_t v) { return (v + 255) & ~size_t(255); };
  DenseLayout L;
  const int U = T * sp.top_k;
  L.s_gu = (sp.transposed & TSB_T_GATE_UP) ? col_slices(2 * sp.inter, sp.hidden, U, vec_of(sp.fmt_gate_up)) : 0;
  L.s_dn = (sp.transposed & TSB_T_DOWN) ? col_slices(sp.hidden, sp.inter, U, vec_of(sp.fmt_down)) : 1;
  L.err = 0;
  L.counter = 4;
  L.logits = 256;
  L.act = L.logits + al(sizeof(float) * (size_t)T * sp.n_experts);
  L.part = L.act + al(sizeof(float) * (size_t)U * sp.inter);
  const size_t p_gu = (size_t)L.s_gu * U * 2 * sp.inter, p_dn = (size_t)L.s_dn * U * sp.hidden;
  L.total = L.part + al(sizeof(float) * (p_gu > p_dn ? p_gu : p_dn));
  return L;
}

int launch_dense_layer(const TsbMoeSpec& sp, const TsbExpert* ex, const void* x, int T, const void* router_w,
                       const float* router_b, int32_t* ids, float* wts, void* out, char* ws, const DenseLayout& L,
                       cudaStream_t st) {
  const int H = sp.hidden, I = sp.inter;
  if (sp.hidden > 16384 || sp.inter > 16384) return set_error(TSB_ERR_UNSUPPORTED, "dense experts: hidden and inter must be <= 16384");
  int32_t* err = reinterpret_cast<int32_t*>(ws + L.err);
  if (router_w) {
    const int rc = launch_router(x, router_w, router_b, H, sp.n_experts, T, sp.top_k,
                                 reinterpret_cast<float*>(ws + L.logits), ids, wts,
                                 reinterpret_cast<unsigned*>(ws + L.counter), st);
    if (rc) return rc;
  }
  DenseArgs a{};
  a.experts = ex;
  a.ids = ids;
  a.wts = wts;
  a.x = static_cast<const uint16_t*>(x);
  a.act = reinterpret_cast<float*>(ws + L.act);
  a.part = reinterpret_cast<float*>(ws + L.part);
  a.out = out;
  a.err = err;
  a.H = H;
  a.I = I;
  a.E = sp.n_experts;
  a.k = sp.top_k;
  a.U = T * sp.top_k;
  a.layout = sp.gate_up_layout;
  a.activation = sp.activation;
  a.limit = sp.limit;
  a.alpha = sp.alpha;
  a.out_f32 = sp.out_f32;
  a.S = 1;
  a.kslice = 0;
  const bool tgu = sp.transposed & TSB_T_GATE_UP, tdn = sp.transposed & TSB_T_DOWN;
  cudaError_t e;
  switch (sp.fmt_gate_up) {
    case TSB_FMT_F32: e = run_gate_up<TSB_FMT_F32>(a, tgu, L.s_gu, st); break;
    case TSB_FMT_F16: e = run_gate_up<TSB_FMT_F16>(a, tgu, L.s_gu, st); break;
    default: e = run_gate_up<TSB_FMT_BF16>(a, tgu, L.s_gu, st); break;
  }
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  switch (sp.fmt_down) {
    case TSB_FMT_F32: e = run_down<TSB_FMT_F32>(a, tdn, L.s_dn, st); break;
    case TSB_FMT_F16: e = run_down<TSB_FMT_F16>(a, tdn, L.s_dn, st); break;
    default: e = run_down<TSB_FMT_BF16>(a, tdn, L.s_dn, st); break;
  }
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  a.S = L.s_dn;
  dense_combine<<<dim3((H + 255) / 256, T), 256, 0, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  return TSB_OK;
}

}  // namespace tsb
