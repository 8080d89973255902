// Decode-side kernels and launchers: plain quantised matvec, router, fused
// gate/up + activation, fused down + weighted top-k combine.
#include <algorithm>
#include <cstdio>

#include "../../include/tsb_moe.h"
#include "moe_math.cuh"
#include "qmv_engine.cuh"
#include "tsb_internal.h"

namespace tsb {

// ------------------------------------------------------------------ config
constexpr int kNCW = 16;
constexpr int kNStage = 4;
constexpr int kStageBytes = 32768;
constexpr int kNStageWide = 5;
constexpr int kWarpNW = 8;          // warps of the warp-owned variant
constexpr int kWarpBuf = 10240;     // bytes per warp buffer (two per warp)   // stages of whole-row single/diagonal-vector plans
constexpr int kGroupsWide = 4;   // consumer groups of those plans

__device__ __forceinline__ float load_act(const void* p, int dtype, int64_t i) {
  if (dtype == TSB_DT_F32) return static_cast<const float*>(p)[i];
  if (dtype == TSB_DT_BF16) return bf16_bits_to_f32(static_cast<const uint16_t*>(p)[i]);
  return __half2float(static_cast<const __half*>(p)[i]);
}

__device__ __forceinline__ void store_out(void* p, int dtype, int64_t i, float v) {
  if (dtype == TSB_DT_F32) static_cast<float*>(p)[i] = v;
  else if (dtype == TSB_DT_BF16) static_cast<uint16_t*>(p)[i] = f32_to_bf16_bits(v);
  else static_cast<__half*>(p)[i] = __float2half_rn(v);
}


// Expert id from a routing table, validated: an id outside [0, E) (a corrupt
// caller-provided table) records kDevBadPlan and yields -1 so the tile holds no rows.
__device__ __forceinline__ int safe_expert(const int32_t* ids, int i, int E, int* err) {
  const int e = ids[i];
  if ((unsigned)e >= (unsigned)E) {
    if (err && e >= 0) atomicExch(err, kDevBadPlan);  // negative: a skipped slot
    return -1;
  }
  return e;
}

// ------------------------------------------------------------------ plans
template <int F>
struct PlanMatvec {
  StageGeom geom;
  int* err;
  static constexpr bool kProducerWaits = false;
  static constexpr bool kXIndependent = true;
  const uint8_t* w;
  const uint8_t* s;
  int64_t N, mat_bytes;
  const void* x;
  int x_dtype, nv, x_vec_ok;
  int64_t x_stride;
  void* y;
  int y_dtype;
  int64_t y_stride;

  __device__ int num_vectors() const { return nv; }
  __device__ XSrc xsrc() const { return XSrc{x, x_stride, x_dtype, x_vec_ok}; }
  __device__ int num_blocks() const { return (int)((N + 15) / 16); }
  __device__ int nseg(int) const { return 1; }
  __device__ void fill_cache(SlotCache*, int) const {}
  __device__ Seg seg(const SlotCache*, int rb, int) const {
    return Seg{w, s, 16 * (int64_t)rb, (int)(N - 16 * (int64_t)rb < 16 ? N - 16 * (int64_t)rb : 16), mat_bytes};
  }
  __device__ void rowmap(int, int m, int& sg, int& lr) const { sg = 0; lr = m; }
  __device__ void columns(int, int g, int t, int& vb, int& v0, int& v1, int& na, int& nb) const {
    vb = min(g, nv - 1);
    v0 = min(2 * t, nv - 1);
    v1 = min(2 * t + 1, nv - 1);
    na = nb = 0;
  }
  __device__ void epilogue(const SlotCache*, int rb, const float* rd, int nw, int lane) const {
    if (nv == 1) {
      const int64_t row = 16 * (int64_t)rb + lane;
      if (lane >= 16 || row >= N) return;
      float v = 0.f;
      for (int i = 0; i < nw; ++i) v += rd[i * 16 + lane];
      store_out(y, y_dtype, row, v);
      return;
    }
    for (int c = lane; c < 128; c += 32) {
      const int m = c >> 3, n = c & 7;
      const int64_t row = 16 * (int64_t)rb + m;
      if (row >= N || n >= nv) continue;
      float v = 0.f;
      for (int i = 0; i < nw; ++i) v += rd[i * 128 + c];
      store_out(y, y_dtype, n * y_stride + row, v);
    }
  }
};

template <int F>
struct PlanGateUp {
  StageGeom geom;
  int* err;
  static constexpr bool kProducerWaits = true;  // expert ids come from the router kernel
  static constexpr bool kXIndependent = true;   // x was written before the router ran
  const TsbExpert* experts;
  const int32_t* ids;
  int n_experts;
  int top_k, I, layout, act;
  float limit, alpha;
  const uint16_t* x;  // bf16 [H]
  int x_vec_ok;
  float* act_out;     // [top_k, I]
  int64_t gu_bytes, up_bytes;
  int tpe;  // row blocks per expert

  __device__ int num_vectors() const { return 1; }
  __device__ XSrc xsrc() const { return XSrc{x, 0, TSB_DT_BF16, x_vec_ok}; }
  __device__ int num_blocks() const { return top_k * tpe; }
  __device__ int nseg(int) const { return layout == TSB_GU_INTERLEAVED ? 1 : 2; }
  __device__ void fill_cache(SlotCache* c, int lane) const {
    if (lane >= top_k) return;
    const int e = safe_expert(ids, lane, n_experts, err);
    const TsbExpert& E = experts[e < 0 ? 0 : e];
    SlotCache s;
    s.w[0] = static_cast<const uint8_t*>(E.gate);
    s.w[1] = static_cast<const uint8_t*>(E.up);
    s.s[0] = static_cast<const uint8_t*>(E.gate_scales);
    s.s[1] = static_cast<const uint8_t*>(E.up_scales);
    s.b[0] = E.gate_bias;
    s.b[1] = E.up_bias;
    s.e = e;
    s.pad = 0;
    c[lane] = s;
  }
  __device__ Seg seg(const SlotCache* c, int rb, int s) const {
    const int u = rb / tpe, j0 = 8 * (rb % tpe);
    const SlotCache& C = c[u];
    const int nr = C.e < 0 ? 0 : min(8, I - j0);
    if (layout == TSB_GU_INTERLEAVED) return Seg{C.w[0], C.s[0], 2 * (int64_t)j0, 2 * nr, gu_bytes};
    if (layout == TSB_GU_CHUNKED) return Seg{C.w[0], C.s[0], (int64_t)(s ? I + j0 : j0), nr, gu_bytes};
    if (s == 0) return Seg{C.w[0], C.s[0], (int64_t)j0, nr, gu_bytes};
    return Seg{C.w[1], C.s[1], (int64_t)j0, nr, up_bytes};
  }
  // Fragment rows g and g+8 must be source rows 8 apart (they share one
  // superblock-phase counter when K % 256 != 0), so interleaved rows keep
  // their order: A row m = gate_up row 2*j0 + m, and the epilogue pairs rows
  // 2i (gate) and 2i+1 (up).
  __device__ void rowmap(int, int m, int& sg, int& lr) const {
    if (layout == TSB_GU_INTERLEAVED) {
      sg = 0;
      lr = m;
    } else {
      sg = m >> 3;
      lr = m & 7;
    }
  }
  __device__ void columns(int, int, int, int& vb, int& v0, int& v1, int& na, int& nb) const {
    vb = v0 = v1 = 0;
    na = nb = 0;
  }
  __device__ void epilogue(const SlotCache* c, int rb, const float* rd, int nw, int lane) const {
    if (lane >= 8) return;
    const int u = rb / tpe, j = 8 * (rb % tpe) + lane;
    if (j >= I) return;
    const int rg = layout == TSB_GU_INTERLEAVED ? 2 * lane : lane;
    const int ru = layout == TSB_GU_INTERLEAVED ? 2 * lane + 1 : lane + 8;
    float gate = 0.f, up = 0.f;
    for (int i = 0; i < nw; ++i) {
      gate += rd[i * 16 + rg];
      up += rd[i * 16 + ru];
    }
    const SlotCache& C = c[u];
    if (C.e < 0) { act_out[(int64_t)u * I + j] = 0.f; return; }
    if (C.b[0]) gate += C.b[0][j];
    if (C.b[1]) up += C.b[1][j];
    act_out[(int64_t)u * I + j] = act_fn(act, gate, up, limit, alpha);
  }
};

template <int F>
struct PlanDownT1 {
  StageGeom geom;
  int* err;
  // Expert ids were written two kernels back (router) or before the chain
  // started, so weight streaming may begin before the gate/up kernel ends.
  static constexpr bool kProducerWaits = false;
  static constexpr bool kXIndependent = false;  // activations come from the gate/up kernel
  const TsbExpert* experts;
  const int32_t* ids;
  const float* wts;
  int n_experts;
  int top_k, rpe, H, I;
  const float* act;  // [top_k, I]
  int act_cg;        // act written by other CTAs of this grid: load through L2 (0 here)
  void* out;         // [H], bf16 or fp32 (out_f32)
  int out_f32;
  int64_t dn_bytes;

  __device__ int num_vectors() const { return top_k; }
  __device__ XSrc xsrc() const { return XSrc{act, I, TSB_DT_F32, 1, act_cg}; }
  __device__ int num_blocks() const { return (H + rpe - 1) / rpe; }
  __device__ int nseg(int) const { return top_k; }
  __device__ void fill_cache(SlotCache* c, int lane) const {
    if (lane >= top_k) return;
    const int e = safe_expert(ids, lane, n_experts, err);
    const TsbExpert& E = experts[e < 0 ? 0 : e];
    SlotCache s;
    s.w[0] = static_cast<const uint8_t*>(E.down);
    s.w[1] = nullptr;
    s.s[0] = static_cast<const uint8_t*>(E.down_scales);
    s.s[1] = nullptr;
    s.b[0] = E.down_bias;
    s.b[1] = nullptr;
    s.e = e;
    s.pad = 0;
    c[lane] = s;
  }
  __device__ Seg seg(const SlotCache* c, int rb, int s) const {
    const SlotCache& C = c[s];
    const int h0 = rpe * rb;
    return Seg{C.w[0], C.s[0], (int64_t)h0, C.e < 0 ? 0 : min(rpe, H - h0), dn_bytes};
  }
  __device__ void rowmap(int, int m, int& sg, int& lr) const {
    sg = m / rpe;
    lr = m % rpe;
    if (sg >= top_k) sg = -1;
  }
  __device__ void columns(int, int g, int, int& vb, int& v0, int& v1, int& na, int& nb) const {
    vb = g < top_k ? g : 0;
    v0 = v1 = 0;
    na = (g / rpe < top_k) ? g / rpe : -1;
    nb = ((g + 8) / rpe < top_k) ? (g + 8) / rpe : -1;
  }
  __device__ void epilogue(const SlotCache* c, int rb, const float* rd, int nw, int lane) const {
    if (lane >= rpe) return;
    const int h = rpe * rb + lane;
    if (h >= H) return;
    float o = 0.f;
    for (int k = 0; k < top_k; ++k) {
      float v = 0.f;
      for (int i = 0; i < nw; ++i) v += rd[i * 16 + k * rpe + lane];
      const SlotCache& C = c[k];
      if (C.e < 0) continue;
      if (C.b[0]) v += C.b[0][h];
      o = fmaf(wts[k], v, o);
    }
    if (out_f32)
      static_cast<float*>(out)[h] = o;
    else
      static_cast<uint16_t*>(out)[h] = f32_to_bf16_bits(o);
  }
};

// ------------------------------------------------------------------ router
// logits[t, e] = bf16(x[t] . W[e] + b[e]) with one CTA per (token, expert): the
// four warps split H and issue all their loads before reducing, so a logit
// costs one memory round trip.  The last CTA to finish selects the top-k per
// token (ties -> lower expert id; NaN sorts lowest) and softmaxes the k
// selected logits (tinyserve/_model_hooks.py:466-473).
__global__ void __launch_bounds__(128) router_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ W,
                                                     const float* __restrict__ b, int H, int E, int T, int top_k,
                                                     float* logits, int32_t* ids, float* wts, unsigned* counter) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int p = blockIdx.x;
  const int t = p / E, e = p % E;
  const int n8 = H / 8;
  const int per = (n8 + 3) / 4;
  const int i0 = warp * per, i1 = min(n8, i0 + per);
  const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)t * H);
  const uint4* wr = reinterpret_cast<const uint4*>(W + (int64_t)e * H);
  constexpr int kU = 8;
  float acc = 0.f;
  for (int base = i0 + lane; base < i1; base += 32 * kU) {
    uint4 a[kU], w[kU];
#pragma unroll
    for (int j = 0; j < kU; ++j) {
      const int i = base + 32 * j;
      if (i < i1) {
        a[j] = xr[i];
        w[j] = __ldg(wr + i);
      } else {
        a[j] = make_uint4(0, 0, 0, 0);
        w[j] = make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int j = 0; j < kU; ++j) {
      const uint32_t av[4] = {a[j].x, a[j].y, a[j].z, a[j].w}, wv[4] = {w[j].x, w[j].y, w[j].z, w[j].w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc = fmaf(__uint_as_float(av[q] << 16), __uint_as_float(wv[q] << 16), acc);
        acc = fmaf(__uint_as_float(av[q] & 0xFFFF0000u), __uint_as_float(wv[q] & 0xFFFF0000u), acc);
      }
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  __shared__ float part[4];
  __shared__ int s_last;
  if (lane == 0) part[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float l = (part[0] + part[1]) + (part[2] + part[3]);
    if (b) l += b[e];
    logits[p] = bf16_bits_to_f32(f32_to_bf16_bits(l));
    __threadfence();
    s_last = (atomicAdd(counter, 1u) == gridDim.x - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int tt = warp; tt < T; tt += 4) {
    const float* lg = logits + (int64_t)tt * E;
    float sel[8];
    int sid[8];
    uint32_t taken = 0;  // bit j: expert lane + 32*j already selected (E <= 1024)
    for (int k = 0; k < top_k; ++k) {
      float best = -INFINITY;
      int bi = 0x7fffffff;
      for (int j = 0; lane + 32 * j < E; ++j) {
        if ((taken >> j) & 1u) continue;
        const int ee = lane + 32 * j;
        float v = __ldcg(lg + ee);
        if (v != v) v = -INFINITY;  // NaN sorts lowest; ties (incl. all -inf) go to the lower id
        if (v > best || (v == best && ee < bi)) { best = v; bi = ee; }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
      }
      sel[k] = best;
      sid[k] = bi;
      if (bi != 0x7fffffff && (bi & 31) == lane) taken |= 1u << (bi >> 5);
    }
    if (lane == 0) {
      const float mx = sel[0];
      float den = 0.f, ex[8];
      for (int k = 0; k < top_k; ++k) { ex[k] = __expf(sel[k] - mx); den += ex[k]; }
      for (int k = 0; k < top_k; ++k) {
        ids[(int64_t)tt * top_k + k] = sid[k];
        wts[(int64_t)tt * top_k + k] = ex[k] / den;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) *counter = 0u;
}

// ------------------------------------------------------------------ launch helpers
template <typename Kern, typename... Args>
static cudaError_t launch(Kern k, int grid, int block, size_t smem, cudaStream_t st, bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

static int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int F>
static bool choose_geom(int K, int nseg, int rows_per_seg, StageGeom& G, int kData = kStageBytes - 256) {
  // kData: stage bytes minus its RowInfo header
  int slot, scb, ssl;
  G.K = K;
  G.rps = rows_per_seg;
  auto take = [&](int KC) {
    G.KC = KC;
    G.slot = slot;
    G.sc_base = scb;
    G.sslot = ssl;
  };
  if (host_stage_bytes<F>(K, K, nseg, rows_per_seg, slot, scb, ssl) <= kData) {
    take(K);
    return true;
  }
  for (int KC = (K / 256) * 256; KC >= 256; KC -= 256) {
    if (host_stage_bytes<F>(K, KC, nseg, rows_per_seg, slot, scb, ssl) <= kData) {
      take(KC);
      return true;
    }
  }
  return false;
}

template <int F, int MODE, class P>
static cudaError_t run_plan(const P& plan, int nblocks, int nv, cudaStream_t st, bool pdl) {
  const int grid = std::max(1, std::min(nblocks, num_sms()));
  if (plan.geom.KC >= plan.geom.K) {
    // Single-vector whole-row plans: kGroupsWide consumer groups (each warp
    // covers a longer K range of its row block) over a kNStageWide-deep ring,
    // when that fits in shared memory.
    using SW = SmemPlan<kNCW, kNStageWide, kStageBytes, MODE, F>;
    if (MODE == COLS_DUP && SW::total(plan.geom.K, nv) <= 227 * 1024) {
      const int smem = SW::total(plan.geom.K, nv);
      // With few row blocks per CTA (small matrices) fewer groups keep all
      // consumer warps on the blocks there are.
      const int per_cta = (nblocks + grid - 1) / grid;
      auto kern = per_cta >= 3           ? qmv_kernel<F, MODE, kNCW, kNStageWide, kStageBytes, kGroupsWide, P>
                  : per_cta >= 2         ? qmv_kernel<F, MODE, kNCW, kNStageWide, kStageBytes, 2, P>
                                         : qmv_kernel<F, MODE, kNCW, kNStageWide, kStageBytes, 1, P>;
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
      return launch(kern, grid, 32 * (kNCW + kNStageWide), (size_t)smem, st, pdl, plan);
    }
    const int smem = SmemPlan<kNCW, kNStage, kStageBytes, MODE, F>::total(plan.geom.K, nv);
    auto kern = qmv_kernel<F, MODE, kNCW, kNStage, kStageBytes, 2, P>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    return launch(kern, grid, 32 * (kNCW + kNStage), (size_t)smem, st, pdl, plan);
  }
  // K-chunked rows: two consumer groups over the deeper ring when the ring is
  // still phase-safe for them ((groups - 1) * chunks + 1 <= stages, see
  // qmv_kernel), so each warp covers twice as many steps of a stage.
  {
    using SW = SmemPlan<kNCW, kNStageWide, kStageBytes, MODE, F>;
    const int nkc = (plan.geom.K + plan.geom.KC - 1) / plan.geom.KC;
    if (MODE != COLS_FULL && (2 - 1) * nkc + 1 <= kNStageWide && SW::total(plan.geom.K, nv) <= 227 * 1024) {
      const int smem = SW::total(plan.geom.K, nv);
      auto kern = qmv_kernel<F, MODE, kNCW, kNStageWide, kStageBytes, 2, P>;
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
      return launch(kern, grid, 32 * (kNCW + kNStageWide), (size_t)smem, st, pdl, plan);
    }
  }
  const int smem = SmemPlan<kNCW, kNStage, kStageBytes, MODE, F>::total(plan.geom.K, nv);
  auto kern = qmv_kernel<F, MODE, kNCW, kNStage, kStageBytes, 1, P>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  return launch(kern, grid, 32 * (kNCW + kNStage), (size_t)smem, st, pdl, plan);
}

int max_vectors_for(int K) {
  // one vector: single-column layout; several: 8-column partial sums (largest coefficients: Q6_K)
  using S1 = SmemPlan<kNCW, kNStage, kStageBytes, COLS_DUP, FMT_Q6_K>;
  using S8 = SmemPlan<kNCW, kNStage, kStageBytes, COLS_FULL, FMT_Q6_K>;
  const int limit = 227 * 1024;
  const int n8 = (limit - S8::off_x) / S8::x_bytes(K, 1);
  if (n8 >= 2) return std::min(8, n8);
  return (limit - S1::off_x) >= S1::x_bytes(K, 1) ? 1 : 0;
}

// ------------------------------------------------------------------ matvec
template <int F>
static int matvec_t(const void* w, const void* s, int64_t N, int64_t K, const void* x, int xdt, int nv, int64_t xs,
                    void* y, int ydt, int64_t ys, int32_t* err, cudaStream_t st) {
  PlanMatvec<F> p{};
  if (!choose_geom<F>((int)K, 1, 16, p.geom)) return set_error(TSB_ERR_UNSUPPORTED, "row too long for a stage");
  p.err = err;
  p.w = static_cast<const uint8_t*>(w);
  p.s = static_cast<const uint8_t*>(s);
  p.N = N;
  int64_t db, sb;
  weight_bytes_of(F, N, K, db, sb);
  p.mat_bytes = db;
  p.x = x;
  p.x_dtype = xdt;
  p.nv = nv;
  p.x_stride = xs;
  {
    const size_t es = xdt == TSB_DT_F32 ? 4 : 2, need = es * 4;
    p.x_vec_ok = (reinterpret_cast<uintptr_t>(x) % need == 0) && ((xs * es) % need == 0);
  }
  p.y = y;
  p.y_dtype = ydt;
  p.y_stride = ys;
  const int nb = (int)((N + 15) / 16);
  cudaError_t e = nv == 1 ? run_plan<F, COLS_DUP>(p, nb, nv, st, false) : run_plan<F, COLS_FULL>(p, nb, nv, st, false);
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  return TSB_OK;
}

int launch_matvec(int fmt, const void* w, const void* s, int64_t N, int64_t K, const void* x, int xdt, int nv,
                  int64_t xs, void* y, int ydt, int64_t ys, int32_t* err, cudaStream_t st) {
  switch (fmt) {
    case FMT_Q8_0: return matvec_t<FMT_Q8_0>(w, s, N, K, x, xdt, nv, xs, y, ydt, ys, err, st);
    case FMT_Q4_K: return matvec_t<FMT_Q4_K>(w, s, N, K, x, xdt, nv, xs, y, ydt, ys, err, st);
    case FMT_Q5_K: return matvec_t<FMT_Q5_K>(w, s, N, K, x, xdt, nv, xs, y, ydt, ys, err, st);
    case FMT_Q6_K: return matvec_t<FMT_Q6_K>(w, s, N, K, x, xdt, nv, xs, y, ydt, ys, err, st);
    case FMT_MXFP4: return matvec_t<FMT_MXFP4>(w, s, N, K, x, xdt, nv, xs, y, ydt, ys, err, st);
  }
  return set_error(TSB_ERR_UNSUPPORTED, "unsupported format");
}

// ------------------------------------------------------------------ MoE decode (T = 1)
template <int F>
static int gate_up_t(const TsbMoeSpec& sp, const TsbExpert* ex, const int32_t* ids, const void* x, float* act,
                     int32_t* err, cudaStream_t st, bool pdl) {
  PlanGateUp<F> p{};
  const bool inter = sp.gate_up_layout == TSB_GU_INTERLEAVED;
  if (!choose_geom<F>(sp.hidden, inter ? 1 : 2, inter ? 16 : 8, p.geom))
    return set_error(TSB_ERR_UNSUPPORTED, "hidden size too large for a stage");
  p.err = err;
  p.experts = ex;
  p.ids = ids;
  p.n_experts = sp.n_experts;
  p.top_k = sp.top_k;
  p.I = sp.inter;
  p.layout = sp.gate_up_layout;
  p.act = sp.activation;
  p.limit = sp.limit;
  p.alpha = sp.alpha;
  p.x = static_cast<const uint16_t*>(x);
  p.x_vec_ok = reinterpret_cast<uintptr_t>(x) % 8 == 0;
  p.act_out = act;
  int64_t db, sb;
  weight_bytes_of(F, (sp.gate_up_layout == TSB_GU_SEPARATE ? 1 : 2) * (int64_t)sp.inter, sp.hidden, db, sb);
  p.gu_bytes = db;
  weight_bytes_of(F, sp.inter, sp.hidden, db, sb);
  p.up_bytes = db;
  p.tpe = (sp.inter + 7) / 8;
  cudaError_t e = run_plan<F, COLS_DUP>(p, sp.top_k * p.tpe, 1, st, pdl);
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  return TSB_OK;
}

template <int F>
static int down_t(const TsbMoeSpec& sp, const TsbExpert* ex, const int32_t* ids, const float* wts, const float* act,
                  void* out, int32_t* err, cudaStream_t st, bool pdl) {
  PlanDownT1<F> p{};
  int kp = 1;
  while (kp < sp.top_k) kp <<= 1;
  p.rpe = 16 / kp;
  if (!choose_geom<F>(sp.inter, sp.top_k, p.rpe, p.geom))
    return set_error(TSB_ERR_UNSUPPORTED, "intermediate size too large for a stage");
  p.err = err;
  p.experts = ex;
  p.ids = ids;
  p.wts = wts;
  p.n_experts = sp.n_experts;
  p.top_k = sp.top_k;
  p.H = sp.hidden;
  p.I = sp.inter;
  p.act = act;
  p.out = out;
  p.out_f32 = sp.out_f32 != 0;
  int64_t db, sb;
  weight_bytes_of(F, sp.hidden, sp.inter, db, sb);
  p.dn_bytes = db;
  cudaError_t e = run_plan<F, COLS_DIAG>(p, (sp.hidden + p.rpe - 1) / p.rpe, sp.top_k, st, pdl);
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  return TSB_OK;
}

#define TSB_DISPATCH(fmt, CALL)                              \
  switch (fmt) {                                             \
    case FMT_Q8_0: { constexpr int F_ = FMT_Q8_0; return CALL; } \
    case FMT_Q4_K: { constexpr int F_ = FMT_Q4_K; return CALL; } \
    case FMT_Q5_K: { constexpr int F_ = FMT_Q5_K; return CALL; } \
    case FMT_Q6_K: { constexpr int F_ = FMT_Q6_K; return CALL; } \
    case FMT_MXFP4: { constexpr int F_ = FMT_MXFP4; return CALL; } \
  }                                                          \
  return set_error(TSB_ERR_UNSUPPORTED, "unsupported format");

int launch_gate_up(const TsbMoeSpec& sp, const TsbExpert* ex, const int32_t* ids, const void* x, float* act,
                   int32_t* err, cudaStream_t st, bool pdl) {
  TSB_DISPATCH(sp.fmt_gate_up, gate_up_t<F_>(sp, ex, ids, x, act, err, st, pdl))
}

int launch_down(const TsbMoeSpec& sp, const TsbExpert* ex, const int32_t* ids, const float* wts, const float* act,
                void* out, int32_t* err, cudaStream_t st, bool pdl) {
  TSB_DISPATCH(sp.fmt_down, down_t<F_>(sp, ex, ids, wts, act, out, err, st, pdl))
}

int launch_router(const void* x, const void* W, const float* b, int H, int E, int T, int top_k, float* logits,
                  int32_t* ids, float* wts, unsigned* counter, cudaStream_t st) {
  const int grid = E * T;
  router_kernel<<<grid, 128, 0, st>>>(static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(W), b, H, E, T,
                                      top_k, logits, ids, wts, counter);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  return TSB_OK;
}

}  // namespace tsb

// ============================================================================
// Fused batch-1 MoE layer: one persistent cooperative kernel per layer.
//
//   1. every CTA stages x and computes the router logits (all of them when the
//      router matrix is small, else its slice followed by a grid barrier),
//      picks the top-k and softmaxes them -- identical in every CTA;
//   2. the producer warp starts streaming gate/up rows of the chosen experts
//      as soon as the routing is known, and keeps streaming the down rows into
//      the stage ring while consumers finish gate/up;
//   3. consumers run gate/up + activation, meet at a grid barrier (act is then
//      complete in global memory), stage act and run down + weighted combine.
// All CTAs are co-resident (cooperative launch, one CTA per SM); the grid
// barrier's waits are bounded and record kDevWaitTimeout when exceeded.
// ============================================================================
namespace tsb {


}  // namespace tsb
