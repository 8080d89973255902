// Batch-1 decode attention over a float8 (e4m3) or bf16 KV cache, and the
// residual + RMSNorm step between sublayers: the per-token caller side of the
// expert layers in a whole-model GPT-OSS decode.
//
// Semantics followed (GPT-OSS as tinyserve runs it through Hugging Face with
// its StaticKVCache, tinyserve/static_kv_cache.py:28-147): RoPE with the
// halves rotated (x1*cos - x2*sin, x2*cos + x1*sin), keys and values stored in
// the cache's type and read back exactly, grouped-query attention (G query
// heads per KV head), scores scaled by 1/sqrt(D), a learned per-head "sink"
// logit that joins the softmax denominator only, causal masking, and for
// sliding layers only the last `window` positions.
//
// Design (one launch per layer, graph-capturable: the position is read from
// device memory):
//  * grid (S, n_kv): CTA (s, h) takes the s-th slice of the live positions
//    [lo, pos] of KV head h for all G query heads of the group.  Each CTA
//    applies RoPE to its q rows and to the new key itself (the new key/value
//    never go through memory inside the launch); CTA (0, h) stores them in the
//    cache at `pos` for later steps.
//  * scores: a warp per position, lane l holds dims 2l, 2l+1; G dot products
//    reduced with shuffles; probabilities relative to the slice maximum.
//  * P.V: thread (g, l) accumulates dims 2l, 2l+1 of head g over the slice.
//  * the last CTA of a KV head (acq_rel counter) merges the S partial
//    (max, sum, o) triples with the sink and writes bf16 outputs; the counter
//    is reset for the next call.
// Memory-bound on the cache slice (D bytes per position per KV head for e4m3).
#include <cuda_fp8.h>

#include <cstdlib>

#include "../../include/tsb_moe.h"
#include "tsb_common.cuh"
#include "tsb_internal.h"

namespace tsb {
namespace {

constexpr int kD = 64;         // head dimension (GPT-OSS)
constexpr int kThreads = 256;  // 8 warps

struct AttnArgs {
  const uint16_t* qkv;   // bf16 [nq + 2 nkv, D] (projection output, before RoPE)
  const uint16_t* cos;   // bf16 [max_seq, D/2]
  const uint16_t* sin;
  const int64_t* pos;    // device scalar
  void* kc;              // [nkv, max_seq, D] cache
  void* vc;
  const float* sinks;    // [nq]
  uint16_t* out;         // bf16 [nq, D]
  float* part;           // [batch][nkv, S, G, D + 2]
  unsigned* counters;    // [batch][nkv]
  const int32_t* slots;  // [batch] cache slot of each row (nullptr: slot 0)
  int64_t slot_stride;   // cache elements between slots
  int32_t* err;
  int nq, nkv, G, S, max_seq, window, cs_max;
  float scale;
};

template <bool FP8>
__device__ __forceinline__ float2 load2(const void* base, int64_t idx) {  // idx even
  if constexpr (FP8) {
    const __nv_fp8x2_storage_t v = *reinterpret_cast<const __nv_fp8x2_storage_t*>(static_cast<const uint8_t*>(base) + idx);
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(v, __NV_E4M3);
    return __half22float2(*reinterpret_cast<const __half2*>(&h));
  } else {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(static_cast<const uint16_t*>(base) + idx);
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
  }
}

// The value a cache of this type holds for x (x already rounded to bf16, as the
// projection's bf16 output is): e4m3 round-to-nearest-even, no saturation
// (out-of-range values become NaN, as a plain cast does), or x itself.
template <bool FP8>
__device__ __forceinline__ float cache_round(float x, uint8_t* byte) {
  if constexpr (FP8) {
    const __nv_fp8_storage_t b = __nv_cvt_float_to_fp8(x, __NV_NOSAT, __NV_E4M3);
    *byte = b;
    const __half_raw h = __nv_cvt_fp8_to_halfraw(b, __NV_E4M3);
    return __half2float(*reinterpret_cast<const __half*>(&h));
  } else {
    *byte = 0;
    return x;
  }
}

__device__ __forceinline__ float bf(uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }
__device__ __forceinline__ float round_bf16(float x) { return bf(f32_to_bf16_bits(x)); }

template <bool FP8>
__global__ void __launch_bounds__(kThreads) gqa_decode_kernel(const AttnArgs a0) {
  extern __shared__ float sm[];
  // batch row b: its token's projections, position, cache slot, output and scratch
  AttnArgs a = a0;
  {
    const int b = blockIdx.z;
    const int64_t slot = a0.slots ? a0.slots[b] : 0;
    constexpr int EB0 = FP8 ? 1 : 2;
    a.qkv = a0.qkv + (int64_t)b * (a0.nq + 2 * a0.nkv) * kD;
    a.pos = a0.pos + b;
    a.out = a0.out + (int64_t)b * a0.nq * kD;
    a.kc = static_cast<uint8_t*>(a0.kc) + slot * a0.slot_stride * EB0;
    a.vc = static_cast<uint8_t*>(a0.vc) + slot * a0.slot_stride * EB0;
    a.part = a0.part + (int64_t)b * a0.nkv * a0.S * a0.G * (kD + 2);
    a.counters = a0.counters + (int64_t)b * a0.nkv;
  }
  const int G = a.G, h = blockIdx.y, s = blockIdx.x;
  float* qs = sm;                 // [G][D]
  float* knew = qs + G * kD;      // [D]
  float* vnew = knew + kD;        // [D]
  float* sc = vnew + kD;          // [G][cs_max]
  __shared__ float s_m[16], s_l[16];
  __shared__ int s_last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t pos = *a.pos;
  if (pos < 0 || pos >= a.max_seq) {
    if (tid == 0 && a.err) atomicExch(a.err, kDevBadPlan);
    return;
  }
  const int64_t lo64 = pos - a.window + 1;
  const int lo = (a.window > 0 && lo64 > 0) ? (int)lo64 : 0;
  const int len = (int)pos - lo + 1;
  const int cs = (len + a.S - 1) / a.S;
  const int c0 = lo + s * cs, c1 = min((int)pos + 1, c0 + cs);
  const int n = max(0, c1 - c0);
  const int64_t hb = (int64_t)h * a.max_seq * kD;
  // stage the slice's keys and values in shared memory with every thread's
  // 16-byte loads in flight at once; rows padded by 16 B so the per-position
  // row reads of the score pass are bank-conflict free
  constexpr int EB = FP8 ? 1 : 2;         // bytes per cached element
  constexpr int RB = kD * EB + 16;        // padded row bytes
  constexpr int C16 = kD * EB / 16;       // 16-byte chunks per row
  uint8_t* ks = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sc + G * a.cs_max) + 15) & ~uintptr_t(15));
  uint8_t* vs = ks + (size_t)a.cs_max * RB;
  {
    const uint8_t* kg = static_cast<const uint8_t*>(a.kc) + (hb + (int64_t)c0 * kD) * EB;
    const uint8_t* vg = static_cast<const uint8_t*>(a.vc) + (hb + (int64_t)c0 * kD) * EB;
    // all of a thread's loads (up to 4 chunks of each) before any store
    for (int base = 0; base < n * C16; base += 4 * kThreads) {
      uint4 kv[4], vv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = base + u * kThreads + tid;
        if (i < n * C16) {
          const int j = i / C16, c = i % C16;
          kv[u] = *reinterpret_cast<const uint4*>(kg + (size_t)j * kD * EB + c * 16);
          vv[u] = *reinterpret_cast<const uint4*>(vg + (size_t)j * kD * EB + c * 16);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = base + u * kThreads + tid;
        if (i < n * C16) {
          const int j = i / C16, c = i % C16;
          *reinterpret_cast<uint4*>(ks + (size_t)j * RB + c * 16) = kv[u];
          *reinterpret_cast<uint4*>(vs + (size_t)j * RB + c * 16) = vv[u];
        }
      }
    }
  }
  
  // everything above reads only cache rows written by earlier steps;
  // the projection output comes from the previous kernel
  pdl_wait();
  pdl_launch_dependents();
  // RoPE: q rows of the group, the new key; the new value as is
  const uint16_t* cr = a.cos + pos * (kD / 2);
  const uint16_t* sr = a.sin + pos * (kD / 2);
  for (int i = tid; i < (G + 2) * (kD / 2); i += kThreads) {
    const int r = i / (kD / 2), d = i % (kD / 2);
    if (r < G + 1) {
      const int row = r < G ? h * G + r : a.nq + h;
      const float x1 = bf(a.qkv[row * kD + d]), x2 = bf(a.qkv[row * kD + d + kD / 2]);
      const float c = bf(cr[d]), sn = bf(sr[d]);
      float y1 = x1 * c - x2 * sn, y2 = x2 * c + x1 * sn;
      if (r < G) {
        qs[r * kD + d] = y1;
        qs[r * kD + d + kD / 2] = y2;
      } else {
        uint8_t b1, b2;
        y1 = cache_round<FP8>(round_bf16(y1), &b1);
        y2 = cache_round<FP8>(round_bf16(y2), &b2);
        knew[d] = y1;
        knew[d + kD / 2] = y2;
        if (s == 0) {
          const int64_t o = ((int64_t)h * a.max_seq + pos) * kD;
          if constexpr (FP8) {
            static_cast<uint8_t*>(a.kc)[o + d] = b1;
            static_cast<uint8_t*>(a.kc)[o + d + kD / 2] = b2;
          } else {
            static_cast<uint16_t*>(a.kc)[o + d] = f32_to_bf16_bits(y1);
            static_cast<uint16_t*>(a.kc)[o + d + kD / 2] = f32_to_bf16_bits(y2);
          }
        }
      }
    } else {
      const int row = a.nq + a.nkv + h;
      for (int dd = d; dd < kD; dd += kD / 2) {
        uint8_t b;
        const float v = cache_round<FP8>(bf(a.qkv[row * kD + dd]), &b);
        vnew[dd] = v;
        if (s == 0) {
          const int64_t o = ((int64_t)h * a.max_seq + pos) * kD + dd;
          if constexpr (FP8)
            static_cast<uint8_t*>(a.vc)[o] = b;
          else
            static_cast<uint16_t*>(a.vc)[o] = a.qkv[row * kD + dd];
        }
      }
    }
  }
  __syncthreads();
  // the current position's key/value come from the prologue, not the cache
  if (pos >= c0 && pos < c1) {
    const int j = (int)pos - c0;
    for (int d = tid; d < kD; d += kThreads) {
      if constexpr (FP8) {
        ks[(size_t)j * RB + d] = __nv_cvt_float_to_fp8(knew[d], __NV_NOSAT, __NV_E4M3);
        vs[(size_t)j * RB + d] = __nv_cvt_float_to_fp8(vnew[d], __NV_NOSAT, __NV_E4M3);
      } else {
        reinterpret_cast<uint16_t*>(ks + (size_t)j * RB)[d] = f32_to_bf16_bits(knew[d]);
        reinterpret_cast<uint16_t*>(vs + (size_t)j * RB)[d] = f32_to_bf16_bits(vnew[d]);
      }
    }
  }
  __syncthreads();
  // scores: one position per thread, all G heads (q broadcast from shared memory)
  for (int j = tid; j < n; j += kThreads) {
    float kr[kD];
#pragma unroll
    for (int d = 0; d < kD; d += 2) {
      const float2 k2 = load2<FP8>(ks + (size_t)j * RB, d);
      kr[d] = k2.x;
      kr[d + 1] = k2.y;
    }
    for (int g = 0; g < G; ++g) {
      const float4* q4 = reinterpret_cast<const float4*>(qs + g * kD);
      float acc = 0.f;
#pragma unroll
      for (int d4 = 0; d4 < kD / 4; ++d4) {
        const float4 q = q4[d4];
        acc = fmaf(q.x, kr[4 * d4], acc);
        acc = fmaf(q.y, kr[4 * d4 + 1], acc);
        acc = fmaf(q.z, kr[4 * d4 + 2], acc);
        acc = fmaf(q.w, kr[4 * d4 + 3], acc);
      }
      sc[g * a.cs_max + j] = acc * a.scale;
    }
  }
  __syncthreads();
  // per-head slice max and sum of exp
  for (int g = warp; g < G; g += kThreads / 32) {
    float m = -INFINITY;
    for (int j = lane; j < n; j += 32) m = fmaxf(m, sc[g * a.cs_max + j]);
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    for (int j = lane; j < n; j += 32) {
      const float e = __expf(sc[g * a.cs_max + j] - m);
      sc[g * a.cs_max + j] = e;
      l += e;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) {
      s_m[g] = m;
      s_l[g] = l;
    }
  }
  __syncthreads();
  // P.V: thread (g, lane) -> dims 2 lane, 2 lane + 1 of head g
  for (int g = warp; g < G; g += kThreads / 32) {
    float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
    const float* pg = sc + g * a.cs_max;
    int j = 0;
    for (; j + 1 < n; j += 2) {
      const float2 va = load2<FP8>(vs + (size_t)j * RB, 2 * lane);
      const float2 vb = load2<FP8>(vs + (size_t)(j + 1) * RB, 2 * lane);
      o0 = fmaf(pg[j], va.x, o0);
      o1 = fmaf(pg[j], va.y, o1);
      o2 = fmaf(pg[j + 1], vb.x, o2);
      o3 = fmaf(pg[j + 1], vb.y, o3);
    }
    if (j < n) {
      const float2 va = load2<FP8>(vs + (size_t)j * RB, 2 * lane);
      o0 = fmaf(pg[j], va.x, o0);
      o1 = fmaf(pg[j], va.y, o1);
    }
    o0 += o2;
    o1 += o3;
    float* dst = a.part + (((int64_t)h * a.S + s) * G + g) * (kD + 2);
    dst[2 * lane] = o0;
    dst[2 * lane + 1] = o1;
    if (lane == 0) {
      dst[kD] = s_m[g];
      dst[kD + 1] = s_l[g];
    }
  }
  // the last CTA of this KV head merges the slices
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    unsigned prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(a.counters + h) : "memory");
    s_last = prev == (unsigned)(a.S - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int g = warp; g < G; g += kThreads / 32) {
    const float* base = a.part + (int64_t)h * a.S * G * (kD + 2);
    const float sink = a.sinks[h * G + g];
    float M = sink;
    for (int t = 0; t < a.S; ++t) M = fmaxf(M, base[(t * G + g) * (kD + 2) + kD]);
    float den = __expf(sink - M), o0 = 0.f, o1 = 0.f;
    for (int t = 0; t < a.S; ++t) {
      const float* q = base + (t * G + g) * (kD + 2);
      const float w = q[kD + 1] > 0.f ? __expf(q[kD] - M) : 0.f;
      den = fmaf(w, q[kD + 1], den);
      o0 = fmaf(w, q[2 * lane], o0);
      o1 = fmaf(w, q[2 * lane + 1], o1);
    }
    const float inv = 1.f / den;
    uint16_t* o = a.out + (h * G + g) * kD;
    o[2 * lane] = f32_to_bf16_bits(o0 * inv);
    o[2 * lane + 1] = f32_to_bf16_bits(o1 * inv);
  }
  if (tid == 0) a.counters[h] = 0u;
}

// x[r] += delta[r] (fp32 residual, delta bf16 or fp32, optional);
// out[r] = bf16(w * x[r] * rsqrt(mean(x[r]^2) + eps)).  One CTA per row; each
// thread keeps its (at most kPer) elements in registers so all loads of the
// row are in flight together.
constexpr int kNormThreads = 256, kPer = 16;

__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(float* __restrict__ x, const void* __restrict__ delta,
                                                                   int delta_f32, const float* __restrict__ w, float eps,
                                                                   int H, uint16_t* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  const int r = blockIdx.x;
  float* xr = x + (int64_t)r * H;
  float v[kPer];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int i = threadIdx.x + k * kNormThreads;
    v[k] = 0.f;
    if (i < H) {
      float d = 0.f;
      if (delta)
        d = delta_f32 ? static_cast<const float*>(delta)[(int64_t)r * H + i]
                      : bf(static_cast<const uint16_t*>(delta)[(int64_t)r * H + i]);
      v[k] = xr[i] + d;
    }
  }
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int i = threadIdx.x + k * kNormThreads;
    if (i < H) {
      xr[i] = v[k];
      ss = fmaf(v[k], v[k], ss);
    }
  }
  __shared__ float red[kNormThreads / 32];
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int k = 0; k < kNormThreads / 32; ++k) t += red[k];
  const float inv = rsqrtf(t / H + eps);
  if (out) {
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = threadIdx.x + k * kNormThreads;
      if (i < H) out[(int64_t)r * H + i] = f32_to_bf16_bits(w[i] * (v[k] * inv));
    }
  }
}

// y[n] = bf16(W[n, :] . x + bias[n]) for bf16 W [N, K] (row-major): one warp
// per row, the row's 16-byte chunks loaded in batches of 8 per lane before any
// arithmetic (the first batch before waiting for the previous kernel, since
// the weights do not depend on it), the input vector staged once per CTA as
// fp32 in shared memory.  Three forms share the body:
//  GV_PLAIN    x is a bf16 vector;
//  GV_NORM     x = bf16(RMSNorm(x_in + delta) * norm_w), computed by every CTA
//              from the fp32 residual stream; CTA 0 stores x_in + delta to
//              x_out (the residual for the rest of the layer);
//  GV_RESIDUAL resid[n] += bf16(y[n]) (y is not stored); the last CTA to finish
//              writes h_out = bf16(RMSNorm(resid) * norm_w) for the next sublayer.
constexpr int kGemvWarps = 8;
enum { GV_PLAIN = 0, GV_NORM = 1, GV_RESIDUAL = 2 };

// Vector staging helpers: each thread issues up to 4 independent 16-byte loads
// before storing any of them, so a staging pass costs one memory round trip
// (a load/store loop would serialise them: the shared-memory stores may alias
// the loads as far as the compiler knows).
__device__ __forceinline__ void stage_bf16_f32(float* __restrict__ xs, const uint16_t* __restrict__ x, int K) {
  const uint4* src = reinterpret_cast<const uint4*>(x);
  const int n16 = K / 8;
  for (int base = 0; base < n16; base += 4 * (int)blockDim.x) {
    uint4 r[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = base + u * blockDim.x + threadIdx.x;
      if (i < n16) r[u] = src[i];
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = base + u * blockDim.x + threadIdx.x;
      if (i < n16) {
        float4* d = reinterpret_cast<float4*>(xs + 8 * i);
        d[0] = make_float4(__uint_as_float(r[u].x << 16), __uint_as_float(r[u].x & 0xFFFF0000u),
                           __uint_as_float(r[u].y << 16), __uint_as_float(r[u].y & 0xFFFF0000u));
        d[1] = make_float4(__uint_as_float(r[u].z << 16), __uint_as_float(r[u].z & 0xFFFF0000u),
                           __uint_as_float(r[u].w << 16), __uint_as_float(r[u].w & 0xFFFF0000u));
      }
    }
  }
}

// xs = v = a + b (b nullable; fp32, K % 4 == 0); returns this thread's sum of v^2.
// When out is given it receives v too.  CG: read a through L2 (data other CTAs
// of the running kernel wrote).
template <bool CG = false>
__device__ __forceinline__ float stage_sum_f32(float* __restrict__ xs, const float* __restrict__ a,
                                               const float* __restrict__ b, float* __restrict__ out, int K) {
  const float4* pa = reinterpret_cast<const float4*>(a);
  const float4* pb = reinterpret_cast<const float4*>(b);
  const int n4 = K / 4;
  float ss = 0.f;
  for (int base = 0; base < n4; base += 4 * (int)blockDim.x) {
    float4 ra[4], rb[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = base + u * blockDim.x + threadIdx.x;
      if (i < n4) {
        ra[u] = CG ? __ldcg(pa + i) : pa[i];
        rb[u] = b ? pb[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = base + u * blockDim.x + threadIdx.x;
      if (i < n4) {
        const float4 v = make_float4(ra[u].x + rb[u].x, ra[u].y + rb[u].y, ra[u].z + rb[u].z, ra[u].w + rb[u].w);
        reinterpret_cast<float4*>(xs)[i] = v;
        if (out) reinterpret_cast<float4*>(out)[i] = v;
        ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
      }
    }
  }
  return ss;
}

// xs[i] = round_bf16(w[i] * xs[i] * inv) (store_bf16 == nullptr) or
// store_bf16[i] = bf16(w[i] * xs[i] * inv); K % 4 == 0.
__device__ __forceinline__ void apply_norm(float* __restrict__ xs, const float* __restrict__ w, float inv, int K,
                                           uint16_t* __restrict__ store_bf16) {
  const float4* pw = reinterpret_cast<const float4*>(w);
  const int n4 = K / 4;
  for (int base = 0; base < n4; base += 4 * (int)blockDim.x) {
    float4 rw[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = base + u * blockDim.x + threadIdx.x;
      if (i < n4) rw[u] = pw[i];
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = base + u * blockDim.x + threadIdx.x;
      if (i < n4) {
        const float4 v = reinterpret_cast<const float4*>(xs)[i];
        const float o[4] = {rw[u].x * (v.x * inv), rw[u].y * (v.y * inv), rw[u].z * (v.z * inv), rw[u].w * (v.w * inv)};
        if (store_bf16) {
          const uint2 pk = make_uint2(f32_to_bf16_bits(o[0]) | ((uint32_t)f32_to_bf16_bits(o[1]) << 16),
                                      f32_to_bf16_bits(o[2]) | ((uint32_t)f32_to_bf16_bits(o[3]) << 16));
          reinterpret_cast<uint2*>(store_bf16)[i] = pk;
        } else {
          reinterpret_cast<float4*>(xs)[i] = make_float4(round_bf16(o[0]), round_bf16(o[1]), round_bf16(o[2]), round_bf16(o[3]));
        }
      }
    }
  }
}

struct GemvArgs {
  const uint16_t* W;
  const uint16_t* bias;
  int N, K;
  const uint16_t* x;     // GV_PLAIN / GV_RESIDUAL
  uint16_t* y;           // GV_PLAIN / GV_NORM
  const float* x_in;     // GV_NORM
  const float* delta;    // GV_NORM (nullable)
  float* x_out;          // GV_NORM
  float* resid;          // GV_RESIDUAL
  const float* norm_w;   // GV_NORM / GV_RESIDUAL
  float eps;
  uint16_t* h_out;       // GV_RESIDUAL
  unsigned* counter;     // GV_RESIDUAL
};

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
  for (int k = 0; k < (int)(blockDim.x >> 5); ++k) t += red[k];
  return t;
}

template <int MODE>
__global__ void __launch_bounds__(kGemvWarps * 32, MODE == GV_PLAIN ? 4 : 3) gemv_bf16_kernel(GemvArgs a) {
  extern __shared__ float xs[];
  __shared__ float red[kGemvWarps];
  __shared__ int s_last;
  const int lane = threadIdx.x & 31;
  const int K = a.K, N = a.N;
  const int n = min((int)(blockIdx.x * kGemvWarps + (threadIdx.x >> 5)), N - 1);  // tail warps redo the last row
  const uint4* row = reinterpret_cast<const uint4*>(a.W + (int64_t)n * K);
  const int nc = K / 8;
  uint4 w[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const int c = u * 32 + lane;
    w[u] = c < nc ? __ldcs(row + c) : make_uint4(0, 0, 0, 0);
  }
  if constexpr (MODE == GV_NORM) {
    // the norm weights are constants too: staged before the wait
    stage_sum_f32(xs + K, a.norm_w, nullptr, nullptr, K);
  }
  pdl_wait();
  pdl_launch_dependents();
  if constexpr (MODE == GV_NORM) {
    const float ss = stage_sum_f32(xs, a.x_in, a.delta, blockIdx.x == 0 ? a.x_out : nullptr, K);
    const float inv = rsqrtf(block_sum(ss, red) / K + a.eps);
    apply_norm(xs, xs + K, inv, K, nullptr);
  } else {
    stage_bf16_f32(xs, a.x, K);
  }
  __syncthreads();
  float acc = 0.f;
  for (int c0 = 0; c0 < nc; c0 += 8 * 32) {
    if (c0 > 0) {
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = c0 + u * 32 + lane;
        w[u] = c < nc ? __ldcs(row + c) : make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int c = c0 + u * 32 + lane;
      if (c < nc) {
        const float4* xv = reinterpret_cast<const float4*>(xs + 8 * c);
        const float4 xa = xv[0], xb = xv[1];
        acc = fmaf(__uint_as_float(w[u].x << 16), xa.x, acc);
        acc = fmaf(__uint_as_float(w[u].x & 0xFFFF0000u), xa.y, acc);
        acc = fmaf(__uint_as_float(w[u].y << 16), xa.z, acc);
        acc = fmaf(__uint_as_float(w[u].y & 0xFFFF0000u), xa.w, acc);
        acc = fmaf(__uint_as_float(w[u].z << 16), xb.x, acc);
        acc = fmaf(__uint_as_float(w[u].z & 0xFFFF0000u), xb.y, acc);
        acc = fmaf(__uint_as_float(w[u].w << 16), xb.z, acc);
        acc = fmaf(__uint_as_float(w[u].w & 0xFFFF0000u), xb.w, acc);
      }
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  const bool mine = lane == 0 && (int)(blockIdx.x * kGemvWarps + (threadIdx.x >> 5)) < N;
  const uint16_t yb = f32_to_bf16_bits(acc + (a.bias ? bf(a.bias[n]) : 0.f));
  if constexpr (MODE != GV_RESIDUAL) {
    if (mine) a.y[n] = yb;
  } else {
    if (mine) a.resid[n] += bf(yb);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned prev;
      asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(a.counter) : "memory");
      s_last = prev == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // other CTAs' residual rows, read through L2 (the acq_rel counter above
    // orders them after their writes)
    const float ss = stage_sum_f32<true>(xs, a.resid, nullptr, nullptr, N);
    const float inv = rsqrtf(block_sum(ss, red) / N + a.eps);
    apply_norm(xs, a.norm_w, inv, N, a.h_out);
    if (threadIdx.x == 0) *a.counter = 0u;
  }
}

// Launch with programmatic stream serialisation: the kernel may start while
// the previous kernel on the stream finishes; it waits (griddepcontrol.wait)
// before reading that kernel's outputs.
// TSB_DECODE_PDL=0 launches them plainly (for A/B timing).
bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("TSB_DECODE_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

template <typename Kern, typename... Args>
cudaError_t launch_pdl(Kern k, dim3 grid, int block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, args...);
}


// ---------------------------------------------------------------------------
// RMSNorm + q|k|v projection + decode attention of one token in one launch.
// One thread-block cluster of CN CTAs per KV head h:
//  1. every CTA normalises the residual (x_in + delta; CTA 0 of cluster 0
//     stores it to x_out) and computes its share of the head group's
//     (G + 2) * 64 projection rows (the group's q heads, its k and v rows),
//     warp per row as in gemv_bf16_kernel, bf16-rounded with the bias;
//  2. each row's value is stored into every CTA of the cluster (distributed
//     shared memory), a cluster barrier makes the group's q/k/v complete in
//     all of them;
//  3. every CTA runs the decode attention of gqa_decode_kernel over its
//     slice of the positions (the slice's cached K/V were staged in shared
//     memory before the dependency wait), CTA 0 stores the new key/value;
//  4. the slices' (max, sum, o) go to CTA 0's shared memory, a second
//     cluster barrier, and CTA 0 merges them with the sink logits.
// Every CTA passes both cluster barriers (no early exit once running), so no
// barrier waits on a CTA that left.
struct QkvAttnArgs {
  const float* x_in;
  const float* delta;
  float* x_out;
  const float* norm_w;
  float eps;
  const uint16_t* W;      // [(nq + 2 nkv) * D, H]
  const uint16_t* bias;   // [(nq + 2 nkv) * D] or null
  const uint16_t* cos;
  const uint16_t* sin;
  const int64_t* pos;
  void* kc;
  void* vc;
  const float* sinks;
  uint16_t* out;          // [nq * D]
  int nq, nkv, G, H, CN, max_seq, window, cs_max;
  float scale;
};

__device__ __forceinline__ void st_remote_f32(float* local, uint32_t rank, float v) {
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(local)), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ra), "f"(v) : "memory");
}
__device__ __forceinline__ uint32_t my_cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_barrier_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

template <bool FP8>
__global__ void __launch_bounds__(kThreads, 1) qkv_attn_kernel(const QkvAttnArgs a) {
  extern __shared__ __align__(16) float sm2[];
  const int G = a.G, H = a.H, CN = a.CN;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = (int)my_cluster_rank(), h = blockIdx.x / CN;
  const int R = (G + 2) * kD;                       // projection rows of the head group
  float* xs = sm2;                                  // [H] normalised input
  float* nws = xs + H;                              // [H] norm weights
  float* qkv = nws + H;                             // [R] the group's projections (all CTAs)
  float* qs = qkv + R;                              // [G][D] roped q
  float* knew = qs + G * kD;                        // [D]
  float* vnew = knew + kD;                          // [D]
  float* sc = vnew + kD;                            // [G][cs_max]
  float* mrg = sc + G * a.cs_max;                   // [CN][G][D + 2] (read in CTA 0)
  constexpr int EB = FP8 ? 1 : 2, RB = kD * EB + 16, C16 = kD * EB / 16;
  uint8_t* ks = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(mrg + (size_t)CN * G * (kD + 2)) + 15) &
                                           ~uintptr_t(15));
  uint8_t* vs = ks + (size_t)a.cs_max * RB;
  __shared__ float red[kThreads / 32];
  __shared__ float s_m[16], s_l[16];
  // this CTA is running: remote stores into it may start once every CTA of
  // the cluster has arrived here (the wait comes before the first such store)
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  const int64_t pos = *a.pos;  // written before the graph / launch by the host
  const bool pos_ok = pos >= 0 && pos < a.max_seq;
  const int64_t lo64 = pos - a.window + 1;
  const int lo = (a.window > 0 && lo64 > 0) ? (int)lo64 : 0;
  const int len = pos_ok ? (int)pos - lo + 1 : 0;
  const int cs = (len + CN - 1) / CN;
  const int c0 = lo + c * cs, c1 = min((int)pos + 1, c0 + cs);
  const int n = pos_ok ? max(0, c1 - c0) : 0;
  const int64_t hb = (int64_t)h * a.max_seq * kD;
  // ---- independent of the previous kernel: norm weights, the K/V slice
  stage_sum_f32(nws, a.norm_w, nullptr, nullptr, H);
  {
    const uint8_t* kg = static_cast<const uint8_t*>(a.kc) + (hb + (int64_t)c0 * kD) * EB;
    const uint8_t* vg = static_cast<const uint8_t*>(a.vc) + (hb + (int64_t)c0 * kD) * EB;
    for (int base = 0; base < n * C16; base += 4 * kThreads) {
      uint4 kv[4], vv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = base + u * kThreads + tid;
        if (i < n * C16) {
          const int j = i / C16, q = i % C16;
          kv[u] = *reinterpret_cast<const uint4*>(kg + (size_t)j * kD * EB + q * 16);
          vv[u] = *reinterpret_cast<const uint4*>(vg + (size_t)j * kD * EB + q * 16);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = base + u * kThreads + tid;
        if (i < n * C16) {
          const int j = i / C16, q = i % C16;
          *reinterpret_cast<uint4*>(ks + (size_t)j * RB + q * 16) = kv[u];
          *reinterpret_cast<uint4*>(vs + (size_t)j * RB + q * 16) = vv[u];
        }
      }
    }
  }
  pdl_wait();
  pdl_launch_dependents();
  // ---- 1. RMSNorm of the residual
  {
    const float ss = stage_sum_f32(xs, a.x_in, a.delta, (h == 0 && c == 0) ? a.x_out : nullptr, H);
    const float inv = rsqrtf(block_sum(ss, red) / H + a.eps);
    apply_norm(xs, nws, inv, H, nullptr);
  }
  __syncthreads();
  // ---- 1b. this CTA's projection rows, stored into every CTA of the cluster
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
  const int rpc = (R + CN - 1) / CN;
  const int nc = H / 8;
  for (int lr = c * rpc + warp; lr < min(R, (c + 1) * rpc); lr += kThreads / 32) {
    const int grow = lr < G * kD ? h * G * kD + lr
                     : lr < (G + 1) * kD ? a.nq * kD + h * kD + (lr - G * kD)
                                         : (a.nq + a.nkv) * kD + h * kD + (lr - (G + 1) * kD);
    const uint4* row = reinterpret_cast<const uint4*>(a.W + (int64_t)grow * H);
    float acc = 0.f;
    for (int cb = 0; cb < nc; cb += 8 * 32) {
      uint4 w[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int q = cb + u * 32 + lane;
        w[u] = q < nc ? __ldcs(row + q) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int q = cb + u * 32 + lane;
        if (q < nc) {
          const float4* xv = reinterpret_cast<const float4*>(xs + 8 * q);
          const float4 xa = xv[0], xb = xv[1];
          acc = fmaf(__uint_as_float(w[u].x << 16), xa.x, acc);
          acc = fmaf(__uint_as_float(w[u].x & 0xFFFF0000u), xa.y, acc);
          acc = fmaf(__uint_as_float(w[u].y << 16), xa.z, acc);
          acc = fmaf(__uint_as_float(w[u].y & 0xFFFF0000u), xa.w, acc);
          acc = fmaf(__uint_as_float(w[u].z << 16), xb.x, acc);
          acc = fmaf(__uint_as_float(w[u].z & 0xFFFF0000u), xb.y, acc);
          acc = fmaf(__uint_as_float(w[u].w << 16), xb.z, acc);
          acc = fmaf(__uint_as_float(w[u].w & 0xFFFF0000u), xb.w, acc);
        }
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    const float v = round_bf16(acc + (a.bias ? bf(a.bias[grow]) : 0.f));
    for (int r = lane; r < CN; r += 32) st_remote_f32(qkv + lr, (uint32_t)r, v);
  }
  cluster_barrier_sync();  // the group's q/k/v are complete in every CTA
  // ---- 3. attention over this CTA's slice (gqa_decode_kernel's steps)
  if (pos_ok) {
    const uint16_t* cr = a.cos + pos * (kD / 2);
    const uint16_t* sr = a.sin + pos * (kD / 2);
    for (int i = tid; i < (G + 2) * (kD / 2); i += kThreads) {
      const int r = i / (kD / 2), d = i % (kD / 2);
      if (r <= G) {
        const float x1 = qkv[r * kD + d], x2 = qkv[r * kD + d + kD / 2];
        const float cc = bf(cr[d]), sn = bf(sr[d]);
        float y1 = x1 * cc - x2 * sn, y2 = x2 * cc + x1 * sn;
        if (r < G) {
          qs[r * kD + d] = y1;
          qs[r * kD + d + kD / 2] = y2;
        } else {
          uint8_t b1, b2;
          y1 = cache_round<FP8>(round_bf16(y1), &b1);
          y2 = cache_round<FP8>(round_bf16(y2), &b2);
          knew[d] = y1;
          knew[d + kD / 2] = y2;
          if (c == 0) {
            const int64_t o = ((int64_t)h * a.max_seq + pos) * kD;
            if constexpr (FP8) {
              static_cast<uint8_t*>(a.kc)[o + d] = b1;
              static_cast<uint8_t*>(a.kc)[o + d + kD / 2] = b2;
            } else {
              static_cast<uint16_t*>(a.kc)[o + d] = f32_to_bf16_bits(y1);
              static_cast<uint16_t*>(a.kc)[o + d + kD / 2] = f32_to_bf16_bits(y2);
            }
          }
        }
      } else {
        for (int dd = d; dd < kD; dd += kD / 2) {
          uint8_t b;
          const float v = cache_round<FP8>(qkv[(G + 1) * kD + dd], &b);
          vnew[dd] = v;
          if (c == 0) {
            const int64_t o = ((int64_t)h * a.max_seq + pos) * kD + dd;
            if constexpr (FP8)
              static_cast<uint8_t*>(a.vc)[o] = b;
            else
              static_cast<uint16_t*>(a.vc)[o] = f32_to_bf16_bits(v);
          }
        }
      }
    }
    __syncthreads();
    if (pos >= c0 && pos < c1) {
      const int j = (int)pos - c0;
      for (int d = tid; d < kD; d += kThreads) {
        if constexpr (FP8) {
          ks[(size_t)j * RB + d] = __nv_cvt_float_to_fp8(knew[d], __NV_NOSAT, __NV_E4M3);
          vs[(size_t)j * RB + d] = __nv_cvt_float_to_fp8(vnew[d], __NV_NOSAT, __NV_E4M3);
        } else {
          reinterpret_cast<uint16_t*>(ks + (size_t)j * RB)[d] = f32_to_bf16_bits(knew[d]);
          reinterpret_cast<uint16_t*>(vs + (size_t)j * RB)[d] = f32_to_bf16_bits(vnew[d]);
        }
      }
    }
    __syncthreads();
    for (int j = tid; j < n; j += kThreads) {
      float kr[kD];
#pragma unroll
      for (int d = 0; d < kD; d += 2) {
        const float2 k2 = load2<FP8>(ks + (size_t)j * RB, d);
        kr[d] = k2.x;
        kr[d + 1] = k2.y;
      }
      for (int g = 0; g < G; ++g) {
        const float4* q4 = reinterpret_cast<const float4*>(qs + g * kD);
        float acc = 0.f;
#pragma unroll
        for (int d4 = 0; d4 < kD / 4; ++d4) {
          const float4 q = q4[d4];
          acc = fmaf(q.x, kr[4 * d4], acc);
          acc = fmaf(q.y, kr[4 * d4 + 1], acc);
          acc = fmaf(q.z, kr[4 * d4 + 2], acc);
          acc = fmaf(q.w, kr[4 * d4 + 3], acc);
        }
        sc[g * a.cs_max + j] = acc * a.scale;
      }
    }
    __syncthreads();
    for (int g = warp; g < G; g += kThreads / 32) {
      float m = -INFINITY;
      for (int j = lane; j < n; j += 32) m = fmaxf(m, sc[g * a.cs_max + j]);
#pragma unroll
      for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      float l = 0.f;
      for (int j = lane; j < n; j += 32) {
        const float e = __expf(sc[g * a.cs_max + j] - m);
        sc[g * a.cs_max + j] = e;
        l += e;
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
      if (lane == 0) {
        s_m[g] = m;
        s_l[g] = l;
      }
    }
    __syncthreads();
  }
  // ---- 4. this slice's (o, max, sum) into CTA 0's shared memory
  for (int g = warp; g < G; g += kThreads / 32) {
    float o0 = 0.f, o1 = 0.f;
    if (pos_ok) {
      const float* pg = sc + g * a.cs_max;
      for (int j = 0; j < n; ++j) {
        const float2 va = load2<FP8>(vs + (size_t)j * RB, 2 * lane);
        o0 = fmaf(pg[j], va.x, o0);
        o1 = fmaf(pg[j], va.y, o1);
      }
    }
    float* dst = mrg + ((size_t)c * G + g) * (kD + 2);
    st_remote_f32(dst + 2 * lane, 0u, o0);
    st_remote_f32(dst + 2 * lane + 1, 0u, o1);
    if (lane == 0) {
      st_remote_f32(dst + kD, 0u, pos_ok && n > 0 ? s_m[g] : -INFINITY);
      st_remote_f32(dst + kD + 1, 0u, pos_ok && n > 0 ? s_l[g] : 0.f);
    }
  }
  cluster_barrier_sync();
  if (c != 0 || !pos_ok) return;
  for (int g = warp; g < G; g += kThreads / 32) {
    const float sink = a.sinks[h * G + g];
    float M = sink;
    for (int t = 0; t < CN; ++t) M = fmaxf(M, mrg[((size_t)t * G + g) * (kD + 2) + kD]);
    float den = __expf(sink - M), o0 = 0.f, o1 = 0.f;
    for (int t = 0; t < CN; ++t) {
      const float* q = mrg + ((size_t)t * G + g) * (kD + 2);
      const float w = q[kD + 1] > 0.f ? __expf(q[kD] - M) : 0.f;
      den = fmaf(w, q[kD + 1], den);
      o0 = fmaf(w, q[2 * lane], o0);
      o1 = fmaf(w, q[2 * lane + 1], o1);
    }
    const float inv = 1.f / den;
    uint16_t* o = a.out + (h * G + g) * kD;
    o[2 * lane] = f32_to_bf16_bits(o0 * inv);
    o[2 * lane + 1] = f32_to_bf16_bits(o1 * inv);
  }
}

size_t qkv_attn_smem(int G, int H, int CN, int max_seq, bool fp8) {
  const int cs_max = (max_seq + CN - 1) / CN;
  const size_t rowb = (fp8 ? kD : 2 * kD) + 16;
  return sizeof(float) * (2 * (size_t)H + (size_t)(G + 2) * kD + (size_t)G * kD + 2 * kD + (size_t)G * cs_max +
                          (size_t)CN * G * (kD + 2)) + 16 + 2 * rowb * cs_max;
}

}  // namespace

// Position slices per KV head: about 128 positions each (8 KV heads x 33
// slices = 264 CTAs at a 4 K context, two per SM), at most 64.
int attn_slices(int max_seq) {
  int S = (max_seq + 127) / 128;
  return S < 1 ? 1 : (S > 64 ? 64 : S);
}

}  // namespace tsb

using namespace tsb;

static size_t attn_ws_bytes(int nq, int nkv, int max_seq, int batch) {
  if (nq <= 0 || nkv <= 0 || max_seq <= 0 || batch <= 0 || nq % nkv) return 0;
  const int S = attn_slices(max_seq), G = nq / nkv;
  const size_t cnt = ((size_t)batch * nkv * 4 + 255) & ~size_t(255);
  return 256 + cnt + sizeof(float) * (size_t)batch * nkv * S * G * (kD + 2);
}

extern "C" size_t tsb_gqa_decode_batch_workspace(int32_t n_q_heads, int32_t n_kv_heads, int32_t max_seq, int32_t batch) {
  return attn_ws_bytes(n_q_heads, n_kv_heads, max_seq, batch);
}

extern "C" size_t tsb_gqa_decode_workspace(int32_t n_q_heads, int32_t n_kv_heads, int32_t max_seq) {
  return attn_ws_bytes(n_q_heads, n_kv_heads, max_seq, 1);
}

extern "C" int tsb_gqa_decode_attention_batch(const void* qkv, int32_t n_q_heads, int32_t n_kv_heads,
                                              int32_t head_dim, const void* cos, const void* sin, const int64_t* pos,
                                              const int32_t* slots, int64_t slot_stride, void* k_cache,
                                              void* v_cache, int32_t cache_fp8, int32_t max_seq, int32_t window,
                                              const float* sinks, float scale, void* out, int32_t batch,
                                              void* workspace, size_t workspace_bytes, void* stream) {
  if (!qkv || !cos || !sin || !pos || !k_cache || !v_cache || !sinks || !out || !workspace)
    return set_error(TSB_ERR_INVALID, "null pointer");
  if (head_dim != kD) return set_error(TSB_ERR_UNSUPPORTED, "head_dim must be 64");
  if (n_kv_heads <= 0 || n_q_heads <= 0 || n_q_heads % n_kv_heads || n_q_heads / n_kv_heads > 16 || n_kv_heads > 65535)
    return set_error(TSB_ERR_INVALID, "n_q_heads must be a multiple of n_kv_heads, at most 16 per KV head");
  if (max_seq <= 0 || window < 0) return set_error(TSB_ERR_INVALID, "bad max_seq / window");
  if (batch <= 0 || batch > 65535) return set_error(TSB_ERR_INVALID, "batch must be in [1, 65535]");
  if (slots && slot_stride < (int64_t)n_kv_heads * max_seq * kD) return set_error(TSB_ERR_INVALID, "slot_stride too small");
  if (cache_fp8 != 0 && cache_fp8 != 1) return set_error(TSB_ERR_INVALID, "cache_fp8 must be 0 or 1");
  if (workspace_bytes < attn_ws_bytes(n_q_heads, n_kv_heads, max_seq, batch))
    return set_error(TSB_ERR_WORKSPACE, "workspace too small");
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return set_error(TSB_ERR_INVALID, "workspace must be 256-byte aligned");
  AttnArgs a{};
  a.qkv = static_cast<const uint16_t*>(qkv);
  a.cos = static_cast<const uint16_t*>(cos);
  a.sin = static_cast<const uint16_t*>(sin);
  a.pos = pos;
  a.kc = k_cache;
  a.vc = v_cache;
  a.sinks = sinks;
  a.out = static_cast<uint16_t*>(out);
  a.slots = slots;
  a.slot_stride = slot_stride;
  char* ws = static_cast<char*>(workspace);
  a.err = reinterpret_cast<int32_t*>(ws);
  a.counters = reinterpret_cast<unsigned*>(ws + 256);
  a.part = reinterpret_cast<float*>(ws + 256 + (((size_t)batch * n_kv_heads * 4 + 255) & ~size_t(255)));
  a.nq = n_q_heads;
  a.nkv = n_kv_heads;
  a.G = n_q_heads / n_kv_heads;
  a.S = attn_slices(max_seq);
  a.max_seq = max_seq;
  a.window = window;
  a.cs_max = (max_seq + a.S - 1) / a.S;
  a.scale = scale;
  const size_t rowb = (cache_fp8 ? kD : 2 * kD) + 16;
  const size_t smem = sizeof(float) * ((size_t)a.G * kD + 2 * kD + (size_t)a.G * a.cs_max) + 16 + 2 * rowb * a.cs_max;
  if (smem > 200 * 1024) return set_error(TSB_ERR_UNSUPPORTED, "max_seq too large for the decode-attention slices");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid(a.S, n_kv_heads, batch);
  cudaError_t e;
  if (cache_fp8) {
    if (smem > 48 * 1024) cudaFuncSetAttribute(gqa_decode_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    e = launch_pdl(gqa_decode_kernel<true>, grid, kThreads, smem, st, a);
  } else {
    if (smem > 48 * 1024) cudaFuncSetAttribute(gqa_decode_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    e = launch_pdl(gqa_decode_kernel<false>, grid, kThreads, smem, st, a);
  }
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  return TSB_OK;
}

extern "C" int tsb_gqa_decode_attention(const void* qkv, int32_t n_q_heads, int32_t n_kv_heads, int32_t head_dim,
                                        const void* cos, const void* sin, const int64_t* pos, void* k_cache,
                                        void* v_cache, int32_t cache_fp8, int32_t max_seq, int32_t window,
                                        const float* sinks, float scale, void* out, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  return tsb_gqa_decode_attention_batch(qkv, n_q_heads, n_kv_heads, head_dim, cos, sin, pos, nullptr, 0, k_cache,
                                        v_cache, cache_fp8, max_seq, window, sinks, scale, out, 1, workspace,
                                        workspace_bytes, stream);
}

extern "C" int tsb_add_rmsnorm(float* x, const void* delta, int32_t delta_dtype, const float* weight, float eps,
                               int32_t rows, int32_t hidden, void* out, void* stream) {
  if (!x || !weight) return set_error(TSB_ERR_INVALID, "null pointer");
  if (rows < 0 || hidden <= 0) return set_error(TSB_ERR_INVALID, "bad shape");
  if (hidden > kNormThreads * kPer) return set_error(TSB_ERR_UNSUPPORTED, "hidden must be <= 4096");
  if (delta && delta_dtype != TSB_DT_F32 && delta_dtype != TSB_DT_BF16)
    return set_error(TSB_ERR_INVALID, "delta must be fp32 or bf16");
  if (rows == 0) return TSB_OK;
  const cudaError_t e = launch_pdl(add_rmsnorm_kernel, dim3(rows), kNormThreads, 0, static_cast<cudaStream_t>(stream),
                                   x, delta, (int)(delta_dtype == TSB_DT_F32), weight, eps, (int)hidden,
                                   static_cast<uint16_t*>(out));
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  return TSB_OK;
}

static int run_gemv(int mode, GemvArgs a, void* stream) {
  if (!a.W) return set_error(TSB_ERR_INVALID, "null pointer");
  if (a.N <= 0 || a.K <= 0 || a.K % 8 || a.K > 16384) return set_error(TSB_ERR_INVALID, "N must be positive, K a positive multiple of 8 up to 16384");
  if (reinterpret_cast<uintptr_t>(a.W) & 15) return set_error(TSB_ERR_INVALID, "weight must be 16-byte aligned");
  if (mode == GV_RESIDUAL && (a.N > 16384 || a.N % 4)) return set_error(TSB_ERR_INVALID, "N must be a multiple of 4, <= 16384, for the residual form");
  const int smem_elems = mode == GV_RESIDUAL ? (a.K > a.N ? a.K : a.N) : (mode == GV_NORM ? 2 * a.K : a.K);
  const size_t smem = sizeof(float) * smem_elems;
  const dim3 grid((a.N + kGemvWarps - 1) / kGemvWarps);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  switch (mode) {
    case GV_NORM:
      if (smem > 48 * 1024) cudaFuncSetAttribute(gemv_bf16_kernel<GV_NORM>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      e = launch_pdl(gemv_bf16_kernel<GV_NORM>, grid, kGemvWarps * 32, smem, st, a);
      break;
    case GV_RESIDUAL:
      if (smem > 48 * 1024) cudaFuncSetAttribute(gemv_bf16_kernel<GV_RESIDUAL>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      e = launch_pdl(gemv_bf16_kernel<GV_RESIDUAL>, grid, kGemvWarps * 32, smem, st, a);
      break;
    default:
      if (smem > 48 * 1024) cudaFuncSetAttribute(gemv_bf16_kernel<GV_PLAIN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      e = launch_pdl(gemv_bf16_kernel<GV_PLAIN>, grid, kGemvWarps * 32, smem, st, a);
  }
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  return TSB_OK;
}

extern "C" int tsb_gemv_bf16(const void* weight, const void* bias, int32_t N, int32_t K, const void* x, void* y,
                             void* stream) {
  if (N == 0) return TSB_OK;
  if (!x || !y) return set_error(TSB_ERR_INVALID, "null pointer");
  GemvArgs a{};
  a.W = static_cast<const uint16_t*>(weight);
  a.bias = static_cast<const uint16_t*>(bias);
  a.N = N;
  a.K = K;
  a.x = static_cast<const uint16_t*>(x);
  a.y = static_cast<uint16_t*>(y);
  return run_gemv(GV_PLAIN, a, stream);
}

extern "C" int tsb_norm_gemv_bf16(const float* x_in, const float* delta, float* x_out, const float* norm_weight,
                                  float eps, const void* weight, const void* bias, int32_t N, int32_t K, void* y,
                                  void* stream) {
  if (!x_in || !x_out || !norm_weight || !y) return set_error(TSB_ERR_INVALID, "null pointer");
  if (x_out == x_in || (delta && x_out == delta)) return set_error(TSB_ERR_INVALID, "x_out must not alias x_in or delta");
  GemvArgs a{};
  a.W = static_cast<const uint16_t*>(weight);
  a.bias = static_cast<const uint16_t*>(bias);
  a.N = N;
  a.K = K;
  a.y = static_cast<uint16_t*>(y);
  a.x_in = x_in;
  a.delta = delta;
  a.x_out = x_out;
  a.norm_w = norm_weight;
  a.eps = eps;
  return run_gemv(GV_NORM, a, stream);
}

extern "C" int tsb_gemv_bf16_residual(const void* weight, const void* bias, int32_t N, int32_t K, const void* x,
                                      float* resid, const float* norm_weight, float eps, void* h_out,
                                      uint32_t* counter, void* stream) {
  if (!x || !resid || !norm_weight || !h_out || !counter) return set_error(TSB_ERR_INVALID, "null pointer");
  GemvArgs a{};
  a.W = static_cast<const uint16_t*>(weight);
  a.bias = static_cast<const uint16_t*>(bias);
  a.N = N;
  a.K = K;
  a.x = static_cast<const uint16_t*>(x);
  a.resid = resid;
  a.norm_w = norm_weight;
  a.eps = eps;
  a.h_out = static_cast<uint16_t*>(h_out);
  a.counter = counter;
  return run_gemv(GV_RESIDUAL, a, stream);
}

extern "C" int tsb_norm_qkv_attention(const float* x_in, const float* delta, float* x_out, const float* norm_weight,
                                      float eps, const void* weight, const void* bias, int32_t hidden,
                                      int32_t n_q_heads, int32_t n_kv_heads, int32_t head_dim, const void* cos,
                                      const void* sin, const int64_t* pos, void* k_cache, void* v_cache,
                                      int32_t cache_fp8, int32_t max_seq, int32_t window, const float* sinks,
                                      float scale, void* out, void* stream) {
  if (!x_in || !x_out || !norm_weight || !weight || !cos || !sin || !pos || !k_cache || !v_cache || !sinks || !out)
    return set_error(TSB_ERR_INVALID, "null pointer");
  if (x_out == x_in || (delta && x_out == delta)) return set_error(TSB_ERR_INVALID, "x_out must not alias x_in or delta");
  if (head_dim != kD) return set_error(TSB_ERR_UNSUPPORTED, "head_dim must be 64");
  if (n_kv_heads <= 0 || n_q_heads <= 0 || n_q_heads % n_kv_heads || n_q_heads / n_kv_heads > 16)
    return set_error(TSB_ERR_INVALID, "n_q_heads must be a multiple of n_kv_heads, at most 16 per KV head");
  if (hidden <= 0 || hidden % 8 || hidden > 8192) return set_error(TSB_ERR_INVALID, "hidden must be a multiple of 8, <= 8192");
  if (max_seq <= 0 || window < 0) return set_error(TSB_ERR_INVALID, "bad max_seq / window");
  if (cache_fp8 != 0 && cache_fp8 != 1) return set_error(TSB_ERR_INVALID, "cache_fp8 must be 0 or 1");
  if (reinterpret_cast<uintptr_t>(weight) & 15) return set_error(TSB_ERR_INVALID, "weight must be 16-byte aligned");
  const int G = n_q_heads / n_kv_heads;
  // cluster size: 16 CTAs per KV head when the device can co-schedule all
  // of the grid's clusters that way, else 8 (the portable maximum)
  int CN = 0;
  size_t smem = 0;
  auto kern = cache_fp8 ? qkv_attn_kernel<true> : qkv_attn_kernel<false>;
  {
    for (int cand : {16, 8}) {
      const size_t sm = qkv_attn_smem(G, hidden, cand, max_seq, cache_fp8);
      if (sm > 220 * 1024) continue;
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
      if (cand > 8) cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(n_kv_heads * cand);
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = sm;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = cand;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) == cudaSuccess && clusters >= n_kv_heads) {
        CN = cand;
        break;
      }
      cudaGetLastError();
    }
  }
  if (CN == 0) return set_error(TSB_ERR_UNSUPPORTED, "the fused q|k|v + attention kernel does not fit this shape");
  smem = qkv_attn_smem(G, hidden, CN, max_seq, cache_fp8);
  if (smem > 220 * 1024) return set_error(TSB_ERR_UNSUPPORTED, "max_seq too large for the fused kernel");
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  QkvAttnArgs a{};
  a.x_in = x_in;
  a.delta = delta;
  a.x_out = x_out;
  a.norm_w = norm_weight;
  a.eps = eps;
  a.W = static_cast<const uint16_t*>(weight);
  a.bias = static_cast<const uint16_t*>(bias);
  a.cos = static_cast<const uint16_t*>(cos);
  a.sin = static_cast<const uint16_t*>(sin);
  a.pos = pos;
  a.kc = k_cache;
  a.vc = v_cache;
  a.sinks = sinks;
  a.out = static_cast<uint16_t*>(out);
  a.nq = n_q_heads;
  a.nkv = n_kv_heads;
  a.G = G;
  a.H = hidden;
  a.CN = CN;
  a.max_seq = max_seq;
  a.window = window;
  a.cs_max = (max_seq + CN - 1) / CN;
  a.scale = scale;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_kv_heads * CN);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = CN;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  return TSB_OK;
}
