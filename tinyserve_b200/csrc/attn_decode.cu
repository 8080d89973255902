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
  float* part;           // [nkv, S, G, D + 2]
  unsigned* counters;    // [nkv]
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
__global__ void __launch_bounds__(kThreads) gqa_decode_kernel(AttnArgs a) {
  extern __shared__ float sm[];
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
  const int n = max(0, c1 - c0);
  const int64_t hb = (int64_t)h * a.max_seq * kD;
  // scores: warp per position
  for (int j = warp; j < n; j += kThreads / 32) {
    const int p = c0 + j;
    float2 k2;
    if (p == pos)
      k2 = make_float2(knew[2 * lane], knew[2 * lane + 1]);
    else
      k2 = load2<FP8>(a.kc, hb + (int64_t)p * kD + 2 * lane);
    for (int g = 0; g < G; ++g) {
      float v = qs[g * kD + 2 * lane] * k2.x + qs[g * kD + 2 * lane + 1] * k2.y;
#pragma unroll
      for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) sc[g * a.cs_max + j] = v * a.scale;
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
    float o0 = 0.f, o1 = 0.f;
    const float* pg = sc + g * a.cs_max;
    for (int j = 0; j < n; ++j) {
      const int p = c0 + j;
      float2 v2;
      if (p == pos)
        v2 = make_float2(vnew[2 * lane], vnew[2 * lane + 1]);
      else
        v2 = load2<FP8>(a.vc, hb + (int64_t)p * kD + 2 * lane);
      o0 = fmaf(pg[j], v2.x, o0);
      o1 = fmaf(pg[j], v2.y, o1);
    }
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
// out[r] = bf16(w * x[r] * rsqrt(mean(x[r]^2) + eps)).  One CTA per row.
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(float* x, const void* delta, int delta_f32, const float* w,
                                                          float eps, int H, uint16_t* out) {
  const int r = blockIdx.x;
  float* xr = x + (int64_t)r * H;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float v = xr[i];
    if (delta)
      v += delta_f32 ? static_cast<const float*>(delta)[(int64_t)r * H + i]
                     : bf(static_cast<const uint16_t*>(delta)[(int64_t)r * H + i]);
    xr[i] = v;
    ss = fmaf(v, v, ss);
  }
  __shared__ float red[8];
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / H + eps);
  if (out)
    for (int i = threadIdx.x; i < H; i += blockDim.x) out[(int64_t)r * H + i] = f32_to_bf16_bits(w[i] * (xr[i] * inv));
}

}  // namespace

int attn_slices(int max_seq) {
  int S = (max_seq + 255) / 256;
  return S < 1 ? 1 : (S > 64 ? 64 : S);
}

}  // namespace tsb

using namespace tsb;

extern "C" size_t tsb_gqa_decode_workspace(int32_t n_q_heads, int32_t n_kv_heads, int32_t max_seq) {
  if (n_q_heads <= 0 || n_kv_heads <= 0 || max_seq <= 0 || n_q_heads % n_kv_heads) return 0;
  const int S = attn_slices(max_seq), G = n_q_heads / n_kv_heads;
  return 256 + sizeof(float) * (size_t)n_kv_heads * S * G * (kD + 2);
}

extern "C" int tsb_gqa_decode_attention(const void* qkv, int32_t n_q_heads, int32_t n_kv_heads, int32_t head_dim,
                                        const void* cos, const void* sin, const int64_t* pos, void* k_cache,
                                        void* v_cache, int32_t cache_fp8, int32_t max_seq, int32_t window,
                                        const float* sinks, float scale, void* out, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  if (!qkv || !cos || !sin || !pos || !k_cache || !v_cache || !sinks || !out || !workspace)
    return set_error(TSB_ERR_INVALID, "null pointer");
  if (head_dim != kD) return set_error(TSB_ERR_UNSUPPORTED, "head_dim must be 64");
  if (n_kv_heads <= 0 || n_q_heads <= 0 || n_q_heads % n_kv_heads || n_q_heads / n_kv_heads > 16 || n_kv_heads > 65535)
    return set_error(TSB_ERR_INVALID, "n_q_heads must be a multiple of n_kv_heads, at most 16 per KV head");
  if (max_seq <= 0 || window < 0) return set_error(TSB_ERR_INVALID, "bad max_seq / window");
  if (cache_fp8 != 0 && cache_fp8 != 1) return set_error(TSB_ERR_INVALID, "cache_fp8 must be 0 or 1");
  if (workspace_bytes < tsb_gqa_decode_workspace(n_q_heads, n_kv_heads, max_seq))
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
  char* ws = static_cast<char*>(workspace);
  a.err = reinterpret_cast<int32_t*>(ws);
  a.counters = reinterpret_cast<unsigned*>(ws + 4);
  a.part = reinterpret_cast<float*>(ws + 256);
  a.nq = n_q_heads;
  a.nkv = n_kv_heads;
  a.G = n_q_heads / n_kv_heads;
  a.S = attn_slices(max_seq);
  a.max_seq = max_seq;
  a.window = window;
  a.cs_max = (max_seq + a.S - 1) / a.S;
  a.scale = scale;
  if (n_kv_heads > 60) return set_error(TSB_ERR_UNSUPPORTED, "at most 60 KV heads (counter space)");
  const size_t smem = sizeof(float) * ((size_t)a.G * kD + 2 * kD + (size_t)a.G * a.cs_max);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (cache_fp8) {
    if (smem > 48 * 1024) cudaFuncSetAttribute(gqa_decode_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    gqa_decode_kernel<true><<<dim3(a.S, n_kv_heads), kThreads, smem, st>>>(a);
  } else {
    if (smem > 48 * 1024) cudaFuncSetAttribute(gqa_decode_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    gqa_decode_kernel<false><<<dim3(a.S, n_kv_heads), kThreads, smem, st>>>(a);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  return TSB_OK;
}

extern "C" int tsb_add_rmsnorm(float* x, const void* delta, int32_t delta_dtype, const float* weight, float eps,
                               int32_t rows, int32_t hidden, void* out, void* stream) {
  if (!x || !weight) return set_error(TSB_ERR_INVALID, "null pointer");
  if (rows < 0 || hidden <= 0) return set_error(TSB_ERR_INVALID, "bad shape");
  if (delta && delta_dtype != TSB_DT_F32 && delta_dtype != TSB_DT_BF16)
    return set_error(TSB_ERR_INVALID, "delta must be fp32 or bf16");
  if (rows == 0) return TSB_OK;
  add_rmsnorm_kernel<<<rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, delta, delta_dtype == TSB_DT_F32, weight,
                                                                           eps, hidden, static_cast<uint16_t*>(out));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  return TSB_OK;
}
