// Grouped (prefill) MoE layer: T tokens, each routed to top_k experts.
//
// Replaces the reference's batched expert path
// (tinyserve/expert_pipeline.py:166-239 execute_layer_experts_batched with
// group_tokens_by_expert, tinyserve/_fast_cache.pyx:60-85): tokens are grouped
// by expert on the GPU, every expert runs one grouped GEMM over its tokens on
// the tcgen05 tensor cores, and the k expert outputs of a token are combined in
// slot order.
//
// Stages (all on one stream, nothing returns to the host):
//   route_count / route_place  deterministic grouping: expert e owns permuted
//                              rows [start_e, start_e + count_e), padded to 128 (256 for CTA pairs);
//                              inside an expert, rows keep (token, slot) order
//   gather_rows                token rows -> permuted fp16 tiles, each row
//                              scaled by a power of two (exact) so that its
//                              largest element sits in [2^14, 2^15)
//   tile_weights<F>            each routed expert's weights decoded bit-exactly
//                              (same arithmetic as tsb_dequant) and rounded to
//                              fp16 tiles
//   grouped_gemm (gate/up)     D = X_e W_gu^T on tcgen05, fp32 accumulators in
//                              tensor memory; epilogue undoes the row scale,
//                              adds biases, applies the activation and writes
//                              fp16 activation tiles
//   grouped_gemm (down)        D = A_e W_dn^T; epilogue adds the bias, writes
//                              fp32 rows
//   combine                    out[t] = sum_j w[t,j] * Y[row(t,j)], j ascending
//
// Numerics: the products run in fp16 x fp16 with fp32 accumulation.  Weight
// rounding to fp16 (11-bit significand) keeps layer outputs within ~3e-4
// relative L2 of fp32 math on the dequantised weights; bf16 operands (8-bit)
// would not meet 1e-3.  MXFP4 weights within the fp16 range are exact.
//
// Operand tiles live in HBM already in the tensor core's shared-memory image
// (K-major, 128-byte swizzle, 64 K-elements per 128-byte row), so a pipeline
// stage is two plain bulk copies (cp.async.bulk, no tensor map) completing on
// an mbarrier.
#include <algorithm>
#include <cstdio>
#include <cstdlib>

#include "../../include/tsb_moe.h"
#include "moe_math.cuh"
#include "qformats.cuh"
#include "tc05.cuh"
#include "tsb_internal.h"

namespace tsb {

constexpr int kBM = 128;                  // permuted rows per tile (tensor-memory lanes)
constexpr int kBK = 64;                   // K elements per k-block (one 128-byte row)
constexpr int kATile = kBM * 128;         // 16 KB
constexpr int kBTileMax = 256 * 128;      // 32 KB (N tile <= 256 rows)
constexpr int kStage = kATile + kBTileMax;
constexpr int kNS = 4;                    // pipeline depth
// warp 0 producer, warp 1 MMA, warps 4-7 and kEpiB..kEpiB+3 epilogue (two sets
// splitting the accumulator's columns; warp w reads tensor-memory lanes
// 32*(w%4)..), warps 8-15 in-GEMM decode (BF variant)
constexpr int kEpiB = 8, kEpiBFused = 16;
constexpr int kGemmThreads = 384;
constexpr int kTmemCols = 512;            // two accumulators of <= 256 columns
constexpr size_t kGemmSmem = 1024 + (size_t)kNS * kStage + 256;

// ------------------------------------------------------------------ routing
// Grouping of the T*k (token, slot) entries by expert, in three small kernels
// over chunks of kRouteChunk entries:
//   route_chunk_count  per-chunk histogram (shared-memory atomics; integer
//                      counts, so the order of the atomics does not matter)
//   route_scan         per expert: total, exclusive prefix over chunks and the
//                      expert's first row (experts padded to 128- or 256-row blocks);
//                      padding rows, row-block owners and the block count
//   route_chunk_place  one warp per chunk walks its entries in index order and
//                      gives each the next row of its expert (warp match +
//                      popcount), so inside an expert rows keep (token, slot)
//                      order and the grouping is deterministic
// Ids outside [0, E) are reported in the error word and get row_of = -1 (they
// contribute nothing, as in decode).
constexpr int kRouteChunk = 1024;

__global__ void __launch_bounds__(256) route_chunk_count(const int32_t* __restrict__ ids, int n, int E,
                                                         int* __restrict__ ccount, int* __restrict__ row_of, int* err) {
  extern __shared__ int hist[];
  const int c = blockIdx.x;
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  for (int j = threadIdx.x; j < kRouteChunk; j += blockDim.x) {
    const int i = c * kRouteChunk + j;
    if (i >= n) break;
    const int v = ids[i];
    if ((unsigned)v < (unsigned)E) {
      atomicAdd(&hist[v], 1);
    } else {
      // negative ids: slots this call skips (another rank's experts);
      // ids >= E: a routing error
      row_of[i] = -1;
      if (v >= 0) atomicExch(err, kDevBadPlan);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) ccount[(size_t)c * E + e] = hist[e];
}

__global__ void __launch_bounds__(1024) route_scan(int nchunks, int E, int* __restrict__ ccount,
                                                   int* __restrict__ counts, int* __restrict__ row_src,
                                                   int* __restrict__ mb_expert, int* __restrict__ total_mb,
                                                   int pad) {
  __shared__ int wsum[32];
  const int e = threadIdx.x;
  int tot = 0;
  if (e < E) {
    for (int c = 0; c < nchunks; ++c) {  // exclusive prefix over chunks, in place
      const int v = ccount[(size_t)c * E + e];
      ccount[(size_t)c * E + e] = tot;
      tot += v;
    }
    counts[e] = tot;
  }
  // exclusive scan of the padded totals over experts (block-wide)
  const int padded = (e < E) ? (tot + pad - 1) / pad * pad : 0;
  const int lane = e & 31, warp = e >> 5;
  int inc = padded;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += u;
  }
  if (lane == 31) wsum[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    const int v = wsum[lane];
    int w = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += u;
    }
    wsum[lane] = w - v;
  }
  __syncthreads();
  const int start = wsum[warp] + inc - padded;
  if (e < E) {
    for (int c = 0; c < nchunks; ++c) ccount[(size_t)c * E + e] += start;
    for (int r = tot; r < padded; ++r) row_src[start + r] = -1;
    for (int b = 0; b < padded / kBM; ++b) mb_expert[start / kBM + b] = e;
    if (e == E - 1) *total_mb = (start + padded) / kBM;
  }
}

__global__ void __launch_bounds__(32) route_chunk_place(const int32_t* __restrict__ ids, int n, int top_k, int E,
                                                        const int* __restrict__ cbase, int* __restrict__ row_of,
                                                        int* __restrict__ row_src) {
  extern __shared__ int running[];
  const int c = blockIdx.x, lane = threadIdx.x;
  for (int e = lane; e < E; e += 32) running[e] = cbase[(size_t)c * E + e];
  __syncwarp();
  for (int j = 0; j < kRouteChunk; j += 32) {
    const int i = c * kRouteChunk + j + lane;
    const int v = i < n ? ids[i] : -1;
    const bool ok = (unsigned)v < (unsigned)E;
    const unsigned peers = __match_any_sync(0xffffffffu, ok ? v : -1 - lane);
    if (ok) {
      const int r = running[v] + __popc(peers & ((1u << lane) - 1u));
      row_of[i] = r;
      row_src[r] = i / top_k;
    }
    __syncwarp();
    if (ok && lane == __ffs(peers) - 1) running[v] += __popc(peers);
    __syncwarp();
  }
}

// One warp per permuted row: copy token row x[src] (bf16) into the fp16 A
// tiles, scaled by 2^-shift (shift = exponent of the row's largest |x| - 14,
// so the row uses the fp16 range fully and nothing overflows).  Padding rows
// are zero.  K columns beyond H are zero.
__global__ void __launch_bounds__(256) gather_rows_kernel(const uint16_t* __restrict__ x, int H, int KB,
                                                          const int* __restrict__ row_src,
                                                          const int* __restrict__ total_mb, uint8_t* __restrict__ Xp,
                                                          int8_t* __restrict__ row_shift) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int R = blockIdx.x * 8 + warp;
  if (R >= *total_mb * kBM) return;
  const int src = row_src[R];
  const int mb = R / kBM, m = R % kBM;
  const int n8 = H / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)(src < 0 ? 0 : src) * H);
  uint32_t mx = 0;  // max |x| as bits (bf16 magnitude << 16 orders like the value)
  if (src >= 0) {
    for (int c = lane; c < n8; c += 32) {
      const uint4 v = xr[c];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        mx = max(mx, (w[q] << 16) & 0x7FFF0000u);
        mx = max(mx, w[q] & 0x7FFF0000u);
      }
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  int sh = 0;
  if (mx != 0 && mx < 0x7F800000u) sh = max(-100, min(100, (int)(mx >> 23) - 127 - 14));
  const float sc = __uint_as_float((uint32_t)(127 - sh) << 23);  // 2^-sh, exact
  uint8_t* rowp = Xp + (size_t)mb * KB * kATile + (size_t)m * 128;
  for (int c = lane; c < KB * 8; c += 32) {
    uint4 o = make_uint4(0, 0, 0, 0);
    if (src >= 0 && c < n8) {
      const uint4 v = xr[c];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      uint32_t h[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float lo = __fmul_rn(__uint_as_float(w[q] << 16), sc);
        const float hi = __fmul_rn(__uint_as_float(w[q] & 0xFFFF0000u), sc);
        const __half2 p = __halves2half2(__float2half_rn(lo), __float2half_rn(hi));
        h[q] = *reinterpret_cast<const uint32_t*>(&p);
      }
      o = make_uint4(h[0], h[1], h[2], h[3]);
    }
    *reinterpret_cast<uint4*>(rowp + (size_t)(c >> 3) * kATile + (((c & 7) ^ (m & 7)) << 4)) = o;
  }
  if (lane == 0) row_shift[R] = (int8_t)sh;
}

// ------------------------------------------------------------------ weights
// Eight consecutive elements (flat index q0, a multiple of 8) of a weight
// stream, decoded with tsb_dequant's arithmetic (gguf_dequant_torch.py:118-249,
// mxfp4.py:20-44).
template <int F>
__device__ __forceinline__ void deq8(const uint8_t* __restrict__ w, const uint8_t* __restrict__ s, int64_t q0,
                                     float (&v)[8]) {
  const int l0 = (int)(q0 & 31);
  if (F == FMT_Q8_0) {
    const uint8_t* b = w + (q0 >> 5) * 34;
    const float d = half_bits_to_f32((uint16_t)(b[0] | (b[1] << 8)));
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(d, (float)(int8_t)b[2 + l0 + i]);
  } else if (F == FMT_Q4_K || F == FMT_Q5_K) {
    const uint8_t* b = w + (q0 >> 8) * FmtT<F>::BB;
    const int j = (int)((q0 >> 5) & 7);
    const float d = half_bits_to_f32((uint16_t)(b[0] | (b[1] << 8)));
    const float dmin = half_bits_to_f32((uint16_t)(b[2] | (b[3] << 8)));
    int sc, m;
    kq_scale_min(b + 4, j, sc, m);
    const float dsc = __fmul_rn(d, (float)sc), dm = __fmul_rn(dmin, (float)m);
    const uint8_t* qs = b + (F == FMT_Q4_K ? 16 : 48) + 32 * (j >> 1) + l0;
    const int sh = 4 * (j & 1);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int q = (qs[i] >> sh) & 0xF;
      if (F == FMT_Q5_K) q |= ((b[16 + l0 + i] >> j) & 1) << 4;
      v[i] = __fsub_rn(__fmul_rn(dsc, (float)q), dm);
    }
  } else if (F == FMT_Q6_K) {
    const uint8_t* b = w + (q0 >> 8) * 210;
    const int g = (int)((q0 >> 5) & 7), h = g >> 2, gg = g & 3;
    const float d = half_bits_to_f32((uint16_t)(b[208] | (b[209] << 8)));
    const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192) + 2 * g;
    const float dd = __fmul_rn(d, (float)sc[l0 < 16 ? 0 : 1]);  // 8 elements never straddle l = 16
    const uint8_t* ql = b + 64 * h + 32 * (gg & 1) + l0;
    const uint8_t* qh = b + 128 + 32 * h + l0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int q = (((ql[i] >> (4 * (gg >> 1))) & 0xF) | (((qh[i] >> (2 * gg)) & 3) << 4)) - 32;
      v[i] = __fmul_rn(dd, (float)q);
    }
  } else {  // MXFP4
    const uint8_t* b = w + (q0 >> 5) * 16 + (l0 >> 1);
    const int e = (int)s[q0 >> 5] - 127;
    const int e1 = e / 2, e2 = e - e1;
    const float p1 = __uint_as_float((uint32_t)(e1 + 127) << 23), p2 = __uint_as_float((uint32_t)(e2 + 127) << 23);
    const uint32_t q = *reinterpret_cast<const uint32_t*>(b);  // 4-byte aligned: l0 is a multiple of 8
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      // e2m1 -> f16 is exact, so this is the table value of each code
      const uint32_t h = cvt_e2m1x2((q >> (8 * i)) & 0xFF);
      v[2 * i] = __fmul_rn(__fmul_rn(half_bits_to_f32((uint16_t)(h & 0xFFFF)), p1), p2);
      v[2 * i + 1] = __fmul_rn(__fmul_rn(half_bits_to_f32((uint16_t)(h >> 16)), p1), p2);
    }
  }
}

struct TileWArgs {
  const TsbExpert* experts;
  const int* counts;
  int proj;     // 0: gate/up, 1: down
  int layout;   // TSB_GU_*
  int I;        // intermediate size
  int N;        // output rows of the projection (2I or H)
  int K;        // input columns (H or I)
  int KB;       // k-blocks (K rounded up to 64, / 64)
  int NT;       // rows per N tile
  uint8_t* out;
  int64_t estride;  // bytes per expert
};

// One CTA per (N tile, group of kTileKB k-blocks) of one expert (blockIdx.y):
// eight threads per tile row, one 16-byte chunk (8 elements) per k-block each,
// so a warp writes four whole 128-byte rows per k-block.  A thread decodes its
// chunk of all kTileKB k-blocks before storing any, which keeps kTileKB
// independent loads in flight per thread.  For the gate/up projection a tile's
// first NT/2 rows are gate features and the next NT/2 the same up features,
// whatever the source layout.
constexpr int kTileKB = 4;

template <int F>
__global__ void __launch_bounds__(256) tile_weights_kernel(const TileWArgs a) {
  const int e = blockIdx.y;
  if (a.counts[e] == 0) return;
  const TsbExpert& E = a.experts[e];
  const int nkq = (a.KB + kTileKB - 1) / kTileKB;
  const int nt = blockIdx.x / nkq, kb0 = (blockIdx.x % nkq) * kTileKB;
  const int half = a.NT / 2;
  uint8_t* base = a.out + (int64_t)e * a.estride + (int64_t)nt * a.KB * a.NT * 128;
  for (int q = threadIdx.x; q < a.NT * 8; q += blockDim.x) {
    const int r = q >> 3, c = q & 7;
    const uint8_t* w;
    const uint8_t* s;
    int64_t row;
    if (a.proj == 1) {
      w = static_cast<const uint8_t*>(E.down);
      s = static_cast<const uint8_t*>(E.down_scales);
      row = (int64_t)nt * a.NT + r;
    } else {
      const bool up = r >= half;
      const int64_t j = (int64_t)nt * half + (up ? r - half : r);
      if (a.layout == TSB_GU_SEPARATE) {
        w = static_cast<const uint8_t*>(up ? E.up : E.gate);
        s = static_cast<const uint8_t*>(up ? E.up_scales : E.gate_scales);
        row = j;
      } else {
        w = static_cast<const uint8_t*>(E.gate);
        s = static_cast<const uint8_t*>(E.gate_scales);
        row = a.layout == TSB_GU_INTERLEAVED ? 2 * j + (up ? 1 : 0) : (up ? a.I + j : j);
      }
    }
    uint4 o[kTileKB];
#pragma unroll
    for (int i = 0; i < kTileKB; ++i) {
      const int k0 = (kb0 + i) * kBK + c * 8;
      o[i] = make_uint4(0, 0, 0, 0);
      if (kb0 + i < a.KB && k0 < a.K) {
        float v[8];
        deq8<F>(w, s, row * a.K + k0, v);
        uint32_t h[4];
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const __half2 p = __halves2half2(__float2half_rn(v[2 * m]), __float2half_rn(v[2 * m + 1]));
          h[m] = *reinterpret_cast<const uint32_t*>(&p);
        }
        o[i] = make_uint4(h[0], h[1], h[2], h[3]);
      }
    }
#pragma unroll
    for (int i = 0; i < kTileKB; ++i)
      if (kb0 + i < a.KB)
        *reinterpret_cast<uint4*>(base + ((int64_t)(kb0 + i) * a.NT + r) * 128 + sw128_off(0, c ^ (r & 7))) = o[i];
  }
}

// ------------------------------------------------------------------ grouped GEMM
struct GemmArgs {
  const uint8_t* A;        // [mb][kb] tiles of 128 rows x 64 fp16
  int KB;                  // k-blocks
  const uint8_t* W;        // per expert: [nt][kb] tiles of NT rows x 64 fp16
  int64_t w_estride;       // bytes per expert
  int NT;                  // N tile (<= 256, multiple of 16)
  int ntiles;              // N tiles per expert
  const int* mb_expert;
  const int* total_mb;
  const int* row_src;
  const int8_t* row_shift;
  const TsbExpert* experts;
  int mode;                // 0: gate/up -> activation tiles, 1: down -> fp32 rows
  uint8_t* act;            // mode 0 output tiles
  int KBo;                 // mode 0: k-blocks of the activation tiles
  int act_kind;
  float limit, alpha;
  float* Y;                // mode 1 output [rows, H]
  int H;
  int* err;
  // in-kernel weight decode (MXFP4): source geometry
  int Kw;                  // weight columns (H for gate/up, I for down)
  int I;
  int layout;              // TSB_GU_*
};

// Bounded wait by a whole warp with a warp-uniform outcome: if any lane gave up,
// every lane does, so the warp never splits around a warp-wide instruction.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err) {
  const bool ok = mbar_wait(bar, parity, err);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ float pow2f(int e) {  // 2^e for |e| <= 126, exact
  return __uint_as_float((uint32_t)(127 + e) << 23);
}

// Power-of-two scale of a row's intermediate activations.  Rows whose largest
// |x| is below 2^-3 (x shift < -17) could give activations in or below the fp16
// subnormal range; they are stored multiplied by 2^-ash (ash < 0) and the down
// epilogue multiplies by 2^ash.  For small arguments clamp-SwiGLU is linear
// in the row scale ((u+1) g sigmoid(a g) ~ g / 2) and silu(g) u quadratic.
// Rows at or above that size are stored as they are (clamp-SwiGLU is bounded
// by (limit + 1) * limit).
__device__ __forceinline__ int act_shift(int xsh, int kind) {
  const int s = min(0, xsh + 17);
  return kind == TSB_ACT_SWIGLU_OAI ? s : max(-120, 2 * s);
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 p = __halves2half2(__float2half_rn(a), __float2half_rn(b));
  return *reinterpret_cast<const uint32_t*>(&p);
}

// Four MXFP4 bytes (8 e2m1 codes, low nibble first) times 2^e as eight fp16
// values, the fp16 rounding of tsb_dequant's exact fp32 value: e2m1 -> f16 is
// exact and, when 2^e is itself an fp16 number (-24 <= e <= 15), one correctly
// rounded f16 multiply gives that rounding; other exponents take the fp32 route.
struct MxScale {
  uint32_t s2;  // 2^e as f16x2 (fast route)
  int e;
  bool fast;
};
__device__ __forceinline__ MxScale mx_scale(uint32_t byte) {
  MxScale m;
  m.e = (int)byte - 127;
  m.fast = m.e >= -24 && m.e <= 15;
  const uint32_t sb = m.e >= -14 ? (uint32_t)(m.e + 15) << 10 : 1u << ((m.e + 24) & 31);
  m.s2 = sb | (sb << 16);
  return m;
}

__device__ __noinline__ uint4 mx_chunk_slow(uint32_t q4, int e) {
  uint32_t h[4];
  const int e1 = e / 2, e2 = e - e1;
  const float p1 = __uint_as_float((uint32_t)(e1 + 127) << 23), p2 = __uint_as_float((uint32_t)(e2 + 127) << 23);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t c = cvt_e2m1x2((q4 >> (8 * i)) & 0xFFu);
    const float lo = __fmul_rn(__fmul_rn(half_bits_to_f32((uint16_t)(c & 0xFFFF)), p1), p2);
    const float hi = __fmul_rn(__fmul_rn(half_bits_to_f32((uint16_t)(c >> 16)), p1), p2);
    const __half2 p = __halves2half2(__float2half_rn(lo), __float2half_rn(hi));
    h[i] = *reinterpret_cast<const uint32_t*>(&p);
  }
  return make_uint4(h[0], h[1], h[2], h[3]);
}

__device__ __forceinline__ uint4 mx_chunk(uint32_t q4, const MxScale& m) {
  if (!m.fast) return mx_chunk_slow(q4, m.e);
  uint32_t h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = h2mul(cvt_e2m1x2((q4 >> (8 * i)) & 0xFFu), m.s2);
  return make_uint4(h[0], h[1], h[2], h[3]);
}

// Source of B row r (0 <= r < NT) of tile column nt for the in-kernel decode:
// MXFP4 blocks and E8M0 scales of the weight row (gate/up tiles hold NT/2 gate
// rows then the same NT/2 up rows).
__device__ __forceinline__ void mx_row(const GemmArgs& g, const TsbExpert& E, int nt, int r, const uint8_t*& w,
                                       const uint8_t*& s) {
  const int64_t nblk = g.Kw / 32;
  int64_t row;
  const void* wm;
  const void* sm;
  if (g.mode == 1) {
    wm = E.down;
    sm = E.down_scales;
    row = (int64_t)nt * g.NT + r;
  } else {
    const int half = g.NT / 2;
    const bool up = r >= half;
    const int64_t j = (int64_t)nt * half + (up ? r - half : r);
    if (g.layout == TSB_GU_SEPARATE) {
      wm = up ? E.up : E.gate;
      sm = up ? E.up_scales : E.gate_scales;
      row = j;
    } else {
      wm = E.gate;
      sm = E.gate_scales;
      row = g.layout == TSB_GU_INTERLEAVED ? 2 * j + (up ? 1 : 0) : (up ? g.I + j : j);
    }
  }
  w = static_cast<const uint8_t*>(wm) + row * nblk * 16;
  s = static_cast<const uint8_t*>(sm) + row * nblk;
}

// Epilogue for one 128-row accumulator: thread m of the 128 reads its row of
// tensor memory at tl (lane quarter already added) for columns [c_lo, c_hi) of
// the gate/up halves (mode 0) or of the N tile (mode 1) and writes the
// activation tiles or the fp32 output rows of row block mb, N tile nt.
__device__ __forceinline__ void epilogue_rows(const GemmArgs& g, int mb, int nt, uint32_t tl, int m, bool setB) {
  const int R = mb * kBM + m;
  const int src = g.row_src[R];
  const TsbExpert& E = g.experts[g.mb_expert[mb]];
  const int xsh = src >= 0 ? g.row_shift[R] : 0;
  const int ash = act_shift(xsh, g.act_kind);
  if (g.mode == 0) {
    const int half = g.NT / 2, j0 = nt * half;
    const float sc = pow2f(xsh);
    const float asc = pow2f(-ash);
    const float* gb = E.gate_bias;
    const float* ub = E.up_bias;
    const int cs = (half / 2 + 7) / 8 * 8;
    for (int c = setB ? cs : 0; c < (setB ? half : cs); c += 8) {
      uint32_t gr[8], ur[8];
      tmem_ld8(tl + c, gr);
      tmem_ld8(tl + half + c, ur);
      tmem_ld_wait();
      if (src >= 0) {
        const int j = j0 + c;
        float a[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float gv = __fmul_rn(__uint_as_float(gr[i]), sc), uv = __fmul_rn(__uint_as_float(ur[i]), sc);
          if (gb) gv += gb[j + i];
          if (ub) uv += ub[j + i];
          a[i] = __fmul_rn(act_fn(g.act_kind, gv, uv, g.limit, g.alpha), asc);
        }
        const uint4 o = make_uint4(pack_h2(a[0], a[1]), pack_h2(a[2], a[3]), pack_h2(a[4], a[5]),
                                   pack_h2(a[6], a[7]));
        uint8_t* dst = g.act + ((size_t)mb * g.KBo + j / kBK) * kATile + sw128_off(m, (j % kBK) / 8);
        *reinterpret_cast<uint4*>(dst) = o;
      }
    }
  } else {
    const float* db = E.down_bias;
    const float dsc = pow2f(ash);
    const int cs = (g.NT / 2 + 7) / 8 * 8;
    for (int c = setB ? cs : 0; c < (setB ? g.NT : cs); c += 8) {
      uint32_t r[8];
      tmem_ld8(tl + c, r);
      tmem_ld_wait();
      if (src >= 0) {
        const int h = nt * g.NT + c;
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(__uint_as_float(r[i]), dsc) + (db ? db[h + i] : 0.f);
        float4* dst = reinterpret_cast<float4*>(g.Y + (size_t)R * g.H + h);
        dst[0] = make_float4(v[0], v[1], v[2], v[3]);
        dst[1] = make_float4(v[4], v[5], v[6], v[7]);
      }
    }
  }
}

// Persistent: CTA c takes tiles c, c + grid, ... of the (row block, N tile)
// grid, N fastest so that neighbouring CTAs share the token tile in L2.
// Warp 0 (one lane) streams A and W k-blocks into a kNS-stage ring; warp 1
// (one lane) issues 4 MMAs (K = 16 each) per k-block into one of two
// tensor-memory accumulators; warps 4-7 drain the other accumulator (warp
// 4+q reads lanes 32q..32q+31, i.e. rows 32q..32q+31 of the tile).
//
// BF = FMT_MXFP4: the B operand is decoded inside the kernel.  Warps 8-15 (one
// thread per B row) read each k-block's raw MXFP4 bytes and scales straight
// from the expert's weight stream (kPf k-blocks ahead, in registers), write
// the fp16 row into the stage's swizzled B tile and arrive on bfull; the MMA
// waits for both the A copy and the B decode of a stage.
constexpr int kNSFused = 3;                 // A/B stages of the in-kernel decode variant
constexpr int kRawItems = 4;                // k-blocks per raw copy (the decode loop assumes 4)
static_assert(kRawItems == 4, "scale-byte selection in the decode loop is written for 4 k-blocks per copy");
constexpr int kRawSlots = 2;
constexpr int kRawPitch = kRawItems * 32 + 16;   // 144 B: row pitch off the 128-byte bank period
constexpr int kRawSlot = 256 * kRawPitch;
constexpr size_t kGemmSmemFused = 1024 + (size_t)kNSFused * kStage + (size_t)kRawSlots * kRawSlot + 256;

template <int BF>
__global__ void __launch_bounds__(BF ? 640 : 384, 1) grouped_gemm_kernel(const GemmArgs g) {
  constexpr int EB = BF ? kEpiBFused : kEpiB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int NS = BF ? kNSFused : kNS;
  uint8_t* raw = smem + (size_t)NS * kStage;  // BF: kRawSlots x kRawSlot raw-weight ring
  uint64_t* bars = reinterpret_cast<uint64_t*>(raw + (BF ? kRawSlots * kRawSlot : 0));
  uint64_t* full = bars;
  uint64_t* empty = bars + NS;
  uint64_t* tfull = bars + 2 * NS;
  uint64_t* tempty = bars + 2 * NS + 2;
  uint64_t* fin = bars + 2 * NS + 4;
  uint64_t* bfull = bars + 2 * NS + 5;
  uint64_t* rfull = bars + 3 * NS + 5;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 3 * NS + 5 + kRawSlots);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);
    }
    mbar_init(fin, 1);
    if (BF) {
      for (int s = 0; s < NS; ++s) mbar_init(&bfull[s], 8);
      for (int s = 0; s < kRawSlots; ++s) mbar_init(&rfull[s], 8);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  const int total_tiles = *g.total_mb * g.ntiles;
  const uint32_t btile = (uint32_t)g.NT * 128u;

  if (warp == 0 && lane == 0) {
    uint32_t it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x) {
      const int mb = tile / g.ntiles, nt = tile % g.ntiles;
      const int e = g.mb_expert[mb];
      const uint8_t* a = g.A + (size_t)mb * g.KB * kATile;
      const uint8_t* b = BF ? nullptr : g.W + e * g.w_estride + (size_t)nt * g.KB * btile;
      for (int kb = 0; kb < g.KB; ++kb, ++it) {
        const int s = it % NS;
        if (!mbar_wait(&empty[s], ((it / NS) & 1) ^ 1, g.err)) { ok = false; break; }
        uint8_t* sa = smem + (size_t)s * kStage;
        mbar_arrive_expect_tx(&full[s], kATile + (BF ? 0u : btile));
        bulk_g2s(sa, a + (size_t)kb * kATile, kATile, &full[s]);
        if (!BF) bulk_g2s(sa + kATile, b + (size_t)kb * btile, btile, &full[s]);
      }
    }
  } else if (warp == 1 && lane == 0) {
    const uint32_t idesc = idesc_f16(kBM, g.NT, 0);
    uint32_t it = 0, tc = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x, ++tc) {
      const int buf = tc & 1;
      if (!mbar_wait(&tempty[buf], ((tc >> 1) & 1) ^ 1, g.err)) { ok = false; break; }
      tc_fence_after();
      const uint32_t d = tbase + (uint32_t)buf * 256u;
      for (int kb = 0; kb < g.KB; ++kb, ++it) {
        const int s = it % NS;
        if (!mbar_wait(&full[s], (it / NS) & 1, g.err)) { ok = false; break; }
        if (BF && !mbar_wait(&bfull[s], (it / NS) & 1, g.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + (size_t)s * kStage), sb = sa + kATile;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_f16(d, sw128_desc(sa + 32 * kk), sw128_desc(sb + 32 * kk), idesc, (kb | kk) != 0);
        umma_commit(&empty[s]);
      }
      if (ok) umma_commit(&tfull[buf]);
    }
    // Every MMA issued above completes before tensor memory is released.
    umma_commit(fin);
    mbar_wait(fin, 0, g.err);
  } else if ((warp >= 4 && warp < 8) || (warp >= EB && warp < EB + 4)) {
    const int q = warp & 3;
    const bool setB = warp >= EB;
    const int m = 32 * q + lane;
    uint32_t tc = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++tc) {
      const int buf = tc & 1;
      if (!warp_wait(&tfull[buf], (tc >> 1) & 1, g.err)) break;
      tc_fence_after();
      const int mb = tile / g.ntiles, nt = tile % g.ntiles;
      const uint32_t tl = tbase + (uint32_t)buf * 256u + ((uint32_t)(32 * q) << 16);
      epilogue_rows(g, mb, nt, tl, m, setB);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
  } else if (BF && warp >= 8 && warp < 16) {
    // Raw MXFP4 bytes of this thread's B row arrive kRawItems k-blocks at a
    // time (one bulk copy per row, kRawSlots groups ahead); E8M0 scales are
    // read with plain loads one group ahead.  Groups never straddle tiles.
    const int r = threadIdx.x - 256;
    const bool active = r < g.NT;
    const int mine = (int)blockIdx.x < total_tiles ? (total_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int gpt = (g.KB + kRawItems - 1) / kRawItems;  // groups per tile
    const int groups = mine * gpt;
    const int64_t rowbytes = (int64_t)(g.Kw / 32) * 16;
    const int wrows = max(0, min(32, g.NT - 32 * (warp - 8)));  // active rows of this warp
    int row_tile = -1;
    const uint8_t* row_w = nullptr;
    const uint8_t* row_s = nullptr;
    // Issue group q (raw copy into slot q % kRawSlots) and start loading its
    // scale bytes (combined only when the group is decoded).
    auto issue = [&](int q, uint32_t (&sb)[2 * kRawItems]) {
#pragma unroll
      for (int i = 0; i < 2 * kRawItems; ++i) sb[i] = 0;
      if (q >= groups) return;
      const int tile = blockIdx.x + (q / gpt) * gridDim.x;
      const int g0 = (q % gpt) * kRawItems;
      const int nk = min(kRawItems, g.KB - g0);
      const uint32_t bytes = (uint32_t)min((int64_t)nk * 32, rowbytes - (int64_t)g0 * 32);
      uint64_t* bar = &rfull[q % kRawSlots];
      if (lane == 0) mbar_arrive_expect_tx(bar, bytes * (uint32_t)wrows);
      __syncwarp();
      if (active) {
        if (tile != row_tile) {  // row pointers change once per tile
          const int mb = tile / g.ntiles, nt = tile % g.ntiles;
          mx_row(g, g.experts[g.mb_expert[mb]], nt, r, row_w, row_s);
          row_tile = tile;
        }
        const uint8_t* w = row_w;
        const uint8_t* sp = row_s;
        bulk_g2s(raw + (size_t)(q % kRawSlots) * kRawSlot + (size_t)r * kRawPitch, w + (size_t)g0 * 32, bytes, bar);
        const int nb = (int)(bytes / 16);  // 32-blocks present in this group
#pragma unroll
        for (int i = 0; i < 2 * kRawItems; ++i)
          if (i < nb) sb[i] = __ldg(sp + 2 * g0 + i);
      }
    };
    uint32_t scA[2 * kRawItems], scB[2 * kRawItems];
    issue(0, scA);
    issue(1, scB);
    uint32_t it = 0;
    bool ok = true;
    auto consume = [&](int q, const uint32_t (&sb)[2 * kRawItems]) {
      const int g0 = (q % gpt) * kRawItems;
      const int nk = min(kRawItems, g.KB - g0);
      const int slot = q % kRawSlots;
      if (!warp_wait(&rfull[slot], (q / kRawSlots) & 1, g.err)) { ok = false; return; }
      const uint8_t* rrow = raw + (size_t)slot * kRawSlot + (size_t)r * kRawPitch;
#pragma unroll 1
      for (int sub = 0; sub < nk; ++sub) {
        const int s = it % NS;
        if (!warp_wait(&empty[s], ((it / NS) & 1) ^ 1, g.err)) { ok = false; return; }
        if (active) {
          const uint4 lo = *reinterpret_cast<const uint4*>(rrow + 32 * sub);
          const uint4 hi = (g0 + sub) * kBK + 32 < g.Kw ? *reinterpret_cast<const uint4*>(rrow + 32 * sub + 16)
                                                        : make_uint4(0, 0, 0, 0);
          const uint32_t sbp = (sub & 2) ? ((sub & 1) ? (sb[6] | sb[7] << 8) : (sb[4] | sb[5] << 8))
                                         : ((sub & 1) ? (sb[2] | sb[3] << 8) : (sb[0] | sb[1] << 8));
          const MxScale m0 = mx_scale(sbp & 0xFF), m1 = mx_scale(sbp >> 8);
          uint8_t* brow = smem + (size_t)s * kStage + kATile + (size_t)r * 128;
          const uint32_t r7 = (uint32_t)(r & 7);
          const uint32_t q8[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
          for (int c = 0; c < 8; ++c)
            *reinterpret_cast<uint4*>(brow + ((c ^ r7) << 4)) = mx_chunk(q8[c], c < 4 ? m0 : m1);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bfull[s]);
        ++it;
      }
      __syncwarp();
    };
    for (int q = 0; ok && q < groups; q += 2) {
      consume(q, scA);
      if (!ok) break;
      issue(q + 2, scA);
      if (q + 1 >= groups) break;
      consume(q + 1, scB);
      if (!ok) break;
      issue(q + 3, scB);
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

// ---------------------------------------------------------------- CTA-pair GEMM
// The same grouped GEMM with two CTAs of a cluster sharing every MMA
// (tcgen05.mma.cta_group::2, M = 256): CTA r of the pair stages the 128 token
// rows of row block 2p + r and half of the N tile's weight rows (NT / 2 rows),
// so a stage is 16 KB + NT * 64 B and the ring is kNSPair deep.  Experts are
// padded to 256 rows, so a pair's two row blocks share one expert.
//   warp 0 (both CTAs)  stage loads into the CTA's own ring
//   warp 2 (CTA 1)      relays "stage s landed" to CTA 0's pfull[s]
//   warp 1 (CTA 0)      waits full[s] + pfull[s], issues the pair's MMAs and
//                       commits to both CTAs' empty[s] (and tfull[buf])
//   warps 4-11          epilogue of the CTA's own 128 rows; release the
//                       accumulator on CTA 0's tempty[buf] (8 + 8 arrivals)
// No cluster-multicast operations are used.
constexpr int kNSPair = 6;
constexpr int kPairStage = kATile + 128 * 128;  // token tile + up to 128 weight rows
constexpr size_t kPairSmem = 1024 + (size_t)kNSPair * kPairStage + 256;

__global__ void __launch_bounds__(kGemmThreads, 1) grouped_gemm_pair_kernel(const GemmArgs g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int NS = kNSPair;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)NS * kPairStage);
  uint64_t* full = bars;
  uint64_t* pfull = bars + NS;
  uint64_t* empty = bars + 2 * NS;
  uint64_t* tfull = bars + 3 * NS;
  uint64_t* tempty = bars + 3 * NS + 2;
  uint64_t* fin = bars + 3 * NS + 4;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 3 * NS + 5);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&pfull[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 16);
    }
    mbar_init(fin, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tslot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any remote arrival
  tc_fence_after();
  const uint32_t tbase = *tslot;
  const int total_tiles = (*g.total_mb / 2) * g.ntiles;
  const int half_rows = g.NT / 2;
  const uint32_t bhalf = (uint32_t)half_rows * 128u;
  const uint32_t btile = (uint32_t)g.NT * 128u;

  if (warp == 0 && lane == 0) {
    uint32_t it = 0;
    bool ok = true;
    for (int tile = pair; ok && tile < total_tiles; tile += npairs) {
      const int pp = tile / g.ntiles, nt = tile % g.ntiles;
      const int mb = 2 * pp + (int)rank;
      const int e = g.mb_expert[mb];
      const uint8_t* a = g.A + (size_t)mb * g.KB * kATile;
      const uint8_t* b = g.W + e * g.w_estride + (size_t)nt * g.KB * btile + rank * bhalf;
      for (int kb = 0; kb < g.KB; ++kb, ++it) {
        const int s = it % NS;
        if (!mbar_wait(&empty[s], ((it / NS) & 1) ^ 1, g.err)) { ok = false; break; }
        uint8_t* sa = smem + (size_t)s * kPairStage;
        mbar_arrive_expect_tx(&full[s], kATile + bhalf);
        bulk_g2s(sa, a + (size_t)kb * kATile, kATile, &full[s]);
        bulk_g2s(sa + kATile, b + (size_t)kb * btile, bhalf, &full[s]);
      }
    }
  } else if (warp == 2 && lane == 0 && rank == 1) {
    uint32_t it = 0;
    bool ok = true;
    for (int tile = pair; ok && tile < total_tiles; tile += npairs) {
      for (int kb = 0; kb < g.KB; ++kb, ++it) {
        const int s = it % NS;
        if (!mbar_wait(&full[s], (it / NS) & 1, g.err)) { ok = false; break; }
        mbar_arrive_cluster_relaxed(mapa_shared(smem_u32(&pfull[s]), 0));
      }
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    const uint32_t idesc = idesc_f16(2 * kBM, g.NT, 0);
    uint32_t it = 0, tc = 0;
    bool ok = true;
    for (int tile = pair; ok && tile < total_tiles; tile += npairs, ++tc) {
      const int buf = tc & 1;
      if (!mbar_wait_cluster(&tempty[buf], ((tc >> 1) & 1) ^ 1, g.err)) { ok = false; break; }
      tc_fence_after();
      const uint32_t d = tbase + (uint32_t)buf * 256u;
      for (int kb = 0; kb < g.KB; ++kb, ++it) {
        const int s = it % NS;
        if (!mbar_wait(&full[s], (it / NS) & 1, g.err)) { ok = false; break; }
        if (!mbar_wait_cluster_relaxed(&pfull[s], (it / NS) & 1, g.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + (size_t)s * kPairStage), sb = sa + kATile;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_f16_pair(d, sw128_desc(sa + 32 * kk), sw128_desc(sb + 32 * kk), idesc, (kb | kk) != 0);
        umma_commit_pair(smem_u32(&empty[s]));
        umma_commit_pair(mapa_shared(smem_u32(&empty[s]), 1));
      }
      if (ok) {
        umma_commit_pair(smem_u32(&tfull[buf]));
        umma_commit_pair(mapa_shared(smem_u32(&tfull[buf]), 1));
      }
    }
    // Every MMA of the pair completes before either CTA releases tensor memory.
    umma_commit_pair(smem_u32(fin));
    umma_commit_pair(mapa_shared(smem_u32(fin), 1));
  } else if ((warp >= 4 && warp < 8) || (warp >= kEpiB && warp < kEpiB + 4)) {
    const int q = warp & 3;
    const bool setB = warp >= kEpiB;
    const int m = 32 * q + lane;
    const uint32_t tempty0 = mapa_shared(smem_u32(&tempty[0]), 0);
    uint32_t tc = 0;
    for (int tile = pair; tile < total_tiles; tile += npairs, ++tc) {
      const int buf = tc & 1;
      if (!warp_wait(&tfull[buf], (tc >> 1) & 1, g.err)) break;
      tc_fence_after();
      const int pp = tile / g.ntiles, nt = tile % g.ntiles;
      const int mb = 2 * pp + (int)rank;
      const uint32_t tl = tbase + (uint32_t)buf * 256u + ((uint32_t)(32 * q) << 16);
      epilogue_rows(g, mb, nt, tl, m, setB);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty0 + (uint32_t)buf * 8u);
    }
  }
  // Both CTAs wait for the pair's last MMAs (fin) before leaving; the cluster
  // barrier keeps either CTA from freeing tensor memory while the other runs.
  if (threadIdx.x == 32) mbar_wait(fin, 0, g.err);
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tbase, kTmemCols);
  }
}

// out[t] = sum_j w[t,j] * Y[row_of[t,j]], j ascending (fmaf chain from 0, the
// decode combine's order); rows of invalid experts are skipped.
__global__ void __launch_bounds__(256) combine_kernel(const float* __restrict__ Y, int H,
                                                      const int* __restrict__ row_of, const float* __restrict__ wts,
                                                      int top_k, void* __restrict__ out, int out_f32) {
  const int t = blockIdx.x;
  for (int h4 = threadIdx.x; h4 < H / 4; h4 += blockDim.x) {
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < top_k; ++j) {
      const int r = row_of[t * top_k + j];
      if (r < 0) continue;
      const float w = wts[t * top_k + j];
      const float4 y = reinterpret_cast<const float4*>(Y + (size_t)r * H)[h4];
      o.x = fmaf(w, y.x, o.x);
      o.y = fmaf(w, y.y, o.y);
      o.z = fmaf(w, y.z, o.z);
      o.w = fmaf(w, y.w, o.w);
    }
    if (out_f32) {
      reinterpret_cast<float4*>(static_cast<float*>(out) + (size_t)t * H)[h4] = o;
    } else {
      const uint32_t lo = f32_to_bf16_bits(o.x) | ((uint32_t)f32_to_bf16_bits(o.y) << 16);
      const uint32_t hi = f32_to_bf16_bits(o.z) | ((uint32_t)f32_to_bf16_bits(o.w) << 16);
      reinterpret_cast<uint2*>(static_cast<uint16_t*>(out) + (size_t)t * H)[h4] = make_uint2(lo, hi);
    }
  }
}

// ------------------------------------------------------------------ router (T tokens)
// One 16-warp CTA per token: x staged once in shared memory, warp w computes
// logits[e] = bf16(x . W[e] + b[e]) for experts w, w + 16, ... two at a time
// with all of a lane's loads of both rows in flight (a token's logits cost a
// few memory round trips, not one per expert); then warp 0 takes the top-k
// (ties -> lower id, NaN lowest) and a softmax over the k selected logits, the
// decode router's rule (tinyserve/_model_hooks.py:466-473).
constexpr int kRouteThreads = 512;

__global__ void __launch_bounds__(kRouteThreads, 2) prefill_router_kernel(const uint16_t* __restrict__ x,
                                                                       const uint16_t* __restrict__ W,
                                                                       const float* __restrict__ b, int H, int E,
                                                                       int T, int top_k, int32_t* __restrict__ ids,
                                                                       float* __restrict__ wts) {
  extern __shared__ float slog[];  // [E] logits, then x as uint4 [H / 8]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x;
  float* lg = slog;
  uint4* xs = reinterpret_cast<uint4*>(slog + ((E + 3) & ~3));
  const int n8 = H / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)t * H);
  for (int c = threadIdx.x; c < n8; c += kRouteThreads) xs[c] = xr[c];
  __syncthreads();
  auto dot8 = [](uint4 a, uint4 w, float acc) {
    const uint32_t av[4] = {a.x, a.y, a.z, a.w}, wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      acc = fmaf(__uint_as_float(av[q] << 16), __uint_as_float(wv[q] << 16), acc);
      acc = fmaf(__uint_as_float(av[q] & 0xFFFF0000u), __uint_as_float(wv[q] & 0xFFFF0000u), acc);
    }
    return acc;
  };
  for (int e0 = warp; e0 < E; e0 += 2 * (kRouteThreads / 32)) {
    const int e1 = e0 + kRouteThreads / 32;
    const uint4* w0 = reinterpret_cast<const uint4*>(W + (int64_t)e0 * H);
    const uint4* w1 = reinterpret_cast<const uint4*>(W + (int64_t)(e1 < E ? e1 : e0) * H);
    float a0 = 0.f, a1 = 0.f;
    for (int c0 = 0; c0 < n8; c0 += 4 * 32) {
      uint4 r0[4], r1[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = c0 + u * 32 + lane;
        r0[u] = c < n8 ? __ldg(w0 + c) : make_uint4(0, 0, 0, 0);
        r1[u] = c < n8 ? __ldg(w1 + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < n8) {
          const uint4 xv = xs[c];
          a0 = dot8(xv, r0[u], a0);
          a1 = dot8(xv, r1[u], a1);
        }
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      a0 += __shfl_xor_sync(0xffffffffu, a0, o);
      a1 += __shfl_xor_sync(0xffffffffu, a1, o);
    }
    if (lane == 0) {
      if (b) a0 += b[e0];
      lg[e0] = bf16_bits_to_f32(f32_to_bf16_bits(a0));
      if (e1 < E) {
        if (b) a1 += b[e1];
        lg[e1] = bf16_bits_to_f32(f32_to_bf16_bits(a1));
      }
    }
  }
  __syncthreads();
  if (warp != 0) return;
  __syncwarp();
  float sel[8];
  int sid[8];
  uint32_t taken = 0;
  for (int k = 0; k < top_k; ++k) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int j = 0; lane + 32 * j < E; ++j) {
      if ((taken >> j) & 1u) continue;
      const int ee = lane + 32 * j;
      float v = lg[ee];
      if (v != v) v = -INFINITY;
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
      ids[(int64_t)t * top_k + k] = sid[k];
      wts[(int64_t)t * top_k + k] = ex[k] / den;
    }
  }
}

// ------------------------------------------------------------------ host side
// Largest N tile <= 256 (multiple of 16) dividing `rows`; for the gate/up
// projection the tile holds `pair` = 2 halves (gate, up) of NT/2 features each,
// and NT/2 must divide I.
static int pick_nt(int rows, bool pair) {
  for (int nt = 256; nt >= 16; nt -= 16) {
    if (pair ? (rows % (nt / 2) == 0 && (nt / 2) % 8 == 0) : rows % nt == 0) return nt;
  }
  return 0;
}

// Where the MXFP4 weights are decoded.  Decoding inside the GEMM repeats the
// decode for every 128-row block of an expert; decoding once into fp16 tiles
// costs a write and re-read of the tiles through HBM.  With at most ~2 row
// blocks per expert on average (T*k <= 256*E: batched decode, short prompts)
// the in-GEMM decode wins; above that the tiles do.  TSB_PREFILL_FUSED=0/1
// forces one or the other.
static bool fused_mxfp4(const TsbMoeSpec& sp, int T) {
  static const int force = [] {
    const char* v = getenv("TSB_PREFILL_FUSED");
    return v ? (v[0] == '1' ? 1 : 0) : -1;
  }();
  if (force >= 0) return force == 1;
  return (int64_t)T * sp.top_k <= (int64_t)256 * sp.n_experts;
}

// Two-CTA GEMMs on the tiled path, opt-in with TSB_PREFILL_PAIR=1.  Per row
// they run about 5% faster than the one-CTA kernel, but experts padded to 256
// rows add 8% rows under Zipf routing of 4096 tokens over 32 experts, so the
// one-CTA kernel stays the default.
static bool pair_gemm() {
  static const bool on = [] {
    const char* v = getenv("TSB_PREFILL_PAIR");
    return v && v[0] == '1';
  }();
  return on;
}

PrefillLayout prefill_layout(const TsbMoeSpec& sp, int T) {
  PrefillLayout L{};
  auto al = [](size_t v) { return (v + 1023) & ~size_t(1023); };
  const int64_t n = (int64_t)T * sp.top_k;
  const bool fgu = sp.fmt_gate_up == FMT_MXFP4 && fused_mxfp4(sp, T);
  const bool fdn = sp.fmt_down == FMT_MXFP4 && fused_mxfp4(sp, T);
  L.pair = !fgu && !fdn && pair_gemm();
  L.pad = L.pair ? 2 * kBM : kBM;
  L.mb_max = (int)((n + (int64_t)sp.n_experts * (L.pad - 1)) / L.pad) * (L.pad / kBM);
  L.rows_max = (int64_t)L.mb_max * kBM;
  L.kbh = (sp.hidden + kBK - 1) / kBK;
  L.kbi = (sp.inter + kBK - 1) / kBK;
  L.nt_gu = pick_nt(sp.inter, true);
  L.nt_dn = pick_nt(sp.hidden, false);
  size_t o = 0;
  L.err = o;          // int32 error word
  L.total_mb = 4;     // int32
  o = 256;
  L.counts = o;   o = al(o + 4 * (size_t)sp.n_experts);
  L.ccount = o;   o = al(o + 4 * (size_t)sp.n_experts * (size_t)((n + kRouteChunk - 1) / kRouteChunk));
  L.mb_expert = o; o = al(o + 4 * (size_t)L.mb_max);
  L.row_of = o;   o = al(o + 4 * (size_t)n);
  L.row_src = o;  o = al(o + 4 * (size_t)L.rows_max);
  L.row_shift = o; o = al(o + (size_t)L.rows_max);
  L.xp = o;       o = al(o + (size_t)L.mb_max * L.kbh * kATile);
  L.act = o;      o = al(o + (size_t)L.mb_max * L.kbi * kATile);
  L.y = o;        o = al(o + 4 * (size_t)L.rows_max * sp.hidden);
  L.fused_gu = fgu;
  L.fused_dn = fdn;
  L.wgu_estride = fgu ? 0 : (int64_t)2 * sp.inter * L.kbh * 128;
  L.wdn_estride = fdn ? 0 : (int64_t)sp.hidden * L.kbi * 128;
  L.wgu = o;      o = al(o + (size_t)sp.n_experts * L.wgu_estride);
  L.wdn = o;      o = al(o + (size_t)sp.n_experts * L.wdn_estride);
  L.total = o;
  return L;
}

static int num_sms() {
  static int n = [] {
    int dev = 0, v = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v;
  }();
  return n;
}

template <int F>
static void launch_tile_weights(const TileWArgs& a, int E, cudaStream_t st) {
  tile_weights_kernel<F><<<dim3((a.N / a.NT) * ((a.KB + kTileKB - 1) / kTileKB), E), 256, 0, st>>>(a);
}

static int tile_weights(int fmt, const TileWArgs& a, int E, cudaStream_t st) {
  switch (fmt) {
    case FMT_Q8_0: launch_tile_weights<FMT_Q8_0>(a, E, st); break;
    case FMT_Q4_K: launch_tile_weights<FMT_Q4_K>(a, E, st); break;
    case FMT_Q5_K: launch_tile_weights<FMT_Q5_K>(a, E, st); break;
    case FMT_Q6_K: launch_tile_weights<FMT_Q6_K>(a, E, st); break;
    case FMT_MXFP4: launch_tile_weights<FMT_MXFP4>(a, E, st); break;
    default: return set_error(TSB_ERR_UNSUPPORTED, "unsupported format");
  }
  return TSB_OK;
}

template <int BF>
static int launch_gemm(const GemmArgs& g, int tiles_max, cudaStream_t st) {
  static bool attr = [] {
    return cudaFuncSetAttribute(grouped_gemm_kernel<BF>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)(BF ? kGemmSmemFused : kGemmSmem)) == cudaSuccess;
  }();
  if (!attr) return set_error(TSB_ERR_CUDA, "cannot enable the grouped GEMM's shared memory");
  const int grid = std::max(1, std::min(tiles_max, num_sms()));
  grouped_gemm_kernel<BF><<<grid, BF ? 640 : kGemmThreads, BF ? kGemmSmemFused : kGemmSmem, st>>>(g);
  return TSB_OK;
}

static int launch_gemm_pair(const GemmArgs& g, int tiles_max, cudaStream_t st) {
  static bool attr = [] {
    return cudaFuncSetAttribute(grouped_gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)kPairSmem) == cudaSuccess;
  }();
  if (!attr) return set_error(TSB_ERR_CUDA, "cannot enable the pair GEMM's shared memory");
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = kPairSmem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  // The kernel is persistent: launch only as many pairs as can be resident at
  // once (clusters are placed inside one GPC, so this can be below SMs / 2).
  static const int resident = [&] {
    cudaLaunchConfig_t q = cfg;
    q.gridDim = dim3(num_sms());
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, grouped_gemm_pair_kernel, &q) != cudaSuccess || n < 1) n = num_sms() / 2;
    return n;
  }();
  const int pairs = std::max(1, std::min(tiles_max / 2, resident));
  cfg.gridDim = dim3(2 * pairs);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, grouped_gemm_pair_kernel, g);
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  return TSB_OK;
}

int launch_route(const TsbMoeSpec& sp, const void* x, int T, const void* rw, const float* rb, int32_t* ids,
                 float* wts, cudaStream_t st) {
  const size_t sm = sizeof(float) * (size_t)((sp.n_experts + 3) & ~3) + 2 * (size_t)sp.hidden;
  if (sm > 48 * 1024) cudaFuncSetAttribute(prefill_router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  prefill_router_kernel<<<T, kRouteThreads, sm, st>>>(static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(rw),
                                                       rb, sp.hidden, sp.n_experts, T, sp.top_k, ids, wts);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  return TSB_OK;
}

int launch_moe_prefill(const TsbMoeSpec& sp, const TsbExpert* ex, const void* x, int T, const void* rw,
                       const float* rb, int32_t* ids, float* wts, void* out, char* ws, const PrefillLayout& L,
                       cudaStream_t st) {
  const int E = sp.n_experts, k = sp.top_k, n = T * k;
  int32_t* err = reinterpret_cast<int32_t*>(ws + L.err);
  int* total_mb = reinterpret_cast<int*>(ws + L.total_mb);
  int* counts = reinterpret_cast<int*>(ws + L.counts);
  int* mb_expert = reinterpret_cast<int*>(ws + L.mb_expert);
  int* row_of = reinterpret_cast<int*>(ws + L.row_of);
  int* row_src = reinterpret_cast<int*>(ws + L.row_src);
  int8_t* row_shift = reinterpret_cast<int8_t*>(ws + L.row_shift);
  uint8_t* xp = reinterpret_cast<uint8_t*>(ws + L.xp);
  uint8_t* act = reinterpret_cast<uint8_t*>(ws + L.act);
  float* Y = reinterpret_cast<float*>(ws + L.y);
  uint8_t* wgu = reinterpret_cast<uint8_t*>(ws + L.wgu);
  uint8_t* wdn = reinterpret_cast<uint8_t*>(ws + L.wdn);

  if (rw) {
    const int rc = launch_route(sp, x, T, rw, rb, ids, wts, st);
    if (rc) return rc;
  }
  int* ccount = reinterpret_cast<int*>(ws + L.ccount);
  const int nchunks = (n + kRouteChunk - 1) / kRouteChunk;
  route_chunk_count<<<nchunks, 256, 4 * E, st>>>(ids, n, E, ccount, row_of, err);
  route_scan<<<1, 1024, 0, st>>>(nchunks, E, ccount, counts, row_src, mb_expert, total_mb, L.pad);
  route_chunk_place<<<nchunks, 32, 4 * E, st>>>(ids, n, k, E, ccount, row_of, row_src);
  gather_rows_kernel<<<(int)((L.rows_max + 7) / 8), 256, 0, st>>>(static_cast<const uint16_t*>(x), sp.hidden, L.kbh,
                                                                  row_src, total_mb, xp, row_shift);
  if (sp.inter % kBK) {
    // K padding of the activation tiles must read as zero.
    cudaMemsetAsync(act, 0, (size_t)L.mb_max * L.kbi * kATile, st);
  }
  TileWArgs tg{ex, counts, 0, sp.gate_up_layout, sp.inter, 2 * sp.inter, sp.hidden, L.kbh, L.nt_gu, wgu,
               L.wgu_estride};
  const bool fgu = L.fused_gu, fdn = L.fused_dn;
  int rc = fgu ? TSB_OK : tile_weights(sp.fmt_gate_up, tg, E, st);
  if (rc) return rc;
  TileWArgs td{ex, counts, 1, sp.gate_up_layout, sp.inter, sp.hidden, sp.inter, L.kbi, L.nt_dn, wdn, L.wdn_estride};
  rc = fdn ? TSB_OK : tile_weights(sp.fmt_down, td, E, st);
  if (rc) return rc;

  GemmArgs g{};
  g.A = xp;
  g.KB = L.kbh;
  g.W = wgu;
  g.w_estride = L.wgu_estride;
  g.NT = L.nt_gu;
  g.ntiles = 2 * sp.inter / L.nt_gu;
  g.mb_expert = mb_expert;
  g.total_mb = total_mb;
  g.row_src = row_src;
  g.row_shift = row_shift;
  g.experts = ex;
  g.mode = 0;
  g.act = act;
  g.KBo = L.kbi;
  g.act_kind = sp.activation;
  g.limit = sp.limit;
  g.alpha = sp.alpha;
  g.err = err;
  g.Kw = sp.hidden;
  g.I = sp.inter;
  g.layout = sp.gate_up_layout;
  rc = fgu ? launch_gemm<FMT_MXFP4>(g, L.mb_max * g.ntiles, st)
      : L.pair ? launch_gemm_pair(g, L.mb_max * g.ntiles, st)
               : launch_gemm<0>(g, L.mb_max * g.ntiles, st);
  if (rc) return rc;
  GemmArgs d = g;
  d.A = act;
  d.KB = L.kbi;
  d.W = wdn;
  d.w_estride = L.wdn_estride;
  d.NT = L.nt_dn;
  d.ntiles = sp.hidden / L.nt_dn;
  d.mode = 1;
  d.Y = Y;
  d.H = sp.hidden;
  d.Kw = sp.inter;
  rc = fdn ? launch_gemm<FMT_MXFP4>(d, L.mb_max * d.ntiles, st)
      : L.pair ? launch_gemm_pair(d, L.mb_max * d.ntiles, st)
               : launch_gemm<0>(d, L.mb_max * d.ntiles, st);
  if (rc) return rc;
  combine_kernel<<<T, 256, 0, st>>>(Y, sp.hidden, row_of, wts, k, out, sp.out_f32 != 0);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  return TSB_OK;
}

}  // namespace tsb
