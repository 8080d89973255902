// Batch-1 MoE decode on a decode-packed copy of 4-bit K-quant experts.
//
// The generic decode engine reads the GGUF block stream as stored
// (tinyserve/gguf_dequant_torch.py:180-205): with K % 256 != 0 rows start at
// different superblock phases and every 32-element step rebuilds its scale
// from the 12-byte packed scales, which costs ~120 instructions per 512
// weights.  Here the experts are repacked once (tsb_moe_pack) into the order
// the tensor-core fragments consume, with each (row, 32-element sub-block)'s
// fold coefficients already formed, so the inner loop is a shared-memory
// read, a handful of bit operations, four MMAs and eight FMAs per 1024 weights.
//
// Packed unit: one 16-row block x one 64-element k-block = 768 bytes
//   [0, 512)    codes: lane L (g = L/4, t = L%4) owns 16 bytes = 32 codes in
//               mma.m16n8k16 A-fragment order (see pack_unit_kernel)
//   [512, 768)  fold coefficients: for sub-block sb (0, 1) and row pair g,
//               float4 (s_g, s_g+8, o_g, o_g+8) at 512 + 128 sb + 16 g
// A row's contribution from a sub-block is s * sum(q*x) - dmin*m * sum(x);
// the codes of sub-block 0 decode to 1024+q and those of sub-block 1 to 64+q
// (one LOP3 per f16 pair: 0x6400|q and 0x5400|q<<4), so the MMA yields
// C = sum(q*x) + off * X and the fold is s*C - (off*s + dmin*m)*X with
// o = off*s + dmin*m stored.  s = d*sc and dmin*m are the products the
// reference decoder forms (gguf_dequant_torch.py:195-203), in fp32.
//
// Gate/up row blocks hold 8 gate rows then the 8 up rows of the same outputs,
// so the SwiGLU pair of output j sits in one lane's accumulators (rows g and
// g+8 of the fragment).  Down row blocks are 16 consecutive rows.
//
// Work: warp tasks (slot, row block, k-range); each task writes its 16 fp32
// partial sums, and the last task of a row block (atomic counter, reset after
// use) reduces the partials in fixed order and runs the epilogue, so results
// do not depend on scheduling.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "../../include/tsb_moe.h"
#include "moe_math.cuh"
#include "qformats.cuh"
#include "tsb_common.cuh"
#include "tsb_internal.h"

namespace tsb {

constexpr int kPkThreads = 512;
constexpr int kPkWarps = kPkThreads / 32;
constexpr int kUnitBytes = 768;
constexpr int kMaxSplit = 16;

bool packable(const TsbMoeSpec& sp) {
  return sp.fmt_gate_up == FMT_Q4_K && sp.fmt_down == FMT_Q4_K && sp.hidden % 64 == 0 && sp.inter % 64 == 0 &&
         sp.hidden > 0 && sp.inter > 0 && sp.n_experts >= 1 && sp.top_k >= 1 && sp.top_k <= 8;
}

PackGeom pack_geom(const TsbMoeSpec& sp) {
  PackGeom G{};
  G.rgu = (sp.inter + 7) / 8;
  G.rdn = (sp.hidden + 15) / 16;
  G.kbh = sp.hidden / 64;
  G.kbi = sp.inter / 64;
  G.gu_off = 0;
  G.dn_off = (int64_t)G.rgu * G.kbh * kUnitBytes;
  G.expert_bytes = (G.dn_off + (int64_t)G.rdn * G.kbi * kUnitBytes + 255) & ~int64_t(255);
  return G;
}

// ------------------------------------------------------------------ packing
// Q4_K element f of a flat stream: code, and the sub-block's (d*sc, dmin*m).
__device__ __forceinline__ int q4k_code(const uint8_t* w, int64_t f) {
  const uint8_t* b = w + (f >> 8) * 144;
  const int i = (int)(f & 255), j = i >> 5, l = i & 31;
  return (b[16 + 32 * (j >> 1) + l] >> (4 * (j & 1))) & 15;
}
__device__ __forceinline__ void q4k_coef(const uint8_t* w, int64_t f, float& s, float& o) {
  const uint8_t* b = w + (f >> 8) * 144;
  const int j = (int)((f & 255) >> 5);
  const float d = half_bits_to_f32((uint16_t)(b[0] | (b[1] << 8)));
  const float dmin = half_bits_to_f32((uint16_t)(b[2] | (b[3] << 8)));
  int sc, m;
  kq_scale_min(b + 4, j, sc, m);
  s = __fmul_rn(d, (float)sc);
  o = __fmul_rn(dmin, (float)m);
}

struct PackArgs {
  const TsbExpert* experts;
  uint8_t* packed;
  PackGeom G;
  int H, I, layout;
  int64_t units_gu, units_per_expert;
};

// Source (stream, row) of packed row m of a row block; null when past the end.
__device__ __forceinline__ const uint8_t* src_row(const PackArgs& a, const TsbExpert& E, bool down, int rb, int m,
                                                  int64_t& row) {
  if (down) {
    row = 16 * rb + m;
    return row < a.H ? static_cast<const uint8_t*>(E.down) : nullptr;
  }
  const int j = 8 * rb + (m & 7);
  if (j >= a.I) return nullptr;
  const bool up = m >= 8;
  if (a.layout == TSB_GU_INTERLEAVED) {
    row = 2 * (int64_t)j + (up ? 1 : 0);
    return static_cast<const uint8_t*>(E.gate);
  }
  if (a.layout == TSB_GU_CHUNKED) {
    row = (up ? a.I : 0) + (int64_t)j;
    return static_cast<const uint8_t*>(E.gate);
  }
  row = j;
  return static_cast<const uint8_t*>(up ? E.up : E.gate);
}

// One warp per packed unit.  Lane L's 32 codes: for family fam (0: sub-block
// 0, decoded as 1024+q; 1: sub-block 1, decoded as 64+q), fragment register
// m (0..7) and half h, the code of row g + 8*(r&1), column
// 16*(2 fam + m/4) + 2t + 8*(r/2) + h (r = m%4) sits in word m/2 at bit
// 8*(m%2) + 16h + 4 fam.
__global__ void __launch_bounds__(256) pack_unit_kernel(const PackArgs a, int64_t nunits) {
  const int64_t unit = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (unit >= nunits) return;
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int64_t e = unit / a.units_per_expert;
  int64_t r = unit % a.units_per_expert;
  const bool down = r >= a.units_gu;
  if (down) r -= a.units_gu;
  const int KB = down ? a.G.kbi : a.G.kbh;
  const int rb = (int)(r / KB), kb = (int)(r % KB);
  const int K = down ? a.I : a.H;
  const TsbExpert E = a.experts[e];
  uint8_t* dst = a.packed + e * a.G.expert_bytes + (down ? a.G.dn_off : a.G.gu_off) + r * kUnitBytes;

  uint32_t word[4] = {0, 0, 0, 0};
  int64_t row_lo = 0, row_hi = 0;
  const uint8_t* w_lo = src_row(a, E, down, rb, g, row_lo);
  const uint8_t* w_hi = src_row(a, E, down, rb, g + 8, row_hi);
#pragma unroll
  for (int fam = 0; fam < 2; ++fam)
#pragma unroll
    for (int m = 0; m < 8; ++m)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int rr = m & 3;
        const int col = 16 * (2 * fam + (m >> 2)) + 2 * t + 8 * (rr >> 1) + h;
        const uint8_t* w = (rr & 1) ? w_hi : w_lo;
        const int64_t row = (rr & 1) ? row_hi : row_lo;
        const int q = w ? q4k_code(w, row * K + 64 * (int64_t)kb + col) : 0;
        word[m >> 1] |= (uint32_t)q << (8 * (m & 1) + 16 * h + 4 * fam);
      }
  *reinterpret_cast<uint4*>(dst + 16 * lane) = make_uint4(word[0], word[1], word[2], word[3]);

  if (lane < 16) {
    const int sb = lane >> 3, gg = lane & 7;
    float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int hi = 0; hi < 2; ++hi) {
      int64_t row = 0;
      const uint8_t* w = src_row(a, E, down, rb, gg + 8 * hi, row);
      if (!w) continue;
      float s, o;
      q4k_coef(w, row * K + 64 * (int64_t)kb + 32 * sb, s, o);
      c[hi] = s;
      c[2 + hi] = fmaf(sb ? 64.f : 1024.f, s, o);
    }
    *reinterpret_cast<float4*>(dst + 512 + 128 * sb + 16 * gg) = make_float4(c[0], c[1], c[2], c[3]);
  }
}

int launch_pack(const TsbMoeSpec& sp, const TsbExpert* experts, void* packed, cudaStream_t st) {
  PackArgs a{};
  a.experts = experts;
  a.packed = static_cast<uint8_t*>(packed);
  a.G = pack_geom(sp);
  a.H = sp.hidden;
  a.I = sp.inter;
  a.layout = sp.gate_up_layout;
  a.units_gu = (int64_t)a.G.rgu * a.G.kbh;
  a.units_per_expert = a.units_gu + (int64_t)a.G.rdn * a.G.kbi;
  const int64_t n = a.units_per_expert * sp.n_experts;
  pack_unit_kernel<<<(unsigned)((n + 7) / 8), 256, 0, st>>>(a, n);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  return TSB_OK;
}

// ------------------------------------------------------------------ decode
struct PkArgs {
  const uint8_t* packed;
  int64_t expert_bytes, sec_off;
  int R, KB, S, nkb, ntasks;
  const int32_t* ids;
  const float* wts;
  const TsbExpert* experts;
  int n_experts, top_k;
  int* err;
  const void* x;      // mode 0: bf16 [H]; mode 1: fp32 [top_k, I]
  int nv;             // staged vectors: 1 (gate/up) or top_k (down)
  float* part;        // [ntasks, 16]
  unsigned* cnt;      // per output row block, zero between calls
  int mode, I, H, act;
  float limit, alpha;
  float* act_out;     // mode 0: fp32 [top_k, I]
  uint16_t* out;      // mode 1: bf16 [H]
  // routing inside the gate/up launch (null: ids and wts are inputs)
  const uint16_t* router_w;  // bf16 [E, H]
  const float* router_b;     // fp32 [E] or null
  // 0x64006400 and 0x54005400 (f16x2 1024 and 64), passed as arguments so the
  // compiler keeps them in registers: each code decode is then one LOP3 with
  // the mask as its immediate, (w & mask) | magic.
  uint32_t magic1024, magic64;
};

// Each warp streams its units through a private ring of kSlots slots of
// kSlotUnits units (one cp.async.bulk copy per slot, completing on the slot's
// mbarrier): up to kSlots * kSlotUnits * 768 bytes in flight per warp.  The
// ring is refilled across the warp's tasks, so it does not drain between them.
constexpr int kSlotUnits = 4, kSlots = 2;
constexpr int kSlotBytes = kSlotUnits * kUnitBytes;

// Slot waits spin on mbarrier.test_wait (no suspend): a warp waits for its
// own next slot every two units, so a sleeping wait's wake-up delay would sit
// on the critical path.  Bounded: after kSpinPolls polls (seconds) it records
// kDevWaitTimeout and returns false.
constexpr uint32_t kSpinPolls = 1u << 26;
__device__ __forceinline__ bool pk_warp_wait(uint64_t* bar, uint32_t parity, int* err) {
  bool ok = false;
  for (uint32_t i = 0; i < kSpinPolls && !ok; ++i) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(r)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    ok = r != 0;
  }
  if (!ok && err) atomicExch(err, kDevWaitTimeout);
  return __all_sync(0xffffffffu, ok);
}
// D = A * B with a zero accumulator input (no per-use register clearing).
__device__ __forceinline__ void mma_f16_z(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
}

// One 768-byte unit: decode the 32 codes of this lane, four MMAs against the
// staged vector, fold into the two row accumulators.
__device__ __forceinline__ void unit_fma(const uint8_t* u, int oq, int oc, const uint8_t* xb, const float2 xs,
                                         uint32_t M1, uint32_t M2, float& acc_lo, float& acc_hi) {
  const uint4 q = *reinterpret_cast<const uint4*>(u + oq);
  const float4 c0 = *reinterpret_cast<const float4*>(u + oc);
  const float4 c1 = *reinterpret_cast<const float4*>(u + oc + 128);
  const uint4 b01 = *reinterpret_cast<const uint4*>(xb);
  const uint4 b23 = *reinterpret_cast<const uint4*>(xb + 16);
  uint32_t l0[4], l1[4], h0[4], h1[4];
  {
    const uint32_t w0 = q.x, w1 = q.y, w2 = q.z, w3 = q.w;
    const uint32_t v0 = w0 >> 8, v1 = w1 >> 8, v2 = w2 >> 8, v3 = w3 >> 8;
    l0[0] = (w0 & 0x000F000Fu) | M1;
    l0[1] = (v0 & 0x000F000Fu) | M1;
    l0[2] = (w1 & 0x000F000Fu) | M1;
    l0[3] = (v1 & 0x000F000Fu) | M1;
    l1[0] = (w2 & 0x000F000Fu) | M1;
    l1[1] = (v2 & 0x000F000Fu) | M1;
    l1[2] = (w3 & 0x000F000Fu) | M1;
    l1[3] = (v3 & 0x000F000Fu) | M1;
    h0[0] = (w0 & 0x00F000F0u) | M2;
    h0[1] = (v0 & 0x00F000F0u) | M2;
    h0[2] = (w1 & 0x00F000F0u) | M2;
    h0[3] = (v1 & 0x00F000F0u) | M2;
    h1[0] = (w2 & 0x00F000F0u) | M2;
    h1[1] = (v2 & 0x00F000F0u) | M2;
    h1[2] = (w3 & 0x00F000F0u) | M2;
    h1[3] = (v3 & 0x00F000F0u) | M2;
  }
  float d0[4], d1[4];
  mma_f16_z(d0, l0, b01.x, b01.y);
  mma_f16(d0, l1, b01.z, b01.w);
  mma_f16_z(d1, h0, b23.x, b23.y);
  mma_f16(d1, h1, b23.z, b23.w);
  acc_lo = fmaf(c0.x, d0[0], acc_lo);
  acc_lo = fmaf(-c0.z, xs.x, acc_lo);
  acc_hi = fmaf(c0.y, d0[2], acc_hi);
  acc_hi = fmaf(-c0.w, xs.x, acc_hi);
  acc_lo = fmaf(c1.x, d1[0], acc_lo);
  acc_lo = fmaf(-c1.z, xs.y, acc_lo);
  acc_hi = fmaf(c1.y, d1[2], acc_hi);
  acc_hi = fmaf(-c1.w, xs.y, acc_hi);
}

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Shared memory per staged vector v: xf (KB x 128 B: for k-block kb and quad
// lane t, the eight B-fragment registers of the four MMAs) and X (KB x 8 B:
// the two sub-block sums); then 32 zero bytes (the B operand of lanes whose
// fragment column is not the token's), the per-vector unscale factors and
// the warps' rings.
__host__ __device__ inline size_t pk_zero_off(int nv, int KB) { return ((size_t)nv * KB * 136 + 15) & ~size_t(15); }
__host__ __device__ inline size_t pk_ring_off(int nv, int KB) { return pk_zero_off(nv, KB) + 128; }
__host__ __device__ inline size_t pk_smem(int nv, int KB) {
  return pk_ring_off(nv, KB) + (size_t)kPkWarps * kSlots * kSlotBytes;
}

// Four consecutive elements [k, k+4) of staged vector v as floats.
template <int MODE>
__device__ __forceinline__ float4 vec4(const PkArgs& a, int v, int k) {
  if (MODE == 0) {
    const uint2 r = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(a.x) + k);
    return make_float4(__uint_as_float(r.x << 16), __uint_as_float(r.x & 0xFFFF0000u), __uint_as_float(r.y << 16),
                       __uint_as_float(r.y & 0xFFFF0000u));
  }
  return __ldcg(reinterpret_cast<const float4*>(static_cast<const float*>(a.x) + (int64_t)v * a.I + k));
}

// Thread i owns float4 groups q = i + 512 u of the flat range of all staged
// vectors; vector v = q / K4.
template <int MODE>
__device__ __forceinline__ float4 stage_load(const PkArgs& a, int q, int K4, int total) {
  const int v = q / K4;
  return q < total ? vec4<MODE>(a, v, 4 * (q - v * K4)) : make_float4(0.f, 0.f, 0.f, 0.f);
}

// Pass 2 of one group: scale, round to fp16, sub-block sum over eight lanes,
// store into the fragment-order image.  All lanes of the warp call it.
template <int MODE>
__device__ __forceinline__ void stage_store(const PkArgs& a, uint8_t* sm, const float* s_scale, int q, int K4,
                                            int total, float4 f, int lane) {
  const int v = min(q / K4, a.nv - 1), m = q - v * K4;
  const float sc = s_scale[v];
  const __half2 h01 = __floats2half2_rn(f.x * sc, f.y * sc);
  const __half2 h23 = __floats2half2_rn(f.z * sc, f.w * sc);
  const float2 g01 = __half22float2(h01), g23 = __half22float2(h23);
  float sum = (g01.x + g01.y) + (g23.x + g23.y);
  sum += __shfl_xor_sync(0xffffffffu, sum, 1);
  sum += __shfl_xor_sync(0xffffffffu, sum, 2);
  sum += __shfl_xor_sync(0xffffffffu, sum, 4);
  if (q >= total) return;
  float* X = reinterpret_cast<float*>(sm + (size_t)a.nv * a.KB * 128);
  if ((lane & 7) == 0) X[(size_t)v * 2 * a.KB + (m >> 3)] = sum;
  // k = 4m: k-block kb = m/16, MMA j = (m/4)%4, w0 = 4*(m%4) in [0,16):
  // pairs (w0, w0+1) and (w0+2, w0+3) go to quad lanes tt and tt+1 of half w0/8
  const int kb = m >> 4, j = (m >> 2) & 3, w0 = 4 * (m & 3);
  const int tt = (w0 & 7) >> 1, hf = w0 >> 3;
  const int i0 = ((kb * 4 + tt) * 4 + j) * 2 + hf;
  uint32_t* xf = reinterpret_cast<uint32_t*>(sm + (size_t)v * a.KB * 128);
  xf[i0] = *reinterpret_cast<const uint32_t*>(&h01);
  xf[i0 + 8] = *reinterpret_cast<const uint32_t*>(&h23);
}

// Max |x| per vector over this thread's groups, then the block-wide
// power-of-two scales (max|x| in [2^14, 2^15), exact in fp32).
__device__ __forceinline__ void stage_scales(const PkArgs& a, float (&mx)[8], float* inv, float* s_scale,
                                             float (*red)[kPkWarps], int warp, int lane) {
#pragma unroll
  for (int v = 0; v < 8; ++v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) mx[v] = fmaxf(mx[v], __shfl_xor_sync(0xffffffffu, mx[v], o));
    if (lane == 0) red[v][warp] = mx[v];
  }
  __syncthreads();
  if (threadIdx.x < a.nv) {
    const int v = threadIdx.x;
    float m = red[v][0];
    for (int i = 1; i < kPkWarps; ++i) m = fmaxf(m, red[v][i]);
    const int ex = (int)((__float_as_uint(m) >> 23) & 255u);
    int sx = (m > 0.f && ex != 255) ? 14 - (ex - 127) : 0;
    sx = max(-126, min(126, sx));
    s_scale[v] = __uint_as_float((uint32_t)(sx + 127) << 23);
    inv[v] = __uint_as_float((uint32_t)(127 - sx) << 23);
  }
  __syncthreads();
}

__device__ __forceinline__ void max_into(float (&mx)[8], int v, float4 f) {
  const float m = fmaxf(fmaxf(fabsf(f.x), fabsf(f.y)), fmaxf(fabsf(f.z), fabsf(f.w)));
#pragma unroll
  for (int w = 0; w < 8; ++w)
    if (w == v) mx[w] = fmaxf(mx[w], m);
}

// Staging of all vectors: max |x| per vector, then scale, round to fp16,
// permute into fragment order and sum per sub-block; two block barriers.  When
// the vectors fit in kStageRegs groups per thread (the GPT-OSS shapes: 720 and
// 2880 groups) the groups are loaded once and kept in registers for both
// passes; otherwise each pass loads kStageU groups per thread at a time.
// The eight groups of a 32-element sub-block sit on eight consecutive lanes
// (vector length K4 is a multiple of 16 groups), so three shuffles sum it.
constexpr int kStageU = 4, kStageRegs = 8;

template <int MODE>
__device__ void stage_vectors(const PkArgs& a, uint8_t* sm, float* inv, int warp, int lane) {
  __shared__ float red[8][kPkWarps];
  __shared__ float s_scale[8];
  const int K4 = 16 * a.KB, total = a.nv * K4;
  float mx[8];
#pragma unroll
  for (int v = 0; v < 8; ++v) mx[v] = 0.f;
  if (total <= kStageRegs * kPkThreads) {
    float4 f[kStageRegs];
#pragma unroll
    for (int u = 0; u < kStageRegs; ++u) f[u] = stage_load<MODE>(a, threadIdx.x + u * kPkThreads, K4, total);
#pragma unroll
    for (int u = 0; u < kStageRegs; ++u) {
      const int q = threadIdx.x + u * kPkThreads;
      if (q < total) max_into(mx, q / K4, f[u]);
    }
    stage_scales(a, mx, inv, s_scale, red, warp, lane);
#pragma unroll
    for (int u = 0; u < kStageRegs; ++u) {
      if ((int)(threadIdx.x - lane) + u * kPkThreads >= total) break;  // warp-uniform
      stage_store<MODE>(a, sm, s_scale, threadIdx.x + u * kPkThreads, K4, total, f[u], lane);
    }
    return;
  }
  for (int q0 = threadIdx.x; q0 < total; q0 += kStageU * kPkThreads) {
    float4 f[kStageU];
#pragma unroll
    for (int u = 0; u < kStageU; ++u) f[u] = stage_load<MODE>(a, q0 + u * kPkThreads, K4, total);
#pragma unroll
    for (int u = 0; u < kStageU; ++u) {
      const int q = q0 + u * kPkThreads;
      if (q < total) max_into(mx, q / K4, f[u]);
    }
  }
  stage_scales(a, mx, inv, s_scale, red, warp, lane);
  // all lanes stay in the loop for the shuffles (a sub-block's eight lanes are
  // all in range or all out)
  for (int q0 = threadIdx.x - lane; q0 < total; q0 += kStageU * kPkThreads) {
    float4 f[kStageU];
#pragma unroll
    for (int u = 0; u < kStageU; ++u) f[u] = stage_load<MODE>(a, q0 + lane + u * kPkThreads, K4, total);
#pragma unroll
    for (int u = 0; u < kStageU; ++u) {
      if (q0 + u * kPkThreads >= total) break;  // warp-uniform
      stage_store<MODE>(a, sm, s_scale, q0 + lane + u * kPkThreads, K4, total, f[u], lane);
    }
  }
}

// Routing of one token inside every gate/up CTA (tinyserve/_model_hooks.py:466-473):
// warp w computes the logits of experts w, w+16, ... (bf16 x . bf16 W[e] in
// fp32, + bias, rounded to bf16 as the reference's bf16 Linear returns them)
// into shared memory, then warp 0 selects the top-k (ties -> lower id, NaN
// lowest) and softmaxes the k selected logits.  Every CTA reaches the same
// result from the same arithmetic; CTA 0 publishes ids / weights.
__device__ void route_in_cta(const PkArgs& a, float* s_logit, int* s_e, float* s_w, int warp, int lane) {
  const int H = a.H, n8 = H / 8;
  const uint4* xr = static_cast<const uint4*>(a.x);
  constexpr int kU = 12;  // 384 16-byte groups per pass: one pass for H <= 3072
  for (int e = warp; e < a.n_experts; e += kPkWarps) {
    const uint4* wr = reinterpret_cast<const uint4*>(a.router_w + (int64_t)e * H);
    float acc = 0.f;
    for (int base = lane; base < n8; base += 32 * kU) {
      uint4 xv[kU], wv[kU];
#pragma unroll
      for (int j = 0; j < kU; ++j) {
        const int i = base + 32 * j;
        xv[j] = i < n8 ? __ldg(xr + i) : make_uint4(0, 0, 0, 0);
        wv[j] = i < n8 ? __ldg(wr + i) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int j = 0; j < kU; ++j) {
        const uint32_t av[4] = {xv[j].x, xv[j].y, xv[j].z, xv[j].w}, bv[4] = {wv[j].x, wv[j].y, wv[j].z, wv[j].w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc = fmaf(__uint_as_float(av[q] << 16), __uint_as_float(bv[q] << 16), acc);
          acc = fmaf(__uint_as_float(av[q] & 0xFFFF0000u), __uint_as_float(bv[q] & 0xFFFF0000u), acc);
        }
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) s_logit[e] = bf16_bits_to_f32(f32_to_bf16_bits(a.router_b ? acc + a.router_b[e] : acc));
  }
  __syncthreads();
  if (warp != 0) return;
  float sel[8];
  int sid[8];
  uint32_t taken = 0;  // bit j: expert lane + 32*j already selected (E <= 1024)
  for (int k = 0; k < a.top_k; ++k) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int j = 0; lane + 32 * j < a.n_experts; ++j) {
      if ((taken >> j) & 1u) continue;
      const int ee = lane + 32 * j;
      float v = s_logit[ee];
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
    for (int k = 0; k < a.top_k; ++k) { ex[k] = __expf(sel[k] - mx); den += ex[k]; }
    for (int k = 0; k < a.top_k; ++k) {
      s_e[k] = sid[k];
      s_w[k] = ex[k] / den;
      if (blockIdx.x == 0) {
        const_cast<int32_t*>(a.ids)[k] = sid[k];
        const_cast<float*>(a.wts)[k] = ex[k] / den;
      }
    }
    // published before this CTA lets the down kernel launch, whose L2
    // prefetch reads them (a hint; its real reads follow its PDL wait)
    if (blockIdx.x == 0) __threadfence();
  }
}

template <int MODE>
__global__ void __launch_bounds__(kPkThreads, 1) packed_matvec_kernel(const PkArgs a) {
  extern __shared__ uint4 smem4[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(smem4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  uint8_t* zero = sm + pk_zero_off(a.nv, a.KB);
  uint8_t* ring = sm + pk_ring_off(a.nv, a.KB) + (size_t)warp * kSlots * kSlotBytes;
  float* inv = reinterpret_cast<float*>(zero + 32);
  __shared__ int s_e[8];
  __shared__ uint64_t s_bar[kPkWarps][kSlots];
  uint64_t* bar = s_bar[warp];
  if (threadIdx.x < 8) reinterpret_cast<uint32_t*>(zero)[threadIdx.x] = 0u;
  if (lane < kSlots) mbar_init(&bar[lane], 1);
  fence_barrier_init();

  const int gw0 = blockIdx.x * kPkWarps + warp, nw = gridDim.x * kPkWarps;
  auto task_ptr = [&](int task, int e, int& kb0, int& kb1) {
    const int rem = task % (a.R * a.S), rb = rem / a.S, s = rem % a.S;
    kb0 = s * a.nkb;
    kb1 = min(a.KB, kb0 + a.nkb);
    return a.packed + (int64_t)e * a.expert_bytes + a.sec_off + ((int64_t)rb * a.KB + kb0) * kUnitBytes;
  };
  auto expert_of = [&](int u, bool report) {
    const int e = a.ids[u];
    if ((unsigned)e >= (unsigned)a.n_experts) {
      if (report && a.err) atomicExch(a.err, kDevBadPlan);
      return -1;
    }
    return e;
  };

  __shared__ float s_logit[1024];
  __shared__ float s_w[8];
  bool routed_here = false;
  if (MODE == 0) {
    if (a.router_w) {
      route_in_cta(a, s_logit, s_e, s_w, warp, lane);
      routed_here = true;
    }
    // x does not depend on the router kernel (when there is one): stage it
    // while that runs
    stage_vectors<0>(a, sm, inv, warp, lane);
    pdl_wait();
  } else {
    // Pull this warp's weight ranges into L2 while gate/up finishes.  The ids
    // read here are a hint only (routing inside the gate/up launch may not have
    // published them yet); the ids used below are read after the wait.
    if (lane == 0)
      for (int task = gw0; task < a.ntasks; task += nw) {
        const int e = expert_of(task / (a.R * a.S), false);
        if (e < 0) continue;
        int kb0, kb1;
        const uint8_t* p = task_ptr(task, e, kb0, kb1);
        prefetch_l2(p, (uint32_t)(kb1 - kb0) * kUnitBytes);
      }
    pdl_wait();
  }
  if (!routed_here && threadIdx.x < a.top_k) s_e[threadIdx.x] = expert_of(threadIdx.x, true);
  // bias pointers of the chosen experts, read once per CTA (the epilogues'
  // only other dependent load)
  __shared__ const float* s_bias[2][8];
  if (threadIdx.x < a.top_k) {
    const int e = s_e[threadIdx.x];
    const TsbExpert* E = a.experts + (e < 0 ? 0 : e);
    s_bias[0][threadIdx.x] = e < 0 ? nullptr : (MODE == 0 ? E->gate_bias : E->down_bias);
    s_bias[1][threadIdx.x] = e < 0 ? nullptr : (MODE == 0 ? E->up_bias : nullptr);
  }
  pdl_launch_dependents();
  if (MODE == 1) stage_vectors<1>(a, sm, inv, warp, lane);
  __syncthreads();

  uint32_t issued = 0, consumed = 0;  // slot fills / drains of this warp's ring
  bool bad = false;                   // a slot wait ran out: stop streaming
  // Per-task geometry (one division chain per task, not per slot).
  struct TaskGeo {
    const uint8_t* p;  // first unit
    int n, u, rb, kb0;
  };
  auto geo = [&](int task) {
    TaskGeo G;
    G.u = task / (a.R * a.S);
    const int rem = task - G.u * (a.R * a.S);
    G.rb = rem / a.S;
    G.kb0 = (rem - G.rb * a.S) * a.nkb;
    const int e = s_e[G.u];
    G.n = e < 0 ? 0 : min(a.KB, G.kb0 + a.nkb) - G.kb0;
    G.p = a.packed + (int64_t)(e < 0 ? 0 : e) * a.expert_bytes + a.sec_off +
          ((int64_t)G.rb * a.KB + G.kb0) * kUnitBytes;
    return G;
  };
  // issue cursor: the next (task, group) to fetch, running ahead of the consumer
  int it_task = gw0, it_g = 0;
  TaskGeo it_geo{};
  if (gw0 < a.ntasks) it_geo = geo(gw0);
  auto issue_next = [&]() {
    while (it_task < a.ntasks && it_g * kSlotUnits >= it_geo.n) {
      it_task += nw;
      it_g = 0;
      if (it_task < a.ntasks) it_geo = geo(it_task);
    }
    if (it_task >= a.ntasks) return;
    const uint32_t bytes = (uint32_t)min(kSlotUnits, it_geo.n - it_g * kSlotUnits) * kUnitBytes;
    uint64_t* b = &bar[issued & (kSlots - 1)];
    if (lane == 0) {
      mbar_arrive_expect_tx(b, bytes);
      bulk_g2s(ring + (issued & (kSlots - 1)) * kSlotBytes, it_geo.p + (size_t)it_g * kSlotBytes, bytes, b);
    }
    ++issued;
    ++it_g;
  };
#pragma unroll
  for (int i = 0; i < kSlots; ++i) issue_next();
  const int oq = 16 * lane, oc = 512 + 16 * g;

  for (int task = gw0; task < a.ntasks; task += nw) {
    const TaskGeo G = geo(task);
    const int u = G.u, rb = G.rb, n = G.n, kb0 = G.kb0;
    const int e = s_e[u];
    float acc_lo = 0.f, acc_hi = 0.f, acc_lo1 = 0.f, acc_hi1 = 0.f;
    if (n > 0 && !bad) {
      const int v = MODE == 0 ? 0 : u;
      const uint8_t* xb = g == 0 ? sm + (size_t)v * a.KB * 128 + (size_t)kb0 * 128 + 32 * t : zero;
      const int xstep = g == 0 ? 128 : 0;
      const float2* X = reinterpret_cast<const float2*>(sm + (size_t)a.nv * a.KB * 128) + (size_t)v * a.KB + kb0;
      for (int u0 = 0; u0 < n; u0 += kSlotUnits) {
        const uint32_t sl = consumed & (kSlots - 1);
        if (!pk_warp_wait(&bar[sl], (consumed / kSlots) & 1u, a.err)) {
          bad = true;
          break;
        }
        ++consumed;
        const uint8_t* slot = ring + sl * kSlotBytes;
        if (u0 + kSlotUnits <= n) {
          // full slot: independent units, two accumulator pairs
#pragma unroll
          for (int ui = 0; ui < kSlotUnits; ++ui)
            unit_fma(slot + ui * kUnitBytes, oq, oc, xb + ui * xstep, X[ui], a.magic1024, a.magic64,
                     (ui & 1) ? acc_lo1 : acc_lo, (ui & 1) ? acc_hi1 : acc_hi);
        } else {
          for (int ui = 0; ui < n - u0; ++ui)
            unit_fma(slot + ui * kUnitBytes, oq, oc, xb + ui * xstep, X[ui], a.magic1024, a.magic64, acc_lo,
                     acc_hi);
        }
        xb += kSlotUnits * xstep;
        X += kSlotUnits;
        __syncwarp();  // every lane has read the slot before it is refilled
        issue_next();
      }
    }
    acc_lo += acc_lo1;
    acc_hi += acc_hi1;
    // partial sums of rows g and g+8 live in the t == 0 lanes
    float* P = a.part + (int64_t)task * 16;
    if (t == 0) {
      P[g] = acc_lo;
      P[g + 8] = acc_hi;
    }
    // The warp barrier orders the lanes' partial stores before lane 0's
    // counter update; the update releases them at GPU scope (release is
    // cumulative) and acquires the other tasks' partials for the last one.
    __syncwarp();
    const int slot = MODE == 0 ? u * a.R + rb : rb;
    const unsigned need = MODE == 0 ? (unsigned)a.S : (unsigned)(a.top_k * a.S);
    unsigned last = 0;
    if (lane == 0) {
      unsigned old;
      asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(old) : "l"(a.cnt + slot) : "memory");
      last = old == need - 1;
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) continue;
    if (MODE == 0) {
      const int j = 8 * rb + lane;
      if (lane < 8 && j < a.I) {
        float gate = 0.f, up = 0.f;
        const float* Q = a.part + (int64_t)(u * a.R + rb) * a.S * 16;
        for (int s = 0; s < a.S; ++s) {
          gate += __ldcg(Q + 16 * s + lane);
          up += __ldcg(Q + 16 * s + lane + 8);
        }
        float r = 0.f;
        if (e >= 0) {
          gate *= inv[0];
          up *= inv[0];
          if (s_bias[0][u]) gate += s_bias[0][u][j];
          if (s_bias[1][u]) up += s_bias[1][u][j];
          r = act_fn(a.act, gate, up, a.limit, a.alpha);
        }
        a.act_out[(int64_t)u * a.I + j] = r;
      }
    } else {
      // lane = row (lane & 15) x half (lane >> 4); the halves take alternate
      // (slot, split) partials, all loads issued before the sums, then one shuffle.
      const int r = lane & 15, hf = lane >> 4, h = 16 * rb + r;
      const int nks = a.top_k * a.S;
      float o = 0.f;
      for (int i0 = hf; i0 < nks; i0 += 16) {
        float pv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int i = i0 + 2 * j;
          const int k = i / a.S, sp = i - k * a.S;
          pv[j] = (i < nks && s_e[min(k, 7)] >= 0) ? __ldcg(a.part + ((int64_t)(k * a.R + rb) * a.S + sp) * 16 + r) : 0.f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int i = i0 + 2 * j;
          if (i >= nks) break;
          const int k = i / a.S;
          o = fmaf(a.wts[k] * inv[k], pv[j], o);
        }
      }
      o += __shfl_xor_sync(0xffffffffu, o, 16);
      if (lane < 16 && h < a.H) {
        for (int k = 0; k < a.top_k; ++k) {
          const int ek = s_e[k];
          if (ek < 0) continue;
          const float* bias = s_bias[0][k];
          if (bias) o = fmaf(a.wts[k], bias[h], o);
        }
        a.out[h] = f32_to_bf16_bits(o);
      }
    }
    if (lane == 0) a.cnt[slot] = 0u;
  }
  // copies still in flight after a timed-out wait land before the CTA exits
  while (consumed < issued) {
    if (!pk_warp_wait(&bar[consumed % kSlots], (consumed / kSlots) & 1u, a.err)) break;
    ++consumed;
  }
}

static int num_sms_pk() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// K-split: k-blocks per task a multiple of kSlotUnits (so every slot but a
// row's last is full), the smallest makespan (k-blocks per warp plus one of
// per-task overhead) over the resident warps, at most kMaxSplit tasks per row.
static int choose_nkb(int rows, int KB, int warps) {
  int best = 0;
  double best_t = 1e30;
  const int top = (KB + kSlotUnits - 1) / kSlotUnits * kSlotUnits;
  for (int nkb = kSlotUnits; nkb <= top; nkb += kSlotUnits) {
    const int S = (KB + nkb - 1) / nkb;
    if (S > kMaxSplit) continue;
    const int64_t tasks = (int64_t)rows * S;
    const double waves = (double)((tasks + warps - 1) / warps);
    const double tm = waves * (nkb + 1);
    if (tm < best_t - 1e-9) {
      best_t = tm;
      best = nkb;
    }
  }
  return best;
}

size_t packed_ws_bytes(const TsbMoeSpec& sp) {
  const PackGeom G = pack_geom(sp);
  const int64_t parts =
      (int64_t)sp.top_k * std::max<int64_t>((int64_t)G.rgu * std::min(G.kbh, kMaxSplit), (int64_t)G.rdn * std::min(G.kbi, kMaxSplit));
  const int64_t cnts = std::max<int64_t>((int64_t)sp.top_k * G.rgu, G.rdn);
  return (size_t)(parts * 16 * 4 + cnts * 4 + 512);
}

constexpr size_t kPkSmemMax = 160 * 1024;

// One CTA per SM (measured: two per SM, one task per warp, ran the layer in
// 51 us against 43 us).
constexpr int kPkCtasPerSm = 1;

template <int MODE>
static int launch_pk(PkArgs& a, int rows, cudaStream_t st, bool pdl) {
  const int grid = kPkCtasPerSm * num_sms_pk();
  a.nkb = choose_nkb(rows, a.KB, grid * kPkWarps);
  a.S = (a.KB + a.nkb - 1) / a.nkb;
  a.ntasks = rows * a.S;
  const size_t smem = pk_smem(a.nv, a.KB);
  static bool attr = [] {
    return cudaFuncSetAttribute(packed_matvec_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)kPkSmemMax) == cudaSuccess;
  }();
  if (!attr || smem > kPkSmemMax)
    return set_error(TSB_ERR_UNSUPPORTED, "packed decode: vectors too long for shared memory");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kPkThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, packed_matvec_kernel<MODE>, a);
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  return TSB_OK;
}

int launch_packed_decode(const TsbMoeSpec& sp, const void* packed, const TsbExpert* ex, const void* x,
                         const int32_t* ids, const float* wts, float* act, void* out, int32_t* err, char* pws,
                         cudaStream_t st, const void* router_w, const float* router_b) {
  const PackGeom G = pack_geom(sp);
  PkArgs a{};
  a.packed = static_cast<const uint8_t*>(packed);
  a.expert_bytes = G.expert_bytes;
  a.ids = ids;
  a.wts = wts;
  a.experts = ex;
  a.n_experts = sp.n_experts;
  a.top_k = sp.top_k;
  a.err = err;
  a.I = sp.inter;
  a.H = sp.hidden;
  a.act = sp.activation;
  a.limit = sp.limit;
  a.alpha = sp.alpha;
  a.act_out = act;
  a.out = static_cast<uint16_t*>(out);
  a.cnt = reinterpret_cast<unsigned*>(pws);
  a.magic1024 = 0x64006400u;
  a.magic64 = 0x54005400u;
  const int64_t cnts = std::max<int64_t>((int64_t)sp.top_k * G.rgu, G.rdn);
  a.part = reinterpret_cast<float*>(pws + ((cnts * 4 + 255) & ~int64_t(255)));

  PkArgs gu = a;
  gu.mode = 0;
  gu.sec_off = G.gu_off;
  gu.R = G.rgu;
  gu.KB = G.kbh;
  gu.x = x;
  gu.nv = 1;
  gu.router_w = static_cast<const uint16_t*>(router_w);
  gu.router_b = router_b;
  int rc = launch_pk<0>(gu, sp.top_k * G.rgu, st, false);
  if (rc) return rc;
  PkArgs dn = a;
  dn.mode = 1;
  dn.sec_off = G.dn_off;
  dn.R = G.rdn;
  dn.KB = G.kbi;
  dn.x = act;
  dn.nv = sp.top_k;
  return launch_pk<1>(dn, sp.top_k * G.rdn, st, true);
}

}  // namespace tsb
