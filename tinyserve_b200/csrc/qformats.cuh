// Quantised weight formats: byte layouts, tensor-core fragment decoders and
// bit-exact scalar decoders.
//
// Layouts are the GGUF / HF-MXFP4 ones that tinyserve decodes
// (tinyserve/gguf_dequant_torch.py:95-249, tinyserve/mxfp4.py:5-44):
//   Q8_0  34 B / 32:  d f16 @0, qs int8[32] @2
//   Q4_K 144 B / 256: d @0, dmin @2, scales[12] @4, qs[128] @16
//   Q5_K 176 B / 256: d @0, dmin @2, scales[12] @4, qh[32] @16, qs[128] @48
//   Q6_K 210 B / 256: ql[128] @0, qh[64] @128, scales int8[16] @192, d @208
//   MXFP4: blocks [N, K/32, 16] (low nibble = even element), scales [N, K/32] E8M0
// A weight [N, K] is a flat stream of blocks in row-major element order, so for
// K % 256 != 0 a K-quant superblock can straddle two rows.
//
// Tensor-core decode.  The matvec kernels feed weights to
// mma.sync.m16n8k16 (f16 in, f32 accumulate).  For one 32-element block
// ("step") thread t of a quad supplies 8 weights of one row, in the order
// o[0..7] given by elem_order(); pairs (o0,o1),(o2,o3) feed the first k16 MMA
// and (o4,o5),(o6,o7) the second.  The activation vector is stored in shared
// memory permuted into the same order, so any order is legal; each format
// picks the one that decodes with the fewest instructions.  Integer codes are
// turned into f16 with the magic constant 0x6400 (= 1024.0): the f16 with
// bits 0x6400|u is exactly 1024+u for u < 1024.  The constant offset
// 1024*sum(x) is removed in the per-block fold.
#pragma once
#include "tsb_common.cuh"

namespace tsb {

enum : int { FMT_Q8_0 = 8, FMT_Q4_K = 12, FMT_Q5_K = 13, FMT_Q6_K = 14, FMT_MXFP4 = 39 };

template <int F> struct FmtT;
template <> struct FmtT<FMT_Q8_0> { static constexpr int BE = 32, BB = 34; };
template <> struct FmtT<FMT_Q4_K> { static constexpr int BE = 256, BB = 144; };
template <> struct FmtT<FMT_Q5_K> { static constexpr int BE = 256, BB = 176; };
template <> struct FmtT<FMT_Q6_K> { static constexpr int BE = 256, BB = 210; };
// MXFP4: the nibble stream is 16 B per 32 elements; scales live in their own tensor.
template <> struct FmtT<FMT_MXFP4> { static constexpr int BE = 32, BB = 16; };

// Position (0..31 within the step) of thread t's s-th weight.
template <int F>
__host__ __device__ __forceinline__ int elem_order(int t, int s) {
  if (F == FMT_Q4_K || F == FMT_Q5_K) {
    const int r = (s & 4) | ((s & 1) << 1) | ((s >> 1) & 1);  // 0,2,1,3,4,6,5,7
    return 8 * t + r;
  } else if (F == FMT_Q6_K) {
    const int q = s & 3;
    const int r = ((q & 1) << 1) | (q >> 1);  // 0,2,1,3
    return 16 * (s >> 2) + 4 * t + r;
  } else {
    return 8 * t + s;
  }
}

// Constant removed per block by the fold: magic 1024 plus the format's code bias.
template <int F> struct FoldBias;
template <> struct FoldBias<FMT_Q8_0> { static constexpr float v = 1152.f; };  // 1024 + 128 (int8 -> u8)
template <> struct FoldBias<FMT_Q4_K> { static constexpr float v = 1024.f; };
template <> struct FoldBias<FMT_Q5_K> { static constexpr float v = 1024.f; };
template <> struct FoldBias<FMT_Q6_K> { static constexpr float v = 1056.f; };  // 1024 + 32
template <> struct FoldBias<FMT_MXFP4> { static constexpr float v = 0.f; };

constexpr uint32_t kMagic = 0x64646464u;
// __byte_perm selectors: [x.b0, M, x.b2, M] and [x.b1, M, x.b3, M]
constexpr uint32_t kSel02 = 0x4240u, kSel13 = 0x4341u;
// [x.b0, M, x.b1, M] and [x.b2, M, x.b3, M]
constexpr uint32_t kSel01 = 0x4140u, kSel23 = 0x4342u;

// Where one row's bytes for one step sit in shared memory.
struct RowLoc {
  const uint8_t* blk;   // Q8_0 block / K-quant superblock / MXFP4 16-B block
  int sub;              // K-quants: 32-element sub-block index within the superblock (0..7)
  uint32_t mx_scale;    // MXFP4: E8M0 byte
};

// ---------------------------------------------------------------------------
// A-fragment decode: four f16x2 registers p[0..3] holding weights o0..o7 of
// this thread for one row and one 32-element step.
// ---------------------------------------------------------------------------
template <int F>
__device__ __forceinline__ void decode_a(const RowLoc& L, int t, uint32_t (&p)[4]);

template <>
__device__ __forceinline__ void decode_a<FMT_Q8_0>(const RowLoc& L, int t, uint32_t (&p)[4]) {
  const uint8_t* q = L.blk + 2 + 8 * t;  // 2-byte aligned
  const uint32_t w0 = lds_u32_a2(q) ^ 0x80808080u;
  const uint32_t w1 = lds_u32_a2(q + 4) ^ 0x80808080u;
  p[0] = prmt(w0, kMagic, kSel01);
  p[1] = prmt(w0, kMagic, kSel23);
  p[2] = prmt(w1, kMagic, kSel01);
  p[3] = prmt(w1, kMagic, kSel23);
}

template <>
__device__ __forceinline__ void decode_a<FMT_Q4_K>(const RowLoc& L, int t, uint32_t (&p)[4]) {
  const uint2 w = *reinterpret_cast<const uint2*>(L.blk + 16 + 32 * (L.sub >> 1) + 8 * t);
  const int sh = 4 * (L.sub & 1);
  const uint32_t a = (w.x >> sh) & 0x0F0F0F0Fu;
  const uint32_t b = (w.y >> sh) & 0x0F0F0F0Fu;
  p[0] = prmt(a, kMagic, kSel02);
  p[1] = prmt(a, kMagic, kSel13);
  p[2] = prmt(b, kMagic, kSel02);
  p[3] = prmt(b, kMagic, kSel13);
}

template <>
__device__ __forceinline__ void decode_a<FMT_Q5_K>(const RowLoc& L, int t, uint32_t (&p)[4]) {
  const uint2 w = *reinterpret_cast<const uint2*>(L.blk + 48 + 32 * (L.sub >> 1) + 8 * t);
  const uint2 h = *reinterpret_cast<const uint2*>(L.blk + 16 + 8 * t);
  const int sh = 4 * (L.sub & 1);
  const int rot = (4 - L.sub) & 31;  // bit `sub` of each qh byte -> bit 4
  const uint32_t a = ((w.x >> sh) & 0x0F0F0F0Fu) | (__funnelshift_l(h.x, h.x, rot) & 0x10101010u);
  const uint32_t b = ((w.y >> sh) & 0x0F0F0F0Fu) | (__funnelshift_l(h.y, h.y, rot) & 0x10101010u);
  p[0] = prmt(a, kMagic, kSel02);
  p[1] = prmt(a, kMagic, kSel13);
  p[2] = prmt(b, kMagic, kSel02);
  p[3] = prmt(b, kMagic, kSel13);
}

template <>
__device__ __forceinline__ void decode_a<FMT_Q6_K>(const RowLoc& L, int t, uint32_t (&p)[4]) {
  // sub = 32-element group g (0..7) = half h (g>>2), group-in-half gg (g&3).
  const int h = L.sub >> 2, gg = L.sub & 3;
  const uint8_t* ql = L.blk + 64 * h + 32 * (gg & 1) + 4 * t;
  const uint8_t* qh = L.blk + 128 + 32 * h + 4 * t;
  const int sh = 4 * (gg >> 1);
  const int rot = (4 - 2 * gg) & 31;  // bits (2gg, 2gg+1) of each qh byte -> bits 4,5
  const uint32_t l0 = lds_u32_a2(ql), l1 = lds_u32_a2(ql + 16);
  const uint32_t h0 = lds_u32_a2(qh), h1 = lds_u32_a2(qh + 16);
  const uint32_t a = ((l0 >> sh) & 0x0F0F0F0Fu) | (__funnelshift_l(h0, h0, rot) & 0x30303030u);
  const uint32_t b = ((l1 >> sh) & 0x0F0F0F0Fu) | (__funnelshift_l(h1, h1, rot) & 0x30303030u);
  p[0] = prmt(a, kMagic, kSel02);
  p[1] = prmt(a, kMagic, kSel13);
  p[2] = prmt(b, kMagic, kSel02);
  p[3] = prmt(b, kMagic, kSel13);
}

template <>
__device__ __forceinline__ void decode_a<FMT_MXFP4>(const RowLoc& L, int t, uint32_t (&p)[4]) {
  const uint32_t w = *reinterpret_cast<const uint32_t*>(L.blk + 4 * t);
  p[0] = cvt_e2m1x2(w & 0xFFu);
  p[1] = cvt_e2m1x2((w >> 8) & 0xFFu);
  p[2] = cvt_e2m1x2((w >> 16) & 0xFFu);
  p[3] = cvt_e2m1x2(w >> 24);
}

// ---------------------------------------------------------------------------
// Per-(row, step) fold coefficients: acc += A * (c*xs) - B * sum(x).
// Q6_K has two 16-element scale groups per step (A0,B0 / A1,B1).
// Arithmetic follows the reference decoders: d*sc and dmin*m are formed
// exactly as gguf_dequant_torch.py:195-203 forms them.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void kq_scale_min(const uint8_t* s12, int j, int& sc, int& m) {
  if (j < 4) {
    sc = s12[j] & 63;
    m = s12[j + 4] & 63;
  } else {
    sc = (s12[j + 4] & 0xF) | ((s12[j - 4] >> 6) << 4);
    m = (s12[j + 4] >> 4) | ((s12[j] >> 6) << 4);
  }
}

// Small non-negative integer (< 2^23) to float without the conversion unit:
// the float with bits 0x4B000000 | v is exactly 2^23 + v.
__device__ __forceinline__ float small_u2f(uint32_t v) { return __uint_as_float(0x4B000000u | v) - 8388608.f; }

template <int F>
__device__ __forceinline__ float4 fold_coef(const RowLoc& L) {
  if (F == FMT_Q4_K || F == FMT_Q5_K) {
    // superblocks are 16-B aligned in the stage: read d/dmin and the 12 scale bytes as words
    const uint4 hw = *reinterpret_cast<const uint4*>(L.blk);
    const float2 dd = __half22float2(*reinterpret_cast<const __half2*>(&hw.x));
    const int j = L.sub, sh = 8 * (j & 3);
    // j < 4: sc = s[j] & 63, m = s[j+4] & 63
    // j >= 4: sc = (s[j+4] & 15) | (s[j-4] >> 6) << 4, m = (s[j+4] >> 4) | (s[j] >> 6) << 4
    const uint32_t lo_sc = (hw.y >> sh) & 63u, lo_m = (hw.z >> sh) & 63u;
    const uint32_t hi_sc = ((hw.w >> sh) & 15u) | (((hw.y >> sh) >> 2) & 0x30u);
    const uint32_t hi_m = (((hw.w >> sh) >> 4) & 15u) | (((hw.z >> sh) >> 2) & 0x30u);
    const uint32_t sc = j < 4 ? lo_sc : hi_sc, m = j < 4 ? lo_m : hi_m;
    const float a = dd.x * small_u2f(sc);
    return make_float4(a, fmaf(FoldBias<F>::v, a, dd.y * small_u2f(m)), 0.f, 0.f);
  } else if (F == FMT_Q6_K) {
    const float d = half_bits_to_f32(*reinterpret_cast<const uint16_t*>(L.blk + 208));
    const uint32_t sp = *reinterpret_cast<const uint16_t*>(L.blk + 192 + 2 * L.sub);  // two int8 scales
    const float s0 = small_u2f((sp & 0xFFu) ^ 0x80u) - 128.f;
    const float s1 = small_u2f((sp >> 8) ^ 0x80u) - 128.f;
    const float a0 = d * s0, a1 = d * s1;
    return make_float4(a0, FoldBias<F>::v * a0, a1, FoldBias<F>::v * a1);
  } else if (F == FMT_Q8_0) {
    const float d = half_bits_to_f32(*reinterpret_cast<const uint16_t*>(L.blk));
    return make_float4(d, FoldBias<F>::v * d, 0.f, 0.f);
  } else {
    // E8M0: 2^(s-127); s = 0 is the subnormal 2^-127, s = 255 overflows to +inf.
    const uint32_t s = L.mx_scale;
    const float f = s ? __uint_as_float(s << 23) : __uint_as_float(0x00400000u);
    return make_float4(f, 0.f, 0.f, 0.f);
  }
}

}  // namespace tsb
