// Bit-exact dequantisation kernels.
//
// Each thread decodes one 32-element block of the flat stream and writes 32
// outputs.  The float arithmetic repeats the reference decoder's operation
// order with explicitly rounded intrinsics (no FMA contraction):
//   Q8_0  d * q                          (gguf_dequant_torch.py:118-122)
//   Q4_K  (d*sc)*q - (dmin*m)            (gguf_dequant_torch.py:187-203)
//   Q5_K  (d*sc)*q - (dmin*m)            (gguf_dequant_torch.py:206-227)
//   Q6_K  (d*sc)*q                       (gguf_dequant_torch.py:230-249)
//   MXFP4 ldexp(lut[n], s-127)           (mxfp4.py:20-44), an exact power-of-two
//         scaling done as two exact multiplies so that only the final
//         product can round (to a subnormal) or overflow (to inf).
#include "qformats.cuh"
#include "tsb_internal.h"

namespace tsb {

__constant__ float kFp4Lut[16] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f,
                                  -0.f, -0.5f, -1.f, -1.5f, -2.f, -3.f, -4.f, -6.f};

__device__ __forceinline__ void put(void* out, int odt, int64_t i, float v) {
  if (odt == TSB_DT_F32) static_cast<float*>(out)[i] = v;
  else static_cast<uint16_t*>(out)[i] = f32_to_bf16_bits(v);
}

__device__ __forceinline__ float pow2i(int e) {  // 2^e for -126 <= e <= 127
  return __uint_as_float((uint32_t)(e + 127) << 23);
}

template <int F>
__global__ void dequant_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ s, int64_t nblk32,
                               void* out, int odt) {
  const int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (q >= nblk32) return;
  const int64_t o = q * 32;
  if (F == FMT_Q8_0) {
    const uint8_t* b = w + q * 34;
    const float d = half_bits_to_f32((uint16_t)(b[0] | (b[1] << 8)));
    for (int i = 0; i < 32; ++i) put(out, odt, o + i, __fmul_rn(d, (float)(int8_t)b[2 + i]));
  } else if (F == FMT_Q4_K || F == FMT_Q5_K) {
    const int BB = FmtT<F>::BB;
    const uint8_t* b = w + (q >> 3) * BB;
    const int j = (int)(q & 7);
    const float d = half_bits_to_f32((uint16_t)(b[0] | (b[1] << 8)));
    const float dmin = half_bits_to_f32((uint16_t)(b[2] | (b[3] << 8)));
    int sc, m;
    kq_scale_min(b + 4, j, sc, m);
    const float dsc = __fmul_rn(d, (float)sc), dm = __fmul_rn(dmin, (float)m);
    const uint8_t* qs = b + (F == FMT_Q4_K ? 16 : 48) + 32 * (j >> 1);
    const int sh = 4 * (j & 1);
    for (int l = 0; l < 32; ++l) {
      int v = (qs[l] >> sh) & 0xF;
      if (F == FMT_Q5_K) v |= ((b[16 + l] >> j) & 1) << 4;
      put(out, odt, o + l, __fsub_rn(__fmul_rn(dsc, (float)v), dm));
    }
  } else if (F == FMT_Q6_K) {
    const uint8_t* b = w + (q >> 3) * 210;
    const int g = (int)(q & 7), h = g >> 2, gg = g & 3;
    const float d = half_bits_to_f32((uint16_t)(b[208] | (b[209] << 8)));
    const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192) + 2 * g;
    const float d0 = __fmul_rn(d, (float)sc[0]), d1 = __fmul_rn(d, (float)sc[1]);
    const uint8_t* ql = b + 64 * h + 32 * (gg & 1);
    const uint8_t* qh = b + 128 + 32 * h;
    for (int l = 0; l < 32; ++l) {
      const int v = (((ql[l] >> (4 * (gg >> 1))) & 0xF) | (((qh[l] >> (2 * gg)) & 3) << 4)) - 32;
      put(out, odt, o + l, __fmul_rn(l < 16 ? d0 : d1, (float)v));
    }
  } else {  // MXFP4
    const uint8_t* b = w + q * 16;
    const int e = (int)s[q] - 127;
    const int e1 = e / 2, e2 = e - e1;  // both within [-64, 64]
    const float p1 = pow2i(e1), p2 = pow2i(e2);
    for (int i = 0; i < 16; ++i) {
      const float lo = kFp4Lut[b[i] & 0xF], hi = kFp4Lut[b[i] >> 4];
      put(out, odt, o + 2 * i, __fmul_rn(__fmul_rn(lo, p1), p2));
      put(out, odt, o + 2 * i + 1, __fmul_rn(__fmul_rn(hi, p1), p2));
    }
  }
}

int launch_dequant(int fmt, const void* w, const void* s, int64_t rows, int64_t cols, void* out, int odt,
                   cudaStream_t st) {
  const int64_t n = rows * cols / 32;
  if (n == 0) return TSB_OK;
  const int bs = 128;
  const int64_t grid = (n + bs - 1) / bs;
  const uint8_t* W = static_cast<const uint8_t*>(w);
  const uint8_t* S = static_cast<const uint8_t*>(s);
  switch (fmt) {
    case FMT_Q8_0: dequant_kernel<FMT_Q8_0><<<grid, bs, 0, st>>>(W, S, n, out, odt); break;
    case FMT_Q4_K: dequant_kernel<FMT_Q4_K><<<grid, bs, 0, st>>>(W, S, n, out, odt); break;
    case FMT_Q5_K: dequant_kernel<FMT_Q5_K><<<grid, bs, 0, st>>>(W, S, n, out, odt); break;
    case FMT_Q6_K: dequant_kernel<FMT_Q6_K><<<grid, bs, 0, st>>>(W, S, n, out, odt); break;
    case FMT_MXFP4: dequant_kernel<FMT_MXFP4><<<grid, bs, 0, st>>>(W, S, n, out, odt); break;
    default: return set_error(TSB_ERR_UNSUPPORTED, "unsupported format");
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  return TSB_OK;
}

}  // namespace tsb
