// Internal declarations shared by the C-ABI layer and the kernel files.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

#include "../../include/tsb_moe.h"

namespace tsb {

// Records msg as the calling thread's last error and returns code.
int set_error(int code, const char* msg);

// Data / scale bytes of a [rows, cols] weight (scale bytes are 0 except MXFP4).
void weight_bytes_of(int fmt, int64_t rows, int64_t cols, int64_t& data, int64_t& scales);

int max_vectors_for(int K);

int launch_matvec(int fmt, const void* w, const void* s, int64_t N, int64_t K, const void* x, int xdt, int nv,
                  int64_t xs, void* y, int ydt, int64_t ys, int32_t* err, cudaStream_t st);
int launch_gate_up(const TsbMoeSpec& sp, const TsbExpert* ex, const int32_t* ids, const void* x, float* act,
                   int32_t* err, cudaStream_t st, bool pdl);
int launch_down(const TsbMoeSpec& sp, const TsbExpert* ex, const int32_t* ids, const float* wts, const float* act,
                void* out, int32_t* err, cudaStream_t st, bool pdl);
int launch_router(const void* x, const void* W, const float* b, int H, int E, int T, int top_k, float* logits,
                  int32_t* ids, float* wts, unsigned* counter, cudaStream_t st);
// Workspace layout of tsb_moe_prefill (byte offsets) and its tile geometry.
struct PrefillLayout {
  size_t err, total_mb, counts, ccount, mb_expert, row_of, row_src, row_shift, xp, act, y, wgu, wdn, total;
  int64_t rows_max, wgu_estride, wdn_estride;
  int mb_max, kbh, kbi, nt_gu, nt_dn;
  bool fused_gu, fused_dn;  // MXFP4 decoded inside the GEMM (no fp16 weight tiles)
  bool pair;                // tiled GEMMs on CTA pairs (experts padded to 256 rows)
  int pad;                  // expert row padding: 128, or 256 for CTA pairs
};
PrefillLayout prefill_layout(const TsbMoeSpec& sp, int T);
int launch_moe_prefill(const TsbMoeSpec& sp, const TsbExpert* ex, const void* x, int T, const void* rw,
                       const float* rb, int32_t* ids, float* wts, void* out, char* ws, const PrefillLayout& L,
                       cudaStream_t st);
int launch_route(const TsbMoeSpec& sp, const void* x, int T, const void* rw, const float* rb, int32_t* ids,
                 float* wts, cudaStream_t st);
// Decode-packed experts (batch-1 decode of Q4_K and MXFP4 layers).
bool packable(const TsbMoeSpec& sp);
size_t packed_total_bytes(const TsbMoeSpec& sp);
int launch_pack(const TsbMoeSpec& sp, const TsbExpert* experts, void* packed, cudaStream_t st);
size_t packed_ws_bytes(const TsbMoeSpec& sp);
int launch_packed_decode(const TsbMoeSpec& sp, const void* packed, const TsbExpert* ex, const void* x, int32_t* ids,
                         float* wts, void* out, int out_f32, int32_t* err, char* pws, cudaStream_t st,
                         const void* router_w, const float* router_b);
// Dense (fp32 / fp16 / bf16) expert layers (moe_dense.cu).
bool is_dense_fmt(int fmt);
struct DenseLayout {
  size_t err, counter, logits, act, part, total;
  int s_gu, s_dn;  // K slices of the [in, out] kernels (0 / 1 for [out, in])
};
DenseLayout dense_layout(const TsbMoeSpec& sp, int T);
int launch_dense_layer(const TsbMoeSpec& sp, const TsbExpert* ex, const void* x, int T, const void* router_w,
                       const float* router_b, int32_t* ids, float* wts, void* out, char* ws, const DenseLayout& L,
                       cudaStream_t st);
int launch_dequant(int fmt, const void* w, const void* s, int64_t rows, int64_t cols, void* out, int odt,
                   cudaStream_t st);

}  // namespace tsb
