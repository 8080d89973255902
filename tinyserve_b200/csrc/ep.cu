// Expert-parallel decode over NCCL, as a C-ABI entry point (tsb_ep_moe_decode).
//
// The layer's experts are split evenly over the ranks of a communicator the
// caller owns; every rank brings the same number T of tokens with their
// routing.  One call, all on the caller's stream, no host synchronisation:
//   1. all-gather of the tokens (bf16 [T, H] -> [G*T, H]) and of their
//      routing (ids as int32 bits and weights, one fp32 [T, 2k] block);
//   2. localise: a (token, slot) pair whose expert this rank owns keeps its
//      local id, every other pair gets -1 (the layer kernels skip it);
//   3. this rank's experts over all G*T rows (tsb_moe_decode_packed when a
//      packed copy is given, else tsb_moe_decode), fp32 partial outputs;
//   4. reduce-scatter (sum) of the partials: each rank receives its own T
//      rows, converted to bf16 unless the spec asks for fp32.
// The reference runs every expert of a layer on one GPU
// (tinyserve/expert_pipeline.py:140-164); this is the multi-GPU form of that
// call.
//
// NCCL is resolved at run time (dlopen of libnccl.so.2, preferring a copy the
// process already loaded, e.g. PyTorch's), so the library itself does not
// depend on it.  Only the public NCCL entry points below are used.
#include <dlfcn.h>

#include <cstdint>
#include <cstring>
#include <mutex>

#include "tsb_common.cuh"
#include "tsb_internal.h"

namespace tsb {
namespace {

// NCCL's public C types, as the API passes them (enums by value).
using nccl_comm = void*;
constexpr int kNcclFloat32 = 7, kNcclBfloat16 = 9, kNcclSum = 0;
using AllGatherFn = int (*)(const void*, void*, size_t, int, nccl_comm, cudaStream_t);
using ReduceScatterFn = int (*)(const void*, void*, size_t, int, int, nccl_comm, cudaStream_t);
using ErrStrFn = const char* (*)(int);

struct Nccl {
  AllGatherFn all_gather = nullptr;
  ReduceScatterFn reduce_scatter = nullptr;
  ErrStrFn err_str = nullptr;
  bool ok = false;
};

const Nccl& nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    n.all_gather = reinterpret_cast<AllGatherFn>(dlsym(h, "ncclAllGather"));
    n.reduce_scatter = reinterpret_cast<ReduceScatterFn>(dlsym(h, "ncclReduceScatter"));
    n.err_str = reinterpret_cast<ErrStrFn>(dlsym(h, "ncclGetErrorString"));
    n.ok = n.all_gather && n.reduce_scatter;
  });
  return n;
}

int nccl_error(const Nccl& n, int r) {
  return set_error(TSB_ERR_CUDA, n.err_str ? n.err_str(r) : "NCCL call failed");
}

// routing of this rank's T tokens as one fp32 [T, 2k] block: ids (bits), weights
__global__ void ep_pack_meta(const int32_t* ids, const float* wts, int n, int k, float* meta) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int t = i / k, j = i - t * k;
  meta[(size_t)t * 2 * k + j] = __int_as_float(ids[i]);
  meta[(size_t)t * 2 * k + k + j] = wts[i];
}

// gathered routing -> local ids (-1 where another rank owns the expert) and weights
__global__ void ep_localise(const float* meta, int n, int k, int base, int e_local, int32_t* lid, float* w) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int t = i / k, j = i - t * k;
  const int e = __float_as_int(meta[(size_t)t * 2 * k + j]) - base;
  lid[i] = (e >= 0 && e < e_local) ? e : -1;
  w[i] = meta[(size_t)t * 2 * k + k + j];
}

__global__ void ep_to_bf16(const float* in, size_t n, uint16_t* out) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = f32_to_bf16_bits(in[i]);
}

struct EpLayout {
  size_t x_all, meta, meta_all, lid, w, part, red, inner, total, inner_bytes;
};

// inner layer call: 0 tsb_moe_decode, 1 tsb_moe_decode_packed, 2 tsb_moe_prefill
EpLayout ep_layout(const TsbMoeSpec& sp, int T, int world, int mode) {
  auto al = [](size_t v) { return (v + 255) & ~size_t(255); };
  const size_t R = (size_t)world * T, H = sp.hidden, k = sp.top_k;
  TsbMoeSpec f = sp;
  f.out_f32 = 1;
  EpLayout L{};
  // the layer's own workspace first, so its device error word sits at the
  // start of the whole (tsb_read_device_error(workspace) reads it)
  L.inner = 0;
  L.inner_bytes = mode == 2   ? tsb_moe_prefill_workspace(&f, (int32_t)R)
                  : mode == 1 ? tsb_moe_decode_packed_workspace(&f, (int32_t)R)
                              : tsb_moe_decode_workspace(&f, (int32_t)R);
  L.x_all = al(L.inner + L.inner_bytes);
  L.meta = al(L.x_all + R * H * 2);
  L.meta_all = al(L.meta + (size_t)T * 2 * k * 4);
  L.lid = al(L.meta_all + R * 2 * k * 4);
  L.w = al(L.lid + R * k * 4);
  L.part = al(L.w + R * k * 4);
  L.red = al(L.part + R * H * 4);
  L.total = al(L.red + (size_t)T * H * 4);
  return L;
}

}  // namespace
}  // namespace tsb

extern "C" {

size_t tsb_ep_decode_workspace(const TsbMoeSpec* local_spec, int32_t T, int32_t world, int32_t packed) {
  if (!local_spec || T <= 0 || world <= 0) return 0;
  return tsb::ep_layout(*local_spec, T, world, packed != 0 ? 1 : 0).total;
}

size_t tsb_ep_prefill_workspace(const TsbMoeSpec* local_spec, int32_t T, int32_t world) {
  if (!local_spec || T <= 0 || world <= 0) return 0;
  return tsb::ep_layout(*local_spec, T, world, 2).total;
}

}  // extern "C"

namespace tsb {
namespace {
int ep_call(int mode, const TsbMoeSpec* local_spec, const TsbExpert* local_experts, const void* packed,
            const void* x, int32_t T, const int32_t* ids, const float* weights, void* out, void* nccl_comm,
            int32_t rank, int32_t world, void* workspace, size_t workspace_bytes, void* stream) {
  if (!local_spec || !local_experts || !x || !ids || !weights || !out || !nccl_comm || !workspace)
    return set_error(TSB_ERR_INVALID, "null pointer");
  if (T < 1) return set_error(TSB_ERR_INVALID, "T must be >= 1");
  if (world < 1 || rank < 0 || rank >= world) return set_error(TSB_ERR_INVALID, "rank out of range");
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return set_error(TSB_ERR_INVALID, "workspace must be 256-byte aligned");
  const TsbMoeSpec& sp = *local_spec;
  const EpLayout L = ep_layout(sp, T, world, mode);
  if (workspace_bytes < L.total) return set_error(TSB_ERR_WORKSPACE, "workspace too small");
  const Nccl& n = nccl();
  if (!n.ok) return set_error(TSB_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) not found");

  char* ws = static_cast<char*>(workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int k = sp.top_k, H = sp.hidden, R = world * T;
  auto* x_all = ws + L.x_all;
  auto* meta = reinterpret_cast<float*>(ws + L.meta);
  auto* meta_all = reinterpret_cast<float*>(ws + L.meta_all);
  auto* lid = reinterpret_cast<int32_t*>(ws + L.lid);
  auto* w = reinterpret_cast<float*>(ws + L.w);
  auto* part = reinterpret_cast<float*>(ws + L.part);
  auto* red = reinterpret_cast<float*>(ws + L.red);

  int r = n.all_gather(x, x_all, (size_t)T * H, kNcclBfloat16, nccl_comm, st);
  if (r) return nccl_error(n, r);
  const int nk = T * k;
  ep_pack_meta<<<(nk + 255) / 256, 256, 0, st>>>(ids, weights, nk, k, meta);
  r = n.all_gather(meta, meta_all, (size_t)T * 2 * k, kNcclFloat32, nccl_comm, st);
  if (r) return nccl_error(n, r);
  ep_localise<<<(R * k + 255) / 256, 256, 0, st>>>(meta_all, R * k, k, rank * sp.n_experts, sp.n_experts, lid, w);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));

  TsbMoeSpec f = sp;
  f.out_f32 = 1;
  const int rc = mode == 2   ? tsb_moe_prefill(&f, local_experts, x_all, R, nullptr, nullptr, lid, w, part,
                                                ws + L.inner, L.inner_bytes, stream)
                 : mode == 1 ? tsb_moe_decode_packed(&f, packed, local_experts, x_all, R, nullptr, nullptr, lid, w,
                                                     part, ws + L.inner, L.inner_bytes, stream)
                             : tsb_moe_decode(&f, local_experts, x_all, R, nullptr, nullptr, lid, w, part,
                                              ws + L.inner, L.inner_bytes, stream);
  if (rc) return rc;
  void* dst = sp.out_f32 ? out : red;
  r = n.reduce_scatter(part, dst, (size_t)T * H, kNcclFloat32, kNcclSum, nccl_comm, st);
  if (r) return nccl_error(n, r);
  if (!sp.out_f32) {
    const size_t cnt = (size_t)T * H;
    ep_to_bf16<<<(unsigned)((cnt + 255) / 256), 256, 0, st>>>(red, cnt, static_cast<uint16_t*>(out));
    e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  }
  return TSB_OK;
}
}  // namespace
}  // namespace tsb

extern "C" {

int tsb_ep_moe_decode(const TsbMoeSpec* local_spec, const TsbExpert* local_experts, const void* packed,
                      const void* x, int32_t T, const int32_t* ids, const float* weights, void* out,
                      void* nccl_comm, int32_t rank, int32_t world, void* workspace, size_t workspace_bytes,
                      void* stream) {
  return tsb::ep_call(packed ? 1 : 0, local_spec, local_experts, packed, x, T, ids, weights, out, nccl_comm, rank,
                      world, workspace, workspace_bytes, stream);
}

int tsb_ep_moe_prefill(const TsbMoeSpec* local_spec, const TsbExpert* local_experts, const void* x, int32_t T,
                       const int32_t* ids, const float* weights, void* out, void* nccl_comm, int32_t rank,
                       int32_t world, void* workspace, size_t workspace_bytes, void* stream) {
  return tsb::ep_call(2, local_spec, local_experts, nullptr, x, T, ids, weights, out, nccl_comm, rank, world,
                      workspace, workspace_bytes, stream);
}

}  // extern "C"
