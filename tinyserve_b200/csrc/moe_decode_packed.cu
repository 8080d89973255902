// Batch-1 MoE decode, one persistent launch per token-layer, on a decode-packed
// copy of the experts (Q4_K or MXFP4).
//
// Packed unit = one row block (16 rows of one projection) x one chunk of 256
// columns.  Its codes are laid out so that one 128-bit shared-memory load
// gives a lane the A fragments of four mma.m16n8k16 (f16 in, f32 out), and the
// eight 32-element sub-blocks of the chunk are spread over the MMA's eight N
// columns: the B operand holds the activation vector "diagonally" (column n
// sees only sub-block n's elements), so after the chunk's 16 MMAs the
// accumulator holds, per row, the eight per-sub-block dot products.  The
// per-(row, sub-block) scale fold therefore runs once per 4096 weights rather
// than once per MMA.
//
// Q4_K (tinyserve/gguf_dequant_torch.py:180-205): a row of length K starts at
// superblock phase p = (row*K mod 256)/32; rows are grouped by phase (row maps)
// so that chunk c of every row in a block is exactly one source superblock,
// whose 144 bytes become the unit: codes (128 B per row) and a header of
// fp16 d / dmin and the eight 6-bit (scale, min) pairs widened to bytes
// (20 B per row).  1.03x the Q4_K bytes, plus the superblocks that straddle
// two rows, which both rows carry.  Codes decode to 64+q (0x5400|q<<4): one
// shift and one LOP3 per f16 pair (a 1024+q decode would save the shift but
// makes the accumulator 16x larger across the chunk's 16 chained MMAs and
// doubles the layer error); the offset is removed in the fold:
//   row += s*D_n - (off*s + dmin*m) * X_n,  s = d*sc,  X_n = sum of x over n.
// MXFP4 (tinyserve/mxfp4.py:20-44): e2m1 codes convert exactly with
// cvt.rn.f16x2.e2m1x2; the unit header is the 8 E8M0 scale bytes per row, the
// fold row += 2^(e_n - 127) * D_n.  Exactly the MXFP4 bytes.
//
// One launch per token-layer (cooperative, one CTA per SM):
//   1. every CTA routes the token itself (bf16 logits, top-k, softmax;
//      tinyserve/_model_hooks.py:466-473) and stages x as the f16 B image;
//   2. gate/up tasks (slot, j-group of 16 gate + 16 up rows, chunk range)
//      stream their units through a per-warp cp.async.bulk ring; the last
//      task of a j-group (counter) reduces the partial sums in fixed order,
//      applies the bias and the activation, and publishes 16 activations;
//   3. every CTA waits for all j-groups (a device-wide counter, bounded
//      wait), stages the top_k activation vectors as B images, and runs its
//      down tasks, whose weights its warps' rings and an L2 prefetch issued
//      right after routing have been pulling in meanwhile;
//   4. the last down task of a 32-row group combines slots and splits in
//      fixed order: out[h] = sum_k w_k * (down_k . act_k)[h] + w_k * b_k[h].
// Results do not depend on scheduling.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "../../include/tsb_moe.h"
#include "moe_math.cuh"
#include "qformats.cuh"
#include "tsb_common.cuh"
#include "tsb_internal.h"

namespace tsb {

constexpr int kPkThreads = 512;
constexpr int kPkWarps = kPkThreads / 32;
constexpr int kCopyLane = 31;
constexpr bool kPfGateUp = false, kPfDown = false;  // L2 prefetch of the chunks the ring does not hold yet        // the lane that issues bulk copies and L2 prefetches
constexpr int kSlots = 2;            // ring slots per warp (one chunk = two units each)
constexpr int kPadL = 8, kPadR = 16;  // zero sub-blocks before / after a B image (phase shifts, last chunk)
constexpr int kQ4Hdr = 320, kQ4Unit = 320 + 2048;
constexpr int kMxHdr = 128, kMxUnit = 128 + 2048;

bool packable(const TsbMoeSpec& sp) {
  const bool q4 = sp.fmt_gate_up == FMT_Q4_K && sp.fmt_down == FMT_Q4_K;
  const bool mx = sp.fmt_gate_up == FMT_MXFP4 && sp.fmt_down == FMT_MXFP4;
  return (q4 || mx) && sp.hidden % 32 == 0 && sp.inter % 32 == 0 && sp.hidden > 0 && sp.inter > 0 &&
         sp.hidden <= 16384 && sp.inter <= 16384 && sp.n_experts >= 1 && sp.n_experts <= 1024 && sp.top_k >= 1 &&
         sp.top_k <= 8 && sp.top_k <= sp.n_experts && sp.gate_up_layout >= 0 && sp.gate_up_layout <= 2;
}

// ------------------------------------------------------------------ geometry
static int q4_phase(int64_t row, int K) { return (int)(((row * K) % 256) / 32); }

static int64_t gate_row(const TsbMoeSpec& sp, int j) {
  return sp.gate_up_layout == TSB_GU_INTERLEAVED ? 2 * (int64_t)j : j;
}
static int64_t up_row(const TsbMoeSpec& sp, int j) {
  if (sp.gate_up_layout == TSB_GU_INTERLEAVED) return 2 * (int64_t)j + 1;
  if (sp.gate_up_layout == TSB_GU_CHUNKED) return (int64_t)sp.inter + j;
  return j;
}

// Row maps: gate/up j-groups of 16 outputs whose gate rows share one phase and
// whose up rows share one phase; down groups of 32 outputs of one phase.
struct PkMaps {
  std::vector<int32_t> gu_j, gu_ph, dn_h, dn_ph;
  int C_gu = 0, C_dn = 0;
};

static PkMaps pk_maps(const TsbMoeSpec& sp) {
  PkMaps M;
  const bool q4 = sp.fmt_gate_up == FMT_Q4_K;
  const int H = sp.hidden, I = sp.inter;
  // gate/up: key = gate phase * 8 + up phase
  std::vector<std::vector<int32_t>> b(64);
  for (int j = 0; j < I; ++j) {
    const int pg = q4 ? q4_phase(gate_row(sp, j), H) : 0, pu = q4 ? q4_phase(up_row(sp, j), H) : 0;
    b[pg * 8 + pu].push_back(j);
  }
  int pmax = 0;
  for (int key = 0; key < 64; ++key) {
    const auto& v = b[key];
    if (v.empty()) continue;
    pmax = std::max(pmax, std::max(key / 8, key % 8));
    for (size_t i = 0; i < v.size(); i += 16) {
      for (size_t r = 0; r < 16; ++r) M.gu_j.push_back(i + r < v.size() ? v[i + r] : -1);
      M.gu_ph.push_back(key / 8);
      M.gu_ph.push_back(key % 8);
    }
  }
  M.C_gu = (H / 32 + pmax + 7) / 8;
  std::vector<std::vector<int32_t>> d(8);
  for (int h = 0; h < H; ++h) d[q4 ? q4_phase(h, I) : 0].push_back(h);
  pmax = 0;
  for (int p = 0; p < 8; ++p) {
    const auto& v = d[p];
    if (v.empty()) continue;
    pmax = std::max(pmax, p);
    for (size_t i = 0; i < v.size(); i += 32) {
      for (size_t r = 0; r < 32; ++r) M.dn_h.push_back(i + r < v.size() ? v[i + r] : -1);
      M.dn_ph.push_back(p);
    }
  }
  M.C_dn = (I / 32 + pmax + 7) / 8;
  return M;
}

struct PkGeo {
  int q4, unit, hdr;
  int ngj, ndp, C_gu, C_dn;
  int64_t o_guj, o_guph, o_dnh, o_dnph, maps_bytes;
  int64_t gu_off, dn_off, expert_bytes, total;
};

static PkGeo pk_geo(const TsbMoeSpec& sp, const PkMaps& M) {
  PkGeo G{};
  G.q4 = sp.fmt_gate_up == FMT_Q4_K;
  G.unit = G.q4 ? kQ4Unit : kMxUnit;
  G.hdr = G.q4 ? kQ4Hdr : kMxHdr;
  G.ngj = (int)M.gu_ph.size() / 2;
  G.ndp = (int)M.dn_ph.size();
  G.C_gu = M.C_gu;
  G.C_dn = M.C_dn;
  auto al = [](int64_t v) { return (v + 255) & ~int64_t(255); };
  G.o_guj = 0;
  G.o_guph = al(G.o_guj + 4 * (int64_t)M.gu_j.size());
  G.o_dnh = al(G.o_guph + 4 * (int64_t)M.gu_ph.size());
  G.o_dnph = al(G.o_dnh + 4 * (int64_t)M.dn_h.size());
  G.maps_bytes = al(G.o_dnph + 4 * (int64_t)M.dn_ph.size());
  G.gu_off = 0;
  G.dn_off = (int64_t)G.ngj * G.C_gu * 2 * G.unit;
  G.expert_bytes = al(G.dn_off + (int64_t)G.ndp * G.C_dn * 2 * G.unit);
  G.total = G.maps_bytes + G.expert_bytes * sp.n_experts;
  return G;
}

size_t packed_total_bytes(const TsbMoeSpec& sp) {
  if (!packable(sp)) return 0;
  return (size_t)pk_geo(sp, pk_maps(sp)).total;
}

// ------------------------------------------------------------------ packing
struct PackArgs {
  const TsbExpert* experts;
  uint8_t* packed;  // start of the expert sections
  const int32_t* gu_j;
  const int32_t* gu_ph;
  const int32_t* dn_h;
  const int32_t* dn_ph;
  PkGeo G;
  int H, I, layout;
  int64_t units_gu, units_per_expert;
};

struct SrcRow {
  const uint8_t* w;  // block stream (null: padding row)
  const uint8_t* s;  // MXFP4 scale bytes
  int64_t row;       // row in that stream
  int64_t nrows;     // rows of that stream
  int K, p;          // row length, Q4_K phase
};

__device__ SrcRow pack_src(const PackArgs& a, const TsbExpert& E, bool down, int grp, int rbsel, int r) {
  SrcRow S{};
  if (down) {
    const int h = a.dn_h[grp * 32 + rbsel * 16 + r];
    S.K = a.I;
    S.p = a.dn_ph[grp];
    if (h < 0) return S;
    S.w = static_cast<const uint8_t*>(E.down);
    S.s = static_cast<const uint8_t*>(E.down_scales);
    S.row = h;
    S.nrows = a.H;
    return S;
  }
  const int j = a.gu_j[grp * 16 + r];
  S.K = a.H;
  S.p = a.gu_ph[grp * 2 + rbsel];
  if (j < 0) return S;
  const bool up = rbsel == 1;
  if (a.layout == TSB_GU_SEPARATE) {
    S.w = static_cast<const uint8_t*>(up ? E.up : E.gate);
    S.s = static_cast<const uint8_t*>(up ? E.up_scales : E.gate_scales);
    S.row = j;
    S.nrows = a.I;
  } else {
    S.w = static_cast<const uint8_t*>(E.gate);
    S.s = static_cast<const uint8_t*>(E.gate_scales);
    S.row = a.layout == TSB_GU_INTERLEAVED ? 2 * (int64_t)j + (up ? 1 : 0) : (up ? (int64_t)a.I : 0) + j;
    S.nrows = 2 * (int64_t)a.I;
  }
  return S;
}

// Q4_K superblock of chunk c of a row (null when past the stream).
__device__ __forceinline__ const uint8_t* q4_block(const SrcRow& S, int c) {
  if (!S.w) return nullptr;
  const int64_t sbi = (S.row * S.K - 32 * S.p) / 256 + c;
  if (sbi < 0 || sbi >= S.nrows * S.K / 256) return nullptr;
  return S.w + sbi * 144;
}
__device__ __forceinline__ uint32_t q4_code(const uint8_t* b, int n, int e) {
  return b ? (b[16 + 32 * (n >> 1) + e] >> (4 * (n & 1))) & 15u : 0u;
}
__device__ __forceinline__ uint32_t mx_byte(const SrcRow& S, int c, int n, int bi) {
  const int blk = 8 * c + n;
  if (!S.w || blk >= S.K / 32) return 0u;
  return S.w[S.row * (S.K / 2) + (int64_t)blk * 16 + bi];
}

// One warp per unit.  Lane L = (g, t) owns sub-blocks t and 4 + t of rows g
// and g + 8: 16 code words W[h][rho][i'] (half h: sub-block 4h + t; row
// rho: g, g + 8; i' = 0..3: elements 8i'..8i'+7).  Q4_K (int8 MMA): byte k
// of the word holds elements 8i'+k (low nibble) and 8i'+4+k (high nibble),
// so W & 0x0F0F0F0F and (W >> 4) & 0x0F0F0F0F are the two u8 A registers.
// MXFP4 (f16 MMA): the word is bytes 4i'..4i'+3 of the source block (low
// nibble first), so the e2m1 conversions give the pairs (e0,e1) .. (e6,e7).  Plane j (16 B per
// lane; h = j / 2, i' in {2(j%2), 2(j%2)+1}) holds W[h][0][i'0],
// W[h][1][i'0], W[h][0][i'1], W[h][1][i'1].
__global__ void __launch_bounds__(256) pk_pack_kernel(const PackArgs a, int64_t nunits) {
  const int64_t unit = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (unit >= nunits) return;
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int64_t e = unit / a.units_per_expert;
  int64_t r = unit % a.units_per_expert;
  const bool down = r >= a.units_gu;
  if (down) r -= a.units_gu;
  const int C = down ? a.G.C_dn : a.G.C_gu;
  const int rbsel = (int)(r & 1);
  const int c = (int)((r >> 1) % C);
  const int grp = (int)((r >> 1) / C);
  const TsbExpert E = a.experts[e];
  uint8_t* dst = a.packed + e * a.G.expert_bytes + (down ? a.G.dn_off : a.G.gu_off) + r * a.G.unit;

  uint32_t w[2][2][4];  // [h][rho][i']
  const SrcRow S0 = pack_src(a, E, down, grp, rbsel, g), S1 = pack_src(a, E, down, grp, rbsel, g + 8);
  if (a.G.q4) {
    const uint8_t* blk[2] = {q4_block(S0, c), q4_block(S1, c)};
    const int sh[8] = {0, 8, 16, 24, 4, 12, 20, 28};
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int rho = 0; rho < 2; ++rho)
#pragma unroll
        for (int ip = 0; ip < 4; ++ip) {
          uint32_t v = 0;
#pragma unroll
          for (int q = 0; q < 8; ++q) v |= q4_code(blk[rho], 4 * h + t, 8 * ip + q) << sh[q];
          w[h][rho][ip] = v;
        }
  } else {
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int rho = 0; rho < 2; ++rho) {
        const SrcRow& S = rho ? S1 : S0;
#pragma unroll
        for (int ip = 0; ip < 4; ++ip)
          w[h][rho][ip] = mx_byte(S, c, 4 * h + t, 4 * ip) | mx_byte(S, c, 4 * h + t, 4 * ip + 1) << 8 |
                          mx_byte(S, c, 4 * h + t, 4 * ip + 2) << 16 | mx_byte(S, c, 4 * h + t, 4 * ip + 3) << 24;
      }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int h = j >> 1, i0 = 2 * (j & 1);
    *reinterpret_cast<uint4*>(dst + a.G.hdr + (32 * j + lane) * 16) =
        make_uint4(w[h][0][i0], w[h][1][i0], w[h][0][i0 + 1], w[h][1][i0 + 1]);
  }

  if (lane < 16) {
    const SrcRow S = pack_src(a, E, down, grp, rbsel, lane);
    if (a.G.q4) {
      const uint8_t* b = q4_block(S, c);
      uint32_t dd = 0, pw[4] = {0, 0, 0, 0};
      if (b) {
        dd = (uint32_t)b[0] | (uint32_t)b[1] << 8 | (uint32_t)b[2] << 16 | (uint32_t)b[3] << 24;
        for (int q = 0; q < 4; ++q) {
          int sa, ma, sb, mb;
          kq_scale_min(b + 4, 2 * q, sa, ma);
          kq_scale_min(b + 4, 2 * q + 1, sb, mb);
          pw[q] = (uint32_t)sa | (uint32_t)sb << 8 | (uint32_t)ma << 16 | (uint32_t)mb << 24;
        }
      }
      *reinterpret_cast<uint32_t*>(dst + 4 * lane) = dd;
      *reinterpret_cast<uint4*>(dst + 64 + 16 * lane) = make_uint4(pw[0], pw[1], pw[2], pw[3]);
    } else {
      uint32_t s[2] = {0, 0};
      if (S.w)
        for (int n = 0; n < 8; ++n) {
          const int blk = 8 * c + n;
          if (blk < S.K / 32) s[n >> 2] |= (uint32_t)S.s[S.row * (S.K / 32) + blk] << (8 * (n & 3));
        }
      *reinterpret_cast<uint2*>(dst + 8 * lane) = make_uint2(s[0], s[1]);
    }
  }
}

int launch_pack(const TsbMoeSpec& sp, const TsbExpert* experts, void* packed, cudaStream_t st) {
  const PkMaps M = pk_maps(sp);
  const PkGeo G = pk_geo(sp, M);
  uint8_t* base = static_cast<uint8_t*>(packed);
  // the row maps: small, copied once from host memory (stream-ordered)
  std::vector<uint8_t> maps((size_t)G.maps_bytes, 0);
  memcpy(maps.data() + G.o_guj, M.gu_j.data(), 4 * M.gu_j.size());
  memcpy(maps.data() + G.o_guph, M.gu_ph.data(), 4 * M.gu_ph.size());
  memcpy(maps.data() + G.o_dnh, M.dn_h.data(), 4 * M.dn_h.size());
  memcpy(maps.data() + G.o_dnph, M.dn_ph.data(), 4 * M.dn_ph.size());
  cudaError_t e = cudaMemcpyAsync(base, maps.data(), maps.size(), cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);  // host vector dies on return
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  PackArgs a{};
  a.experts = experts;
  a.packed = base + G.maps_bytes;
  a.gu_j = reinterpret_cast<const int32_t*>(base + G.o_guj);
  a.gu_ph = reinterpret_cast<const int32_t*>(base + G.o_guph);
  a.dn_h = reinterpret_cast<const int32_t*>(base + G.o_dnh);
  a.dn_ph = reinterpret_cast<const int32_t*>(base + G.o_dnph);
  a.G = G;
  a.H = sp.hidden;
  a.I = sp.inter;
  a.layout = sp.gate_up_layout;
  a.units_gu = (int64_t)G.ngj * G.C_gu * 2;
  a.units_per_expert = a.units_gu + (int64_t)G.ndp * G.C_dn * 2;
  const int64_t n = a.units_per_expert * sp.n_experts;
  pk_pack_kernel<<<(unsigned)((n + 7) / 8), 256, 0, st>>>(a, n);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  return TSB_OK;
}

// ------------------------------------------------------------------ decode
// Phase timing (development builds only, -DTSB_PK_TIMING=1): per-CTA
// globaltimer stamps at the phase boundaries and per-warp cycle counts of
// waiting, computing, issuing copies and epilogues, read back with
// tsb_pk_timing_read.  Compiled out of the default build.
#ifndef TSB_PK_TIMING
#define TSB_PK_TIMING 0
#endif
#if TSB_PK_TIMING
#define PK_T(...) __VA_ARGS__
__device__ unsigned long long g_pk_trace[160 * 16];
__device__ unsigned long long g_pk_wtrace[160 * 16 * 8];
#else
#define PK_T(...)
#endif
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

struct PkArgs {
  const uint8_t* packed;  // expert sections
  const int32_t* gu_j;
  const int32_t* dn_h;
  const int32_t* gu_ph;
  const int32_t* dn_ph;
  int64_t gu_off, dn_off, expert_bytes;
  int H, I, E, top_k, ngj, ndp, C_gu, C_dn;
  int Q_gu, Q_dn;          // chunks of one warp's range (gate/up, down)
  int N_gu, N_dn;          // chunks of the whole layer call (gate/up, down)
  int slots_gu, slots_dn;  // partial-sum slots per group (workspace stride)
  int nsb_h;  // padded sub-blocks of the x image
  const uint16_t* x;
  const uint16_t* router_w;
  const float* router_b;
  int32_t* ids;
  float* wts;
  const TsbExpert* experts;
  unsigned* cnt_gu;  // [top_k * ngj]
  unsigned* cnt_dn;  // [ndp]
  unsigned* sync;    // [1] CTAs finished
  float* dact;       // [top_k, I] activations; bit pattern 0 (+0.0) = not yet written
  float* part_gu;    // [top_k * ngj, slots_gu, 32]
  float* part_dn;    // [ndp, slots_dn, 32]
  void* out;
  int out_f32, act_kind;
  float limit, alpha;
  int* err;
};

// Slot waits use mbarrier.try_wait: a waiting warp is suspended in hardware
// until the phase completes (or a time limit passes), so it takes no issue
// slots from the warps that compute.  Bounded: after kWaitPolls polls of up
// to kWaitNs each (seconds in all) it records kDevWaitTimeout and gives up.
constexpr uint32_t kSpinPolls = 1u << 26;  // polls of the device-wide counters (with a short sleep)
constexpr uint32_t kWaitPolls = 1u << 16, kWaitNs = 100000;
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err) {
  bool ok = false;
  for (uint32_t i = 0; i < kWaitPolls && !ok; ++i) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(r)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kWaitNs)
        : "memory");
    ok = r != 0;
  }
  if (!ok && err) atomicExch(err, kDevWaitTimeout);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void mma_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                      uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}
__device__ __forceinline__ void mma_acc(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

// L2 eviction policies: the expert weights are streamed once per token and go
// in as evict-first, so the small data every token re-reads (router
// weights, the row maps, the activations and partial sums) stays in L2.
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint4 ldg_hint(const uint4* p, uint64_t pol) {
  uint4 v;
  asm volatile("ld.global.nc.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(pol));
  return v;
}
// 8 floats (32-byte aligned) with relaxed GPU-scope loads: re-read from L2
// on every call, never served by a stale L1 line.
__device__ __forceinline__ void ld_relaxed_f32x8(const float* p, float (&v)[8]) {
  asm volatile("ld.relaxed.gpu.global.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]) : "l"(p) : "memory");
  asm volatile("ld.relaxed.gpu.global.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7]) : "l"(p + 4) : "memory");
}
__device__ __forceinline__ int ldg_hint_i32(const int32_t* p, uint64_t pol) {
  int v;
  asm volatile("ld.global.nc.L2::cache_hint.b32 %0, [%1], %2;" : "=r"(v) : "l"(p), "l"(pol));
  return v;
}
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
__device__ __forceinline__ void prefetch_l2_hint(const void* p, uint32_t bytes, uint64_t pol) {
  asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;" ::"l"(p), "r"(bytes), "l"(pol)
               : "memory");
}
__device__ __forceinline__ uint32_t u4c(const uint4& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Four f16x2 A registers from one code word (see pk_pack_kernel): element
// pairs (e0,e1), (e2,e3), (e4,e5), (e6,e7).
template <bool Q4>
__device__ __forceinline__ void decode_word(uint32_t w, uint32_t m64, uint32_t (&r)[4]) {
  if (Q4) {
    // every code decodes to 64 + q (0x5400 | q << 4): nibble pairs are moved
    // to bits [7:4] / [23:20] of each half first
    r[0] = ((w << 4) & 0x00F000F0u) | m64;
    r[1] = (w & 0x00F000F0u) | m64;
    r[2] = ((w >> 4) & 0x00F000F0u) | m64;
    r[3] = ((w >> 8) & 0x00F000F0u) | m64;
  } else {
    // the word unpacked into its four bytes in PTX: the conversions read the
    // bytes in place (a shift and a mask per byte otherwise)
    asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %4;\n cvt.rn.f16x2.e2m1x2 %0, b0;\n"
        " cvt.rn.f16x2.e2m1x2 %1, b1;\n cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n}"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
        : "r"(w));
  }
}

// The four MMAs of plane j of one unit.  q: the lane's plane word group
// (rows g, g+8 x two element octets); b0, b1: the B registers of the four
// MMAs, (b01, b23) adjacent.  MMA m covers elements 4m..4m+3 of the lane's
// sub-block: a01 (row g) / a23 (row g+8) elements 4m, 4m+1; a45 / a67
// elements 4m+2, 4m+3.
template <bool Q4, bool FIRST>
__device__ __forceinline__ void plane_mma(const uint4& q, const uint4& b0, const uint4& b1, uint32_t m64,
                                          float (&d)[4]) {
  uint32_t r0[4], r1[4], r2[4], r3[4];
  decode_word<Q4>(q.x, m64, r0);  // row g,   elements 8i'0 .. 8i'0+7
  decode_word<Q4>(q.y, m64, r1);  // row g+8
  decode_word<Q4>(q.z, m64, r2);  // row g,   elements 8i'1 .. 8i'1+7
  decode_word<Q4>(q.w, m64, r3);  // row g+8
  if (FIRST)
    mma_z(d, r0[0], r1[0], r0[1], r1[1], b0.x, b0.y);
  else
    mma_acc(d, r0[0], r1[0], r0[1], r1[1], b0.x, b0.y);
  mma_acc(d, r0[2], r1[2], r0[3], r1[3], b0.z, b0.w);
  mma_acc(d, r2[0], r3[0], r2[1], r3[1], b1.x, b1.y);
  mma_acc(d, r2[2], r3[2], r2[3], r3[3], b1.z, b1.w);
}

// Scale fold of one unit: lane (g, t) holds rows g, g+8 x sub-blocks 2t,
// 2t+1 of the chunk.  Q4_K (codes decoded as 64 + q):
//   row += d * sum_n sc_n * (D_n - 64 X_n) - dmin * sum_n m_n X_n
// MXFP4: row += sum_n 2^(e_n - 127) * D_n.
template <bool Q4>
__device__ __forceinline__ void unit_fold(const uint8_t* u, const float (&d)[4], float xa, float xb, int g, int t,
                                          float& acc0, float& acc1) {
  // MXFP4: xa, xb are the x scales 2^-e of the lane's two sub-blocks
  if (Q4) {
#pragma unroll
    for (int rho = 0; rho < 2; ++rho) {
      const int row = g + 8 * rho;
      const uint32_t dd = *reinterpret_cast<const uint32_t*>(u + 4 * row);
      const uint32_t sm = *reinterpret_cast<const uint32_t*>(u + 64 + 16 * row + 4 * t);
      const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&dd));
      const float ya = fmaf(-64.f, xa, d[2 * rho]), yb = fmaf(-64.f, xb, d[2 * rho + 1]);
      const float uu = fmaf((float)((sm >> 8) & 255u), yb, (float)(sm & 255u) * ya);
      const float vv = fmaf((float)(sm >> 24), xb, (float)((sm >> 16) & 255u) * xa);
      float acc = rho ? acc1 : acc0;
      acc = fmaf(dm.x, uu, acc);
      acc = fmaf(-dm.y, vv, acc);
      if (rho) acc1 = acc; else acc0 = acc;
    }
  } else {
#pragma unroll
    for (int rho = 0; rho < 2; ++rho) {
      const int row = g + 8 * rho;
      const uint32_t e2 = *reinterpret_cast<const uint16_t*>(u + 8 * row + 2 * t);
      const uint32_t ea = e2 & 255u, eb = e2 >> 8;
      const float fa = __uint_as_float(ea ? ea << 23 : 0x00400000u) * xa;
      const float fb = __uint_as_float(eb ? eb << 23 : 0x00400000u) * xb;
      float acc = rho ? acc1 : acc0;
      acc = fmaf(fa, d[2 * rho], acc);
      acc = fmaf(fb, d[2 * rho + 1], acc);
      if (rho) acc1 = acc; else acc0 = acc;
    }
  }
}

// One chunk (two units, A and B, of the same 256 columns).  B operands: lanes
// g == t hold sub-block 8c - p + t for the half-0 MMAs, lanes g == t + 4
// sub-block 8c - p + 4 + t for the half-1 MMAs (element pairs 2m, 2m+1 of MMA
// m as one (b01, b23) register pair); every other lane reads zeros.  Half 0
// fills accumulator columns 0-3, half 1 columns 4-7, so the lane's columns
// 2t, 2t+1 are sub-blocks 2t, 2t+1.  SHARED: both units have the same phase
// (one set of B loads).
template <bool Q4, bool SHARED>
__device__ __forceinline__ void chunk_mma(const uint8_t* uA, const uint8_t* uB, const uint8_t* srcA0,
                                          const uint8_t* srcA1, const uint8_t* srcB0, const uint8_t* srcB1,
                                          size_t strA0, size_t strA1, size_t strB0, size_t strB1, uint32_t m64,
                                          int lane, float (&dA)[4], float (&dB)[4]) {
  float eA[4], eB[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int h = j >> 1, G = 2 * (j & 1);
    const uint8_t* sa = h ? srcA1 : srcA0;
    const size_t za = h ? strA1 : strA0;
    const uint4 qa = lds128(uA + (32 * j + lane) * 16);
    const uint4 qb = lds128(uB + (32 * j + lane) * 16);
    const uint4 ba0 = lds128(sa + G * za), ba1 = lds128(sa + (G + 1) * za);
    uint4 bb0 = ba0, bb1 = ba1;
    if (!SHARED) {
      const uint8_t* sb = h ? srcB1 : srcB0;
      const size_t zb = h ? strB1 : strB0;
      bb0 = lds128(sb + G * zb);
      bb1 = lds128(sb + (G + 1) * zb);
    }
    if (j == 0) {
      plane_mma<Q4, true>(qa, ba0, ba1, m64, dA);
      plane_mma<Q4, true>(qb, bb0, bb1, m64, dB);
    } else if (j == 2) {
      plane_mma<Q4, true>(qa, ba0, ba1, m64, eA);
      plane_mma<Q4, true>(qb, bb0, bb1, m64, eB);
    } else if (j == 1) {
      plane_mma<Q4, false>(qa, ba0, ba1, m64, dA);
      plane_mma<Q4, false>(qb, bb0, bb1, m64, dB);
    } else {
      plane_mma<Q4, false>(qa, ba0, ba1, m64, eA);
      plane_mma<Q4, false>(qb, bb0, bb1, m64, eB);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    dA[i] += eA[i];
    dB[i] += eB[i];
  }
}

// ---- Q4_K on the int8 tensor path (mma.m16n8k32, u8 codes x s8 x bytes)
__device__ __forceinline__ void imma(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                     uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One chunk (two units) of Q4_K: MMA (h, i) covers elements 8i..8i+7 of the
// lane's sub-block 4h + t (k-quad t: 8i..8i+3, k-quad t+4: 8i+4..8i+7).  The
// 14-bit x of a sub-block is split x = 256*hi + lo, both signed bytes; in
// MMA (h, i) column 4h + t carries the hi bytes of sub-block 4h + t and
// column 4(1-h) + t its lo bytes (the B operand of lanes g == t and g == t+4;
// every other lane supplies zeros), so one MMA yields both partial dots and a
// unit takes 8 MMAs.  bX0 / bX1: this lane's B source for half 0 / 1 (its
// plane 0 for the hi or lo pair), zX the plane stride (0 for a zero lane);
// shared: unit B reads unit A's x (both row blocks at the same phase).
// Result per unit and lane: c[r] = 256*hi + lo dot of rows g (r < 2) / g+8,
// sub-blocks 2t, 2t+1 (r & 1); exact in int32.
__device__ __forceinline__ void chunk_imma(const uint8_t* uA, const uint8_t* uB, const uint8_t* bA0,
                                           const uint8_t* bA1, const uint8_t* bB0, const uint8_t* bB1, size_t zA,
                                           size_t zB, bool shared, int lane, int (&cA)[4], int (&cB)[4]) {
  int dA[2][4], dB[2][4];
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int i = 0; i < 4; ++i) dA[h][i] = dB[h][i] = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int h = j >> 1, G = j & 1;  // plane j: MMAs (h, 2G), (h, 2G + 1)
    const uint4 qa = lds128(uA + (32 * j + lane) * 16);
    const uint4 qb = lds128(uB + (32 * j + lane) * 16);
    const uint4 xa = lds128((h ? bA1 : bA0) + G * zA);
    const uint4 xb = shared ? xa : lds128((h ? bB1 : bB0) + G * zB);
    // unit A: words x (row g) / y (row g+8) -> MMA 2G, z / w -> MMA 2G+1
    imma(dA[h], qa.x & 0x0F0F0F0Fu, qa.y & 0x0F0F0F0Fu, (qa.x >> 4) & 0x0F0F0F0Fu, (qa.y >> 4) & 0x0F0F0F0Fu, xa.x,
         xa.y);
    imma(dA[h], qa.z & 0x0F0F0F0Fu, qa.w & 0x0F0F0F0Fu, (qa.z >> 4) & 0x0F0F0F0Fu, (qa.w >> 4) & 0x0F0F0F0Fu, xa.z,
         xa.w);
    imma(dB[h], qb.x & 0x0F0F0F0Fu, qb.y & 0x0F0F0F0Fu, (qb.x >> 4) & 0x0F0F0F0Fu, (qb.y >> 4) & 0x0F0F0F0Fu, xb.x,
         xb.y);
    imma(dB[h], qb.z & 0x0F0F0F0Fu, qb.w & 0x0F0F0F0Fu, (qb.z >> 4) & 0x0F0F0F0Fu, (qb.w >> 4) & 0x0F0F0F0Fu, xb.z,
         xb.w);
  }
  // Lane t < 2 holds the hi dots of sub-blocks 2t, 2t+1 in its half-0
  // columns and the lo dots of sub-blocks 4+2t, 5+2t in its half-1 columns;
  // lane t ^ 2 the reverse.  Swap the lo halves across the pair.
  const bool lowq = (lane & 3) < 2;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int ka = lowq ? dA[0][i] : dA[1][i], sa = lowq ? dA[1][i] : dA[0][i];
    const int kb = lowq ? dB[0][i] : dB[1][i], sb = lowq ? dB[1][i] : dB[0][i];
    cA[i] = ka * 256 + __shfl_xor_sync(0xffffffffu, sa, 2);
    cB[i] = kb * 256 + __shfl_xor_sync(0xffffffffu, sb, 2);
  }
}

// Q4_K fold of one unit: sub-block n's dot product is
//   2^-e_n * (d * sc_n * c_n) - dmin * m_n * X_n,  c_n = 256*hi_n + lo_n
// with X_n = 2^-e_n * sum x_int (the image's float2 per sub-block).
__device__ __forceinline__ void fold_q4(const uint8_t* u, const int (&c)[4], float2 xa, float2 xb, int g, int t,
                                        float& acc0, float& acc1) {
#pragma unroll
  for (int rho = 0; rho < 2; ++rho) {
    const int row = g + 8 * rho;
    const uint32_t dd = *reinterpret_cast<const uint32_t*>(u + 4 * row);
    const uint32_t sm = *reinterpret_cast<const uint32_t*>(u + 64 + 16 * row + 4 * t);
    const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&dd));
    const float fa = (float)c[2 * rho] * xa.x;
    const float fb = (float)c[2 * rho + 1] * xb.x;
    const float uu = fmaf((float)((sm >> 8) & 255u), fb, (float)(sm & 255u) * fa);
    const float vv = fmaf((float)(sm >> 24), xb.y, (float)((sm >> 16) & 255u) * xa.y);
    float acc = rho ? acc1 : acc0;
    acc = fmaf(dm.x, uu, acc);
    acc = fmaf(-dm.y, vv, acc);
    if (rho) acc1 = acc; else acc0 = acc;
  }
}

// Shared memory: per-warp rings, then the B images and their sub-block sums.
// Image of vector v: plane j (MMAs 4j..4j+3) of padded sub-block s at
// img + v*nsb*64 + (j*nsb + s)*16; X at X + v*nsb + s.  Padded sub-block s
// is row-local sub-block s - kPadL.
__host__ __device__ inline size_t pk_ring_bytes(int unit) { return (size_t)kPkWarps * kSlots * 2 * unit; }
__host__ __device__ inline size_t pk_img_bytes(int nvec, int nsb) { return (size_t)nvec * nsb * 64; }
__host__ __device__ inline size_t pk_x_bytes(int nvec, int nsb) { return ((size_t)nvec * nsb * 8 + 15) & ~size_t(15); }
// Down-phase images: each warp stages the 8 activation sub-blocks of one
// down chunk into a small image of its own (kMiniNsb padded sub-blocks, the
// 8 real ones at [kPadL, kPadL + 8)), two buffers per warp.
constexpr int kMiniNsb = kPadL + 8, kMiniBufs = 2;
__host__ __device__ inline size_t pk_mini_bytes() { return pk_img_bytes(1, kMiniNsb) + pk_x_bytes(1, kMiniNsb); }
__host__ __device__ inline size_t pk_smem(int unit, int nsb_h) {
  return pk_ring_bytes(unit) + pk_img_bytes(1, nsb_h) + pk_x_bytes(1, nsb_h) + 64 +
         (size_t)kPkWarps * kMiniBufs * pk_mini_bytes();
}

// Thread-block cluster helpers (distributed shared memory).
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
// Store v into the same shared-memory location of cluster CTA `rank`.
__device__ __forceinline__ void st_cluster(float* local, uint32_t rank, float v) {
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(local)), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ra), "f"(v) : "memory");
}
// Every thread of every CTA of the cluster: prior (remote) shared-memory
// stores are visible to all of them afterwards.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Split form used at kernel start: every CTA arrives once it is running; a
// CTA waits before its first store into another CTA's shared memory.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

// Router logits (tinyserve/_model_hooks.py:466-473), split over the CTAs of
// a thread-block cluster: CTA r of n computes experts r, r + n, ... (one warp
// each: bf16 x . bf16 W[e] in fp32, + bias, rounded to bf16 as the
// reference's bf16 Linear returns them) into its own s_logit, then, once
// every CTA of the cluster is running (the arrive at kernel start), copies
// them into the s_logit of the other CTAs; a cluster barrier follows.
// Called by every thread of the CTA.
__device__ void pk_logits(const PkArgs& a, float* s_logit, int warp, int lane) {
  const int H = a.H, n8 = H / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(a.x);
  const int r = (int)cluster_rank(), n = (int)cluster_size();
  const uint64_t keep = policy_evict_last();
  constexpr int kU = 12;
  for (int e = r + n * warp; e < a.E; e += n * kPkWarps) {
    const uint4* wr = reinterpret_cast<const uint4*>(a.router_w + (int64_t)e * H);
    float acc4[4] = {0.f, 0.f, 0.f, 0.f};  // four independent FMA chains
    for (int base = lane; base < n8; base += 32 * kU) {
      uint4 xv[kU], wv[kU];
#pragma unroll
      for (int j = 0; j < kU; ++j) {
        const int i = base + 32 * j;
        xv[j] = i < n8 ? __ldg(xr + i) : make_uint4(0, 0, 0, 0);
        wv[j] = i < n8 ? ldg_hint(wr + i, keep) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int j = 0; j < kU; ++j) {
        const uint32_t av[4] = {xv[j].x, xv[j].y, xv[j].z, xv[j].w}, bv[4] = {wv[j].x, wv[j].y, wv[j].z, wv[j].w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc4[q] = fmaf(__uint_as_float(av[q] << 16), __uint_as_float(bv[q] << 16), acc4[q]);
          acc4[q] = fmaf(__uint_as_float(av[q] & 0xFFFF0000u), __uint_as_float(bv[q] & 0xFFFF0000u), acc4[q]);
        }
      }
    }
    float acc = (acc4[0] + acc4[1]) + (acc4[2] + acc4[3]);
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) s_logit[e] = bf16_bits_to_f32(f32_to_bf16_bits(a.router_b ? acc + a.router_b[e] : acc));
  }
  __syncwarp();
  PK_T(if (threadIdx.x == 0 && blockIdx.x < 160) g_pk_trace[blockIdx.x * 16 + 8] = gtimer();)
  cluster_wait();
  PK_T(if (threadIdx.x == 0 && blockIdx.x < 160) g_pk_trace[blockIdx.x * 16 + 9] = gtimer();)
  for (int e = r + n * warp; e < a.E; e += n * kPkWarps)
    if (lane < n && lane != r) st_cluster(s_logit + e, (uint32_t)lane, s_logit[e]);
}

// Top-k of the logits in s_logit (ties -> lower id, NaN lowest) and softmax
// over the k selected logits; warp 0 of every CTA reaches the same result,
// CTA 0 publishes ids / weights.
// Order-preserving map of a float to an unsigned key (NaN lowest).
__device__ __forceinline__ uint32_t sort_key(float f) {
  if (f != f) return 0u;
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ uint32_t redux_max(uint32_t v) {
  uint32_t r;
  asm volatile("redux.sync.max.u32 %0, %1, 0xffffffff;" : "=r"(r) : "r"(v));
  return r;
}
__device__ __forceinline__ uint32_t redux_min(uint32_t v) {
  uint32_t r;
  asm volatile("redux.sync.min.u32 %0, %1, 0xffffffff;" : "=r"(r) : "r"(v));
  return r;
}

__device__ void pk_select(const PkArgs& a, const float* s_logit, int* s_e, float* s_w, int lane) {
  // Each pick: every lane's best remaining (key, lowest id) over its experts
  // lane, lane + 32, ...; the warp's largest key (redux.max), then the lowest
  // id holding it (redux.min): ties go to the lower id, NaN ranks lowest.
  uint32_t taken = 0;  // bit j: expert lane + 32*j already selected (E <= 1024)
  float sel[8];
  int sid[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    if (k >= a.top_k) break;
    uint32_t bk = 0u, bid = 0xFFFFFFFFu;
    for (int j = 0; lane + 32 * j < a.E; ++j) {
      if ((taken >> j) & 1u) continue;
      const uint32_t key = sort_key(s_logit[lane + 32 * j]);
      if (bid == 0xFFFFFFFFu || key > bk) { bk = key; bid = lane + 32 * j; }
    }
    const uint32_t mk = redux_max(bid == 0xFFFFFFFFu ? 0u : bk);
    const uint32_t id = redux_min(bid != 0xFFFFFFFFu && bk == mk ? bid : 0xFFFFFFFFu);
    sid[k] = (int)id;
    sel[k] = id < (uint32_t)a.E ? s_logit[id] : -INFINITY;
    if (id < (uint32_t)a.E && (int)(id & 31) == lane) taken |= 1u << (id >> 5);
  }
  if (lane == 0) {
    const float mx = sel[0];
    float ex[8], den = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (k < a.top_k) {
        ex[k] = __expf((sel[k] != sel[k] ? -INFINITY : sel[k]) - mx);
        den += ex[k];
      }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (k >= a.top_k) break;
      const bool ok = (unsigned)sid[k] < (unsigned)a.E;
      s_e[k] = ok ? sid[k] : -1;
      s_w[k] = ex[k] / den;
      if (blockIdx.x == 0) {
        a.ids[k] = sid[k];
        a.wts[k] = ex[k] / den;
      }
    }
  }
}

// Power-of-two scale putting max |v| in [2^14, 2^15) (exact in fp32).
__device__ __forceinline__ void pow2_scale(float m, float& scale, float& inv) {
  const int ex = (int)((__float_as_uint(m) >> 23) & 255u);
  int sx = (m > 0.f && ex != 255) ? 14 - (ex - 127) : 0;
  sx = max(-126, min(126, sx));
  scale = __uint_as_float((uint32_t)(sx + 127) << 23);
  inv = __uint_as_float((uint32_t)(127 - sx) << 23);
}

// B image of one vector of length K (multiple of 32), 64 bytes per 32-element
// sub-block in four 16-byte groups; group G of padded sub-block s sits at
// img + (G*nsb + s)*16, the sub-block's float2 (x scale, scaled sum) at X[s].
//   MXFP4 (f16 MMA): group G = element pairs 4G..4G+3 as f16x2, x scaled by
//     a power of two per sub-block (max |x| in [2^14, 2^15)); X[s] = (2^-e, 0).
//   Q4_K (int8 MMA): x_int = rint(x * 2^e) with e per sub-block (max |x_int|
//     in [2^13, 2^14)), split x_int = 256*hi + lo (both signed bytes):
//     groups 0, 1 = hi bytes of elements 0-15, 16-31, groups 2, 3 = lo bytes;
//     X[s] = (2^-e, 2^-e * sum x_int).
// stage_group writes the 8 elements 8q..8q+7 of sub-block sb; the four groups
// of a sub-block sit on four consecutive lanes (two shuffles combine them).
template <bool Q4>
__device__ __forceinline__ void stage_group(uint8_t* img, float2* X, int nsb, int sb, int q, const float (&v)[8],
                                            bool valid) {
  const int sp = sb + kPadL;
  if (Q4) {
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) m = fmaxf(m, valid ? fabsf(v[i]) : 0.f);
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    const int ex = (int)((__float_as_uint(m) >> 23) & 255u);
    int sx = (m > 0.f && ex != 255) ? 13 - (ex - 127) : 0;
    sx = max(-126, min(126, sx));
    const float sc = __uint_as_float((uint32_t)(sx + 127) << 23);
    uint32_t hi[2] = {0, 0}, lo[2] = {0, 0};
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int xi = valid ? __float2int_rn(v[i] * sc) : 0;
      sum += xi;
      hi[i >> 2] |= (uint32_t)(((xi + 128) >> 8) & 255) << (8 * (i & 3));  // x = 256*hi + lo, lo in [-128, 128)
      lo[i >> 2] |= (uint32_t)(xi & 255) << (8 * (i & 3));
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if (!valid) return;
    *reinterpret_cast<uint2*>(img + ((size_t)(q >> 1) * nsb + sp) * 16 + 8 * (q & 1)) = make_uint2(hi[0], hi[1]);
    *reinterpret_cast<uint2*>(img + ((size_t)(2 + (q >> 1)) * nsb + sp) * 16 + 8 * (q & 1)) = make_uint2(lo[0], lo[1]);
    const float inv = __uint_as_float((uint32_t)(127 - sx) << 23);
    if (q == 0) X[sp] = make_float2(inv, (float)sum * inv);
  } else {
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) m = fmaxf(m, valid ? fabsf(v[i]) : 0.f);
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    float sc, inv;
    pow2_scale(m, sc, inv);
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half2 h = __floats2half2_rn(v[2 * i] * sc, v[2 * i + 1] * sc);
      w[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    if (!valid) return;
    *reinterpret_cast<uint4*>(img + ((size_t)q * nsb + sp) * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    if (q == 0) X[sp] = make_float2(inv, 0.f);
  }
}

__device__ __forceinline__ void zero_pads(uint8_t* img, float2* X, int nsb, int K) {
  const int real = K / 32;
  constexpr int kPad = kPadL + kPadR;
  // 4 planes x (kPadL + kPadR) padded sub-blocks of 16 bytes, plus their sums
  for (int i = threadIdx.x; i < 4 * kPad; i += blockDim.x) {
    const int j = i / kPad, s = i % kPad;
    const int sp = s < kPadL ? s : real + s;  // [0, kPadL) and [kPadL + real, nsb)
    *reinterpret_cast<uint4*>(img + ((size_t)j * nsb + sp) * 16) = make_uint4(0, 0, 0, 0);
    if (j == 0) X[sp] = make_float2(0.f, 0.f);
  }
}

// sum_{s < S} Q[32 s + lane] in order, with up to 8 loads in flight.
__device__ __forceinline__ float sum_parts(const float* Q, int S, int lane) {
  float sum = 0.f;
  for (int s0 = 0; s0 < S; s0 += 8) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = s0 + i < S ? __ldcg(Q + 32 * (s0 + i) + lane) : 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) sum += v[i];
  }
  return sum;
}

template <int F>
__global__ void __launch_bounds__(kPkThreads, 1) pk_layer_kernel(const PkArgs a) {
  constexpr bool Q4 = F == FMT_Q4_K;
  constexpr int UNIT = Q4 ? kQ4Unit : kMxUnit, HDR = Q4 ? kQ4Hdr : kMxHdr;
  extern __shared__ uint4 smem4[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(smem4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  uint8_t* ring = sm + (size_t)warp * kSlots * 2 * UNIT;
  uint8_t* img = sm + pk_ring_bytes(UNIT);  // image of x
  float2* Xs = reinterpret_cast<float2*>(img + pk_img_bytes(1, a.nsb_h));
  uint8_t* zero = reinterpret_cast<uint8_t*>(Xs) + pk_x_bytes(1, a.nsb_h);  // 16-byte aligned
  uint8_t* mini = zero + 64 + (size_t)warp * kMiniBufs * pk_mini_bytes();  // this warp's down images

  __shared__ float s_logit[1024];
  __shared__ int s_e[8];
  __shared__ float s_w[8];
  __shared__ const float* s_bias[3][8];  // gate, up, down bias of each slot's expert
  __shared__ uint64_t s_bar[kPkWarps][kSlots];
  __shared__ int s_last;  // this CTA is the last to finish
  uint64_t* bar = s_bar[warp];
  auto stamp = [&](int i) {
    PK_T(if (threadIdx.x == 0 && blockIdx.x < 160) g_pk_trace[blockIdx.x * 16 + i] = gtimer();)
    (void)i;
  };
  stamp(0);
  PK_T(if (threadIdx.x == 0 && blockIdx.x == 0) g_pk_trace[15] = gridDim.x;)
  if (threadIdx.x < 16) reinterpret_cast<uint32_t*>(zero)[threadIdx.x] = 0u;
  if (lane < kSlots) mbar_init(&bar[lane], 1);
  fence_barrier_init();
  if (a.router_w) cluster_arrive_relaxed();
  // Programmatic dependent launch: the next launch on the stream may start
  // its CTAs (and this prologue) as SMs free up; everything above touches
  // only shared memory.  Before the first global read of data an earlier
  // launch may write (x, ids, the workspace words), wait for that launch to
  // complete.  Without a programmatic predecessor the wait returns at once.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // ---- router logits, split over the cluster (ids given: validated below)
  if (a.router_w) pk_logits(a, s_logit, warp, lane);

  // ---- B image of x (one vector), its scale and sub-block sums, while the
  // other CTAs' logits arrive.  Thread i owns 8-element groups i + 512u.
  {
    constexpr int kXR = 2048 / kPkThreads;  // H <= 16384: at most 2048 groups
    const int ng = a.H / 8;
    uint4 xv[kXR];
#pragma unroll
    for (int u = 0; u < kXR; ++u) {
      const int q = threadIdx.x + u * kPkThreads;
      xv[u] = q < ng ? __ldg(reinterpret_cast<const uint4*>(a.x) + q) : make_uint4(0, 0, 0, 0);
    }
    zero_pads(img, Xs, a.nsb_h, a.H);
#pragma unroll
    for (int u = 0; u < kXR; ++u) {
      const int q0 = threadIdx.x - lane + u * kPkThreads;
      if (q0 >= ng) break;  // warp-uniform
      const int q = q0 + lane;
      const uint32_t wv[4] = {xv[u].x, xv[u].y, xv[u].z, xv[u].w};
      float v[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(wv[i] << 16);
        v[2 * i + 1] = __uint_as_float(wv[i] & 0xFFFF0000u);
      }
      stage_group<Q4>(img, Xs, a.nsb_h, q >> 2, q & 3, v, q < ng);
    }
  }

  // ---- routing: every CTA of the cluster has written its logits into all
  // of them; then top-k in each CTA
  if (a.router_w) {
    PK_T(if (threadIdx.x == 0 && blockIdx.x < 160) g_pk_trace[blockIdx.x * 16 + 10] = gtimer();)
    cluster_sync_all();
    PK_T(if (threadIdx.x == 0 && blockIdx.x < 160) g_pk_trace[blockIdx.x * 16 + 11] = gtimer();)
    if (warp == 0) pk_select(a, s_logit, s_e, s_w, lane);
    PK_T(if (threadIdx.x == 0 && blockIdx.x < 160) g_pk_trace[blockIdx.x * 16 + 12] = gtimer();)
  } else if (threadIdx.x < a.top_k) {
    const int e = a.ids[threadIdx.x];
    const bool ok = (unsigned)e < (unsigned)a.E;
    if (!ok && e >= 0 && blockIdx.x == 0 && a.err) atomicExch(a.err, kDevBadPlan);  // negative: skipped slot
    s_e[threadIdx.x] = ok ? e : -1;
    s_w[threadIdx.x] = a.wts[threadIdx.x];
  }
  __syncthreads();
  PK_T(if (threadIdx.x == 0 && blockIdx.x < 160) g_pk_trace[blockIdx.x * 16 + 13] = gtimer();)

  stamp(1);
  // ---- work split.  The chunks of a phase form one flat list: gate/up
  // chunk i is chunk i % C_gu of j-group (i / C_gu) % ngj of slot
  // i / (C_gu * ngj); down chunk i is chunk r % C_dn of slot r / C_dn of
  // down group i / (top_k * C_dn), r = i % (top_k * C_dn).  Warp gw owns the
  // contiguous range [gw * Q, (gw + 1) * Q) of each list, so no warp streams
  // more than Q chunks.  A group (a gate/up j-group of one slot, or a down
  // group over all slots) is a contiguous run of Cg chunks; the warps whose
  // ranges meet it each publish one partial sum into slot (warp - first
  // warp), and the last to arrive combines them in slot order.
  const int gw = blockIdx.x * kPkWarps + warp;
  const int Cg_gu = a.C_gu, Cg_dn = a.top_k * a.C_dn;
  const int r0_gu = min(a.N_gu, gw * a.Q_gu), r1_gu = min(a.N_gu, r0_gu + a.Q_gu);
  const int r0_dn = min(a.N_dn, gw * a.Q_dn), r1_dn = min(a.N_dn, r0_dn + a.Q_dn);
  // first byte of a chunk (nullptr: the slot is skipped)
  auto chunk_ptr = [&](int down, int i) -> const uint8_t* {
    int k, grp, c;
    if (!down) {
      const int G = i / Cg_gu;
      c = i - G * Cg_gu;
      k = G / a.ngj;
      grp = G - k * a.ngj;
    } else {
      grp = i / Cg_dn;
      const int r = i - grp * Cg_dn;
      k = r / a.C_dn;
      c = r - k * a.C_dn;
    }
    const int e = s_e[k];
    if (e < 0) return nullptr;
    return a.packed + (int64_t)e * a.expert_bytes + (down ? a.dn_off : a.gu_off) +
           ((int64_t)grp * (down ? a.C_dn : a.C_gu) + c) * 2 * UNIT;
  };
  const uint64_t stream_pol = policy_evict_first();
  // issue cursor, running ahead of the consumer through the warp's gate/up
  // range, then its down range
  uint32_t issued = 0, consumed = 0;
  int it_ph = 0, it_i = r0_gu, it_e = r1_gu;
  auto issue_next = [&]() {
    for (;;) {
      if (it_i >= it_e) {
        if (it_ph == 1) return;
        it_ph = 1;
        it_i = r0_dn;
        it_e = r1_dn;
        continue;
      }
      const uint8_t* p = chunk_ptr(it_ph, it_i++);
      if (!p) continue;
      // one chunk: its two units are adjacent in the packed layout.  Lane 31
      // issues every bulk copy; lane 0 does the fences and release atomics,
      // so those never wait behind this warp's copies.
      uint64_t* b = &bar[issued % kSlots];
      if (lane == kCopyLane) {
        mbar_arrive_expect_tx(b, 2 * UNIT);
        bulk_g2s_hint(ring + (issued % kSlots) * 2 * UNIT, p, 2 * UNIT, b, stream_pol);
      }
      ++issued;
      return;
    }
  };
#pragma unroll
  for (int i = 0; i < kSlots; ++i) issue_next();
  // bias pointers of the chosen experts (read by the epilogues only; visible
  // to them through the barriers that precede every epilogue)
  if (threadIdx.x < a.top_k) {
    const int e = s_e[threadIdx.x];
    const TsbExpert* E = a.experts + (e < 0 ? 0 : e);
    s_bias[0][threadIdx.x] = e < 0 ? nullptr : E->gate_bias;
    s_bias[1][threadIdx.x] = e < 0 ? nullptr : E->up_bias;
    s_bias[2][threadIdx.x] = e < 0 ? nullptr : E->down_bias;
  }
  // Down chunks beyond what the ring holds: into L2 while gate/up streams.
  // The ring requests the warp's first kSlots down chunks itself as its last
  // gate/up chunks are consumed.  (Prefetching those, or the gate/up chunks
  // past the ring, measured slower: the extra requests delay the ring's.)
  if (lane == kCopyLane) {
    int skip = kSlots;
    for (int i = r0_dn; i < r1_dn; ++i) {
      const uint8_t* p = chunk_ptr(1, i);
      if (!p) continue;
      if (skip > 0) {
        --skip;
        continue;
      }
      prefetch_l2_hint(p, 2 * UNIT, stream_pol);
    }
  }

  __syncthreads();  // the x image is complete

  // 0x54005400 (f16x2 64.0) as a register operand: each decode is one LOP3
  const uint32_t m64 = 0x54005400u;
  stamp(2);
  bool bad = false;
  PK_T(long long cy_wait = 0, cy_comp = 0, n_units = 0, cy_epi = 0, cy_issue = 0, cy_task = 0;)
  const uint64_t keep_meta = policy_evict_last();

  // One chunk (chunk c of a row group whose first rows start at superblock
  // phases p0 / p1) against the image (im, X, nsb padded sub-blocks): the
  // next ring slot, folded into acc.
  auto run_chunk = [&](const uint8_t* im, const float2* X, int nsb, int c, int p0, int p1, float (&acc)[2][2]) {
    const uint32_t sl = consumed % kSlots;
    PK_T(const long long c0 = clock64();)
    if (!warp_wait(&bar[sl], (consumed / kSlots) & 1u, a.err)) {
      bad = true;
      return;
    }
    PK_T(const long long c1 = clock64(); cy_wait += c1 - c0; n_units += 2;)
    consumed += 1;
    const uint8_t* uA = ring + sl * 2 * UNIT;
    const uint8_t* uB = uA + UNIT;
    // B sources (see chunk_mma): half 0 from lanes g == t, half 1 from g == t + 4
    const size_t pst = (size_t)nsb * 16;
    const int sA = 8 * c - p0 + t + kPadL, sB = 8 * c - p1 + t + kPadL;
    const bool h0 = g == t, h1 = g == t + 4;
    const int xa = 8 * c - p0 + 2 * t + kPadL, xb = 8 * c - p1 + 2 * t + kPadL;
    const uint8_t* a0s = h0 ? im + (size_t)sA * 16 : zero;
    const uint8_t* a1s = h1 ? im + (size_t)(sA + 4) * 16 : zero;
    const size_t z0 = h0 ? pst : 0, z1 = h1 ? pst : 0;
    if (Q4) {
      // hi bytes: lanes g == 4h + t; lo bytes (planes 2, 3): lanes g == 4(1-h) + t
      const bool on = h0 || h1;
      const size_t lo = 2 * pst, zq = on ? pst : 0;
      const uint8_t* qA0 = on ? im + (size_t)sA * 16 + (h1 ? lo : 0) : zero;
      const uint8_t* qA1 = on ? im + (size_t)(sA + 4) * 16 + (h0 ? lo : 0) : zero;
      int cA[4], cB[4];
      const uint8_t* qB0 = on ? im + (size_t)sB * 16 + (h1 ? lo : 0) : zero;
      const uint8_t* qB1 = on ? im + (size_t)(sB + 4) * 16 + (h0 ? lo : 0) : zero;
      chunk_imma(uA + HDR, uB + HDR, qA0, qA1, qB0, qB1, zq, zq, p0 == p1, lane, cA, cB);
      fold_q4(uA, cA, X[xa], X[xa + 1], g, t, acc[0][0], acc[0][1]);
      fold_q4(uB, cB, X[xb], X[xb + 1], g, t, acc[1][0], acc[1][1]);
    } else {
      float dA[4], dB[4];
      chunk_mma<false, true>(uA + HDR, uB + HDR, a0s, a1s, nullptr, nullptr, z0, z1, 0, 0, m64, lane, dA, dB);
      unit_fold<false>(uA, dA, X[xa].x, X[xa + 1].x, g, t, acc[0][0], acc[0][1]);
      unit_fold<false>(uB, dB, X[xb].x, X[xb + 1].x, g, t, acc[1][0], acc[1][1]);
    }
    __syncwarp();  // every lane has read both slots before they are refilled
    PK_T(const long long c2 = clock64(); cy_comp += c2 - c1;)
    issue_next();
    PK_T(cy_issue += clock64() - c2;)
  };

  // Down images of up to two chunks (slot k[u], activation sub-blocks
  // sb0[u] .. sb0[u] + 7, zero outside [0, I/32); u < n) into this warp's
  // buffers (buf0 + u) % 2.  An activation is ready once its word is not +0.0 (the gate/up
  // epilogue never stores that pattern); the loads repeat until every word
  // the warp needs is ready, so one L2 round trip suffices when they are.
  // Bounded: records kDevWaitTimeout and returns false.
  auto stage_down = [&](int n, int buf0, const int (&k)[2], const int (&sb0)[2]) -> bool {
    const int nsbI = a.I / 32, q = lane & 3;
    float v[2][8];
    bool ok = false;
    for (uint32_t it = 0; it < kSpinPolls && !ok; ++it) {
      ok = true;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int sb = sb0[u] + (lane >> 2);
        if (u < n && sb >= 0 && sb < nsbI) {
          const float* src = a.dact + (int64_t)k[u] * a.I + sb * 32 + 8 * q;
          ld_relaxed_f32x8(src, v[u]);
#pragma unroll
          for (int i = 0; i < 8; ++i) ok = ok && __float_as_uint(v[u][i]) != 0u;
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) v[u][i] = 0.f;
        }
      }
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) __nanosleep(32);
    }
    if (!ok) {
      if (lane == 0 && a.err) atomicExch(a.err, kDevWaitTimeout);
      return false;
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (u >= n) break;
      uint8_t* mim = mini + (size_t)((buf0 + u) & 1) * pk_mini_bytes();
      stage_group<Q4>(mim, reinterpret_cast<float2*>(mim + pk_img_bytes(1, kMiniNsb)), kMiniNsb, lane >> 2, q, v[u],
                      true);
    }
    __syncwarp();
    return true;
  };

  // The warp's range of one phase, one group at a time: stream, fold,
  // publish the group's partial sums; the last contributor of a group runs
  // its epilogue.
  // Down chunk i of the flat list: its slot and first activation sub-block;
  // false when the slot is skipped.
  auto dn_chunk = [&](int i, int& k, int& sb0) -> bool {
    const int grp = i / Cg_dn, r = i - grp * Cg_dn;
    k = r / a.C_dn;
    if (s_e[k] < 0) return false;
    sb0 = 8 * (r - k * a.C_dn) - ldg_hint_i32(a.dn_ph + grp, keep_meta);
    return true;
  };
  int dn_m = 0;  // down chunks of this warp consumed so far (buffer dn_m % 2)
  auto run_range = [&](int down) {
    const int Cg = down ? Cg_dn : Cg_gu, Q = down ? a.Q_dn : a.Q_gu;
    const int r1 = down ? r1_dn : r1_gu;
    if (down) {
      // the images of the warp's first two down chunks, in one pass
      int kk[2] = {0, 0}, sb[2] = {0, 0}, n = 0;
      for (int i = r0_dn; i < r1_dn && n < 2; ++i) {
        int k1, s1;
        if (!dn_chunk(i, k1, s1)) continue;
        if (n == 0) {
          kk[0] = k1;
          sb[0] = s1;
        } else {
          kk[1] = k1;
          sb[1] = s1;
        }
        ++n;
      }
      if (n && !stage_down(n, 0, kk, sb)) bad = true;
    }
    for (int i = down ? r0_dn : r0_gu; i < r1 && !bad;) {
      PK_T(const long long ct0 = clock64();)
      const int G = i / Cg, gend = min(r1, (G + 1) * Cg);
      const int grp = down ? G : G % a.ngj;
      // row-block phases and this lane's row-map entry (L2 evict-last:
      // every token re-reads them)
      int p0, p1, map;
      if (down) {
        p0 = p1 = ldg_hint_i32(a.dn_ph + grp, keep_meta);
        map = ldg_hint_i32(a.dn_h + grp * 32 + lane, keep_meta);
      } else {
        p0 = ldg_hint_i32(a.gu_ph + 2 * grp, keep_meta);
        p1 = ldg_hint_i32(a.gu_ph + 2 * grp + 1, keep_meta);
        map = lane < 16 ? ldg_hint_i32(a.gu_j + grp * 16 + lane, keep_meta) : -1;
      }
      float accg[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
      // runs of one slot (a gate/up group is one run), each weighted by its
      // routing weight (1 for gate/up).  One chunk call site for both phases
      // keeps the unrolled chunk body once in the code (instruction cache).
      for (int j = i; j < gend && !bad;) {
        const int r = j - G * Cg, k = down ? r / a.C_dn : G / a.ngj;
        const int kend = down ? min(gend, G * Cg + (k + 1) * a.C_dn) : gend;
        if (s_e[k] >= 0) {
          float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
          for (int jj = j; jj < kend && !bad; ++jj) {
            const uint8_t* im = img;
            const float2* X = Xs;
            int nsb = a.nsb_h, cc = jj - G * Cg, q0 = p0, q1 = p1;
            if (down) {
              // the chunk's 8 activation sub-blocks, in this warp's image
              // (the first two staged before the loop)
              if (dn_m >= 2) {
                int kk[2] = {k, 0}, sb[2] = {8 * (jj - G * Cg - k * a.C_dn) - p0, 0};
                if (!stage_down(1, dn_m & 1, kk, sb)) {
                  bad = true;
                  break;
                }
              }
              im = mini + (size_t)(dn_m & 1) * pk_mini_bytes();
              X = reinterpret_cast<const float2*>(im + pk_img_bytes(1, kMiniNsb));
              nsb = kMiniNsb;
              cc = q0 = q1 = 0;
              ++dn_m;
            }
            run_chunk(im, X, nsb, cc, q0, q1, acc);
          }
          const float w = down ? s_w[k] : 1.f;
#pragma unroll
          for (int rb = 0; rb < 2; ++rb)
#pragma unroll
            for (int q = 0; q < 2; ++q) accg[rb][q] = fmaf(w, acc[rb][q], accg[rb][q]);
        }
        j = kend;
      }
      // partial sums of the group's 32 rows (rb, row): reduce over the quad
#pragma unroll
      for (int rb = 0; rb < 2; ++rb)
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          float v = accg[rb][q];
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          accg[rb][q] = v;
        }
      const int first = G * Cg / Q, count = ((G + 1) * Cg - 1) / Q - first + 1;
      const int slots = down ? a.slots_dn : a.slots_gu;
      float* Pg = (down ? a.part_dn : a.part_gu) + (int64_t)G * slots * 32;
      float* P = Pg + (gw - first) * 32;
      if (t == 0) {
        P[g] = accg[0][0];
        P[g + 8] = accg[0][1];
        P[16 + g] = accg[1][0];
        P[24 + g] = accg[1][1];
      }
      // The warp barrier orders the lanes' partial stores before lane 0's
      // counter update; the update releases them at GPU scope (release is
      // cumulative) and acquires the other contributors' partials for the
      // last one.
      __syncwarp();
      unsigned* cnt = down ? a.cnt_dn + G : a.cnt_gu + G;
      unsigned last = 0;
      if (lane == 0) {
        unsigned old;
        asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(old) : "l"(cnt) : "memory");
        last = old == (unsigned)count - 1;
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      PK_T(cy_task += clock64() - ct0;)
      i = gend;
      if (!last) continue;
      PK_T(const long long ce = clock64();)
      const float sum = sum_parts(Pg, count, lane);
      if (!down) {
        // gate/up epilogue: rows [0,16) gate, [16,32) up of the group's 16
        // outputs; lanes 0-15 hold the gate sums, 16-31 the up sums
        const int k = G / a.ngj;
        const float other = __shfl_xor_sync(0xffffffffu, sum, 16);
        const float gate = sum, up = other;
        const int jo = map;
        float r = 0.f;
        if (jo >= 0 && s_e[k] >= 0) {
          const float gb = s_bias[0][k] ? gate + s_bias[0][k][jo] : gate;
          const float ub = s_bias[1][k] ? up + s_bias[1][k][jo] : up;
          r = act_fn(a.act_kind, gb, ub, a.limit, a.alpha);
        }
        // +0.0 marks "not written": store it as -0.0 (the same number)
        if (jo >= 0) a.dact[(int64_t)k * a.I + jo] = __float_as_uint(r) == 0u ? -0.f : r;
      } else {
        // down epilogue: 32 outputs, the slots already weighted
        const int h = map;
        if (h >= 0) {
          float o = sum;
          for (int k = 0; k < a.top_k; ++k)
            if (s_e[k] >= 0 && s_bias[2][k]) o = fmaf(s_w[k], s_bias[2][k][h], o);
          if (a.out_f32)
            static_cast<float*>(a.out)[h] = o;
          else
            static_cast<uint16_t*>(a.out)[h] = f32_to_bf16_bits(o);
        }
      }
      __syncwarp();
      if (lane == 0) *cnt = 0u;
      PK_T(cy_epi += clock64() - ce;)
    }
  };

  // ---- phase 0: the warp's gate/up range; phase 1: its down range.  One
  // loop, so the range body exists once in the code (instruction cache).
  // No barrier between them: a down chunk waits only for the activation
  // sub-blocks it reads (stage_down), so down work starts where gate/up is
  // complete while other groups still stream.
  PK_T(if (lane == 0 && blockIdx.x < 160) g_pk_wtrace[(blockIdx.x * 16 + warp) * 8 + 7] = gtimer();)
#pragma unroll 1
  for (int phase = 0; phase < 2; ++phase) {
  run_range(phase);
  PK_T(if (lane == 0 && blockIdx.x < 160 && phase == 0) {
    unsigned long long* W = g_pk_wtrace + (blockIdx.x * 16 + warp) * 8;
    W[0] = gtimer();
    W[1] = cy_wait;
    W[2] = cy_comp;
    W[3] = n_units;
    W[4] = cy_issue;
    W[5] = cy_epi;
    W[6] = cy_task;
  })
  }
  __syncthreads();
  stamp(6);


  // copies still in flight land before the CTA exits (bounded: after a
  // timed-out wait, keep waiting on later slots until none is left or the
  // total budget runs out)
  {
    int misses = 0;
    while (consumed < issued && misses < 4) {
      if (!warp_wait(&bar[consumed % kSlots], (consumed / kSlots) & 1u, a.err)) ++misses;
      ++consumed;
    }
  }
  // the last CTA to finish resets the device-wide words for the next call
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned old;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(old) : "l"(a.sync + 1) : "memory");
    s_last = old == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last) {
    for (int i = threadIdx.x; i < a.top_k * a.I / 4; i += kPkThreads)
      reinterpret_cast<float4*>(a.dact)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (threadIdx.x == 0) a.sync[1] = 0u;
    __threadfence();
  }
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

// Partial-sum slots per group: the most warps whose ranges can meet one
// group, for the smallest range length Q any launch uses (the full device's
// warps; a smaller grid only lengthens Q and lowers the count).
static void pk_slots(const TsbMoeSpec& sp, const PkGeo& G, int& sg, int& sd) {
  const int64_t warps = (int64_t)num_sms() * kPkWarps;
  const int64_t Ng = (int64_t)sp.top_k * G.ngj * G.C_gu, Nd = (int64_t)sp.top_k * G.ndp * G.C_dn;
  const int64_t Qg = std::max<int64_t>(1, (Ng + warps - 1) / warps), Qd = std::max<int64_t>(1, (Nd + warps - 1) / warps);
  sg = (int)((G.C_gu + Qg - 1) / Qg + 1);
  sd = (int)(((int64_t)sp.top_k * G.C_dn + Qd - 1) / Qd + 1);
}

// Workspace after the generic layer workspace: counters, device-wide words,
// gate/up and down partial sums.
struct PkWs {
  size_t cnt_gu, cnt_dn, sync, dact, part_gu, part_dn, total;
};
static PkWs pk_ws(const TsbMoeSpec& sp, const PkGeo& G) {
  auto al = [](size_t v) { return (v + 255) & ~size_t(255); };
  PkWs W;
  W.cnt_gu = 0;
  W.cnt_dn = al(W.cnt_gu + 4 * (size_t)sp.top_k * G.ngj);
  W.sync = al(W.cnt_dn + 4 * (size_t)G.ndp);
  W.dact = al(W.sync + 64);
  W.part_gu = al(W.dact + 4 * (size_t)sp.top_k * sp.inter);
  int sg = 0, sd = 0;
  pk_slots(sp, G, sg, sd);
  W.part_dn = al(W.part_gu + 4 * 32 * (size_t)sp.top_k * G.ngj * sg);
  W.total = al(W.part_dn + 4 * 32 * (size_t)G.ndp * sd);
  return W;
}

size_t packed_ws_bytes(const TsbMoeSpec& sp) {
  if (!packable(sp)) return 0;
  return pk_ws(sp, pk_geo(sp, pk_maps(sp))).total;
}

constexpr int kPkSmemMax = 220 * 1024;

// Launch shape: clusters of kPkCluster CTAs (the router split), as many as fit
// co-resident with one CTA per SM (the device-wide barrier between gate/up and
// down needs every CTA resident; its waits are bounded all the same).
constexpr int kPkCluster = 2;

// CTAs of one launch: as many clusters of kPkCluster as the device keeps
// co-resident with one CTA per SM (cudaOccupancyMaxActiveClusters); the
// device-wide barrier between gate/up and down needs every CTA resident.
template <int F>
static int pk_grid(int& grid) {
  static int g = 0;
  static cudaError_t init = [] {
    cudaError_t e = cudaFuncSetAttribute(pk_layer_kernel<F>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPkSmemMax);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(num_sms() / kPkCluster * kPkCluster));
    cfg.blockDim = dim3(kPkThreads);
    cfg.dynamicSmemBytes = kPkSmemMax;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = kPkCluster;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, pk_layer_kernel<F>, &cfg);
    if (e != cudaSuccess) return e;
    g = std::min(clusters, num_sms() / kPkCluster) * kPkCluster;
    return g > 0 ? cudaSuccess : cudaErrorInvalidConfiguration;
  }();
  if (init != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(init));
  grid = g;
  return TSB_OK;
}

template <int F>
static int launch_pk(PkArgs& a, int grid, size_t smem, cudaStream_t st) {
  if (smem > kPkSmemMax) return set_error(TSB_ERR_UNSUPPORTED, "packed decode: layer too large for shared memory");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kPkThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = kPkCluster;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, pk_layer_kernel<F>, a);
  if (e != cudaSuccess) return set_error(TSB_ERR_CUDA, cudaGetErrorString(e));
  return TSB_OK;
}

int launch_packed_decode(const TsbMoeSpec& sp, const void* packed, const TsbExpert* ex, const void* x, int32_t* ids,
                         float* wts, void* out, int out_f32, int32_t* err, char* pws, cudaStream_t st,
                         const void* router_w, const float* router_b) {
  // geometry depends only on the spec: cache the last one
  static thread_local TsbMoeSpec last_sp{};
  static thread_local PkGeo last_G{};
  static thread_local bool have = false;
  if (!have || memcmp(&last_sp, &sp, sizeof sp) != 0) {
    last_G = pk_geo(sp, pk_maps(sp));
    last_sp = sp;
    have = true;
  }
  const PkGeo& G = last_G;
  const PkWs W = pk_ws(sp, G);
  const uint8_t* base = static_cast<const uint8_t*>(packed);
  PkArgs a{};
  a.packed = base + G.maps_bytes;
  a.gu_j = reinterpret_cast<const int32_t*>(base + G.o_guj);
  a.gu_ph = reinterpret_cast<const int32_t*>(base + G.o_guph);
  a.dn_h = reinterpret_cast<const int32_t*>(base + G.o_dnh);
  a.dn_ph = reinterpret_cast<const int32_t*>(base + G.o_dnph);
  a.gu_off = G.gu_off;
  a.dn_off = G.dn_off;
  a.expert_bytes = G.expert_bytes;
  a.H = sp.hidden;
  a.I = sp.inter;
  a.E = sp.n_experts;
  a.top_k = sp.top_k;
  a.ngj = G.ngj;
  a.ndp = G.ndp;
  a.C_gu = G.C_gu;
  a.C_dn = G.C_dn;
  int grid = 0;
  const int rc = G.q4 ? pk_grid<FMT_Q4_K>(grid) : pk_grid<FMT_MXFP4>(grid);
  if (rc) return rc;
  const int warps = grid * kPkWarps;
  a.N_gu = sp.top_k * G.ngj * G.C_gu;
  a.N_dn = sp.top_k * G.ndp * G.C_dn;
  a.Q_gu = std::max(1, (a.N_gu + warps - 1) / warps);
  a.Q_dn = std::max(1, (a.N_dn + warps - 1) / warps);
  pk_slots(sp, G, a.slots_gu, a.slots_dn);
  a.nsb_h = sp.hidden / 32 + kPadL + kPadR;
  a.x = static_cast<const uint16_t*>(x);
  a.router_w = static_cast<const uint16_t*>(router_w);
  a.router_b = router_b;
  a.ids = ids;
  a.wts = wts;
  a.experts = ex;
  a.cnt_gu = reinterpret_cast<unsigned*>(pws + W.cnt_gu);
  a.cnt_dn = reinterpret_cast<unsigned*>(pws + W.cnt_dn);
  a.sync = reinterpret_cast<unsigned*>(pws + W.sync);
  a.dact = reinterpret_cast<float*>(pws + W.dact);
  a.part_gu = reinterpret_cast<float*>(pws + W.part_gu);
  a.part_dn = reinterpret_cast<float*>(pws + W.part_dn);

  a.out = out;
  a.out_f32 = out_f32;
  a.act_kind = sp.activation;
  a.limit = sp.limit;
  a.alpha = sp.alpha;
  a.err = err;
  if (G.q4) return launch_pk<FMT_Q4_K>(a, grid, pk_smem(kQ4Unit, a.nsb_h), st);
  return launch_pk<FMT_MXFP4>(a, grid, pk_smem(kMxUnit, a.nsb_h), st);
}

}  // namespace tsb

#if TSB_PK_TIMING
// Development builds: copy the phase stamps ([160][16]) and per-warp counts
// ([160][16][8]) to host memory.
extern "C" int tsb_pk_timing_read(unsigned long long* stamps, unsigned long long* warps) {
  cudaError_t e = cudaMemcpyFromSymbol(stamps, tsb::g_pk_trace, sizeof(unsigned long long) * 160 * 16);
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(warps, tsb::g_pk_wtrace, sizeof(unsigned long long) * 160 * 16 * 8);
  return (int)e;
}
#endif
