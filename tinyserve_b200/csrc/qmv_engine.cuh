// Pipelined quantised matrix-vector engine for up to 8 activation vectors
// (batch-1 decode and small batches).
//
// One CTA, persistent over "row blocks" (16 weight rows each):
//   warp 0 ........ producer.  For each (row block, k-chunk) it copies the raw
//                   quantised bytes of the 16 rows into a ring of shared-memory
//                   stages with cp.async.bulk (the TMA engine's non-tensor
//                   path), completing on an mbarrier.  The ragged end of a
//                   matrix and MXFP4 scale bytes use plain loads.
//   warps 1..NCW .. consumers.  They split the chunk's 32-element steps.  For
//                   every step each lane decodes its share of the 16 rows
//                   straight into mma.sync A fragments (no dequantised copy of
//                   the weights exists anywhere), multiplies them with up to 8
//                   activation vectors kept in shared memory as f16 (B
//                   fragments), and folds the per-block scales into fp32
//                   accumulators.  After the last chunk of a row block the
//                   warps reduce their partial sums through shared memory and
//                   the plan's epilogue writes the result.
//
// A plan (template parameter P) says which 16 rows a row block holds (up to 8
// segments of rows from different matrices), which activation vector each B
// column reads and what the epilogue does.  The same engine runs the plain
// matvec, the fused gate/up + SwiGLU of an MoE layer and the fused down
// projection + weighted top-k combine.
//
// Stage layout: segment s of a row block occupies the fixed slot
// [s*slot, (s+1)*slot) when chunks cover whole rows (one contiguous copy per
// segment); otherwise row r of segment s occupies [(s*rps+r)*slot, ...) (one
// copy per row, rps = rows per segment).  MXFP4 scale bytes follow at sc_base.  Offsets are closed
// form, so producer and consumers compute them independently.
#pragma once
#include <type_traits>

#include "qformats.cuh"

namespace tsb {

constexpr int kMaxSeg = 8;

struct Seg {
  const uint8_t* w;   // matrix base (16-B aligned)
  const uint8_t* s;   // MXFP4 scale tensor base, else nullptr
  int64_t row0;       // first matrix row held
  int nrows;          // rows held (<= 16)
  int64_t mat_bytes;  // bytes of the whole matrix (clamp for the last copy)
};

// Per-launch table the producer fills once (plan.fill_cache) so that seg() and
// the epilogue never chase pointers through global memory per row block.
struct SlotCache {
  const uint8_t* w[2];  // weight matrices of slot (e.g. gate / up, or down)
  const uint8_t* s[2];  // their MXFP4 scale tensors
  const float* b[2];    // optional biases
  int e;                // expert id (-1: invalid id in the routing table)
  int pad;
};
constexpr int kMaxSlots = 8;

struct Piece {
  int64_t cs;     // first kept source byte (16-B aligned, relative to the matrix)
  int64_t end;    // one past the last needed source byte
  uint32_t soff;  // stage offset of byte cs
  uint32_t bulk;  // bytes [cs, cs+bulk) arrive through the bulk copy
};

// Launch-constant geometry of a stage.
struct StageGeom {
  int K;        // row length (elements)
  int KC;       // chunk length (elements, multiple of 32)
  int slot;     // bytes per segment (whole-row chunks) or per row (partial chunks)
  int sc_base;  // MXFP4: stage offset of the scale bytes
  int sslot;    // MXFP4: bytes per scale slot (per segment or per row, like `slot`)
  int rps;      // rows per segment (at most)
};

template <int F>
__device__ __forceinline__ void byte_range(int64_t e0, int64_t e1, int64_t& b0, int64_t& b1) {
  using T = FmtT<F>;
  const int64_t q0 = e0 / 32, q1 = e1 / 32;
  if (F == FMT_MXFP4 || F == FMT_Q8_0) {
    b0 = q0 * T::BB;
    b1 = q1 * T::BB;
  } else {
    b0 = (q0 >> 3) * T::BB;
    b1 = ((q1 + 7) >> 3) * T::BB;
  }
}

// Piece for segment `si` (whole-row chunk, r < 0) or for row r of it.
template <int F>
__device__ __forceinline__ Piece make_piece(const Seg& sg, int si, int r, const StageGeom& G, int k0, int k1) {
  int64_t b0, b1;
  uint32_t soff;
  if (r < 0) {
    byte_range<F>(sg.row0 * G.K, (sg.row0 + sg.nrows) * G.K, b0, b1);
    soff = (uint32_t)(si * G.slot);
  } else {
    const int64_t rr = sg.row0 + r;
    byte_range<F>(rr * G.K + k0, rr * G.K + k1, b0, b1);
    soff = (uint32_t)((si * G.rps + r) * G.slot);
  }
  Piece p;
  p.cs = b0 & ~int64_t(15);
  p.end = b1;
  int64_t be = (b1 + 15) & ~int64_t(15);
  const int64_t mat_al = sg.mat_bytes & ~int64_t(15);
  if (be > mat_al) be = mat_al;
  if (be < p.cs) be = p.cs;
  p.bulk = (uint32_t)(be - p.cs);
  p.soff = soff;
  return p;
}

// MXFP4 scale bytes of segment `si` (whole rows, r < 0) or of row r, as a piece
// of the scale tensor.  The scale tensor need not be 16-B aligned, so alignment
// is taken on absolute addresses (cs may be up to 15 bytes before the tensor;
// those bytes lie inside the same allocation, whose start is 256-B aligned).
template <int F>
__device__ __forceinline__ Piece make_scale_piece(const Seg& sg, int si, int r, const StageGeom& G, int k0, int k1) {
  const int64_t bpr = G.K / 32;  // scale bytes per row
  int64_t b0, b1;
  uint32_t soff;
  if (r < 0) {
    b0 = sg.row0 * bpr;
    b1 = (sg.row0 + sg.nrows) * bpr;
    soff = (uint32_t)(G.sc_base + si * G.sslot);
  } else {
    b0 = (sg.row0 + r) * bpr + k0 / 32;
    b1 = b0 + (k1 - k0) / 32;
    soff = (uint32_t)(G.sc_base + (si * G.rps + r) * G.sslot);
  }
  const int64_t base = (int64_t)reinterpret_cast<uintptr_t>(sg.s);
  Piece p;
  p.cs = ((base + b0) & ~int64_t(15)) - base;
  p.end = b1;
  int64_t be = ((base + b1 + 15) & ~int64_t(15)) - base;
  const int64_t mat_end = ((base + sg.mat_bytes / 16) & ~int64_t(15)) - base;  // scales = blocks / 16
  if (be > mat_end) be = mat_end;
  if (be < p.cs) be = p.cs;
  p.bulk = (uint32_t)(be - p.cs);
  p.soff = soff;
  return p;
}

// Per-row addressing within a stage for the current chunk.
struct RowInfo {
  int32_t off;   // stage offset of the block (Q8_0/MXFP4) or superblock (K-quants) holding element k0
  int32_t sub0;  // K-quants: 32-block index of element k0 inside that superblock
  int32_t soff;  // MXFP4: stage offset of this row's scale bytes for the chunk
  int32_t valid;
};

template <int F>
__device__ __forceinline__ RowInfo row_info(const Seg& sg, int si, int lr, const StageGeom& G, int k0, int k1) {
  RowInfo ri{0, 0, 0, 0};
  if (si < 0 || lr >= sg.nrows) return ri;
  const bool whole = (k0 == 0 && k1 == G.K);
  const Piece p = make_piece<F>(sg, si, whole ? -1 : lr, G, k0, k1);
  const int64_t r = sg.row0 + lr;
  const int64_t q = (r * G.K + k0) / 32;
  using T = FmtT<F>;
  if (F == FMT_MXFP4 || F == FMT_Q8_0) {
    ri.off = (int32_t)(p.soff + (q * T::BB - p.cs));
  } else {
    ri.off = (int32_t)(p.soff + ((q >> 3) * T::BB - p.cs));
    ri.sub0 = (int32_t)(q & 7);
  }
  if (F == FMT_MXFP4) {
    const int cb = (k1 - k0) / 32;
    (void)cb;
    const Piece sp = make_scale_piece<F>(sg, si, whole ? -1 : lr, G, k0, k1);
    ri.soff = (int32_t)(sp.soff + (((sg.row0 + lr) * (int64_t)(G.K / 32) + k0 / 32) - sp.cs));
  }
  ri.valid = 1;
  return ri;
}

template <int F>
__device__ __forceinline__ RowLoc row_loc(const uint8_t* stage, const RowInfo& ri, int u) {
  RowLoc L;
  using T = FmtT<F>;
  if (F == FMT_MXFP4 || F == FMT_Q8_0) {
    L.blk = stage + ri.off + u * T::BB;
    L.sub = 0;
    L.mx_scale = (F == FMT_MXFP4) ? stage[ri.soff + u] : 0u;
  } else {
    const int s = ri.sub0 + u;
    L.blk = stage + ri.off + (s >> 3) * T::BB;
    L.sub = s & 7;
    L.mx_scale = 0u;
  }
  return L;
}

// How the lane's B column and folded C values map to activation vectors.
enum ColMode : int {
  COLS_DUP = 0,   // all B columns read vector 0; each lane folds c0 (row g) and c2 (row g+8)
  COLS_FULL = 1,  // B column n reads vector n; all four C values folded
  COLS_DIAG = 2,  // row m's useful column is n(m) (top-k combine tiles)
};

// Convert NV activation vectors (each K long) into shared memory:
//   xq  [U][NV][32] f16 in the format's element order (64 B per step and vector)
//   xsx [U][NV] float4 {xs, sx0, sx1, 0}: xs = power-of-two scale applied before
//       rounding to f16 (keeps the block maximum in (2^14, 2^15]); sx0 / sx1 =
//       sums of the f16 values actually fed to the tensor cores, rescaled by xs
//       (sx1 only for Q6_K, whose 16-element halves carry separate scales).
// Each thread owns 4 consecutive elements per round (8 threads per 32-block);
// all rounds of a batch are loaded before any is processed, so the global
// load latency is paid once per batch rather than once per block.
struct XSrc {
  const void* p;   // vector 0
  int64_t stride;  // elements between vectors
  int dtype;       // TSB_DT_F32 (0) / TSB_DT_BF16 (1) / TSB_DT_F16 (2)
  int vec_ok;      // rows 16-B (fp32) / 8-B (16-bit) aligned: vector loads allowed
  int cg;          // fp32 source written by other CTAs of this grid: load through L2 (ld.global.cg)
};

__device__ __forceinline__ float4 load4(const XSrc& X, int v, int k) {
  const int64_t i = v * X.stride + k;
  if (X.dtype == 0) {
    if (X.vec_ok) {
      const float4* q = reinterpret_cast<const float4*>(static_cast<const float*>(X.p) + i);
      return X.cg ? __ldcg(q) : *q;
    }
    const float* q = static_cast<const float*>(X.p) + i;
    return make_float4(q[0], q[1], q[2], q[3]);
  }
  uint32_t a, b;
  if (X.vec_ok) {
    const uint2 w = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(X.p) + i);
    a = w.x;
    b = w.y;
  } else {
    const uint16_t* q = static_cast<const uint16_t*>(X.p) + i;
    a = q[0] | ((uint32_t)q[1] << 16);
    b = q[2] | ((uint32_t)q[3] << 16);
  }
  if (X.dtype == 1)
    return make_float4(__uint_as_float(a << 16), __uint_as_float(a & 0xFFFF0000u), __uint_as_float(b << 16),
                       __uint_as_float(b & 0xFFFF0000u));
  const __half2 h0 = *reinterpret_cast<__half2*>(&a), h1 = *reinterpret_cast<__half2*>(&b);
  const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
  return make_float4(f0.x, f0.y, f1.x, f1.y);
}

template <int F>
__device__ void stage_x(uint8_t* xq_raw, float4* xsx, int K, int nv, const XSrc& X, int tid, int nthreads) {
  constexpr int kBatch = 8;
  __half* xq = reinterpret_cast<__half*>(xq_raw);
  const int total4 = nv * K / 4;
  const int p = (tid & 7) * 4;  // position of this thread's first element in its block
  int dst[4];
  for (int i = 0; i < 4; ++i)
    for (int t = 0; t < 4; ++t)
      for (int s = 0; s < 8; ++s)
        if (elem_order<F>(t, s) == p + i) dst[i] = 8 * t + s;
  for (int r0 = 0; r0 * nthreads < total4; r0 += kBatch) {
    float4 v[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int f = (r0 + j) * nthreads + tid;
      v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (f < total4) v[j] = load4(X, (4 * f) / K, (4 * f) % K);
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      if ((r0 + j) * nthreads >= total4) break;  // uniform across the CTA
      const int f = (r0 + j) * nthreads + tid;
      float amax = fmaxf(fmaxf(fabsf(v[j].x), fabsf(v[j].y)), fmaxf(fabsf(v[j].z), fabsf(v[j].w)));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
      // e = exponent such that amax * 2^-e lies in (2^14, 2^15], from the float's
      // exponent bits (clamped so 2^-e and 2^e stay normal floats); scaling by a
      // power of two is exact.
      int e = 0;
      if (amax > 0.f && amax <= 3.0e38f) {
        const int ex = (int)((__float_as_uint(amax) >> 23) & 255u) - 126;  // amax = m * 2^ex, m in [0.5, 1)
        e = min(126, max(-126, ex - 15));
      }
      const float inv = __uint_as_float((uint32_t)(127 - e) << 23);
      const float xv[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
      float hs = 0.f;
      __half hh[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        hh[i] = __float2half_rn(xv[i] * inv);
        hs += __half2float(hh[i]);
      }
      float s_all = hs, s_lo = (p < 16) ? hs : 0.f;
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        s_all += __shfl_xor_sync(0xffffffffu, s_all, o);
        s_lo += __shfl_xor_sync(0xffffffffu, s_lo, o);
      }
      if (f < total4) {
        const int vv = (4 * f) / K, u = ((4 * f) % K) / 32;
        __half* blk = xq + (size_t)(u * nv + vv) * 32;
#pragma unroll
        for (int i = 0; i < 4; ++i) blk[dst[i]] = hh[i];
        if (p == 0) {
          const float xs = __uint_as_float((uint32_t)(127 + e) << 23);
          if (F == FMT_Q6_K)
            xsx[u * nv + vv] = make_float4(xs, s_lo * xs, (s_all - s_lo) * xs, 0.f);
          else
            xsx[u * nv + vv] = make_float4(xs, s_all * xs, 0.f, 0.f);
        }
      }
    }
  }
}

// Producer tables for whole-row plans: the row headers, bulk pieces and byte
// totals of the next kPtabUnits units are computed ahead, one lane per item, so
// that filling a stage is only a header copy, expect_tx and 1-2 bulk copies.
constexpr int kPtabUnits = 4;
struct PtabPiece {
  const uint8_t* src;
  uint32_t bytes;
  uint32_t soff;  // bit 31: the piece also has a plain-load tail (matrix end)
};
constexpr int kPtabBytes = kPtabUnits * 16 * 16 + kPtabUnits * 16 * (int)sizeof(PtabPiece) + kPtabUnits * 4;

// Shared-memory map of one CTA.
//   bars     full[NSTAGE], empty[NSTAGE] mbarriers
//   cnt      per-stage counters of warps done with a row block (last one runs the epilogue)
//   red      per-stage partial sums: [NSTAGE][NCW][16] (one column) or [..][128] (8 columns)
//   coef     per-warp fold coefficients of the current coefficient chunk
//   stages   NSTAGE x STAGE_BYTES; each stage starts with a 256-B header of 16 RowInfo
//   x        staged activation vectors
template <int NCW, int NSTAGE, int STAGE_BYTES, int MODE, int F>
struct SmemPlan {
  static constexpr int kCoefCh = (F == FMT_Q6_K) ? 8 : 16;  // steps per coefficient chunk
  static constexpr int kCoefW = (F == FMT_Q6_K) ? 16 : 8;  // bytes per coefficient entry
  static constexpr int kRedW = (MODE == COLS_FULL) ? 128 : 16;
  static constexpr int kRed = NSTAGE * NCW * kRedW * 4;
  static constexpr int kCoef = NCW * 16 * kCoefCh * kCoefW;
  static constexpr int kHdr = 256;
  static constexpr int off_bars = 0;
  static constexpr int off_cnt = 128;
  static constexpr int off_red = 256;
  static constexpr int off_cache = off_red + kRed;
  static constexpr int off_ptab = off_cache + kMaxSlots * (int)sizeof(SlotCache);
  static constexpr int off_coef = ((off_ptab + NSTAGE * kPtabBytes + 15) / 16) * 16;  // one table per producer
  static constexpr int off_stage = ((off_coef + kCoef + 127) / 128) * 128;
  static constexpr int off_x = off_stage + NSTAGE * STAGE_BYTES;
  static __host__ __device__ constexpr int x_bytes(int K, int nv) { return (K / 32) * nv * (64 + 16); }
  static __host__ __device__ constexpr int total(int K, int nv) { return off_x + x_bytes(K, nv); }
};

// Plan interface (all device-side, const):
//   StageGeom geom; int* err;
//   static constexpr bool kProducerWaits;   row blocks depend on the previous kernel's output
//   static constexpr bool kXIndependent;    activations were written before the previous kernel
//   int num_vectors() const;                activation vectors (<= 8)
//   XSrc xsrc() const;                      where the activation vectors live
//   int num_blocks() const;                 row blocks
//   void fill_cache(SlotCache* c, int lane) const;   producer warp, once, before any seg()
//   int nseg(int rb) const;  Seg seg(const SlotCache*, int rb, int s) const;
//   void rowmap(int rb, int m, int& s, int& lr) const;   A-row m -> (segment, row)  (s<0: none)
//   void columns(int rb, int g, int t, int& vb, int& v0, int& v1, int& na, int& nb) const;
//   void epilogue(const SlotCache*, int rb, const float* red, int nwarps, int lane) const;
//       run by the last warp to finish the row block; red[w*W + i] = warp w's partial
//       sums, W = 16 (i = A-row, one column) or 128 (i = row*8 + column).
// NG consumer groups of NCW/NG warps: row block i goes to group i % NG, and the
// warps of a group split its K range.  NG = 2 when a row block is one stage
// (whole rows), so two row blocks are in flight and each warp covers twice as
// many steps; NG = 1 for k-chunked rows (a group must see all chunks of its rows).
// Shared-memory pointers of the engine (one CTA).
struct EngSmem {
  uint8_t* ptab;  // producer tables (kPtabBytes): headers and bulk pieces of upcoming units
  uint64_t* full;
  uint64_t* empty;
  int* cnt;
  float* red;
  uint8_t* stages;
  uint8_t* coef;  // 2 KB per consumer warp
};

// Number of stage units (row block x k-chunk) this CTA processes for a plan.
template <class P>
__device__ __forceinline__ int eng_units(const P& plan) {
  const int nb = plan.num_blocks();
  const int mine = nb > (int)blockIdx.x ? (nb - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  return mine * ((plan.geom.K + plan.geom.KC - 1) / plan.geom.KC);
}

// Producer warp: stream every row block of this CTA for `plan` into the stage
// ring, continuing the ring position `it`.  Returns false if a wait timed out.
// With np producer warps, producer p fills the ring positions it with
// it % np == p (np == NSTAGE: producer p owns stage p); every producer walks
// the same unit sequence so the positions agree with the consumers'.
template <int F, int MODE, int NCW, int NSTAGE, int STAGE_BYTES, int NG, class P>
__device__ __forceinline__ bool eng_produce(const P& plan, const SlotCache* cache, const EngSmem& S, int& it, int lane,
                                            int* err, int np = 1, int pidx = 0) {
  using SP = SmemPlan<NCW, NSTAGE, STAGE_BYTES, MODE, F>;
  constexpr int WPG = NCW / NG;
  static_assert(NCW % NG == 0, "groups must split the consumer warps evenly");
  uint64_t* full = S.full;
  uint64_t* empty = S.empty;
  const StageGeom G = plan.geom;
  const int K = G.K, KC = G.KC;
  const int nkc = (K + KC - 1) / KC;
  const int nblocks = plan.num_blocks();
  uint8_t* stages = S.stages;
  if (nkc == 1) {
    // whole rows: table-driven
    int4* htab = reinterpret_cast<int4*>(S.ptab);
    PtabPiece* ptab = reinterpret_cast<PtabPiece*>(S.ptab + kPtabUnits * 256);
    uint32_t* ttab = reinterpret_cast<uint32_t*>(S.ptab + kPtabUnits * 256 + kPtabUnits * 16 * sizeof(PtabPiece));
    constexpr int kPiecesPerSeg = (F == FMT_MXFP4) ? 2 : 1;
    int u = 0;
    for (int rb0 = blockIdx.x; rb0 < nblocks; rb0 += kPtabUnits * gridDim.x) {
      // ---- precompute up to kPtabUnits units (lane = item within a unit)
      __syncwarp();
      for (int j = 0; j < kPtabUnits; ++j) {
        const int rb = rb0 + j * gridDim.x;
        if (rb >= nblocks) break;
        if ((it + j) % np != pidx) continue;  // another producer's stage
        const int ns = plan.nseg(rb);
        uint32_t bytes = 0;
        if (lane < 16) {
          int rs, rl;
          plan.rowmap(rb, lane, rs, rl);
          Seg sg{};
          if (rs >= 0) sg = plan.seg(cache, rb, rs);
          const RowInfo ri = row_info<F>(sg, rs, rl, G, 0, K);
          htab[j * 16 + lane] = make_int4(ri.off, ri.sub0, ri.soff, ri.valid);
        } else if (lane - 16 < ns * kPiecesPerSeg) {
          const int i = lane - 16, s = i % ns;
          const Seg sg = plan.seg(cache, rb, s);
          const Piece p = (i < ns) ? make_piece<F>(sg, s, -1, G, 0, K) : make_scale_piece<F>(sg, s, -1, G, 0, K);
          PtabPiece q;
          q.src = ((i < ns) ? sg.w : sg.s) + p.cs;
          q.bytes = p.bulk;
          q.soff = p.soff | ((p.cs + p.bulk < p.end) ? 0x80000000u : 0u);
          ptab[j * 16 + i] = q;
          bytes = p.bulk;
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) bytes += __shfl_xor_sync(0xffffffffu, bytes, o);
        if (lane == 0) ttab[j] = bytes;
      }
      __syncwarp();
      // ---- fill stages from the tables
      for (int j = 0; j < kPtabUnits; ++j, ++u, ++it) {
        const int rb = rb0 + j * gridDim.x;
        if (rb >= nblocks) break;
        if (it % np != pidx) continue;
        const int ns = plan.nseg(rb);
        const int st = it % NSTAGE;
        const uint32_t ph = ((it / NSTAGE) & 1) ^ 1;
        if (!mbar_wait(&empty[st], ph, err)) return false;
        uint8_t* stage = stages + st * STAGE_BYTES;
        uint8_t* data = stage + SP::kHdr;
        if (lane < 16) reinterpret_cast<int4*>(stage)[lane] = htab[j * 16 + lane];
        if (lane < ns * kPiecesPerSeg) {
          const PtabPiece q = ptab[j * 16 + lane];
          if (q.soff & 0x80000000u) {  // ragged end of the matrix: plain loads for the tail
            const int s = lane % ns;
            const Seg sg = plan.seg(cache, rb, s);
            const Piece p = (lane < ns) ? make_piece<F>(sg, s, -1, G, 0, K) : make_scale_piece<F>(sg, s, -1, G, 0, K);
            const uint8_t* src = (lane < ns) ? sg.w : sg.s;
            for (int64_t b = p.cs + p.bulk; b < p.end; ++b) data[p.soff + (b - p.cs)] = src[b];
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_expect_tx(&full[st], ttab[j]);
        __syncwarp();
        if (lane < ns * kPiecesPerSeg) {
          const PtabPiece q = ptab[j * 16 + lane];
          if (q.bytes) bulk_g2s(data + (q.soff & 0x7FFFFFFFu), q.src, q.bytes, &full[st]);
        }
      }
    }
    return true;
  }
    for (int rb = blockIdx.x; rb < nblocks; rb += gridDim.x) {
      const int ns = plan.nseg(rb);
      int rs = -1, rl = 0;
      Seg rseg{};
      if (lane < 16) {
        plan.rowmap(rb, lane, rs, rl);
        if (rs >= 0) rseg = plan.seg(cache, rb, rs);
      }
      for (int kc = 0; kc < nkc; ++kc, ++it) {
        if (it % np != pidx) continue;
        const int k0 = kc * KC, k1 = min(K, k0 + KC);
        const bool whole = (k0 == 0 && k1 == K);
        const int st = it % NSTAGE;
        const uint32_t ph = ((it / NSTAGE) & 1) ^ 1;
        if (!mbar_wait(&empty[st], ph, err)) return false;
        uint8_t* stage = stages + st * STAGE_BYTES;
        uint8_t* data = stage + SP::kHdr;
        if (lane < 16) {
          const RowInfo ri = row_info<F>(rseg, rs, rl, G, k0, k1);
          reinterpret_cast<int4*>(stage)[lane] = make_int4(ri.off, ri.sub0, ri.soff, ri.valid);
        }
        // pieces: one per segment (whole rows) or one per row; lane i owns pieces i, i+32, ...
        const int npc = whole ? ns : ns * G.rps;
        uint32_t mybulk = 0;
        for (int i = lane; i < npc; i += 32) {
          const int s = whole ? i : i / G.rps, r = whole ? -1 : i % G.rps;
          const Seg sg = plan.seg(cache, rb, s);
          if (!whole && r >= sg.nrows) continue;
          const Piece p = make_piece<F>(sg, s, r, G, k0, k1);
          mybulk += p.bulk;
          for (int64_t b = p.cs + p.bulk; b < p.end; ++b) data[p.soff + (b - p.cs)] = sg.w[b];
        }
        if (F == FMT_MXFP4) {
          for (int i = lane; i < npc; i += 32) {
            const int s = whole ? i : i / G.rps, r = whole ? -1 : i % G.rps;
            const Seg sg = plan.seg(cache, rb, s);
            if (!whole && r >= sg.nrows) continue;
            const Piece p = make_scale_piece<F>(sg, s, r, G, k0, k1);
            mybulk += p.bulk;
            for (int64_t b = p.cs + p.bulk; b < p.end; ++b) data[p.soff + (b - p.cs)] = sg.s[b];
          }
        }
        uint32_t total = mybulk;
#pragma unroll
        for (int o = 16; o; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
        __syncwarp();
        if (lane == 0) mbar_arrive_expect_tx(&full[st], total);
        __syncwarp();
        for (int i = lane; i < npc; i += 32) {
          const int s = whole ? i : i / G.rps, r = whole ? -1 : i % G.rps;
          const Seg sg = plan.seg(cache, rb, s);
          if (!whole && r >= sg.nrows) continue;
          const Piece p = make_piece<F>(sg, s, r, G, k0, k1);
          if (p.bulk) bulk_g2s(data + p.soff, sg.w + p.cs, p.bulk, &full[st]);
          if (F == FMT_MXFP4) {
            const Piece q = make_scale_piece<F>(sg, s, r, G, k0, k1);
            if (q.bulk) bulk_g2s(data + q.soff, sg.s + q.cs, q.bulk, &full[st]);
          }
        }
      }
    }
  return true;
}

// One stage chunk of one row block for one consumer warp: steps [u_beg, u_end)
// of the chunk (ub = its first 32-block), accumulated into acc.  Shared by the
// stage-ring engine and the warp-owned variant.
template <int F, int MODE, class SP>
__device__ __forceinline__ void consume_chunk(const uint8_t* stage, int u_beg, int u_end, int ub, int nv, int vb,
                                              int v0, int v1, int n_a, int n_b, const uint4* xq, const float4* xsx,
                                              uint8_t* coef, float (&acc)[4], int lane) {
  const int g = lane >> 2, t = lane & 3;
  constexpr bool kKQ = (F == FMT_Q4_K || F == FMT_Q5_K || F == FMT_Q6_K);
  const uint8_t* data = stage + SP::kHdr;
  const int4* hdr = reinterpret_cast<const int4*>(stage);
  const int4 h0 = hdr[g], h1 = hdr[g + 8];
  const RowInfo r0{h0.x, h0.y, h0.z, h0.w}, r1{h1.x, h1.y, h1.z, h1.w};

  // Running per-row positions.  Rows outside the matrix (valid == 0) read
  // the stage from offset 0 instead of branching: every decoded A value is
  // finite (magic f16 <= 1279, e2m1 <= 6), and their fold coefficient is 0.
  // Rows g and g+8 are 8 rows apart and 8*K/32 is a multiple of 8 for any
  // K % 32 == 0, so both rows sit at the same 32-block phase within their
  // superblocks: one sub-block counter serves both.
  using T = FmtT<F>;
  const uint8_t* pA = data + (r0.valid ? r0.off : 0);
  const uint8_t* pB = data + (r1.valid ? r1.off : 0);
  int sA = 0;
  if (kKQ) {
    sA = (r0.valid ? r0.sub0 : r1.sub0) + u_beg;
    pA += (sA >> 3) * T::BB;
    pB += (sA >> 3) * T::BB;
    sA &= 7;
  } else {
    pA += u_beg * T::BB;
    pB += u_beg * T::BB;
  }
  const uint8_t* scA = data + r0.soff + u_beg;  // MXFP4 scale bytes
  const uint8_t* scB = data + r1.soff + u_beg;
  const uint4* xqp = xq + ((size_t)(ub + u_beg) * nv + vb) * 4 + t;
  const float4* xsp = xsx + (size_t)(ub + u_beg) * nv;

  for (int uc = u_beg; uc < u_end; uc += SP::kCoefCh) {
    const int nst = min(SP::kCoefCh, u_end - uc);
    if (F == FMT_Q4_K || F == FMT_Q5_K) {
      // One task per (row, superblock): decode d, dmin and the 12 scale bytes
      // once and emit the coefficients of the sub-blocks that fall in this
      // chunk of steps (16 steps from any phase span at most 3 superblocks).
      __syncwarp();
      float2* cf = reinterpret_cast<float2*>(coef);
      for (int task = lane; task < 48; task += 32) {
        const int m = task / 3, j = task - 3 * (task / 3);
        const int4 q = hdr[m];
        if (!q.w) {
          if (j == 0)
            for (int u = 0; u < nst; ++u) cf[m * SP::kCoefCh + u] = make_float2(0.f, 0.f);
          continue;
        }
        const int sb = ((q.y + uc) >> 3) + j;  // superblock index relative to the row's first
        const int ubase = sb * 8 - q.y - uc;   // chunk step of sub-block 0 of this superblock
        if (ubase >= nst) continue;
        const uint4 hw = *reinterpret_cast<const uint4*>(data + q.x + sb * FmtT<F>::BB);
        const float2 dd = __half22float2(*reinterpret_cast<const __half2*>(&hw.x));
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int u = ubase + i;
          if (u < 0 || u >= nst) continue;
          const int sh = 8 * (i & 3);
          uint32_t sc, mn;
          if (i < 4) {
            sc = (hw.y >> sh) & 63u;
            mn = (hw.z >> sh) & 63u;
          } else {
            sc = ((hw.w >> sh) & 15u) | (((hw.y >> sh) >> 2) & 0x30u);
            mn = (((hw.w >> sh) >> 4) & 15u) | (((hw.z >> sh) >> 2) & 0x30u);
          }
          const float a = dd.x * small_u2f(sc);
          cf[m * SP::kCoefCh + u] = make_float2(a, fmaf(FoldBias<F>::v, a, dd.y * small_u2f(mn)));
        }
      }
      __syncwarp();
    } else if (kKQ) {
      __syncwarp();
#pragma unroll
      for (int e0 = 0; e0 < 16 * SP::kCoefCh; e0 += 32) {
        const int e = e0 + lane;
        const int m = e / SP::kCoefCh, s = e % SP::kCoefCh;
        const int4 q = hdr[m];
        const RowInfo ri{q.x, q.y, q.z, q.w};
        float4 c = make_float4(0.f, 0.f, 0.f, 0.f);
        if (ri.valid && s < nst) c = fold_coef<F>(row_loc<F>(data, ri, uc + s));
        if (F == FMT_Q6_K) reinterpret_cast<float4*>(coef)[m * SP::kCoefCh + s] = c;
        else reinterpret_cast<float2*>(coef)[m * SP::kCoefCh + s] = make_float2(c.x, c.y);
      }
      __syncwarp();
    }
#pragma unroll 2
    for (int s = 0; s < nst; ++s) {
      const uint4 b = *xqp;
      xqp += nv * 4;
      RowLoc la, lb;
      la.blk = pA; la.sub = sA; la.mx_scale = (F == FMT_MXFP4) ? scA[0] : 0u;
      lb.blk = pB; lb.sub = sA; lb.mx_scale = (F == FMT_MXFP4) ? scB[0] : 0u;
      uint32_t pa[4], pb[4];
      decode_a<F>(la, t, pa);
      decode_a<F>(lb, t, pb);
      float c1[4] = {0.f, 0.f, 0.f, 0.f};
      float c2[4] = {0.f, 0.f, 0.f, 0.f};
      const uint32_t a1[4] = {pa[0], pb[0], pa[1], pb[1]};
      const uint32_t a2[4] = {pa[2], pb[2], pa[3], pb[3]};
      mma_f16(c1, a1, b.x, b.y);
      if (F == FMT_Q6_K) mma_f16(c2, a2, b.z, b.w);
      else mma_f16(c1, a2, b.z, b.w);
      float4 ka, kb;
      if (kKQ) {
        if (F == FMT_Q6_K) {
          ka = reinterpret_cast<const float4*>(coef)[g * SP::kCoefCh + s];
          kb = reinterpret_cast<const float4*>(coef)[(g + 8) * SP::kCoefCh + s];
        } else {
          const float2 qa = reinterpret_cast<const float2*>(coef)[g * SP::kCoefCh + s];
          const float2 qb = reinterpret_cast<const float2*>(coef)[(g + 8) * SP::kCoefCh + s];
          ka = make_float4(qa.x, qa.y, 0.f, 0.f);
          kb = make_float4(qb.x, qb.y, 0.f, 0.f);
        }
      } else {
        ka = fold_coef<F>(la);
        kb = fold_coef<F>(lb);
        ka.x = r0.valid ? ka.x : 0.f; ka.y = r0.valid ? ka.y : 0.f;
        kb.x = r1.valid ? kb.x : 0.f; kb.y = r1.valid ? kb.y : 0.f;
      }
      // advance both rows by one 32-element step
      if (kKQ) {
        if (++sA == 8) { sA = 0; pA += T::BB; pB += T::BB; }
      } else {
        pA += T::BB;
        pB += T::BB;
      }
      if (F == FMT_MXFP4) { ++scA; ++scB; }
      auto fold = [&](float& a, float cv1, float cv2, const float4& k, const float4& q) {
        if (F == FMT_Q6_K) {
          a = fmaf(k.x, cv1 * q.x, a);
          a = fmaf(-k.y, q.y, a);
          a = fmaf(k.z, cv2 * q.x, a);
          a = fmaf(-k.w, q.z, a);
        } else if (F == FMT_MXFP4) {
          a = fmaf(k.x * q.x, cv1, a);
        } else {
          a = fmaf(k.x, cv1 * q.x, a);
          a = fmaf(-k.y, q.y, a);
        }
      };
      if (MODE == COLS_DUP) {
        const float4 q0 = xsp[0];
        fold(acc[0], c1[0], c2[0], ka, q0);
        fold(acc[2], c1[2], c2[2], kb, q0);
      } else if (MODE == COLS_FULL) {
        const float4 qv0 = xsp[v0], qv1 = xsp[v1];
        fold(acc[0], c1[0], c2[0], ka, qv0);
        fold(acc[1], c1[1], c2[1], ka, qv1);
        fold(acc[2], c1[2], c2[2], kb, qv0);
        fold(acc[3], c1[3], c2[3], kb, qv1);
      } else {
        const bool oa = n_a & 1, ob = n_b & 1;
        const float4 qa_ = xsp[n_a < 0 ? 0 : n_a], qb_ = xsp[n_b < 0 ? 0 : n_b];
        fold(acc[0], oa ? c1[1] : c1[0], oa ? c2[1] : c2[0], ka, qa_);
        fold(acc[2], ob ? c1[3] : c1[2], ob ? c2[3] : c2[2], kb, qb_);
      }
      xsp += nv;
    }
  }
}

// Consumer warp cw: process this CTA's row blocks of `plan` (its group's share),
// whose stage units start at ring position it0.  Returns false on a timeout.
template <int F, int MODE, int NCW, int NSTAGE, int STAGE_BYTES, int NG, class P>
__device__ __forceinline__ bool eng_consume(const P& plan, const SlotCache* cache, const EngSmem& S, int it0,
                                            const uint4* xq, const float4* xsx, int cw, int lane, int* err) {
  using SP = SmemPlan<NCW, NSTAGE, STAGE_BYTES, MODE, F>;
  constexpr int WPG = NCW / NG;
  static_assert(NCW % NG == 0, "groups must split the consumer warps evenly");
  uint64_t* full = S.full;
  uint64_t* empty = S.empty;
  const StageGeom G = plan.geom;
  const int K = G.K, KC = G.KC;
  const int nkc = (K + KC - 1) / KC;
  const int nblocks = plan.num_blocks();
  uint8_t* stages = S.stages;
  int* cnt = S.cnt;
  float* red = S.red;
  const int nv = plan.num_vectors();
  const int grp = cw / WPG, wg = cw % WPG;
  const int g = lane >> 2, t = lane & 3;
  uint8_t* coef = S.coef + cw * 2048;
  constexpr bool kKQ = (F == FMT_Q4_K || F == FMT_Q5_K || F == FMT_Q6_K);
  int bi = 0;
  for (int rb = blockIdx.x; rb < nblocks; rb += gridDim.x, ++bi) {
    if (bi % NG != grp) continue;
    int it = it0 + bi * nkc;
    int vb, v0, v1, n_a, n_b;
    plan.columns(rb, g, t, vb, v0, v1, n_a, n_b);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};

    for (int kc = 0; kc < nkc; ++kc, ++it) {
      const int k0 = kc * KC, k1 = min(K, k0 + KC);
      const int st = it % NSTAGE;
      const uint32_t ph = (it / NSTAGE) & 1;
      const int Uc = (k1 - k0) / 32, ub = k0 / 32;
      const int u_beg = (wg * Uc) / WPG, u_end = ((wg + 1) * Uc) / WPG;
      if (!mbar_wait(&full[st], ph, err)) return false;
      const uint8_t* stage = stages + st * STAGE_BYTES;
      consume_chunk<F, MODE, SP>(stage, u_beg, u_end, ub, nv, vb, v0, v1, n_a, n_b, xq, xsx, coef, acc, lane);
      if (kc + 1 < nkc) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        continue;
      }
      // Last chunk of the row block: publish partials; the last warp to do so runs
      // the epilogue (fixed summation order, so results are deterministic).  The
      // stage is released only after that, so the partial-sum slot `st` cannot be
      // reused before the epilogue has read it.
      float* rd = red + st * (NCW * SP::kRedW);
      float* mine = rd + wg * SP::kRedW;
      if (MODE == COLS_FULL) {
        mine[g * 8 + 2 * t] = acc[0];
        mine[g * 8 + 2 * t + 1] = acc[1];
        mine[(g + 8) * 8 + 2 * t] = acc[2];
        mine[(g + 8) * 8 + 2 * t + 1] = acc[3];
      } else if (MODE == COLS_DUP) {
        if (t == 0) {
          mine[g] = acc[0];
          mine[g + 8] = acc[2];
        }
      } else {
        if (n_a >= 0 && (n_a >> 1) == t) mine[g] = acc[0];
        if (n_b >= 0 && (n_b >> 1) == t) mine[g + 8] = acc[2];
      }
      __syncwarp();
      int last = 0;
      if (lane == 0) {
        __threadfence_block();
        last = (atomicAdd(&cnt[st], 1) == WPG - 1);
        __threadfence_block();
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      if (last) {
        plan.epilogue(cache, rb, rd, WPG, lane);
        __syncwarp();
        if (lane == 0) cnt[st] = 0;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
  }
  return true;
}

template <int F, int MODE, int NCW, int NSTAGE, int STAGE_BYTES, int NG, class P>
__global__ void __launch_bounds__(32 * (NCW + NSTAGE), 1) qmv_kernel(const P plan) {
  // Waits use only the parity of a stage's phase, so a consumer may wait for
  // ring position p only once position p - NSTAGE has been filled (else it
  // matches that older phase of the same parity and reads another unit).
  // Fills are in ring order and a group waits for p only after consuming its
  // previous position p', so the condition holds when p - p' <= NSTAGE: the
  // largest gap is (NG - 1) * nkc + 1 (the other groups' row blocks), which the
  // launcher keeps <= NSTAGE (nkc = 1 for whole-row plans: NG <= NSTAGE).
  static_assert(NG <= NSTAGE, "more consumer groups than stages aliases mbarrier phases");
  using SP = SmemPlan<NCW, NSTAGE, STAGE_BYTES, MODE, F>;
  constexpr int WPG = NCW / NG;
  extern __shared__ __align__(128) uint8_t smem[];
  EngSmem S;
  S.full = reinterpret_cast<uint64_t*>(smem + SP::off_bars);
  S.empty = S.full + NSTAGE;
  S.cnt = reinterpret_cast<int*>(smem + SP::off_cnt);
  S.red = reinterpret_cast<float*>(smem + SP::off_red);
  S.stages = smem + SP::off_stage;
  S.coef = smem + SP::off_coef;
  SlotCache* cache = reinterpret_cast<SlotCache*>(smem + SP::off_cache);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int K = plan.geom.K;
  const int nv = plan.num_vectors();
  uint8_t* xq_raw = smem + SP::off_x;
  float4* xsx = reinterpret_cast<float4*>(xq_raw + (size_t)(K / 32) * nv * 64);
  int* err = plan.err;
  if (tid == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], WPG);
      S.cnt[s] = 0;
    }
    fence_barrier_init();
  }
  __syncthreads();
  // Warps 0..NSTAGE-1 are producers (producer p fills stage p); the rest consume.
  if (warp < NSTAGE) {
    if (P::kProducerWaits) pdl_wait();
    if (warp == 0) plan.fill_cache(cache, lane);
    named_bar_sync(2, 32 * NSTAGE);  // slot cache ready for every producer
    S.ptab = smem + SP::off_ptab + warp * kPtabBytes;
    int it = 0;
    eng_produce<F, MODE, NCW, NSTAGE, STAGE_BYTES, NG>(plan, cache, S, it, lane, err, NSTAGE, warp);
    return;
  }
  const int ctid = tid - 32 * NSTAGE;
  if (!P::kXIndependent) pdl_wait();
  stage_x<F>(xq_raw, xsx, K, nv, plan.xsrc(), ctid, 32 * NCW);
  named_bar_sync(1, 32 * NCW);
  if (P::kXIndependent) pdl_wait();
  pdl_launch_dependents();
  eng_consume<F, MODE, NCW, NSTAGE, STAGE_BYTES, NG>(plan, cache, S, 0, reinterpret_cast<const uint4*>(xq_raw), xsx,
                                                     warp - NSTAGE, lane, err);
}

// Host-side geometry (excluding the 256-B RowInfo header): stage slot size for a given chunk.
template <int F>
inline int host_slot_bytes(int K, int KC, int rows_per_seg) {
  using T = FmtT<F>;
  const bool whole = (KC >= K);
  const int64_t elems = whole ? (int64_t)rows_per_seg * K : KC;
  int64_t bytes;
  if (F == FMT_MXFP4 || F == FMT_Q8_0) bytes = elems / 32 * T::BB + 32;
  else bytes = (elems / 256 + 2) * T::BB + 32;
  return (int)((bytes + 15) & ~int64_t(15));
}

template <int F>
inline int host_stage_bytes(int K, int KC, int nseg, int rows_per_seg, int& slot, int& sc_base, int& sslot) {
  const bool whole = (KC >= K);
  slot = host_slot_bytes<F>(K, KC, rows_per_seg);
  sc_base = whole ? nseg * slot : nseg * rows_per_seg * slot;
  int total = sc_base;
  sslot = 0;
  if (F == FMT_MXFP4) {
    const int cb = (whole ? K : KC) / 32;
    sslot = ((whole ? rows_per_seg * cb : cb) + 32 + 15) & ~15;
    total += (whole ? nseg : nseg * rows_per_seg) * sslot;
  }
  return total;
}

}  // namespace tsb
