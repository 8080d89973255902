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
    ri.soff = G.sc_base + si * (((G.rps * cb) + 15) & ~15) + lr * cb;
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
template <int F, typename LoadFn>
__device__ void stage_x(uint8_t* xq_raw, float4* xsx, int K, int nv, LoadFn load, int tid, int nthreads) {
  const int U = K / 32;
  const int lane = tid & 31, wid = tid >> 5, nw = nthreads >> 5;
  __half* xq = reinterpret_cast<__half*>(xq_raw);
  int dst = 0;
  for (int t = 0; t < 4; ++t)
    for (int s = 0; s < 8; ++s)
      if (elem_order<F>(t, s) == lane) dst = 8 * t + s;
  for (int job = wid; job < U * nv; job += nw) {
    const int u = job / nv, v = job % nv;
    const float x = load(v, 32 * u + lane);
    float amax = fabsf(x);
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    int e = 0;
    if (amax > 0.f && amax <= 3.0e38f) {
      int ex;
      frexpf(amax, &ex);
      e = ex - 15;
    }
    const __half h = __float2half_rn(ldexpf(x, -e));
    const float hv = __half2float(h);
    xq[(size_t)(u * nv + v) * 32 + dst] = h;
    float s_all = hv, s_lo = (lane < 16) ? hv : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      s_all += __shfl_xor_sync(0xffffffffu, s_all, o);
      s_lo += __shfl_xor_sync(0xffffffffu, s_lo, o);
    }
    if (lane == 0) {
      const float xs = ldexpf(1.f, e);
      if (F == FMT_Q6_K)
        xsx[u * nv + v] = make_float4(xs, s_lo * xs, (s_all - s_lo) * xs, 0.f);
      else
        xsx[u * nv + v] = make_float4(xs, s_all * xs, 0.f, 0.f);
    }
  }
}

// Shared-memory map of one CTA.
template <int NCW, int NSTAGE, int STAGE_BYTES>
struct SmemPlan {
  static constexpr int kCoefCh = 8;  // steps per coefficient chunk
  static constexpr int kRed = 2 * NCW * 128 * 4;
  static constexpr int kCoef = NCW * 16 * kCoefCh * 16;
  static constexpr int kRinfo = NCW * 16 * 16;
  static constexpr int off_bars = 0;
  static constexpr int off_red = 128;
  static constexpr int off_coef = off_red + kRed;
  static constexpr int off_rinfo = off_coef + kCoef;
  static constexpr int off_stage = ((off_rinfo + kRinfo + 127) / 128) * 128;
  static constexpr int off_x = off_stage + NSTAGE * STAGE_BYTES;
  static __host__ __device__ constexpr int x_bytes(int K, int nv) { return (K / 32) * nv * (64 + 16); }
  static __host__ __device__ constexpr int total(int K, int nv) { return off_x + x_bytes(K, nv); }
};

// Plan interface (all device-side, const):
//   int K; StageGeom geom; int* err;
//   static constexpr bool kProducerWaits;   tiles depend on the previous kernel's output
//   int num_vectors() const;                activation vectors (<= 8)
//   float load_x(int v, int k) const;       activation v, element k (fp32)
//   int num_blocks() const;                 row blocks
//   int nseg(int rb) const;  Seg seg(int rb, int s) const;
//   void rowmap(int rb, int m, int& s, int& lr) const;   A-row m -> (segment, row)  (s<0: none)
//   void columns(int rb, int g, int t, int& vb, int& v0, int& v1, int& na, int& nb) const;
//   void epilogue(int rb, const float* red, int nwarps, int ct) const;
//       ct = consumer thread (0 .. 32*NCW-1); red[w*128 + m*8 + n] = warp w's partial sum.
template <int F, int MODE, int NCW, int NSTAGE, int STAGE_BYTES, class P>
__global__ void __launch_bounds__(32 * (NCW + 1), 1) qmv_kernel(const P plan) {
  using SP = SmemPlan<NCW, NSTAGE, STAGE_BYTES>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + SP::off_bars);
  uint64_t* empty = full + NSTAGE;
  float* red = reinterpret_cast<float*>(smem + SP::off_red);
  uint8_t* stages = smem + SP::off_stage;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const StageGeom G = plan.geom;
  const int K = G.K, KC = G.KC;
  const int nkc = (K + KC - 1) / KC;
  const int nv = plan.num_vectors();
  uint8_t* xq_raw = smem + SP::off_x;
  float4* xsx = reinterpret_cast<float4*>(xq_raw + (size_t)(K / 32) * nv * 64);
  int* err = plan.err;

  if (tid == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NCW);
    }
    fence_barrier_init();
  }
  __syncthreads();
  const int nblocks = plan.num_blocks();

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    if (P::kProducerWaits) pdl_wait();
    int it = 0;
    for (int rb = blockIdx.x; rb < nblocks; rb += gridDim.x) {
      const int ns = plan.nseg(rb);
      for (int kc = 0; kc < nkc; ++kc, ++it) {
        const int k0 = kc * KC, k1 = min(K, k0 + KC);
        const bool whole = (k0 == 0 && k1 == K);
        const int st = it % NSTAGE;
        const uint32_t ph = ((it / NSTAGE) & 1) ^ 1;
        if (!mbar_wait(&empty[st], ph, err)) return;
        uint8_t* stage = stages + st * STAGE_BYTES;
        uint32_t total = 0;
        // pass 1: plain-load ragged ends and scales, count bulk bytes
        for (int s = 0; s < ns; ++s) {
          const Seg sg = plan.seg(rb, s);
          const int npr = whole ? 1 : sg.nrows;
          for (int r = 0; r < npr; ++r) {
            const Piece p = make_piece<F>(sg, s, whole ? -1 : r, G, k0, k1);
            total += p.bulk;
            for (int64_t b = p.cs + p.bulk + lane; b < p.end; b += 32) stage[p.soff + (b - p.cs)] = sg.w[b];
          }
          if (F == FMT_MXFP4) {
            const int cb = (k1 - k0) / 32;
            const int base = G.sc_base + s * (((G.rps * cb) + 15) & ~15);
            for (int r = 0; r < sg.nrows; ++r) {
              const uint8_t* sp = sg.s + (sg.row0 + r) * (int64_t)(K / 32) + k0 / 32;
              for (int b = lane; b < cb; b += 32) stage[base + r * cb + b] = sp[b];
            }
          }
        }
        __syncwarp();
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[st], total);
          for (int s = 0; s < ns; ++s) {
            const Seg sg = plan.seg(rb, s);
            const int npr = whole ? 1 : sg.nrows;
            for (int r = 0; r < npr; ++r) {
              const Piece p = make_piece<F>(sg, s, whole ? -1 : r, G, k0, k1);
              if (p.bulk) bulk_g2s(stage + p.soff, sg.w + p.cs, p.bulk, &full[st]);
            }
          }
        }
      }
    }
    return;
  }

  // ------------------------------ consumers ------------------------------
  const int ctid = tid - 32;
  pdl_wait();
  stage_x<F>(xq_raw, xsx, K, nv, [&](int v, int k) { return plan.load_x(v, k); }, ctid, 32 * NCW);
  named_bar_sync(1, 32 * NCW);
  pdl_launch_dependents();

  const int cw = warp - 1;
  const int g = lane >> 2, t = lane & 3;
  float4* coef = reinterpret_cast<float4*>(smem + SP::off_coef) + cw * 16 * SP::kCoefCh;
  int4* rinfo = reinterpret_cast<int4*>(smem + SP::off_rinfo) + cw * 16;
  const uint4* xq = reinterpret_cast<const uint4*>(xq_raw);
  constexpr bool kKQ = (F == FMT_Q4_K || F == FMT_Q5_K || F == FMT_Q6_K);

  int it = 0, blk = 0;
  for (int rb = blockIdx.x; rb < nblocks; rb += gridDim.x, ++blk) {
    int vb, v0, v1, n_a, n_b;
    plan.columns(rb, g, t, vb, v0, v1, n_a, n_b);
    // this lane's two rows (A rows g and g+8) and their segments
    int sa, la_r, sb, lb_r;
    plan.rowmap(rb, g, sa, la_r);
    plan.rowmap(rb, g + 8, sb, lb_r);
    Seg sega{}, segb{};
    if (sa >= 0) sega = plan.seg(rb, sa);
    if (sb >= 0) segb = plan.seg(rb, sb);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};

    for (int kc = 0; kc < nkc; ++kc, ++it) {
      const int k0 = kc * KC, k1 = min(K, k0 + KC);
      const int st = it % NSTAGE;
      const uint32_t ph = (it / NSTAGE) & 1;
      const RowInfo r0 = row_info<F>(sega, sa, la_r, G, k0, k1);
      const RowInfo r1 = row_info<F>(segb, sb, lb_r, G, k0, k1);
      if (kKQ) {
        // row table for the coefficient pass: lane m < 16 fills entry m
        __syncwarp();
        if (lane < 16) {
          int s_, l_;
          plan.rowmap(rb, lane, s_, l_);
          Seg sg{};
          if (s_ >= 0) sg = plan.seg(rb, s_);
          const RowInfo ri = row_info<F>(sg, s_, l_, G, k0, k1);
          rinfo[lane] = make_int4(ri.off, ri.sub0, ri.soff, ri.valid);
        }
      }
      const int Uc = (k1 - k0) / 32, ub = k0 / 32;
      const int u_beg = (cw * Uc) / NCW, u_end = ((cw + 1) * Uc) / NCW;
      if (!mbar_wait(&full[st], ph, err)) return;
      const uint8_t* stage = stages + st * STAGE_BYTES;

      for (int uc = u_beg; uc < u_end; uc += SP::kCoefCh) {
        const int nst = min(SP::kCoefCh, u_end - uc);
        if (kKQ) {
          __syncwarp();
          for (int e = lane; e < 16 * nst; e += 32) {
            const int m = e / nst, s = e % nst;
            const int4 q = rinfo[m];
            const RowInfo ri{q.x, q.y, q.z, q.w};
            float4 c = make_float4(0.f, 0.f, 0.f, 0.f);
            if (ri.valid) c = fold_coef<F>(row_loc<F>(stage, ri, uc + s));
            coef[m * SP::kCoefCh + s] = c;
          }
          __syncwarp();
        }
#pragma unroll 2
        for (int s = 0; s < nst; ++s) {
          const int u = uc + s;   // step within the chunk
          const int ug = ub + u;  // step within the row
          const uint4 b = xq[((size_t)ug * nv + vb) * 4 + t];
          uint32_t pa[4] = {kMagic, kMagic, kMagic, kMagic};
          uint32_t pb[4] = {kMagic, kMagic, kMagic, kMagic};
          RowLoc la{}, lb{};
          if (r0.valid) { la = row_loc<F>(stage, r0, u); decode_a<F>(la, t, pa); }
          if (r1.valid) { lb = row_loc<F>(stage, r1, u); decode_a<F>(lb, t, pb); }
          if (F == FMT_MXFP4) {
            if (!r0.valid) pa[0] = pa[1] = pa[2] = pa[3] = 0u;
            if (!r1.valid) pb[0] = pb[1] = pb[2] = pb[3] = 0u;
          }
          float c1[4] = {0.f, 0.f, 0.f, 0.f};
          float c2[4] = {0.f, 0.f, 0.f, 0.f};
          const uint32_t a1[4] = {pa[0], pb[0], pa[1], pb[1]};
          const uint32_t a2[4] = {pa[2], pb[2], pa[3], pb[3]};
          mma_f16(c1, a1, b.x, b.y);
          if (F == FMT_Q6_K) mma_f16(c2, a2, b.z, b.w);
          else mma_f16(c1, a2, b.z, b.w);
          float4 ka, kb;
          if (kKQ) {
            ka = coef[g * SP::kCoefCh + s];
            kb = coef[(g + 8) * SP::kCoefCh + s];
          } else {
            ka = r0.valid ? fold_coef<F>(la) : make_float4(0.f, 0.f, 0.f, 0.f);
            kb = r1.valid ? fold_coef<F>(lb) : make_float4(0.f, 0.f, 0.f, 0.f);
          }
          auto fold = [&](float& a, float cv1, float cv2, const float4& k, int v) {
            const float4 q = xsx[ug * nv + v];
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
            fold(acc[0], c1[0], c2[0], ka, 0);
            fold(acc[2], c1[2], c2[2], kb, 0);
          } else if (MODE == COLS_FULL) {
            fold(acc[0], c1[0], c2[0], ka, v0);
            fold(acc[1], c1[1], c2[1], ka, v1);
            fold(acc[2], c1[2], c2[2], kb, v0);
            fold(acc[3], c1[3], c2[3], kb, v1);
          } else {
            const bool oa = n_a & 1, ob = n_b & 1;
            fold(acc[0], oa ? c1[1] : c1[0], oa ? c2[1] : c2[0], ka, n_a < 0 ? 0 : n_a);
            fold(acc[2], ob ? c1[3] : c1[2], ob ? c2[3] : c2[2], kb, n_b < 0 ? 0 : n_b);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }

    // cross-warp reduction of this row block
    float* rd = red + (blk & 1) * (NCW * 128);
    float* mine = rd + cw * 128;
    if (MODE == COLS_DIAG) {
      if (n_a >= 0 && (n_a >> 1) == t) mine[g * 8 + n_a] = acc[0];
      if (n_b >= 0 && (n_b >> 1) == t) mine[(g + 8) * 8 + n_b] = acc[2];
    } else {
      mine[g * 8 + 2 * t] = acc[0];
      mine[g * 8 + 2 * t + 1] = acc[1];
      mine[(g + 8) * 8 + 2 * t] = acc[2];
      mine[(g + 8) * 8 + 2 * t + 1] = acc[3];
    }
    named_bar_sync(1, 32 * NCW);
    plan.epilogue(rb, rd, NCW, ctid);
  }
}

// Host-side geometry: stage slot size for a given chunk.
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
inline int host_stage_bytes(int K, int KC, int nseg, int rows_per_seg, int& slot, int& sc_base) {
  const bool whole = (KC >= K);
  slot = host_slot_bytes<F>(K, KC, rows_per_seg);
  sc_base = whole ? nseg * slot : nseg * rows_per_seg * slot;
  int total = sc_base;
  if (F == FMT_MXFP4) {
    const int cb = (whole ? K : KC) / 32;
    total += nseg * (((rows_per_seg * cb) + 15) & ~15);
  }
  return total;
}

}  // namespace tsb
