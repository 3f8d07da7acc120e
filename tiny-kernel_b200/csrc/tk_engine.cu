// tk_engine.cu -- persistent, warp-specialised, TMA-fed INT4 fused-dequant GEMV engine
// for sm_100a.
//
// Computes the qmatmul_int4 contraction of the reference (src/kernels/shaders.zig:442-501)
//     y[m][n] = sum_g scale[g][n] * sum_{k in g} x[m][k] * (q[k][n] - zero[g][n])
// on the reference's packed layout, and the INT4 Llama FFN built from it
// (src/bench.zig:266-341 gate/up composition plus the down projection).
//
// Design (one CTA per SM: 8 consumer warps + weight, record and flush warps):
//  * A work unit is one k-step (8 packed rows = 16 k) of a 1024-column wide tile of one
//    matrix.  Within a phase, units are ordered tile-major, matrix, group, step; CTA b of P
//    owns units [U*b/P, U*(b+1)/P) (stream-K), so every SM streams the same number of bytes.
//    Units are visited group by group ("items"); the iteration is incremental.
//  * The CTA has one ring of S stages (full + empty mbarrier each).  A stage holds one
//    item: the packed rows of the group as 1040-byte TMA box rows (u64 tensor map; one
//    box for a whole group, or one per k-step for a partial group) -- long rows are what
//    lets TMA stream near the HBM read limit -- plus the group's f16 scales (2 KB), zero
//    points (512 B) and activation record.  Weight-warp lane 0 issues the boxes, lanes 8-9
//    the scales and zero points; the record warp adds the record.
//  * Consumer warp j computes slice j (128 columns) of every stage.
//    - m <= 2 (the dp2a path): lane l owns columns 4l..4l+3 of the slice.  It copies its
//      packed bytes of every row, the scales, zero points and the activation record into
//      registers and releases the stage at once (a held stage is a stage not streaming),
//      then computes.  Two rows' bytes are interleaved with one PRMT per column pair so a
//      column's two k pairs sit in adjacent bytes; masking gives the low nibbles (even k)
//      and 16 x the high nibbles (odd k); dp2a multiplies them by the activations
//      quantised to int16 per group (scale 2^-e, max |x| * 2^e in [2^14, 2^15)), two k per
//      instruction, into exact int32 sums.  Per group:
//        v = 2^-e * (sum_even + (sum_odd16 >> 4) - z * sum_k xq_k)     (exact integers)
//        y += scale * v.
//    - m = 3, 4 (the int8 tensor-core path): m16n8k32 u8 x s8 MMAs on nibble planes
//      against activations split into int8 hi + lo / 256 parts.
//  * Split-K partial sums go to a scratch buffer and each finished segment bumps a counter
//    per 128-column sub-tile.  An output sub-tile is reduced (in phase and CTA order, so
//    deterministically) by the warp that counts its last segment, which stores y
//    (+ residual).  The gate/up sub-tiles are not reduced by their producers: the record warp
//    of every CTA that needs an h sub-tile waits for its counter to be complete, reduces it
//    in the same fixed order, applies silu(gate) * up and writes its items' records straight
//    into their stages -- two L2 round trips between the last gate/up segment and the down
//    projection.  The last CTA to finish returns those counters to zero.
//  * No grid-wide barrier: every CTA builds its own prologue records.  The FFN splits
//    gate/up into tile ranges so the down projection of an early range overlaps the
//    production of the last one.
// Every spin-wait is bounded by a global-timer timeout and reports through p.err.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <mutex>

#include "tk_dp2a.cuh"
#include "tk_engine.h"
#include "tk_internal.h"
#include "tk_ptx.cuh"

namespace tk {

namespace {

constexpr int kNC = kSlices;  // consumer warps: one per 128-column slice

// The phase list as the kernel reads it: a copy in shared memory (dynamic indexing into the
// kernel parameters would go through the constant cache on every access).
struct PhaseTable {
  const PhaseParams* ph;
  int n;
};

// ---- stream-K bookkeeping --------------------------------------------------------------

// Stream-K arithmetic is 32-bit: the host admits a phase only when units * CTAs < 2^31, so
// every product below fits (64-bit division is a long software sequence on the GPU).

// CTA whose stream-K range holds unit u (ranges [U*b/W, U*(b+1)/W), all non-empty)
__device__ __forceinline__ int cta_of_unit(unsigned u, unsigned units, unsigned W) {
  return (int)(((u + 1) * W - 1) / units);
}

__device__ __forceinline__ unsigned phase_ctas(const PhaseParams& P, unsigned Wtot) {
  return (unsigned)P.units < Wtot ? (unsigned)P.units : Wtot;
}

// Number of CTA ranges of phase P holding units of (global) column unit cu = wide tile *
// nmat + matrix; 0 when the phase does not cover cu.
__device__ __forceinline__ int nseg_of_cu(const PhaseParams& P, int cu, unsigned Wtot) {
  const int c = cu - P.wt0 * P.nmat;
  if (c < 0 || c >= P.tiles * P.nmat) return 0;
  const unsigned W = phase_ctas(P, Wtot), U = (unsigned)P.units;
  const unsigned per = (unsigned)(P.groups * P.spg);
  const unsigned a = (unsigned)c * per;
  return cta_of_unit(a + per - 1, U, W) - cta_of_unit(a, U, W) + 1;
}

// Segments of column unit cu summed over the phases that reduce together with phase ph.
__device__ __forceinline__ int red_segments(const PhaseTable& T, int ph, int cu, unsigned Wtot) {
  const PhaseParams& P = T.ph[ph];
  int n = 0;
  for (int q = P.red_first; q < P.red_first + P.red_count; ++q) n += nseg_of_cu(T.ph[q], cu, Wtot);
  return n;
}

// Index within its reduction of CTA b's segment of column unit cu in phase ph (earlier
// phases of the reduction first, then CTA order).
__device__ __forceinline__ int segment_index(const PhaseTable& T, int ph, int cu, int b,
                                             unsigned Wtot) {
  const PhaseParams& P = T.ph[ph];
  int off = 0;
  for (int q = P.red_first; q < ph; ++q) off += nseg_of_cu(T.ph[q], cu, Wtot);
  const unsigned W = phase_ctas(P, Wtot);
  const unsigned a = (unsigned)(cu - P.wt0 * P.nmat) * (unsigned)(P.groups * P.spg);
  return off + b - cta_of_unit(a, (unsigned)P.units, W);
}

__device__ __forceinline__ int active_slices(const PhaseParams& P, int wtile) {
  const int rem = (P.N - wtile * kWideCols) / kTileCols;
  return rem < kSlices ? rem : kSlices;
}

// Partial sums of segment `seg` of column unit cu, slice `slice`: [MT][128] floats.
template <int MT>
__device__ __forceinline__ float* partial_slot(const PhaseParams& P, int cu, int seg, int slice) {
  return P.partials + (((size_t)cu * P.maxseg + seg) * kSlices + slice) * MT * kTileCols;
}

// Walks one CTA's items (one group of one wide tile each) through all phases.  The fields of
// the current phase that per-item paths read are copied in at the phase switch: a shared-memory
// read on a per-item path waits behind the consumers' bulk of stage reads.
struct ItemIter {
  int ph;       // phase of the current item; == nphases when exhausted
  int i, n;     // index within the phase, items in the phase
  int cu, grp;  // global column unit (tile * nmat + mat) and global group of the item
  int s0, s1;   // k-step range of the current item within its group
  int last_s1;  // s1 of the phase's last item
  int nmat, g0, g1, spg, N, frag_bytes, epi;
  bool rec_pro;  // the phase's records are the prologue's (else built from partial sums)
};

// Slices of the current item's wide tile that hold columns (8 except in a ragged last tile).
__device__ __forceinline__ int item_slices(const ItemIter& it) {
  const int rem = (it.N - (it.cu >> (it.nmat - 1)) * kWideCols) / kTileCols;
  return rem < kSlices ? rem : kSlices;
}

__device__ __forceinline__ void iter_seek(ItemIter& it, const PhaseTable& T, int w, unsigned Wtot) {
  while (it.ph < T.n) {
    const PhaseParams& P = T.ph[it.ph];
    const unsigned W = phase_ctas(P, Wtot), U = (unsigned)P.units;
    if ((unsigned)w < W) {
      const unsigned beg = U * (unsigned)w / W, end = U * (unsigned)(w + 1) / W;
      const unsigned fg0 = beg / (unsigned)P.spg, fgl = (end - 1) / (unsigned)P.spg;
      const unsigned cl = fg0 / (unsigned)P.groups;
      it.nmat = P.nmat;
      it.g0 = P.g0;
      it.g1 = P.g1;
      it.spg = P.spg;
      it.N = P.N;
      it.frag_bytes = P.frag_bytes;
      it.epi = P.epi;
      it.rec_pro = P.src_count == 0;
      it.i = 0;
      it.n = (int)(fgl - fg0 + 1);
      it.cu = (int)cl + P.wt0 * P.nmat;
      it.grp = P.g0 + (int)(fg0 - cl * (unsigned)P.groups);
      it.s0 = (int)(beg - fg0 * (unsigned)P.spg);
      it.last_s1 = (int)(end - fgl * (unsigned)P.spg);
      it.s1 = it.n == 1 ? it.last_s1 : P.spg;
      return;
    }
    ++it.ph;
  }
}

__device__ __forceinline__ void iter_start(ItemIter& it, const PhaseTable& T, int w, unsigned Wtot) {
  it.ph = 0;
  it.i = it.n = it.cu = it.grp = it.s0 = it.s1 = it.last_s1 = 0;
  it.nmat = 1;
  it.g0 = it.g1 = it.spg = it.N = it.frag_bytes = it.epi = 0;
  it.rec_pro = true;
  iter_seek(it, T, w, Wtot);
}

__device__ __forceinline__ void iter_next(ItemIter& it, const PhaseTable& T, int w, unsigned Wtot) {
  if (++it.i < it.n) {
    if (++it.grp == it.g1) {
      it.grp = it.g0;
      ++it.cu;
    }
    it.s0 = 0;
    it.s1 = it.i == it.n - 1 ? it.last_s1 : it.spg;
    return;
  }
  ++it.ph;
  iter_seek(it, T, w, Wtot);
}

// Bytes the weight warp's copies bring into a stage for item `it` (box rows, scales, zeros);
// the record warp adds the activation record (P.frag_bytes).
__device__ __forceinline__ uint32_t item_weight_bytes(const ItemIter& it) {
  return (uint32_t)((it.s1 - it.s0) * kStepRows * kRowBytes +
                    item_slices(it) * (kScaleBytes + kZeroBytes));
}

// The weight warp's copy of its current phase's pointers.
struct WeightPhase {
  int map_base;
  const uint16_t* scales[kMaxMats];
  const uint8_t* zeros[kMaxMats];
};

// Weight-warp lane `lane` issues its share of item `it`'s weight-side copies: lane 0 the TMA
// box(es), lane 8 the scales, lane 9 the zero points.
__device__ __forceinline__ void issue_weights(const TmapPack& maps, const WeightPhase& W,
                                              const ItemIter& it, uint8_t* tile, uint8_t* aux,
                                              uint64_t* bar, uint64_t pol, int lane) {
  const int mat = it.cu & (it.nmat - 1);
  const int wt = it.cu >> (it.nmat - 1);
  const int col0 = wt * kWideCols;
  if (lane == 0) {
    const int row0 = it.grp * it.spg * kStepRows;
    const int x = wt * (kWideCols / 8);  // u64 element of the tile's first byte
    if (it.s0 == 0 && it.s1 == it.spg) {
      tma_load_2d(tile, &maps.map[W.map_base + 2 * mat], bar, x, row0, pol);
    } else {
      for (int s = it.s0; s < it.s1; ++s)
        tma_load_2d(tile + s * kStepRows * kRowBytes, &maps.map[W.map_base + 2 * mat + 1], bar, x,
                    row0 + s * kStepRows, pol);
    }
  } else if (lane == 8) {
    bulk_load(aux, W.scales[mat] + (size_t)it.grp * it.N + col0,
              (uint32_t)(item_slices(it) * kScaleBytes), bar, pol);
  } else if (lane == 9) {
    bulk_load(aux + kSlices * kScaleBytes, W.zeros[mat] + (size_t)it.grp * (it.N / 2) + col0 / 2,
              (uint32_t)(item_slices(it) * kZeroBytes), bar, pol);
  }
}

__device__ __forceinline__ uint8_t* frag_slot(uint8_t* aux) {
  return aux + kSlices * (kScaleBytes + kZeroBytes);
}

// The record warp's copy of its current phase's record source.
struct RecordPhase {
  const uint8_t* frag_in;
  long long frag_cta_stride;
  int src_first, src_count;
};

__device__ __forceinline__ void issue_frag(const RecordPhase& R, const ItemIter& it, int b,
                                           uint8_t* aux, uint64_t* bar, uint64_t pol) {
  bulk_load(frag_slot(aux), R.frag_in + b * R.frag_cta_stride + (size_t)it.grp * it.frag_bytes,
            (uint32_t)it.frag_bytes, bar, pol);
}

__device__ __forceinline__ void trace_event(const EngineParams& p, int ev) {
  if (p.trace) p.trace[(size_t)blockIdx.x * kTraceEvents + ev] = global_timer_ns();
}

// ---- activation records ------------------------------------------------------------------

// int8 tensor-core path.  Warp-collective: lane l holds v[0..3] = values 4l..4l+3 of a
// 128-value activation chunk of token `tok`.  Writes the records of the chunk's 128/gs
// groups into `rec` (the record of the chunk's first group, records `rec_bytes` apart).  Per
// k pair p the MMA sees x[2p+1] against the high nibble and x[2p] against the low nibble of
// the packed byte.  The group's values are scaled by 2^e (max |x| of the group in [32, 64))
// and split into int8 hi + lo / 256 parts.
template <int MT>
__device__ __forceinline__ void build_records_mma(const float (&v)[4], int tok, int gs,
                                                  uint8_t* rec, int rec_bytes, int lane,
                                                  int gi_only) {
  const int gl = gs >> 2;  // lanes per group
  // k pairs 2l and 2l + 1 of the chunk: odd k (high nibble) and even k (low nibble)
  const float b[4] = {v[1], v[0], v[3], v[2]};
  float mx = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
  for (int off = 1; off < gl; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  // e with max |x| * 2^e in [32, 64): from the exponent field (subnormal or zero maxima and
  // non-finite values are clamped to the range the scale stays a normal power of two in)
  int e = 6 - ((int)((__float_as_uint(mx) >> 23) & 0xffu) - 126);
  e = e < -100 ? -100 : (e > 100 ? 100 : e);
  const float up = __uint_as_float((uint32_t)(127 + e) << 23);    // 2^e
  const float down = __uint_as_float((uint32_t)(127 - e) << 23);  // 2^-e
  int hi[4], lo[4];
  int sh = 0, sl = 0;  // sums of the hi and lo parts (zero-point term)
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float w = b[i] * up;
    hi[i] = __float2int_rn(w);
    int l = __float2int_rn((w - (float)hi[i]) * 256.f);
    lo[i] = l < -127 ? -127 : (l > 127 ? 127 : l);
    sh += hi[i];
    sl += lo[i];
  }
  // this lane's two k pairs are bytes 2 j .. 2 j + 1 (j = (lambda >> 2) & 1) of word h of t:
  // 16-bit pieces {odd hi, odd lo, even hi, even lo}, two per shuffle word
  const uint32_t p_odd = (uint32_t)(hi[0] & 0xff) | ((uint32_t)(hi[2] & 0xff) << 8) |
                         ((uint32_t)(lo[0] & 0xff) << 16) | ((uint32_t)(lo[2] & 0xff) << 24);
  const uint32_t p_even = (uint32_t)(hi[1] & 0xff) | ((uint32_t)(hi[3] & 0xff) << 8) |
                          ((uint32_t)(lo[1] & 0xff) << 16) | ((uint32_t)(lo[3] & 0xff) << 24);
  const int gi = lane / gl, lg = lane - gi * gl;  // group within the chunk, lane within it
  const int kbl = lg & 15;                        // lane within its 32-pair block
  const int kb = lg >> 4;
  const int t = kbl & 3, j = (kbl >> 2) & 1, h = kbl >> 3;
  // the partner lane holds the other two bytes of the same words (none when gs == 16)
  uint32_t q_odd = __shfl_xor_sync(0xffffffffu, p_odd, 4);
  uint32_t q_even = __shfl_xor_sync(0xffffffffu, p_even, 4);
  if (gl <= 4) q_odd = q_even = 0u;
  uint8_t* r = rec + (size_t)gi * rec_bytes;
  const bool store = gi_only < 0 || gi == gi_only;
  if (j == 0 && store) {
    const uint32_t o1h = (p_odd & 0xffffu) | (q_odd << 16);
    const uint32_t o1l = (p_odd >> 16) | (q_odd & 0xffff0000u);
    const uint32_t o2h = (p_even & 0xffffu) | (q_even << 16);
    const uint32_t o2l = (p_even >> 16) | (q_even & 0xffff0000u);
    uint32_t* bh = reinterpret_cast<uint32_t*>(r) + ((kb * 4 + t) * 2 * MT + 2 * tok) * 4;
    uint32_t* bl = bh + 4;  // the lo column of the same token
    bh[h] = o1h;
    bh[2 + h] = o2h;
    bl[h] = o1l;
    bl[2 + h] = o2l;
    if (gs <= 32) {  // kappa half 1 is beyond the group: zero
      bh[1] = 0u;
      bh[3] = 0u;
      bl[1] = 0u;
      bl[3] = 0u;
    }
  }
  // per 16-k step (4 lanes): the sums of the quantised values' hi and lo parts, so the
  // zero-point term -z * sum(x) is formed exactly from the same values the MMA sees
  sh += __shfl_xor_sync(0xffffffffu, sh, 1);
  sl += __shfl_xor_sync(0xffffffffu, sl, 1);
  sh += __shfl_xor_sync(0xffffffffu, sh, 2);
  sl += __shfl_xor_sync(0xffffffffu, sl, 2);
  const int spg = gs >> 4;
  const int kbg = spg >= 4 ? spg / 4 : 1;
  int2* sums = reinterpret_cast<int2*>(r + 128 * MT * kbg);
  if ((lg & 3) == 0 && store) sums[(lg >> 2) * MT + tok] = make_int2(sh, sl);
  if (lg == 0 && store) reinterpret_cast<float*>(sums + spg * MT)[tok] = down;
}

// Records of the groups of a 128-value chunk (all of them, or only group gi_only: the other
// lanes still take part in the shuffles but store nothing).
template <int MT>
__device__ __forceinline__ void build_records(const float (&v)[4], int tok, int gs, uint8_t* rec,
                                              int rec_bytes, int lane, int gi_only = -1) {
  if constexpr (MT <= 2) build_records_dp<MT>(v, tok, gs, rec, rec_bytes, lane, gi_only);
  else build_records_mma<MT>(v, tok, gs, rec, rec_bytes, lane, gi_only);
}

// ---- int8 tensor-core path (m = 3, 4) ------------------------------------------------------

// Row (k pair within a 32-pair block) that MMA K index kappa = 16 h + 4 t + i reads:
// 16 h + 2 t + (i & 1) + 8 (i >> 1).  For a fixed i the 4 t values land 2 rows apart, so the
// 16-byte loads of a quarter warp (g in {0,1}, t in 0..3) hit 8 distinct 16-byte bank slots of
// the 1040-byte-strided stage rows.
__device__ __forceinline__ int kappa_row(int h, int t, int i) {
  return 16 * h + 2 * t + (i & 1) + 8 * (i >> 1);
}

// The 32 k pairs (rows) of block `kb` of one slice for this lane, 16 MMAs of m16n8k32 u8 x s8:
// MMA j (0..7) covers columns 16 g + 2 j, 16 g + 2 j + 1 (A rows g, g + 8) for B-column class
// j / (2 MT); each j gets the high-nibble MMA and the low-nibble MMA into its own accumulator.
// Rows outside [r0, r1) (a partial item) or beyond `nrows` (groups of < 64 k) read as zero.
template <int MT>
__device__ __forceinline__ void compute_kblock(const uint8_t* blk, const uint4* recb, int kb0,
                                               int nrows, int r0, int r1, int g, int t,
                                               const uint32_t (&cls_mask)[4 / MT], int cB,
                                               int (&D)[8][4]) {
  uint4 R[2][4];
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int rr = kappa_row(h, t, i);
      const int ar = kb0 + rr;
      R[h][i] = (rr < nrows && ar >= r0 && ar < r1)
                    ? *reinterpret_cast<const uint4*>(blk + rr * kRowBytes + 16 * g)
                    : make_uint4(0u, 0u, 0u, 0u);
    }
  const uint4 bf = recb[t * 2 * MT + cB];
  constexpr int NCL = 4 / MT;
  uint32_t b1x[NCL], b1y[NCL], b2x[NCL], b2y[NCL];
#pragma unroll
  for (int c = 0; c < NCL; ++c) {
    b1x[c] = bf.x & cls_mask[c];
    b1y[c] = bf.y & cls_mask[c];
    b2x[c] = bf.z & cls_mask[c];
    b2y[c] = bf.w & cls_mask[c];
  }
#pragma unroll
  for (int wd = 0; wd < 4; ++wd) {  // word wd: columns 16 g + 4 wd .. + 3
    uint32_t C0[4], C1[4];
    transpose4x4(word(R[0][0], wd), word(R[0][1], wd), word(R[0][2], wd), word(R[0][3], wd), C0);
    transpose4x4(word(R[1][0], wd), word(R[1][1], wd), word(R[1][2], wd), word(R[1][3], wd), C1);
#pragma unroll
    for (int pr = 0; pr < 2; ++pr) {
      const int j = 2 * wd + pr;
      const uint32_t a0 = C0[2 * pr], a1 = C0[2 * pr + 1], a2 = C1[2 * pr], a3 = C1[2 * pr + 1];
      mma_16832_u8s8(D[j], (a0 >> 4) & 0x0F0F0F0Fu, (a1 >> 4) & 0x0F0F0F0Fu,
                     (a2 >> 4) & 0x0F0F0F0Fu, (a3 >> 4) & 0x0F0F0F0Fu, b1x[j / (2 * MT)],
                     b1y[j / (2 * MT)]);
      mma_16832_u8s8(D[j], a0 & 0x0F0F0F0Fu, a1 & 0x0F0F0F0Fu, a2 & 0x0F0F0F0Fu,
                     a3 & 0x0F0F0F0Fu, b2x[j / (2 * MT)], b2y[j / (2 * MT)]);
    }
  }
}

// Applies the group's scales and zero points to the MMA sums and resets them.  The sums of
// row pair r are spread over the classes c (accumulator c * 2 MT + r); the other classes hold
// zeros in this lane's positions, so they are folded by addition.
template <int MT>
__device__ __forceinline__ void group_epilogue(const uint8_t* scales, const uint8_t* zeros,
                                               const int2* sums, const float* gscale, int s0,
                                               int s1, int tokE, int colbase, int (&D)[8][4],
                                               float (&y)[4 * MT]) {
  constexpr int NCL = 4 / MT;
  int sbh = 0, sbl = 0;
  for (int s = s0; s < s1; ++s) {
    const int2 v = sums[s * MT + tokE];
    sbh += v.x;
    sbl += v.y;
  }
  const float esc = gscale[tokE];
  const __half* sc = reinterpret_cast<const __half*>(scales) + colbase;
  const uint8_t* zp = zeros + colbase / 2;
#pragma unroll
  for (int r = 0; r < 2 * MT; ++r) {
    int d0 = D[r][0], d1 = D[r][1], d2 = D[r][2], d3 = D[r][3];
#pragma unroll
    for (int c = 1; c < NCL; ++c) {
      d0 += D[c * 2 * MT + r][0];
      d1 += D[c * 2 * MT + r][1];
      d2 += D[c * 2 * MT + r][2];
      d3 += D[c * 2 * MT + r][3];
    }
    const float2 sf = __half22float2(*reinterpret_cast<const __half2*>(sc + 2 * r));
    const int zz = zp[r];
    const int za = zz & 15, zb = zz >> 4;
    // sum_k xq_k * (q_k - z), exact in int32 per part, then one rounding each
    const float va = fmaf((float)(d1 - za * sbl), 0x1p-8f, (float)(d0 - za * sbh)) * esc;
    const float vb = fmaf((float)(d3 - zb * sbl), 0x1p-8f, (float)(d2 - zb * sbh)) * esc;
    y[2 * r] = fmaf(sf.x, va, y[2 * r]);
    y[2 * r + 1] = fmaf(sf.y, vb, y[2 * r + 1]);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) D[j][0] = D[j][1] = D[j][2] = D[j][3] = 0;
}

// ---- split-K reduction -----------------------------------------------------------------------

// Stores this lane's partial sums of a slice: dp2a path y[4 m + i] -> [m][4 lane + i];
// tensor-core path y[4 i + c] -> [tokE][colbase + 4 i + c].
template <int MT>
__device__ __forceinline__ void store_partials(float* slot, const float (&y)[4 * MT], int lane,
                                               int tokE, int colbase) {
  if constexpr (MT <= 2) {
#pragma unroll
    for (int m = 0; m < MT; ++m)
      *reinterpret_cast<float4*>(slot + m * kTileCols + 4 * lane) =
          make_float4(y[4 * m], y[4 * m + 1], y[4 * m + 2], y[4 * m + 3]);
  } else {
    float* dst = slot + tokE * kTileCols + colbase;
#pragma unroll
    for (int i = 0; i < MT; ++i)
      *reinterpret_cast<float4*>(dst + 4 * i) =
          make_float4(y[4 * i], y[4 * i + 1], y[4 * i + 2], y[4 * i + 3]);
  }
}

// Sums this lane's 4 columns of token `tok` over the segments of one sub-tile of a reduction:
// ns0 segments of column unit cu0 into a0 and, when two_mats, ns1 segments of cu0 + 1 into a1
// (a single matrix takes 16 segments per batch into a0).  16 loads in flight per batch; the
// sums run in a fixed order, so every warp that reduces a sub-tile gets the same bits.
template <int MT>
__device__ __forceinline__ void sum_partials(const PhaseParams& P, int cu0, int ns0,
                                             int ns1, bool two_mats, int slice, int tok, int lane,
                                             float4& a0, float4& a1) {
  constexpr size_t kSegStride = (size_t)kSlices * MT * kTileCols;
  constexpr int kB = 8;
  const float* base0 = partial_slot<MT>(P, cu0, 0, slice) + tok * kTileCols + 4 * lane;
  const float* base1 =
      two_mats ? partial_slot<MT>(P, cu0 + 1, 0, slice) + tok * kTileCols + 4 * lane : base0;
  if (!two_mats) ns1 = ns0;
  const int step = two_mats ? kB : 2 * kB;
  a0 = make_float4(0.f, 0.f, 0.f, 0.f);
  a1 = a0;
  for (int s0 = 0; s0 < ns0 || s0 < ns1; s0 += step) {
    const int s1 = two_mats ? s0 : s0 + kB;  // first segment of the batch's second half
    float4 v0[kB], v1[kB];
#pragma unroll
    for (int i = 0; i < kB; ++i) {
      v0[i] = s0 + i < ns0 ? __ldcg(reinterpret_cast<const float4*>(base0 + (s0 + i) * kSegStride))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
      v1[i] = s1 + i < ns1 ? __ldcg(reinterpret_cast<const float4*>(base1 + (s1 + i) * kSegStride))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float4 t0 = make_float4(0.f, 0.f, 0.f, 0.f), t1 = t0;
#pragma unroll
    for (int i = 0; i < kB; ++i) {
      t0.x += v0[i].x;
      t0.y += v0[i].y;
      t0.z += v0[i].z;
      t0.w += v0[i].w;
      t1.x += v1[i].x;
      t1.y += v1[i].y;
      t1.z += v1[i].z;
      t1.w += v1[i].w;
    }
    a0.x += t0.x;
    a0.y += t0.y;
    a0.z += t0.z;
    a0.w += t0.w;
    if (two_mats) {
      a1.x += t1.x;
      a1.y += t1.y;
      a1.z += t1.z;
      a1.w += t1.w;
    } else {
      a0.x += t1.x;
      a0.y += t1.y;
      a0.z += t1.z;
      a0.w += t1.w;
    }
  }
}

// The last warp to finish an output sub-tile (kEpiStore): reduction of the partials + store.
template <int MT, int GS>
__device__ void fixup_tile(const EngineParams& p, const PhaseTable& T, int ph, int wt, int slice,
                           unsigned Wtot, int lane) {
  const PhaseParams& P = T.ph[ph];
  const int cu0 = wt * P.nmat;
  const int ns0 = red_segments(T, ph, cu0, Wtot);
  const int ns1 = P.nmat > 1 ? red_segments(T, ph, cu0 + 1, Wtot) : 0;
  const int col = wt * kWideCols + slice * kTileCols + 4 * lane;
  for (int tok = 0; tok < MT; ++tok) {
    float4 a0, a1;
    sum_partials<MT>(P, cu0, ns0, ns1, P.nmat > 1, slice, tok, lane, a0, a1);
    if (tok < p.m) {
      if (P.residual) {
        const float4 r = *reinterpret_cast<const float4*>(P.residual + (size_t)tok * P.ldr + col);
        a0.x = r.x + a0.x;
        a0.y = r.y + a0.y;
        a0.z = r.z + a0.z;
        a0.w = r.w + a0.w;
      }
      *reinterpret_cast<float4*>(P.out + (size_t)tok * P.ldo + col) = a0;
    }
  }
}

// h = silu(gate) * up for this lane's 4 columns of sub-tile (wt, slice) of the kEpiSiluMul
// phase `a` (gate/up column units 2 wt, 2 wt + 1), every token (0 beyond the live ones).
template <int MT>
__device__ __forceinline__ void reduce_silu_mul(const PhaseTable& T, int a, int wt, int slice,
                                                unsigned Wtot, int lane, int m,
                                                float (&h)[MT][4]) {
  const PhaseParams& A = T.ph[a];
  const int cu0 = 2 * wt;
  const int ns0 = red_segments(T, a, cu0, Wtot);
  const int ns1 = red_segments(T, a, cu0 + 1, Wtot);
#pragma unroll
  for (int tok = 0; tok < MT; ++tok) {
    float4 g, u;
    sum_partials<MT>(A, cu0, ns0, ns1, true, slice, tok, lane, g, u);
    const float gv[4] = {g.x, g.y, g.z, g.w}, uv[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) h[tok][i] = tok < m ? gv[i] / (1.0f + expf(-gv[i])) * uv[i] : 0.f;
  }
}

// Counts one finished segment of sub-tile (wt, slice) of phase ph's reduction; returns true
// to the last of them.
__device__ __forceinline__ bool count_segment(const PhaseTable& T, int ph, int wt, int slice,
                                              unsigned Wtot) {
  const PhaseParams& P = T.ph[ph];
  unsigned total = 0;
  for (int mi = 0; mi < P.nmat; ++mi)
    total += (unsigned)red_segments(T, ph, wt * P.nmat + mi, Wtot);
  const unsigned prev = atomicAdd(&P.counters[wt * kSlices + slice], 1u);
  return prev == total - 1;
}

// Consumer warps: x (optionally rmsnorm'ed, src/kernels/shaders.zig:16-56) -> records.
// x and the norm weight are read first and the weight producer is held at named barrier 2
// until every consumer has them in registers: reads issued after the weight stream starts
// queue behind megabytes of TMA traffic.
template <int MT, int GS>
__device__ void prologue(const EngineParams& p, int warp, int lane, float* s_red, float* s_rms,
                         uint8_t* rec0s) {
  const int nchunks = p.K0 / kTileCols;
  constexpr int kLocal = 4;  // 128-value chunks held in registers per consumer warp and token
  float4 xv[MT][kLocal], wv[kLocal];
  float ss[MT];
#pragma unroll
  for (int i = 0; i < kLocal; ++i) {
    const int ch = warp + i * kNC;
    const bool in = ch < nchunks;
    wv[i] = (in && p.do_norm) ? *reinterpret_cast<const float4*>(p.norm_w + ch * kTileCols + 4 * lane)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int tok = 0; tok < MT; ++tok)
      xv[tok][i] = (in && tok < p.m) ? *reinterpret_cast<const float4*>(
                                           p.x + (size_t)tok * p.ldx + ch * kTileCols + 4 * lane)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int tok = 0; tok < MT; ++tok) {
    float v = 0.f;
#pragma unroll
    for (int i = 0; i < kLocal; ++i) {
      const float4 a = xv[tok][i];
      v = fmaf(a.x, a.x, fmaf(a.y, a.y, fmaf(a.z, a.z, fmaf(a.w, a.w, v))));
    }
    // chunks beyond the register window (K0 > kLocal * kNC * 128) are read again later
    if (tok < p.m)
      for (int ch = warp + kLocal * kNC; ch < nchunks; ch += kNC) {
        const float4 a =
            *reinterpret_cast<const float4*>(p.x + (size_t)tok * p.ldx + ch * kTileCols + 4 * lane);
        v = fmaf(a.x, a.x, fmaf(a.y, a.y, fmaf(a.z, a.z, fmaf(a.w, a.w, v))));
      }
    ss[tok] = v;
  }
  // every consumer thread has its x values: release the weight producer
  named_barrier_arrive(2, (kNC + 1) * 32);
  float rms[MT];
#pragma unroll
  for (int tok = 0; tok < MT; ++tok) rms[tok] = 1.f;
  if (p.do_norm) {
#pragma unroll
    for (int tok = 0; tok < MT; ++tok) {
      float v = ss[tok];
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == 0) s_red[tok * kNC + warp] = v;
    }
    named_barrier(1, kNC * 32);
    if (threadIdx.x < MT) {
      float tot = 0.f;
      for (int i = 0; i < kNC; ++i) tot += s_red[threadIdx.x * kNC + i];
      s_rms[threadIdx.x] = rsqrtf(tot / (float)p.K0 + p.eps);
    }
    named_barrier(1, kNC * 32);
#pragma unroll
    for (int tok = 0; tok < MT; ++tok) rms[tok] = s_rms[tok];
  }
  uint8_t* recs = p.rec0_smem ? rec0s : p.frag0 + (long long)blockIdx.x * p.frag0_cta_stride;
  auto emit = [&](float4 a, float4 w, int tok, int ch) {
    float v[4] = {a.x, a.y, a.z, a.w};
    if (p.do_norm) {
      v[0] = v[0] * rms[tok] * w.x;
      v[1] = v[1] * rms[tok] * w.y;
      v[2] = v[2] * rms[tok] * w.z;
      v[3] = v[3] * rms[tok] * w.w;
    }
    build_records<MT>(v, tok, GS, recs + (size_t)(ch * kTileCols / GS) * p.frag0_bytes,
                      p.frag0_bytes, lane);
  };
#pragma unroll
  for (int tok = 0; tok < MT; ++tok) {
#pragma unroll
    for (int i = 0; i < kLocal; ++i) {
      const int ch = warp + i * kNC;
      if (ch < nchunks) emit(xv[tok][i], wv[i], tok, ch);
    }
    for (int ch = warp + kLocal * kNC; ch < nchunks; ch += kNC) {
      const float4 a = tok < p.m ? *reinterpret_cast<const float4*>(p.x + (size_t)tok * p.ldx +
                                                                     ch * kTileCols + 4 * lane)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 w = p.do_norm
                           ? *reinterpret_cast<const float4*>(p.norm_w + ch * kTileCols + 4 * lane)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
      emit(a, w, tok, ch);
    }
  }
  // records in global memory are read back by this CTA's record warp through the async proxy
  if (!p.rec0_smem) fence_proxy_async();
}

// Bounded warp-collective wait for an mbarrier phase that also gives up when the CTA aborts.
__device__ __forceinline__ bool wait_slot(uint64_t* bar, uint32_t parity, const volatile int* abort,
                                          unsigned* err, unsigned long long timeout_ns) {
  bool done = mbar_try_wait(bar, parity);
  if (!done) {
    const uint64_t t0 = global_timer_ns();
    while (!(done = mbar_try_wait(bar, parity))) {
      if (*abort) break;
      if (global_timer_ns() - t0 > timeout_ns) {
        if ((threadIdx.x & 31) == 0) atomicOr(err, kErrTmaWait);
        break;
      }
    }
  }
  return __all_sync(0xffffffffu, done);
}

// Warp roles: warps 0..kNC-1 consume stages, warp kNC (weight warp) streams the packed weights,
// scales and zero points of every item, warp kNC+1 (record warp) copies each item's activation
// record once it is ready, warp kNC+2 (flush warp) completes every split-K segment: the
// consumers only store their partial sums and move on; the flush warp makes them visible and
// counts them, and for each sub-tile whose last segment it counted it posts a fixup job to the
// consumer warp of that slice, which runs it between items (the eight slices' reductions run in
// parallel and no consumer waits on a global round trip of the counting).  Each stage's full
// barrier takes one arrival from each producer warp.
constexpr int kWeightWarp = kNC;
constexpr int kRecordWarp = kNC + 1;
constexpr int kFlushWarp = kNC + 2;
constexpr int kThreads = (kNC + 3) * 32;
constexpr int kFlushSlots = 4;  // flush events in flight between the consumers and the flush warp
constexpr int kJobSlots = 16;   // fixup jobs in flight from the flush warp to one consumer warp

// An item ends a split-K segment: the last item of its column unit or of the CTA's range.
__device__ __forceinline__ bool ends_segment(const ItemIter& it) {
  return it.grp == it.g1 - 1 || it.i == it.n - 1;
}

template <int MT, int GS>
__global__ void __launch_bounds__(kThreads, 1)
    int4_engine_kernel(const __grid_constant__ TmapPack maps, const __grid_constant__ EngineParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ PhaseParams s_ph[kMaxPhases];
  __shared__ float s_red[MT * kNC];
  __shared__ float s_rms[MT];
  __shared__ volatile long long s_armed;   // items whose weights the weight warp has armed
  __shared__ volatile int s_wdone;         // weight warp has left its loop (s_armed final)
  __shared__ volatile int s_records;       // this CTA's prologue records are written
  __shared__ volatile int s_abort;
  __shared__ volatile int s_never;         // stays 0: a wait that must not be cut short
  __shared__ uint64_t s_fbar[kFlushSlots];  // flush events (kNC consumer arrivals)
  __shared__ volatile int s_fdone;         // flush events the flush warp has completed
  __shared__ volatile int s_job[kNC][kJobSlots];  // fixup jobs per slice: (phase << 16) | tile
  __shared__ volatile int s_job_head[kNC];        // jobs posted (flush warp)
  __shared__ volatile int s_job_tail[kNC];        // jobs done (consumer warp)
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.stages;
  uint8_t* tiles = smem;
  uint8_t* auxs = smem + (size_t)S * p.tile_stage_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(auxs + (size_t)S * p.aux_stage_bytes);
  uint64_t* empty = full + S;
  uint8_t* rec0s = reinterpret_cast<uint8_t*>(empty + S) + 16 - (smem_addr(empty + S) & 15u);
  {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(p.ph);
    uint32_t* dst = reinterpret_cast<uint32_t*>(s_ph);
    const int words = p.nphases * (int)(sizeof(PhaseParams) / 4);
    for (int i = threadIdx.x; i < words; i += blockDim.x) dst[i] = src[i];
  }
  const PhaseTable T{s_ph, p.nphases};
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 2);
      mbar_init(&empty[i], kNC);
    }
    for (int i = 0; i < kFlushSlots; ++i) mbar_init(&s_fbar[i], kNC);
    s_fdone = 0;
    for (int i = 0; i < kNC; ++i) s_job_head[i] = s_job_tail[i] = 0;
    fence_mbar_init();
    s_records = 0;
    s_abort = 0;
    s_never = 0;
    s_armed = 0;
    s_wdone = 0;
    trace_event(p, 0);
  }
  __syncthreads();
  const unsigned Ptot = gridDim.x;
  const int b = blockIdx.x;
  // consumer ring position (function scope for the drain at the end)
  int slot = 0;
  uint32_t parity = 0;
  long long consumed = 0;

  if (warp == kWeightWarp) {
    // ---------------------------- weight producer warp ---------------------------------
    const uint64_t pol_stream = l2_evict_first();
    ItemIter wi;
    iter_start(wi, T, b, Ptot);
    long long G = 0;
    int wslot = 0;
    uint32_t wround = 0;
    // The first two stages go out at once; the rest wait until the consumers have read x
    // (reads issued behind megabytes of stage traffic would stall the prologue).
    constexpr long long kEarlyStages = 2;
    bool x_read = false;
    WeightPhase W{};
    int wph = -1;
    while (wi.ph < T.n) {
      if (!x_read && G >= kEarlyStages) {
        named_barrier(2, (kNC + 1) * 32);
        x_read = true;
      }
      if (wround > 0 && !wait_slot(&empty[wslot], (wround - 1) & 1, &s_abort, p.err, p.timeout_ns)) {
        s_abort = 1;
        break;
      }
      if (s_abort) break;
      if (wi.ph != wph) {
        wph = wi.ph;
        const PhaseParams& P = T.ph[wph];
        W.map_base = P.map_base;
        for (int i = 0; i < kMaxMats; ++i) {
          W.scales[i] = P.scales[i];
          W.zeros[i] = P.zeros[i];
        }
        // The items of a phase fed by partial sums wait for those sums (the gate/up -> down
        // transition) while HBM has nothing to stream: bring all of this CTA's items of the
        // phase into L2 now, so that their copies into the ring come from L2 afterwards.
        if (p.prefetch_l2 && !wi.rec_pro && lane == 0) {
          ItemIter pi = wi;
          for (int n = 0; pi.ph == wph && n < 64; ++n) {
            const int mat = pi.cu & (pi.nmat - 1);
            const int wt = pi.cu >> (pi.nmat - 1);
            tma_prefetch_2d(&maps.map[W.map_base + 2 * mat], wt * (kWideCols / 8),
                            pi.grp * pi.spg * kStepRows);
            iter_next(pi, T, b, Ptot);
          }
        }
      }
      if (lane == 0) {
        if (G == 0) trace_event(p, 7);
        mbar_arrive_expect_tx(&full[wslot], item_weight_bytes(wi));
      }
      __syncwarp();
      issue_weights(maps, W, wi, tiles + (size_t)wslot * p.tile_stage_bytes,
                    auxs + (size_t)wslot * p.aux_stage_bytes, &full[wslot], pol_stream, lane);
      __syncwarp();
      ++G;
      if (lane == 0) s_armed = G;
      iter_next(wi, T, b, Ptot);
      if (++wslot == S) {
        wslot = 0;
        ++wround;
      }
    }
    if (!x_read) named_barrier(2, (kNC + 1) * 32);
    if (lane == 0) {
      s_armed = G;
      __threadfence_block();
      s_wdone = 1;
      trace_event(p, 8);
    }
  } else if (warp == kRecordWarp) {
    // ---------------------------- record producer warp ---------------------------------
    // Prologue records: already in shared memory (plain arrival) or copied per item from this
    // CTA's global copy.  Records of h: once the gate/up segment counter of the item's h
    // sub-tile is complete, the warp reduces the sub-tile (kept for the sub-tile's other group)
    // and writes the item's record straight into the stage.
    const uint64_t pol_keep = l2_evict_last();
    ItemIter fi;
    iter_start(fi, T, b, Ptot);
    long long F = 0;
    int fslot = 0;
    bool aborted = false;
    uint64_t t_wait = 0;
    RecordPhase RP{};
    int rph = -1;
    int h_sub = -1;   // h sub-tile whose values are in hv
    int h_src = 0;    // its producing phase
    float hv[MT][4];  // this lane's 4 h values of h_sub, per token
    unsigned src_done = 0;  // producing phases seen complete (bit per phase): no more polls
    while (fi.ph < T.n) {
      if (s_abort) {
        aborted = true;
        break;
      }
      if (fi.ph != rph) {
        rph = fi.ph;
        const PhaseParams& P = T.ph[rph];
        RP.frag_in = P.frag_in;
        RP.frag_cta_stride = P.frag_cta_stride;
        RP.src_first = P.src_first;
        RP.src_count = P.src_count;
      }
      // only items whose weights are armed (their slot is free and the full barrier is in
      // the phase this arrival belongs to)
      bool go = F < s_armed;
      if (go && fi.rec_pro && p.rec0_smem) {
        // the consumers read this item's record from shared memory: complete the arrival
        if (lane == 0) mbar_arrive(&full[fslot]);
        __syncwarp();
        ++F;
        iter_next(fi, T, b, Ptot);
        fslot = fslot + 1 == S ? 0 : fslot + 1;
        t_wait = 0;
        continue;
      }
      if (go && fi.rec_pro) {
        go = s_records != 0;
        if (go) {
          fence_proxy_async();  // records were written by generic stores
          if (lane == 0) {
            uint8_t* aux = auxs + (size_t)fslot * p.aux_stage_bytes;
            mbar_arrive_expect_tx(&full[fslot], (uint32_t)fi.frag_bytes);
            issue_frag(RP, fi, b, aux, &full[fslot], pol_keep);
          }
          __syncwarp();
        }
      } else if (go) {
        const int h0 = fi.grp * GS;  // first h column of the item's group
        const int wt_h = h0 / kWideCols, sl_h = (h0 % kWideCols) / kTileCols;
        const int sub = wt_h * kSlices + sl_h;
        if (sub != h_sub) {
          int a = RP.src_first;
          while (a + 1 < RP.src_first + RP.src_count && wt_h >= T.ph[a].wt1) ++a;
          const PhaseParams& A = T.ph[a];
          if (!(src_done >> a & 1u)) {
            // the sub-tile's count, and the whole producing phase's (one complete phase
            // means no more polls for its sub-tiles)
            const unsigned total = (unsigned)(red_segments(T, a, 2 * wt_h, Ptot) +
                                              red_segments(T, a, 2 * wt_h + 1, Ptot));
            const unsigned ptotal = (unsigned)A.done_total;
            unsigned v = 0, pv = 0;
            if (lane == 0) {
              v = ld_acquire_u32(&A.counters[sub]);
              pv = ld_acquire_u32(&p.phase_done[a]);
            }
            v = __shfl_sync(0xffffffffu, v, 0);
            pv = __shfl_sync(0xffffffffu, pv, 0);
            if (pv == ptotal) src_done |= 1u << a;
            go = v == total || pv == ptotal;
          }
          if (go) {
            reduce_silu_mul<MT>(T, a, wt_h, sl_h, Ptot, lane, p.m, hv);
            h_sub = sub;
            h_src = a;
          }
        }
        if (go) {
          const int gi = (h0 % kTileCols) / GS;  // the item's group within the sub-tile
          uint8_t* rec = frag_slot(auxs + (size_t)fslot * p.aux_stage_bytes);
#pragma unroll
          for (int tok = 0; tok < MT; ++tok)
            build_records<MT>(hv[tok], tok, GS, rec - (size_t)gi * fi.frag_bytes, fi.frag_bytes,
                              lane, gi);
          // h itself, once: by the item of output tile 0
          const PhaseParams& A = T.ph[h_src];
          if (A.out && fi.cu == 0 && lane / (GS / 4) == gi) {
            for (int tok = 0; tok < p.m && tok < MT; ++tok)
              *reinterpret_cast<float4*>(A.out + (size_t)tok * A.ldo + wt_h * kWideCols +
                                         sl_h * kTileCols + 4 * lane) =
                  make_float4(hv[tok][0], hv[tok][1], hv[tok][2], hv[tok][3]);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&full[fslot]);
        }
      }
      if (go) {
        ++F;
        iter_next(fi, T, b, Ptot);
        fslot = fslot + 1 == S ? 0 : fslot + 1;
        t_wait = 0;
      } else {
        const uint64_t now = global_timer_ns();
        if (t_wait == 0) {
          t_wait = now;
        } else if (now - t_wait > p.timeout_ns) {
          if (lane == 0) atomicOr(p.err, kErrFlagWait);
          s_abort = 1;
          aborted = true;
          break;
        }
        __nanosleep(32);
      }
    }
    if (aborted) {
      // Complete every stage the weight warp armed (a plain arrival in place of the record) so
      // that every copy in flight lands before the CTA exits.
      const uint64_t t0 = global_timer_ns();
      while (!s_wdone && global_timer_ns() - t0 < p.timeout_ns) __nanosleep(64);
      const long long G = s_armed;
      for (; F < G; ++F) {
        if (lane == 0) mbar_arrive(&full[fslot]);
        fslot = fslot + 1 == S ? 0 : fslot + 1;
      }
    }
  } else if (warp == kFlushWarp) {
    // ------------------------------- flush warp ----------------------------------------
    ItemIter hi;
    iter_start(hi, T, b, Ptot);
    int k = 0;
    bool fok = true;
    while (fok && hi.ph < T.n) {
      if (ends_segment(hi)) {
        const PhaseParams& P = T.ph[hi.ph];
        if (!wait_slot(&s_fbar[k % kFlushSlots], (uint32_t)(k / kFlushSlots) & 1u, &s_abort, p.err,
                       p.timeout_ns)) {
          s_abort = 1;
          break;
        }
        __threadfence();  // the consumers' partial sums (acquired through the barrier)
        const int wt = hi.cu >> (P.nmat - 1);
        const int ns = active_slices(P, wt);
        if (P.epi == kEpiSiluMul) {
          // the consumers of h reduce it once the sub-tile's count is complete
          if (lane < ns) atomicAdd(&P.counters[wt * kSlices + lane], 1u);
          if (lane == 0) atomicAdd(&p.phase_done[hi.ph], (unsigned)ns);
          __syncwarp();
          if (lane == 0) s_fdone = k + 1;
          ++k;
          iter_next(hi, T, b, Ptot);
          continue;
        }
        const bool last = lane < ns && count_segment(T, hi.ph, wt, lane, Ptot);
        if (__ballot_sync(0xffffffffu, last)) __threadfence();  // the other CTAs' partials
        if (last) {
          // lane = slice: post the fixup to that slice's consumer warp
          const int h = s_job_head[lane];
          const uint64_t t0 = global_timer_ns();
          while (h - s_job_tail[lane] >= kJobSlots && !s_abort) {
            if (global_timer_ns() - t0 > p.timeout_ns) {
              atomicOr(p.err, kErrFlagWait);
              s_abort = 1;
              break;
            }
          }
          s_job[lane][h % kJobSlots] = (hi.ph << 16) | wt;
          __threadfence_block();
          s_job_head[lane] = h + 1;
        }
        fok = __all_sync(0xffffffffu, !s_abort);
        if (lane == 0) s_fdone = k + 1;
        ++k;
      }
      iter_next(hi, T, b, Ptot);
    }
  } else {
    // ------------------------------- consumer warps ------------------------------------
    const int slice = warp;
    // tensor-core path lane roles
    const int g = lane >> 2, t = lane & 3, q = g >> 1;
    const int cB = 2 * (q % MT) + (g & 1);
    const int tokE = t % MT;
    const int colbase = 16 * g + 4 * MT * (t / MT);
    uint32_t cls_mask[4 / MT];
#pragma unroll
    for (int c = 0; c < 4 / MT; ++c) cls_mask[c] = (q / MT == c) ? 0xffffffffu : 0u;

    ItemIter it;
    iter_start(it, T, b, Ptot);
    bool ok = true;
    int fk = 0;  // flush events handed to the flush warp
    // Fixup jobs the flush warp posted for this slice: reduce the sub-tile's partials, run its
    // epilogue and return its counter to zero for the next launch.
    int job_tail = 0;  // jobs of this slice run so far (s_job_tail mirrors it for the flush warp)
    auto run_jobs = [&]() {
      for (;;) {
        const int h = __shfl_sync(0xffffffffu, lane == 0 ? s_job_head[slice] : 0, 0);
        if (job_tail == h) break;
        const int job = s_job[slice][job_tail % kJobSlots];
        __threadfence_block();
        const int jph = job >> 16, jwt = job & 0xffff;
        fixup_tile<MT, GS>(p, T, jph, jwt, slice, Ptot, lane);
        __syncwarp();
        if (lane == 0) atomicExch(&T.ph[jph].counters[jwt * kSlices + slice], 0u);
        ++job_tail;
        __syncwarp();
        if (lane == 0) s_job_tail[slice] = job_tail;
      }
    };
    // Runs fixup jobs until the flush warp has completed `n` flush events (bounded; gives up
    // on an abort).  Lane 0 decides, so the warp leaves the loop together.
    auto wait_flushes = [&](int n) {
      const uint64_t t0 = global_timer_ns();
      for (;;) {
        int st = 0;
        if (lane == 0) {
          if (s_fdone >= n) st = 1;
          else if (s_abort) st = 2;
          else if (global_timer_ns() - t0 > p.timeout_ns) {
            atomicOr(p.err, kErrFlagWait);
            s_abort = 1;
            st = 2;
          }
        }
        st = __shfl_sync(0xffffffffu, st, 0);
        run_jobs();
        if (st) break;
      }
    };
    // Waits for stage `sl` in phase `par`; runs fixup jobs meanwhile (another CTA may be waiting
    // for the records one of them produces).  Returns false on an abort or a timeout.
    auto wait_full = [&](int sl, uint32_t par) -> bool {
      if (__all_sync(0xffffffffu, mbar_try_wait(&full[sl], par))) return true;
      const uint64_t t0 = global_timer_ns();
      for (;;) {
        run_jobs();
        if (__all_sync(0xffffffffu, mbar_try_wait_hint(&full[sl], par, 256))) return true;
        int st = 0;
        if (lane == 0) {
          if (s_abort) st = 1;
          else if (global_timer_ns() - t0 > p.timeout_ns) {
            atomicOr(p.err, kErrTmaWait);
            st = 1;
          }
        }
        if (__shfl_sync(0xffffffffu, st, 0)) return false;
      }
    };
    // Ends a split-K segment: stores this slice's partial sums and hands the segment to the
    // flush warp (which counts it; the reduction runs later as a fixup job).
    float y[4 * MT];
#pragma unroll
    for (int i = 0; i < 4 * MT; ++i) y[i] = 0.f;
    auto hand_off = [&](const PhaseParams& P, int ph, int cu, bool active) {
      if (active)
        store_partials<MT>(partial_slot<MT>(P, cu, segment_index(T, ph, cu, b, Ptot), slice), y,
                           lane, tokE, colbase);
#pragma unroll
      for (int i = 0; i < 4 * MT; ++i) y[i] = 0.f;
      __syncwarp();
      // the event slot is free once the flush warp has completed event fk - kFlushSlots
      wait_flushes(fk - kFlushSlots + 1);
      if (lane == 0) mbar_arrive(&s_fbar[fk % kFlushSlots]);
      ++fk;
    };
    // Stage pointers of the item in slot sl.
    auto stage_tile = [&](int sl) {
      return tiles + (size_t)sl * p.tile_stage_bytes + slice * kTileCols;
    };
    auto stage_aux = [&](int sl) { return auxs + (size_t)sl * p.aux_stage_bytes; };
    const bool rec0_smem = p.rec0_smem != 0;
    auto item_rec = [&](const ItemIter& x, int sl) -> const uint8_t* {
      return (x.rec_pro && rec0_smem) ? rec0s + (size_t)x.grp * x.frag_bytes
                                      : frag_slot(stage_aux(sl));
    };

    prologue<MT, GS>(p, warp, lane, s_red, s_rms, rec0s);
    named_barrier(1, kNC * 32);
    if (threadIdx.x == 0) {
      __threadfence_block();
      s_records = 1;
      trace_event(p, 1);
    }

    if constexpr (MT <= 2) {
      // Software-pipelined over chunks of HB rows: the shared-memory loads of the next chunk
      // (possibly of the next item) are issued before the dp2a work of the current one, and a
      // stage is released as soon as its last chunk is loaded.
      constexpr int R = GS / 2;                    // packed rows per item
      constexpr int HB = R <= 32 ? R / 2 : 16;     // rows per chunk
      constexpr int NCH = R / HB;                  // chunks per item (2 or 4)
      uint32_t wA[HB], wB[HB];
      uint4 XA[MT][HB / 4], XB[MT][HB / 4];
      DpMeta<MT> Mc, Mn;
      bool have = it.ph < T.n;
      if (have) {
        if (!wait_full(slot, parity)) {
          ok = false;
          s_abort = 1;
          have = false;
        } else {
          if (threadIdx.x == 0) trace_event(p, 9);
          const uint8_t* rec = item_rec(it, slot);
          dp_load_meta<MT, GS>(stage_aux(slot), rec, slice, lane, it.s0, it.s1, Mc);
          dp_load_rows<HB>(stage_tile(slot), 0, it.s0 * kStepRows, it.s1 * kStepRows, lane, wA);
          dp_load_x<MT, HB>(rec, dp_tok_stride(GS), 0, XA);
        }
      }
      while (have) {
        const int r0 = it.s0 * kStepRows, r1 = it.s1 * kStepRows;
        const uint8_t* tl = stage_tile(slot);
        const uint8_t* rec = item_rec(it, slot);
        const bool seg_end = ends_segment(it);
        // the fixup-job queue head, read now and looked at after this item's work
        const int jh = lane == 0 ? s_job_head[slice] : 0;
        ItemIter nx = it;
        iter_next(nx, T, b, Ptot);
        const int nslot = slot + 1 == S ? 0 : slot + 1;
        const uint32_t npar = slot + 1 == S ? parity ^ 1u : parity;
        const bool prefetch = !seg_end && nx.ph < T.n;
        bool next_loaded = false;
        int aL[MT][4], aH[MT][4];
#pragma unroll
        for (int m = 0; m < MT; ++m)
#pragma unroll
          for (int i = 0; i < 4; ++i) aL[m][i] = aH[m][i] = 0;
#pragma unroll
        for (int c = 0; c < NCH; c += 2) {
          dp_load_rows<HB>(tl, (c + 1) * HB, r0, r1, lane, wB);
          dp_load_x<MT, HB>(rec, dp_tok_stride(GS), (c + 1) * HB, XB);
          bool nready = false;
          if (c + 2 == NCH) {
            // every byte of this stage is loaded (in issue order before the arrival)
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            // probe the next stage now; the answer is looked at after this chunk's work
            if (prefetch) nready = mbar_test_wait(&full[nslot], npar);
          }
          dp_compute<MT, HB>(wA, XA, aL, aH);
          if (c + 2 < NCH) {
            dp_load_rows<HB>(tl, (c + 2) * HB, r0, r1, lane, wA);
            dp_load_x<MT, HB>(rec, dp_tok_stride(GS), (c + 2) * HB, XA);
          } else if (prefetch) {
            // the next item's first chunk, while this item's last chunk computes (a segment
            // end is handed off first: other CTAs may wait for it)
            if (!__all_sync(0xffffffffu, nready) && !wait_full(nslot, npar)) {
              ok = false;
            } else {
              const uint8_t* nrec = item_rec(nx, nslot);
              dp_load_meta<MT, GS>(stage_aux(nslot), nrec, slice, lane, nx.s0, nx.s1, Mn);
              dp_load_rows<HB>(stage_tile(nslot), 0, nx.s0 * kStepRows, nx.s1 * kStepRows, lane, wA);
              dp_load_x<MT, HB>(nrec, dp_tok_stride(GS), 0, XA);
              next_loaded = true;
            }
          }
          dp_compute<MT, HB>(wB, XB, aL, aH);
        }
        dp_epilogue<MT>(Mc, aL, aH, y);
        ++consumed;
        slot = nslot;  // ring position of item `consumed` (the drain after an error starts here)
        parity = npar;
        if (seg_end) hand_off(T.ph[it.ph], it.ph, it.cu, slice < item_slices(it));
        if (__shfl_sync(0xffffffffu, jh, 0) != job_tail) run_jobs();
        if (!ok) {
          s_abort = 1;
          break;
        }
        if (nx.ph >= T.n) break;
        if (!next_loaded) {
          if (!wait_full(slot, parity)) {
            ok = false;
            s_abort = 1;
            break;
          }
          const uint8_t* nrec = item_rec(nx, slot);
          dp_load_meta<MT, GS>(stage_aux(slot), nrec, slice, lane, nx.s0, nx.s1, Mn);
          dp_load_rows<HB>(stage_tile(slot), 0, nx.s0 * kStepRows, nx.s1 * kStepRows, lane, wA);
          dp_load_x<MT, HB>(nrec, dp_tok_stride(GS), 0, XA);
        }
        it = nx;
        Mc = Mn;
      }
    } else {
      int D[8][4];
#pragma unroll
      for (int r = 0; r < 8; ++r) D[r][0] = D[r][1] = D[r][2] = D[r][3] = 0;
      while (ok && it.ph < T.n) {
        if (!wait_full(slot, parity)) {
          ok = false;
          s_abort = 1;
          break;
        }
        if (consumed == 0 && threadIdx.x == 0) trace_event(p, 9);
        const bool active = slice < item_slices(it);
        const uint8_t* ax = stage_aux(slot);
        const uint8_t* tl = stage_tile(slot);
        const uint8_t* rec = item_rec(it, slot);
        if (active) {
          constexpr int spg = GS / 16;
          constexpr int kbg = spg >= 4 ? spg / 4 : 1;    // 32-pair blocks per group
          constexpr int nrows = spg >= 4 ? 32 : 8 * spg;  // valid rows per block
          const uint4* rb = reinterpret_cast<const uint4*>(rec);
          const int r0 = it.s0 * kStepRows, r1 = it.s1 * kStepRows;
          for (int kb = 0; kb < kbg; ++kb) {
            if (kb * 32 >= r1 || kb * 32 + 32 <= r0) continue;
            compute_kblock<MT>(tl + (size_t)kb * 32 * kRowBytes, rb + kb * 4 * 2 * MT, kb * 32,
                               nrows, r0, r1, g, t, cls_mask, cB, D);
          }
          const int2* sums = reinterpret_cast<const int2*>(rec + 128 * MT * kbg);
          group_epilogue<MT>(ax + slice * kScaleBytes,
                             ax + kSlices * kScaleBytes + slice * kZeroBytes, sums,
                             reinterpret_cast<const float*>(sums + spg * MT), it.s0, it.s1,
                             tokE, colbase, D, y);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        ++consumed;
        if (++slot == S) {
          slot = 0;
          parity ^= 1u;
        }
        const int cu = it.cu, ph = it.ph;
        const bool flush = ends_segment(it);
        iter_next(it, T, b, Ptot);
        if (flush) hand_off(T.ph[ph], ph, cu, active);
        run_jobs();
      }
    }
    // every flush event completed by the flush warp and every fixup job of this slice run
    wait_flushes(fk);
    if (threadIdx.x == 0) trace_event(p, 5);
  }
  __syncthreads();
  if (warp < kNC) {
    // Only after an error: wait for the stages that were armed but not consumed, so no copy
    // is in flight when the CTA exits.
    for (long long G = consumed; G < s_armed; ++G) {
      wait_slot(&full[slot], parity, &s_never, p.err, p.timeout_ns);
      if (++slot == S) {
        slot = 0;
        parity ^= 1u;
      }
    }
  }
  if (threadIdx.x == 0) {
    // the last CTA to finish (every CTA's reads of the counters are done) returns the
    // kEpiSiluMul segment counters to zero for the next launch and counts the launch
    __threadfence();
    if (atomicAdd(&p.sync->done, 1u) == gridDim.x - 1) {
      __threadfence();
      for (int i = 0; i < p.zero_count; ++i) p.zero_counters[i] = 0u;
      atomicExch(&p.sync->done, 0u);
      atomicAdd(&p.sync->epoch, 1u);
    }
    trace_event(p, 6);
  }
}

template <int MT, int GS>
cudaError_t launch_mt(const TmapPack& maps, const EngineParams& p, int grid, size_t smem,
                      cudaStream_t stream) {
  auto kern = int4_engine_kernel<MT, GS>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, maps, p);
}

template <int MT, int GS>
cudaError_t prepare_mt(size_t smem, int* blocks) {
  auto kern = int4_engine_kernel<MT, GS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, kern, kThreads, smem);
}

// (MT, GS) instantiations: MT in {1, 2, 4} tokens, GS in {16, 32, 64, 128}.
template <int MT>
cudaError_t occupancy_gs(int gs, size_t smem, int* blocks) {
  switch (gs) {
    case 16: return prepare_mt<MT, 16>(smem, blocks);
    case 32: return prepare_mt<MT, 32>(smem, blocks);
    case 64: return prepare_mt<MT, 64>(smem, blocks);
    case 128: return prepare_mt<MT, 128>(smem, blocks);
    default: return cudaErrorInvalidValue;
  }
}

template <int MT>
cudaError_t launch_gs(int gs, const TmapPack& maps, const EngineParams& p, int grid, size_t smem,
                      cudaStream_t stream) {
  switch (gs) {
    case 16: return launch_mt<MT, 16>(maps, p, grid, smem, stream);
    case 32: return launch_mt<MT, 32>(maps, p, grid, smem, stream);
    case 64: return launch_mt<MT, 64>(maps, p, grid, smem, stream);
    case 128: return launch_mt<MT, 128>(maps, p, grid, smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

int engine_warps_per_cta() { return kNC; }

size_t engine_smem_bytes(int stages, int tile_stage_bytes, int aux_stage_bytes, int rec0_bytes) {
  return 1024 + (size_t)stages * ((size_t)tile_stage_bytes + aux_stage_bytes + 16) + 16 +
         (size_t)rec0_bytes;
}

// Deepest ring that fits (bytes in flight are what keeps HBM busy), with the prologue
// records in shared memory when they fit beside it.
bool engine_plan_smem(int tile_stage_bytes, int aux_stage_bytes, int rec0_bytes, int smem_limit,
                      int* stages, int* rec0_smem, size_t* smem) {
  for (int s = kMaxStages; s >= 2; --s) {
    const size_t with = engine_smem_bytes(s, tile_stage_bytes, aux_stage_bytes, rec0_bytes);
    if (with <= (size_t)smem_limit) {
      *stages = s;
      *rec0_smem = 1;
      *smem = with;
      return true;
    }
    const size_t without = engine_smem_bytes(s, tile_stage_bytes, aux_stage_bytes, 0);
    if (without <= (size_t)smem_limit) {
      *stages = s;
      *rec0_smem = 0;
      *smem = without;
      return true;
    }
  }
  return false;
}

// The shared-memory attribute and the occupancy query cost host time ahead of every launch, so
// they are redone only when an instantiation is launched on a device with another shared-memory
// size than its last one (the attribute always holds the size of the latest launch).
cudaError_t engine_occupancy(int mt, int gs, size_t smem, int* blocks) {
  constexpr int kMaxDevices = 64;
  struct Last {
    size_t smem;
    int blocks;
    unsigned gen;
  };
  static std::mutex mu;
  static Last last[kMaxDevices][3][4] = {};  // [device][MT 1, 2, 4][GS 16, 32, 64, 128]
  const int mi = mt == 1 ? 0 : mt == 2 ? 1 : mt == 4 ? 2 : -1;
  const int gi = gs == 16 ? 0 : gs == 32 ? 1 : gs == 64 ? 2 : gs == 128 ? 3 : -1;
  if (mi < 0 || gi < 0) return cudaErrorInvalidValue;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  Last* L = dev >= 0 && dev < kMaxDevices ? &last[dev][mi][gi] : nullptr;
  const unsigned gen = attr_generation(dev);
  if (L && L->blocks > 0 && L->smem == smem && L->gen == gen) {
    *blocks = L->blocks;
    return cudaSuccess;
  }
  switch (mt) {
    case 1: e = occupancy_gs<1>(gs, smem, blocks); break;
    case 2: e = occupancy_gs<2>(gs, smem, blocks); break;
    default: e = occupancy_gs<4>(gs, smem, blocks); break;
  }
  if (L) *L = (e == cudaSuccess) ? Last{smem, *blocks, gen} : Last{0, 0, 0};
  return e;
}

cudaError_t engine_launch(int mt, int gs, const TmapPack& maps, const EngineParams& p, int grid,
                          size_t smem, cudaStream_t stream) {
  switch (mt) {
    case 1: return launch_gs<1>(gs, maps, p, grid, smem, stream);
    case 2: return launch_gs<2>(gs, maps, p, grid, smem, stream);
    case 4: return launch_gs<4>(gs, maps, p, grid, smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace tk
