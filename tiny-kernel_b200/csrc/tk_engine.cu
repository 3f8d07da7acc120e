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
//  * Split-K partial sums go to a scratch buffer; the last warp to finish a 128-column
//    sub-tile (an atomic counter per sub-tile) adds the partials in phase and CTA order
//    (deterministic) and runs the epilogue: store (+ residual), or silu(gate) * up -> the
//    next phase's records plus a ready flag for that sub-tile.
//  * No grid-wide barrier: every CTA builds its own prologue records; the record warp
//    issues a record copy for an h group only once the flag of its h sub-tile equals
//    epoch + 1 (epoch = launches completed, advanced by the last CTA to finish).  The FFN
//    splits gate/up into tile ranges so the down projection of an early range overlaps
//    the reduction of the last one.
// Every spin-wait is bounded by a global-timer timeout and reports through p.err.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "tk_engine.h"
#include "tk_ptx.cuh"

namespace tk {

namespace {

constexpr int kNC = kSlices;  // consumer warps: one per 128-column slice

// ---- stream-K bookkeeping --------------------------------------------------------------

// CTA whose stream-K range holds unit u (ranges [U*b/W, U*(b+1)/W), all non-empty)
__device__ __forceinline__ long long cta_of_unit(long long u, long long units, long long W) {
  return ((u + 1) * W - 1) / units;
}

__device__ __forceinline__ long long phase_ctas(const PhaseParams& P, long long Wtot) {
  return P.units < Wtot ? P.units : Wtot;
}

// Number of CTA ranges of phase P holding units of (global) column unit cu = wide tile *
// nmat + matrix; 0 when the phase does not cover cu.
__device__ __forceinline__ int nseg_of_cu(const PhaseParams& P, long long cu, long long Wtot) {
  const long long c = cu - (long long)P.wt0 * P.nmat;
  if (c < 0 || c >= (long long)P.tiles * P.nmat) return 0;
  const long long W = phase_ctas(P, Wtot);
  const long long per = (long long)P.groups * P.spg;
  const long long a = c * per;
  return (int)(cta_of_unit(a + per - 1, P.units, W) - cta_of_unit(a, P.units, W) + 1);
}

// Segments of column unit cu summed over the phases that reduce together with phase ph.
__device__ __forceinline__ int red_segments(const EngineParams& p, int ph, long long cu,
                                            long long Wtot) {
  const PhaseParams& P = p.ph[ph];
  int n = 0;
  for (int q = P.red_first; q < P.red_first + P.red_count; ++q) n += nseg_of_cu(p.ph[q], cu, Wtot);
  return n;
}

// Index within its reduction of CTA b's segment of column unit cu in phase ph (earlier
// phases of the reduction first, then CTA order).
__device__ __forceinline__ int segment_index(const EngineParams& p, int ph, long long cu,
                                             long long b, long long Wtot) {
  const PhaseParams& P = p.ph[ph];
  int off = 0;
  for (int q = P.red_first; q < ph; ++q) off += nseg_of_cu(p.ph[q], cu, Wtot);
  const long long W = phase_ctas(P, Wtot);
  const long long a = (cu - (long long)P.wt0 * P.nmat) * P.groups * P.spg;
  return off + (int)(b - cta_of_unit(a, P.units, W));
}

__device__ __forceinline__ int active_slices(const PhaseParams& P, int wtile) {
  const int rem = (P.N - wtile * kWideCols) / kTileCols;
  return rem < kSlices ? rem : kSlices;
}

// Partial sums of segment `seg` of column unit cu, slice `slice`: [MT][128] floats.
template <int MT>
__device__ __forceinline__ float* partial_slot(const PhaseParams& P, long long cu, int seg,
                                               int slice) {
  return P.partials + (((size_t)cu * P.maxseg + seg) * kSlices + slice) * MT * kTileCols;
}

// Walks one CTA's items (one group of one wide tile each) through all phases.
struct ItemIter {
  int ph;       // phase of the current item; == nphases when exhausted
  int i, n;     // index within the phase, items in the phase
  int cu, grp;  // global column unit (tile * nmat + mat) and global group of the item
  int s0, s1;   // k-step range of the current item within its group
  int last_s1;  // s1 of the phase's last item
};

__device__ __forceinline__ void iter_seek(ItemIter& it, const EngineParams& p, long long w,
                                          long long Wtot) {
  while (it.ph < p.nphases) {
    const PhaseParams& P = p.ph[it.ph];
    const long long W = phase_ctas(P, Wtot);
    if (w < W) {
      const long long beg = P.units * w / W, end = P.units * (w + 1) / W;
      const long long fg0 = beg / P.spg, fgl = (end - 1) / P.spg;
      const long long cl = fg0 / P.groups;
      it.i = 0;
      it.n = (int)(fgl - fg0 + 1);
      it.cu = (int)(cl + (long long)P.wt0 * P.nmat);
      it.grp = P.g0 + (int)(fg0 - cl * P.groups);
      it.s0 = (int)(beg - fg0 * P.spg);
      it.last_s1 = (int)(end - fgl * P.spg);
      it.s1 = it.n == 1 ? it.last_s1 : P.spg;
      return;
    }
    ++it.ph;
  }
}

__device__ __forceinline__ void iter_start(ItemIter& it, const EngineParams& p, long long w,
                                           long long Wtot) {
  it.ph = 0;
  it.i = it.n = it.cu = it.grp = it.s0 = it.s1 = it.last_s1 = 0;
  iter_seek(it, p, w, Wtot);
}

__device__ __forceinline__ void iter_next(ItemIter& it, const EngineParams& p, long long w,
                                          long long Wtot) {
  const PhaseParams& P = p.ph[it.ph];
  if (++it.i < it.n) {
    if (++it.grp == P.g1) {
      it.grp = P.g0;
      ++it.cu;
    }
    it.s0 = 0;
    it.s1 = it.i == it.n - 1 ? it.last_s1 : P.spg;
    return;
  }
  ++it.ph;
  iter_seek(it, p, w, Wtot);
}

// Bytes the weight warp's copies bring into a stage for item `it` (box rows, scales, zeros);
// the record warp adds the activation record (P.frag_bytes).
__device__ __forceinline__ uint32_t item_weight_bytes(const PhaseParams& P, const ItemIter& it) {
  const int ns = active_slices(P, it.cu >> (P.nmat - 1));
  return (uint32_t)((it.s1 - it.s0) * kStepRows * kRowBytes + ns * (kScaleBytes + kZeroBytes));
}

// Weight-warp lane `lane` issues its share of item `it`'s weight-side copies: lane 0 the TMA
// box(es), lane 8 the scales, lane 9 the zero points.
__device__ __forceinline__ void issue_weights(const TmapPack& maps, const PhaseParams& P,
                                              const ItemIter& it, uint8_t* tile, uint8_t* aux,
                                              uint64_t* bar, uint64_t pol, int lane) {
  const int mat = it.cu & (P.nmat - 1);
  const int wt = it.cu >> (P.nmat - 1);
  const int col0 = wt * kWideCols;
  if (lane == 0) {
    const int row0 = it.grp * P.spg * kStepRows;
    const int x = wt * (kWideCols / 8);  // u64 element of the tile's first byte
    if (it.s0 == 0 && it.s1 == P.spg) {
      tma_load_2d(tile, &maps.map[P.map_base + 2 * mat], bar, x, row0, pol);
    } else {
      for (int s = it.s0; s < it.s1; ++s)
        tma_load_2d(tile + s * kStepRows * kRowBytes, &maps.map[P.map_base + 2 * mat + 1], bar, x,
                    row0 + s * kStepRows, pol);
    }
  } else if (lane == 8) {
    const int ns = active_slices(P, wt);
    bulk_load(aux, P.scales[mat] + (size_t)it.grp * P.N + col0, (uint32_t)(ns * kScaleBytes), bar,
              pol);
  } else if (lane == 9) {
    const int ns = active_slices(P, wt);
    bulk_load(aux + kSlices * kScaleBytes, P.zeros[mat] + (size_t)it.grp * (P.N / 2) + col0 / 2,
              (uint32_t)(ns * kZeroBytes), bar, pol);
  }
}

__device__ __forceinline__ uint8_t* frag_slot(uint8_t* aux) {
  return aux + kSlices * (kScaleBytes + kZeroBytes);
}

__device__ __forceinline__ void issue_frag(const PhaseParams& P, const ItemIter& it, long long b,
                                           uint8_t* aux, uint64_t* bar, uint64_t pol) {
  bulk_load(frag_slot(aux), P.frag_in + b * P.frag_cta_stride + (size_t)it.grp * P.frag_bytes,
            (uint32_t)P.frag_bytes, bar, pol);
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
                                                  uint8_t* rec, int rec_bytes, int lane) {
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
  if (j == 0) {
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
  if ((lg & 3) == 0) sums[(lg >> 2) * MT + tok] = make_int2(sh, sl);
  if (lg == 0) reinterpret_cast<float*>(sums + spg * MT)[tok] = down;
}

// dp2a path.  Warp-collective, same lane contract as build_records_mma: lane l holds values
// 4l..4l+3 of a 128-value chunk of token `tok`.  A group's lane lg writes X[lg] of the
// group's record (its four values are k = 4lg..4lg+3 of the group: packed rows 2lg, 2lg+1).
template <int MT>
__device__ __forceinline__ void build_records_dp(const float (&v)[4], int tok, int gs,
                                                 uint8_t* rec, int rec_bytes, int lane) {
  const int gl = gs >> 2;  // lanes per group
  float mx = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
  for (int off = 1; off < gl; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  // e with max |x| * 2^e in [2^14, 2^15) from the exponent field (zero, subnormal and
  // non-finite maxima are clamped to the range the scale stays a normal power of two in)
  int e = 141 - (int)((__float_as_uint(mx) >> 23) & 0xffu);
  e = e < -100 ? -100 : (e > 100 ? 100 : e);
  const float up = __uint_as_float((uint32_t)(127 + e) << 23);    // 2^e
  const float down = __uint_as_float((uint32_t)(127 - e) << 23);  // 2^-e
  int q[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = __float2int_rn(v[i] * up);
    q[i] = t < -32767 ? -32767 : (t > 32767 ? 32767 : t);
  }
  const int gi = lane / gl, lg = lane - gi * gl;
  uint8_t* r = rec + (size_t)gi * rec_bytes + (size_t)tok * dp_tok_stride(gs);
  reinterpret_cast<uint2*>(r)[lg] =
      make_uint2(((uint32_t)q[0] & 0xffffu) | ((uint32_t)q[2] << 16),
                 ((uint32_t)q[1] & 0xffffu) | ((uint32_t)q[3] << 16));
  // per 16-k step (4 lanes): the sum of the quantised values, for the zero-point term
  int s = q[0] + q[1] + q[2] + q[3];
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  s += __shfl_xor_sync(0xffffffffu, s, 2);
  if ((lg & 3) == 0) reinterpret_cast<int*>(r + 2 * gs)[lg >> 2] = s;
  if (lg == 0) *reinterpret_cast<float*>(r + 2 * gs + gs / 4) = down;
}

template <int MT>
__device__ __forceinline__ void build_records(const float (&v)[4], int tok, int gs, uint8_t* rec,
                                              int rec_bytes, int lane) {
  if constexpr (MT <= 2) build_records_dp<MT>(v, tok, gs, rec, rec_bytes, lane);
  else build_records_mma<MT>(v, tok, gs, rec, rec_bytes, lane);
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

// ---- dp2a path (m = 1, 2) ---------------------------------------------------------------------

// Packed bytes of rows [rb, rb + RB) of this lane's 4 columns; rows outside [r0, r1) are 0.
template <int RB>
__device__ __forceinline__ void dp_load_rows(const uint8_t* tl, int rb, int r0, int r1, int lane,
                                             uint32_t (&w)[RB]) {
  if (r0 <= rb && r1 >= rb + RB) {
#pragma unroll
    for (int r = 0; r < RB; ++r)
      w[r] = *reinterpret_cast<const uint32_t*>(tl + (size_t)(rb + r) * kRowBytes + 4 * lane);
  } else {
#pragma unroll
    for (int r = 0; r < RB; ++r) {
      const int rr = rb + r;
      w[r] = (rr >= r0 && rr < r1)
                 ? *reinterpret_cast<const uint32_t*>(tl + (size_t)rr * kRowBytes + 4 * lane)
                 : 0u;
    }
  }
}

// Activation pairs of row pairs [rb/2, rb/2 + RB/2) of every token (two row pairs per uint4).
template <int MT, int RB>
__device__ __forceinline__ void dp_load_x(const uint8_t* rec, int tok_stride, int rb,
                                          uint4 (&X)[MT][RB / 4]) {
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    const uint4* xp = reinterpret_cast<const uint4*>(rec + (size_t)m * tok_stride) + rb / 4;
#pragma unroll
    for (int q = 0; q < RB / 4; ++q) X[m][q] = xp[q];
  }
}

// Row pair j = (2j, 2j+1): p0 = {r c0, r+1 c0, r c1, r+1 c1}, p1 the same for c2, c3.  The low
// nibbles (even k) meet x[4j], x[4j+2]; 16 x the high nibbles (odd k) meet x[4j+1], x[4j+3].
template <int MT, int RB>
__device__ __forceinline__ void dp_compute(const uint32_t (&w)[RB], const uint4 (&X)[MT][RB / 4],
                                           int (&aL)[MT][4], int (&aH)[MT][4]) {
#pragma unroll
  for (int j = 0; j < RB / 2; ++j) {
    const uint32_t p0 = prmt(w[2 * j], w[2 * j + 1], 0x5140);
    const uint32_t p1 = prmt(w[2 * j], w[2 * j + 1], 0x7362);
    const uint32_t l0 = p0 & 0x0F0F0F0Fu, h0 = p0 & 0xF0F0F0F0u;
    const uint32_t l1 = p1 & 0x0F0F0F0Fu, h1 = p1 & 0xF0F0F0F0u;
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const uint32_t xe = (j & 1) ? X[m][j >> 1].z : X[m][j >> 1].x;
      const uint32_t xo = (j & 1) ? X[m][j >> 1].w : X[m][j >> 1].y;
      aL[m][0] = dp2a_lo(xe, l0, aL[m][0]);
      aL[m][1] = dp2a_hi(xe, l0, aL[m][1]);
      aL[m][2] = dp2a_lo(xe, l1, aL[m][2]);
      aL[m][3] = dp2a_hi(xe, l1, aL[m][3]);
      aH[m][0] = dp2a_lo(xo, h0, aH[m][0]);
      aH[m][1] = dp2a_hi(xo, h0, aH[m][1]);
      aH[m][2] = dp2a_lo(xo, h1, aH[m][2]);
      aH[m][3] = dp2a_hi(xo, h1, aH[m][3]);
    }
  }
}

// One item of one slice on the dp2a path: R = packed rows per group (gs / 2).  Loads every
// stage byte it needs, releases the stage (empty barrier), then computes; groups of 128 k
// (R = 64) are computed in two 32-row blocks before the release.  y[4 m + i] accumulates
// column 4 lane + i of token m.
template <int MT, int R>
__device__ __forceinline__ void dp_item(const uint8_t* tl, const uint8_t* rec, const uint8_t* scp,
                                        const uint8_t* zpp, int s0, int s1, int lane,
                                        uint64_t* empty_bar, float (&y)[4 * MT]) {
  constexpr int gs = 2 * R;
  constexpr int RB = R < 32 ? R : 32;
  constexpr int tok_stride = dp_tok_stride(gs);
  const int r0 = s0 * kStepRows, r1 = s1 * kStepRows;
  const uint2 sc = *reinterpret_cast<const uint2*>(scp + 8 * lane);
  const uint32_t zz = *reinterpret_cast<const uint16_t*>(zpp + 2 * lane);
  int sx[MT];
  float esc[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    const uint8_t* rt = rec + (size_t)m * tok_stride;
    const int* sums = reinterpret_cast<const int*>(rt + 2 * gs);
    int a = 0;
    for (int s = s0; s < s1; ++s) a += sums[s];
    sx[m] = a;
    esc[m] = *reinterpret_cast<const float*>(rt + 2 * gs + gs / 4);
  }
  int aL[MT][4], aH[MT][4];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int i = 0; i < 4; ++i) aL[m][i] = aH[m][i] = 0;
  if constexpr (R <= 32) {
    uint32_t w[RB];
    uint4 X[MT][RB / 4];
    dp_load_rows<RB>(tl, 0, r0, r1, lane, w);
    dp_load_x<MT, RB>(rec, tok_stride, 0, X);
    __syncwarp();
    if (lane == 0) mbar_arrive(empty_bar);
    dp_compute<MT, RB>(w, X, aL, aH);
  } else {
    for (int rb = 0; rb < R; rb += 32) {
      if (rb >= r1 || rb + 32 <= r0) continue;
      uint32_t w[32];
      uint4 X[MT][8];
      dp_load_rows<32>(tl, rb, r0, r1, lane, w);
      dp_load_x<MT, 32>(rec, tok_stride, rb, X);
      dp_compute<MT, 32>(w, X, aL, aH);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty_bar);
  }
  const float2 s01 = __half22float2(*reinterpret_cast<const __half2*>(&sc.x));
  const float2 s23 = __half22float2(*reinterpret_cast<const __half2*>(&sc.y));
  const float s[4] = {s01.x, s01.y, s23.x, s23.y};
  const int z[4] = {(int)(zz & 15u), (int)((zz >> 4) & 15u), (int)((zz >> 8) & 15u),
                    (int)((zz >> 12) & 15u)};
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      // sum_k xq_k * (q_k - z): exact in int32, then one rounding
      const int t = aL[m][i] + (aH[m][i] >> 4) - z[i] * sx[m];
      y[4 * m + i] = fmaf(s[i] * esc[m], (float)t, y[4 * m + i]);
    }
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

// The last warp to finish a sub-tile: deterministic reduction of the partials + epilogue.
template <int MT>
__device__ void fixup_tile(const EngineParams& p, int ph, int wt, int slice, long long Wtot,
                           int lane, unsigned epoch) {
  const PhaseParams& P = p.ph[ph];
  const int m = p.m;
  for (int tok = 0; tok < MT; ++tok) {
    float acc[kMaxMats][4];
#pragma unroll
    for (int mi = 0; mi < kMaxMats; ++mi) acc[mi][0] = acc[mi][1] = acc[mi][2] = acc[mi][3] = 0.f;
    for (int mi = 0; mi < P.nmat; ++mi) {
      const long long cu = (long long)wt * P.nmat + mi;
      const int ns = red_segments(p, ph, cu, Wtot);
      const float* base = partial_slot<MT>(P, cu, 0, slice) + tok * kTileCols + 4 * lane;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      // eight segments' loads in flight at a time; the sum stays in segment order
      for (int s0 = 0; s0 < ns; s0 += 8) {
        float4 v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          v[i] = s0 + i < ns ? __ldcg(reinterpret_cast<const float4*>(
                                   base + (size_t)(s0 + i) * kSlices * MT * kTileCols))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          a0 += v[i].x;
          a1 += v[i].y;
          a2 += v[i].z;
          a3 += v[i].w;
        }
      }
      acc[mi][0] = a0;
      acc[mi][1] = a1;
      acc[mi][2] = a2;
      acc[mi][3] = a3;
    }
    const int sub0 = wt * kWideCols + slice * kTileCols;  // first column of the sub-tile
    const int col = sub0 + 4 * lane;
    if (P.epi == kEpiStore) {
      if (tok < m) {
        float4 o = make_float4(acc[0][0], acc[0][1], acc[0][2], acc[0][3]);
        if (P.residual) {
          const float4 r = *reinterpret_cast<const float4*>(P.residual + (size_t)tok * P.ldr + col);
          o.x = r.x + o.x;
          o.y = r.y + o.y;
          o.z = r.z + o.z;
          o.w = r.w + o.w;
        }
        *reinterpret_cast<float4*>(P.out + (size_t)tok * P.ldo + col) = o;
      }
    } else {
      float h[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float gv = acc[0][i];
        h[i] = (tok < m) ? gv / (1.0f + expf(-gv)) * acc[1][i] : 0.f;
      }
      if (P.out && tok < m)
        *reinterpret_cast<float4*>(P.out + (size_t)tok * P.ldo + col) = make_float4(h[0], h[1], h[2], h[3]);
      build_records<MT>(h, tok, P.next_gs,
                        P.frag_out + (size_t)(sub0 / P.next_gs) * P.next_frag_bytes,
                        P.next_frag_bytes, lane);
    }
  }
  if (P.epi == kEpiSiluMul) {
    fence_proxy_async();  // the records are read by other CTAs through TMA
    __syncwarp();
    if (lane == 0) {
      __threadfence();
      atomicExch(&P.ready_out[wt * kSlices + slice], epoch + 1);
    }
  }
}

// Counts one finished segment of sub-tile (wt, slice) of phase ph's reduction; returns true
// to the last of them.
__device__ __forceinline__ bool count_segment(const EngineParams& p, int ph, int wt, int slice,
                                              long long Wtot) {
  const PhaseParams& P = p.ph[ph];
  unsigned total = 0;
  for (int mi = 0; mi < P.nmat; ++mi)
    total += (unsigned)red_segments(p, ph, (long long)wt * P.nmat + mi, Wtot);
  const unsigned prev = atomicAdd(&P.counters[wt * kSlices + slice], 1u);
  return prev == total - 1;
}

// End of a CTA's range in phase ph: store the segment, count it, reduce if last.
template <int MT>
__device__ __forceinline__ void flush_segment(const EngineParams& p, int ph, int cu, long long b,
                                              long long Wtot, int slice, float (&y)[4 * MT],
                                              int lane, int tokE, int colbase, unsigned epoch) {
  const PhaseParams& P = p.ph[ph];
  const int seg = segment_index(p, ph, cu, b, Wtot);
  const int wt = cu >> (P.nmat - 1);
  const int sub = wt * kSlices + slice;
  store_partials<MT>(partial_slot<MT>(P, cu, seg, slice), y, lane, tokE, colbase);
  __threadfence();
  __syncwarp();
  unsigned last = 0;
  if (lane == 0) last = count_segment(p, ph, wt, slice, Wtot) ? 1u : 0u;
  last = __shfl_sync(0xffffffffu, last, 0);
  if (last) {
    __threadfence();
    fixup_tile<MT>(p, ph, wt, slice, Wtot, lane, epoch);
    __syncwarp();
    if (lane == 0) atomicExch(&P.counters[sub], 0u);
  }
#pragma unroll
  for (int i = 0; i < 4 * MT; ++i) y[i] = 0.f;
}

// Consumer warps: x (optionally rmsnorm'ed, src/kernels/shaders.zig:16-56) -> records.
// x and the norm weight are read first and the weight producer is held at named barrier 2
// until every consumer has them in registers: reads issued after the weight stream starts
// queue behind megabytes of TMA traffic.
template <int MT>
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
    build_records<MT>(v, tok, p.gs0, recs + (size_t)(ch * kTileCols / p.gs0) * p.frag0_bytes,
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
// record once it is ready, warp kNC+2 (flush warp) completes the split-K segments that end in
// the middle of a CTA's range (the consumers only store their partial sums and move on; the
// flush warp makes them visible, counts them and runs the tile epilogue when it is last).  Each
// stage's full barrier takes one arrival from each producer warp.
constexpr int kWeightWarp = kNC;
constexpr int kRecordWarp = kNC + 1;
constexpr int kFlushWarp = kNC + 2;
constexpr int kThreads = (kNC + 3) * 32;
constexpr int kFlushSlots = 4;  // flush events in flight between the consumers and the flush warp

// An item ends its column unit in the middle of the CTA's range of the phase (its split-K
// segment is handed to the flush warp) rather than at the end of the range.
__device__ __forceinline__ bool mid_range_flush(const PhaseParams& P, const ItemIter& it) {
  return it.grp == P.g1 - 1 && it.i != it.n - 1;
}

template <int MT>
__global__ void __launch_bounds__(kThreads, 1)
    int4_engine_kernel(const __grid_constant__ TmapPack maps, const __grid_constant__ EngineParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ float s_red[MT * kNC];
  __shared__ float s_rms[MT];
  __shared__ unsigned s_epoch;
  __shared__ volatile long long s_armed;   // items whose weights the weight warp has armed
  __shared__ volatile int s_wdone;         // weight warp has left its loop (s_armed final)
  __shared__ volatile int s_records;       // this CTA's prologue records are written
  __shared__ volatile int s_abort;
  __shared__ volatile int s_never;         // stays 0: a wait that must not be cut short
  __shared__ uint64_t s_fbar[kFlushSlots];  // mid-range flush events (kNC consumer arrivals)
  __shared__ volatile int s_fdone;         // flush events the flush warp has completed
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.stages;
  uint8_t* tiles = smem;
  uint8_t* auxs = smem + (size_t)S * p.tile_stage_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(auxs + (size_t)S * p.aux_stage_bytes);
  uint64_t* empty = full + S;
  uint8_t* rec0s = reinterpret_cast<uint8_t*>(empty + S) + 16 - (smem_addr(empty + S) & 15u);
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 2);
      mbar_init(&empty[i], kNC);
    }
    for (int i = 0; i < kFlushSlots; ++i) mbar_init(&s_fbar[i], kNC);
    s_fdone = 0;
    fence_mbar_init();
    s_records = 0;
    s_abort = 0;
    s_never = 0;
    s_armed = 0;
    s_wdone = 0;
    s_epoch = ld_acquire_u32(&p.sync->epoch);
    trace_event(p, 0);
  }
  __syncthreads();
  const unsigned epoch = s_epoch;
  const long long Ptot = gridDim.x;
  const long long b = blockIdx.x;
  // consumer ring position (function scope for the drain at the end)
  int slot = 0;
  uint32_t parity = 0;
  long long consumed = 0;

  if (warp == kWeightWarp) {
    // ---------------------------- weight producer warp ---------------------------------
    const uint64_t pol_stream = l2_evict_first();
    ItemIter wi;
    iter_start(wi, p, b, Ptot);
    long long G = 0;
    int wslot = 0;
    uint32_t wround = 0;
    named_barrier(2, (kNC + 1) * 32);  // the consumers have read x
    while (wi.ph < p.nphases) {
      if (wround > 0 && !wait_slot(&empty[wslot], (wround - 1) & 1, &s_abort, p.err, p.timeout_ns)) {
        s_abort = 1;
        break;
      }
      if (s_abort) break;
      const PhaseParams& P = p.ph[wi.ph];
      if (lane == 0) {
        if (G == 0) trace_event(p, 7);
        mbar_arrive_expect_tx(&full[wslot], item_weight_bytes(P, wi));
      }
      __syncwarp();
      issue_weights(maps, P, wi, tiles + (size_t)wslot * p.tile_stage_bytes,
                    auxs + (size_t)wslot * p.aux_stage_bytes, &full[wslot], pol_stream, lane);
      __syncwarp();
      ++G;
      if (lane == 0) s_armed = G;
      iter_next(wi, p, b, Ptot);
      if (++wslot == S) {
        wslot = 0;
        ++wround;
      }
    }
    if (lane == 0) {
      s_armed = G;
      __threadfence_block();
      s_wdone = 1;
      trace_event(p, 8);
    }
  } else if (warp == kRecordWarp) {
    // ---------------------------- record producer warp ---------------------------------
    const uint64_t pol_keep = l2_evict_last();
    ItemIter fi;
    iter_start(fi, p, b, Ptot);
    long long F = 0;
    int fslot = 0;
    bool aborted = false;
    uint64_t t_wait = 0;
    while (fi.ph < p.nphases) {
      if (s_abort) {
        aborted = true;
        break;
      }
      // only items whose weights are armed (their slot is free and the full barrier is in
      // the phase this arrival belongs to)
      bool go = F < s_armed;
      const PhaseParams& P = p.ph[fi.ph];
      if (go && P.ready_in == nullptr && p.rec0_smem) {
        // the consumers read this item's record from shared memory: complete the arrival
        if (lane == 0) mbar_arrive(&full[fslot]);
        __syncwarp();
        ++F;
        iter_next(fi, p, b, Ptot);
        fslot = fslot + 1 == S ? 0 : fslot + 1;
        t_wait = 0;
        continue;
      }
      if (go) {
        if (P.ready_in == nullptr) {
          go = s_records != 0;
        } else {
          unsigned v = 0;
          if (lane == 0) v = ld_acquire_u32(&P.ready_in[fi.grp * P.gs / kTileCols]);
          go = __shfl_sync(0xffffffffu, v, 0) == epoch + 1;
        }
      }
      if (go) {
        fence_proxy_async();  // records were written by generic stores
        if (lane == 0) {
          uint8_t* aux = auxs + (size_t)fslot * p.aux_stage_bytes;
          mbar_arrive_expect_tx(&full[fslot], (uint32_t)P.frag_bytes);
          issue_frag(P, fi, b, aux, &full[fslot], pol_keep);
        }
        __syncwarp();
        ++F;
        iter_next(fi, p, b, Ptot);
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
    iter_start(hi, p, b, Ptot);
    int k = 0;
    while (hi.ph < p.nphases) {
      const PhaseParams& P = p.ph[hi.ph];
      if (mid_range_flush(P, hi)) {
        if (!wait_slot(&s_fbar[k % kFlushSlots], (uint32_t)(k / kFlushSlots) & 1u, &s_abort, p.err,
                       p.timeout_ns)) {
          s_abort = 1;
          break;
        }
        __threadfence();  // the consumers' partial sums (acquired through the barrier)
        const int wt = hi.cu >> (P.nmat - 1);
        const int ns = active_slices(P, wt);
        const bool last = lane < ns && count_segment(p, hi.ph, wt, lane, Ptot);
        unsigned won = __ballot_sync(0xffffffffu, last);
        if (won) __threadfence();
        while (won) {
          const int sl = __ffs(won) - 1;
          won &= won - 1;
          fixup_tile<MT>(p, hi.ph, wt, sl, Ptot, lane, epoch);
          __syncwarp();
          if (lane == 0) atomicExch(&P.counters[wt * kSlices + sl], 0u);
        }
        __syncwarp();
        if (lane == 0) s_fdone = k + 1;
        ++k;
      }
      iter_next(hi, p, b, Ptot);
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
    iter_start(it, p, b, Ptot);
    bool ok = true;
    int fk = 0;  // mid-range flush events handed to the flush warp

    prologue<MT>(p, warp, lane, s_red, s_rms, rec0s);
    named_barrier(1, kNC * 32);
    if (threadIdx.x == 0) {
      __threadfence_block();
      s_records = 1;
      trace_event(p, 1);
    }

    float y[4 * MT];
#pragma unroll
    for (int i = 0; i < 4 * MT; ++i) y[i] = 0.f;
    int D[8][4];
#pragma unroll
    for (int r = 0; r < 8; ++r) D[r][0] = D[r][1] = D[r][2] = D[r][3] = 0;
    int cur_ph = -1;
    while (ok && it.ph < p.nphases) {
      const int ph = it.ph;
      const PhaseParams& P = p.ph[ph];
      if (ph != cur_ph) {
        if (cur_ph >= 0 && threadIdx.x == 0) trace_event(p, 3 + (cur_ph ? 2 : 0));
        cur_ph = ph;
      }
      if (!wait_slot(&full[slot], parity, &s_abort, p.err, p.timeout_ns)) {
        ok = false;
        s_abort = 1;
        break;
      }
      if (consumed == 0 && threadIdx.x == 0) trace_event(p, 9);
      const int wt = it.cu >> (P.nmat - 1);
      const bool active = slice < active_slices(P, wt);
      const uint8_t* ax = auxs + (size_t)slot * p.aux_stage_bytes;
      const uint8_t* tl = tiles + (size_t)slot * p.tile_stage_bytes + slice * kTileCols;
      const uint8_t* rec = (P.ready_in == nullptr && p.rec0_smem)
                               ? rec0s + (size_t)it.grp * P.frag_bytes
                               : frag_slot(const_cast<uint8_t*>(ax));
      if constexpr (MT <= 2) {
        if (active) {
          const uint8_t* scp = ax + slice * kScaleBytes;
          const uint8_t* zpp = ax + kSlices * kScaleBytes + slice * kZeroBytes;
          switch (P.gs) {
            case 16: dp_item<MT, 8>(tl, rec, scp, zpp, it.s0, it.s1, lane, &empty[slot], y); break;
            case 32: dp_item<MT, 16>(tl, rec, scp, zpp, it.s0, it.s1, lane, &empty[slot], y); break;
            case 64: dp_item<MT, 32>(tl, rec, scp, zpp, it.s0, it.s1, lane, &empty[slot], y); break;
            default: dp_item<MT, 64>(tl, rec, scp, zpp, it.s0, it.s1, lane, &empty[slot], y); break;
          }
        } else {
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[slot]);
        }
      } else {
        if (active) {
          const int kbg = P.spg >= 4 ? P.spg / 4 : 1;    // 32-pair blocks per group
          const int nrows = P.spg >= 4 ? 32 : 8 * P.spg;  // valid rows per block
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
                             reinterpret_cast<const float*>(sums + P.spg * MT), it.s0, it.s1,
                             tokE, colbase, D, y);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
      }
      ++consumed;
      if (++slot == S) {
        slot = 0;
        parity ^= 1u;
      }
      const int cu = it.cu;
      const bool mid = mid_range_flush(P, it);
      const bool last_of_range = it.i == it.n - 1;
      iter_next(it, p, b, Ptot);
      if (mid) {
        // store the partial sums and hand the segment to the flush warp
        if (active)
          store_partials<MT>(partial_slot<MT>(P, cu, segment_index(p, ph, cu, b, Ptot), slice), y,
                             lane, tokE, colbase);
#pragma unroll
        for (int i = 0; i < 4 * MT; ++i) y[i] = 0.f;
        __syncwarp();
        if (lane == 0) {
          // the event slot is free once the flush warp has completed event fk - kFlushSlots
          const uint64_t t0 = global_timer_ns();
          while (s_fdone < fk - kFlushSlots + 1 && !s_abort) {
            if (global_timer_ns() - t0 > p.timeout_ns) {
              atomicOr(p.err, kErrFlagWait);
              s_abort = 1;
              break;
            }
          }
          mbar_arrive(&s_fbar[fk % kFlushSlots]);
        }
        ++fk;
      } else if (last_of_range) {
        if (active)
          flush_segment<MT>(p, ph, cu, b, Ptot, slice, y, lane, tokE, colbase, epoch);
#pragma unroll
        for (int i = 0; i < 4 * MT; ++i) y[i] = 0.f;
      }
    }
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
    // the last CTA to finish advances the epoch (the next launch's ready flags)
    __threadfence();
    if (atomicAdd(&p.sync->done, 1u) == gridDim.x - 1) {
      atomicExch(&p.sync->done, 0u);
      __threadfence();
      atomicExch(&p.sync->epoch, epoch + 1);
    }
    trace_event(p, 6);
  }
}

template <int MT>
cudaError_t launch_mt(const TmapPack& maps, const EngineParams& p, int grid, size_t smem,
                      cudaStream_t stream) {
  auto kern = int4_engine_kernel<MT>;
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

template <int MT>
cudaError_t prepare_mt(size_t smem, int* blocks) {
  auto kern = int4_engine_kernel<MT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, kern, kThreads, smem);
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

cudaError_t engine_occupancy(int mt, size_t smem, int* blocks) {
  switch (mt) {
    case 1: return prepare_mt<1>(smem, blocks);
    case 2: return prepare_mt<2>(smem, blocks);
    case 4: return prepare_mt<4>(smem, blocks);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t engine_launch(int mt, const TmapPack& maps, const EngineParams& p, int grid,
                          size_t smem, cudaStream_t stream) {
  switch (mt) {
    case 1: return launch_mt<1>(maps, p, grid, smem, stream);
    case 2: return launch_mt<2>(maps, p, grid, smem, stream);
    case 4: return launch_mt<4>(maps, p, grid, smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace tk
