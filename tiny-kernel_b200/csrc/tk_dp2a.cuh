// tk_dp2a.cuh -- the dp2a consumer arithmetic shared by the streaming kernels (1-2 rows).
//
// qmatmul_int4 (src/kernels/shaders.zig:442-501) on the reference's packed layout with the
// activations quantised to int16 per group (one power-of-two scale 2^-e, max |x| * 2^e in
// [2^14, 2^15)).  Lane l of a consumer warp owns columns 4l .. 4l+3 of a 128-column slice.  One
// PRMT per column pair interleaves two packed rows so that a column's two k pairs sit in adjacent
// bytes; masking gives the low nibbles (even k) and 16 x the high nibbles (odd k); dp2a multiplies
// them by the int16 activations, two k per instruction, into exact int32 sums.  Per group:
//     v = 2^-e * (sum_even + (sum_odd16 >> 4) - z * sum_k xq_k)     (exact integers)
//     y += scale * v.
#pragma once
#include <cuda_fp16.h>

#include <cstdint>

#include "tk_engine.h"
#include "tk_ptx.cuh"

namespace tk {
namespace {

// dp2a path.  Warp-collective, same lane contract as build_records_mma: lane l holds values
// 4l..4l+3 of a 128-value chunk of token `tok`.  A group's lane lg writes X[lg] of the
// group's record (its four values are k = 4lg..4lg+3 of the group: packed rows 2lg, 2lg+1).
template <int MT>
__device__ __forceinline__ void build_records_dp(const float (&v)[4], int tok, int gs,
                                                 uint8_t* rec, int rec_bytes, int lane,
                                                 int gi_only) {
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
  const bool store = gi_only < 0 || gi == gi_only;
  uint8_t* r = rec + (size_t)gi * rec_bytes + (size_t)tok * dp_tok_stride(gs);
  if (store)
    reinterpret_cast<uint2*>(r)[lg] =
        make_uint2(((uint32_t)q[0] & 0xffffu) | ((uint32_t)q[2] << 16),
                   ((uint32_t)q[1] & 0xffffu) | ((uint32_t)q[3] << 16));
  // per 16-k step (4 lanes): the sum of the quantised values, for the zero-point term
  int s = q[0] + q[1] + q[2] + q[3];
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  s += __shfl_xor_sync(0xffffffffu, s, 2);
  if ((lg & 3) == 0 && store) reinterpret_cast<int*>(r + 2 * gs)[lg >> 2] = s;
  if (lg == 0 && store) *reinterpret_cast<float*>(r + 2 * gs + gs / 4) = down;
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

// Packed bytes of rows [rb, rb + RB) of this lane's 4 columns, whatever the item's row range
// (the decode kernel fills a partial item's other k-steps with zero rows).
template <int RB>
__device__ __forceinline__ void dp_load_rows_all(const uint8_t* tl, int rb, int lane,
                                                 uint32_t (&w)[RB]) {
#pragma unroll
  for (int r = 0; r < RB; ++r)
    w[r] = *reinterpret_cast<const uint32_t*>(tl + (size_t)(rb + r) * kRowBytes + 4 * lane);
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

// Per-item values of the dp2a path that stay in registers from the item's first loads to its
// epilogue: this lane's 4 scales and 4 zero points, and per token the sum of the quantised
// activations over the item's k-steps and 2^-e.
template <int MT>
struct DpMeta {
  uint2 sc;
  uint32_t zz;
  int sx[MT];
  float esc[MT];
};

template <int MT, int GS>
__device__ __forceinline__ void dp_load_meta(const uint8_t* ax, const uint8_t* rec, int slice,
                                             int lane, int s0, int s1, DpMeta<MT>& M) {
  constexpr int tok_stride = dp_tok_stride(GS);
  constexpr int spg = GS / 16;
  M.sc = *reinterpret_cast<const uint2*>(ax + slice * kScaleBytes + 8 * lane);
  M.zz = *reinterpret_cast<const uint16_t*>(ax + kSlices * kScaleBytes + slice * kZeroBytes + 2 * lane);
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    const uint8_t* rt = rec + (size_t)m * tok_stride;
    const int* sums = reinterpret_cast<const int*>(rt + 2 * GS);
    int a = 0;
#pragma unroll
    for (int s = 0; s < spg; ++s) {
      const int v = sums[s];
      a += (s >= s0 && s < s1) ? v : 0;
    }
    M.sx[m] = a;
    M.esc[m] = *reinterpret_cast<const float*>(rt + 2 * GS + GS / 4);
  }
}

// y[4 m + i] (column 4 lane + i of token m) += scale * 2^-e * sum_k xq_k * (q_k - z)
template <int MT>
__device__ __forceinline__ void dp_epilogue(const DpMeta<MT>& M, const int (&aL)[MT][4],
                                            const int (&aH)[MT][4], float (&y)[4 * MT]) {
  const float2 s01 = __half22float2(*reinterpret_cast<const __half2*>(&M.sc.x));
  const float2 s23 = __half22float2(*reinterpret_cast<const __half2*>(&M.sc.y));
  const float s[4] = {s01.x, s01.y, s23.x, s23.y};
  const int z[4] = {(int)(M.zz & 15u), (int)((M.zz >> 4) & 15u), (int)((M.zz >> 8) & 15u),
                    (int)((M.zz >> 12) & 15u)};
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      // exact in int32, then one rounding
      const int t = aL[m][i] + (aH[m][i] >> 4) - z[i] * M.sx[m];
      y[4 * m + i] = fmaf(s[i] * M.esc[m], (float)t, y[4 * m + i]);
    }
}

}  // namespace
}  // namespace tk
