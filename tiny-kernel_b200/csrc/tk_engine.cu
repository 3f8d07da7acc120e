// tk_engine.cu -- persistent, warp-specialised, TMA-fed INT4 fused-dequant GEMV engine
// for sm_100a.
//
// Computes the qmatmul_int4 contraction of the reference (src/kernels/shaders.zig:442-501)
//     y[m][n] = sum_g scale[g][n] * sum_{k in g} x[m][k] * (q[k][n] - zero[g][n])
// on the reference's packed layout, and the INT4 Llama FFN built from it
// (src/bench.zig:266-341 gate/up composition plus the down projection).
//
// Design (one CTA per SM: 8 consumer warps + 1 producer warp):
//  * A work unit is one k-step (8 packed rows = 16 k) of a 1024-column wide tile of one
//    matrix.  Units are ordered tile-major, matrix, group, step; CTA b of P owns units
//    [U*b/P, U*(b+1)/P) (stream-K), so every SM streams the same number of bytes.  Units
//    are visited group by group ("items"); the iteration is incremental (no divisions).
//  * The CTA has one ring of S stages (full + empty mbarrier each).  A stage holds one
//    item: the packed rows of the group as 1040-byte TMA box rows (u64 tensor map; one
//    box for a whole group, or one per k-step for a partial group) -- long rows are what
//    lets TMA stream near the HBM read limit -- plus the group's f16 scales (2 KB), zero
//    points (512 B) and activation record.  Producer lane 0 issues the boxes, lanes 8-10
//    the rest.  Consecutive 1040-byte rows sit 16 bytes apart modulo 128, which makes the
//    fragment loads bank-conflict free without a swizzle.
//  * Consumer warp j computes slice j of every stage.  The weight nibbles become m16n8k16
//    A fragments with one PRMT and two LOPs per 4 nibbles: each nibble lands in the
//    mantissa of an f16 subnormal, so the MMA sees q * 2^-24 exactly (even k) or
//    16 q * 2^-24 (odd k; the activations carry the 1/16).  Zero points are applied per
//    group in f32 as  - z * sum_k x_k.
//  * Activations arrive as precomputed B fragments: x is scaled by a power of two per
//    group and split x = hi + lo into two f16 values (B columns 2c, 2c+1), so the
//    products keep ~22 significant bits and accumulate in f32 in the tensor core.
//  * Split-K partial sums go to a scratch buffer; the last warp to finish a 128-column
//    sub-tile (an atomic counter per sub-tile) adds the partials in CTA order
//    (deterministic) and runs the epilogue: store (+ residual), or silu(gate) * up -> the
//    next phase's records plus a ready flag for that sub-tile.
//  * No grid-wide barrier: every CTA builds its own phase-0 records in a private scratch
//    slice; the producer issues a phase-1 record copy only once the flag of the h
//    sub-tile it reads equals epoch + 1 (epoch = launches completed, advanced by the last
//    CTA to finish), so weights of both phases stream without a pause.
// Every spin-wait is bounded by a global-timer timeout and reports through p.err.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "tk_engine.h"
#include "tk_ptx.cuh"

namespace tk {

namespace {

constexpr int kNC = kSlices;  // consumer warps per CTA (plus one producer warp)

// CTA whose stream-K range holds unit u (ranges [U*b/W, U*(b+1)/W), all non-empty)
__device__ __forceinline__ long long cta_of_unit(long long u, long long units, long long W) {
  return ((u + 1) * W - 1) / units;
}

__device__ __forceinline__ long long phase_ctas(const PhaseParams& P, long long Wtot) {
  return P.units < Wtot ? P.units : Wtot;
}

// Number of CTAs whose ranges intersect column unit cu (= wide tile * nmat + mat).
__device__ __forceinline__ int nseg_of_cu(const PhaseParams& P, long long cu, long long Wtot) {
  const long long W = phase_ctas(P, Wtot);
  const long long per = (long long)P.groups * P.spg;
  const long long a = cu * per;
  return (int)(cta_of_unit(a + per - 1, P.units, W) - cta_of_unit(a, P.units, W) + 1);
}

__device__ __forceinline__ int active_slices(const PhaseParams& P, int wtile) {
  const int rem = (P.N - wtile * kWideCols) / kTileCols;
  return rem < kSlices ? rem : kSlices;
}

// Walks one CTA's items (one group of one wide tile each) through all phases.
struct ItemIter {
  int ph;       // phase of the current item; == nphases when exhausted
  int i, n;     // index within the phase, items in the phase
  int cu, grp;  // column unit (tile * nmat + mat) and group of the current item
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
      it.i = 0;
      it.n = (int)(fgl - fg0 + 1);
      it.cu = (int)(fg0 / P.groups);
      it.grp = (int)(fg0 - (long long)it.cu * P.groups);
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
    if (++it.grp == P.groups) {
      it.grp = 0;
      ++it.cu;
    }
    it.s0 = 0;
    it.s1 = it.i == it.n - 1 ? it.last_s1 : P.spg;
    return;
  }
  ++it.ph;
  iter_seek(it, p, w, Wtot);
}

// Total bytes a stage receives for item `it` (box rows, scales, zeros, record).
__device__ __forceinline__ uint32_t item_bytes(const PhaseParams& P, const ItemIter& it) {
  const int ns = active_slices(P, it.cu >> (P.nmat - 1));
  return (uint32_t)((it.s1 - it.s0) * kStepRows * kRowBytes + ns * (kScaleBytes + kZeroBytes) +
                    P.frag_bytes);
}

// Producer lane `lane` issues its share of item `it`'s weight-side copies: lane 0 the TMA
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

// Warp-collective bounded wait on a stage barrier.
__device__ __forceinline__ bool wait_stage(uint64_t* bar, uint32_t parity, unsigned* err,
                                           unsigned long long timeout_ns) {
  bool done = mbar_try_wait(bar, parity);
  if (!done) {
    const uint64_t t0 = global_timer_ns();
    while (!(done = mbar_try_wait(bar, parity))) {
      if (global_timer_ns() - t0 > timeout_ns) break;
    }
  }
  const bool all = __all_sync(0xffffffffu, done);
  if (!all && (threadIdx.x & 31) == 0) atomicOr(err, kErrTmaWait);
  return all;
}

__device__ __forceinline__ uint32_t pack_half2(__half lo, __half hi) {
  return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

// Warp-collective: lane l holds v[0..3] = values 4l..4l+3 of a 128-value activation
// chunk of token `tok`.  Writes the B fragments and metadata of the 128/gs groups of the
// chunk into `rec` (record of the chunk's first group).  k order inside a k-step follows
// the A-fragment construction: MMA k index (2t, 2t+1, 2t+8, 2t+9) <-> step-local k
// (4t, 4t+2, 4t+1, 4t+3); odd k carry an extra 1/16.
template <int MT>
__device__ __forceinline__ void build_records(const float (&v)[4], int tok, int gs,
                                              uint8_t* rec, int rec_bytes, int lane) {
  const int gl = gs >> 2;  // lanes per group
  float mx = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
  for (int off = 1; off < gl; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  int e = 0;
  if (mx > 0.f && mx <= 3.0e38f) {
    int E;
    frexpf(mx, &E);
    e = 14 - E;  // max |x * 2^e| in [2^13, 2^14)
    e = e < -100 ? -100 : (e > 100 ? 100 : e);
  }
  const float x0 = ldexpf(v[0], e), x1 = ldexpf(v[1], e);
  const float x2 = ldexpf(v[2], e), x3 = ldexpf(v[3], e);
  const float o1 = ldexpf(v[1], e - 4), o3 = ldexpf(v[3], e - 4);
  const __half h0 = __float2half_rn(x0), h2 = __float2half_rn(x2);
  const __half h1 = __float2half_rn(o1), h3 = __float2half_rn(o3);
  const __half l0 = __float2half_rn(x0 - __half2float(h0));
  const __half l2 = __float2half_rn(x2 - __half2float(h2));
  const __half l1 = __float2half_rn(o1 - __half2float(h1));
  const __half l3 = __float2half_rn(o3 - __half2float(h3));
  const int gi = lane / gl, lg = lane - gi * gl;
  const int s = lg >> 2, t = lg & 3;
  const int spg = gs >> 4;
  uint8_t* r = rec + (size_t)gi * rec_bytes;
  uint2* b = reinterpret_cast<uint2*>(r);
  b[(s * 4 + t) * 2 * MT + 2 * tok + 0] = make_uint2(pack_half2(h0, h2), pack_half2(h1, h3));
  b[(s * 4 + t) * 2 * MT + 2 * tok + 1] = make_uint2(pack_half2(l0, l2), pack_half2(l1, l3));
  float sum = (x0 + x1) + (x2 + x3);
  sum += __shfl_xor_sync(0xffffffffu, sum, 1);
  sum += __shfl_xor_sync(0xffffffffu, sum, 2);
  if (t == 0) {
    float2* meta = reinterpret_cast<float2*>(r + spg * 4 * 2 * MT * 8);
    meta[s * MT + tok] = make_float2(sum * 0x1p-24f, ldexpf(1.0f, 24 - e));
  }
}

// One k-step of one slice for this lane: 2 x 16 B smem loads, 8 MMAs.  `step` points at
// the step's first box row plus the slice's byte offset; row r of the step is at
// r * kRowBytes.
template <int MT>
__device__ __forceinline__ void compute_step(const uint8_t* step, const uint2* fragb, int g, int t,
                                             const uint32_t (&cls_mask)[4 / MT], int cB,
                                             float (&D)[2 * MT][4]) {
  const uint4 U = *reinterpret_cast<const uint4*>(step + (2 * t) * kRowBytes + 16 * g);
  const uint4 V = *reinterpret_cast<const uint4*>(step + (2 * t + 1) * kRowBytes + 16 * g);
  const uint2 bf = fragb[t * 2 * MT + cB];
  constexpr int NCL = 4 / MT;
  uint32_t bx[NCL], by[NCL];
#pragma unroll
  for (int c = 0; c < NCL; ++c) {
    bx[c] = bf.x & cls_mask[c];
    by[c] = bf.y & cls_mask[c];
  }
  const uint32_t uw[4] = {U.x, U.y, U.z, U.w};
  const uint32_t vw[4] = {V.x, V.y, V.z, V.w};
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int wd = j >> 1;
    const uint32_t bA = (j & 1) * 2, bB = bA + 1;
    const uint32_t pA = prmt(uw[wd], vw[wd], bA | (bA << 4) | ((bA + 4) << 8) | ((bA + 4) << 12));
    const uint32_t pB = prmt(uw[wd], vw[wd], bB | (bB << 4) | ((bB + 4) << 8) | ((bB + 4) << 12));
    mma_16816(D[j % (2 * MT)], pA & 0x000F000Fu, pB & 0x000F000Fu, pA & 0x00F000F0u,
              pB & 0x00F000F0u, bx[j / (2 * MT)], by[j / (2 * MT)]);
  }
}

// Applies the group's scales and zero points to the MMA sums and resets them.
template <int MT>
__device__ __forceinline__ void group_epilogue(const uint8_t* scales, const uint8_t* zeros,
                                               const float2* meta, int s0, int s1, int tokE,
                                               int colbase, float (&D)[2 * MT][4],
                                               float (&y)[4 * MT]) {
  float sxs = 0.f;
  for (int s = s0; s < s1; ++s) sxs += meta[s * MT + tokE].x;
  const float gsc = meta[s0 * MT + tokE].y;
  const __half* sc = reinterpret_cast<const __half*>(scales) + colbase;
  const uint8_t* zp = zeros + colbase / 2;
#pragma unroll
  for (int r = 0; r < 2 * MT; ++r) {
    const float2 sf = __half22float2(*reinterpret_cast<const __half2*>(sc + 2 * r));
    const uint32_t zz = zp[r];
    const float za = (float)(zz & 15u), zb = (float)(zz >> 4);
    const float va = D[r][0] + D[r][1];
    const float vb = D[r][2] + D[r][3];
    y[2 * r] = fmaf(sf.x * gsc, fmaf(-za, sxs, va), y[2 * r]);
    y[2 * r + 1] = fmaf(sf.y * gsc, fmaf(-zb, sxs, vb), y[2 * r + 1]);
    D[r][0] = D[r][1] = D[r][2] = D[r][3] = 0.f;
  }
}

// The last warp to finish a tile: deterministic reduction of the partials + epilogue.
template <int MT>
__device__ void fixup_tile(const PhaseParams& P, int m, int wt, int slice, long long Wtot,
                           int lane, unsigned epoch) {
  for (int tok = 0; tok < MT; ++tok) {
    float acc[kMaxMats][4];
#pragma unroll
    for (int mi = 0; mi < kMaxMats; ++mi) acc[mi][0] = acc[mi][1] = acc[mi][2] = acc[mi][3] = 0.f;
    for (int mi = 0; mi < P.nmat; ++mi) {
      const long long cu = (long long)wt * P.nmat + mi;
      const int ns = nseg_of_cu(P, cu, Wtot);
      const float* base =
          P.partials + (((size_t)cu * P.maxseg * kSlices + slice) * MT + tok) * 128 + 4 * lane;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      for (int s = 0; s < ns; ++s) {
        const float4 v =
            __ldcg(reinterpret_cast<const float4*>(base + (size_t)s * kSlices * MT * 128));
        a0 += v.x;
        a1 += v.y;
        a2 += v.z;
        a3 += v.w;
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

template <int MT>
__device__ __forceinline__ void flush_segment(const PhaseParams& P, int m, int cu, long long b,
                                              long long Wtot, int slice, float (&y)[4 * MT],
                                              int lane, int tokE, int colbase, unsigned epoch) {
  const long long W = phase_ctas(P, Wtot);
  const long long a = (long long)cu * P.groups * P.spg;
  const int seg = (int)(b - cta_of_unit(a, P.units, W));
  const int wt = cu >> (P.nmat - 1);
  const int sub = wt * kSlices + slice;
  float* dst =
      P.partials + ((((size_t)cu * P.maxseg + seg) * kSlices + slice) * MT + tokE) * 128 + colbase;
#pragma unroll
  for (int i = 0; i < MT; ++i)
    *reinterpret_cast<float4*>(dst + 4 * i) = make_float4(y[4 * i], y[4 * i + 1], y[4 * i + 2], y[4 * i + 3]);
  __threadfence();
  __syncwarp();
  unsigned last = 0;
  if (lane == 0) {
    unsigned total = 0;
    for (int mi = 0; mi < P.nmat; ++mi)
      total += (unsigned)nseg_of_cu(P, (long long)wt * P.nmat + mi, Wtot);
    const unsigned prev = atomicAdd(&P.counters[sub], 1u);
    last = (prev == total - 1) ? 1u : 0u;
  }
  last = __shfl_sync(0xffffffffu, last, 0);
  if (last) {
    __threadfence();
    fixup_tile<MT>(P, m, wt, slice, Wtot, lane, epoch);
    __syncwarp();
    if (lane == 0) atomicExch(&P.counters[sub], 0u);
  }
#pragma unroll
  for (int i = 0; i < 4 * MT; ++i) y[i] = 0.f;
}

// Consumer warps: x (optionally rmsnorm'ed, src/kernels/shaders.zig:16-56) -> records.
template <int MT>
__device__ void prologue(const EngineParams& p, int warp, int lane, float* s_red, float* s_rms) {
  if (p.do_norm) {
    for (int tok = 0; tok < p.m; ++tok) {
      const float* xr = p.x + (size_t)tok * p.ldx;
      float ss = 0.f;
      for (int i = threadIdx.x; i < p.K0; i += kNC * 32) {
        const float v = xr[i];
        ss = fmaf(v, v, ss);
      }
      for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      if (lane == 0) s_red[warp] = ss;
      named_barrier(1, kNC * 32);
      if (threadIdx.x == 0) {
        float tot = 0.f;
        for (int i = 0; i < kNC; ++i) tot += s_red[i];
        s_rms[tok] = rsqrtf(tot / (float)p.K0 + p.eps);
      }
      named_barrier(1, kNC * 32);
    }
  }
  const int nchunks = p.K0 / kTileCols;
  uint8_t* recs = p.frag0 + (long long)blockIdx.x * p.frag0_cta_stride;
  for (int c = warp; c < MT * nchunks; c += kNC) {
    const int tok = (int)(c / nchunks), ch = (int)(c - (long long)tok * nchunks);
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (tok < p.m) {
      const float4 xv =
          *reinterpret_cast<const float4*>(p.x + (size_t)tok * p.ldx + ch * kTileCols + 4 * lane);
      v[0] = xv.x;
      v[1] = xv.y;
      v[2] = xv.z;
      v[3] = xv.w;
      if (p.do_norm) {
        const float4 wv = *reinterpret_cast<const float4*>(p.norm_w + ch * kTileCols + 4 * lane);
        const float rms = s_rms[tok];
        v[0] = v[0] * rms * wv.x;
        v[1] = v[1] * rms * wv.y;
        v[2] = v[2] * rms * wv.z;
        v[3] = v[3] * rms * wv.w;
      }
    }
    build_records<MT>(v, tok, p.gs0, recs + (size_t)(ch * kTileCols / p.gs0) * p.frag0_bytes,
                      p.frag0_bytes, lane);
  }
  fence_proxy_async();  // read back by this CTA's producer through TMA
}

template <int MT>
__global__ void __launch_bounds__((kNC + 1) * 32, 1)
    int4_engine_kernel(const __grid_constant__ TmapPack maps, const __grid_constant__ EngineParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ float s_red[kNC];
  __shared__ float s_rms[MT];
  __shared__ long long s_issued;
  __shared__ unsigned s_epoch;
  __shared__ volatile int s_records;  // this CTA's phase-0 records are written
  __shared__ volatile int s_abort;
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.stages;
  uint8_t* tiles = smem;
  uint8_t* auxs = smem + (size_t)S * p.tile_stage_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(auxs + (size_t)S * p.aux_stage_bytes);
  uint64_t* empty = full + S;
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kNC);
    }
    fence_mbar_init();
    s_records = 0;
    s_abort = 0;
    s_issued = 0;
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

  if (warp == kNC) {
    // ------------------------------- producer warp -------------------------------------
    const uint64_t pol_stream = l2_evict_first();
    const uint64_t pol_keep = l2_evict_last();
    ItemIter wi, fi;  // next item whose weights / whose activation record to issue
    iter_start(wi, p, b, Ptot);
    fi = wi;
    long long G = 0, F = 0;  // items with weights issued / with records issued
    int wslot = 0, fslot = 0;
    uint32_t wround = 0;
    bool aborted = false;
    uint64_t t_idle = 0;
    uint32_t spins = 0;
    while (wi.ph < p.nphases || F < G) {
      if (s_abort) {
        aborted = true;
        break;
      }
      bool progress = false;
      if (wi.ph < p.nphases) {
        bool free_slot = wround == 0;
        if (!free_slot) free_slot = mbar_test_wait(&empty[wslot], (wround - 1) & 1);
        free_slot = __shfl_sync(0xffffffffu, free_slot, 0);
        if (free_slot) {
          const PhaseParams& P = p.ph[wi.ph];
          uint8_t* aux = auxs + (size_t)wslot * p.aux_stage_bytes;
          if (lane == 0) {
            if (G == 0) trace_event(p, 7);
            mbar_arrive_expect_tx(&full[wslot], item_bytes(P, wi));
          }
          __syncwarp();
          issue_weights(maps, P, wi, tiles + (size_t)wslot * p.tile_stage_bytes, aux, &full[wslot],
                        pol_stream, lane);
          ++G;
          iter_next(wi, p, b, Ptot);
          if (++wslot == S) {
            wslot = 0;
            ++wround;
          }
          progress = true;
        }
      }
      if (F < G) {
        const PhaseParams& P = p.ph[fi.ph];
        bool ready;
        if (P.ready_in == nullptr) {
          ready = s_records != 0;
        } else {
          ready = ld_acquire_u32(&P.ready_in[fi.grp * P.gs / kTileCols]) == epoch + 1;
        }
        ready = __shfl_sync(0xffffffffu, ready, 0);
        if (ready) {
          fence_proxy_async();  // records were written by generic stores
          if (lane == 10)
            issue_frag(P, fi, b, auxs + (size_t)fslot * p.aux_stage_bytes, &full[fslot], pol_keep);
          ++F;
          iter_next(fi, p, b, Ptot);
          fslot = fslot + 1 == S ? 0 : fslot + 1;
          progress = true;
        }
      }
      if (progress) {
        t_idle = 0;
        spins = 0;
      } else if ((++spins & 63u) == 0) {
        const uint64_t now = __shfl_sync(0xffffffffu, global_timer_ns(), 0);
        if (t_idle == 0) {
          t_idle = now;
        } else if (now - t_idle > p.timeout_ns) {
          if (lane == 0) atomicOr(p.err, kErrFlagWait);
          aborted = true;
          break;
        }
        __nanosleep(64);
      }
    }
    if (aborted) {
      // complete the armed stages so every issued copy lands before the CTA exits
      while (F < G) {
        if (lane == 10)
          issue_frag(p.ph[fi.ph], fi, b, auxs + (size_t)fslot * p.aux_stage_bytes, &full[fslot],
                     pol_keep);
        ++F;
        iter_next(fi, p, b, Ptot);
        fslot = fslot + 1 == S ? 0 : fslot + 1;
      }
    }
    if (lane == 0) {
      s_issued = G;
      trace_event(p, 8);
    }
  } else {
    // ------------------------------- consumer warps ------------------------------------
    const int slice = warp;
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

    prologue<MT>(p, warp, lane, s_red, s_rms);
    named_barrier(1, kNC * 32);
    if (threadIdx.x == 0) {
      __threadfence_block();
      s_records = 1;
      trace_event(p, 1);
    }

    for (int ph = 0; ph < p.nphases && ok; ++ph) {
      const PhaseParams& P = p.ph[ph];
      float D[2 * MT][4];
      float y[4 * MT];
#pragma unroll
      for (int r = 0; r < 2 * MT; ++r) D[r][0] = D[r][1] = D[r][2] = D[r][3] = 0.f;
#pragma unroll
      for (int i = 0; i < 4 * MT; ++i) y[i] = 0.f;
      while (it.ph == ph) {
        if (!wait_stage(&full[slot], parity, p.err, p.timeout_ns)) {
          ok = false;
          s_abort = 1;
          break;
        }
        if (consumed == 0 && threadIdx.x == 0) trace_event(p, 9);
        const int wt = it.cu >> (P.nmat - 1);
        const bool active = slice < active_slices(P, wt);
        const uint8_t* ax = auxs + (size_t)slot * p.aux_stage_bytes;
        if (active) {
          const uint8_t* tl = tiles + (size_t)slot * p.tile_stage_bytes + slice * kTileCols;
          const uint2* fb = reinterpret_cast<const uint2*>(frag_slot(const_cast<uint8_t*>(ax)));
          for (int s = it.s0; s < it.s1; ++s)
            compute_step<MT>(tl + s * kStepRows * kRowBytes, fb + s * 4 * 2 * MT, g, t, cls_mask,
                             cB, D);
          const float2* meta = reinterpret_cast<const float2*>(fb + P.spg * 4 * 2 * MT);
          group_epilogue<MT>(ax + slice * kScaleBytes,
                             ax + kSlices * kScaleBytes + slice * kZeroBytes, meta, it.s0, it.s1,
                             tokE, colbase, D, y);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        ++consumed;
        if (++slot == S) {
          slot = 0;
          parity ^= 1u;
        }
        const int cu = it.cu;
        const bool last_of_cu = (it.i == it.n - 1) || (it.grp == P.groups - 1);
        iter_next(it, p, b, Ptot);
        if (last_of_cu && active)
          flush_segment<MT>(P, p.m, cu, b, Ptot, slice, y, lane, tokE, colbase, epoch);
      }
      if (threadIdx.x == 0) trace_event(p, 3 + 2 * ph);
    }
  }
  __syncthreads();
  if (warp < kNC) {
    // Only after an error: wait for the stages the producer armed but the consumers did
    // not take (the producer completed their records before leaving), so no copy is in
    // flight when the CTA exits.
    for (long long G = consumed; G < s_issued; ++G) {
      wait_stage(&full[slot], parity, p.err, p.timeout_ns);
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
  cfg.blockDim = dim3((kNC + 1) * 32);
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
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, kern, (kNC + 1) * 32, smem);
}

}  // namespace

int engine_warps_per_cta() { return kNC; }

size_t engine_smem_bytes(int stages, int tile_stage_bytes, int aux_stage_bytes) {
  return 1024 + (size_t)stages * ((size_t)tile_stage_bytes + aux_stage_bytes + 16);
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
