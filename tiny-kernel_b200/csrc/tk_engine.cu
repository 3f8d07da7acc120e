// tk_engine.cu -- persistent, TMA-fed INT4 fused-dequant GEMV engine for sm_100a.
//
// Computes the qmatmul_int4 contraction of the reference (src/kernels/shaders.zig:442-501)
//     y[m][n] = sum_g scale[g][n] * sum_{k in g} x[m][k] * (q[k][n] - zero[g][n])
// on the reference's packed layout, and the INT4 Llama FFN built from it
// (src/bench.zig:266-341 gate/up composition plus the down projection).
//
// Design (one CTA per SM, NW consumer warps, each warp with its own TMA ring):
//  * A work unit is one k-step (8 packed rows = 16 k) of a 128-column tile of one matrix.
//    Units are ordered tile-major, matrix, group, step; warp w of W owns units
//    [U*w/W, U*(w+1)/W) (stream-K), so every SM streams the same number of bytes.
//  * Per group the warp's lane 0 issues: one 8-row x 128 B TMA tensor box per k-step
//    (128B swizzle), one 256 B bulk copy of the group's f16 scales and one 64 B bulk copy
//    of its zero points, and one bulk copy of the group's activation record.
//  * The weight nibbles are turned into m16n8k16 A fragments with one PRMT and two LOPs
//    per 4 nibbles: each nibble lands in the mantissa of an f16 subnormal, so the MMA sees
//    q * 2^-24 exactly (even k) or 16 q * 2^-24 (odd k; the activations carry the 1/16).
//    Zero points are applied per group in f32 as  - z * sum_k x_k.
//  * Activations arrive as precomputed B fragments: x is scaled by a power of two per
//    group and split x = hi + lo into two f16 values (B columns 2c, 2c+1), so the
//    products keep ~22 significant bits and accumulate in f32 in the tensor core.
//  * Split-K partial sums go to a scratch buffer; the last warp to finish a tile (an
//    atomic counter per tile) adds the partials in warp order (deterministic) and runs
//    the epilogue: store (+ residual), or silu(gate) * up -> the next phase's records.
//  * Phases are separated by a grid barrier; the next phase's weight loads are issued
//    before the barrier so HBM keeps streaming across it.
// Every spin-wait is bounded by a global-timer timeout and reports through p.err.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "tk_engine.h"
#include "tk_ptx.cuh"

namespace tk {

namespace {

constexpr int kNW = 8;  // consumer warps per CTA

struct Item {
  long long cu;  // tile * nmat + mat
  int tile, mat, grp, s0, s1;
};

struct Range {
  long long beg, end, fg0;
  int n;
};

__device__ __forceinline__ long long warp_of_unit(long long u, long long units, long long W) {
  return ((u + 1) * W - 1) / units;
}

__device__ __forceinline__ long long phase_warps(const PhaseParams& P, long long Wtot) {
  return P.units < Wtot ? P.units : Wtot;
}

__device__ __forceinline__ Range warp_range(const PhaseParams& P, long long w, long long Wtot) {
  Range r;
  const long long W = phase_warps(P, Wtot);
  if (w >= W) {
    r.beg = r.end = r.fg0 = 0;
    r.n = 0;
    return r;
  }
  r.beg = P.units * w / W;
  r.end = P.units * (w + 1) / W;
  r.fg0 = r.beg / P.spg;
  r.n = (int)((r.end - 1) / P.spg - r.fg0 + 1);
  return r;
}

__device__ __forceinline__ Item make_item(const PhaseParams& P, const Range& r, int i) {
  Item it;
  const long long fg = r.fg0 + i;
  const long long gstart = fg * P.spg;
  it.s0 = (int)(r.beg > gstart ? r.beg - gstart : 0);
  it.s1 = (int)(r.end - gstart < P.spg ? r.end - gstart : P.spg);
  it.cu = fg / P.groups;
  it.grp = (int)(fg - it.cu * P.groups);
  it.tile = (int)(it.cu / P.nmat);
  it.mat = (int)(it.cu - (long long)it.tile * P.nmat);
  return it;
}

__device__ __forceinline__ int nseg_of_cu(const PhaseParams& P, long long cu, long long Wtot) {
  const long long W = phase_warps(P, Wtot);
  const long long per = (long long)P.groups * P.spg;
  const long long a = cu * per;
  return (int)(warp_of_unit(a + per - 1, P.units, W) - warp_of_unit(a, P.units, W) + 1);
}

// lane 0 only
__device__ __forceinline__ void issue_item(const TmapPack& maps, const PhaseParams& P,
                                           const Item& it, uint8_t* tile, uint8_t* aux,
                                           uint64_t* bar, bool weights, bool frag,
                                           uint64_t pol_stream, uint64_t pol_keep) {
  if (weights) {
    const uint32_t bytes =
        (uint32_t)((it.s1 - it.s0) * kStepBytes + kScaleBytes + kZeroBytes + P.frag_bytes);
    mbar_arrive_expect_tx(bar, bytes);
    const CUtensorMap* map = &maps.map[P.map_base + it.mat];
    const int row0 = it.grp * P.spg * kStepRows;
    for (int s = it.s0; s < it.s1; ++s)
      tma_load_2d(tile + s * kStepBytes, map, bar, it.tile * kTileCols, row0 + s * kStepRows,
                  pol_stream);
    const uint16_t* sc = P.scales[it.mat] + (size_t)it.grp * P.N + (size_t)it.tile * kTileCols;
    bulk_load(aux, sc, kScaleBytes, bar, pol_stream);
    const uint8_t* zp =
        P.zeros[it.mat] + (size_t)it.grp * (P.N / 2) + (size_t)it.tile * (kTileCols / 2);
    bulk_load(aux + kScaleBytes, zp, kZeroBytes, bar, pol_stream);
  }
  if (frag) {
    bulk_load(aux + kScaleBytes + kZeroBytes, P.frag_in + (size_t)it.grp * P.frag_bytes,
              (uint32_t)P.frag_bytes, bar, pol_keep);
  }
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

// Grid-wide barrier for a cooperative launch; generation counter, self-resetting.
__device__ bool grid_sync(GridBar* gb, unsigned* err, unsigned long long timeout_ns) {
  __shared__ int s_ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    const unsigned gen = ld_acquire_u32(&gb->gen);
    __threadfence();
    const unsigned prev = atomicAdd(&gb->count, 1u);
    if (prev == gridDim.x - 1) {
      atomicExch(&gb->count, 0u);
      __threadfence();
      atomicAdd(&gb->gen, 1u);
    } else {
      const uint64_t t0 = global_timer_ns();
      while (ld_acquire_u32(&gb->gen) == gen) {
        __nanosleep(64);
        if (global_timer_ns() - t0 > timeout_ns) {
          atomicOr(err, kErrGridBarrier);
          ok = 0;
          break;
        }
      }
    }
    __threadfence();
    if (ld_acquire_u32(err) != 0) ok = 0;
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
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

// One k-step of one tile for this lane: 2 x 16 B smem loads, 8 MMAs.
template <int MT>
__device__ __forceinline__ void compute_step(const uint8_t* tile_step, const uint2* fragb, int g,
                                             int t, const uint32_t (&cls_mask)[4 / MT], int cB,
                                             float (&D)[2 * MT][4]) {
  const uint4 U = *reinterpret_cast<const uint4*>(tile_step + (2 * t) * 128 + ((g ^ (2 * t)) << 4));
  const uint4 V =
      *reinterpret_cast<const uint4*>(tile_step + (2 * t + 1) * 128 + ((g ^ (2 * t + 1)) << 4));
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
__device__ __forceinline__ void group_epilogue(const uint8_t* aux, const float2* meta, int s0,
                                               int s1, int tokE, int colbase,
                                               float (&D)[2 * MT][4], float (&y)[4 * MT]) {
  float sxs = 0.f;
  for (int s = s0; s < s1; ++s) sxs += meta[s * MT + tokE].x;
  const float gsc = meta[s0 * MT + tokE].y;
  const __half* sc = reinterpret_cast<const __half*>(aux) + colbase;
  const uint8_t* zp = aux + kScaleBytes + colbase / 2;
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
__device__ void fixup_tile(const PhaseParams& P, int m, int tile, long long Wtot, int lane) {
  for (int tok = 0; tok < MT; ++tok) {
    float acc[kMaxMats][4];
#pragma unroll
    for (int mi = 0; mi < kMaxMats; ++mi) acc[mi][0] = acc[mi][1] = acc[mi][2] = acc[mi][3] = 0.f;
    for (int mi = 0; mi < P.nmat; ++mi) {
      const long long cu = (long long)tile * P.nmat + mi;
      const int ns = nseg_of_cu(P, cu, Wtot);
      const float* base = P.partials + ((size_t)cu * P.maxseg * MT + tok) * 128 + 4 * lane;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      for (int s = 0; s < ns; ++s) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(base + (size_t)s * MT * 128));
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
    const int col = tile * kTileCols + 4 * lane;
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
                        P.frag_out + (size_t)(tile * kTileCols / P.next_gs) * P.next_frag_bytes,
                        P.next_frag_bytes, lane);
    }
  }
  if (P.epi == kEpiSiluMul) fence_proxy_async();
}

template <int MT>
__device__ __forceinline__ void flush_segment(const PhaseParams& P, int m, const Item& it,
                                              long long w, long long Wtot, float (&y)[4 * MT],
                                              int lane, int tokE, int colbase) {
  const long long W = phase_warps(P, Wtot);
  const long long a = it.cu * (long long)P.groups * P.spg;
  const int seg = (int)(w - warp_of_unit(a, P.units, W));
  float* dst = P.partials + (((size_t)it.cu * P.maxseg + seg) * MT + tokE) * 128 + colbase;
#pragma unroll
  for (int i = 0; i < MT; ++i)
    *reinterpret_cast<float4*>(dst + 4 * i) = make_float4(y[4 * i], y[4 * i + 1], y[4 * i + 2], y[4 * i + 3]);
  __threadfence();
  __syncwarp();
  unsigned last = 0;
  if (lane == 0) {
    unsigned total = 0;
    for (int mi = 0; mi < P.nmat; ++mi) total += (unsigned)nseg_of_cu(P, (long long)it.tile * P.nmat + mi, Wtot);
    const unsigned prev = atomicAdd(&P.counters[it.tile], 1u);
    last = (prev == total - 1) ? 1u : 0u;
  }
  last = __shfl_sync(0xffffffffu, last, 0);
  if (last) {
    __threadfence();
    fixup_tile<MT>(P, m, it.tile, Wtot, lane);
    __syncwarp();
    if (lane == 0) atomicExch(&P.counters[it.tile], 0u);
  }
#pragma unroll
  for (int i = 0; i < 4 * MT; ++i) y[i] = 0.f;
}

// x (optionally rmsnorm'ed, src/kernels/shaders.zig:16-56) -> activation records frag0.
template <int MT>
__device__ void prologue(const EngineParams& p, int warp, int lane, float* s_red, float* s_rms) {
  if (p.do_norm) {
    for (int tok = 0; tok < p.m; ++tok) {
      const float* xr = p.x + (size_t)tok * p.ldx;
      float ss = 0.f;
      for (int i = threadIdx.x; i < p.K0; i += kNW * 32) {
        const float v = xr[i];
        ss = fmaf(v, v, ss);
      }
      for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      if (lane == 0) s_red[warp] = ss;
      __syncthreads();
      if (threadIdx.x == 0) {
        float tot = 0.f;
        for (int i = 0; i < kNW; ++i) tot += s_red[i];
        s_rms[tok] = rsqrtf(tot / (float)p.K0 + p.eps);
      }
      __syncthreads();
    }
  }
  const int nchunks = p.K0 / kTileCols;
  const long long Wtot = (long long)gridDim.x * kNW;
  const long long w = (long long)blockIdx.x * kNW + warp;
  for (long long c = w; c < (long long)MT * nchunks; c += Wtot) {
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
    build_records<MT>(v, tok, p.gs0, p.frag0 + (size_t)(ch * kTileCols / p.gs0) * p.frag0_bytes,
                      p.frag0_bytes, lane);
  }
  fence_proxy_async();
}

template <int MT>
__global__ void __launch_bounds__(kNW * 32, 1)
    int4_engine_kernel(const __grid_constant__ TmapPack maps, const __grid_constant__ EngineParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ float s_red[kNW];
  __shared__ float s_rms[MT];
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.stages;
  uint8_t* my_tiles = smem + (size_t)warp * S * p.tile_stage_bytes;
  uint8_t* my_aux = smem + (size_t)kNW * S * p.tile_stage_bytes + (size_t)warp * S * p.aux_stage_bytes;
  uint64_t* my_bars =
      reinterpret_cast<uint64_t*>(smem + (size_t)kNW * S * (p.tile_stage_bytes + p.aux_stage_bytes)) +
      warp * S;
  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&my_bars[s], 1);
    fence_mbar_init();
  }
  __syncwarp();

  const long long Wtot = (long long)gridDim.x * kNW;
  const long long w = (long long)blockIdx.x * kNW + warp;
  const uint64_t pol_stream = l2_evict_first();
  const uint64_t pol_keep = l2_evict_last();
  const int g = lane >> 2, t = lane & 3, q = g >> 1;
  const int cB = 2 * (q % MT) + (g & 1);
  const int tokE = t % MT;
  const int colbase = 16 * g + 4 * MT * (t / MT);
  uint32_t cls_mask[4 / MT];
#pragma unroll
  for (int c = 0; c < 4 / MT; ++c) cls_mask[c] = (q / MT == c) ? 0xffffffffu : 0u;

  Range rng[kMaxPhases];
  long long first[kMaxPhases + 1];
  first[0] = 0;
  for (int ph = 0; ph < kMaxPhases; ++ph) {
    if (ph < p.nphases) {
      rng[ph] = warp_range(p.ph[ph], w, Wtot);
    } else {
      rng[ph].n = 0;
      rng[ph].beg = rng[ph].end = rng[ph].fg0 = 0;
    }
    first[ph + 1] = first[ph] + rng[ph].n;
  }

  long long issued = 0, consumed = 0;
  int passed = -1;  // highest phase whose activation records are complete
  bool ok = true;

  // Issues ring items (in order) while a slot is free, up to phase `max_ph`.
  auto issue_more = [&](int max_ph) {
    while (issued - consumed < S) {
      int ph = 0;
      while (ph < p.nphases && issued >= first[ph + 1]) ++ph;
      if (ph >= p.nphases || ph > max_ph) break;
      if (lane == 0) {
        const int slot = (int)(issued % S);
        const Item it = make_item(p.ph[ph], rng[ph], (int)(issued - first[ph]));
        issue_item(maps, p.ph[ph], it, my_tiles + (size_t)slot * p.tile_stage_bytes,
                   my_aux + (size_t)slot * p.aux_stage_bytes, &my_bars[slot], true, ph <= passed,
                   pol_stream, pol_keep);
      }
      ++issued;
    }
  };

  issue_more(0);  // phase-0 weights stream while the prologue runs
  prologue<MT>(p, warp, lane, s_red, s_rms);

  for (int ph = 0; ph < p.nphases; ++ph) {
    if (!grid_sync(p.bar, p.err, p.timeout_ns)) {
      ok = false;
      break;
    }
    const PhaseParams& P = p.ph[ph];
    passed = ph;
    // activation records of this phase are ready: complete the deferred stages
    if (lane == 0) {
      fence_proxy_async();  // records were written by other CTAs' generic stores
      const long long hi = issued < first[ph + 1] ? issued : first[ph + 1];
      for (long long G = consumed > first[ph] ? consumed : first[ph]; G < hi; ++G) {
        const int slot = (int)(G % S);
        const Item it = make_item(P, rng[ph], (int)(G - first[ph]));
        issue_item(maps, P, it, my_tiles + (size_t)slot * p.tile_stage_bytes,
                   my_aux + (size_t)slot * p.aux_stage_bytes, &my_bars[slot], false, true,
                   pol_stream, pol_keep);
      }
    }
    __syncwarp();
    issue_more(ph + 1);

    float D[2 * MT][4];
    float y[4 * MT];
#pragma unroll
    for (int r = 0; r < 2 * MT; ++r) D[r][0] = D[r][1] = D[r][2] = D[r][3] = 0.f;
#pragma unroll
    for (int i = 0; i < 4 * MT; ++i) y[i] = 0.f;

    const Range& R = rng[ph];
    for (int i = 0; i < R.n; ++i) {
      const int slot = (int)(consumed % S);
      const uint32_t parity = (uint32_t)((consumed / S) & 1);
      if (!wait_stage(&my_bars[slot], parity, p.err, p.timeout_ns)) {
        ok = false;
        break;
      }
      const Item it = make_item(P, R, i);
      const uint8_t* tl = my_tiles + (size_t)slot * p.tile_stage_bytes;
      const uint8_t* ax = my_aux + (size_t)slot * p.aux_stage_bytes;
      const uint2* fb = reinterpret_cast<const uint2*>(ax + kScaleBytes + kZeroBytes);
      for (int s = it.s0; s < it.s1; ++s)
        compute_step<MT>(tl + s * kStepBytes, fb + s * 4 * 2 * MT, g, t, cls_mask, cB, D);
      const float2* meta = reinterpret_cast<const float2*>(fb + P.spg * 4 * 2 * MT);
      group_epilogue<MT>(ax, meta, it.s0, it.s1, tokE, colbase, D, y);
      ++consumed;
      __syncwarp();
      if (lane == 0) fence_proxy_async();
      issue_more(ph + 1);
      const bool last_of_cu = (i == R.n - 1) || ((R.fg0 + i + 1) / P.groups != it.cu);
      if (last_of_cu) flush_segment<MT>(P, p.m, it, w, Wtot, y, lane, tokE, colbase);
    }
  }

  if (!ok) {
    // Complete and drain every stage still in flight before the CTA exits.
    if (lane == 0) {
      for (long long G = consumed; G < issued; ++G) {
        int ph = 0;
        while (ph < p.nphases && G >= first[ph + 1]) ++ph;
        if (ph < p.nphases && ph > passed) {
          const int slot = (int)(G % S);
          const Item it = make_item(p.ph[ph], rng[ph], (int)(G - first[ph]));
          issue_item(maps, p.ph[ph], it, my_tiles + (size_t)slot * p.tile_stage_bytes,
                     my_aux + (size_t)slot * p.aux_stage_bytes, &my_bars[slot], false, true,
                     pol_stream, pol_keep);
        }
      }
    }
    __syncwarp();
    for (long long G = consumed; G < issued; ++G)
      wait_stage(&my_bars[G % S], (uint32_t)((G / S) & 1), p.err, p.timeout_ns);
  }
}

template <int MT>
cudaError_t launch_mt(const TmapPack& maps, const EngineParams& p, int grid, size_t smem,
                      cudaStream_t stream) {
  auto kern = int4_engine_kernel<MT>;
  static size_t configured = 0;
  if (configured < smem) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kNW * 32);
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
cudaError_t occupancy_mt(size_t smem, int* blocks) {
  auto kern = int4_engine_kernel<MT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, kern, kNW * 32, smem);
}

}  // namespace

int engine_warps_per_cta() { return kNW; }

size_t engine_smem_bytes(int stages, int tile_stage_bytes, int aux_stage_bytes) {
  return 1024 + (size_t)kNW * stages * ((size_t)tile_stage_bytes + aux_stage_bytes + 8);
}

cudaError_t engine_occupancy(int mt, size_t smem, int* blocks) {
  switch (mt) {
    case 1: return occupancy_mt<1>(smem, blocks);
    case 2: return occupancy_mt<2>(smem, blocks);
    case 4: return occupancy_mt<4>(smem, blocks);
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
