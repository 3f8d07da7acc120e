// tk_decode.cu -- the batch 1-2 decode kernel: qmatmul_int4 and the INT4 Llama FFN in one
// persistent launch per call, with a counter-free split-K exchange (tk_decode.h).
//
// Warp roles (one CTA per SM, 288 threads):
//   warp 8 (producer)   lane 0 issues every copy of the CTA: first the prologue data (x rows and
//                       the norm weight, 1-D bulk copies into the first ring stages), then per
//                       work item the packed rows (2-D TMA box of 1040-byte rows), the f16 scales
//                       and the packed zero points of a 1024-column tile and one group.  Items of
//                       phase B are copied as soon as a stage is free: their weights do not
//                       depend on h, so they land while phase A finishes and h is assembled.
//   warps 0-7 (consumers) slice w = 128 columns of every item, dp2a arithmetic (tk_dp2a.cuh).
//                       prologue: rmsnorm + the int16 records of every group of x, in smem;
//                       phase A, then (FFN) the phase-B records: h = silu(gate) * up summed from
//                       the tagged gate/up partials of the other CTAs, one item per warp, in
//                       parallel; phase B; finally the y reduction tasks of this CTA.
// Split-K exchange: a segment (one CTA's contiguous k range of one column unit) stores its
// partial sums as 64-bit words (tag << 32 | float bits) with plain stores; a reader loads the
// words of every segment it needs and retries until all carry this launch's tag, then sums them
// in segment order (deterministic: every reader gets the same bits).  The tag is the launch's
// epoch + 1: CTA b reads epoch[b] at its start and, at its end, writes epoch[b + k * grid] for
// every k, so every slot advances once per launch whatever the grid size, and no CTA writes a
// slot another CTA of the same launch reads.
// Every wait is bounded by a global-timer timeout and reports through p.err.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <mutex>

#include "tk_decode.h"
#include "tk_internal.h"
#include "tk_dp2a.cuh"
#include "tk_ptx.cuh"

namespace tk {

namespace {

constexpr int kNC = kDecConsumers;
constexpr int kProducerWarp = kNC;

// CTA whose stream-K range holds unit u (ranges [U*b/W, U*(b+1)/W))
__device__ __forceinline__ int dec_cta_of_unit(unsigned u, unsigned units, unsigned W) {
  return (int)(((u + 1) * W - 1) / units);
}

// Segments (CTA ranges) of column unit cu, and the first one's CTA.
__device__ __forceinline__ int dec_nseg(const DecPhase& P, int cu, int* first) {
  const unsigned per = (unsigned)(P.groups * P.spg);
  const unsigned a = (unsigned)cu * per;
  const int c0 = dec_cta_of_unit(a, P.units, P.ctas);
  if (first) *first = c0;
  return dec_cta_of_unit(a + per - 1, P.units, P.ctas) - c0 + 1;
}

// One CTA's walk over its items (one group of one column unit each) through the phases.
struct It {
  int ph;       // phase of the item; p.nph: done
  int i, n;     // item index within the phase, the CTA's items in the phase
  int cu, grp;  // column unit (phase tile * nmat + matrix) and group, both within the phase
  int s0, s1;   // k-steps [s0, s1) of the group
  int last_s1;
  int groups, spg, nmat, N, wt0, g0;  // the phase's sizes and offsets
};

__device__ __forceinline__ void it_seek(It& it, const DecodeParams& p, unsigned b) {
  while (it.ph < p.nph) {
    const DecPhase& P = p.ph[it.ph];
    if (b < P.ctas) {
      const unsigned U = P.units, W = P.ctas;
      const unsigned beg = U * b / W, end = U * (b + 1) / W;
      const unsigned fg0 = beg / (unsigned)P.spg, fgl = (end - 1) / (unsigned)P.spg;
      const unsigned cl = fg0 / (unsigned)P.groups;
      it.groups = P.groups;
      it.spg = P.spg;
      it.nmat = P.nmat;
      it.N = P.N;
      it.wt0 = P.wt0;
      it.g0 = P.g0;
      it.i = 0;
      it.n = (int)(fgl - fg0 + 1);
      it.cu = (int)cl;
      it.grp = (int)(fg0 - cl * (unsigned)P.groups);
      it.s0 = (int)(beg - fg0 * (unsigned)P.spg);
      it.last_s1 = (int)(end - fgl * (unsigned)P.spg);
      it.s1 = it.n == 1 ? it.last_s1 : P.spg;
      return;
    }
    ++it.ph;
  }
}

// The groups CTA b's ranges of the A phases touch (the x records it needs): per A phase an
// interval [gf, gl] of a column unit's groups, wrapping past the last group when gl < gf, or all.
struct NeedGroups {
  int gf[kDecMaxPhases], gl[kDecMaxPhases];
  bool all;
};

__device__ __forceinline__ NeedGroups a_range_groups(const DecodeParams& p, unsigned b) {
  NeedGroups n;
  n.all = false;
#pragma unroll
  for (int q = 0; q < kDecMaxPhases; ++q) {
    n.gf[q] = 1;  // empty unless set
    n.gl[q] = 0;
    const DecPhase& P = p.ph[q];
    if (q >= p.na || b >= P.ctas) continue;
    const unsigned beg = P.units * b / P.ctas, end = P.units * (b + 1) / P.ctas;
    if (end - beg >= (unsigned)(P.groups * P.spg)) n.all = true;  // every group of a unit
    n.gf[q] = (int)((beg / (unsigned)P.spg) % (unsigned)P.groups);
    n.gl[q] = (int)(((end - 1) / (unsigned)P.spg) % (unsigned)P.groups);
  }
  return n;
}

// Whether a group in [g0, g1) is among the needed ones.
__device__ __forceinline__ bool needs_groups(const DecodeParams& p, const NeedGroups& n, unsigned b,
                                             int g0, int g1) {
  if (n.all) return true;
#pragma unroll
  for (int q = 0; q < kDecMaxPhases; ++q) {
    if (q >= p.na || b >= p.ph[q].ctas) continue;
    const int gf = n.gf[q], gl = n.gl[q];
    if (gf <= gl ? (g0 <= gl && g1 > gf)    // [gf, gl]
                 : (g1 > gf || g0 <= gl))   // [gf, G) and [0, gl]
      return true;
  }
  return false;
}

// Items (groups touched) of CTA b's range in phase P.
__device__ __forceinline__ int phase_items(const DecPhase& P, unsigned b) {
  if (b >= P.ctas) return 0;
  const unsigned beg = P.units * b / P.ctas, end = P.units * (b + 1) / P.ctas;
  return (int)((end - 1) / (unsigned)P.spg - beg / (unsigned)P.spg + 1);
}

__device__ __forceinline__ void it_start(It& it, const DecodeParams& p, unsigned b) {
  it.ph = 0;
  it.i = it.n = it.cu = it.grp = it.s0 = it.s1 = it.last_s1 = 0;
  it.groups = it.spg = it.nmat = 1;
  it.N = it.wt0 = it.g0 = 0;
  it_seek(it, p, b);
}

__device__ __forceinline__ void it_next(It& it, const DecodeParams& p, unsigned b) {
  if (++it.i < it.n) {
    if (++it.grp == it.groups) {
      it.grp = 0;
      ++it.cu;
    }
    it.s0 = 0;
    it.s1 = it.i == it.n - 1 ? it.last_s1 : it.spg;
    return;
  }
  ++it.ph;
  it_seek(it, p, b);
}

// Absolute 1024-column tile of the item (of N) and its absolute group (of K).
__device__ __forceinline__ int it_tile(const It& it) { return it.wt0 + (it.cu >> (it.nmat - 1)); }
__device__ __forceinline__ int it_group(const It& it) { return it.g0 + it.grp; }

// 128-column slices of the item's tile that hold columns (8 except in a ragged last tile).
__device__ __forceinline__ int it_slices(const It& it) {
  const int rem = (it.N - it_tile(it) * kWideCols) / kTileCols;
  return rem < kSlices ? rem : kSlices;
}

__device__ __forceinline__ bool it_seg_end(const It& it) {
  return it.grp == it.groups - 1 || it.i == it.n - 1;
}

__device__ __forceinline__ void dec_trace(const DecodeParams& p, int ev) {
  if (p.trace) p.trace[(size_t)blockIdx.x * kTraceEvents + ev] = global_timer_ns();
}

// Packed rows + scales + zero points of item `it` into one stage (producer lane 0).
__device__ __forceinline__ void issue_item(const TmapPack& maps, const DecPhase& P, const It& it,
                                           uint8_t* tile, uint8_t* aux, uint64_t* bar,
                                           uint64_t pol) {
  const int mat = it.cu & (it.nmat - 1);
  const int wt = it_tile(it);
  const int ns = it_slices(it);
  const uint32_t bytes = (uint32_t)(it.spg * kStepRows * kRowBytes +
                                    ns * (kScaleBytes + kZeroBytes));
  mbar_arrive_expect_tx(bar, bytes);
  const int row0 = it_group(it) * it.spg * kStepRows;
  const int x = wt * (kWideCols / 8);  // u64 element of the tile's first byte
  if (it.s0 == 0 && it.s1 == it.spg) {
    tma_load_2d(tile, &maps.map[P.map_base + 2 * mat], bar, x, row0, pol);
  } else {
    // a partial item: its k-steps, and zero rows for the group's others (so the consumers need
    // no row masks: zero codes contribute nothing, and the zero-point sums cover its k-steps only)
    for (int s = 0; s < it.spg; ++s) {
      if (s >= it.s0 && s < it.s1)
        tma_load_2d(tile + s * kStepRows * kRowBytes, &maps.map[P.map_base + 2 * mat + 1], bar, x,
                    row0 + s * kStepRows, pol);
      else
        tma_load_2d(tile + s * kStepRows * kRowBytes, &maps.map[kZeroMap], bar, 0, 0, pol);
    }
  }
  const int col0 = wt * kWideCols;
  const size_t g = (size_t)it_group(it);
  bulk_load(aux, P.scales[mat] + g * P.N + col0, (uint32_t)(ns * kScaleBytes), bar, pol);
  bulk_load(aux + kSlices * kScaleBytes, P.zeros[mat] + g * (P.N / 2) + col0 / 2,
            (uint32_t)(ns * kZeroBytes), bar, pol);
}

__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// issue_item's copies as L2 prefetches (weights, scales, zero points: read-only inputs).
__device__ __forceinline__ void prefetch_item(const TmapPack& maps, const DecPhase& P, const It& it) {
  const int mat = it.cu & (it.nmat - 1);
  const int wt = it_tile(it);
  const int ns = it_slices(it);
  const int row0 = it_group(it) * it.spg * kStepRows;
  const int x = wt * (kWideCols / 8);
  if (it.s0 == 0 && it.s1 == it.spg) {
    tma_prefetch_2d(&maps.map[P.map_base + 2 * mat], x, row0);
  } else {
    for (int s = it.s0; s < it.s1; ++s)
      tma_prefetch_2d(&maps.map[P.map_base + 2 * mat + 1], x, row0 + s * kStepRows);
  }
  const int col0 = wt * kWideCols;
  const size_t g = (size_t)it_group(it);
  bulk_prefetch_l2(P.scales[mat] + g * P.N + col0, (uint32_t)(ns * kScaleBytes));
  bulk_prefetch_l2(P.zeros[mat] + g * (P.N / 2) + col0 / 2, (uint32_t)(ns * kZeroBytes));
}

__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ unsigned long long tagged(float v, unsigned tag) {
  return ((unsigned long long)tag << 32) | __float_as_uint(v);
}

__device__ __forceinline__ void st_cg_u64x2(unsigned long long* p, unsigned long long a,
                                            unsigned long long b) {
  asm volatile("st.global.cg.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}

__device__ __forceinline__ ulonglong2 ld_cg_u64x2(const unsigned long long* p) {
  ulonglong2 v;
  asm volatile("ld.global.cg.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
  return v;
}

// System-scope relaxed accesses of the peer exchange (single-copy atomic 64-bit words).
__device__ __forceinline__ void st_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long ld_cg_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.global.cg.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Tagged partial words of segment `seg` of column unit cu, token tok: 1024 columns.
template <int MT>
__device__ __forceinline__ unsigned long long* dec_part(const DecPhase& P, int cu, int seg, int tok) {
  return P.part + (((size_t)cu * P.maxseg + seg) * MT + tok) * kWideCols;
}

// Bounded wait for a stage; false on an abort or a timeout.
__device__ __forceinline__ bool dec_wait_full(uint64_t* bar, uint32_t par, volatile int* abort,
                                              unsigned* err, unsigned long long timeout_ns,
                                              int lane) {
  if (__all_sync(0xffffffffu, mbar_try_wait(bar, par))) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    if (__all_sync(0xffffffffu, mbar_try_wait_hint(bar, par, 1000))) return true;
    int st = 0;
    if (lane == 0) {
      if (*abort) st = 1;
      else if (global_timer_ns() - t0 > timeout_ns) {
        atomicOr(err, kErrTmaWait);
        st = 1;
      }
    }
    if (__shfl_sync(0xffffffffu, st, 0)) return false;
  }
}

// Per-stage item descriptors, written by the producer lane before it arms a stage (the stage's
// full barrier orders them before the consumers' reads): everything a consumer needs about the
// item in the stage, so the consumer loop carries no work-split iterator.
//   x: absolute group of the item (x records) | item index within the phase << 16 (h records)
//   y: first k-step | end k-step << 8 | segment end << 16 | column slices of the tile << 24
//   z: column unit | segment (this CTA's range within the unit) << 16
__shared__ uint4 s_desc[kMaxStages];

__device__ __forceinline__ uint4 item_desc(const DecPhase& P, const It& it, unsigned b) {
  uint4 d;
  d.x = (unsigned)it_group(it) | ((unsigned)it.i << 16);
  const bool seg_end = it_seg_end(it);
  d.y = (unsigned)it.s0 | ((unsigned)it.s1 << 8) | ((unsigned)seg_end << 16) |
        ((unsigned)it_slices(it) << 24);
  int c0 = 0;
  if (seg_end) dec_nseg(P, it.cu, &c0);
  d.z = (unsigned)it.cu | ((unsigned)((int)b - c0) << 16);
  d.w = 0u;
  return d;
}

// Consumer warp `slice`: the n items of this CTA in phase P, dp2a arithmetic; each finished
// segment's partial sums are stored as tagged words.  Records: the group's (rec_by_item == 0:
// rec + absolute group * frag_bytes, the x records) or the item's (rec + i * frag_bytes, the
// phase's h records).  Returns false on an abort.
template <int MT, int GS>
__device__ bool consume_phase(const DecodeParams& p, const DecPhase& P, int n, int slice, int lane,
                              uint8_t* tiles, uint8_t* auxs, uint64_t* full, uint64_t* empty,
                              int& slot, uint32_t& parity, long long& consumed, const uint8_t* rec,
                              bool rec_by_item, unsigned tag, volatile int* abort,
                              unsigned long long* wait_ns, unsigned long long* first_ns,
                              unsigned long long* last_ns) {
  constexpr int R = GS / 2;  // packed rows per group
  // rows per chunk: 16 at one row (the chunk pair fully unrolled), 8 at two, 4 at four (a rolled
  // loop over chunk pairs, which keeps the rows' accumulators and chunks in registers)
  constexpr int HB = MT == 1 ? (R <= 32 ? R / 2 : 16)
                             : MT == 2 ? (R <= 16 ? R / 2 : 8) : (R <= 8 ? R / 2 : 4);
  constexpr int NCH = R / HB;  // chunks per item (2 to 8)
  constexpr int kPairUnroll = MT == 1 ? NCH / 2 : 1;
  constexpr int tok_stride = dp_tok_stride(GS);
  if (n <= 0) return true;
  const int S = p.stages;
  const int fb = p.frag_bytes;
  auto stage_tile = [&](int sl) { return tiles + (size_t)sl * p.tile_stage_bytes + slice * kTileCols; };
  auto stage_aux = [&](int sl) { return auxs + (size_t)sl * p.aux_stage_bytes; };
  auto item_rec = [&](const uint4& d) {
    return rec + (size_t)(rec_by_item ? (d.x >> 16) : (d.x & 0xffffu)) * fb;
  };
  uint32_t wA[HB], wB[HB];
  uint4 XA[MT][HB / 4], XB[MT][HB / 4];
  DpMeta<MT> Mc, Mn;
  float y[4 * MT];
#pragma unroll
  for (int i = 0; i < 4 * MT; ++i) y[i] = 0.f;
  // stage waits, timed for the trace (consumer warp 0 when tracing)
  auto wait_stage = [&](int sl, uint32_t par) -> bool {
    if (!wait_ns) return dec_wait_full(&full[sl], par, abort, p.err, p.timeout_ns, lane);
    const unsigned long long t0 = global_timer_ns();
    const bool r = dec_wait_full(&full[sl], par, abort, p.err, p.timeout_ns, lane);
    const unsigned long long t1 = global_timer_ns();
    *wait_ns += t1 - t0;
    *last_ns = t1;
    return r;
  };
  // the first chunk (rows, activations) and the metadata of the item described by d in stage sl
  auto load_first = [&](int sl, const uint4& d, DpMeta<MT>& M) {
    const uint8_t* r = item_rec(d);
    const int s0 = (int)(d.y & 0xffu), s1 = (int)((d.y >> 8) & 0xffu);
    dp_load_meta<MT, GS>(stage_aux(sl), r, slice, lane, s0, s1, M);
    dp_load_rows_all<HB>(stage_tile(sl), 0, lane, wA);
    dp_load_x<MT, HB>(r, tok_stride, 0, XA);
  };
  if (!wait_stage(slot, parity)) return false;
  if (wait_ns) *first_ns = global_timer_ns();
  uint4 d = s_desc[slot];
  load_first(slot, d, Mc);
  for (int i = 0;; ++i) {
    const uint8_t* tl = stage_tile(slot);
    const uint8_t* r = item_rec(d);
    const bool seg_end = (d.y >> 16) & 1u;
    const bool more = i + 1 < n;
    const int nslot = slot + 1 == S ? 0 : slot + 1;
    const uint32_t npar = slot + 1 == S ? parity ^ 1u : parity;
    const bool prefetch = !seg_end && more;
    bool next_loaded = false, ok = true;
    uint4 nd = d;
    int aL[MT][4], aH[MT][4];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int q = 0; q < 4; ++q) aL[m][q] = aH[m][q] = 0;
#pragma unroll kPairUnroll
    for (int c = 0; c < NCH; c += 2) {
      dp_load_rows_all<HB>(tl, (c + 1) * HB, lane, wB);
      dp_load_x<MT, HB>(r, tok_stride, (c + 1) * HB, XB);
      bool nready = false;
      if (c + 2 == NCH) {
        // every byte of this stage is loaded (in issue order before the arrival)
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (prefetch) nready = mbar_test_wait(&full[nslot], npar);
      }
      dp_compute<MT, HB>(wA, XA, aL, aH);
      if (c + 2 < NCH) {
        dp_load_rows_all<HB>(tl, (c + 2) * HB, lane, wA);
        dp_load_x<MT, HB>(r, tok_stride, (c + 2) * HB, XA);
      } else if (prefetch) {
        // the next item's first chunk while this item's last chunk computes
        if (!__all_sync(0xffffffffu, nready) && !wait_stage(nslot, npar)) {
          ok = false;
        } else {
          nd = s_desc[nslot];
          load_first(nslot, nd, Mn);
          next_loaded = true;
        }
      }
      dp_compute<MT, HB>(wB, XB, aL, aH);
    }
    dp_epilogue<MT>(Mc, aL, aH, y);
    ++consumed;
    slot = nslot;
    parity = npar;
    if (seg_end) {
      if (slice < (int)(d.y >> 24)) {
        const int cu = (int)(d.z & 0xffffu), seg = (int)(d.z >> 16);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          unsigned long long* dst = dec_part<MT>(P, cu, seg, m) + slice * kTileCols + 4 * lane;
          st_cg_u64x2(dst, tagged(y[4 * m], tag), tagged(y[4 * m + 1], tag));
          st_cg_u64x2(dst + 2, tagged(y[4 * m + 2], tag), tagged(y[4 * m + 3], tag));
        }
      }
#pragma unroll
      for (int q = 0; q < 4 * MT; ++q) y[q] = 0.f;
    }
    if (!ok) return false;
    if (!more) return true;
    if (!next_loaded) {
      if (!wait_stage(slot, parity)) return false;
      nd = s_desc[slot];
      load_first(slot, nd, Mn);
    }
    d = nd;
    Mc = Mn;
  }
}

// Bounded poll step shared by the readers of tagged partials: returns 1 to retry, 0 to give up
// (timeout -> error bit and abort, or another warp aborted).  t0 = 0 starts the clock.
__device__ __forceinline__ bool dec_poll_again(uint64_t& t0, volatile int* abort, unsigned* err,
                                               unsigned long long timeout_ns, int lane,
                                               unsigned bit = kErrDecPoll) {
  const uint64_t now = global_timer_ns();
  if (t0 == 0) t0 = now;
  int st = 0;
  if (lane == 0) {
    if (*abort) st = 1;
    else if (now - t0 > timeout_ns) {
      atomicOr(err, bit);
      *abort = 1;
      st = 1;
    }
  }
  if (__shfl_sync(0xffffffffu, st, 0)) return false;
  __nanosleep(64);
  return true;
}

// One reduction task of the output phases (phases [q0, q1): the B phases, or qmatmul's one
// phase): 8 output columns, 4 lanes per column; lane (c, j) sums the segments j, j + 4, j + 8,
// ... of column c phase by phase in order, then the four lanes combine their sums in a fixed
// tree, so the result's bits do not depend on timing.  Returns false on an abort.
// The fused tensor-parallel exchange of one output word (row m, column col) held by the four
// lanes of a column: lane j stores it to ranks j, j + 4; then every lane reads the tp_n ranks'
// words of the column from this rank's area, retrying until all carry the tag, and sums them
// in rank order.  Returns false on an abort.
__device__ bool tp_exchange(const DecodeParams& p, int m, int col, int j, int lane, unsigned ttag,
                            volatile int* abort, float& acc) {
  const size_t off = (size_t)m * p.ldo + col;
  const size_t par = ttag & 1u;
  const unsigned long long w = tagged(acc, ttag);
  for (int q = j; q < p.tp_n; q += 4)
    st_sys_u64(p.tp_recv[q] + (par * p.tp_n + p.tp_rank) * p.tp_words + off, w);
  const unsigned long long* own = p.tp_recv[p.tp_rank] + par * p.tp_n * p.tp_words + off;
  uint64_t t0 = 0;
  for (;;) {
    unsigned long long v[kDecMaxRanks];
    bool ok = true;
#pragma unroll
    for (int q = 0; q < kDecMaxRanks; ++q) {
      v[q] = q < p.tp_n ? ld_sys_u64(own + (size_t)q * p.tp_words) : ((unsigned long long)ttag << 32);
      ok = ok && (unsigned)(v[q] >> 32) == ttag;
    }
    if (__all_sync(0xffffffffu, ok)) {
      float s = 0.f;
#pragma unroll
      for (int q = 0; q < kDecMaxRanks; ++q)
        if (q < p.tp_n) s += __uint_as_float((unsigned)v[q]);
      acc = s;
      return true;
    }
    if (!dec_poll_again(t0, abort, p.err, p.timeout_ns, lane, kErrDecPeer)) return false;
  }
}

template <int MT>
__device__ bool reduce_task(const DecodeParams& p, int q0, int q1, int task, unsigned tag,
                            unsigned ttag, int lane, volatile int* abort, const float* res_stash) {
  constexpr int B = kDecReduceBatch / MT;  // segments per lane per batch
  const int col = task * 8 + (lane >> 2), j = lane & 3;
  const int cu = col / kWideCols, cl = col % kWideCols;  // output phases cover every tile
#pragma unroll 1
  for (int m = 0; m < MT; ++m) {
    float acc = 0.f;
#pragma unroll 1
    for (int q = q0; q < q1; ++q) {
    const DecPhase& L = p.ph[q];
    const int ns = dec_nseg(L, cu, nullptr);
    for (int base = 0; base < ns; base += 4 * B) {
      uint64_t t0 = 0;
      for (;;) {
        unsigned long long v[B];
#pragma unroll
        for (int i = 0; i < B; ++i) {
          const int s = base + j + 4 * i;
          v[i] = s < ns ? ld_cg_u64(dec_part<MT>(L, cu, s, m) + cl) : ((unsigned long long)tag << 32);
        }
        bool ok = true;
#pragma unroll
        for (int i = 0; i < B; ++i) ok = ok && (unsigned)(v[i] >> 32) == tag;
        if (__all_sync(0xffffffffu, ok)) {
#pragma unroll
          for (int i = 0; i < B; ++i) acc += __uint_as_float((unsigned)v[i]);
          break;
        }
        if (!dec_poll_again(t0, abort, p.err, p.timeout_ns, lane)) return false;
      }
    }
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    // this rank's partial y, summed over the group's ranks (m < p.m is warp-uniform)
    if (p.tp_n > 1 && m < p.m && !tp_exchange(p, m, col, j, lane, ttag, abort, acc)) return false;
    if (j == 0 && m < p.m) {
      if (p.residual)
        acc = (res_stash ? res_stash[m * 8 + (lane >> 2)] : p.residual[(size_t)m * p.ldr + col]) + acc;
      p.out[(size_t)m * p.ldo + col] = acc;
    }
  }
  return true;
}

// The record of one item of B phase na + j (absolute h group `grp`), built by one warp from the
// gate/up partials of A phase j:
// h = silu(sum of the gate segments) * (sum of the up segments) over the group's GS columns,
// quantised into the dp2a record at `rec`; write_h: also store h to h_out.  Lanes: li = lane & 15
// owns columns 4 li .. 4 li + 3 of the group; for GS <= 64 lanes 0-15 sum the gate segments and
// lanes 16-31 the up segments at the same time, for GS = 128 every lane sums both.  Segments are
// loaded 8 / MT at a time, all of a batch in flight, and summed in segment order.
template <int MT, int GS>
__device__ bool build_h_record(const DecodeParams& p, int j, int grp, bool write_h, uint8_t* rec,
                               unsigned tag, int lane, volatile int* abort, int part = 0,
                               int nparts = 1, float* xbuf = nullptr, int bar = 0) {
  constexpr int kSB = MT >= 4 ? 1 : 8 / MT;  // segments in flight per batch
  constexpr bool kSplit = GS / 4 <= 16;  // a half warp per matrix
  constexpr int kMats = kSplit ? 1 : 2;  // matrices summed per lane
  const DecPhase& A = p.ph[j];
  const int c0 = grp * GS;  // first h column of the group (absolute)
  // the A phase's tile (phase-local) and column within it
  const int ta = c0 / kWideCols - A.wt0, cl = c0 % kWideCols;
  const int li = kSplit ? (lane & 15) : lane;
  const bool owner = li < GS / 4;
  bool failed = false;
  float acc[kMats][MT][4];
#pragma unroll
  for (int q = 0; q < kMats; ++q)
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[q][m][0] = acc[q][m][1] = acc[q][m][2] = acc[q][m][3] = 0.f;
#pragma unroll
  for (int q = 0; q < kMats; ++q) {
    const int mat = kSplit ? (lane >> 4) : q;
    const int cu = ta * 2 + mat;
    const int nst = dec_nseg(A, cu, nullptr);
    // this warp's share of the segments (all of them, or a contiguous part)
    const int sa = nst * part / nparts, ns = nst * (part + 1) / nparts;
    // warp-uniform batch bound: the larger of the two matrices' segment ends
    const int nsw = kSplit ? max(ns, __shfl_xor_sync(0xffffffffu, ns, 16)) : ns;
    const int saw = kSplit ? min(sa, __shfl_xor_sync(0xffffffffu, sa, 16)) : sa;
    for (int base = saw; base < nsw && !failed; base += kSB) {
      uint64_t t0 = 0;
      for (;;) {
        ulonglong2 va[kSB][MT], vb[kSB][MT];
#pragma unroll
        for (int i = 0; i < kSB; ++i)
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            if (owner && base + i >= sa && base + i < ns) {
              const unsigned long long* src = dec_part<MT>(A, cu, base + i, m) + cl + 4 * li;
              va[i][m] = ld_cg_u64x2(src);
              vb[i][m] = ld_cg_u64x2(src + 2);
            } else {
              const unsigned long long t = (unsigned long long)tag << 32;
              va[i][m] = vb[i][m] = make_ulonglong2(t, t);
            }
          }
        bool ok = true;
#pragma unroll
        for (int i = 0; i < kSB; ++i)
#pragma unroll
          for (int m = 0; m < MT; ++m)
            ok = ok && (unsigned)(va[i][m].x >> 32) == tag && (unsigned)(va[i][m].y >> 32) == tag &&
                 (unsigned)(vb[i][m].x >> 32) == tag && (unsigned)(vb[i][m].y >> 32) == tag;
        if (__all_sync(0xffffffffu, ok)) {
#pragma unroll
          for (int i = 0; i < kSB; ++i)
#pragma unroll
            for (int m = 0; m < MT; ++m) {
              acc[q][m][0] += __uint_as_float((unsigned)va[i][m].x);
              acc[q][m][1] += __uint_as_float((unsigned)va[i][m].y);
              acc[q][m][2] += __uint_as_float((unsigned)vb[i][m].x);
              acc[q][m][3] += __uint_as_float((unsigned)vb[i][m].y);
            }
          break;
        }
        if (!dec_poll_again(t0, abort, p.err, p.timeout_ns, lane)) {
          failed = true;  // a part still meets its partners at the barrier below
          break;
        }
      }
    }
  }
  if (nparts > 1) {
    // the parts' sums meet in shared memory (the x records' area, free after the A phases) and
    // the first part's warp adds them in part order
    float* mine = xbuf + (size_t)part * (kMats * MT * 4 * 32);
#pragma unroll
    for (int q = 0; q < kMats; ++q)
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int i = 0; i < 4; ++i) mine[((q * MT + m) * 4 + i) * 32 + lane] = acc[q][m][i];
    named_barrier(bar, nparts * 32);
    if (failed || *abort) return false;
    if (part != 0) return true;
#pragma unroll
    for (int q = 0; q < kMats; ++q)
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float s = 0.f;
          for (int r = 0; r < nparts; ++r)
            s += xbuf[(size_t)r * (kMats * MT * 4 * 32) + ((q * MT + m) * 4 + i) * 32 + lane];
          acc[q][m][i] = s;
        }
  } else if (failed) {
    return false;
  }
  const bool holder = lane < GS / 4;  // lanes 0 .. GS/4 - 1 hold the group's h
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    float h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float g = acc[0][m][i];
      // GS <= 64: the up sums live in lanes 16-31
      const float u = kSplit ? __shfl_down_sync(0xffffffffu, acc[0][m][i], 16) : acc[kMats - 1][m][i];
      h[i] = (holder && m < p.m) ? g / (1.0f + expf(-g)) * u : 0.f;
    }
    build_records_dp<MT>(h, m, GS, rec, p.frag_bytes, lane, 0);
    if (write_h && holder && m < p.m)
      *reinterpret_cast<float4*>(p.h_out + (size_t)m * p.ldh + c0 + 4 * lane) =
          make_float4(h[0], h[1], h[2], h[3]);
  }
  return true;
}

// x in pinned host memory: every CTA reads only its share of x over the host link and publishes
// it as tagged words (x_dev, device memory); then the CTA's consumer threads gather the whole of x
// from there (L2), eight words in flight per thread, retrying until every word carries this
// launch's tag, into the prologue area.  One read of x over the link per launch, not one per CTA.
template <int MT>
__device__ bool gather_host_x(const DecodeParams& p, uint8_t* tiles, unsigned b, unsigned tag,
                              volatile int* abort) {
  constexpr int kT = kNC * 32, kB = 8;
  const int n = p.m * p.ph[0].K;  // floats
  const int i0 = (int)((long long)n * b / gridDim.x), i1 = (int)((long long)n * (b + 1) / gridDim.x);
  for (int i = i0 + (int)threadIdx.x; i < i1; i += kT) {
    const int m = i / p.ph[0].K, c = i - m * p.ph[0].K;
    p.x_dev[i] = tagged(p.x[(size_t)m * p.ldx + c], tag);
  }
  float* xs = reinterpret_cast<float*>(tiles);
  for (int base = (int)threadIdx.x; base < n; base += kT * kB) {
    uint64_t t0 = 0;
    for (;;) {
      unsigned long long v[kB];
#pragma unroll
      for (int j = 0; j < kB; ++j)
        v[j] = base + j * kT < n ? ld_cg_u64(p.x_dev + base + j * kT) : ((unsigned long long)tag << 32);
      bool ok = true;
#pragma unroll
      for (int j = 0; j < kB; ++j) ok = ok && (unsigned)(v[j] >> 32) == tag;
      if (ok) {
#pragma unroll
        for (int j = 0; j < kB; ++j)
          if (base + j * kT < n) xs[base + j * kT] = __uint_as_float((unsigned)v[j]);
        break;
      }
      const uint64_t now = global_timer_ns();
      if (t0 == 0) t0 = now;
      if (*abort) return false;
      if (now - t0 > p.timeout_ns) {
        atomicOr(p.err, kErrDecPoll);
        return false;
      }
      __nanosleep(32);
    }
  }
  return true;
}

template <int MT, int GS>
__global__ void __launch_bounds__(kDecThreads, 1)
    int4_decode_kernel(const __grid_constant__ TmapPack maps, const __grid_constant__ DecodeParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ float s_red[MT * kNC];
  __shared__ float s_rms[MT];
  __shared__ volatile long long s_armed;  // items (prologue stages included) armed by the producer
  __shared__ volatile int s_abort;
  __shared__ volatile int s_never;
  __shared__ unsigned s_tag;
  __shared__ unsigned s_ttag;
  __shared__ float s_res[kDecMaxTasksPerCta * 8 * MT];  // residual of this CTA's tasks (host x)
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.stages;
  uint8_t* tiles = smem;
  uint8_t* auxs = smem + (size_t)S * p.tile_stage_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(auxs + (size_t)S * p.aux_stage_bytes);
  uint64_t* empty = full + S;
  uint8_t* rec0 = reinterpret_cast<uint8_t*>(empty + S);  // 16-byte aligned (S barriers each)
  uint8_t* recb = rec0 + (size_t)p.ph[0].groups * p.frag_bytes;
  const unsigned b = blockIdx.x;
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kNC);
    }
    fence_mbar_init();
    s_armed = p.pro_stages;
    s_abort = 0;
    s_never = 0;
  }
  __syncthreads();
  if (warp == kProducerWarp && lane == 0) {
    // the first ring's worth of weight items into L2 while a preceding launch may still run
    It it;
    it_start(it, p, b);
    for (int i = 0; i < S && it.ph < p.nph; ++i) {
      prefetch_item(maps, p.ph[it.ph], it);
      it_next(it, p, b);
    }
  }
  if (threadIdx.x == 0) {
    // the next launch of the stream may be scheduled now; this one reads nothing a preceding
    // kernel writes before that kernel has completed
    griddep_launch_dependents();
    if (p.norm_w) bulk_prefetch_l2(p.norm_w, (uint32_t)p.ph[0].K * 4u);  // a read-only input
    griddep_wait();
    // the prologue copies go out first (x rows, then the norm weight, contiguous over the first
    // pro_stages stages' tiles): everything the consumers do first waits for them
    const uint32_t xrow = (uint32_t)p.ph[0].K * 4u;
    const uint32_t total = (p.x_host ? 0u : xrow * (uint32_t)p.m) + (p.norm_w ? xrow : 0u);
    const uint64_t pol = l2_evict_first();
    if (total) mbar_arrive_expect_tx(&full[0], total);
    else mbar_arrive(&full[0]);
    for (int m = 0; m < (p.x_host ? 0 : p.m); ++m)
        bulk_load(tiles + (size_t)m * xrow, p.x + (size_t)m * p.ldx, xrow, &full[0], pol);
    if (p.norm_w) bulk_load(tiles + (size_t)p.m * xrow, p.norm_w, xrow, &full[0], pol);
    for (int i = 1; i < p.pro_stages; ++i) mbar_arrive(&full[i]);
    s_tag = p.epoch[b] + 1u;
    s_ttag = p.tp_n > 1 ? p.tp_epoch[b] + 1u : 0u;
    dec_trace(p, 0);
  }
  __syncthreads();
  const unsigned tag = s_tag;
  int slot = 0;
  uint32_t parity = 0;
  long long consumed = 0;

  if (warp == kProducerWarp) {
    // ------------------------------- producer ---------------------------------------------
    if (lane == 0) {
      const uint64_t pol = l2_evict_first();
      const int P0 = p.pro_stages;  // stages the prologue copies (issued by thread 0) occupy
      long long G = P0;
      int ws = P0 % S;
      uint32_t wround = (uint32_t)(P0 / S);
      It it;
      it_start(it, p, b);
      dec_trace(p, 7);
      while (it.ph < p.nph) {
        if (wround > 0) {
          // bounded wait for the consumers to free the slot
          bool ok = mbar_try_wait(&empty[ws], (wround - 1) & 1);
          if (!ok) {
            const uint64_t t0 = global_timer_ns();
            // suspended in the wait (time hint) rather than spinning: the producer shares an SM
            // sub-partition with two consumer warps
            while (!(ok = mbar_try_wait_hint(&empty[ws], (wround - 1) & 1, 2000))) {
              if (s_abort) break;
              if (global_timer_ns() - t0 > p.timeout_ns) {
                atomicOr(p.err, kErrTmaWait);
                s_abort = 1;
                break;
              }
            }
          }
          if (!ok) break;
        }
        if (s_abort) break;
        const DecPhase& P = p.ph[it.ph];
        s_desc[ws] = item_desc(P, it, b);
        issue_item(maps, P, it, tiles + (size_t)ws * p.tile_stage_bytes,
                   auxs + (size_t)ws * p.aux_stage_bytes, &full[ws], pol);
        s_armed = ++G;
        it_next(it, p, b);
        if (++ws == S) {
          ws = 0;
          ++wround;
        }
      }
      s_armed = G;
      dec_trace(p, 8);
    }
    __syncwarp();
  } else {
    // ------------------------------- consumers --------------------------------------------
    const int slice = warp;
    volatile int* abort = &s_abort;
    if (p.x_host) {
      if (!gather_host_x<MT>(p, tiles, b, tag, abort)) *abort = 1;
      if (threadIdx.x == 0) dec_trace(p, 15);
    }
    // prologue: wait for x (and the norm weight), then the records of every group of x; the
    // consumer warps take the same branch (an abort is published before the barrier)
    if (!dec_wait_full(&full[0], 0, abort, p.err, p.timeout_ns, lane) && lane == 0) *abort = 1;
    named_barrier(1, kNC * 32);
    bool ok = *abort == 0;
    const bool pro_landed = ok;
    if (ok && p.x_host && p.residual) {
      // keep the residual of this CTA's reduction tasks (the prologue area is reused)
      for (int i = threadIdx.x; i < kDecMaxTasksPerCta * 8 * MT; i += kNC * 32) {
        const int k = i / (8 * MT), m = (i / 8) % MT, c = i % 8;
        const int t = (int)b + (int)gridDim.x * k;
        if (t < p.red_tasks && m < p.m)
          s_res[i] = reinterpret_cast<const float*>(tiles)[(size_t)m * p.ph[0].K + t * 8 + c];
      }
    }
    if (ok) {
      const float* xs = reinterpret_cast<const float*>(tiles);
      const float* ws = xs + (size_t)p.m * p.ph[0].K;
      const int nchunks = p.ph[0].K / kTileCols;
      float rms[MT];
#pragma unroll
      for (int m = 0; m < MT; ++m) rms[m] = 1.f;
      if (p.norm_w) {
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          float v = 0.f;
          if (m < p.m)
            for (int ch = warp; ch < nchunks; ch += kNC) {
              const float4 a = *reinterpret_cast<const float4*>(xs + (size_t)m * p.ph[0].K + ch * kTileCols + 4 * lane);
              v = fmaf(a.x, a.x, fmaf(a.y, a.y, fmaf(a.z, a.z, fmaf(a.w, a.w, v))));
            }
          for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
          if (lane == 0) s_red[m * kNC + warp] = v;
        }
        named_barrier(1, kNC * 32);
        if (threadIdx.x < MT) {
          float tot = 0.f;
          for (int i = 0; i < kNC; ++i) tot += s_red[threadIdx.x * kNC + i];
          s_rms[threadIdx.x] = rsqrtf(tot / (float)p.ph[0].K + p.eps);
        }
        named_barrier(1, kNC * 32);
#pragma unroll
        for (int m = 0; m < MT; ++m) rms[m] = s_rms[m];
      }
      // the records of the groups this CTA's gate/up (or matvec) range touches
      const NeedGroups need = a_range_groups(p, b);
      for (int ch = warp; ch < nchunks; ch += kNC) {
        if (!needs_groups(p, need, b, ch * kTileCols / GS, (ch + 1) * kTileCols / GS)) continue;
        float4 w4 = make_float4(1.f, 1.f, 1.f, 1.f);
        if (p.norm_w) w4 = *reinterpret_cast<const float4*>(ws + ch * kTileCols + 4 * lane);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          float v[4] = {0.f, 0.f, 0.f, 0.f};
          if (m < p.m) {
            const float4 a = *reinterpret_cast<const float4*>(xs + (size_t)m * p.ph[0].K + ch * kTileCols + 4 * lane);
            if (p.norm_w) {
              v[0] = a.x * rms[m] * w4.x;
              v[1] = a.y * rms[m] * w4.y;
              v[2] = a.z * rms[m] * w4.z;
              v[3] = a.w * rms[m] * w4.w;
            } else {
              v[0] = a.x;
              v[1] = a.y;
              v[2] = a.z;
              v[3] = a.w;
            }
          }
          build_records_dp<MT>(v, m, GS, rec0 + (size_t)(ch * kTileCols / GS) * p.frag_bytes,
                               p.frag_bytes, lane, -1);
        }
      }
    }
    // every consumer has read the prologue data and written its records: free the stages
    named_barrier(1, kNC * 32);
    __syncwarp();
    if (lane == 0)
      for (int i = 0; i < p.pro_stages; ++i) mbar_arrive(&empty[i]);
    if (pro_landed) {
      slot = p.pro_stages % S;
      parity = (uint32_t)((p.pro_stages / S) & 1);
      consumed = p.pro_stages;
    }
    if (threadIdx.x == 0) dec_trace(p, 1);
    if (s_abort) ok = false;

    // trace of consumer warp 0: stage waits per phase, item counts, first / last phase-B stage
    const bool tw = p.trace && warp == 0;
    // the A phases (x records), then per B phase its records and its items: one inlined copy of
    // the item loop for each kind (a single copy with the kind chosen at run time measured slower)
    unsigned long long wt = 0, ft = 0, lt = 0;
    int nitems = 0;
#pragma unroll 1
    for (int q = 0; q < p.na; ++q) {
      const int n = phase_items(p.ph[q], b);
      nitems += n;
      if (ok)
        ok = consume_phase<MT, GS>(p, p.ph[q], n, slice, lane, tiles, auxs, full, empty, slot,
                                   parity, consumed, rec0, false, tag, abort,
                                   tw ? &wt : nullptr, &ft, &lt);
    }
    if (threadIdx.x == 0) {
      dec_trace(p, 2);
      if (p.trace) {
        p.trace[(size_t)blockIdx.x * kTraceEvents + 10] = wt;
        p.trace[(size_t)blockIdx.x * kTraceEvents + 12] = (unsigned long long)nitems;
      }
    }
    wt = 0;
    nitems = 0;
    const int nb = p.nph - p.na;
#pragma unroll 1
    for (int j = 0; j < nb; ++j) {
      const int q = p.na + j;
      uint8_t* recq = recb + (size_t)j * p.recb_items * p.frag_bytes;
      // the records of this CTA's items of B phase q: warp w builds items w, w + 8, ...
      // With fewer items than warps (small phases: tensor-parallel shards) the warps of an item
      // share its gate/up segments (parts of a contiguous range each, summed in part order in the
      // x records' area, which the A phases no longer need).
      const int nbi = phase_items(p.ph[q], b);
      constexpr int kPartFloats = (GS / 4 <= 16 ? 1 : 2) * MT * 4 * 32;
      int parts = nbi > 0 && nbi < kNC ? kNC / nbi : 1;
      if ((size_t)nbi * parts * kPartFloats * sizeof(float) > (size_t)p.ph[0].groups * p.frag_bytes)
        parts = 1;
      if (ok && nbi > 0) {
        It bi;
        bi.ph = q;
        it_seek(bi, p, b);
        for (int i = 0; bi.ph == q && ok; ++i) {
          if (parts > 1 ? i == warp / parts : i % kNC == warp)
            ok = build_h_record<MT, GS>(
                p, j, it_group(bi), p.h_out && it_tile(bi) == 0 && bi.s0 == 0,
                recq + (size_t)i * p.frag_bytes, tag, lane, abort, warp % parts, parts,
                reinterpret_cast<float*>(rec0) + (size_t)i * parts * kPartFloats, 2 + i);
          it_next(bi, p, b);
        }
      }
      if (!ok) *abort = 1;
      named_barrier(1, kNC * 32);
      if (*abort) ok = false;
      if (threadIdx.x == 0 && j == 0) dec_trace(p, 3);
      const int n = phase_items(p.ph[q], b);
      nitems += n;
      if (ok)
        ok = consume_phase<MT, GS>(p, p.ph[q], n, slice, lane, tiles, auxs, full, empty, slot,
                                   parity, consumed, recq, true, tag, abort,
                                   tw ? &wt : nullptr, &ft, &lt);
    }
    if (threadIdx.x == 0 && nb > 0) {
      dec_trace(p, 4);
      if (p.trace) {
        unsigned long long* tr = p.trace + (size_t)blockIdx.x * kTraceEvents;
        tr[9] = ft;
        tr[11] = wt;
        tr[13] = (unsigned long long)nitems;
        tr[14] = lt;
      }
    }
    if (!ok) *abort = 1;
    // the y reduction tasks of this CTA (8 columns each) over the output phases
    const int q0 = nb > 0 ? p.na : 0, q1 = p.nph;
    for (int k = warp; ok; k += kNC) {
      const int t = (int)b + (int)gridDim.x * k;
      if (t >= p.red_tasks) break;
      ok = reduce_task<MT>(p, q0, q1, t, tag, s_ttag, lane, abort,
                           (p.x_host && p.residual) ? s_res + k * 8 * MT : nullptr);
    }
    if (threadIdx.x == 0) dec_trace(p, 5);
  }
  __syncthreads();
  if (warp < kNC) {
    // after an abort: wait for the stages armed but not consumed, so no copy is in flight when
    // the CTA exits
    const long long armed = s_armed;
    for (long long G = consumed; G < armed; ++G) {
      dec_wait_full(&full[slot], parity, &s_never, p.err, p.timeout_ns, lane);
      if (++slot == S) {
        slot = 0;
        parity ^= 1u;
      }
    }
  }
  if (threadIdx.x == 0) {
    for (unsigned j = b; j < (unsigned)kDecEpochSlots; j += gridDim.x) p.epoch[j] = tag;
    if (p.tp_n > 1)
      for (unsigned j = b; j < (unsigned)kDecEpochSlots; j += gridDim.x) p.tp_epoch[j] = s_ttag;
    // a CTA that gave up tells the host directly (its bits are in p.err as well)
    if (p.err_host && s_abort) *reinterpret_cast<volatile unsigned*>(p.err_host) = 1u;
    dec_trace(p, 6);
  }
}

template <int MT, int GS>
cudaError_t dec_launch_mt(const TmapPack& maps, const DecodeParams& p, int grid, size_t smem,
                          cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kDecThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (p.pdl) {
    // every CTA must become resident (they wait on one another): one CTA per SM and grid <= SMs
    // give that on a device this launch does not share; the bounded waits end in an error
    // otherwise
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
  } else {
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, int4_decode_kernel<MT, GS>, maps, p);
}

template <int MT, int GS>
cudaError_t dec_prepare_mt(size_t smem, int* blocks) {
  auto kern = int4_decode_kernel<MT, GS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, kern, kDecThreads, smem);
}

template <int MT>
cudaError_t dec_occupancy_gs(int gs, size_t smem, int* blocks) {
  switch (gs) {
    case 16: return dec_prepare_mt<MT, 16>(smem, blocks);
    case 32: return dec_prepare_mt<MT, 32>(smem, blocks);
    case 64: return dec_prepare_mt<MT, 64>(smem, blocks);
    case 128: return dec_prepare_mt<MT, 128>(smem, blocks);
    default: return cudaErrorInvalidValue;
  }
}

template <int MT>
cudaError_t dec_launch_gs(int gs, const TmapPack& maps, const DecodeParams& p, int grid,
                          size_t smem, cudaStream_t stream) {
  switch (gs) {
    case 16: return dec_launch_mt<MT, 16>(maps, p, grid, smem, stream);
    case 32: return dec_launch_mt<MT, 32>(maps, p, grid, smem, stream);
    case 64: return dec_launch_mt<MT, 64>(maps, p, grid, smem, stream);
    case 128: return dec_launch_mt<MT, 128>(maps, p, grid, smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

size_t decode_smem_bytes(int stages, int tile_stage_bytes, int aux_stage_bytes, int rec0_bytes,
                         int recb_bytes) {
  return 1024 + (size_t)stages * ((size_t)tile_stage_bytes + aux_stage_bytes + 16) +
         (size_t)rec0_bytes + (size_t)recb_bytes;
}

// The attribute and occupancy query are redone only when an instantiation is launched with
// another shared-memory size than its last one on a device.
cudaError_t decode_occupancy(int mt, int gs, size_t smem, int* blocks) {
  constexpr int kMaxDevices = 64;
  struct Last {
    size_t smem;
    int blocks;
    unsigned gen;
  };
  static Last last[kMaxDevices][3][4] = {};
  const int mi = mt == 1 ? 0 : mt == 2 ? 1 : mt == 4 ? 2 : -1;
  const int gi = gs == 16 ? 0 : gs == 32 ? 1 : gs == 64 ? 2 : gs == 128 ? 3 : -1;
  if (mi < 0 || gi < 0) return cudaErrorInvalidValue;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  Last* L = dev >= 0 && dev < kMaxDevices ? &last[dev][mi][gi] : nullptr;
  const unsigned gen = attr_generation(dev);
  if (L && L->blocks > 0 && L->smem == smem && L->gen == gen) {
    *blocks = L->blocks;
    return cudaSuccess;
  }
  e = mt == 1 ? dec_occupancy_gs<1>(gs, smem, blocks)
      : mt == 2 ? dec_occupancy_gs<2>(gs, smem, blocks) : dec_occupancy_gs<4>(gs, smem, blocks);
  if (L) *L = (e == cudaSuccess) ? Last{smem, *blocks, gen} : Last{0, 0, 0};
  return e;
}

cudaError_t decode_launch(int mt, int gs, const TmapPack& maps, const DecodeParams& p, int grid,
                          size_t smem, cudaStream_t stream) {
  switch (mt) {
    case 1: return dec_launch_gs<1>(gs, maps, p, grid, smem, stream);
    case 2: return dec_launch_gs<2>(gs, maps, p, grid, smem, stream);
    case 4: return dec_launch_gs<4>(gs, maps, p, grid, smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace tk
