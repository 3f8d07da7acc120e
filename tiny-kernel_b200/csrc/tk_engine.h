// tk_engine.h -- parameters shared by the host launcher and the persistent INT4 engine.
//
// The engine runs a list of "phases" of INT4 fused-dequant GEMV in one persistent,
// cooperative launch (one CTA per SM):
//   qmatmul_int4 (src/kernels/shaders.zig:442-501):   prologue(x -> records) | phase 0
//   INT4 FFN (src/bench.zig:266-341 + down proj):     prologue(rmsnorm(x) -> records) |
//                                                     gate+up over tile range 0 -> silu*up -> h |
//                                                     ... | gate+up over tile range P-1 |
//                                                     down over the h groups of range 0 | ... |
//                                                     down over the h groups of range P-1
// A phase covers the wide tiles [wt0, wt1) of N and the groups [g0, g1) of K of its matrices.
// Work unit = one k-step (16 k values = 8 packed rows) of a 1024-column wide tile of one
// matrix; each CTA owns a contiguous range of every phase's units (stream-K) and its 8
// consumer warps take one 128-column slice each.  Partial sums of a 128-column sub-tile are
// reduced deterministically (in phase and CTA order); the phases [red_first, red_first +
// red_count) add into the same outputs.  An output (y) sub-tile is reduced by the last warp to
// finish it.  The gate/up partial sums are not reduced by their producers: every CTA that
// consumes an h sub-tile waits for its segment counter to be complete and reduces it itself
// (silu(gate) * up, then the records of its own items).  There is no grid-wide barrier.
// Splitting the gate/up tiles into P ranges lets the down projection of range j run while
// later ranges are still being produced.
#pragma once
#include <cstdint>
#include <cuda.h>

namespace tk {

constexpr int kTileCols = 128;   // output columns per slice == bytes per packed row slice
constexpr int kSlices = 8;       // slices per wide tile == consumer warps per CTA
constexpr int kWideCols = kTileCols * kSlices;  // 1024 columns per wide tile
constexpr int kStepRows = 8;     // packed rows (k pairs) per k-step
// A wide tile's packed row is read as one 1040-byte TMA box row (130 u64): 1024 payload
// bytes plus 16 bytes of the next tile, so consecutive rows land 16 bytes apart modulo
// 128 in shared memory and the fragment loads are bank-conflict free.
constexpr int kRowBytes = 1040;
constexpr int kRowElems = kRowBytes / 8;  // u64 elements per box row
constexpr int kMaxPhases = 8;
constexpr int kMaxStages = 16;  // ring stages per CTA (the deepest that fits is taken)
constexpr int kMaxMats = 2;
constexpr int kScaleBytes = kTileCols * 2;  // f16 scales of one slice, one group
constexpr int kZeroBytes = kTileCols / 2;   // packed zero points of one slice, one group

// Device-side event trace (per CTA, global-timer ns), written when EngineParams.trace
// is set: start, prologue done, (unused), phase-0 items done, (unused), phase-1 items
// done, end, producer first issue, producer last issue, first stage landed.
constexpr int kTraceEvents = 16;

// error bits written to the device error word
constexpr unsigned kErrTmaWait = 1u;
constexpr unsigned kErrFlagWait = 2u;

// One group's activation record for the int8 tensor-core path (MT = 4):
//   uint4 b[kbg][4 (t)][2*MT (token, hi/lo)]   kbg = max(1, gs / 64) blocks of 32 k pairs;
//         .x/.y = high-nibble B (odd k) for kappa halves 0/1, .z/.w = low-nibble B (even k),
//         each an int8 hi or lo part, 4 k pairs per word
//   int2  sums[spg][MT]   sums of the int8 hi and lo parts over each 16-k step (zero points)
//   float scale[MT]       2^-e of the group's int8 split
// padded to 16 bytes.
__host__ __device__ constexpr int frag_record_bytes(int spg, int mt) {
  return (128 * mt * (spg >= 4 ? spg / 4 : 1) + 8 * mt * spg + 4 * mt + 15) & ~15;
}

// One group's activation record for the dp2a path (MT = 1, 2), per token (token stride
// dp_tok_stride(gs)): the group's gs values quantised to int16 with one power-of-two scale
// (max |x| * 2^e in [2^14, 2^15)),
//   uint2 X[gs / 4]   X[j] = {x[4j] | x[4j+2] << 16, x[4j+1] | x[4j+3] << 16}: the even-k and
//                     odd-k halves of packed rows 2j, 2j+1 as dp2a's two 16-bit lanes
//   int   sums[spg]   sum of the quantised values over each 16-k step (zero points)
//   float esc         2^-e
__host__ __device__ constexpr int dp_tok_stride(int gs) { return (2 * gs + gs / 4 + 4 + 15) & ~15; }

// Record bytes per group for MT tokens on the path the engine takes for MT.
__host__ __device__ constexpr int record_bytes(int gs, int mt) {
  return mt <= 2 ? mt * dp_tok_stride(gs) : frag_record_bytes(gs / 16, mt);
}

enum EpilogueKind : int {
  kEpiStore = 0,    // out[tok][col] = sum (+ residual[tok][col]), by the last segment's warp
  kEpiSiluMul = 1,  // partial sums stay in `partials`; a phase with src_count > 0 builds its
                    // records from silu(mat0) * mat1 of them (and writes h to `out` if set)
};

// Launch-to-launch synchronisation state (device memory, zeroed once).
struct SyncState {
  unsigned epoch;  // launches completed
  unsigned pad0[31];
  unsigned done;   // CTAs finished in the current launch
  unsigned pad1[31];
};

struct PhaseParams {
  int K, N, gs, nmat;
  int spg;          // k-steps per group = gs / 16
  int wt0, wt1;     // wide tiles [wt0, wt1) of N
  int g0, g1;       // groups [g0, g1) of K
  int tiles;        // wt1 - wt0; the last tile of N may have fewer than 8 slices
  int groups;       // g1 - g0
  long long units;  // tiles * nmat * groups * spg
  int red_first;    // phases [red_first, red_first + red_count) reduce into the same outputs
  int red_count;
  int map_base;     // tensor maps of matrix i: map[map_base + 2i] (group box), +1 (step box)
  const uint16_t* scales[kMaxMats];
  const uint8_t* zeros[kMaxMats];
  const uint8_t* frag_in;     // prologue records in global memory, one per group of K
  long long frag_cta_stride;  // bytes between CTAs' private copies
  int frag_bytes;             // record bytes per group
  int src_first, src_count;   // src_count > 0: records built from the kEpiSiluMul partial sums
                              // of phases [src_first, src_first + src_count); else the prologue's
  int done_total;             // kEpiSiluMul: sum over its column units of segments * slices
  float* partials;         // [N/1024 * nmat][maxseg][kSlices][MT][128], shared by the reduction
  unsigned* counters;      // [N / 128] per sub-tile, zero between launches, shared likewise
  int maxseg;              // segments per column unit summed over the reduction's phases
  int epi;
  float* out;              // kEpiStore: y; kEpiSiluMul: optional h
  int ldo;
  const float* residual;   // kEpiStore: optional
  int ldr;
};

struct EngineParams {
  int m;        // live tokens (rows of x), <= MT of the instantiation
  int nphases;
  PhaseParams ph[kMaxPhases];
  // prologue: every CTA turns x[m][K0] (optionally rmsnorm'ed) into its own records at
  // frag0 + blockIdx.x * frag0_cta_stride, group size gs0
  const float* x;
  int ldx;
  int K0;
  const float* norm_w;
  float eps;
  int do_norm;
  uint8_t* frag0;
  long long frag0_cta_stride;
  int gs0;
  int frag0_bytes;
  // phase-0 records in shared memory (built by the consumers, read with plain loads) when
  // rec0_smem, else in frag0 (global, one copy per CTA) and copied per stage by TMA
  int rec0_smem;
  // shared-memory ring
  int stages;
  int tile_stage_bytes;
  int aux_stage_bytes;
  // segment counters the last CTA to finish returns to zero (the kEpiSiluMul reductions'),
  // and per kEpiSiluMul phase the (segment, slice) pairs it has completed (inside that range)
  int prefetch_l2;  // 1: at the switch to a phase fed by partial sums (the down projection), the
                    // weight warp prefetches all of its items of that phase into L2
  unsigned* zero_counters;
  int zero_count;
  unsigned* phase_done;  // [kMaxPhases]
  // sync + errors
  unsigned long long* trace;  // optional [gridDim.x][kTraceEvents] globaltimer stamps
  SyncState* sync;
  unsigned* err;
  unsigned long long timeout_ns;
};

struct TmapPack {
  CUtensorMap map[7];  // per matrix: group-box map, step-box map; [6]: one k-step of zero rows
};
constexpr int kZeroMap = 6;

}  // namespace tk
