// tk_engine.h -- parameters shared by the host launcher and the persistent INT4 engine.
//
// The engine runs one or two "phases" of INT4 fused-dequant GEMV in one persistent,
// cooperative launch (one CTA per SM):
//   qmatmul_int4 (src/kernels/shaders.zig:442-501):   prologue(x -> fragments) | phase 0
//   INT4 FFN (src/bench.zig:266-341 + down proj):     prologue(rmsnorm(x) -> fragments) |
//                                                     phase 0 gate+up -> silu*up -> h |
//                                                     phase 1 down (+ residual)
// Work unit = one k-step (16 k values = 8 packed rows) of one 128-column tile of one
// matrix; each warp owns a contiguous range of k-steps (stream-K), partial sums of a
// tile are reduced deterministically (in warp order) by the last warp to finish it.
#pragma once
#include <cstdint>
#include <cuda.h>

namespace tk {

constexpr int kTileCols = 128;   // output columns per tile == bytes per packed row slice
constexpr int kStepRows = 8;     // packed rows (k pairs) per k-step
constexpr int kStepBytes = 1024; // one k-step of one tile: 8 rows x 128 B (TMA box)
constexpr int kMaxPhases = 2;
constexpr int kMaxMats = 2;
constexpr int kScaleBytes = kTileCols * 2;  // f16 scales of one tile, one group
constexpr int kZeroBytes = kTileCols / 2;   // packed zero points of one tile, one group

// error bits written to the device error word
constexpr unsigned kErrTmaWait = 1u;
constexpr unsigned kErrGridBarrier = 2u;

// One group's activation record: the B-operand fragments of the m16n8k16 MMA for every
// k-step of the group, followed by per-step metadata:
//   uint2  b[spg][4 (t)][2*MT (token, hi/lo)]
//   float2 meta[spg][MT]  = {sum_k xs_k * 2^-24 over the step, 2^(24 - e) for the group}
// padded to 16 bytes.
__host__ __device__ constexpr int frag_record_bytes(int spg, int mt) {
  return (spg * 72 * mt + 15) & ~15;
}

enum EpilogueKind : int {
  kEpiStore = 0,    // out[tok][col] = sum (+ residual[tok][col])
  kEpiSiluMul = 1,  // h = silu(mat0) * mat1 -> optional h out + next phase's records
};

struct GridBar {
  unsigned count;
  unsigned pad0[31];
  unsigned gen;
  unsigned pad1[31];
};

struct PhaseParams {
  int K, N, gs, nmat;
  int spg;      // k-steps per group = gs / 16
  int groups;   // K / gs
  int tiles;    // N / 128
  long long units;  // tiles * nmat * groups * spg
  int map_base;     // tensor map index of matrix 0 in TmapPack
  const uint16_t* scales[kMaxMats];
  const uint8_t* zeros[kMaxMats];
  const uint8_t* frag_in;  // activation records, one per group of K
  int frag_bytes;
  float* partials;         // [tiles*nmat][maxseg][MT][128]
  unsigned* counters;      // [tiles], zero between launches
  int maxseg;
  int epi;
  float* out;              // kEpiStore: y; kEpiSiluMul: optional h
  int ldo;
  const float* residual;   // kEpiStore: optional
  int ldr;
  uint8_t* frag_out;       // kEpiSiluMul: records for the next phase
  int next_gs;
  int next_frag_bytes;
};

struct EngineParams {
  int m;        // live tokens (rows of x), <= MT of the instantiation
  int nphases;
  PhaseParams ph[kMaxPhases];
  // prologue: x[m][K0] (optionally rmsnorm'ed) -> records frag0 with group size gs0
  const float* x;
  int ldx;
  int K0;
  const float* norm_w;
  float eps;
  int do_norm;
  uint8_t* frag0;
  int gs0;
  int frag0_bytes;
  // shared-memory ring
  int stages;
  int tile_stage_bytes;
  int aux_stage_bytes;
  // sync + errors
  GridBar* bar;
  unsigned* err;
  unsigned long long timeout_ns;
};

struct TmapPack {
  CUtensorMap map[3];
};

}  // namespace tk
