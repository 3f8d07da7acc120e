// tk_decode.h -- parameters of the batch 1-2 decode kernel (tk_decode.cu).
//
// One persistent launch (one CTA per SM, all resident) computes either
//   qmatmul_int4 (src/kernels/shaders.zig:442-501):  phase A = y[m][N] = x . W
// or the INT4 Llama FFN (src/bench.zig:266-341 + the down projection and residual of
// src/model/llama.zig:220-231):
//   prologue rmsnorm(x) -> phase A gate/up -> h = silu(gate) * up -> phase B down (+ x).
// Work is split stream-K over k-steps (16 k values) of 1024-column tiles, as in the streaming
// engine (tk_engine.h), but the split-K exchange is counter-free: every segment of partial sums
// is stored as (value, tag) pairs in one 64-bit word, the tag being the launch's epoch, so a
// reader knows a value is this launch's by looking at the value itself -- no counters, fences
// or flags between the producer of a partial and its reader, and nothing to reset between
// launches.  The phase-B records (h) are built by the consumer warps of every CTA straight from
// the gate/up partials; the output y is reduced by 32-column tasks spread over all CTAs.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "tk_engine.h"

namespace tk {

constexpr int kDecConsumers = 8;                      // consumer warps (one per 128-col slice)
constexpr int kDecThreads = (kDecConsumers + 1) * 32;  // + the producer warp
constexpr int kDecEpochSlots = 1024;  // launch counters: CTA b reads slot b, writes b + k*grid
constexpr int kDecMaxItemsB = 64;     // phase-B items of one CTA whose records live in smem
constexpr int kDecReduceBatch = 16;   // partials in flight per lane of a reduction task (/ rows)
constexpr int kDecMaxTasksPerCta = 16;  // reduction tasks per CTA whose residual smem holds

// error bits of the device error word (shared with the engine's)
constexpr unsigned kErrDecPoll = 16u;  // a tagged partial never arrived
constexpr unsigned kErrDecPeer = 32u;  // a peer rank's tagged output never arrived
constexpr int kDecMaxRanks = 8;        // ranks of a fused tensor-parallel exchange

struct DecPhase {
  int K, N;           // contraction size and output columns of the whole matrix
  int nmat;           // 1, or 2 (gate and up at the same columns)
  int wt0, tiles;     // the phase's 1024-column tiles [wt0, wt0 + tiles) of N
  int g0, groups;     // the phase's groups [g0, g0 + groups) of K
  int spg;            // k-steps (16 k) per group
  unsigned units;     // tiles * nmat * groups * spg
  unsigned ctas;      // min(grid, units): CTAs that hold a range of this phase
  int map_base;       // tensor maps of matrix i: map[map_base + 2i] (group box), +1 (k-step box)
  const uint16_t* scales[2];
  const uint8_t* zeros[2];
  unsigned long long* part;  // tagged partial sums [tiles * nmat][maxseg][MT][1024]
  int maxseg;
};

// Phases of a launch: A phases (x records: qmatmul_int4's one phase, or the FFN's gate/up over
// consecutive column ranges), then B phases (the FFN's down projection over the h groups of the
// A phase with the same index, records built from that A phase's partial sums).  Splitting the
// FFN in two lets B0's records be built long after A0 has finished everywhere and B0's work hide
// the wait for A1's last partial sums.
constexpr int kDecMaxPhases = 4;

struct DecodeParams {
  int m;     // live rows (<= MT)
  int nph;   // phases
  int na;    // A phases (ph[0 .. na)); B phases ph[na .. nph), nph - na == na or 0
  DecPhase ph[kDecMaxPhases];
  const float* x;  // [m][ldx], K = ph[0].K
  int ldx;
  const float* norm_w;  // non-null: rmsnorm(x) with eps first (the FFN)
  float eps;
  float* out;  // y [m][ldo] of the last phase
  int ldo;
  const float* residual;  // optional, added to y
  int ldr;
  int x_host;                 // x (and the residual, which is x) and out are pinned host memory
  unsigned long long* x_dev;  // x_host: [m * K] tagged words through which the CTAs share x
  unsigned* err_host;         // optional pinned host word set nonzero by a CTA that failed
  float* h_out;  // optional f32 h [m][ldh]
  int ldh;
  // shared memory: S stages of (tile | aux), then the records
  int stages, tile_stage_bytes, aux_stage_bytes;
  int pro_stages;  // the first stages hold the prologue copies: x rows, then the norm weight
  int frag_bytes;  // record bytes per group
  int recb_items;  // records per CTA per B phase (the largest item count of a CTA's range)
  int red_tasks;   // 8-column reduction tasks over the last phases' outputs
  unsigned* epoch;  // [kDecEpochSlots]
  unsigned* err;
  unsigned long long timeout_ns;
  unsigned long long* trace;  // optional [grid][kTraceEvents] global-timer stamps
  // 1: launched with programmatic stream serialization (the launch may start while the
  // preceding kernel of the stream finishes; it reads nothing that kernel may write before
  // griddepcontrol.wait, only L2-prefetches its first weight items), not as a cooperative launch;
  // 0: a cooperative launch
  int pdl;
  // Tensor-parallel exchange fused into the reduction (tp_n > 1, the FFN of one rank's shard):
  // each reduction task stores its columns' partial y as tagged words into every rank's area
  // (plain peer stores over NVLink), then sums the tp_n ranks' words of those columns in rank
  // order -- every rank gets the same bits.  The tag is this rank's group launch count + 1
  // (every rank of the group makes the same sequence of these launches); the area has two
  // halves by the tag's parity, so a rank a launch ahead never overwrites words a peer has yet
  // to read.
  int tp_n, tp_rank;
  unsigned long long* tp_recv[kDecMaxRanks];  // rank r's area, mapped here: [2][tp_n][tp_words]
  int tp_words;                               // words per (parity, source rank) >= m * ldo
  unsigned* tp_epoch;                         // this rank's group launch counters [kDecEpochSlots]
};

// Dynamic shared memory of a launch with these sizes (1024-byte alignment slack included).
size_t decode_smem_bytes(int stages, int tile_stage_bytes, int aux_stage_bytes, int rec0_bytes,
                         int recb_bytes);
cudaError_t decode_occupancy(int mt, int gs, size_t smem, int* blocks);
cudaError_t decode_launch(int mt, int gs, const TmapPack& maps, const DecodeParams& p, int grid,
                          size_t smem, cudaStream_t stream);

}  // namespace tk
