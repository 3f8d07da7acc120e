// tk_gemm.h -- parameters of the batch >= 5 INT4 GEMM (tcgen05 / tensor memory).
//
// Y[M][N] = X[M][K] . W[K][N] with W in the reference's packed INT4 layout
// (src/kernels/shaders.zig:442-501): the weights are dequantised to f16 ((q - z) * scale, one
// rounding) and multiplied on the 5th-generation tensor cores with f32 accumulators in tensor
// memory.  MMA M = 128 output columns (the dequantised weights, A), MMA N = a tile of NT tokens
// (the f16 activations, B, K-major, 128-byte swizzle).  Token tiles up to 64: A is written into
// tensor memory (int4_gemm_tm_kernel); 128 and 256: A is written into shared memory, MN-major
// with the 128-byte swizzle (int4_gemm_kernel).
// A CTA computes two 128-column tiles (two matrices at the same columns -- gate and up -- or
// 256 adjacent columns of one matrix) for NT tokens over a range of K.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>

namespace tk {

constexpr int kGemmTileCols = 128;  // MMA M: output columns per tile
constexpr int kGemmTiles = 2;       // tiles per CTA
constexpr int kGemmKStep = 64;      // k per pipeline stage (32 packed rows)
constexpr int kGemmDequantWarps = 16;  // warp d: tile d/8, k rows 8(d%8) .. 8(d%8)+7 of a step
constexpr int kGemmThreads = 64 + 32 * kGemmDequantWarps;  // warp 0 TMA, warp 1 MMA, dequant
constexpr int kGemmATileBytes = kGemmTileCols * kGemmKStep * 2;  // one dequantised f16 tile
constexpr int kGemmMaxRawStages = 12;
constexpr int kGemmMaxAStages = 4;

enum GemmEpilogue : int {
  kGemmStore = 0,    // out[m][n] = acc (+ residual[m][n])
  kGemmSiluMul = 1,  // h = silu(tile 0) * tile 1 -> h16 (f16, the next GEMM's activations), h32
  kGemmPartial = 2,  // out[split][m][n] = acc (reduced by a separate pass)
};

struct GemmParams {
  int M, K, N, gs;
  int splits;  // the K steps are split evenly over gridDim.z
  int pair;    // 1: tile t from matrix t at the same columns; 0: matrix 0, 256 adjacent columns
  const uint16_t* scales[kGemmTiles];
  const uint8_t* zeros[kGemmTiles];
  int epi;
  float* out;
  const float* residual;
  __half* h16;
  float* h32;
  int raw_stages;      // ring of TMA copies: activations, packed weights, scales, zero points
  int raw_stage_bytes;
  int a_stages;        // ring of dequantised A tiles (both tiles of a step)
  int aux_stages;      // tensor-memory kernel: ring of scales / zero points (8 groups a stage)
  int tm;              // 1: the tensor-memory kernel
  unsigned* err;
  unsigned long long timeout_ns;
  unsigned long long* trace;  // optional per-CTA cycle counts (kTraceEvents slots per CTA)
  int trace_ctas;             // CTAs (in launch order) that record
};

struct GemmMaps {
  CUtensorMap x;                 // f16 activations [rows][K], box 64 x NT, 128-byte swizzle
  CUtensorMap w[kGemmTiles];     // packed weights [K/2][N] u8, box 128 x 32
  CUtensorMap sc[kGemmTiles];    // scales [K/gs][N] f16, box 128 x 8 groups (tensor-memory kernel)
  CUtensorMap ze[kGemmTiles];    // zero points [K/gs][N/2] u8, box 64 x 8 groups (ditto)
};

// Tensor-memory kernel (token tiles up to kGemmTmemMaxNT, K a multiple of 128): the
// dequantised A tiles live in tensor memory; a step is 128 k (64 packed rows); the weights
// arrive with the 128-byte swizzle; scales and zero points arrive 8 groups at a time in their
// own ring.
constexpr int kGemmTmemMaxNT = 64;   // 128- and 256-token tiles: the shared-memory kernel
constexpr int kGemmTmKStep = 128;
constexpr int kGemmTmDequantWarps = 16;  // warp d: tile d/8, column half (d/4)%2, lane quarter (d+2)%4
constexpr int kGemmTmThreads = 64 + 32 * kGemmTmDequantWarps;
constexpr int kGemmTmWeightTile = kGemmTileCols * kGemmTmKStep / 2;  // 8 KB of packed rows
constexpr int kGemmAuxGroups = 8;
constexpr int kGemmAuxStageBytes = kGemmTiles * kGemmAuxGroups * (256 + 64);  // 5120
constexpr int kGemmMaxAuxStages = 4;
constexpr int kGemmTmemMaxAStages = 3;
// activations (two 64-k chunks of nt rows), then both packed-weight tiles
__host__ __device__ constexpr int gemm_tm_raw_stage_bytes(int nt) {
  return 2 * nt * 128 + kGemmTiles * kGemmTmWeightTile;
}
// Steps (128 k) covered by one stage of the scale / zero-point ring (8 groups).
__host__ __device__ constexpr int gemm_aux_steps(int gs) { return gs / 16; }
// The tensor-memory kernel takes token tiles up to 64 and K in whole 128-k steps.
__host__ __device__ constexpr bool gemm_use_tm(int nt, int k) {
  return nt <= kGemmTmemMaxNT && k % kGemmTmKStep == 0;
}

// Shared-memory bytes of one stage of the TMA ring for a token tile of nt (1024-aligned):
// activations (nt rows of 64 f16), packed rows of both tiles (4 KB each), scales and zero
// points of up to 4 groups per tile.
__host__ __device__ constexpr int gemm_raw_stage_bytes(int nt) {
  return (nt * 128 + kGemmTiles * 4096 + kGemmTiles * 4 * (256 + 64) + 1023) & ~1023;
}
// Order of k in the GEMM activations (x16, h16): inside every aligned four k the middle two are
// swapped, so position j holds k = gemm_kperm(j) (the map is its own inverse).  The
// tensor-memory dequantiser builds each f16 pair of an A cell from one byte of two adjacent
// packed rows -- k and k + 2 from the low nibbles, k + 1 and k + 3 from the high ones -- with
// one byte permute for two cells; the shared-memory dequantiser stores its k rows in the same
// order.  Only the activations' order changes: a row's dot product is the same sum.
__host__ __device__ constexpr int gemm_kperm(int j) { return (j & ~3) | ((j & 1) << 1) | ((j >> 1) & 1); }
__host__ __device__ constexpr long long gemm_kperm(long long j) {
  return (j & ~3ll) | ((j & 1) << 1) | ((j >> 1) & 1);
}

// One stage of the dequantised ring: both A tiles.
constexpr int kGemmAStageBytes = kGemmTiles * kGemmATileBytes;

}  // namespace tk
