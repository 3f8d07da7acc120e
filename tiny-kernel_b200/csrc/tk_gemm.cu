// tk_gemm.cu -- batch >= 5 INT4 GEMM on the 5th-generation tensor cores (tcgen05).
//
// Computes the qmatmul_int4 contraction of the reference (src/kernels/shaders.zig:442-501)
//     y[m][n] = sum_g scale[g][n] * sum_{k in g} x[m][k] * (q[k][n] - zero[g][n])
// for many rows at once, on the reference's packed layout, as a GEMM whose A operand (128
// output columns x 64 k) is dequantised in shared memory and whose B operand is the f16
// activations (NT tokens x 64 k); f32 accumulators live in tensor memory.
//
// One CTA = two 128-column tiles x NT tokens x a range of K, 18 warps:
//   warp 0      TMA producer: activations (f16, 128-byte swizzle), packed weights of both
//               tiles, the step's scales and zero points -> the raw ring (full_r)
//   warps 2-17  dequantisers: warp d turns packed rows 4(d%8) .. 4(d%8)+3 of tile d/8 (k rows
//               8(d%8) .. 8(d%8)+7, one swizzle atom row group) into f16 A rows; lane l takes
//               the 4 columns 4l .. 4l+3 of a packed row with one 32-bit load.  Nibble pairs
//               become f16 by exponent constants: low nibbles q as 0x6400 | q = 1024 + q, high
//               nibbles in place as 0x5400 | q << 4 = 64 + q; (q - z) is exact, times the scale
//               one rounding.  The pairs are columns (4l, 4l+2) and (4l+1, 4l+3), so the A
//               tile's M order is permuted inside each group of 4 columns (0, 2, 1, 3).  A is
//               MN-major with the 128-byte swizzle (full_a); after the last step these warps
//               are the epilogue
//   warp 1      tensor-memory allocation and MMA issue: 2 tiles x 4 tcgen05.mma.kind::f16
//               (128 x NT x 16) per step, committed to the A stage's and the raw stage's empty
//               barriers
// The raw ring is deep (the HBM latency), the A ring short (it only decouples dequantisation
// from the MMAs).  Epilogue: tcgen05.ld of each thread's tensor-memory lane (an output column)
// for 8 tokens at a time, the four warps of a lane quarter taking every fourth token chunk;
// store (+ residual), silu(gate) * up (the FFN's h, f16 for the next GEMM and optionally f32),
// or a split-K partial.  Every wait is bounded and reports through p.err.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <mutex>

#include "tk_engine.h"
#include "tk_gemm.h"
#include "tk_internal.h"
#include "tk_ptx.cuh"

namespace tk {

namespace {

constexpr unsigned kErrGemmWait = 4u;

// Bounded wait of one thread for an mbarrier phase; false (and the error bit) on timeout.
__device__ __forceinline__ bool gemm_wait(uint64_t* bar, uint32_t parity, unsigned* err,
                                          unsigned long long timeout_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > timeout_ns) {
      atomicOr(err, kErrGemmWait);
      return false;
    }
  }
  return true;
}

// Raw stage layout (1024-byte aligned): activations (NT rows of 64 f16, the 128-byte swizzle
// needs the 1024-byte alignment), packed rows of both tiles (32 x 128 bytes each), scales
// (tile, group-in-step: 128 f16), zero points (tile, group-in-step: 64 bytes).
template <int NT>
struct RawLayout {
  static constexpr int X = 0;
  static constexpr int P = NT * 128;
  static constexpr int SC = P + kGemmTiles * 4096;
  static constexpr int ZE = SC + kGemmTiles * 4 * 256;
};

// Byte offset of element (m, k) of an MN-major A tile (128 x 64 f16, 128-byte swizzle): swizzle
// atoms of 64 m x 8 k (eight 128-byte k rows, 16-byte chunk c of row r stored at c ^ r), the
// two m atoms 1024 bytes apart (LBO), the eight k atoms 2048 bytes apart (SBO).
__host__ __device__ constexpr uint32_t a_offset(int m, int k) {
  return (uint32_t)((k >> 3) * 2048 + (m >> 6) * 1024 + (k & 7) * 128 +
                    ((((m & 63) >> 3) ^ (k & 7)) << 4) + (m & 7) * 2);
}

// Output column of tensor-memory lane (A row) l: inside each group of 4, rows hold columns
// 0, 2, 1, 3.
__device__ __forceinline__ int lane_column(int l) { return (l & ~3) | ((l & 1) << 1) | ((l >> 1) & 1); }

__device__ __forceinline__ uint32_t hsubmul(uint32_t q, uint32_t z, uint32_t s) {
  const __half2 h = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&q),
                                    *reinterpret_cast<const __half2*>(&z)),
                            *reinterpret_cast<const __half2*>(&s));
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Bounded wait that also adds the cycles it took to *acc when `timed` (tracing: the clock is
// read only then).
__device__ __forceinline__ bool gemm_wait_timed(uint64_t* bar, uint32_t parity, unsigned* err,
                                                unsigned long long timeout_ns, long long* acc,
                                                bool timed) {
  if (!timed) return gemm_wait(bar, parity, err, timeout_ns);
  const long long c0 = clock64();
  const bool ok = gemm_wait(bar, parity, err, timeout_ns);
  *acc += clock64() - c0;
  return ok;
}

// Ring position: stage index and phase parity, advanced without divisions.
struct RingPos {
  int s = 0;
  uint32_t ph = 0;
  __device__ __forceinline__ void next(int n) {
    if (++s == n) {
      s = 0;
      ph ^= 1u;
    }
  }
};

template <int NT>
__global__ void __launch_bounds__(kGemmThreads, 1)
    int4_gemm_kernel(const __grid_constant__ GemmMaps maps, const __grid_constant__ GemmParams p) {
  using L = RawLayout<NT>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full_r[kGemmMaxRawStages], empty_r[kGemmMaxRawStages];
  __shared__ uint64_t full_a[kGemmMaxAStages], empty_a[kGemmMaxAStages];
  __shared__ uint64_t done_bar;
  __shared__ uint32_t tmem_slot;
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint8_t* aring = smem;
  uint8_t* rring = smem + (size_t)p.a_stages * kGemmAStageBytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int SR = p.raw_stages, SA = p.a_stages;
  const int gps = p.gs >= kGemmKStep ? 1 : kGemmKStep / p.gs;  // groups per step
  // this CTA's tiles, tokens and K steps
  const int col0 = p.pair ? blockIdx.x * kGemmTileCols : blockIdx.x * kGemmTiles * kGemmTileCols;
  const int colt[2] = {col0, p.pair ? col0 : col0 + kGemmTileCols};
  const int m0 = blockIdx.y * NT;
  const int steps = p.K / kGemmKStep;
  const int ks0 = (int)((long long)steps * blockIdx.z / p.splits);
  const int ks1 = (int)((long long)steps * (blockIdx.z + 1) / p.splits);
  const int nsteps = ks1 - ks0;
  constexpr uint32_t kTmemCols = NT * 2 <= 32 ? 32 : (NT * 2 <= 64 ? 64 : (NT * 2 <= 128 ? 128 : (NT * 2 <= 256 ? 256 : 512)));

  if (threadIdx.x == 0) {
    for (int i = 0; i < SR; ++i) {
      mbar_init(&full_r[i], 1);
      mbar_init(&empty_r[i], kGemmDequantWarps + 1);  // dequantisers (packed rows) + MMA (x)
    }
    for (int i = 0; i < SA; ++i) {
      mbar_init(&full_a[i], kGemmDequantWarps);
      mbar_init(&empty_a[i], 1);
    }
    mbar_init(&done_bar, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&tmem_slot, kTmemCols);
  tcgen05_fence_before();
  __syncthreads();
  tcgen05_fence_after();
  const uint32_t tmem = tmem_slot;
  const int cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  unsigned long long* trace = (p.trace && cta < p.trace_ctas) ? p.trace + (size_t)cta * kTraceEvents : nullptr;
  const bool tr = trace != nullptr;
  const long long t_start = tr ? clock64() : 0;
  long long tw0 = 0, tw1 = 0;  // cycles in this warp's two kinds of waits (traced)

  if (warp == 0) {
    // ------------------------------- TMA producer -------------------------------------
    // the warp runs converged; one elected lane issues the copies
    const bool leader = elect_one();
    const uint64_t pol_w = l2_evict_first(), pol_x = l2_evict_last();
    const uint32_t bytes =
        (uint32_t)(NT * 128 + kGemmTiles * 4096 + gps * kGemmTiles * (256 + 64));
    RingPos r;
    int i = 0;
    for (; i < nsteps; ++i, r.next(SR)) {
      bool ok = true;
      if (i >= SR && lane == 0)
        ok = gemm_wait_timed(&empty_r[r.s], r.ph ^ 1u, p.err, p.timeout_ns, &tw0, tr);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      uint8_t* st = rring + (size_t)r.s * p.raw_stage_bytes;
      const int k0 = (ks0 + i) * kGemmKStep;
      const int g0 = k0 / p.gs;
      if (leader) {
        mbar_arrive_expect_tx(&full_r[r.s], bytes);
        tma_load_2d(st + L::X, &maps.x, &full_r[r.s], k0, m0, pol_x);
        for (int t = 0; t < kGemmTiles; ++t)
          tma_load_2d(st + L::P + t * 4096, &maps.w[t], &full_r[r.s], colt[t], k0 / 2, pol_w);
        for (int t = 0; t < kGemmTiles; ++t)
          for (int gi = 0; gi < gps; ++gi) {
            bulk_load(st + L::SC + (t * 4 + gi) * 256,
                      p.scales[t] + (size_t)(g0 + gi) * p.N + colt[t], 256, &full_r[r.s], pol_w);
            bulk_load(st + L::ZE + (t * 4 + gi) * 64,
                      p.zeros[t] + (size_t)(g0 + gi) * (p.N / 2) + colt[t] / 2, 64, &full_r[r.s],
                      pol_w);
          }
      }
      __syncwarp();
    }
    // no copy may be in flight when the CTA exits (only an error path gets here early)
    if (lane == 0) {
      for (int j = (i > SR ? i - SR : 0); j < i; ++j)
        gemm_wait(&full_r[j % SR], (uint32_t)((j / SR) & 1), p.err, p.timeout_ns);
      if (trace) {
        trace[0] = (unsigned long long)tw0;
        trace[1] = (unsigned long long)(clock64() - t_start);
      }
    }
  } else if (warp == 1) {
    // --------------------------------- MMA issue ----------------------------------------
    // converged warp, one elected lane issues (see elect_one)
    constexpr uint32_t idesc = umma_idesc_f16_amn(kGemmTileCols, NT);
    const bool leader = elect_one();
    RingPos ra, rr;
    for (int i = 0; i < nsteps; ++i, ra.next(SA), rr.next(SR)) {
      bool ok = true;
      if (lane == 0)
        ok = gemm_wait_timed(&full_a[ra.s], ra.ph, p.err, p.timeout_ns, &tw0, tr) &&
             gemm_wait_timed(&full_r[rr.s], rr.ph, p.err, p.timeout_ns, &tw1, tr);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      tcgen05_fence_after();
      const uint32_t xa = smem_addr(rring + (size_t)rr.s * p.raw_stage_bytes + L::X);
      const uint32_t ab = smem_addr(aring + (size_t)ra.s * kGemmAStageBytes);
      if (leader) {
#pragma unroll
        for (int t = 0; t < kGemmTiles; ++t) {
#pragma unroll
          for (int kk = 0; kk < kGemmKStep / 16; ++kk)
            umma_f16(tmem + (uint32_t)(t * NT),
                     umma_smem_desc(ab + t * kGemmATileBytes + kk * 4096, 1024, 2048, 2),
                     umma_smem_desc(xa + kk * 32, 16, 1024, 2), idesc,
                     (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&empty_a[ra.s]);
        umma_commit(&empty_r[rr.s]);
      }
      __syncwarp();
    }
    if (leader) umma_commit(&done_bar);
    __syncwarp();
    if (trace && lane == 0) {
      trace[2] = (unsigned long long)tw0;
      trace[3] = (unsigned long long)tw1;
      trace[4] = (unsigned long long)(clock64() - t_start);
    }
  } else {
    // --------------------------- dequantisers, then epilogue ------------------------------
    const int dq = warp - 2;
    const int t = dq >> 3;  // tile
    const int kg = dq & 7;  // k rows 8kg .. 8kg+7 of each step (packed rows 4kg .. 4kg+3)
    const int gi = (8 * kg) / (p.gs >= kGemmKStep ? kGemmKStep : p.gs);  // group in step
    // shared-memory offsets of this lane inside a stage: packed row 4kg, scales, zero points,
    // and its A row group (the swizzle chunk of k row j is chunk ^ j)
    const uint32_t p_off = (uint32_t)(L::P + t * 4096 + kg * 4 * 128 + lane * 4);
    const uint32_t sc_off = (uint32_t)(L::SC + (t * 4 + gi) * 256 + lane * 8);
    const uint32_t ze_off = (uint32_t)(L::ZE + (t * 4 + gi) * 64 + lane * 2);
    const uint32_t a_base = (uint32_t)(t * kGemmATileBytes) + a_offset(4 * lane, 8 * kg);
    const uint32_t chunk = (uint32_t)((lane & 15) >> 1);
    const uint32_t rring_s = smem_addr(rring), aring_s = smem_addr(aring);
    RingPos rr, ra;
    for (int i = 0; i < nsteps; ++i, rr.next(SR), ra.next(SA)) {
      if (!gemm_wait_timed(&full_r[rr.s], rr.ph, p.err, p.timeout_ns, &tw0, tr)) break;
      if (i >= SA && !gemm_wait_timed(&empty_a[ra.s], ra.ph ^ 1u, p.err, p.timeout_ns, &tw1, tr))
        break;
      const uint32_t st = rring_s + (uint32_t)rr.s * (uint32_t)p.raw_stage_bytes;
      // scales of columns 4l .. 4l+3 as (4l, 4l+2) and (4l+1, 4l+3) pairs; zero points the
      // same, once as 1024 + z (low nibbles) and once as 64 + z (high nibbles)
      const uint32_t sx = ld_shared_u32(st + sc_off), sy = ld_shared_u32(st + sc_off + 4);
      const uint32_t zz = ld_shared_u32(st + (ze_off & ~3u)) >> ((ze_off & 2u) * 8);
      const uint32_t s02 = __byte_perm(sx, sy, 0x5410), s13 = __byte_perm(sx, sy, 0x7632);
      const uint32_t z02 = (zz & 0xFu) | ((zz & 0xF00u) << 8);
      const uint32_t z13 = ((zz >> 4) & 0xFu) | ((zz & 0xF000u) << 4);
      const uint32_t zl02 = 0x64006400u | z02, zh02 = 0x54005400u | (z02 << 4);
      const uint32_t zl13 = 0x64006400u | z13, zh13 = 0x54005400u | (z13 << 4);
      const uint32_t ab = aring_s + (uint32_t)ra.s * (uint32_t)kGemmAStageBytes + a_base;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const uint32_t w = ld_shared_u32(st + p_off + r * 128);
        const uint32_t w8 = w >> 8;
        const uint32_t e0 = hsubmul((w & 0x000F000Fu) | 0x64006400u, zl02, s02);
        const uint32_t e1 = hsubmul((w8 & 0x000F000Fu) | 0x64006400u, zl13, s13);
        const uint32_t o0 = hsubmul((w & 0x00F000F0u) | 0x54005400u, zh02, s02);
        const uint32_t o1 = hsubmul((w8 & 0x00F000F0u) | 0x54005400u, zh13, s13);
        // k rows 2r and 2r+1 of the group at A rows gemm_kperm(2r), gemm_kperm(2r+1) (the
        // activations' k order): row j at j * 128, chunk ^ j
        constexpr int je[4] = {gemm_kperm(0), gemm_kperm(2), gemm_kperm(4), gemm_kperm(6)};
        constexpr int jo[4] = {gemm_kperm(1), gemm_kperm(3), gemm_kperm(5), gemm_kperm(7)};
        const uint32_t ce = ((chunk ^ (uint32_t)je[r]) - chunk) << 4;
        const uint32_t co = ((chunk ^ (uint32_t)jo[r]) - chunk) << 4;
        st_shared_v2(ab + (uint32_t)je[r] * 128u + ce, e0, e1);
        st_shared_v2(ab + (uint32_t)jo[r] * 128u + co, o0, o1);
      }
      fence_proxy_async_smem();  // the A tiles are read by tcgen05.mma (async proxy)
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&full_a[ra.s]);
        mbar_arrive(&empty_r[rr.s]);
      }
    }
    if (trace && warp == 2 && lane == 0) {
      trace[5] = (unsigned long long)tw0;
      trace[6] = (unsigned long long)tw1;
      trace[7] = (unsigned long long)(clock64() - t_start);
    }
    // epilogue: this warp's 32 tensor-memory lanes are A rows q*32 .. q*32+31; the four warps
    // of a lane quarter take every fourth chunk of 8 tokens
    bool ok = true;
    if (lane == 0) ok = nsteps > 0 && gemm_wait(&done_bar, 0u, p.err, p.timeout_ns);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (ok) {
      tcgen05_fence_after();
      const int q = warp & 3;
      const int cl = lane_column(q * 32 + lane);
      const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16);
      for (int j = dq >> 2; j < NT / 8; j += kGemmDequantWarps / 4) {
        uint32_t v0[8], v1[8];
        tmem_ld8(tl + (uint32_t)(0 * NT + j * 8), v0);
        tmem_ld8(tl + (uint32_t)(1 * NT + j * 8), v1);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int tok = m0 + j * 8 + e;
          if (tok >= p.M) continue;
          const float a0 = __uint_as_float(v0[e]), a1 = __uint_as_float(v1[e]);
          if (p.epi == kGemmSiluMul) {
            const float h = a0 / (1.0f + expf(-a0)) * a1;
            const size_t o = (size_t)tok * p.N + colt[0] + cl;
            p.h16[(size_t)tok * p.N + gemm_kperm(colt[0] + cl)] = __float2half_rn(h);
            if (p.h32) p.h32[o] = h;
          } else if (p.epi == kGemmStore) {
            const size_t o0 = (size_t)tok * p.N + colt[0] + cl, o1 = (size_t)tok * p.N + colt[1] + cl;
            p.out[o0] = p.residual ? p.residual[o0] + a0 : a0;
            p.out[o1] = p.residual ? p.residual[o1] + a1 : a1;
          } else {
            const size_t base = ((size_t)blockIdx.z * p.M + tok) * p.N;
            p.out[base + colt[0] + cl] = a0;
            p.out[base + colt[1] + cl] = a1;
          }
        }
      }
    }
  }
  tcgen05_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// ------------------------------------------------------------------------------------------
// Tensor-memory variant (token tiles up to 64, K in whole 128-k steps).  The A operand
// (dequantised weights) is written to tensor memory with tcgen05.st and read from there by
// tcgen05.mma, so shared memory carries only the TMA copies, the dequantisers' reads and the
// MMA's activation reads.  A step is 128 k.
//   warp 0      TMA: per step the activations (two 64-k chunks) and the two packed-weight tiles
//               (128 columns x 64 packed rows, 128-byte swizzle) -> raw ring; every
//               gemm_aux_steps(gs) steps the scales and zero points of 8 groups of both tiles
//               -> aux ring
//   warp 1      tensor-memory allocation, MMA issue (A from tensor memory): 2 tiles x 8
//               tcgen05.mma.kind::f16 (128 x NT x 16) per step
//   warps 2-17  dequantisers, then the epilogue.  Warp w writes tensor-memory lanes
//               32(w%4) .. +31 (its lane quarter) of tile t, columns 32ch .. 32ch+31 (packed
//               rows of the step), (t, ch) from (w-2)/4.  Lane l (j = l/4, u = l%4) loads the
//               32-bit words of packed rows 32ch + 8c + 2u + e (c in 0..3, e in {0,1}) at
//               columns 32q + 4j .. 32q + 4j + 3 (rows 2 apart inside a quad: with the swizzle
//               the warp's loads hit 32 distinct banks) and stores their cells with
//               tcgen05.st.16x256b, whose thread layout holds exactly those: column
//               32ch + 8c + 2u + e' of lanes j + 8i' + 16h for byte i = 2h + i'.  So
//               tensor-memory lane 32q + l holds output column 32q + 4(l%8) + l/8.
//   The two words of a lane at packed rows 2p and 2p + 1 (e = 0, 1) give the cells of tensor-memory
//   columns 2p (e' = 0) and 2p + 1 (e' = 1): one byte permute puts byte i of both words in bytes
//   0 and 2, and one mask + or makes the f16 pair (1024 + lo, 1024 + lo') -- k = 4p, 4p + 2 -- or
//   (64 + hi, 64 + hi') -- k = 4p + 1, 4p + 3 -- by the exponent constants 0x6400 / 0x5400; minus
//   (1024 + z, 1024 + z) or (64 + z, 64 + z) (exact), times (s, s) (one rounding).  The MMA's k
//   order is thus 4p, 4p + 2, 4p + 1, 4p + 3: the activations' order (gemm_kperm).
// A step's tensor-memory stores are completed (tcgen05.wait::st) and the step handed to the MMA
// warp at the end of the same step: the MMA of step i then overlaps the cells of step i + 1, and
// the dequantisers' wait for a free A stage (three steps back) stays short.  (Completing them
// after the next step's cells instead hides the store latency but puts a whole step between the
// cells and the MMA, and the three-stage chain then set the pace: 1.0 us per step.)
__device__ __forceinline__ int tm_lane_column(int l) { return 4 * (l & 7) + (l >> 3); }

template <int NT>
__global__ void __launch_bounds__(kGemmTmThreads, 1)
    int4_gemm_tm_kernel(const __grid_constant__ GemmMaps maps, const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full_r[kGemmMaxRawStages], empty_r[kGemmMaxRawStages];
  __shared__ uint64_t full_x[kGemmMaxAuxStages], empty_x[kGemmMaxAuxStages];
  __shared__ uint64_t full_a[kGemmTmemMaxAStages], empty_a[kGemmTmemMaxAStages];
  __shared__ uint64_t done_bar;
  __shared__ uint32_t tmem_slot;
  constexpr int kX = 0, kP = 2 * NT * 128;  // raw stage: activations, then the packed tiles
  constexpr int kRaw = gemm_tm_raw_stage_bytes(NT);
  constexpr int SA = NT >= 128 ? 2 : 3;
  constexpr uint32_t kAcol0 = 2 * NT;       // tensor-memory columns: accumulators, A stages
  constexpr uint32_t kAStageCols = kGemmTiles * kGemmTmKStep / 2;  // 128
  constexpr uint32_t kTmemCols = 512;
  static_assert(kAcol0 + SA * kAStageCols <= kTmemCols, "tensor memory");
  // traced: global-timer stamps of the CTA's entry, its setup, the dequantisers' loop end, the
  // epilogue end and the exit (slots 10-14)
  const unsigned long long g_entry = p.trace ? global_timer_ns() : 0ull;
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint8_t* rring = smem;
  uint8_t* xring = smem + (size_t)p.raw_stages * kRaw;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int SR = p.raw_stages, SX = p.aux_stages;
  const int spa = gemm_aux_steps(p.gs);
  const int lg = __ffs(p.gs) - 1;  // group sizes are powers of two: no divisions in the loops
  const int col0 = p.pair ? blockIdx.x * kGemmTileCols : blockIdx.x * kGemmTiles * kGemmTileCols;
  const int colt[2] = {col0, p.pair ? col0 : col0 + kGemmTileCols};
  const int m0 = blockIdx.y * NT;
  const int steps = p.K / kGemmTmKStep;
  const int ks0 = (int)((long long)steps * blockIdx.z / p.splits);
  const int ks1 = (int)((long long)steps * (blockIdx.z + 1) / p.splits);
  const int nsteps = ks1 - ks0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < SR; ++i) {
      mbar_init(&full_r[i], 1);
      mbar_init(&empty_r[i], kGemmTmDequantWarps + 1);  // dequantisers (weights) + MMA (x)
    }
    for (int i = 0; i < SX; ++i) {
      mbar_init(&full_x[i], 1);
      mbar_init(&empty_x[i], kGemmTmDequantWarps);
    }
    for (int i = 0; i < SA; ++i) {
      mbar_init(&full_a[i], kGemmTmDequantWarps);
      mbar_init(&empty_a[i], 1);
    }
    mbar_init(&done_bar, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&tmem_slot, kTmemCols);
  tcgen05_fence_before();
  __syncthreads();
  tcgen05_fence_after();
  const uint32_t tmem = tmem_slot;
  const int cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  unsigned long long* trace = (p.trace && cta < p.trace_ctas) ? p.trace + (size_t)cta * kTraceEvents : nullptr;
  const bool tr = trace != nullptr;
  const long long t_start = tr ? clock64() : 0;
  long long tw0 = 0, tw1 = 0;  // traced wait cycles
  if (tr && threadIdx.x == 0) {
    trace[10] = g_entry;
    trace[11] = global_timer_ns();
  }

  if (warp == 0) {
    // ------------------------------- TMA producer -------------------------------------
    const bool leader = elect_one();
    const uint64_t pol_w = l2_evict_first(), pol_x = l2_evict_last();
    RingPos r, rx;
    int i = 0, na = 0, ia = 0;  // ia: steps into the current scale stage
    bool ok = true;
    for (; i < nsteps; ++i, r.next(SR), ia = (ia + 1 == spa) ? 0 : ia + 1) {
      if (ia == 0) {
        if (na >= SX && lane == 0)
          ok = gemm_wait_timed(&empty_x[rx.s], rx.ph ^ 1u, p.err, p.timeout_ns, &tw0, tr);
        if (!__shfl_sync(0xffffffffu, ok, 0)) break;
        const int gb = ((ks0 + i) * kGemmTmKStep) >> lg;
        uint8_t* xs = xring + (size_t)rx.s * kGemmAuxStageBytes;
        if (leader) {
          mbar_arrive_expect_tx(&full_x[rx.s], (uint32_t)kGemmAuxStageBytes);
          for (int t = 0; t < kGemmTiles; ++t) {
            tma_load_2d(xs + t * 2048, &maps.sc[t], &full_x[rx.s], colt[t], gb, pol_w);
            tma_load_2d(xs + 4096 + t * 512, &maps.ze[t], &full_x[rx.s], colt[t] / 2, gb, pol_w);
          }
        }
        __syncwarp();
        rx.next(SX);
        ++na;
      }
      if (i >= SR && lane == 0)
        ok = gemm_wait_timed(&empty_r[r.s], r.ph ^ 1u, p.err, p.timeout_ns, &tw0, tr);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      uint8_t* st = rring + (size_t)r.s * kRaw;
      const int k0 = (ks0 + i) * kGemmTmKStep;
      if (leader) {
        mbar_arrive_expect_tx(&full_r[r.s], (uint32_t)kRaw);
        tma_load_2d(st + kX, &maps.x, &full_r[r.s], k0, m0, pol_x);
        tma_load_2d(st + kX + NT * 128, &maps.x, &full_r[r.s], k0 + 64, m0, pol_x);
        for (int t = 0; t < kGemmTiles; ++t)
          tma_load_2d(st + kP + t * kGemmTmWeightTile, &maps.w[t], &full_r[r.s], colt[t], k0 / 2,
                      pol_w);
      }
      __syncwarp();
    }
    // no copy may be in flight when the CTA exits (only an error path gets here early)
    if (lane == 0) {
      for (int j = (i > SR ? i - SR : 0); j < i; ++j)
        gemm_wait(&full_r[j % SR], (uint32_t)((j / SR) & 1), p.err, p.timeout_ns);
      for (int j = (na > SX ? na - SX : 0); j < na; ++j)
        gemm_wait(&full_x[j % SX], (uint32_t)((j / SX) & 1), p.err, p.timeout_ns);
      if (trace) {
        trace[0] = (unsigned long long)tw0;
        trace[1] = (unsigned long long)(clock64() - t_start);
      }
    }
  } else if (warp == 1) {
    // --------------------------------- MMA issue ----------------------------------------
    constexpr uint32_t idesc = umma_idesc_f16(kGemmTileCols, NT);
    const bool leader = elect_one();
    RingPos ra, rr;
    for (int i = 0; i < nsteps; ++i, ra.next(SA), rr.next(SR)) {
      bool ok = true;
      if (lane == 0)
        ok = gemm_wait_timed(&full_a[ra.s], ra.ph, p.err, p.timeout_ns, &tw0, tr) &&
             gemm_wait_timed(&full_r[rr.s], rr.ph, p.err, p.timeout_ns, &tw1, tr);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      tcgen05_fence_after();
      const uint32_t xa = smem_addr(rring + (size_t)rr.s * kRaw + kX);
      const uint32_t ta = tmem + kAcol0 + kAStageCols * (uint32_t)ra.s;
      if (leader) {
        // one descriptor per step: the k offsets add to its address field (shared-memory
        // addresses stay below 256 KB, so the 14-bit field never carries)
        const uint64_t bdesc = umma_smem_desc(xa, 16, 1024, 2);
#pragma unroll
        for (int t = 0; t < kGemmTiles; ++t) {
#pragma unroll
          for (int kk = 0; kk < kGemmTmKStep / 16; ++kk)
            umma_f16_ts(tmem + (uint32_t)(t * NT), ta + (uint32_t)(64 * t + 8 * kk),
                        bdesc + (uint64_t)((((kk >> 2) * (NT * 128) + (kk & 3) * 32)) >> 4),
                        idesc, (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&empty_a[ra.s]);
        umma_commit(&empty_r[rr.s]);
      }
      __syncwarp();
    }
    if (leader) umma_commit(&done_bar);
    __syncwarp();
    if (trace && lane == 0) {
      trace[2] = (unsigned long long)tw0;
      trace[3] = (unsigned long long)tw1;
      trace[4] = (unsigned long long)(clock64() - t_start);
    }
  } else {
    // --------------------------- dequantisers, then epilogue ------------------------------
    const int q = warp & 3;              // tensor-memory lane quarter
    const int pidx = (warp - 2) >> 2;    // (tile, column half)
    const int t = pidx >> 1, ch = pidx & 1;
    const int j = lane >> 2, u = lane & 3;
    const int cbase = 32 * q + 4 * j;  // this lane's 4 output columns (within the tile)
    // swizzled shared-memory offsets (inside a raw stage) of packed rows 32ch + 8c + 2u + e at
    // columns cbase .. cbase + 3: chunk (cbase / 16) ^ (row % 8), row % 8 = 2u + e; + c * 1024
    uint32_t w_off[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int row = 2 * u + e;
      w_off[e] = (uint32_t)(kP + t * kGemmTmWeightTile + ch * 4096 + row * 128 +
                            (((cbase >> 4) ^ row) << 4) + (cbase & 15));
    }
    const uint32_t rbase = smem_addr(rring), xbase = smem_addr(xring);
    // tensor-memory address of this warp's block: lanes 32q (+16h), columns 32ch of tile t
    const uint32_t tl = tmem + ((uint32_t)(32 * q) << 16) + kAcol0 + (uint32_t)(64 * t + 32 * ch);
    const uint32_t gmask = (uint32_t)p.gs - 1u;
    RingPos rr, ra, rx;
    int gb = 0;
    int pend_r = -1, pend_a = -1, pend_x = -1;  // stages of the step whose stores are pending
    long long t_comp = 0, t_cells = 0;          // traced: cycles completing stores, computing
    auto complete_pending = [&]() {
      const long long c0 = tr ? clock64() : 0;
      tmem_st_wait();
      tcgen05_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&full_a[pend_a]);
        mbar_arrive(&empty_r[pend_r]);
        if (pend_x >= 0) mbar_arrive(&empty_x[pend_x]);
      }
      if (tr) t_comp += clock64() - c0;
    };
    int ia = 0;  // steps into the current scale stage
    for (int i = 0; i < nsteps; ++i, rr.next(SR), ra.next(SA)) {
      if (ia == 0) {
        if (!gemm_wait_timed(&full_x[rx.s], rx.ph, p.err, p.timeout_ns, &tw0, tr)) break;
        gb = ((ks0 + i) * kGemmTmKStep) >> lg;
      }
      if (!gemm_wait_timed(&full_r[rr.s], rr.ph, p.err, p.timeout_ns, &tw0, tr)) break;
      if (i >= SA && !gemm_wait_timed(&empty_a[ra.s], ra.ph ^ 1u, p.err, p.timeout_ns, &tw1, tr)) break;
      tcgen05_fence_after();
      const long long c_cells = tr ? clock64() : 0;
      const uint32_t st = rbase + (uint32_t)rr.s * (uint32_t)kRaw;
      const uint32_t xs = xbase + (uint32_t)rx.s * (uint32_t)kGemmAuxStageBytes;
      const int k0 = (ks0 + i) * kGemmTmKStep;
      uint32_t h0[16], h1[16];  // the two 16x256b.x4 stores (lane halves h = 0, 1)
      uint32_t sp[4], zl[4], zh[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (c == 0 || ((uint32_t)(16 * c) & gmask) == 0u) {
          // scales and zero points of this lane's 4 columns in the group of k = k0 + 64ch + 16c
          const int g = ((k0 + 64 * ch + 16 * c) >> lg) - gb;
          const uint32_t sx = ld_shared_u32(xs + t * 2048 + g * 256 + cbase * 2);
          const uint32_t sy = ld_shared_u32(xs + t * 2048 + g * 256 + cbase * 2 + 4);
          const uint32_t zw = ld_shared_u32(xs + 4096 + t * 512 + g * 64 + ((cbase >> 1) & ~3));
          const uint32_t zz = zw >> ((cbase & 4) ? 16 : 0);  // nibbles of columns cbase .. +3
          sp[0] = __byte_perm(sx, sx, 0x1010);
          sp[1] = __byte_perm(sx, sx, 0x3232);
          sp[2] = __byte_perm(sy, sy, 0x1010);
          sp[3] = __byte_perm(sy, sy, 0x3232);
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            const uint32_t z = (zz >> (4 * b)) & 0xFu;
            zl[b] = 0x64006400u + z * 0x00010001u;  // (1024 + z, 1024 + z)
            zh[b] = 0x54005400u + z * 0x00100010u;  // (64 + z, 64 + z)
          }
        }
        const uint32_t w0 = ld_shared_u32(st + w_off[0] + (uint32_t)(c * 1024));
        const uint32_t w1 = ld_shared_u32(st + w_off[1] + (uint32_t)(c * 1024));
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const uint32_t v = __byte_perm(w0, w1, (uint32_t)(b | (b << 4) | ((4 + b) << 8) | ((4 + b) << 12)));
          const uint32_t lo = hsubmul((v & 0x000F000Fu) | 0x64006400u, zl[b], sp[b]);
          const uint32_t hi = hsubmul((v & 0x00F000F0u) | 0x54005400u, zh[b], sp[b]);
          // byte b = 2h + i' -> store h, registers 4c + 2i' + e' (e' = 0: lo, 1: hi)
          if (b < 2) {
            h0[4 * c + 2 * (b & 1)] = lo;
            h0[4 * c + 2 * (b & 1) + 1] = hi;
          } else {
            h1[4 * c + 2 * (b & 1)] = lo;
            h1[4 * c + 2 * (b & 1) + 1] = hi;
          }
        }
      }
      if (tr) t_cells += clock64() - c_cells;
      const uint32_t ta = tl + kAStageCols * (uint32_t)ra.s;
      tmem_st_16x256b_x4(ta, h0);
      tmem_st_16x256b_x4(ta + (16u << 16), h1);
      pend_r = rr.s;
      pend_a = ra.s;
      const bool last_of_stage = ia + 1 == spa;
      pend_x = (last_of_stage || i == nsteps - 1) ? rx.s : -1;
      complete_pending();
      if (last_of_stage) {
        rx.next(SX);
        ia = 0;
      } else {
        ++ia;
      }
    }
    if (trace && warp == 2 && lane == 0) {
      trace[5] = (unsigned long long)tw0;
      trace[6] = (unsigned long long)tw1;
      trace[7] = (unsigned long long)(clock64() - t_start);
      trace[8] = (unsigned long long)t_comp;
      trace[9] = (unsigned long long)t_cells;
      trace[12] = global_timer_ns();
    }
    // epilogue: lane quarter q, the four warps of a quarter take every fourth 8-token chunk
    bool ok = true;
    if (lane == 0) ok = nsteps > 0 && gemm_wait(&done_bar, 0u, p.err, p.timeout_ns);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (ok) {
      tcgen05_fence_after();
      const int cl = 32 * q + tm_lane_column(lane);
      const uint32_t td = tmem + ((uint32_t)(32 * q) << 16);
      for (int jj = pidx; jj < NT / 8; jj += 4) {
        uint32_t v0[8], v1[8];
        tmem_ld8(td + (uint32_t)(0 * NT + jj * 8), v0);
        tmem_ld8(td + (uint32_t)(1 * NT + jj * 8), v1);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int tok = m0 + jj * 8 + e;
          if (tok >= p.M) continue;
          const float a0 = __uint_as_float(v0[e]), a1 = __uint_as_float(v1[e]);
          if (p.epi == kGemmSiluMul) {
            const float h = a0 / (1.0f + expf(-a0)) * a1;
            const size_t o = (size_t)tok * p.N + colt[0] + cl;
            p.h16[(size_t)tok * p.N + gemm_kperm(colt[0] + cl)] = __float2half_rn(h);
            if (p.h32) p.h32[o] = h;
          } else if (p.epi == kGemmStore) {
            const size_t o0 = (size_t)tok * p.N + colt[0] + cl, o1 = (size_t)tok * p.N + colt[1] + cl;
            p.out[o0] = p.residual ? p.residual[o0] + a0 : a0;
            p.out[o1] = p.residual ? p.residual[o1] + a1 : a1;
          } else {
            const size_t base = ((size_t)blockIdx.z * p.M + tok) * p.N;
            p.out[base + colt[0] + cl] = a0;
            p.out[base + colt[1] + cl] = a1;
          }
        }
      }
    }
  }
  if (tr && warp == 2 && lane == 0) trace[13] = global_timer_ns();
  tcgen05_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
  if (tr && threadIdx.x == 0) trace[14] = global_timer_ns();
}

// The dynamic shared-memory attribute of instantiation `slot` (0-2: tensor-memory kernel at 16,
// 32, 64 tokens; 3-4: shared-memory kernel at 128, 256), set again only when it is launched on a
// device with another size than its last launch there: the call costs host time ahead of every
// launch otherwise (or in an earlier CUDA context of the device: attr_generation).
cudaError_t set_smem_attr(const void* kern, int slot, size_t smem) {
  constexpr int kMaxDevices = 64, kSlots = 5;
  static std::mutex mu;
  struct Last {
    size_t smem;
    unsigned gen;
  };
  static Last last[kMaxDevices][kSlots] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  Last* L = dev >= 0 && dev < kMaxDevices ? &last[dev][slot] : nullptr;
  const unsigned gen = attr_generation(dev);
  if (L && L->smem == smem && L->gen == gen) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (L) *L = e == cudaSuccess ? Last{smem, gen} : Last{0, 0};
  return e;
}

template <int NT>
cudaError_t launch_tm(const GemmMaps& maps, const GemmParams& p, dim3 grid, size_t smem,
                      cudaStream_t st) {
  auto kern = int4_gemm_tm_kernel<NT>;
  cudaError_t e = set_smem_attr(reinterpret_cast<const void*>(kern), NT == 16 ? 0 : NT == 32 ? 1 : 2,
                                smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, kGemmTmThreads, smem, st>>>(maps, p);
  return cudaGetLastError();
}

template <int NT>
cudaError_t launch_nt(const GemmMaps& maps, const GemmParams& p, dim3 grid, size_t smem,
                      cudaStream_t st) {
  auto kern = int4_gemm_kernel<NT>;
  cudaError_t e = set_smem_attr(reinterpret_cast<const void*>(kern), NT == 128 ? 3 : 4, smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, kGemmThreads, smem, st>>>(maps, p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t gemm_launch(int nt, const GemmMaps& maps, const GemmParams& p, dim3 grid, size_t smem,
                        cudaStream_t st) {
  if (p.tm) {
    switch (nt) {
      case 16: return launch_tm<16>(maps, p, grid, smem, st);
      case 32: return launch_tm<32>(maps, p, grid, smem, st);
      case 64: return launch_tm<64>(maps, p, grid, smem, st);
      default: return cudaErrorInvalidValue;
    }
  }
  // K is a multiple of 128 on every path that reaches the GEMM (the engine's column tiles), so
  // the shared-memory-operand kernel serves the 128- and 256-token tiles
  if (nt == 128) return launch_nt<128>(maps, p, grid, smem, st);
  if (nt == 256) return launch_nt<256>(maps, p, grid, smem, st);
  return cudaErrorInvalidValue;
}

}  // namespace tk
