// tk_gemm.cu -- batch >= 16 INT4 GEMM on the 5th-generation tensor cores (tcgen05).
//
// Computes the qmatmul_int4 contraction of the reference (src/kernels/shaders.zig:442-501)
//     y[m][n] = sum_g scale[g][n] * sum_{k in g} x[m][k] * (q[k][n] - zero[g][n])
// for many rows at once, on the reference's packed layout, as a GEMM whose A operand (128
// output columns x 64 k) is dequantised in shared memory and whose B operand is the f16
// activations (NT tokens x 64 k); f32 accumulators live in tensor memory.
//
// One CTA = two 128-column tiles x NT tokens x a range of K, 10 warps:
//   warp 0     TMA producer: activations (f16, 128-byte swizzle), packed weights of both
//              tiles, the step's scales and zero points -> the raw ring (full_r)
//   warps 2-9  dequantisers: warp d turns packed rows 8(d%4) .. 8(d%4)+7 of tile d/4 into 16
//              f16 k rows of the A tile; lane l takes the 4 columns 4l .. 4l+3 of a row with one
//              32-bit load and makes ((q - z) * scale, one rounding) by the exponent trick
//              0x6400 | q = 1024 + q on nibble pairs (columns 4l, 4l+2 and 4l+1, 4l+3), so the
//              A tile's M order is permuted inside each group of 4 columns (0, 2, 1, 3); A is
//              MN-major with the 128-byte swizzle (full_a); after the last step they are the
//              epilogue
//   warp 1     tensor-memory allocation and MMA issue: 2 tiles x 4 tcgen05.mma.kind::f16
//              (128 x NT x 16) per step, committed to the A stage's and the raw stage's empty
//              barriers
// The raw ring is deep (the HBM latency), the A ring short (it only decouples dequantisation
// from the MMAs).  Epilogue: tcgen05.ld of each thread's tensor-memory lane (an output column)
// for 8 tokens at a time, the two warps of a lane quarter taking alternate token chunks;
// store (+ residual), silu(gate) * up (the FFN's h, f16 for the next GEMM and optionally f32),
// or a split-K partial.  Every wait is bounded and reports through p.err.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "tk_engine.h"
#include "tk_gemm.h"
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
__device__ __forceinline__ uint32_t a_offset(int m, int k) {
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

  if (warp == 0) {
    // ------------------------------- TMA producer -------------------------------------
    if (lane == 0) {
      const uint64_t pol_w = l2_evict_first(), pol_x = l2_evict_last();
      const uint32_t bytes =
          (uint32_t)(NT * 128 + kGemmTiles * 4096 + gps * kGemmTiles * (256 + 64));
      int i = 0;
      for (; i < nsteps; ++i) {
        const int s = i % SR, r = i / SR;
        if (r > 0 && !gemm_wait(&empty_r[s], (uint32_t)((r - 1) & 1), p.err, p.timeout_ns)) break;
        uint8_t* st = rring + (size_t)s * p.raw_stage_bytes;
        const int k0 = (ks0 + i) * kGemmKStep;
        mbar_arrive_expect_tx(&full_r[s], bytes);
        tma_load_2d(st + L::X, &maps.x, &full_r[s], k0, m0, pol_x);
        for (int t = 0; t < kGemmTiles; ++t)
          tma_load_2d(st + L::P + t * 4096, &maps.w[t], &full_r[s], colt[t], k0 / 2, pol_w);
        const int g0 = k0 / p.gs;
        for (int t = 0; t < kGemmTiles; ++t)
          for (int gi = 0; gi < gps; ++gi) {
            bulk_load(st + L::SC + (t * 4 + gi) * 256,
                      p.scales[t] + (size_t)(g0 + gi) * p.N + colt[t], 256, &full_r[s], pol_w);
            bulk_load(st + L::ZE + (t * 4 + gi) * 64,
                      p.zeros[t] + (size_t)(g0 + gi) * (p.N / 2) + colt[t] / 2, 64, &full_r[s],
                      pol_w);
          }
      }
      // no copy may be in flight when the CTA exits (only an error path gets here early)
      for (int j = (i > SR ? i - SR : 0); j < i; ++j)
        gemm_wait(&full_r[j % SR], (uint32_t)((j / SR) & 1), p.err, p.timeout_ns);
    }
  } else if (warp == 1) {
    // --------------------------------- MMA issue ----------------------------------------
    constexpr uint32_t idesc = umma_idesc_f16_amn(kGemmTileCols, NT);
    for (int i = 0; i < nsteps; ++i) {
      const int sa = i % SA, sr = i % SR;
      bool ok = true;
      if (lane == 0)
        ok = gemm_wait(&full_a[sa], (uint32_t)((i / SA) & 1), p.err, p.timeout_ns) &&
             gemm_wait(&full_r[sr], (uint32_t)((i / SR) & 1), p.err, p.timeout_ns);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      tcgen05_fence_after();
      if (lane == 0) {
        const uint32_t xa = smem_addr(rring + (size_t)sr * p.raw_stage_bytes + L::X);
        const uint32_t ab = smem_addr(aring + (size_t)sa * kGemmAStageBytes);
#pragma unroll
        for (int t = 0; t < kGemmTiles; ++t) {
#pragma unroll
          for (int kk = 0; kk < kGemmKStep / 16; ++kk)
            umma_f16(tmem + (uint32_t)(t * NT),
                     umma_smem_desc(ab + t * kGemmATileBytes + kk * 4096, 1024, 2048, 2),
                     umma_smem_desc(xa + kk * 32, 16, 1024, 2), idesc,
                     (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&empty_a[sa]);
        umma_commit(&empty_r[sr]);
      }
      __syncwarp();
    }
    if (lane == 0) umma_commit(&done_bar);
  } else {
    // --------------------------- dequantisers, then epilogue ------------------------------
    const int dq = warp - 2;
    const int t = dq >> 2;        // tile
    const int kq = dq & 3;        // k rows 16kq .. 16kq+15 of each step
    const int gi = (16 * kq) / (p.gs >= kGemmKStep ? kGemmKStep : p.gs);  // group in step
    for (int i = 0; i < nsteps; ++i) {
      const int sr = i % SR, sa = i % SA;
      if (!gemm_wait(&full_r[sr], (uint32_t)((i / SR) & 1), p.err, p.timeout_ns)) break;
      if (i >= SA && !gemm_wait(&empty_a[sa], (uint32_t)((i / SA - 1) & 1), p.err, p.timeout_ns))
        break;
      const uint8_t* st = rring + (size_t)sr * p.raw_stage_bytes;
      // scales of columns 4l .. 4l+3 as (4l, 4l+2) and (4l+1, 4l+3) pairs; zero points the same
      const uint2 sc = *reinterpret_cast<const uint2*>(st + L::SC + (t * 4 + gi) * 256 + lane * 8);
      const uint32_t zz = *reinterpret_cast<const uint16_t*>(st + L::ZE + (t * 4 + gi) * 64 + lane * 2);
      const uint32_t s02 = __byte_perm(sc.x, sc.y, 0x5410), s13 = __byte_perm(sc.x, sc.y, 0x7632);
      const uint32_t z02 = 0x64006400u | (zz & 0xFu) | ((zz & 0xF00u) << 8);
      const uint32_t z13 = 0x64006400u | ((zz >> 4) & 0xFu) | ((zz & 0xF000u) << 4);
      const uint8_t* pk = st + L::P + t * 4096 + kq * 8 * 128 + lane * 4;
      uint8_t* at = aring + (size_t)sa * kGemmAStageBytes + t * kGemmATileBytes;
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(pk + r * 128);
        const int k = kq * 16 + 2 * r;
        const uint32_t e0 = hsubmul((w & 0x000F000Fu) | 0x64006400u, z02, s02);
        const uint32_t e1 = hsubmul(((w >> 8) & 0x000F000Fu) | 0x64006400u, z13, s13);
        const uint32_t o0 = hsubmul(((w >> 4) & 0x000F000Fu) | 0x64006400u, z02, s02);
        const uint32_t o1 = hsubmul(((w >> 12) & 0x000F000Fu) | 0x64006400u, z13, s13);
        *reinterpret_cast<uint2*>(at + a_offset(4 * lane, k)) = make_uint2(e0, e1);
        *reinterpret_cast<uint2*>(at + a_offset(4 * lane, k + 1)) = make_uint2(o0, o1);
      }
      fence_proxy_async_smem();  // the A tiles are read by tcgen05.mma (async proxy)
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&full_a[sa]);
        mbar_arrive(&empty_r[sr]);
      }
    }
    // epilogue: this warp's 32 tensor-memory lanes are A rows q*32 .. q*32+31; the two warps
    // of a lane quarter take alternate chunks of 8 tokens
    bool ok = true;
    if (lane == 0) ok = nsteps > 0 && gemm_wait(&done_bar, 0u, p.err, p.timeout_ns);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (ok) {
      tcgen05_fence_after();
      const int q = warp & 3;
      const int cl = lane_column(q * 32 + lane);
      const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16);
      for (int j = dq >> 2; j < NT / 8; j += 2) {
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
            p.h16[o] = __float2half_rn(h);
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

template <int NT>
cudaError_t launch_nt(const GemmMaps& maps, const GemmParams& p, dim3 grid, size_t smem,
                      cudaStream_t st) {
  auto kern = int4_gemm_kernel<NT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, kGemmThreads, smem, st>>>(maps, p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t gemm_launch(int nt, const GemmMaps& maps, const GemmParams& p, dim3 grid, size_t smem,
                        cudaStream_t st) {
  switch (nt) {
    case 16: return launch_nt<16>(maps, p, grid, smem, st);
    case 32: return launch_nt<32>(maps, p, grid, smem, st);
    case 64: return launch_nt<64>(maps, p, grid, smem, st);
    case 128: return launch_nt<128>(maps, p, grid, smem, st);
    case 256: return launch_nt<256>(maps, p, grid, smem, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace tk
