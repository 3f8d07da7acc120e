// tk_simple.cu -- CUDA-core kernels for the small ops of the path and the fallback GEMV.
//
//  * qmatmul_int4_generic: any legal qmatmul_int4 shape (k % group == 0, group % 8 == 0,
//    n even).  One thread per output column; accumulates in exactly the order of the
//    reference shader (src/kernels/shaders.zig:481-497): acc += (x * scale) * (q - zero),
//    k ascending, with no FMA contraction, so it matches the f32 oracle bit for bit.
//  * dequant_int4: the test hook for dequantisation bit-exactness (shaders.zig:474-495).
//  * rmsnorm, fused_rmsnorm_rope, silu_mul, add: shaders.zig:16-56, 124-182, 344-357,
//    812-824; one CTA per row for the reductions.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdint>

#include "tk_gemm.h"
#include "tk_internal.h"

namespace tk {
namespace {

__global__ void qmatmul_int4_generic_kernel(const float* __restrict__ x,
                                            const uint8_t* __restrict__ w,
                                            const __half* __restrict__ s,
                                            const uint8_t* __restrict__ z, float* __restrict__ out,
                                            int k, int n, int gs) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  const int row = blockIdx.y;
  if (col >= n) return;
  const float* xr = x + (size_t)row * k;
  const int shift = (col & 1) * 4;
  const int ng = k / gs;
  float acc = 0.0f;
  for (int g = 0; g < ng; ++g) {
    const float scale = __half2float(s[(size_t)g * n + col]);
    const float fz = (float)((z[(size_t)g * (n / 2) + col / 2] >> shift) & 15);
    for (int i = 0; i < gs; i += 2) {
      const int kk = g * gs + i;
      const uint32_t p = w[(size_t)(kk / 2) * n + col];
      acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(xr[kk], scale), __fsub_rn((float)(p & 15u), fz)));
      acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(xr[kk + 1], scale), __fsub_rn((float)(p >> 4), fz)));
    }
  }
  out[(size_t)row * n + col] = acc;
}

__global__ void dequant_int4_kernel(const uint8_t* __restrict__ w, const __half* __restrict__ s,
                                    const uint8_t* __restrict__ z, float* __restrict__ out, int k,
                                    int n, int gs) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  const int kp = blockIdx.y;  // packed row = k pair
  if (col >= n) return;
  const int kk = 2 * kp;
  const int g = kk / gs;
  const float scale = __half2float(s[(size_t)g * n + col]);
  const float fz = (float)((z[(size_t)g * (n / 2) + col / 2] >> ((col & 1) * 4)) & 15);
  const uint32_t p = w[(size_t)kp * n + col];
  out[(size_t)kk * n + col] = __fmul_rn(scale, __fsub_rn((float)(p & 15u), fz));
  out[(size_t)(kk + 1) * n + col] = __fmul_rn(scale, __fsub_rn((float)(p >> 4), fz));
}

// Block-wide sum, deterministic: warp shuffles then the warps' partials in order.
__device__ float block_sum(float v, float* red) {
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float tot = 0.0f;
  const int nw = blockDim.x >> 5;
  for (int i = 0; i < nw; ++i) tot += red[i];
  __syncthreads();
  return tot;
}

__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                               float* __restrict__ out, int dim, float eps) {
  __shared__ float red[32];
  const size_t off = (size_t)blockIdx.x * dim;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float v = x[off + i];
    ss = fmaf(v, v, ss);
  }
  const float tot = block_sum(ss, red);
  const float rms = rsqrtf(tot / (float)dim + eps);
  for (int i = threadIdx.x; i < dim; i += blockDim.x) out[off + i] = x[off + i] * rms * w[i];
}

// fp32 matvec, W [N][K] row-major (src/kernels/shaders.zig:184-266): out[n] = sum_k W[n][k] x[k].
// One warp per row (the NMAT matrices' rows share the x loads), float4 streams of each row with
// four independent partial sums per lane, a butterfly sum at the end.  x is re-read from L1.
// vec: K % 4 == 0 and 16-byte aligned rows; otherwise scalar loads.
template <int NMAT>
__global__ void __launch_bounds__(256) matvec_f32_kernel(const float* __restrict__ x,
                                                         const float* __restrict__ W0,
                                                         const float* __restrict__ W1,
                                                         float* __restrict__ out0,
                                                         float* __restrict__ out1, int K, int N,
                                                         int vec) {
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  for (int n = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); n < N; n += warps) {
    float acc[NMAT][4];
#pragma unroll
    for (int m = 0; m < NMAT; ++m) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0.f;
    const float* r0 = W0 + (size_t)n * K;
    const float* r1 = NMAT > 1 ? W1 + (size_t)n * K : nullptr;
    if (vec) {
      const float4* x4 = reinterpret_cast<const float4*>(x);
      const float4* a4 = reinterpret_cast<const float4*>(r0);
      const float4* b4 = reinterpret_cast<const float4*>(r1);
      const int K4 = K >> 2;
      int k = lane;
      // four float4 per lane per iteration (2 KB of each row in flight per warp)
      constexpr int U = 4;
      for (; k + 32 * (U - 1) < K4; k += 32 * U) {
        float4 xa[U], wa[U], va[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          xa[u] = __ldg(x4 + k + 32 * u);
          wa[u] = __ldcs(a4 + k + 32 * u);
          if (NMAT > 1) va[u] = __ldcs(b4 + k + 32 * u);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          acc[0][0] = fmaf(wa[u].x, xa[u].x, acc[0][0]);
          acc[0][1] = fmaf(wa[u].y, xa[u].y, acc[0][1]);
          acc[0][2] = fmaf(wa[u].z, xa[u].z, acc[0][2]);
          acc[0][3] = fmaf(wa[u].w, xa[u].w, acc[0][3]);
          if (NMAT > 1) {
            acc[NMAT - 1][0] = fmaf(va[u].x, xa[u].x, acc[NMAT - 1][0]);
            acc[NMAT - 1][1] = fmaf(va[u].y, xa[u].y, acc[NMAT - 1][1]);
            acc[NMAT - 1][2] = fmaf(va[u].z, xa[u].z, acc[NMAT - 1][2]);
            acc[NMAT - 1][3] = fmaf(va[u].w, xa[u].w, acc[NMAT - 1][3]);
          }
        }
      }
      for (; k < K4; k += 32) {
        const float4 xa = __ldg(x4 + k);
        const float4 wa = __ldcs(a4 + k);
        acc[0][0] = fmaf(wa.x, xa.x, acc[0][0]);
        acc[0][1] = fmaf(wa.y, xa.y, acc[0][1]);
        acc[0][2] = fmaf(wa.z, xa.z, acc[0][2]);
        acc[0][3] = fmaf(wa.w, xa.w, acc[0][3]);
        if (NMAT > 1) {
          const float4 v1 = __ldcs(b4 + k);
          acc[NMAT - 1][0] = fmaf(v1.x, xa.x, acc[NMAT - 1][0]);
          acc[NMAT - 1][1] = fmaf(v1.y, xa.y, acc[NMAT - 1][1]);
          acc[NMAT - 1][2] = fmaf(v1.z, xa.z, acc[NMAT - 1][2]);
          acc[NMAT - 1][3] = fmaf(v1.w, xa.w, acc[NMAT - 1][3]);
        }
      }
    } else {
      for (int k = lane; k < K; k += 32) {
        const float xv = __ldg(x + k);
        acc[0][k & 3] = fmaf(r0[k], xv, acc[0][k & 3]);
        if (NMAT > 1) acc[NMAT - 1][k & 3] = fmaf(r1[k], xv, acc[NMAT - 1][k & 3]);
      }
    }
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
      float v = (acc[m][0] + acc[m][1]) + (acc[m][2] + acc[m][3]);
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == 0) (m == 0 ? out0 : out1)[n] = v;
    }
  }
}

// GGUF Q4_0 blocks (f16 d, 16 bytes of nibbles; 32 weights of one output row n) -> the
// qmatmul_int4 layout with group size 32: scale d, zero point 8, codes unchanged, so
// s * (q - z) = d * (q - 8) exactly.  Thread t of a block handles output column n0 + t of one
// 32-k block kb: 16 packed bytes at rows 16kb .. 16kb+15 (128 threads -> 128 contiguous bytes
// per row store).  order 0: weight 2i = low nibble of qs[i], 2i+1 = high nibble (the reference
// loader, src/model/llama.zig:341-353); order 1: weight i = low nibble, i + 16 = high nibble.
__global__ void __launch_bounds__(128) repack_q4_0_kernel(const uint8_t* __restrict__ blocks,
                                                          uint8_t* __restrict__ w,
                                                          uint16_t* __restrict__ s,
                                                          uint8_t* __restrict__ z, int N, int K,
                                                          int order) {
  const int n = blockIdx.x * 128 + threadIdx.x;
  const int kb = blockIdx.y;
  if (n >= N) return;
  const uint8_t* blk = blocks + ((size_t)n * (K / 32) + kb) * 18;
  const uint16_t d = (uint16_t)(blk[0] | (blk[1] << 8));
  uint8_t q[32];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint8_t b = blk[2 + i];
    if (order == 0) {
      q[2 * i] = b & 0xF;
      q[2 * i + 1] = b >> 4;
    } else {
      q[i] = b & 0xF;
      q[i + 16] = b >> 4;
    }
  }
#pragma unroll
  for (int p = 0; p < 16; ++p)
    w[(size_t)(16 * kb + p) * N + n] = (uint8_t)(q[2 * p] | (q[2 * p + 1] << 4));
  s[(size_t)kb * N + n] = d;
  if ((n & 1) == 0) z[(size_t)kb * (N / 2) + n / 2] = 0x88;
}

// ---- paged decode attention (src/kernels/shaders.zig:503-587) -----------------------------
// One CTA per (head, sequence), 8 warps; warp w takes the KV blocks w, w+8, ... of the sequence
// (16 tokens each, through the block table) and keeps its own online softmax (running max, sum
// of exponentials, 4 output dims per lane: d = lane + 32i); the CTA merges the 8 states.
// Layout as the shader: q/o [batch][heads][head_dim], caches [block][heads][16][head_dim].
constexpr int kKvBlock = 16;

__global__ void __launch_bounds__(256) paged_attention_kernel(
    const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
    const int* __restrict__ block_tables, const int* __restrict__ context_lens,
    float* __restrict__ o, int num_heads, int head_dim, int max_blocks, float scale) {
  __shared__ float s_m[8], s_s[8];
  __shared__ float s_acc[8][128];
  const int head = blockIdx.x, b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ctx = min(max(context_lens[b], 0), max_blocks * kKvBlock);  // the table's reach
  const int nblocks = (ctx + kKvBlock - 1) / kKvBlock;
  float qv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int d = lane + 32 * i;
    qv[i] = d < head_dim ? q[((size_t)b * num_heads + head) * head_dim + d] : 0.f;
  }
  float m = -INFINITY, sum = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int blk = warp; blk < nblocks; blk += 8) {
    const int phys = block_tables[(size_t)b * max_blocks + blk];
    const size_t base = ((size_t)phys * num_heads + head) * kKvBlock * head_dim;
    const int ntok = min(kKvBlock, ctx - blk * kKvBlock);
    for (int t0 = 0; t0 < ntok; t0 += 4) {
      float kv[4][4], vv[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int d = lane + 32 * i;
          const bool in = t0 + j < ntok && d < head_dim;
          const size_t off = base + (size_t)(t0 + j) * head_dim + d;
          kv[j][i] = in ? kc[off] : 0.f;
          vv[j][i] = in ? vc[off] : 0.f;
        }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (t0 + j >= ntok) break;
        float sc = qv[0] * kv[j][0] + qv[1] * kv[j][1] + qv[2] * kv[j][2] + qv[3] * kv[j][3];
        for (int off = 16; off > 0; off >>= 1) sc += __shfl_xor_sync(0xffffffffu, sc, off);
        sc *= scale;
        const float nm = fmaxf(m, sc);
        const float f = expf(m - nm), pr = expf(sc - nm);
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i] = acc[i] * f + pr * vv[j][i];
        sum = sum * f + pr;
        m = nm;
      }
    }
  }
  if (lane == 0) {
    s_m[warp] = m;
    s_s[warp] = sum;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (lane + 32 * i < 128) s_acc[warp][lane + 32 * i] = acc[i];
  __syncthreads();
  if (threadIdx.x < head_dim) {
    const int d = threadIdx.x;
    float M = -INFINITY;
    for (int w = 0; w < 8; ++w) M = fmaxf(M, s_m[w]);
    float S = 0.f, A = 0.f;
    if (M != -INFINITY)
      for (int w = 0; w < 8; ++w) {
        const float f = s_m[w] == -INFINITY ? 0.f : expf(s_m[w] - M);
        S += s_s[w] * f;
        A += s_acc[w][d] * f;
      }
    o[((size_t)b * num_heads + head) * head_dim + d] = S > 0.f ? A / S : 0.f;  // empty context: 0
  }
}

// ---- sampler (src/kernels/shaders.zig:826-943) -------------------------------------------
// One CTA of 1024 threads; vocabularies are small next to the weights (128K f32 = 512 KB).
constexpr int kSampleThreads = 1024;

// (value, index) pair that wins: the larger value, the smaller index on ties.
__device__ __forceinline__ void argmax_merge(float& v, unsigned& i, float ov, unsigned oi) {
  if (ov > v || (ov == v && oi < i)) {
    v = ov;
    i = oi;
  }
}

__global__ void __launch_bounds__(kSampleThreads) argmax_kernel(const float* __restrict__ x, int n,
                                                                unsigned* __restrict__ out) {
  __shared__ float sv[32];
  __shared__ unsigned si[32];
  float v = -INFINITY;
  unsigned idx = 0xFFFFFFFFu;
  for (int i = threadIdx.x; i < n; i += blockDim.x) argmax_merge(v, idx, x[i], (unsigned)i);
  for (int off = 16; off > 0; off >>= 1)
    argmax_merge(v, idx, __shfl_xor_sync(0xffffffffu, v, off), __shfl_xor_sync(0xffffffffu, idx, off));
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[w] = v;
    si[w] = idx;
  }
  __syncthreads();
  if (w == 0) {
    v = lane < (int)(blockDim.x >> 5) ? sv[lane] : -INFINITY;
    idx = lane < (int)(blockDim.x >> 5) ? si[lane] : 0xFFFFFFFFu;
    for (int off = 16; off > 0; off >>= 1)
      argmax_merge(v, idx, __shfl_xor_sync(0xffffffffu, v, off), __shfl_xor_sync(0xffffffffu, idx, off));
    if (lane == 0) out[0] = idx == 0xFFFFFFFFu ? 0u : idx;  // all -inf / NaN: index 0
  }
}

// Block-wide reduction of one float (op 0: max, op 1: sum); every thread gets the result.
__device__ __forceinline__ float block_reduce(float v, int op, float* red) {
  for (int off = 16; off > 0; off >>= 1) {
    const float o = __shfl_xor_sync(0xffffffffu, v, off);
    v = op == 0 ? fmaxf(v, o) : v + o;
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  v = lane < nw ? red[lane] : (op == 0 ? -INFINITY : 0.f);
  for (int off = 16; off > 0; off >>= 1) {
    const float o = __shfl_xor_sync(0xffffffffu, v, off);
    v = op == 0 ? fmaxf(v, o) : v + o;
  }
  return v;
}

// probs = softmax(logits / temperature); sampled = the first i whose cumulative probability
// exceeds random_val (vocab - 1 if none).  The cumulative sums are a block scan over contiguous
// per-thread chunks, so the chosen index can differ from a sequential f32 sum only when
// random_val lies within rounding of a boundary.
__global__ void __launch_bounds__(kSampleThreads) softmax_sample_kernel(
    const float* __restrict__ logits, float* __restrict__ probs, unsigned* __restrict__ sampled,
    int n, float temperature, float random_val) {
  __shared__ float red[32];
  __shared__ float scan[kSampleThreads];
  __shared__ unsigned s_pick;
  const float inv_t = 1.0f / temperature;
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < n; i += blockDim.x) mx = fmaxf(mx, logits[i] * inv_t);
  mx = block_reduce(mx, 0, red);
  float sum = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) sum += expf(logits[i] * inv_t - mx);
  sum = block_reduce(sum, 1, red);
  const float inv_sum = 1.0f / sum;
  for (int i = threadIdx.x; i < n; i += blockDim.x) probs[i] = expf(logits[i] * inv_t - mx) * inv_sum;
  __syncthreads();
  // contiguous chunk of this thread, its probability mass, an inclusive block scan
  const int per = (n + blockDim.x - 1) / blockDim.x;
  const int c0 = min(n, (int)threadIdx.x * per), c1 = min(n, c0 + per);
  float part = 0.f;
  for (int i = c0; i < c1; ++i) part += probs[i];
  scan[threadIdx.x] = part;
  if (threadIdx.x == 0) s_pick = (unsigned)(n - 1);
  __syncthreads();
  for (int off = 1; off < (int)blockDim.x; off <<= 1) {
    const float add = threadIdx.x >= (unsigned)off ? scan[threadIdx.x - off] : 0.f;
    __syncthreads();
    scan[threadIdx.x] += add;
    __syncthreads();
  }
  const float before = threadIdx.x ? scan[threadIdx.x - 1] : 0.f;
  if (c0 < c1 && random_val >= before && random_val < scan[threadIdx.x]) {
    float cum = before;
    unsigned pick = (unsigned)(c1 - 1);
    for (int i = c0; i < c1; ++i) {
      cum += probs[i];
      if (random_val < cum) {
        pick = (unsigned)i;
        break;
      }
    }
    atomicMin(&s_pick, pick);
  }
  __syncthreads();
  if (threadIdx.x == 0) sampled[0] = s_pick;
}

// rmsnorm of one row, written as f16 in the GEMM's k order (the activations of the tensor-core
// GEMM).
__global__ void rmsnorm_f16_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                   __half* __restrict__ out, int dim, float eps) {
  __shared__ float red[32];
  const size_t off = (size_t)blockIdx.x * dim;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float v = x[off + i];
    ss = fmaf(v, v, ss);
  }
  const float tot = block_sum(ss, red);
  const float rms = rsqrtf(tot / (float)dim + eps);
  for (int i = threadIdx.x; i < dim; i += blockDim.x)
    out[off + gemm_kperm(i)] = __float2half_rn(x[off + i] * rms * w[i]);
}

__global__ void fused_rmsnorm_rope_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                          const float* __restrict__ cosc,
                                          const float* __restrict__ sinc, float* __restrict__ out,
                                          int dim, int head_dim, int pos, float eps) {
  __shared__ float red[32];
  const size_t off = (size_t)blockIdx.x * dim;
  const int half_head = head_dim / 2;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float v = x[off + i];
    ss = fmaf(v, v, ss);
  }
  const float tot = block_sum(ss, red);
  const float rms = rsqrtf(tot / (float)dim + eps);
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float normed = x[off + i] * rms * w[i];
    const int ph = i % head_dim;
    if (ph < half_head) {
      const float pair = x[off + i + half_head] * rms * w[i + half_head];
      const float c = cosc[(size_t)pos * half_head + ph];
      const float s = sinc[(size_t)pos * half_head + ph];
      out[off + i] = normed * c - pair * s;
    } else {
      const float pair = x[off + i - half_head] * rms * w[i - half_head];
      const int fi = ph - half_head;
      const float c = cosc[(size_t)pos * half_head + fi];
      const float s = sinc[(size_t)pos * half_head + fi];
      out[off + i] = normed * c + pair * s;
    }
  }
}

__global__ void silu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u,
                                float* __restrict__ out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float gv = g[i];
  out[i] = gv / (1.0f + expf(-gv)) * u[i];
}

__global__ void add_kernel(const float* __restrict__ a, const float* __restrict__ b,
                           float* __restrict__ out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  out[i] = a[i] + b[i];
}

// x as f16 in the GEMM's k order (rows of a multiple of 4 elements).
__global__ void f32_to_f16_kernel(const float* __restrict__ x, __half* __restrict__ y, long long n) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[gemm_kperm(i)] = __float2half_rn(x[i]);
}

// y[m][n] = sum over splits (in split order) of part[split][m][n] (+ residual[m][n])
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int splits, long long mn,
                                     const float* __restrict__ residual, float* __restrict__ y) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= mn) return;
  float a = 0.f;
  for (int s = 0; s < splits; ++s) a += part[(long long)s * mn + i];
  y[i] = residual ? residual[i] + a : a;
}

}  // namespace

cudaError_t launch_f32_to_f16(const float* x, __half* y, long long n, cudaStream_t st) {
  f32_to_f16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(x, y, n);
  return cudaGetLastError();
}

cudaError_t launch_splitk_reduce(const float* part, int splits, long long mn, const float* residual,
                                 float* y, cudaStream_t st) {
  splitk_reduce_kernel<<<(unsigned)((mn + 255) / 256), 256, 0, st>>>(part, splits, mn, residual, y);
  return cudaGetLastError();
}

cudaError_t launch_qmatmul_int4_generic(const float* x, const uint8_t* w, const uint16_t* s,
                                        const uint8_t* z, float* out, int m, int k, int n,
                                        int gs, cudaStream_t st) {
  dim3 grid((n + 127) / 128, m);
  qmatmul_int4_generic_kernel<<<grid, 128, 0, st>>>(x, w, reinterpret_cast<const __half*>(s), z,
                                                    out, k, n, gs);
  return cudaGetLastError();
}

cudaError_t launch_dequant_int4(const uint8_t* w, const uint16_t* s, const uint8_t* z,
                                float* out, int k, int n, int gs, cudaStream_t st) {
  dim3 grid((n + 127) / 128, k / 2);
  dequant_int4_kernel<<<grid, 128, 0, st>>>(w, reinterpret_cast<const __half*>(s), z, out, k, n,
                                            gs);
  return cudaGetLastError();
}

cudaError_t launch_rmsnorm(const float* x, const float* w, float* out, int rows, int dim,
                           float eps, cudaStream_t st) {
  rmsnorm_kernel<<<rows, 256, 0, st>>>(x, w, out, dim, eps);
  return cudaGetLastError();
}

cudaError_t launch_matvec_f32(const float* x, const float* W0, const float* W1, float* out0,
                              float* out1, int K, int N, int sm_count, cudaStream_t st) {
  const int vec = (K % 4 == 0) && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(W0) |
                                    reinterpret_cast<uintptr_t>(W1)) % 16 == 0);
  // 8 warps (rows) per block; enough blocks to cover the SMs a few times, rows strided
  const int blocks = std::max(1, std::min((N + 7) / 8, sm_count * 8));
  if (W1)
    matvec_f32_kernel<2><<<blocks, 256, 0, st>>>(x, W0, W1, out0, out1, K, N, vec);
  else
    matvec_f32_kernel<1><<<blocks, 256, 0, st>>>(x, W0, nullptr, out0, nullptr, K, N, vec);
  return cudaGetLastError();
}

cudaError_t launch_repack_q4_0(const uint8_t* blocks, uint8_t* w, uint16_t* s, uint8_t* z, int N,
                               int K, int order, cudaStream_t st) {
  const dim3 grid((unsigned)((N + 127) / 128), (unsigned)(K / 32));
  repack_q4_0_kernel<<<grid, 128, 0, st>>>(blocks, w, s, z, N, K, order);
  return cudaGetLastError();
}

cudaError_t launch_paged_attention(const float* q, const float* kc, const float* vc,
                                   const int* block_tables, const int* context_lens, float* o,
                                   int batch, int num_heads, int head_dim, int max_blocks,
                                   float scale, cudaStream_t st) {
  paged_attention_kernel<<<dim3((unsigned)num_heads, (unsigned)batch), 256, 0, st>>>(
      q, kc, vc, block_tables, context_lens, o, num_heads, head_dim, max_blocks, scale);
  return cudaGetLastError();
}

cudaError_t launch_argmax(const float* x, int n, unsigned* out, cudaStream_t st) {
  argmax_kernel<<<1, kSampleThreads, 0, st>>>(x, n, out);
  return cudaGetLastError();
}

cudaError_t launch_softmax_sample(const float* logits, float* probs, unsigned* sampled, int n,
                                  float temperature, float random_val, cudaStream_t st) {
  softmax_sample_kernel<<<1, kSampleThreads, 0, st>>>(logits, probs, sampled, n, temperature,
                                                      random_val);
  return cudaGetLastError();
}

cudaError_t launch_rmsnorm_f16(const float* x, const float* w, __half* out, int rows, int dim,
                               float eps, cudaStream_t st) {
  rmsnorm_f16_kernel<<<rows, 512, 0, st>>>(x, w, out, dim, eps);
  return cudaGetLastError();
}

cudaError_t launch_fused_rmsnorm_rope(const float* x, const float* w, const float* cosc,
                                      const float* sinc, float* out, int rows, int dim,
                                      int head_dim, int pos, float eps, cudaStream_t st) {
  fused_rmsnorm_rope_kernel<<<rows, 256, 0, st>>>(x, w, cosc, sinc, out, dim, head_dim, pos, eps);
  return cudaGetLastError();
}

cudaError_t launch_silu_mul(const float* g, const float* u, float* out, int n, cudaStream_t st) {
  silu_mul_kernel<<<(n + 255) / 256, 256, 0, st>>>(g, u, out, n);
  return cudaGetLastError();
}

cudaError_t launch_add(const float* a, const float* b, float* out, int n, cudaStream_t st) {
  add_kernel<<<(n + 255) / 256, 256, 0, st>>>(a, b, out, n);
  return cudaGetLastError();
}

}  // namespace tk
