// tk_allreduce.cu -- one-shot all-reduce (sum, f32) over NVLink peer memory for the tensor-parallel
// FFN's exchange step (the [M][hidden] partial outputs: 16 KB at batch 1).
//
// Every rank maps every peer's receive area (CUDA IPC).  CTA c owns chunk c of the vector:
//   1. reads its chunk's epoch counter e (local, advanced by this CTA once per call, so a CUDA
//      graph replays correctly without any host-side state) and uses buffer parity e & 1;
//   2. stores its chunk of the local vector into every rank's receive slot [parity][my rank]
//      (peer stores over NVLink; its own slot too), then -- after a system-scope fence -- writes e
//      into every rank's flag [my rank][c] with release semantics;
//   3. waits (bounded) until its own flags [p][c] >= e for every rank p, then sums the ranks'
//      slots in rank order (every rank gets bit-identical sums) into the local vector.
// A rank can run at most one epoch ahead of another on a chunk (it needs the slower rank's flag
// of the previous epoch), so two parities suffice.  No TMA and no multicast.
#include <cuda_runtime.h>

#include <cstdint>

#include "tk_internal.h"

namespace tk {

namespace {

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long p2p_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__global__ void __launch_bounds__(256) p2p_allreduce_kernel(const P2PParams p) {
  __shared__ unsigned s_e;
  __shared__ int s_ok;
  const int c = blockIdx.x;
  const int off = c * p.chunk;
  const int len = min(p.chunk, p.count - off);
  if (threadIdx.x == 0) {
    s_e = p.counters[c] + 1u;
    s_ok = 1;
  }
  __syncthreads();
  const unsigned e = s_e;
  const size_t par = e & 1u;
  const float* src = p.buf + off;
  const bool vec = ((p.count | p.chunk) & 3) == 0 && (reinterpret_cast<uintptr_t>(p.buf) & 15) == 0;
  // 2. push this chunk to every rank's slot [par][rank]
  for (int r = 0; r < p.nranks; ++r) {
    float* dst = p.recv[r] + (par * p.nranks + p.rank) * p.slot_floats + off;
    if (vec) {
      for (int i = threadIdx.x * 4; i < len; i += blockDim.x * 4)
        *reinterpret_cast<float4*>(dst + i) = *reinterpret_cast<const float4*>(src + i);
    } else {
      for (int i = threadIdx.x; i < len; i += blockDim.x) dst[i] = src[i];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int r = 0; r < p.nranks; ++r) st_release_sys(p.flags[r] + p.rank * kP2PMaxChunks + c, e);
    // 3. wait for every rank's chunk
    const unsigned long long t0 = p2p_timer_ns();
    for (int r = 0; r < p.nranks && s_ok; ++r) {
      const unsigned* f = p.flags[p.rank] + r * kP2PMaxChunks + c;
      while ((int)(ld_acquire_sys(f) - e) < 0) {
        if (p2p_timer_ns() - t0 > p.timeout_ns) {
          atomicOr(p.err, kErrP2PWait);
          s_ok = 0;
          break;
        }
      }
    }
    __threadfence();
  }
  __syncthreads();
  if (!s_ok) return;  // the error word reports it; the vector is left as it was
  const float* base = p.recv[p.rank] + par * p.nranks * p.slot_floats + off;
  float* out = p.buf + off;
  for (int i = threadIdx.x; i < len; i += blockDim.x) {
    float v = base[i];
    for (int r = 1; r < p.nranks; ++r) v += base[(size_t)r * p.slot_floats + i];
    out[i] = v;
  }
  if (threadIdx.x == 0) p.counters[c] = e;
}

}  // namespace

cudaError_t launch_p2p_allreduce(const P2PParams& p, cudaStream_t st) {
  const int nchunks = (p.count + p.chunk - 1) / p.chunk;
  p2p_allreduce_kernel<<<nchunks, 256, 0, st>>>(p);
  return cudaGetLastError();
}

}  // namespace tk
