// tk_internal.h -- declarations shared by the translation units of libtkcuda.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include <cuda_fp16.h>

#include "tk_engine.h"
#include "tk_gemm.h"

namespace tk {

// tk_runtime.cu -- generation of the per-device kernel attribute caches (dynamic shared memory,
// occupancy): tk_device_create bumps it for its device, so an attribute set in an earlier CUDA
// context of the device (before a cudaDeviceReset) is set again on the next launch.
unsigned attr_generation(int dev);
void bump_attr_generation(int dev);

// tk_engine.cu
int engine_warps_per_cta();
size_t engine_smem_bytes(int stages, int tile_stage_bytes, int aux_stage_bytes, int rec0_bytes);
// Picks the deepest ring (up to kMaxStages) that fits a smem budget, with the prologue records
// in shared memory when they fit beside it.  Returns false when not even 2 stages fit.
bool engine_plan_smem(int tile_stage_bytes, int aux_stage_bytes, int rec0_bytes, int smem_limit,
                      int* stages, int* rec0_smem, size_t* smem);
// The kernel is instantiated per tokens (mt in {1, 2, 4}) and group size (16, 32, 64, 128).
cudaError_t engine_occupancy(int mt, int gs, size_t smem, int* blocks);
cudaError_t engine_launch(int mt, int gs, const TmapPack& maps, const EngineParams& p, int grid,
                          size_t smem, cudaStream_t stream);

// tk_simple.cu -- CUDA-core kernels: reference-order fallbacks and the small ops.
cudaError_t launch_qmatmul_int4_generic(const float* x, const uint8_t* w, const uint16_t* s,
                                        const uint8_t* z, float* out, int m, int k, int n,
                                        int gs, cudaStream_t st);
cudaError_t launch_dequant_int4(const uint8_t* w, const uint16_t* s, const uint8_t* z,
                                float* out, int k, int n, int gs, cudaStream_t st);
cudaError_t launch_rmsnorm(const float* x, const float* w, float* out, int rows, int dim,
                           float eps, cudaStream_t st);
cudaError_t launch_fused_rmsnorm_rope(const float* x, const float* w, const float* cosc,
                                      const float* sinc, float* out, int rows, int dim,
                                      int head_dim, int pos, float eps, cudaStream_t st);
cudaError_t launch_silu_mul(const float* g, const float* u, float* out, int n, cudaStream_t st);
cudaError_t launch_add(const float* a, const float* b, float* out, int n, cudaStream_t st);
cudaError_t launch_f32_to_f16(const float* x, __half* y, long long n, cudaStream_t st);
cudaError_t launch_matvec_f32(const float* x, const float* W0, const float* W1, float* out0,
                              float* out1, int K, int N, int sm_count, cudaStream_t st);
// One-shot peer-memory all-reduce (tk_allreduce.cu).
constexpr int kP2PMaxRanks = 8;
constexpr int kP2PMaxChunks = 512;
constexpr int kP2PChunkFloats = 512;
constexpr size_t kP2PMaxFloats = (size_t)kP2PMaxChunks * kP2PChunkFloats;  // 1 MB of f32
constexpr unsigned kErrP2PWait = 8u;
struct P2PParams {
  float* buf;                       // the local vector, summed in place
  int count, chunk, nranks, rank;
  size_t slot_floats;               // floats per receive slot (one rank, one parity)
  float* recv[kP2PMaxRanks];        // rank r's receive area, mapped here: [2][nranks][slot]
  unsigned* flags[kP2PMaxRanks];    // rank r's flags, mapped here: [nranks][kP2PMaxChunks]
  unsigned* counters;               // local epoch per chunk [kP2PMaxChunks]
  unsigned* err;
  unsigned long long timeout_ns;
};
cudaError_t launch_p2p_allreduce(const P2PParams& p, cudaStream_t st);
cudaError_t launch_repack_q4_0(const uint8_t* blocks, uint8_t* w, uint16_t* s, uint8_t* z, int N,
                               int K, int order, cudaStream_t st);
cudaError_t launch_paged_attention(const float* q, const float* kc, const float* vc,
                                   const int* block_tables, const int* context_lens, float* o,
                                   int batch, int num_heads, int head_dim, int max_blocks,
                                   float scale, cudaStream_t st);
cudaError_t launch_argmax(const float* x, int n, unsigned* out, cudaStream_t st);
cudaError_t launch_softmax_sample(const float* logits, float* probs, unsigned* sampled, int n,
                                  float temperature, float random_val, cudaStream_t st);
cudaError_t launch_rmsnorm_f16(const float* x, const float* w, __half* out, int rows, int dim,
                               float eps, cudaStream_t st);
cudaError_t launch_splitk_reduce(const float* part, int splits, long long mn, const float* residual,
                                 float* y, cudaStream_t st);

// tk_gemm.cu -- batch >= 5 GEMM (tcgen05); nt = token tile in {16, 32, 64, 128, 256}
cudaError_t gemm_launch(int nt, const GemmMaps& maps, const GemmParams& p, dim3 grid, size_t smem,
                        cudaStream_t st);

}  // namespace tk
