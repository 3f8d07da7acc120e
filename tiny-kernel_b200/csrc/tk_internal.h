// tk_internal.h -- declarations shared by the translation units of libtkcuda.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "tk_engine.h"

namespace tk {

// tk_engine.cu
int engine_warps_per_cta();
size_t engine_smem_bytes(int stages, int tile_stage_bytes, int aux_stage_bytes, int rec0_bytes);
// Picks the ring depth and where phase-0 records live for a smem budget: records in shared
// memory with >= 4 stages when they fit, else records in global memory with up to 5 stages.
// Returns false when not even 2 stages fit.
bool engine_plan_smem(int tile_stage_bytes, int aux_stage_bytes, int rec0_bytes, int smem_limit,
                      int* stages, int* rec0_smem, size_t* smem);
cudaError_t engine_occupancy(int mt, size_t smem, int* blocks);
cudaError_t engine_launch(int mt, const TmapPack& maps, const EngineParams& p, int grid,
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

}  // namespace tk
