/*
 * tk_cuda.h -- C ABI of the B200 (sm_100a) INT4 GEMV / INT4 Llama-FFN path.
 *
 * This header is the drop-in boundary that replaces the Metal runtime under the
 * reference's Zig kernel API (Lulzx/tiny-kernel):
 *
 *   reference (Zig + Metal)                         this ABI
 *   ---------------------------------------------   ----------------------------------
 *   src/main.zig:17-23        tk.init / tk.deinit   tk_device_create / tk_device_destroy
 *   src/metal/device.zig:42-45  Device.name         tk_device_name
 *   src/metal/device.zig:85-91  Device.createBuffer tk_buffer_alloc / tk_buffer_free
 *   src/metal/device.zig:123-133 Buffer.slice       tk_buffer_upload / tk_buffer_download
 *   src/kernels/quantized.zig:15-50 QMatMulInt4     tk_qmatmul_int4(_async)
 *   src/kernels/rmsnorm.zig:15-42   RMSNorm         tk_rmsnorm(_async)
 *   src/kernels/fused.zig:15-50     FusedRMSNormRoPE tk_fused_rmsnorm_rope(_async)
 *   src/kernels/fused.zig:187-212   FusedSiluMul    tk_silu_mul(_async)
 *   src/bench.zig:266-341  INT4 FFN composition     tk_int4_ffn(_async)   (adds the down projection)
 *
 * Conventions
 *  - Every entry point returns TK_OK (0) or a negative TK_ERR_* status; the text of
 *    the last failure on the calling thread is available from tk_last_error_string().
 *  - All tensor pointers are DEVICE pointers (from tk_buffer_alloc or any CUDA
 *    allocation) unless a function says otherwise.  Buffers are owned by the caller,
 *    as Buffer(T) is in the reference (bench.zig:225-240, `defer x.deinit()`).
 *  - The plain entry points are synchronous, like the reference's forward()
 *    (commit + waitUntilCompleted, quantized.zig:47-49): outputs are ready on return.
 *    The *_async variants enqueue on the given CUDA stream (NULL = the device's
 *    stream) and return immediately.
 *  - f16 scales are passed as raw IEEE binary16 bit patterns (uint16_t).
 *  - The library caches per-device state for the life of the process (kernel attributes, the
 *    allocation-free entry point's scratch address): cudaDeviceReset while it is loaded is not
 *    supported.
 *
 * Environment (read once, at tk_device_create; for tuning and tests, none is needed):
 *   TK_WAIT_TIMEOUT_MS  bound of every device-side wait (default 2000); a wait that runs out
 *                       reports TK_ERR_TIMEOUT
 *   TK_GEMM=0           route every batch through the streaming engine (no tcgen05 GEMM)
 *   TK_ENGINE_CTAS      CTAs of the streaming engine's launches (default: one per SM; smaller
 *                       FFN shards take a divisor of their work, see tk_int4_ffn)
 *   TK_ENGINE_STAGES    cap on the engine's shared-memory ring depth (default: deepest fit)
 *   TK_FFN_SPLIT        gate/up tile ranges of the engine's FFN, 1..4 (default 1)
 *   TK_DOWN_PREFETCH=0  no L2 prefetch of the down projection at the gate/up -> down switch
 *   TK_DECODE=0         1-2 rows run the streaming engine instead of the decode kernel
 *   TK_DECODE_PDL=0     the decode kernel is a cooperative launch that starts only after the
 *                       preceding kernel of its stream has finished (default: a programmatic
 *                       dependent launch whose CTAs are set up, and prefetch their first weights
 *                       into L2, while that kernel finishes; the kernel still reads nothing the
 *                       preceding kernel may write before it has completed)
 *   TK_TP_NCCL=1        tk_tp groups use NCCL for every exchange (read at tk_tp_create)
 *   TK_TP_FUSED=0       tk_tp groups do not fuse the batch 1-2 FFN's exchange into the decode
 *                       kernel (read at tk_tp_create)
 *   TK_NCCL_LIB         path of the libnccl.so.2 the tk_tp_* calls load
 *
 * INT4 weight layout (identical to qmatmul_int4, src/kernels/shaders.zig:442-501):
 *   w_packed u8 [K/2][N]          byte (k/2)*N + n; even k = low nibble, odd k = high nibble
 *   scales   f16 [K/group][N]     index g*N + n
 *   zeros    u8 [K/group][N/2]    byte g*(N/2) + n/2; even n = low nibble, odd n = high nibble
 *   y[m][n] = sum_k x[m][k] * scale[g][n] * (q[k][n] - zero[g][n]),   g = k / group
 */
#ifndef TK_CUDA_H
#define TK_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TK_ABI_VERSION 1

/* status codes */
#define TK_OK 0
#define TK_ERR_ARG (-1)         /* bad shape, null pointer, misaligned pointer   */
#define TK_ERR_CUDA (-2)        /* a CUDA runtime / driver call failed            */
#define TK_ERR_NCCL (-3)        /* a NCCL call failed                              */
#define TK_ERR_TIMEOUT (-4)     /* a bounded device-side wait gave up              */
#define TK_ERR_UNSUPPORTED (-5) /* shape or feature not supported on this build    */
#define TK_ERR_NOMEM (-6)       /* device or host allocation failed                */

/* buffer kinds for tk_buffer_alloc */
#define TK_MEM_DEVICE 0 /* cudaMalloc: device-resident HBM                          */
#define TK_MEM_SHARED 1 /* cudaMallocManaged: host-visible like MTLStorageModeShared */
#define TK_MEM_HOST 2   /* cudaMallocHost: pinned host memory (staging for copies)  */

/* flags for tk_int4_ffn */
#define TK_FFN_RESIDUAL 1u /* out = x + FFN(x)  (Llama residual, llama.zig:216-231)  */
/* x and out are pinned host memory (TK_MEM_HOST, cudaMallocHost or cudaHostRegister'd; h_out,
 * when given, stays device memory).  At 1-2 rows the decode kernel reads x and writes out over
 * the host link itself (x is read once per call: each CTA reads a share and passes it on to the
 * others through device scratch); other batches copy x in and out through device scratch on the
 * call's stream.  The synchronous tk_int4_ffn records such a call as a CUDA graph (the kernel
 * node, which reports a failure straight to a pinned host word, or copy in, kernels, copy out and
 * the error word's read-back) and replays it when it is called again with the same arguments: one
 * launch and one wait per call.  The recorded graphs (up to 64 per device, least
 * recently used replaced) are dropped when the device's scratch grows; synchronous calls on one
 * device from several threads at once are not supported (the reference is single-threaded,
 * src/metal/device.zig:7).  The reference's buffers are host-visible shared memory
 * (StorageModeShared, src/metal/device.zig:109), which is the use this flag serves. */
#define TK_FFN_HOST_IO 2u

typedef struct tk_device tk_device;

/* One INT4 matrix in the qmatmul_int4 layout above (K and N given by the call). */
typedef struct tk_int4_matrix {
  const uint8_t *w_packed;  /* [K/2][N]       */
  const uint16_t *scales;   /* [K/group][N]   */
  const uint8_t *zeros;     /* [K/group][N/2] */
} tk_int4_matrix;

/* ---- device ---------------------------------------------------------------------- */

/* Replaces tk.init() / Device.init (src/main.zig:17-19, src/metal/device.zig:10-29):
 * selects CUDA device `ordinal`, creates its stream and the scratch the kernels use. */
int tk_device_create(int ordinal, tk_device **out);
/* Replaces tk.deinit() / Device.deinit (src/main.zig:21-23, device.zig:31-40). */
void tk_device_destroy(tk_device *dev);
/* Replaces Device.name (src/metal/device.zig:42-45). Valid until destroy. */
const char *tk_device_name(tk_device *dev);
/* Number of SMs the persistent kernels size their grid to. */
int tk_device_sm_count(tk_device *dev);
/* Kernels enqueued through this device so far (every launch of every entry point, also
 * those recorded into a CUDA graph). No counterpart in the reference. */
uint64_t tk_device_launch_count(tk_device *dev);
/* The device's CUDA stream (cudaStream_t) used by the synchronous entry points. */
void *tk_device_stream(tk_device *dev);
/* Waits for all work queued on the device's stream; returns any deferred kernel error. */
int tk_device_synchronize(tk_device *dev);
/* Reads and clears the device-side error word that bounded waits set (TK_ERR_TIMEOUT). */
int tk_device_check_error(tk_device *dev);

const char *tk_last_error_string(void);
const char *tk_status_string(int status);
int tk_abi_version(void);

/* ---- buffers (Device.createBuffer / Buffer(T), src/metal/device.zig:85-135) ------- */

int tk_buffer_alloc(tk_device *dev, size_t bytes, int kind, void **ptr);
int tk_buffer_free(tk_device *dev, void *ptr);
/* Synchronous host<->device copies on the device's stream. */
int tk_buffer_upload(tk_device *dev, void *dst_device, const void *src_host, size_t bytes);
int tk_buffer_download(tk_device *dev, void *dst_host, const void *src_device, size_t bytes);
/* The same copies queued on `stream` (NULL: the device's stream) without waiting, so a step can
 * queue its upload, its kernels and its download and wait once (tk_device_synchronize): the
 * reference encodes a step into one command buffer, commits it and waits once
 * (CommandBuffer.commit / waitUntilCompleted, src/metal/device.zig:137-153).
 * The host memory must stay valid until the copy has run; with pageable host memory the copy
 * may be partly synchronous, with pinned memory (TK_MEM_HOST) it is not. */
int tk_buffer_upload_async(tk_device *dev, void *dst_device, const void *src_host, size_t bytes,
                           void *stream);
int tk_buffer_download_async(tk_device *dev, void *dst_host, const void *src_device, size_t bytes,
                             void *stream);

/* ---- kernels --------------------------------------------------------------------- */

/* QMatMulInt4.forward (src/kernels/quantized.zig:15-50; kernel shaders.zig:442-501).
 * x f32 [m][k], out f32 [m][n].  The reference computes row 0 only and requires
 * k <= 4096; this entry point computes all m rows and any k with k % group_size == 0,
 * group_size % 8 == 0, n even.  Shapes with n % 128 == 0, k % 128 == 0 and
 * group_size in {16, 32, 64, 128} (16-byte aligned pointers) run TMA-fed kernels: at 1-4 rows
 * the decode kernel (one persistent launch, dp2a on the CUDA cores against activations
 * quantised to int16 per group), from 5 rows the tcgen05 dequant-to-f16 GEMM; shapes either
 * does not take run the streaming engine in chunks of 4 rows (int8 tensor-core MMAs, mma.sync,
 * against int8 hi/lo activation parts; tk_qmatmul_int4_path); other legal shapes run a plain
 * CUDA-core kernel. */
int tk_qmatmul_int4(tk_device *dev, const float *x, const uint8_t *w_packed,
                    const uint16_t *scales, const uint8_t *zeros, float *out, uint32_t m,
                    uint32_t k, uint32_t n, uint32_t group_size);
int tk_qmatmul_int4_async(tk_device *dev, const float *x, const uint8_t *w_packed,
                          const uint16_t *scales, const uint8_t *zeros, float *out,
                          uint32_t m, uint32_t k, uint32_t n, uint32_t group_size,
                          void *stream);

/* RMSNorm.forward (src/kernels/rmsnorm.zig:15-42; kernel shaders.zig:16-56).
 * out[r][i] = x[r][i] * rsqrt(mean_i(x[r]^2) + eps) * weight[i] for r < rows.
 * The reference derives rows from x.count / dim (rmsnorm.zig:33). */
int tk_rmsnorm(tk_device *dev, const float *x, const float *weight, float *out,
               uint32_t rows, uint32_t dim, float eps);
int tk_rmsnorm_async(tk_device *dev, const float *x, const float *weight, float *out,
                     uint32_t rows, uint32_t dim, float eps, void *stream);

/* FusedRMSNormRoPE.forward (src/kernels/fused.zig:15-50; kernel shaders.zig:124-182).
 * rmsnorm, then rotate-half RoPE per head_dim chunk with cos/sin[pos*head_dim/2 + j]. */
int tk_fused_rmsnorm_rope(tk_device *dev, const float *x, const float *weight,
                          const float *cos_cache, const float *sin_cache, float *out,
                          uint32_t rows, uint32_t dim, uint32_t head_dim, uint32_t pos,
                          float eps);
int tk_fused_rmsnorm_rope_async(tk_device *dev, const float *x, const float *weight,
                                const float *cos_cache, const float *sin_cache, float *out,
                                uint32_t rows, uint32_t dim, uint32_t head_dim,
                                uint32_t pos, float eps, void *stream);

/* FusedSiluMul.forward (src/kernels/fused.zig:187-212; kernel shaders.zig:344-357).
 * out[i] = gate[i] / (1 + exp(-gate[i])) * up[i] for i < n (n = gate.count). */
int tk_silu_mul(tk_device *dev, const float *gate, const float *up, float *out, uint32_t n);
int tk_silu_mul_async(tk_device *dev, const float *gate, const float *up, float *out,
                      uint32_t n, void *stream);

/* INT4 Llama FFN (the reference composes gate/up in src/bench.zig:266-341; the down
 * projection and residual follow src/model/llama.zig:220-231):
 *   h   = silu(gate(rmsnorm(x))) * up(rmsnorm(x))      [m][inter]
 *   out = down(h)            (+ x when flags & TK_FFN_RESIDUAL)   [m][hidden]
 * gate/up: K = hidden, N = inter.  down: K = inter, N = hidden.  eps as in RMSNorm.
 * h_out (optional, may be NULL) receives the f32 intermediate.
 * Fast path: hidden % 128 == 0, inter % 128 == 0, group_size in {16,32,64,128}. */
int tk_int4_ffn(tk_device *dev, const float *x, const float *norm_weight,
                const tk_int4_matrix *gate, const tk_int4_matrix *up,
                const tk_int4_matrix *down, float *out, float *h_out, uint32_t m,
                uint32_t hidden, uint32_t inter, uint32_t group_size, float eps,
                uint32_t flags);
int tk_int4_ffn_async(tk_device *dev, const float *x, const float *norm_weight,
                      const tk_int4_matrix *gate, const tk_int4_matrix *up,
                      const tk_int4_matrix *down, float *out, float *h_out, uint32_t m,
                      uint32_t hidden, uint32_t inter, uint32_t group_size, float eps,
                      uint32_t flags, void *stream);

/* ---- tensor parallelism -------------------------------------------------------------
 * The additive tensor-parallel FFN (no counterpart in the reference, which runs on one Apple GPU).
 * One process (or thread) per GPU.  Rank r holds the shard: gate/up columns and down K-rows
 * [r*I/tp, (r+1)*I/tp) of the full FFN (inter_shard = I/tp); x, the norm weight and out are full
 * size on every rank.  tk_int4_ffn_tp computes the shard's partial output and sums it across
 * the ranks in place, on the device's stream or the given one (tk_int4_ffn_tp_exchange says
 * how).  At 1-2 rows on a group whose ranks mapped one another's memory, the exchange is fused
 * into the decode kernel: each reduction task stores its columns' partial sums into every
 * rank's area over NVLink and sums the ranks' values in rank order, in the same launch (every
 * rank gets the same bits; TK_ERR_ARG unless x, the norm weight, out and the matrices are 16-byte
 * aligned); TK_TP_FUSED=0 in the environment at tk_tp_create turns this off.  Otherwise the
 * shard's FFN is followed by tk_tp_allreduce_sum_f32.  With TK_FFN_RESIDUAL the residual is added
 * once: after the sum (fused) or by rank 0 before it.  NCCL (libnccl.so.2) is loaded at the
 * first tk_tp_* call; TK_ERR_NCCL when it is missing or a NCCL call fails.  Every rank must make
 * the same tk_tp_* calls in the same order. */
#define TK_TP_UNIQUE_ID_BYTES 128
typedef struct tk_tp tk_tp;
/* Rank 0 creates the group's id and hands it to the other ranks (any channel). */
int tk_tp_unique_id(uint8_t id[TK_TP_UNIQUE_ID_BYTES]);
/* Joins the group (blocks until all nranks have joined). */
int tk_tp_create(tk_device *dev, int nranks, int rank, const uint8_t id[TK_TP_UNIQUE_ID_BYTES],
                 tk_tp **out);
void tk_tp_destroy(tk_tp *tp);
int tk_int4_ffn_tp(tk_tp *tp, const float *x, const float *norm_weight,
                   const tk_int4_matrix *gate, const tk_int4_matrix *up,
                   const tk_int4_matrix *down, float *out, uint32_t m, uint32_t hidden,
                   uint32_t inter_shard, uint32_t group_size, float eps, uint32_t flags);
int tk_int4_ffn_tp_async(tk_tp *tp, const float *x, const float *norm_weight,
                         const tk_int4_matrix *gate, const tk_int4_matrix *up,
                         const tk_int4_matrix *down, float *out, uint32_t m, uint32_t hidden,
                         uint32_t inter_shard, uint32_t group_size, float eps, uint32_t flags,
                         void *stream);
/* In-place sum of an f32 device buffer across the group (the FFN's exchange step).  Up to
 * 262144 floats it is a one-shot all-reduce over NVLink peer memory (the ranks map one another's
 * receive areas at tk_tp_create; sums in rank order, so every rank gets the same bits; bounded
 * waits report TK_ERR_TIMEOUT through tk_device_check_error); larger buffers, or groups where a
 * rank could not map its peers, or TK_TP_NCCL=1 in the environment, use NCCL.  Once a peer wait
 * of the device has run out (reported by tk_device_check_error or a synchronous call), a group
 * using peer memory refuses further exchanges with TK_ERR_TIMEOUT: its ranks' chunk epochs are
 * out of step, so it must be destroyed and created again. */
int tk_tp_allreduce_sum_f32(tk_tp *tp, float *buf, size_t count, void *stream);
/* 1 when the group uses the peer-memory all-reduce, 0 when NCCL carries every exchange. */
int tk_tp_uses_p2p(tk_tp *tp);
/* The exchange tk_int4_ffn_tp uses for this shape: 2 fused into the decode kernel, 1 the
 * peer-memory all-reduce kernel, 0 NCCL (or nothing to exchange, one rank). */
int tk_int4_ffn_tp_exchange(tk_tp *tp, uint32_t m, uint32_t hidden, uint32_t inter_shard,
                            uint32_t group_size);

/* ---- fp32 matvec ---------------------------------------------------------------------
 * Replaces Matvec.forward(x, W, out, K, N) (src/kernels/fused.zig:62-89, shaders.zig:184-226):
 * out[n] = sum_k W[n*K + k] * x[k], W f32 row-major [N][K] (out_dim, in_dim).  Generalised: any
 * K (the shader stages x in a 4096-float threadgroup array).  fp32 accumulation in a different
 * order than the shader's sequential one. */
int tk_matvec(tk_device *dev, const float *x, const float *W, float *out, uint32_t K, uint32_t N);
int tk_matvec_async(tk_device *dev, const float *x, const float *W, float *out, uint32_t K,
                    uint32_t N, void *stream);
/* Replaces MatvecDual.forward(x, W1, W2, out1, out2, K, N) (fused.zig:102-133,
 * shaders.zig:228-266): two matvecs sharing x, one pass. */
int tk_matvec_dual(tk_device *dev, const float *x, const float *W1, const float *W2,
                   float *out1, float *out2, uint32_t K, uint32_t N);
int tk_matvec_dual_async(tk_device *dev, const float *x, const float *W1, const float *W2,
                         float *out1, float *out2, uint32_t K, uint32_t N, void *stream);

/* ---- GGUF Q4_0 -> qmatmul_int4 layout ---------------------------------------------------
 * The on-disk format on the path's input side (src/model/gguf.zig, src/model/llama.zig:341-353,
 * where the reference decodes Q4_0 to f32 instead).  blocks: n_rows x (k/32) Q4_0 blocks of 18
 * bytes (f16 d, 16 bytes of nibbles), row n = output feature n (the f32 Matvec's [N][K]).  Writes
 * w_packed [k/2][n_rows], scales [k/32][n_rows] (= d), zeros [k/32][n_rows/2] (= 8): a matrix for
 * tk_qmatmul_int4 with group_size 32 whose dequantised weights equal d * (q - 8) exactly.
 * Nibble order inside a block: TK_Q4_0_REFERENCE_ORDER (weight 2i = low nibble of byte i,
 * 2i+1 = high nibble: llama.zig:347-350) or TK_Q4_0_GGML_ORDER (weight i = low nibble,
 * i+16 = high nibble).  k % 32 == 0, n_rows even.  Synchronous. */
#define TK_Q4_0_REFERENCE_ORDER 0
#define TK_Q4_0_GGML_ORDER 1
int tk_repack_q4_0(tk_device *dev, const void *blocks, uint8_t *w_packed, uint16_t *scales,
                   uint8_t *zeros, uint32_t n_rows, uint32_t k, int order);

/* ---- paged decode attention ---------------------------------------------------------------
 * Replaces PagedAttention.forward(q, k_cache, v_cache, block_tables, context_lens, o, batch_size,
 * num_heads, head_dim, max_blocks) (src/kernels/attention.zig:51-100, shaders.zig:503-587):
 * for sequence b and head h, o = softmax(q . K^T / sqrt(head_dim)) V over the sequence's first
 * context_lens[b] tokens; token t lives in physical block block_tables[b * max_blocks + t / 16]
 * of k_cache / v_cache laid out [block][num_heads][16][head_dim].  q, o: [batch][num_heads]
 * [head_dim] f32; head_dim <= 128 (the shader's limit).  A sequence with no tokens gives zeros
 * (the shader divides by a zero sum); a context longer than max_blocks * 16 is cut there (the
 * shader would read past its table row). */
int tk_paged_attention(tk_device *dev, const float *q, const float *k_cache, const float *v_cache,
                       const int32_t *block_tables, const int32_t *context_lens, float *o,
                       uint32_t batch, uint32_t num_heads, uint32_t head_dim, uint32_t max_blocks);
int tk_paged_attention_async(tk_device *dev, const float *q, const float *k_cache,
                             const float *v_cache, const int32_t *block_tables,
                             const int32_t *context_lens, float *o, uint32_t batch,
                             uint32_t num_heads, uint32_t head_dim, uint32_t max_blocks,
                             void *stream);

/* ---- sampler ----------------------------------------------------------------------------
 * Replaces the argmax shader (src/kernels/shaders.zig:889-943; the host loop of
 * src/model/llama.zig:290-303): out[0] = index of the largest of x[0..n).  Ties go to the smallest
 * index (the shader's tie rule follows its thread layout); all -inf or NaN gives 0. */
int tk_argmax(tk_device *dev, const float *x, uint32_t n, uint32_t *out);
int tk_argmax_async(tk_device *dev, const float *x, uint32_t n, uint32_t *out, void *stream);
/* Replaces softmax_sample (shaders.zig:826-887; llama.zig:305-323): probs = softmax(logits /
 * temperature) over vocab entries; sampled[0] = the first i whose cumulative probability exceeds
 * random_val in [0, 1), vocab - 1 if none.  The cumulative sums are computed in a different f32
 * order than the shader's sequential loop: the index can differ only when random_val lies within
 * rounding of a cumulative boundary.  temperature > 0. */
int tk_softmax_sample(tk_device *dev, const float *logits, float *probs, uint32_t *sampled,
                      uint32_t vocab, float temperature, float random_val);
int tk_softmax_sample_async(tk_device *dev, const float *logits, float *probs, uint32_t *sampled,
                            uint32_t vocab, float temperature, float random_val, void *stream);

/* Test hook (bit-exactness of dequantisation, shaders.zig:474-495):
 * out f32 [k][n] = float(scale[g][n]) * (float(q[k][n]) - float(zero[g][n])). */
int tk_dequant_int4(tk_device *dev, const uint8_t *w_packed, const uint16_t *scales,
                    const uint8_t *zeros, float *out, uint32_t k, uint32_t n,
                    uint32_t group_size);

/* ---- profiling ---------------------------------------------------------------------
 * Device-side event trace of the engine (the reference times with a wall clock only,
 * src/bench.zig:4-15).  When enabled, every engine launch overwrites a buffer of
 * sm_count * TK_TRACE_EVENTS global-timer stamps (ns) per CTA: start, prologue done,
 * phase-0 barrier passed, phase-0 items done, phase-1 barrier passed, phase-1 items done,
 * end, producer first issue, producer last issue, first stage landed (0 = not reached).
 * A launch of the batch 1-2 decode kernel uses the slots as: start, prologue records done, phase A
 * done, phase-B records done, phase B done, reduction tasks done, end, producer first issue,
 * producer last issue, first phase-B stage in hand (all ns), then consumer warp 0's ns spent
 * waiting for stages in phase A and in phase B, the CTA's phase-A and phase-B item counts, the
 * ns at which the last phase-B stage was in hand, and (x in host memory) the ns at which the
 * CTA held the whole of x.
 * A launch of the batch >= 5 GEMM overwrites the buffer with SM-clock cycle counts instead,
 * for CTAs x + X * (y + Y * z) below sm_count: TMA producer waiting for free ring stages,
 * producer total, MMA issuer waiting for dequantised tiles, MMA waiting for TMA stages, MMA
 * total, first dequantiser warp waiting for TMA stages, waiting for free A stages, its total,
 * its cycles completing tensor-memory stores, its cycles computing cells; and (the tensor-memory
 * kernel, global-timer ns) the CTA's entry, the end of its set-up, the first dequantiser warp's
 * loop end, its epilogue end and the CTA's exit. */
#define TK_TRACE_EVENTS 16
int tk_device_trace_enable(tk_device *dev, int enable);
int tk_device_trace_read(tk_device *dev, uint64_t *out, size_t max_values, size_t *n_values);

/* ---- allocation-free qmatmul_int4 ---------------------------------------------------
 * No counterpart in the reference (its Metal buffers are always created by the caller
 * through Device.createBuffer; nothing on its path allocates scratch).
 *
 * For callers that cannot call cudaMalloc: a process whose device memory is reserved up
 * front by its own allocator, a latency-critical loop that must not take cudaMalloc's
 * device-wide synchronisation, or a binding that cannot own a tk_device.  Same layout, shapes
 * and errors as tk_qmatmul_int4, on the calling thread's current CUDA device and on `stream`
 * (NULL = the legacy default stream).
 *  - Synchronous: it waits for its work and reads the error word back before it returns.
 *  - Results are within the path's tolerance of tk_qmatmul_int4's, not always identical: every
 *    row count runs the streaming engine in chunks of 4 rows (m >= 5 does not take the
 *    tensor-core GEMM), and shapes the engine does not take run the CUDA-core kernel.
 *  - Its bounded device-side waits give up after a fixed 2 s (TK_WAIT_TIMEOUT_MS is not read).
 * It allocates nothing: the engine's scratch is one static device array of
 * TK_NOALLOC_SCRATCH_BYTES per GPU that loads the library, held until the process exits.
 *  - A shape whose scratch would exceed that size fails with TK_ERR_ARG (config 0,
 *    m=1 k=4096 n=14336 group 64, needs about 3.5 MB); use tk_qmatmul_int4 for those.
 *  - The first call on a device looks up the array's device address (cudaGetSymbolAddress)
 *    and keeps it for the life of the process (cudaDeviceReset is not supported afterwards).
 *  - Every call shares the one array and clears its counters on entry: calls that overlap
 *    on the GPU (other threads, other streams) race and must be serialised by the caller. */
#define TK_NOALLOC_SCRATCH_BYTES (4u << 20)
int tk_qmatmul_int4_noalloc(const float *x, const uint8_t *w_packed, const uint16_t *scales,
                            const uint8_t *zeros, float *out, uint32_t m, uint32_t k,
                            uint32_t n, uint32_t group_size, void *stream);

/* Which path tk_qmatmul_int4 would take for a shape with 16-byte aligned buffers and the
 * default device settings (148 SMs, 227 KB of shared memory per block): 3 = the decode kernel
 * (m <= 4 whose records and ring fit shared memory), 2 = tcgen05 GEMM (m >= 5), 1 = streaming
 * engine (a shape neither of those takes), 0 = CUDA-core fallback, <0 = invalid shape.
 * No counterpart in the reference (one shader serves every shape there). */
int tk_qmatmul_int4_path(uint32_t m, uint32_t k, uint32_t n, uint32_t group_size);

/* The same for tk_int4_ffn over [m][hidden] with an intermediate size inter. */
int tk_int4_ffn_path(uint32_t m, uint32_t hidden, uint32_t inter, uint32_t group_size);

#ifdef __cplusplus
}
#endif
#endif /* TK_CUDA_H */
