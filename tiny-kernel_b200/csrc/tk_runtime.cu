// tk_runtime.cu -- the C ABI of include/tk_cuda.h: device, buffers, scratch, dispatch.
//
// Replaces the reference's Metal runtime (src/metal/device.zig, src/metal/objc.zig) with a
// CUDA device context: one stream per device, a scratch arena for the engine (activation
// records, split-K partials, tile counters, grid barrier, error word) and a cache of TMA
// tensor maps keyed by weight pointer.  Entry points validate their arguments (the
// reference validates none) and report errors as negative status codes.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/tk_cuda.h"
#include "tk_decode.h"
#include "tk_engine.h"
#include "tk_internal.h"

using namespace tk;

namespace {

thread_local std::string g_last_error;

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

#define TK_CUDA_TRY(expr)                                                                     \
  do {                                                                                        \
    cudaError_t e__ = (expr);                                                                 \
    if (e__ != cudaSuccess)                                                                   \
      return fail(TK_ERR_CUDA, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e__), __FILE__, \
                  __LINE__);                                                                  \
  } while (0)

// A kernel launch on a device: counted (tk_device_launch_count), then checked.
#define TK_LAUNCH(dev, expr) \
  do {                       \
    ++(dev)->launches;       \
    TK_CUDA_TRY(expr);       \
  } while (0)

PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;
std::once_flag g_encode_once;

struct ScratchBuf {
  void* ptr = nullptr;
  size_t cap = 0;
};

struct TmapEntry {
  const void* base;
  uint64_t cols, rows;
  uint32_t box_rows;
  CUtensorMap map;
};

constexpr unsigned long long kDefaultTimeoutNs = 2000000000ull;  // 2 s per bounded wait
constexpr unsigned kErrHostSlots = 64;  // synchronising calls in flight at once on one device
// shared memory the engine kernel declares statically (phase table, job queues, barriers)
constexpr int kStaticSmemReserve = 4096;

}  // namespace

// A synchronous host-buffer FFN call recorded as a CUDA graph (upload, kernels, download, the
// error word's read-back): a repeated call with the same arguments is one graph launch and one
// wait.  Keyed by every argument; valid while the device's scratch buffers are not reallocated.
struct FfnGraph {
  const void* ptr[13];  // x, norm weight, gate / up / down (w, s, z), out, h_out
  uint32_t shape[5];    // m, hidden, inter, group size, flags
  uint32_t eps_bits;
  unsigned gen;
  unsigned long long last_use;
  cudaGraphExec_t exec;
  unsigned* err_host;  // pinned, written by the graph's last copy
};

struct tk_device {
  int ordinal = 0;
  cudaStream_t stream = nullptr;
  cudaDeviceProp prop{};
  char name[256] = {0};
  int sm_count = 0;
  int smem_optin = 0;
  unsigned long long timeout_ns = kDefaultTimeoutNs;
  int stages_override = 0;
  int ffn_split = 1;  // gate/up tile ranges of the FFN (TK_FFN_SPLIT, 1..4)
  SyncState* sync = nullptr;
  unsigned* err = nullptr;
  // Pinned host copies of the error word, one slot per synchronising call (a ring), so that the
  // word's read is queued behind the call's work and one wait covers both.
  unsigned* err_host = nullptr;
  std::atomic<unsigned> err_slot{0};
  ScratchBuf frag[1];      // per-CTA prologue records when they do not fit in shared memory
  ScratchBuf partials[2];  // split-K partial sums: [0] first reduction, [1] second
  ScratchBuf counters[2];  // segment counters per 128-column sub-tile of each
  // batch >= 5 GEMM path: f16 activations, f16 h, split-K partials
  ScratchBuf g_x16, g_h16, g_part;
  int gemm_enabled = 1;  // TK_GEMM=0 routes every batch through the engine
  int engine_ctas = 0;    // TK_ENGINE_CTAS: CTAs of the engine's launches (0: one per SM)
  int down_prefetch = 1;  // TK_DOWN_PREFETCH=0 turns off the L2 prefetch of the down projection
  int decode_enabled = 1;  // TK_DECODE=0 routes batch 1-2 through the streaming engine instead
  int decode_pdl = 1;      // TK_DECODE_PDL=0: cooperative launches without programmatic overlap
  ScratchBuf dec;          // decode kernel: launch epochs + tagged partial sums of its phases
  ScratchBuf io;           // TK_FFN_HOST_IO staging of x and out
  ScratchBuf zero_rows;    // one k-step of zero packed rows (the decode kernel's partial items)
  size_t dec_xdev_bytes = 0;  // the decode scratch's tagged host-x area
  // While a synchronous host-buffer call is being recorded into a graph: the pinned word its
  // decode kernel reports a failure to, and whether a kernel took it (if none did, the graph
  // ends with a copy of the device error word instead).
  unsigned* capture_err_host = nullptr;
  bool capture_err_used = false;
  unsigned scratch_gen = 0;  // bumped whenever a scratch buffer is reallocated
  std::vector<struct FfnGraph> ffn_graphs;  // synchronous TK_FFN_HOST_IO calls, recorded
  unsigned long long* trace = nullptr;  // [sm_count][kTraceEvents] when tracing is enabled
  unsigned long long launches = 0;      // kernels enqueued through this device
  // timed-out peer-memory exchanges seen by tk_device_check_error: a tk_tp group created before
  // the latest one is out of step with its peers and refuses further exchanges
  unsigned p2p_timeouts = 0;
  std::vector<TmapEntry> tmaps;
};

namespace {

// CTAs of an engine launch: one per SM unless overridden (TK_ENGINE_CTAS).
int engine_grid(const tk_device* d) {
  return d->engine_ctas > 0 && d->engine_ctas < d->sm_count ? d->engine_ctas : d->sm_count;
}

// CTAs of an FFN launch.  A small FFN (a tensor-parallel shard: under ~60 MB of packed weights)
// is bound by its split-K reduction chains rather than by streaming; there, the largest CTA count
// (>= 60 % of the SMs) that divides the down projection's (column tile, group) items gives every
// CTA whole groups, so no group's item is split between CTAs -- measured per FFN step at hidden
// 4096 on B200: inter 7168 36.1 -> 33.5 us, 3584 31.2 -> 27.9 us, 1792 30.8 -> 24.4 us (112 CTAs);
// the whole 8B FFN keeps one CTA per SM.
int ffn_engine_ctas(const tk_device* d, int hidden, int inter, int gs) {
  if (d->engine_ctas > 0) return engine_grid(d);
  const int sm = d->sm_count;
  if (1.5 * (double)hidden * (double)inter >= 60e6) return sm;
  const long long items = (long long)((hidden + kWideCols - 1) / kWideCols) * (inter / gs);
  for (int c = sm; c * 10 >= sm * 6; --c)
    if (items % c == 0) return c;
  return sm;
}

int set_device(tk_device* d) {
  TK_CUDA_TRY(cudaSetDevice(d->ordinal));
  return TK_OK;
}

cudaStream_t pick_stream(tk_device* d, void* stream) {
  return stream ? static_cast<cudaStream_t>(stream) : d->stream;
}

// Grows a scratch buffer; new memory is zeroed (tile counters must start at zero).
int scratch_ensure(tk_device* d, ScratchBuf& b, size_t need) {
  if (b.cap >= need) return TK_OK;
  TK_CUDA_TRY(cudaStreamSynchronize(d->stream));
  TK_CUDA_TRY(cudaDeviceSynchronize());
  if (b.ptr) TK_CUDA_TRY(cudaFree(b.ptr));
  b.ptr = nullptr;
  b.cap = 0;
  size_t cap = std::max<size_t>(need, 4096);
  TK_CUDA_TRY(cudaMalloc(&b.ptr, cap));
  TK_CUDA_TRY(cudaMemset(b.ptr, 0, cap));
  // the memset runs on the legacy stream, which the device's non-blocking stream does not wait
  // for: finish it before any kernel can use the buffer
  TK_CUDA_TRY(cudaDeviceSynchronize());
  b.cap = cap;
  ++d->scratch_gen;  // graphs recorded over the old buffers are stale
  return TK_OK;
}

int get_encoder() {
  std::call_once(g_encode_once, [] {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode_tiled) return fail(TK_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  return TK_OK;
}

// 2-D tensor map over packed weights [rows = K/2][cols = N bytes] viewed as u64 elements;
// box = 130 u64 (a 1040-byte row: one 1024-column wide tile + 16 bytes) x box_rows rows,
// no swizzle (rows land 16 bytes apart modulo 128 in shared memory).  Cached per pointer.
int weight_tmap(tk_device* d, const void* base, uint64_t cols, uint64_t rows, uint32_t box_rows,
                CUtensorMap* out) {
  for (auto& e : d->tmaps)
    if (e.base == base && e.cols == cols && e.rows == rows && e.box_rows == box_rows) {
      *out = e.map;
      return TK_OK;
    }
  int st = get_encoder();
  if (st != TK_OK) return st;
  TmapEntry e;
  e.base = base;
  e.cols = cols;
  e.rows = rows;
  e.box_rows = box_rows;
  cuuint64_t dims[2] = {cols / 8, rows};
  cuuint64_t strides[1] = {cols};
  cuuint32_t box[2] = {(cuuint32_t)kRowElems, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode_tiled(&e.map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(base),
                              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TK_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  if (d->tmaps.size() >= 512) d->tmaps.erase(d->tmaps.begin());
  d->tmaps.push_back(e);
  *out = e.map;
  return TK_OK;
}

// Both tensor maps of one matrix (group box and k-step box) into maps[idx], maps[idx + 1].
int matrix_tmaps(tk_device* d, const void* w, uint64_t n, uint64_t k, int gs, TmapPack& maps,
                 int idx) {
  int st = weight_tmap(d, w, n, k / 2, (uint32_t)(gs / 2), &maps.map[idx]);
  if (st != TK_OK) return st;
  return weight_tmap(d, w, n, k / 2, (uint32_t)kStepRows, &maps.map[idx + 1]);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_qshape(uint32_t m, uint32_t k, uint32_t n, uint32_t gs) {
  if (m == 0 || k == 0 || n == 0 || gs == 0) return fail(TK_ERR_ARG, "zero dimension");
  if (gs % 8 != 0) return fail(TK_ERR_ARG, "group_size %u is not a multiple of 8", gs);
  if (k % gs != 0) return fail(TK_ERR_ARG, "k=%u is not a multiple of group_size=%u", k, gs);
  if (n % 2 != 0) return fail(TK_ERR_ARG, "n=%u is odd (zero points pack two columns per byte)", n);
  if ((uint64_t)m * k > (1ull << 31) || (uint64_t)k * n > (1ull << 33))
    return fail(TK_ERR_ARG, "shape too large");
  return TK_OK;
}

bool engine_shape(uint32_t k, uint32_t n, uint32_t gs) {
  return n % kTileCols == 0 && k % kTileCols == 0 &&
         (gs == 16 || gs == 32 || gs == 64 || gs == 128);
}

int mt_for(uint32_t m) { return m <= 1 ? 1 : (m <= 2 ? 2 : 4); }

long long warp_of_unit_h(long long u, long long units, long long W) {
  return ((u + 1) * W - 1) / units;
}

// Largest number of CTA ranges that intersect one column unit (wide tile x matrix).
int max_segments(const PhaseParams& P, long long Wtot) {
  const long long W = std::min<long long>(Wtot, P.units);
  const long long per = (long long)P.groups * P.spg;
  int mx = 1;
  for (long long cu = 0; cu < (long long)P.tiles * P.nmat; ++cu) {
    const long long a = cu * per;
    const int ns = (int)(warp_of_unit_h(a + per - 1, P.units, W) - warp_of_unit_h(a, P.units, W) + 1);
    mx = std::max(mx, ns);
  }
  return mx;
}

// Sum over the phase's column units of (CTA ranges holding the unit) * (slices of its tile):
// the (segment, slice) pairs a kEpiSiluMul phase completes.
int phase_done_total(const PhaseParams& P, long long Wtot) {
  const long long W = std::min<long long>(Wtot, P.units);
  const long long per = (long long)P.groups * P.spg;
  long long tot = 0;
  for (long long c = 0; c < (long long)P.tiles * P.nmat; ++c) {
    const long long a = c * per;
    const long long ns = warp_of_unit_h(a + per - 1, P.units, W) - warp_of_unit_h(a, P.units, W) + 1;
    const int wt = P.wt0 + (int)(c / P.nmat);
    tot += ns * std::min(kSlices, (P.N - wt * kWideCols) / kTileCols);
  }
  return (int)tot;
}

// One phase over the wide tiles [wt0, wt1) of N and the groups [g0, g1) of K (all of them
// when wt1 / g1 are negative); a reduction of its own until bind_partials says otherwise.
void fill_phase(PhaseParams& P, int K, int N, int gs, int nmat, int mt, int wt0 = 0, int wt1 = -1,
                int g0 = 0, int g1 = -1) {
  std::memset(&P, 0, sizeof(P));
  P.K = K;
  P.N = N;
  P.gs = gs;
  P.nmat = nmat;
  P.spg = gs / 16;
  P.wt0 = wt0;
  P.wt1 = wt1 < 0 ? (N + kWideCols - 1) / kWideCols : wt1;
  P.g0 = g0;
  P.g1 = g1 < 0 ? K / gs : g1;
  P.tiles = P.wt1 - P.wt0;
  P.groups = P.g1 - P.g0;
  P.units = (long long)P.tiles * nmat * P.groups * P.spg;
  P.frag_bytes = record_bytes(gs, mt);
}

// Split-K scratch of phases [first, first + count) of p, which run over the same matrices:
// one partials buffer indexed by global column unit and one counter per 128-column sub-tile.
// combined: the phases cover disjoint groups of the same outputs and form one reduction (its
// segments are the phases' segments in phase order); otherwise each phase covers its own
// tiles and is a reduction of its own.
int bind_partials(tk_device* d, EngineParams& p, int first, int count, int idx, int mt,
                  long long Wtot, bool combined) {
  int maxseg = 0;
  for (int q = first; q < first + count; ++q) {
    const int ms = max_segments(p.ph[q], Wtot);
    maxseg = combined ? maxseg + ms : std::max(maxseg, ms);
  }
  const PhaseParams& F = p.ph[first];
  const size_t tiles_all = (size_t)(F.N + kWideCols - 1) / kWideCols;
  const size_t pbytes = tiles_all * F.nmat * maxseg * kSlices * mt * kTileCols * sizeof(float);
  int st = scratch_ensure(d, d->partials[idx], pbytes);
  if (st != TK_OK) return st;
  // one counter per 128-column sub-tile, then one per phase (kEpiSiluMul completion)
  st = scratch_ensure(d, d->counters[idx], (size_t)(F.N / kTileCols + kMaxPhases) * sizeof(unsigned));
  if (st != TK_OK) return st;
  for (int q = first; q < first + count; ++q) {
    PhaseParams& P = p.ph[q];
    P.maxseg = maxseg;
    P.partials = static_cast<float*>(d->partials[idx].ptr);
    P.counters = static_cast<unsigned*>(d->counters[idx].ptr);
    P.red_first = combined ? first : q;
    P.red_count = combined ? count : 1;
  }
  return TK_OK;
}

int launch_engine(tk_device* d, int mt, const TmapPack& maps, EngineParams& p, cudaStream_t st,
                  int ctas) {
  int spg_max = 0, fb_max = 0;
  for (int q = 0; q < p.nphases; ++q) {
    // the kernel's stream-K arithmetic is 32-bit
    if (p.ph[q].units * (long long)ctas >= (1LL << 31))
      return fail(TK_ERR_UNSUPPORTED, "phase of %lld work units is too large for one launch",
                  p.ph[q].units);
    spg_max = std::max(spg_max, p.ph[q].spg);
    fb_max = std::max(fb_max, p.ph[q].frag_bytes);
  }
  p.tile_stage_bytes = (spg_max * kStepRows * kRowBytes + 127) & ~127;
  p.aux_stage_bytes = (kSlices * (kScaleBytes + kZeroBytes) + fb_max + 15) & ~15;
  int stages = 0, rec0_smem = 0;
  size_t smem = 0;
  const int rec0_bytes = (p.K0 / p.gs0) * p.frag0_bytes;
  if (!engine_plan_smem(p.tile_stage_bytes, p.aux_stage_bytes, rec0_bytes, d->smem_optin - kStaticSmemReserve,
                        &stages, &rec0_smem, &smem))
    return fail(TK_ERR_UNSUPPORTED, "engine ring does not fit in shared memory");
  if (d->stages_override > 0 && d->stages_override < stages) {
    stages = d->stages_override;
    smem = engine_smem_bytes(stages, p.tile_stage_bytes, p.aux_stage_bytes,
                             rec0_smem ? rec0_bytes : 0);
  }
  p.stages = stages;
  p.rec0_smem = rec0_smem;
  p.prefetch_l2 = d->down_prefetch;
  p.trace = d->trace;
  if (d->trace)
    TK_CUDA_TRY(cudaMemsetAsync(d->trace, 0, (size_t)d->sm_count * kTraceEvents * 8, st));
  p.sync = d->sync;
  p.err = d->err;
  p.timeout_ns = d->timeout_ns;
  int blocks = 0;
  TK_CUDA_TRY(engine_occupancy(mt, p.gs0, smem, &blocks));
  if (blocks < 1) return fail(TK_ERR_UNSUPPORTED, "engine kernel cannot be resident");
  TK_LAUNCH(d, engine_launch(mt, p.gs0, maps, p, ctas, smem, st));
  return TK_OK;
}

int sync_and_check(tk_device* d, cudaStream_t st) {
  // The error word is copied on `st` behind the work, so the one wait also brings the word back
  // (a separate synchronous read would be a second round trip on every synchronous call).
  volatile unsigned* slot = d->err_host + d->err_slot.fetch_add(1u) % kErrHostSlots;
  TK_CUDA_TRY(cudaMemcpyAsync(const_cast<unsigned*>(slot), d->err, sizeof(unsigned),
                              cudaMemcpyDeviceToHost, st));
  TK_CUDA_TRY(cudaStreamSynchronize(st));
  if (*slot == 0) return TK_OK;
  return tk_device_check_error(d);  // reads the word again, reports it and clears the state
}

// One engine launch for <= 4 rows of qmatmul_int4.
int qmatmul_engine_chunk(tk_device* d, const float* x, const uint8_t* w, const uint16_t* s,
                         const uint8_t* z, float* out, int m, int k, int n, int gs,
                         cudaStream_t st) {
  const int mt = mt_for(m);
  const long long Wtot = engine_grid(d);  // one CTA per SM; stream-K ranges are per CTA
  EngineParams p;
  std::memset(&p, 0, sizeof(p));
  p.m = m;
  p.nphases = 1;
  PhaseParams& P = p.ph[0];
  fill_phase(P, k, n, gs, 1, mt);
  P.map_base = 0;
  P.scales[0] = s;
  P.zeros[0] = z;
  const long long rec_stride = (long long)(k / gs) * P.frag_bytes;  // per-CTA records
  int stt = scratch_ensure(d, d->frag[0], (size_t)Wtot * rec_stride);
  if (stt != TK_OK) return stt;
  P.frag_in = static_cast<const uint8_t*>(d->frag[0].ptr);
  P.frag_cta_stride = rec_stride;
  stt = bind_partials(d, p, 0, 1, 0, mt, Wtot, false);
  if (stt != TK_OK) return stt;
  P.epi = kEpiStore;
  P.out = out;
  P.ldo = n;
  p.x = x;
  p.ldx = k;
  p.K0 = k;
  p.do_norm = 0;
  p.frag0 = static_cast<uint8_t*>(d->frag[0].ptr);
  p.frag0_cta_stride = rec_stride;
  p.gs0 = gs;
  p.frag0_bytes = P.frag_bytes;
  TmapPack maps;
  std::memset(&maps, 0, sizeof(maps));
  stt = matrix_tmaps(d, w, n, k, gs, maps, 0);
  if (stt != TK_OK) return stt;
  return launch_engine(d, mt, maps, p, st, (int)Wtot);
}

int ffn_engine_chunk(tk_device* d, const float* x, const float* norm_w, const tk_int4_matrix* gate,
                     const tk_int4_matrix* up, const tk_int4_matrix* down, float* out,
                     float* h_out, int m, int hidden, int inter, int gs, float eps, bool residual,
                     cudaStream_t st) {
  const int mt = mt_for(m);
  const long long Wtot = ffn_engine_ctas(d, hidden, inter, gs);  // stream-K ranges are per CTA
  EngineParams p;
  std::memset(&p, 0, sizeof(p));
  p.m = m;
  // gate/up over nsplit tile ranges, then the down projection over the h groups of each
  // range in the same order: the down work of early ranges runs while the last range's
  // sub-tiles are still being reduced
  const int tiles_i = (inter + kWideCols - 1) / kWideCols;
  const int nsplit = std::max(1, std::min({d->ffn_split, tiles_i, kMaxPhases / 2}));
  p.nphases = 2 * nsplit;
  const int groups_h = inter / gs;
  const long long rec_stride = (long long)(hidden / gs) * record_bytes(gs, mt);  // per-CTA records
  int stt = scratch_ensure(d, d->frag[0], (size_t)Wtot * rec_stride);
  if (stt != TK_OK) return stt;
  for (int j = 0; j < nsplit; ++j) {
    const int t0 = tiles_i * j / nsplit, t1 = tiles_i * (j + 1) / nsplit;
    PhaseParams& A = p.ph[j];
    fill_phase(A, hidden, inter, gs, 2, mt, t0, t1);
    A.map_base = 0;  // gate: maps 0,1; up: maps 2,3
    A.scales[0] = gate->scales;
    A.scales[1] = up->scales;
    A.zeros[0] = gate->zeros;
    A.zeros[1] = up->zeros;
    A.frag_in = static_cast<const uint8_t*>(d->frag[0].ptr);
    A.frag_cta_stride = rec_stride;
    A.epi = kEpiSiluMul;
    A.out = h_out;
    A.ldo = inter;
    const int g0 = std::min(groups_h, t0 * kWideCols / gs);
    const int g1 = j == nsplit - 1 ? groups_h : std::min(groups_h, t1 * kWideCols / gs);
    PhaseParams& B = p.ph[nsplit + j];
    fill_phase(B, inter, hidden, gs, 1, mt, 0, -1, g0, g1);
    B.map_base = 4;  // down: maps 4,5
    B.scales[0] = down->scales;
    B.zeros[0] = down->zeros;
    B.src_first = 0;  // records from silu(gate) * up of the gate/up phases
    B.src_count = nsplit;
    B.epi = kEpiStore;
    B.out = out;
    B.ldo = hidden;
    B.residual = residual ? x : nullptr;
    B.ldr = hidden;
  }
  stt = bind_partials(d, p, 0, nsplit, 0, mt, Wtot, false);
  if (stt != TK_OK) return stt;
  for (int j = 0; j < nsplit; ++j) p.ph[j].done_total = phase_done_total(p.ph[j], Wtot);
  stt = bind_partials(d, p, nsplit, nsplit, 1, mt, Wtot, true);
  if (stt != TK_OK) return stt;
  p.zero_counters = static_cast<unsigned*>(d->counters[0].ptr);
  p.zero_count = inter / kTileCols + kMaxPhases;
  p.phase_done = p.zero_counters + inter / kTileCols;
  p.x = x;
  p.ldx = hidden;
  p.K0 = hidden;
  p.norm_w = norm_w;
  p.eps = eps;
  p.do_norm = 1;
  p.frag0 = static_cast<uint8_t*>(d->frag[0].ptr);
  p.frag0_cta_stride = rec_stride;
  p.gs0 = gs;
  p.frag0_bytes = record_bytes(gs, mt);
  TmapPack maps;
  std::memset(&maps, 0, sizeof(maps));
  stt = matrix_tmaps(d, gate->w_packed, inter, hidden, gs, maps, 0);
  if (stt != TK_OK) return stt;
  stt = matrix_tmaps(d, up->w_packed, inter, hidden, gs, maps, 2);
  if (stt != TK_OK) return stt;
  stt = matrix_tmaps(d, down->w_packed, hidden, inter, gs, maps, 4);
  if (stt != TK_OK) return stt;
  return launch_engine(d, mt, maps, p, st, (int)Wtot);
}

// ---- batch 1-2: the decode kernel (tk_decode.cu) ---------------------------------------------

constexpr int kDecSmemLimit = 227 * 1024;  // B200 opt-in shared memory per block
constexpr int kDefaultGrid = 148;          // B200 SMs (the path queries assume the full device)
// words per (parity, source rank) of the fused tensor-parallel exchange: 2 rows x 16384 columns
constexpr size_t kTpFuseWords = 2 * 16384;

// One phase of the decode kernel: tiles [wt0, wt1) of N (all when wt1 < 0) and groups [g0, g1) of
// K (all when g1 < 0), nmat matrices, on `grid` CTAs.
void dec_fill(DecPhase& P, int K, int N, int gs, int nmat, int grid, int wt0 = 0, int wt1 = -1,
              int g0 = 0, int g1 = -1) {
  std::memset(&P, 0, sizeof(P));
  P.K = K;
  P.N = N;
  P.nmat = nmat;
  P.wt0 = wt0;
  P.tiles = (wt1 < 0 ? (N + kWideCols - 1) / kWideCols : wt1) - wt0;
  P.g0 = g0;
  P.groups = (g1 < 0 ? K / gs : g1) - g0;
  P.spg = gs / 16;
  P.units = (unsigned)((long long)P.tiles * nmat * P.groups * P.spg);
  P.ctas = std::min<unsigned>((unsigned)grid, P.units);
  const long long per = (long long)P.groups * P.spg;
  int mx = 1;
  for (long long cu = 0; cu < (long long)P.tiles * nmat; ++cu) {
    const long long a = cu * per;
    const int ns = (int)(warp_of_unit_h(a + per - 1, P.units, P.ctas) - warp_of_unit_h(a, P.units, P.ctas) + 1);
    mx = std::max(mx, ns);
  }
  P.maxseg = mx;
}

// The most items (groups) any CTA's range of phase P touches.
int dec_max_items(const DecPhase& P) {
  int mx = 0;
  for (unsigned b = 0; b < P.ctas; ++b) {
    const unsigned long long beg = (unsigned long long)P.units * b / P.ctas;
    const unsigned long long end = (unsigned long long)P.units * (b + 1) / P.ctas;
    mx = std::max(mx, (int)((end - 1) / P.spg - beg / P.spg + 1));
  }
  return mx;
}

// The phases of a launch: qmatmul_int4 is one A phase over K x N; the FFN is `split` gate/up phases
// over consecutive tile ranges of the intermediate, then as many down phases over the matching
// h groups (records of B phase j from the partial sums of A phase j).
void dec_phases(DecodeParams& p, bool ffn, int k, int n, int inter, int gs, int grid, int split) {
  if (!ffn) {
    dec_fill(p.ph[0], k, n, gs, 1, grid);
    p.na = p.nph = 1;
    return;
  }
  const int tiles_i = (inter + kWideCols - 1) / kWideCols;
  const int S = std::max(1, std::min({split, tiles_i, kDecMaxPhases / 2}));
  const int groups_h = inter / gs;
  for (int j = 0; j < S; ++j) {
    const int t0 = tiles_i * j / S, t1 = tiles_i * (j + 1) / S;
    dec_fill(p.ph[j], k, inter, gs, 2, grid, t0, t1);
    const int g0 = std::min(groups_h, t0 * kWideCols / gs);
    const int g1 = j == S - 1 ? groups_h : std::min(groups_h, t1 * kWideCols / gs);
    dec_fill(p.ph[S + j], inter, k, gs, 1, grid, 0, -1, g0, g1);
  }
  p.na = S;
  p.nph = 2 * S;
}

struct DecPlan {
  int stages = 0, pro_stages = 0, tile_stage_bytes = 0, aux_stage_bytes = 0;
  int recb_items = 0, frag_bytes = 0;
  size_t smem = 0;
};

// Shared-memory plan of a decode launch; false when the shape does not fit (the caller then takes
// the streaming engine).
bool dec_plan(const DecodeParams& p, int m, int mt, int gs, bool norm, int smem_limit,
              DecPlan* out) {
  DecPlan pl;
  pl.tile_stage_bytes = ((gs / 16) * kStepRows * kRowBytes + 127) & ~127;
  pl.aux_stage_bytes = kSlices * (kScaleBytes + kZeroBytes);
  pl.frag_bytes = mt * dp_tok_stride(gs);  // the int16 records of every row (dp2a at any mt)
  for (int q = p.na; q < p.nph; ++q) pl.recb_items = std::max(pl.recb_items, dec_max_items(p.ph[q]));
  if (pl.recb_items > kDecMaxItemsB) return false;
  const DecPhase& A = p.ph[0];
  const long long pro = (long long)A.K * 4 * (m + (norm ? 1 : 0));
  pl.pro_stages = (int)((pro + pl.tile_stage_bytes - 1) / pl.tile_stage_bytes);
  const int rec0 = A.groups * pl.frag_bytes;
  const int recb = (p.nph - p.na) * pl.recb_items * pl.frag_bytes;
  for (int s = kMaxStages; s >= 2; --s) {
    const size_t need = decode_smem_bytes(s, pl.tile_stage_bytes, pl.aux_stage_bytes, rec0, recb);
    if (need <= (size_t)smem_limit) {
      pl.stages = s;
      pl.smem = need;
      break;
    }
  }
  if (pl.stages < 2 || pl.pro_stages >= pl.stages) return false;
  // 32-bit stream-K arithmetic in the kernel
  for (int q = 0; q < p.nph; ++q)
    if ((long long)p.ph[q].units * p.ph[q].ctas >= (1LL << 31)) return false;
  *out = pl;
  return true;
}

// Gate/up tile ranges of the decode kernel's FFN (TK_FFN_SPLIT, default 1: with the down records
// built by the consumer warps themselves, a second range added a record round trip and twice the
// output segments -- 8B FFN at batch 1 on B200: 28.0 us per step with one range, 34.5 with two).
int dec_split(const tk_device* d) { return d->ffn_split; }

// Can the decode kernel take this call (default device settings)?
// The fused tensor-parallel exchange of a decode launch (DecodeParams::tp_*).
struct TpFuse {
  int n, rank, words;
  unsigned long long* recv[kDecMaxRanks];
  unsigned* epoch;
};

// Rows one decode launch takes, and the instantiation (rows in registers) for m of them.
constexpr int kDecMaxRows = 4;
int dec_mt(int m) { return m <= 2 ? m : 4; }

bool decode_shape(int m, int k, int n, int inter, int gs, int grid, bool ffn) {
  if (m < 1 || m > kDecMaxRows || !(gs == 16 || gs == 32 || gs == 64 || gs == 128)) return false;
  DecodeParams p;
  std::memset(&p, 0, sizeof(p));
  dec_phases(p, ffn, k, n, inter, gs, grid, 1);
  DecPlan pl;
  return dec_plan(p, m, dec_mt(m), gs, ffn, kDecSmemLimit - kStaticSmemReserve, &pl);
}

// One decode launch for m <= 4 rows: qmatmul_int4 (gate == nullptr) or the FFN.  Returns
// TK_ERR_UNSUPPORTED, before enqueuing anything, when the shape does not fit the kernel.
int decode_run(tk_device* d, const float* x, const float* norm_w, float eps,
               const tk_int4_matrix* a0, const tk_int4_matrix* a1, const tk_int4_matrix* down,
               float* out, float* h_out, int m, int k, int n, int inter, int gs, bool residual,
               cudaStream_t st, bool host_io = false, const TpFuse* tpf = nullptr) {
  const bool ffn = down != nullptr;
  const int mt = dec_mt(m);  // instantiations for 1, 2 and 4 rows
  const int grid = engine_grid(d);
  DecodeParams p;
  std::memset(&p, 0, sizeof(p));
  p.m = m;
  dec_phases(p, ffn, k, n, inter, gs, grid, dec_split(d));
  DecPlan pl;
  if (!dec_plan(p, m, mt, gs, ffn, d->smem_optin - kStaticSmemReserve, &pl))
    return fail(TK_ERR_UNSUPPORTED, "shape does not fit the decode kernel");
  if (d->stages_override > 0 && d->stages_override < pl.stages && d->stages_override > pl.pro_stages) {
    pl.stages = d->stages_override;
    pl.smem = decode_smem_bytes(pl.stages, pl.tile_stage_bytes, pl.aux_stage_bytes,
                                p.ph[0].groups * pl.frag_bytes,
                                (p.nph - p.na) * pl.recb_items * pl.frag_bytes);
  }
  // scratch: epochs, then the tagged partials of every phase, then the tagged host x
  const size_t epoch_bytes = kDecEpochSlots * sizeof(unsigned);
  size_t part_bytes[kDecMaxPhases], total = epoch_bytes;
  for (int q = 0; q < p.nph; ++q) {
    const DecPhase& P = p.ph[q];
    part_bytes[q] = (size_t)P.tiles * P.nmat * P.maxseg * mt * kWideCols * 8;
    total += part_bytes[q];
  }
  // host x: the tagged words through which the CTAs share it (the area is kept once sized, so
  // that a device-buffer call after a host-buffer one does not reallocate the scratch)
  const size_t xdev = std::max<size_t>(host_io ? (size_t)m * k * 8 : 0, d->dec_xdev_bytes);
  int stt = scratch_ensure(d, d->dec, total + xdev);
  if (stt != TK_OK) return stt;
  uint8_t* base = static_cast<uint8_t*>(d->dec.ptr);
  p.epoch = reinterpret_cast<unsigned*>(base);
  size_t off = epoch_bytes;
  for (int q = 0; q < p.nph; ++q) {
    p.ph[q].part = reinterpret_cast<unsigned long long*>(base + off);
    off += part_bytes[q];
  }
  d->dec_xdev_bytes = xdev;
  p.x_host = host_io ? 1 : 0;
  p.x_dev = host_io ? reinterpret_cast<unsigned long long*>(base + off) : nullptr;
  TmapPack maps;
  std::memset(&maps, 0, sizeof(maps));
  if ((stt = scratch_ensure(d, d->zero_rows, (size_t)kStepRows * kRowBytes)) != TK_OK) return stt;
  if ((stt = weight_tmap(d, d->zero_rows.ptr, kRowBytes, kStepRows, (uint32_t)kStepRows,
                         &maps.map[kZeroMap])) != TK_OK)
    return stt;
  if ((stt = matrix_tmaps(d, a0->w_packed, ffn ? inter : n, k, gs, maps, 0)) != TK_OK) return stt;
  if (ffn) {
    if ((stt = matrix_tmaps(d, a1->w_packed, inter, k, gs, maps, 2)) != TK_OK) return stt;
    if ((stt = matrix_tmaps(d, down->w_packed, k, inter, gs, maps, 4)) != TK_OK) return stt;
  }
  for (int q = 0; q < p.na; ++q) {
    DecPhase& A = p.ph[q];
    A.map_base = 0;  // gate (or the qmatmul matrix): maps 0, 1; up: maps 2, 3
    A.scales[0] = a0->scales;
    A.zeros[0] = a0->zeros;
    if (ffn) {
      A.scales[1] = a1->scales;
      A.zeros[1] = a1->zeros;
    }
  }
  for (int q = p.na; q < p.nph; ++q) {
    DecPhase& B = p.ph[q];
    B.map_base = 4;  // down: maps 4, 5
    B.scales[0] = down->scales;
    B.zeros[0] = down->zeros;
  }
  p.x = x;
  p.ldx = k;
  p.norm_w = ffn ? norm_w : nullptr;
  p.eps = eps;
  const int n_out = ffn ? k : n;
  p.out = out;
  p.ldo = n_out;
  p.residual = residual ? x : nullptr;
  p.ldr = k;
  p.h_out = ffn ? h_out : nullptr;
  p.ldh = inter;
  p.stages = pl.stages;
  p.tile_stage_bytes = pl.tile_stage_bytes;
  p.aux_stage_bytes = pl.aux_stage_bytes;
  p.pro_stages = pl.pro_stages;
  p.frag_bytes = pl.frag_bytes;
  p.recb_items = pl.recb_items;
  p.red_tasks = n_out / 8;
  if (host_io && residual && p.red_tasks > kDecMaxTasksPerCta * grid)
    return fail(TK_ERR_UNSUPPORTED, "host x with the residual: too many reduction tasks");
  p.err_host = d->capture_err_host;
  if (p.err_host) d->capture_err_used = true;
  p.tp_n = 1;
  if (tpf && tpf->n > 1) {
    if ((size_t)m * n_out > (size_t)tpf->words)
      return fail(TK_ERR_UNSUPPORTED, "fused exchange: output larger than the exchange area");
    p.tp_n = tpf->n;
    p.tp_rank = tpf->rank;
    p.tp_words = tpf->words;
    p.tp_epoch = tpf->epoch;
    for (int r = 0; r < tpf->n; ++r) p.tp_recv[r] = tpf->recv[r];
  }
  p.err = d->err;
  p.timeout_ns = d->timeout_ns;
  p.trace = d->trace;
  p.pdl = d->decode_pdl;
  if (d->trace)
    TK_CUDA_TRY(cudaMemsetAsync(d->trace, 0, (size_t)d->sm_count * kTraceEvents * 8, st));
  int blocks = 0;
  TK_CUDA_TRY(decode_occupancy(mt, gs, pl.smem, &blocks));
  if (blocks < 1) return fail(TK_ERR_UNSUPPORTED, "decode kernel cannot be resident");
  TK_LAUNCH(d, decode_launch(mt, gs, maps, p, grid, pl.smem, st));
  return TK_OK;
}

// ---- batch >= 5: the tcgen05 GEMM path (tk_gemm.cu) ----------------------------------------

// From 5 rows the tcgen05 GEMM: a decode launch takes at most 4 rows, and two of them (batch
// 5-8: 85-122 us per 8B FFN step) cost more than one GEMM over a 16-token tile (about 71 us).
constexpr int kGemmMinRows = 5;

int gemm_nt(int m) { return m <= 16 ? 16 : m <= 32 ? 32 : m <= 64 ? 64 : m <= 128 ? 128 : 256; }

// Shapes the GEMM takes: k in whole 64-steps of whole groups, columns in whole CTA tiles.
bool gemm_shape(uint32_t k, uint32_t n, uint32_t gs, bool pair) {
  return k % kGemmKStep == 0 && (gs == 16 || gs == 32 || gs == 64 || gs == 128) && k % gs == 0 &&
         n % (pair ? kGemmTileCols : kGemmTiles * kGemmTileCols) == 0;
}

// f16 activations [rows][k] for the B operand: box 64 x nt, 128-byte swizzle (rows beyond
// `rows` read as zero).
int act_tmap(const void* base, uint64_t k, uint64_t rows, uint32_t nt, CUtensorMap* out) {
  int st = get_encoder();
  if (st != TK_OK) return st;
  cuuint64_t dims[2] = {k, rows};
  cuuint64_t strides[1] = {k * 2};
  cuuint32_t box[2] = {(cuuint32_t)kGemmKStep, nt};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode_tiled(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims,
                              strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TK_ERR_CUDA, "cuTensorMapEncodeTiled (activations) failed (%d)", (int)r);
  return TK_OK;
}

// Packed weights [k/2][n] for the dequantisers: box 128 columns x 32 packed rows; for the
// tensor-memory kernel 64 packed rows with the 128-byte swizzle.
int gemm_wtmap(const void* w, uint64_t n, uint64_t k, bool tm, CUtensorMap* out) {
  int st = get_encoder();
  if (st != TK_OK) return st;
  const bool swizzle = tm;
  cuuint64_t dims[2] = {n, k / 2};
  cuuint64_t strides[1] = {n};
  cuuint32_t box[2] = {(cuuint32_t)kGemmTileCols, (cuuint32_t)((tm ? kGemmTmKStep : kGemmKStep) / 2)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode_tiled(out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(w), dims,
                              strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TK_ERR_CUDA, "cuTensorMapEncodeTiled (weights) failed (%d)", (int)r);
  return TK_OK;
}

// Scales [k/gs][n] (f16, box 128 columns x 8 groups) and zero points [k/gs][n/2] (u8, box 64 x
// 8 groups) for the tensor-memory kernel's scale ring.
int gemm_auxmaps(const uint16_t* s, const uint8_t* z, uint64_t n, uint64_t k, uint64_t gs,
                 CUtensorMap* sc, CUtensorMap* ze) {
  int st = get_encoder();
  if (st != TK_OK) return st;
  cuuint32_t estr[2] = {1, 1};
  {
    cuuint64_t dims[2] = {n, k / gs};
    cuuint64_t strides[1] = {n * 2};
    cuuint32_t box[2] = {(cuuint32_t)kGemmTileCols, (cuuint32_t)kGemmAuxGroups};
    CUresult r = g_encode_tiled(sc, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint16_t*>(s),
                                dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(TK_ERR_CUDA, "cuTensorMapEncodeTiled (scales) failed (%d)", (int)r);
  }
  {
    cuuint64_t dims[2] = {n / 2, k / gs};
    cuuint64_t strides[1] = {n / 2};
    cuuint32_t box[2] = {(cuuint32_t)(kGemmTileCols / 2), (cuuint32_t)kGemmAuxGroups};
    CUresult r = g_encode_tiled(ze, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(z),
                                dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(TK_ERR_CUDA, "cuTensorMapEncodeTiled (zero points) failed (%d)", (int)r);
  }
  return TK_OK;
}

// Weight maps of tile t: packed weights (swizzled for the tensor-memory kernel) and, for that
// kernel, the scale / zero-point maps.
int gemm_matrix_maps(GemmMaps& maps, int t, const uint8_t* w, const uint16_t* s, const uint8_t* z,
                     int n, int k, int gs, int nt) {
  const bool tm = gemm_use_tm(nt, k);
  int st = gemm_wtmap(w, n, k, tm, &maps.w[t]);
  if (st != TK_OK || !tm) return st;
  return gemm_auxmaps(s, z, n, k, gs, &maps.sc[t], &maps.ze[t]);
}

// One GEMM launch: colblocks CTA column tiles x token tiles x splits.
int gemm_run(tk_device* d, const GemmMaps& maps, GemmParams& p, int nt, int colblocks,
             cudaStream_t st) {
  const int avail = d->smem_optin - kStaticSmemReserve - 1024;
  size_t smem = 0;
  p.tm = gemm_use_tm(nt, p.K) ? 1 : 0;
  if (p.tm) {
    // dequantised tiles in tensor memory: shared memory holds the TMA ring and the scale ring
    p.a_stages = nt >= 128 ? 2 : 3;
    p.aux_stages = 3;
    p.raw_stage_bytes = gemm_tm_raw_stage_bytes(nt);
    p.raw_stages = std::min(kGemmMaxRawStages,
                            (avail - p.aux_stages * kGemmAuxStageBytes) / p.raw_stage_bytes);
    smem = 1024 + (size_t)p.raw_stages * p.raw_stage_bytes + (size_t)p.aux_stages * kGemmAuxStageBytes;
  } else {
    // a short ring of dequantised tiles, the rest of shared memory for the TMA ring
    p.a_stages = nt >= 128 ? 2 : 3;
    p.aux_stages = 0;
    p.raw_stage_bytes = gemm_raw_stage_bytes(nt);
    p.raw_stages = std::min(kGemmMaxRawStages, (avail - p.a_stages * kGemmAStageBytes) / p.raw_stage_bytes);
    smem = 1024 + (size_t)p.a_stages * kGemmAStageBytes + (size_t)p.raw_stages * p.raw_stage_bytes;
  }
  if (p.raw_stages < 2) return fail(TK_ERR_UNSUPPORTED, "GEMM stages do not fit in shared memory");
  p.err = d->err;
  p.timeout_ns = d->timeout_ns;
  p.trace = d->trace;
  p.trace_ctas = d->sm_count;
  if (d->trace)
    TK_CUDA_TRY(cudaMemsetAsync(d->trace, 0, (size_t)d->sm_count * kTraceEvents * 8, st));
  const dim3 grid((unsigned)colblocks, (unsigned)((p.M + nt - 1) / nt), (unsigned)p.splits);
  TK_LAUNCH(d, gemm_launch(nt, maps, p, grid, smem, st));
  return TK_OK;
}

// K splits so that the grid covers the SMs (each split a whole number of 64-k steps).
int gemm_splits(tk_device* d, int ctas, int k, int nt) {
  const int steps = k / (gemm_use_tm(nt, k) ? kGemmTmKStep : kGemmKStep);
  return std::max(1, std::min({steps, d->sm_count / ctas, 16}));
}

// y[m][n] (+)= x[m][k] . W for m >= 5 rows on the tensor cores.
int qmatmul_gemm(tk_device* d, const float* x, const uint8_t* w, const uint16_t* s,
                 const uint8_t* z, float* out, int m, int k, int n, int gs, cudaStream_t st) {
  const int nt = gemm_nt(m);
  int stt = scratch_ensure(d, d->g_x16, (size_t)m * k * 2);
  if (stt != TK_OK) return stt;
  __half* x16 = static_cast<__half*>(d->g_x16.ptr);
  TK_LAUNCH(d, launch_f32_to_f16(x, x16, (long long)m * k, st));
  GemmMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  if ((stt = act_tmap(x16, k, m, nt, &maps.x)) != TK_OK) return stt;
  if ((stt = gemm_matrix_maps(maps, 0, w, s, z, n, k, gs, nt)) != TK_OK) return stt;
  maps.w[1] = maps.w[0];
  maps.sc[1] = maps.sc[0];
  maps.ze[1] = maps.ze[0];
  GemmParams p;
  std::memset(&p, 0, sizeof(p));
  p.M = m;
  p.K = k;
  p.N = n;
  p.gs = gs;
  p.pair = 0;
  p.scales[0] = p.scales[1] = s;
  p.zeros[0] = p.zeros[1] = z;
  const int colblocks = n / (kGemmTiles * kGemmTileCols);
  p.splits = gemm_splits(d, colblocks * ((m + nt - 1) / nt), k, nt);
  if (p.splits == 1) {
    p.epi = kGemmStore;
    p.out = out;
    return gemm_run(d, maps, p, nt, colblocks, st);
  }
  stt = scratch_ensure(d, d->g_part, (size_t)p.splits * m * n * 4);
  if (stt != TK_OK) return stt;
  p.epi = kGemmPartial;
  p.out = static_cast<float*>(d->g_part.ptr);
  if ((stt = gemm_run(d, maps, p, nt, colblocks, st)) != TK_OK) return stt;
  TK_LAUNCH(d, launch_splitk_reduce(p.out, p.splits, (long long)m * n, nullptr, out, st));
  return TK_OK;
}

// The INT4 FFN for m >= 5 rows: rmsnorm (written as f16), gate/up GEMM with silu(gate) * up in its
// epilogue (h in f16 for the down GEMM, and in f32 when asked), down GEMM split over K,
// reduction (+ residual).
int ffn_gemm(tk_device* d, const float* x, const float* norm_w, const tk_int4_matrix* gate,
             const tk_int4_matrix* up, const tk_int4_matrix* down, float* out, float* h_out,
             int m, int hidden, int inter, int gs, float eps, bool residual, cudaStream_t st) {
  const int nt = gemm_nt(m);
  int stt;
  if ((stt = scratch_ensure(d, d->g_x16, (size_t)m * hidden * 2)) != TK_OK) return stt;
  if ((stt = scratch_ensure(d, d->g_h16, (size_t)m * inter * 2)) != TK_OK) return stt;
  __half* x16 = static_cast<__half*>(d->g_x16.ptr);
  __half* h16 = static_cast<__half*>(d->g_h16.ptr);
  TK_LAUNCH(d, launch_rmsnorm_f16(x, norm_w, x16, m, hidden, eps, st));
  // gate/up: tile 0 = gate, tile 1 = up at the same 128 columns
  GemmMaps ma;
  std::memset(&ma, 0, sizeof(ma));
  if ((stt = act_tmap(x16, hidden, m, nt, &ma.x)) != TK_OK) return stt;
  if ((stt = gemm_matrix_maps(ma, 0, gate->w_packed, gate->scales, gate->zeros, inter, hidden, gs,
                              nt)) != TK_OK)
    return stt;
  if ((stt = gemm_matrix_maps(ma, 1, up->w_packed, up->scales, up->zeros, inter, hidden, gs, nt)) !=
      TK_OK)
    return stt;
  GemmParams a;
  std::memset(&a, 0, sizeof(a));
  a.M = m;
  a.K = hidden;
  a.N = inter;
  a.gs = gs;
  a.splits = 1;
  a.pair = 1;
  a.scales[0] = gate->scales;
  a.scales[1] = up->scales;
  a.zeros[0] = gate->zeros;
  a.zeros[1] = up->zeros;
  a.epi = kGemmSiluMul;
  a.h16 = h16;
  a.h32 = h_out;
  if ((stt = gemm_run(d, ma, a, nt, inter / kGemmTileCols, st)) != TK_OK) return stt;
  // down: 256 adjacent output columns per CTA, K split to cover the SMs
  GemmMaps mb;
  std::memset(&mb, 0, sizeof(mb));
  if ((stt = act_tmap(h16, inter, m, nt, &mb.x)) != TK_OK) return stt;
  if ((stt = gemm_matrix_maps(mb, 0, down->w_packed, down->scales, down->zeros, hidden, inter, gs,
                              nt)) != TK_OK)
    return stt;
  mb.w[1] = mb.w[0];
  mb.sc[1] = mb.sc[0];
  mb.ze[1] = mb.ze[0];
  GemmParams b;
  std::memset(&b, 0, sizeof(b));
  b.M = m;
  b.K = inter;
  b.N = hidden;
  b.gs = gs;
  b.pair = 0;
  b.scales[0] = b.scales[1] = down->scales;
  b.zeros[0] = b.zeros[1] = down->zeros;
  const int colblocks = hidden / (kGemmTiles * kGemmTileCols);
  b.splits = gemm_splits(d, colblocks * ((m + nt - 1) / nt), inter, nt);
  if (b.splits == 1) {
    b.epi = kGemmStore;
    b.out = out;
    b.residual = residual ? x : nullptr;
    return gemm_run(d, mb, b, nt, colblocks, st);
  }
  if ((stt = scratch_ensure(d, d->g_part, (size_t)b.splits * m * hidden * 4)) != TK_OK) return stt;
  b.epi = kGemmPartial;
  b.out = static_cast<float*>(d->g_part.ptr);
  if ((stt = gemm_run(d, mb, b, nt, colblocks, st)) != TK_OK) return stt;
  TK_LAUNCH(d, launch_splitk_reduce(b.out, b.splits, (long long)m * hidden, residual ? x : nullptr,
                                   out, st));
  return TK_OK;
}

bool matrix_aligned(const tk_int4_matrix* a) {
  return a && aligned16(a->w_packed) && aligned16(a->scales) && aligned16(a->zeros);
}

}  // namespace

namespace tk {
namespace {
constexpr int kAttrGenDevices = 64;
std::atomic<unsigned> g_attr_gen[kAttrGenDevices];
}  // namespace
// Starts at 1 (a cache entry's 0 never matches); devices beyond the table share generation 1,
// which their callers' caches (also limited to 64 devices) do not keep anyway.
unsigned attr_generation(int dev) {
  return dev >= 0 && dev < kAttrGenDevices ? g_attr_gen[dev].load(std::memory_order_acquire) + 1u : 1u;
}
void bump_attr_generation(int dev) {
  if (dev >= 0 && dev < kAttrGenDevices) g_attr_gen[dev].fetch_add(1u, std::memory_order_acq_rel);
}
}  // namespace tk

extern "C" {

int tk_abi_version(void) { return TK_ABI_VERSION; }

const char* tk_last_error_string(void) { return g_last_error.c_str(); }

const char* tk_status_string(int status) {
  switch (status) {
    case TK_OK: return "ok";
    case TK_ERR_ARG: return "invalid argument";
    case TK_ERR_CUDA: return "CUDA error";
    case TK_ERR_NCCL: return "NCCL error";
    case TK_ERR_TIMEOUT: return "device-side wait timed out";
    case TK_ERR_UNSUPPORTED: return "unsupported";
    case TK_ERR_NOMEM: return "out of memory";
    default: return "unknown status";
  }
}

int tk_device_create(int ordinal, tk_device** out) {
  if (!out) return fail(TK_ERR_ARG, "out is NULL");
  *out = nullptr;
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0)
    return fail(TK_ERR_CUDA, "no CUDA device: %s", cudaGetErrorString(e));
  if (ordinal < 0 || ordinal >= count) return fail(TK_ERR_ARG, "device ordinal %d out of range", ordinal);
  tk_device* d = new tk_device();
  d->ordinal = ordinal;
  auto cleanup = [&](int st) {
    tk_device_destroy(d);
    return st;
  };
  if (cudaSetDevice(ordinal) != cudaSuccess) return cleanup(fail(TK_ERR_CUDA, "cudaSetDevice failed"));
  tk::bump_attr_generation(ordinal);
  if (cudaGetDeviceProperties(&d->prop, ordinal) != cudaSuccess)
    return cleanup(fail(TK_ERR_CUDA, "cudaGetDeviceProperties failed"));
  if (d->prop.major < 10)
    return cleanup(fail(TK_ERR_UNSUPPORTED, "device %d is sm_%d%d; this build targets sm_100a", ordinal,
                        d->prop.major, d->prop.minor));
  std::snprintf(d->name, sizeof(d->name), "%s", d->prop.name);
  d->sm_count = d->prop.multiProcessorCount;
  d->smem_optin = (int)d->prop.sharedMemPerBlockOptin;
  if (const char* env = std::getenv("TK_ENGINE_STAGES")) d->stages_override = std::atoi(env);
  if (const char* env = std::getenv("TK_FFN_SPLIT")) d->ffn_split = std::atoi(env);
  if (const char* env = std::getenv("TK_GEMM")) d->gemm_enabled = std::atoi(env);
  if (const char* env = std::getenv("TK_DOWN_PREFETCH")) d->down_prefetch = std::atoi(env);
  if (const char* env = std::getenv("TK_ENGINE_CTAS")) d->engine_ctas = std::atoi(env);
  if (const char* env = std::getenv("TK_DECODE")) d->decode_enabled = std::atoi(env);
  if (const char* env = std::getenv("TK_DECODE_PDL")) d->decode_pdl = std::atoi(env);
  if (const char* env = std::getenv("TK_WAIT_TIMEOUT_MS"))
    d->timeout_ns = (unsigned long long)std::atoll(env) * 1000000ull;
  if (cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking) != cudaSuccess)
    return cleanup(fail(TK_ERR_CUDA, "cudaStreamCreate failed"));
  if (cudaMalloc(&d->sync, sizeof(SyncState)) != cudaSuccess ||
      cudaMalloc(&d->err, 256) != cudaSuccess ||
      cudaHostAlloc(&d->err_host, kErrHostSlots * sizeof(unsigned), cudaHostAllocDefault) !=
          cudaSuccess)
    return cleanup(fail(TK_ERR_NOMEM, "scratch allocation failed"));
  if (cudaMemset(d->sync, 0, sizeof(SyncState)) != cudaSuccess || cudaMemset(d->err, 0, 256) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess)  // legacy-stream memsets: done before any kernel
    return cleanup(fail(TK_ERR_CUDA, "scratch init failed"));
  *out = d;
  return TK_OK;
}

void tk_device_destroy(tk_device* d) {
  if (!d) return;
  cudaSetDevice(d->ordinal);
  if (d->stream) cudaStreamSynchronize(d->stream);
  for (auto& g : d->ffn_graphs) {
    cudaGraphExecDestroy(g.exec);
    cudaFreeHost(g.err_host);
  }
  for (auto* b : {&d->frag[0], &d->partials[0], &d->partials[1], &d->counters[0],
                  &d->counters[1], &d->g_x16, &d->g_h16, &d->g_part, &d->dec, &d->io, &d->zero_rows})
    if (b->ptr) cudaFree(b->ptr);
  if (d->sync) cudaFree(d->sync);
  if (d->err) cudaFree(d->err);
  if (d->err_host) cudaFreeHost(d->err_host);
  if (d->trace) cudaFree(d->trace);
  if (d->stream) cudaStreamDestroy(d->stream);
  delete d;
}

const char* tk_device_name(tk_device* d) { return d ? d->name : ""; }
int tk_device_sm_count(tk_device* d) { return d ? d->sm_count : 0; }
uint64_t tk_device_launch_count(tk_device* d) { return d ? d->launches : 0; }
void* tk_device_stream(tk_device* d) { return d ? static_cast<void*>(d->stream) : nullptr; }

int tk_device_synchronize(tk_device* d) {
  if (!d) return fail(TK_ERR_ARG, "device is NULL");
  int st = set_device(d);
  if (st != TK_OK) return st;
  return sync_and_check(d, d->stream);
}

int tk_device_check_error(tk_device* d) {
  if (!d) return fail(TK_ERR_ARG, "device is NULL");
  unsigned h = 0;
  TK_CUDA_TRY(cudaMemcpy(&h, d->err, sizeof(h), cudaMemcpyDeviceToHost));
  if (h == 0) return TK_OK;
  if (h & (tk::kErrP2PWait | tk::kErrDecPeer)) ++d->p2p_timeouts;
  // Clear the error word and return the engine's scratch to its launch-ready state.
  TK_CUDA_TRY(cudaDeviceSynchronize());
  TK_CUDA_TRY(cudaMemset(d->err, 0, 256));
  TK_CUDA_TRY(cudaMemset(d->sync, 0, sizeof(SyncState)));
  for (auto* b : {&d->counters[0], &d->counters[1], &d->dec})
    if (b->ptr) TK_CUDA_TRY(cudaMemset(b->ptr, 0, b->cap));
  TK_CUDA_TRY(cudaDeviceSynchronize());  // the memsets (legacy stream) before the next kernel
  return fail(TK_ERR_TIMEOUT, "device-side bounded wait gave up (error bits 0x%x)", h);
}

int tk_device_trace_enable(tk_device* d, int enable) {
  if (!d) return fail(TK_ERR_ARG, "device is NULL");
  int st = set_device(d);
  if (st != TK_OK) return st;
  if (enable && !d->trace) {
    TK_CUDA_TRY(cudaDeviceSynchronize());
    TK_CUDA_TRY(cudaMalloc(&d->trace, (size_t)d->sm_count * kTraceEvents * 8));
    TK_CUDA_TRY(cudaMemset(d->trace, 0, (size_t)d->sm_count * kTraceEvents * 8));
    TK_CUDA_TRY(cudaDeviceSynchronize());
  } else if (!enable && d->trace) {
    TK_CUDA_TRY(cudaDeviceSynchronize());
    TK_CUDA_TRY(cudaFree(d->trace));
    d->trace = nullptr;
  }
  return TK_OK;
}

int tk_device_trace_read(tk_device* d, uint64_t* out, size_t max_values, size_t* n_values) {
  if (!d || !out) return fail(TK_ERR_ARG, "NULL argument");
  if (!d->trace) return fail(TK_ERR_ARG, "tracing is not enabled");
  const size_t n = std::min(max_values, (size_t)d->sm_count * kTraceEvents);
  int st = set_device(d);
  if (st != TK_OK) return st;
  TK_CUDA_TRY(cudaStreamSynchronize(d->stream));
  TK_CUDA_TRY(cudaMemcpy(out, d->trace, n * 8, cudaMemcpyDeviceToHost));
  if (n_values) *n_values = n;
  return TK_OK;
}

int tk_buffer_alloc(tk_device* d, size_t bytes, int kind, void** ptr) {
  if (!d || !ptr) return fail(TK_ERR_ARG, "NULL argument");
  *ptr = nullptr;
  if (bytes == 0) bytes = 16;
  int st = set_device(d);
  if (st != TK_OK) return st;
  cudaError_t e;
  switch (kind) {
    case TK_MEM_DEVICE: e = cudaMalloc(ptr, bytes); break;
    case TK_MEM_SHARED: e = cudaMallocManaged(ptr, bytes); break;
    case TK_MEM_HOST: e = cudaMallocHost(ptr, bytes); break;
    default: return fail(TK_ERR_ARG, "unknown buffer kind %d", kind);
  }
  if (e != cudaSuccess) return fail(TK_ERR_NOMEM, "allocation of %zu bytes failed: %s", bytes, cudaGetErrorString(e));
  return TK_OK;
}

int tk_buffer_free(tk_device* d, void* ptr) {
  if (!d) return fail(TK_ERR_ARG, "device is NULL");
  if (!ptr) return TK_OK;
  cudaPointerAttributes a;
  TK_CUDA_TRY(cudaPointerGetAttributes(&a, ptr));
  if (a.type == cudaMemoryTypeHost) TK_CUDA_TRY(cudaFreeHost(ptr));
  else TK_CUDA_TRY(cudaFree(ptr));
  return TK_OK;
}

int tk_buffer_upload(tk_device* d, void* dst, const void* src, size_t bytes) {
  if (!d || (!dst && bytes) || (!src && bytes)) return fail(TK_ERR_ARG, "NULL argument");
  int st = set_device(d);
  if (st != TK_OK) return st;
  TK_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, d->stream));
  TK_CUDA_TRY(cudaStreamSynchronize(d->stream));
  return TK_OK;
}

int tk_buffer_download(tk_device* d, void* dst, const void* src, size_t bytes) {
  if (!d || (!dst && bytes) || (!src && bytes)) return fail(TK_ERR_ARG, "NULL argument");
  int st = set_device(d);
  if (st != TK_OK) return st;
  TK_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, d->stream));
  TK_CUDA_TRY(cudaStreamSynchronize(d->stream));
  return TK_OK;
}

int tk_buffer_upload_async(tk_device* d, void* dst, const void* src, size_t bytes, void* stream) {
  if (!d || (!dst && bytes) || (!src && bytes)) return fail(TK_ERR_ARG, "NULL argument");
  int st = set_device(d);
  if (st != TK_OK) return st;
  TK_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, pick_stream(d, stream)));
  return TK_OK;
}

int tk_buffer_download_async(tk_device* d, void* dst, const void* src, size_t bytes, void* stream) {
  if (!d || (!dst && bytes) || (!src && bytes)) return fail(TK_ERR_ARG, "NULL argument");
  int st = set_device(d);
  if (st != TK_OK) return st;
  TK_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, pick_stream(d, stream)));
  return TK_OK;
}

int tk_matvec_dual_async(tk_device* d, const float* x, const float* W1, const float* W2, float* out1,
                         float* out2, uint32_t K, uint32_t N, void* stream) {
  if (!d || !x || !W1 || !out1) return fail(TK_ERR_ARG, "NULL argument");
  if ((W2 == nullptr) != (out2 == nullptr)) return fail(TK_ERR_ARG, "W2 and out2 go together");
  if (K == 0 || N == 0) return fail(TK_ERR_ARG, "K and N must be positive");
  int st = set_device(d);
  if (st != TK_OK) return st;
  TK_LAUNCH(d, launch_matvec_f32(x, W1, W2, out1, out2, (int)K, (int)N, d->sm_count,
                                 pick_stream(d, stream)));
  return TK_OK;
}

int tk_matvec_dual(tk_device* d, const float* x, const float* W1, const float* W2, float* out1,
                   float* out2, uint32_t K, uint32_t N) {
  if (!W2 || !out2) return fail(TK_ERR_ARG, "NULL argument");
  int st = tk_matvec_dual_async(d, x, W1, W2, out1, out2, K, N, nullptr);
  if (st != TK_OK) return st;
  return sync_and_check(d, d->stream);
}

int tk_matvec_async(tk_device* d, const float* x, const float* W, float* out, uint32_t K,
                    uint32_t N, void* stream) {
  return tk_matvec_dual_async(d, x, W, nullptr, out, nullptr, K, N, stream);
}

int tk_matvec(tk_device* d, const float* x, const float* W, float* out, uint32_t K, uint32_t N) {
  int st = tk_matvec_async(d, x, W, out, K, N, nullptr);
  if (st != TK_OK) return st;
  return sync_and_check(d, d->stream);
}

int tk_repack_q4_0(tk_device* d, const void* blocks, uint8_t* w, uint16_t* s, uint8_t* z,
                   uint32_t n, uint32_t k, int order) {
  if (!d || !blocks || !w || !s || !z) return fail(TK_ERR_ARG, "NULL argument");
  if (n == 0 || k == 0 || k % 32 || n % 2)
    return fail(TK_ERR_ARG, "Q4_0 repack needs k %% 32 == 0 and an even row count (k=%u, n=%u)", k, n);
  if (order != TK_Q4_0_REFERENCE_ORDER && order != TK_Q4_0_GGML_ORDER)
    return fail(TK_ERR_ARG, "unknown Q4_0 nibble order %d", order);
  int st = set_device(d);
  if (st != TK_OK) return st;
  TK_LAUNCH(d, launch_repack_q4_0(static_cast<const uint8_t*>(blocks), w, s, z, (int)n, (int)k, order,
                                  d->stream));
  return sync_and_check(d, d->stream);
}

int tk_paged_attention_async(tk_device* d, const float* q, const float* kc, const float* vc,
                             const int32_t* bt, const int32_t* cl, float* o, uint32_t batch,
                             uint32_t heads, uint32_t head_dim, uint32_t max_blocks, void* stream) {
  if (!d || !q || !kc || !vc || !bt || !cl || !o) return fail(TK_ERR_ARG, "NULL argument");
  if (batch == 0 || heads == 0 || head_dim == 0 || head_dim > 128 || max_blocks == 0 ||
      batch > 65535 || heads > (1u << 20))
    return fail(TK_ERR_ARG, "paged attention needs batch, heads, max_blocks > 0 and head_dim <= 128");
  int st = set_device(d);
  if (st != TK_OK) return st;
  TK_LAUNCH(d, launch_paged_attention(q, kc, vc, bt, cl, o, (int)batch, (int)heads, (int)head_dim,
                                      (int)max_blocks, 1.0f / sqrtf((float)head_dim),
                                      pick_stream(d, stream)));
  return TK_OK;
}

int tk_paged_attention(tk_device* d, const float* q, const float* kc, const float* vc,
                       const int32_t* bt, const int32_t* cl, float* o, uint32_t batch,
                       uint32_t heads, uint32_t head_dim, uint32_t max_blocks) {
  int st = tk_paged_attention_async(d, q, kc, vc, bt, cl, o, batch, heads, head_dim, max_blocks,
                                    nullptr);
  if (st != TK_OK) return st;
  return sync_and_check(d, d->stream);
}

int tk_argmax_async(tk_device* d, const float* x, uint32_t n, uint32_t* out, void* stream) {
  if (!d || !x || !out) return fail(TK_ERR_ARG, "NULL argument");
  if (n == 0 || n > (1u << 30)) return fail(TK_ERR_ARG, "argmax length %u out of range", n);
  int st = set_device(d);
  if (st != TK_OK) return st;
  TK_LAUNCH(d, launch_argmax(x, (int)n, out, pick_stream(d, stream)));
  return TK_OK;
}

int tk_argmax(tk_device* d, const float* x, uint32_t n, uint32_t* out) {
  int st = tk_argmax_async(d, x, n, out, nullptr);
  if (st != TK_OK) return st;
  return sync_and_check(d, d->stream);
}

int tk_softmax_sample_async(tk_device* d, const float* logits, float* probs, uint32_t* sampled,
                            uint32_t vocab, float temperature, float random_val, void* stream) {
  if (!d || !logits || !probs || !sampled) return fail(TK_ERR_ARG, "NULL argument");
  if (vocab == 0 || vocab > (1u << 30)) return fail(TK_ERR_ARG, "vocabulary size %u out of range", vocab);
  if (!(temperature > 0.f)) return fail(TK_ERR_ARG, "temperature must be positive");
  int st = set_device(d);
  if (st != TK_OK) return st;
  TK_LAUNCH(d, launch_softmax_sample(logits, probs, sampled, (int)vocab, temperature, random_val,
                                     pick_stream(d, stream)));
  return TK_OK;
}

int tk_softmax_sample(tk_device* d, const float* logits, float* probs, uint32_t* sampled,
                      uint32_t vocab, float temperature, float random_val) {
  int st = tk_softmax_sample_async(d, logits, probs, sampled, vocab, temperature, random_val, nullptr);
  if (st != TK_OK) return st;
  return sync_and_check(d, d->stream);
}

int tk_qmatmul_int4_path(uint32_t m, uint32_t k, uint32_t n, uint32_t gs) {
  if (m == 0 || k == 0 || n == 0 || gs == 0 || gs % 8 || k % gs || n % 2) return -1;
  if (!engine_shape(k, n, gs)) return 0;
  if (m >= kGemmMinRows && gemm_shape(k, n, gs, false)) return 2;
  // chunks of up to kDecMaxRows rows, each a decode launch when its instantiation fits
  const int mc = std::min<int>((int)m, kDecMaxRows);
  return decode_shape(mc, (int)k, (int)n, 0, (int)gs, kDefaultGrid, false) ? 3 : 1;
}

int tk_int4_ffn_path(uint32_t m, uint32_t hidden, uint32_t inter, uint32_t gs) {
  if (m == 0 || hidden == 0 || inter == 0 || gs == 0 || gs % 8 || hidden % gs || inter % gs ||
      hidden % 2 || inter % 2)
    return -1;
  if (!engine_shape(hidden, inter, gs) || !engine_shape(inter, hidden, gs)) return 0;
  if (m >= kGemmMinRows && gemm_shape(hidden, inter, gs, true) && gemm_shape(inter, hidden, gs, false))
    return 2;
  const int mc = std::min<int>((int)m, kDecMaxRows);
  return decode_shape(mc, (int)hidden, 0, (int)inter, (int)gs, kDefaultGrid, true) ? 3 : 1;
}

int tk_qmatmul_int4_async(tk_device* d, const float* x, const uint8_t* w, const uint16_t* s,
                          const uint8_t* z, float* out, uint32_t m, uint32_t k, uint32_t n,
                          uint32_t gs, void* stream) {
  if (!d || !x || !w || !s || !z || !out) return fail(TK_ERR_ARG, "NULL argument");
  int st = check_qshape(m, k, n, gs);
  if (st != TK_OK) return st;
  st = set_device(d);
  if (st != TK_OK) return st;
  cudaStream_t cs = pick_stream(d, stream);
  const bool fast = engine_shape(k, n, gs) && aligned16(x) && aligned16(w) && aligned16(s) &&
                    aligned16(z) && aligned16(out);
  if (!fast) {
    TK_LAUNCH(d, launch_qmatmul_int4_generic(x, w, s, z, out, (int)m, (int)k, (int)n, (int)gs, cs));
    return TK_OK;
  }
  if (d->gemm_enabled && m >= kGemmMinRows && gemm_shape(k, n, gs, false))
    return qmatmul_gemm(d, x, w, s, z, out, (int)m, (int)k, (int)n, (int)gs, cs);
  for (uint32_t r = 0; r < m; r += 4) {
    const uint32_t mm = std::min<uint32_t>(4, m - r);
    if ((int)mm <= kDecMaxRows && d->decode_enabled) {
      const tk_int4_matrix a{w, s, z};
      st = decode_run(d, x + (size_t)r * k, nullptr, 0.f, &a, nullptr, nullptr, out + (size_t)r * n,
                      nullptr, (int)mm, (int)k, (int)n, 0, (int)gs, false, cs);
      if (st == TK_OK) continue;
      if (st != TK_ERR_UNSUPPORTED) return st;
    }
    st = qmatmul_engine_chunk(d, x + (size_t)r * k, w, s, z, out + (size_t)r * n, (int)mm, (int)k,
                              (int)n, (int)gs, cs);
    if (st != TK_OK) return st;
  }
  return TK_OK;
}

int tk_qmatmul_int4(tk_device* d, const float* x, const uint8_t* w, const uint16_t* s,
                    const uint8_t* z, float* out, uint32_t m, uint32_t k, uint32_t n, uint32_t gs) {
  int st = tk_qmatmul_int4_async(d, x, w, s, z, out, m, k, n, gs, nullptr);
  if (st != TK_OK) return st;
  return sync_and_check(d, d->stream);
}

int tk_dequant_int4(tk_device* d, const uint8_t* w, const uint16_t* s, const uint8_t* z,
                    float* out, uint32_t k, uint32_t n, uint32_t gs) {
  if (!d || !w || !s || !z || !out) return fail(TK_ERR_ARG, "NULL argument");
  int st = check_qshape(1, k, n, gs);
  if (st != TK_OK) return st;
  st = set_device(d);
  if (st != TK_OK) return st;
  TK_LAUNCH(d, launch_dequant_int4(w, s, z, out, (int)k, (int)n, (int)gs, d->stream));
  return sync_and_check(d, d->stream);
}

int tk_rmsnorm_async(tk_device* d, const float* x, const float* w, float* out, uint32_t rows,
                     uint32_t dim, float eps, void* stream) {
  if (!d || !x || !w || !out) return fail(TK_ERR_ARG, "NULL argument");
  if (rows == 0 || dim == 0) return fail(TK_ERR_ARG, "zero dimension");
  int st = set_device(d);
  if (st != TK_OK) return st;
  TK_LAUNCH(d, launch_rmsnorm(x, w, out, (int)rows, (int)dim, eps, pick_stream(d, stream)));
  return TK_OK;
}

int tk_rmsnorm(tk_device* d, const float* x, const float* w, float* out, uint32_t rows,
               uint32_t dim, float eps) {
  int st = tk_rmsnorm_async(d, x, w, out, rows, dim, eps, nullptr);
  if (st != TK_OK) return st;
  return sync_and_check(d, d->stream);
}

int tk_fused_rmsnorm_rope_async(tk_device* d, const float* x, const float* w, const float* cosc,
                                const float* sinc, float* out, uint32_t rows, uint32_t dim,
                                uint32_t head_dim, uint32_t pos, float eps, void* stream) {
  if (!d || !x || !w || !cosc || !sinc || !out) return fail(TK_ERR_ARG, "NULL argument");
  if (rows == 0 || dim == 0 || head_dim == 0 || head_dim % 2 || dim % head_dim)
    return fail(TK_ERR_ARG, "dim=%u must be a positive multiple of an even head_dim=%u", dim, head_dim);
  int st = set_device(d);
  if (st != TK_OK) return st;
  TK_LAUNCH(d, launch_fused_rmsnorm_rope(x, w, cosc, sinc, out, (int)rows, (int)dim, (int)head_dim,
                                        (int)pos, eps, pick_stream(d, stream)));
  return TK_OK;
}

int tk_fused_rmsnorm_rope(tk_device* d, const float* x, const float* w, const float* cosc,
                          const float* sinc, float* out, uint32_t rows, uint32_t dim,
                          uint32_t head_dim, uint32_t pos, float eps) {
  int st = tk_fused_rmsnorm_rope_async(d, x, w, cosc, sinc, out, rows, dim, head_dim, pos, eps, nullptr);
  if (st != TK_OK) return st;
  return sync_and_check(d, d->stream);
}

int tk_silu_mul_async(tk_device* d, const float* g, const float* u, float* out, uint32_t n,
                      void* stream) {
  if (!d || !g || !u || !out) return fail(TK_ERR_ARG, "NULL argument");
  if (n == 0) return TK_OK;
  int st = set_device(d);
  if (st != TK_OK) return st;
  TK_LAUNCH(d, launch_silu_mul(g, u, out, (int)n, pick_stream(d, stream)));
  return TK_OK;
}

int tk_silu_mul(tk_device* d, const float* g, const float* u, float* out, uint32_t n) {
  int st = tk_silu_mul_async(d, g, u, out, n, nullptr);
  if (st != TK_OK) return st;
  return sync_and_check(d, d->stream);
}

int tk_int4_ffn_async(tk_device* d, const float* x, const float* norm_w, const tk_int4_matrix* gate,
                      const tk_int4_matrix* up, const tk_int4_matrix* down, float* out,
                      float* h_out, uint32_t m, uint32_t hidden, uint32_t inter, uint32_t gs,
                      float eps, uint32_t flags, void* stream) {
  if (!d || !x || !norm_w || !gate || !up || !down || !out) return fail(TK_ERR_ARG, "NULL argument");
  for (const tk_int4_matrix* a : {gate, up, down})
    if (!a->w_packed || !a->scales || !a->zeros) return fail(TK_ERR_ARG, "NULL matrix pointer");
  int st = check_qshape(m, hidden, inter, gs);
  if (st != TK_OK) return st;
  st = check_qshape(m, inter, hidden, gs);
  if (st != TK_OK) return st;
  if (flags & ~(TK_FFN_RESIDUAL | TK_FFN_HOST_IO))
    return fail(TK_ERR_ARG, "unknown flags 0x%x", flags);
  st = set_device(d);
  if (st != TK_OK) return st;
  cudaStream_t cs = pick_stream(d, stream);
  const bool residual = (flags & TK_FFN_RESIDUAL) != 0;
  if (flags & TK_FFN_HOST_IO) {
    // x and out in pinned host memory.  The batch 1-2 decode kernel reads x over the host link
    // itself (each CTA a share, passed on to the others through device memory) and writes out
    // there; the other paths stage both through device scratch with copies.
    const bool aligned = aligned16(x) && aligned16(norm_w) && aligned16(out) &&
                         (!h_out || aligned16(h_out)) && matrix_aligned(gate) &&
                         matrix_aligned(up) && matrix_aligned(down);
    if ((int)m <= kDecMaxRows && d->decode_enabled && aligned && engine_shape(hidden, inter, gs) &&
        engine_shape(inter, hidden, gs)) {
      st = decode_run(d, x, norm_w, eps, gate, up, down, out, h_out, (int)m, (int)hidden, 0,
                      (int)inter, (int)gs, residual, cs, true);
      if (st != TK_ERR_UNSUPPORTED) return st;
    }
    const size_t bytes = (size_t)m * hidden * sizeof(float);
    if ((st = scratch_ensure(d, d->io, 2 * bytes)) != TK_OK) return st;
    float* xd = static_cast<float*>(d->io.ptr);
    float* od = xd + (size_t)m * hidden;
    TK_CUDA_TRY(cudaMemcpyAsync(xd, x, bytes, cudaMemcpyHostToDevice, cs));
    st = tk_int4_ffn_async(d, xd, norm_w, gate, up, down, od, h_out, m, hidden, inter, gs, eps,
                           flags & ~TK_FFN_HOST_IO, stream);
    if (st != TK_OK) return st;
    TK_CUDA_TRY(cudaMemcpyAsync(out, od, bytes, cudaMemcpyDeviceToHost, cs));
    return TK_OK;
  }
  const bool fast = engine_shape(hidden, inter, gs) && engine_shape(inter, hidden, gs) &&
                    aligned16(x) && aligned16(norm_w) && aligned16(out) &&
                    (!h_out || aligned16(h_out)) && matrix_aligned(gate) && matrix_aligned(up) &&
                    matrix_aligned(down);
  if (fast && d->gemm_enabled && m >= kGemmMinRows && gemm_shape(hidden, inter, gs, true) &&
      gemm_shape(inter, hidden, gs, false))
    return ffn_gemm(d, x, norm_w, gate, up, down, out, h_out, (int)m, (int)hidden, (int)inter,
                    (int)gs, eps, residual, cs);
  if (fast) {
    for (uint32_t r = 0; r < m; r += 4) {
      const uint32_t mm = std::min<uint32_t>(4, m - r);
      if ((int)mm <= kDecMaxRows && d->decode_enabled) {
        st = decode_run(d, x + (size_t)r * hidden, norm_w, eps, gate, up, down,
                        out + (size_t)r * hidden, h_out ? h_out + (size_t)r * inter : nullptr,
                        (int)mm, (int)hidden, 0, (int)inter, (int)gs, residual, cs);
        if (st == TK_OK) continue;
        if (st != TK_ERR_UNSUPPORTED) return st;
      }
      st = ffn_engine_chunk(d, x + (size_t)r * hidden, norm_w, gate, up, down,
                            out + (size_t)r * hidden, h_out ? h_out + (size_t)r * inter : nullptr,
                            (int)mm, (int)hidden, (int)inter, (int)gs, eps, residual, cs);
      if (st != TK_OK) return st;
    }
    return TK_OK;
  }
  // CUDA-core composition for shapes the engine does not take.
  float *normed = nullptr, *g = nullptr, *u = nullptr, *h = nullptr, *y = nullptr;
  const size_t mh = (size_t)m * hidden, mi = (size_t)m * inter;
  TK_CUDA_TRY(cudaMallocAsync(&normed, mh * 4, cs));
  TK_CUDA_TRY(cudaMallocAsync(&g, mi * 4, cs));
  TK_CUDA_TRY(cudaMallocAsync(&u, mi * 4, cs));
  TK_CUDA_TRY(cudaMallocAsync(&h, mi * 4, cs));
  TK_CUDA_TRY(cudaMallocAsync(&y, mh * 4, cs));
  TK_LAUNCH(d, launch_rmsnorm(x, norm_w, normed, (int)m, (int)hidden, eps, cs));
  TK_LAUNCH(d, launch_qmatmul_int4_generic(normed, gate->w_packed, gate->scales, gate->zeros, g, (int)m,
                                          (int)hidden, (int)inter, (int)gs, cs));
  TK_LAUNCH(d, launch_qmatmul_int4_generic(normed, up->w_packed, up->scales, up->zeros, u, (int)m,
                                          (int)hidden, (int)inter, (int)gs, cs));
  TK_LAUNCH(d, launch_silu_mul(g, u, h, (int)mi, cs));
  if (h_out) TK_CUDA_TRY(cudaMemcpyAsync(h_out, h, mi * 4, cudaMemcpyDeviceToDevice, cs));
  TK_LAUNCH(d, launch_qmatmul_int4_generic(h, down->w_packed, down->scales, down->zeros, y, (int)m,
                                          (int)inter, (int)hidden, (int)gs, cs));
  if (residual) TK_LAUNCH(d, launch_add(x, y, out, (int)mh, cs));
  else TK_CUDA_TRY(cudaMemcpyAsync(out, y, mh * 4, cudaMemcpyDeviceToDevice, cs));
  for (float* p : {normed, g, u, h, y}) TK_CUDA_TRY(cudaFreeAsync(p, cs));
  return TK_OK;
}

int tk_int4_ffn(tk_device* d, const float* x, const float* norm_w, const tk_int4_matrix* gate,
                const tk_int4_matrix* up, const tk_int4_matrix* down, float* out, float* h_out,
                uint32_t m, uint32_t hidden, uint32_t inter, uint32_t gs, float eps,
                uint32_t flags) {
  const bool graphable = (flags & TK_FFN_HOST_IO) && d && gate && up && down && !d->trace;
  FfnGraph key{};
  if (graphable) {
    const void* ptrs[13] = {x, norm_w, gate->w_packed, gate->scales, gate->zeros, up->w_packed,
                            up->scales, up->zeros, down->w_packed, down->scales, down->zeros, out,
                            h_out};
    std::memcpy(key.ptr, ptrs, sizeof(ptrs));
    const uint32_t shape[5] = {m, hidden, inter, gs, flags};
    std::memcpy(key.shape, shape, sizeof(shape));
    std::memcpy(&key.eps_bits, &eps, sizeof(eps));
    int st = set_device(d);
    if (st != TK_OK) return st;
    static unsigned long long use_clock = 0;
    for (auto& g : d->ffn_graphs)
      if (g.gen == d->scratch_gen && !std::memcmp(g.ptr, key.ptr, sizeof(key.ptr)) &&
          !std::memcmp(g.shape, key.shape, sizeof(key.shape)) && g.eps_bits == key.eps_bits) {
        g.last_use = ++use_clock;
        *static_cast<volatile unsigned*>(g.err_host) = 0u;
        TK_CUDA_TRY(cudaGraphLaunch(g.exec, d->stream));
        TK_CUDA_TRY(cudaStreamSynchronize(d->stream));
        if (*static_cast<volatile unsigned*>(g.err_host) == 0) return TK_OK;
        return tk_device_check_error(d);  // reports the timeout and resets the scratch
      }
  }
  int st = tk_int4_ffn_async(d, x, norm_w, gate, up, down, out, h_out, m, hidden, inter, gs, eps,
                             flags, nullptr);
  if (st != TK_OK) return st;
  st = sync_and_check(d, d->stream);
  if (st != TK_OK || !graphable) return st;
  // The call ran (and sized every scratch buffer): record it for the next identical call.  A
  // failed recording only costs the speed-up.
  unsigned* err_host = nullptr;
  if (cudaHostAlloc(reinterpret_cast<void**>(&err_host), sizeof(unsigned), cudaHostAllocDefault) !=
      cudaSuccess) {
    cudaGetLastError();
    return TK_OK;
  }
  *err_host = 0;
  const unsigned gen = d->scratch_gen;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  bool ok = cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
  if (ok) {
    // the decode kernel reports a failure to err_host itself; the other paths' graphs end with a
    // copy of the device error word
    d->capture_err_host = err_host;
    d->capture_err_used = false;
    const int rs = tk_int4_ffn_async(d, x, norm_w, gate, up, down, out, h_out, m, hidden, inter,
                                     gs, eps, flags, nullptr);
    d->capture_err_host = nullptr;
    const bool copied =
        rs == TK_OK && (d->capture_err_used ||
                        cudaMemcpyAsync(err_host, d->err, sizeof(unsigned), cudaMemcpyDeviceToHost,
                                        d->stream) == cudaSuccess);
    ok = cudaStreamEndCapture(d->stream, &graph) == cudaSuccess && copied;
  }
  if (ok) ok = cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess;
  if (graph) cudaGraphDestroy(graph);
  cudaGetLastError();
  if (!ok || gen != d->scratch_gen) {
    if (exec) cudaGraphExecDestroy(exec);
    cudaFreeHost(err_host);
    return TK_OK;
  }
  key.gen = gen;
  key.exec = exec;
  key.err_host = err_host;
  key.last_use = 0;
  constexpr size_t kMaxGraphs = 64;  // e.g. every layer of a 32-layer decode stack
  if (d->ffn_graphs.size() >= kMaxGraphs) {
    auto lru = std::min_element(d->ffn_graphs.begin(), d->ffn_graphs.end(),
                                [](const FfnGraph& a, const FfnGraph& b) { return a.last_use < b.last_use; });
    cudaGraphExecDestroy(lru->exec);
    cudaFreeHost(lru->err_host);
    d->ffn_graphs.erase(lru);
  }
  d->ffn_graphs.push_back(key);
  return TK_OK;
}

}  // extern "C"

// ---- qmatmul_int4 without any allocation ------------------------------------------------
//
// Some callers cannot call cudaMalloc: a host whose device memory is entirely reserved up
// front by its own allocator (an inference server's memory pool, a framework arena), a
// latency-critical loop where cudaMalloc's implicit device-wide synchronisation is not
// acceptable, or a foreign-language binding that cannot own a tk_device and its arena.
// tk_qmatmul_int4_noalloc serves them: the engine's scratch (split-K partials, tile
// counters, activation records, launch state and error word) lives in the file-scope
// array below instead of in buffers the device context allocates.
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // TK_NOALLOC_SCRATCH_BYTES
constexpr size_t kNoAllocErrBytes = 256;  // the error word's slot at the start of the array
constexpr int kNoAllocMaxDevices = 64;

// One copy per GPU that loads this library, held until the process exits.  In host code
// `g_noalloc_scratch` is only a host-side stand-in for the symbol: its device address comes
// from cudaGetSymbolAddress (noalloc_scratch below) and is what the kernel is given.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
unsigned char* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of the scratch array on the current device (set up once per device).
int noalloc_scratch(int ordinal, unsigned char** out) {
  if (ordinal < 0 || ordinal >= kNoAllocMaxDevices)
    return fail(TK_ERR_UNSUPPORTED, "device ordinal %d is beyond the %d devices supported", ordinal,
                kNoAllocMaxDevices);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[ordinal]) {
    void* p = nullptr;
    TK_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    g_noalloc_ptr[ordinal] = static_cast<unsigned char*>(p);
  }
  *out = g_noalloc_ptr[ordinal];
  return TK_OK;
}

// Tensor map of one matrix's packed weights, encoded on the stack (no cache, no heap).
int noalloc_tmap(const void* base, uint64_t cols, uint64_t rows, uint32_t box_rows,
                 CUtensorMap* out) {
  int st = get_encoder();
  if (st != TK_OK) return st;
  cuuint64_t dims[2] = {cols / 8, rows};
  cuuint64_t strides[1] = {cols};
  cuuint32_t box[2] = {(cuuint32_t)kRowElems, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode_tiled(out, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(base), dims,
                              strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TK_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return TK_OK;
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// One engine launch (<= 4 rows) with every scratch pointer carved from `scratch`.
int noalloc_engine_chunk(unsigned char* scratch, int sm_count, int smem_optin, const float* x,
                         const uint8_t* w, const uint16_t* s, const uint8_t* z, float* out, int m,
                         int k, int n, int gs, cudaStream_t st) {
  const int mt = mt_for(m);
  const long long Wtot = sm_count;
  EngineParams p;
  std::memset(&p, 0, sizeof(p));
  p.m = m;
  p.nphases = 1;
  PhaseParams& P = p.ph[0];
  fill_phase(P, k, n, gs, 1, mt);
  P.maxseg = max_segments(P, Wtot);
  P.red_first = 0;
  P.red_count = 1;
  // layout: error word | launch state | tile counters | partials | per-CTA records.  The error
  // word is cleared once per call (tk_qmatmul_int4_noalloc), before the first chunk, so that a
  // timed-out wait in any chunk is still set when the word is read after the last one.
  const size_t off_sync = kNoAllocErrBytes;
  const size_t off_cnt = off_sync + align256(sizeof(SyncState));
  const size_t off_part = off_cnt + align256((size_t)(n / kTileCols) * sizeof(unsigned));
  const size_t part_bytes =
      (size_t)P.tiles * P.nmat * P.maxseg * kSlices * mt * kTileCols * sizeof(float);
  const size_t off_rec = off_part + align256(part_bytes);
  const long long rec_stride = (long long)P.groups * P.frag_bytes;
  const size_t need = off_rec + (size_t)Wtot * rec_stride;
  if (need > kNoAllocScratchBytes)
    return fail(TK_ERR_ARG,
                "m=%d k=%d n=%d group_size=%d needs %zu bytes of scratch; the allocation-free "
                "entry point has %zu (use tk_qmatmul_int4)",
                m, k, n, gs, need, kNoAllocScratchBytes);
  // the launch state and tile counters must start at zero; the partials and records are
  // written before they are read
  TK_CUDA_TRY(cudaMemsetAsync(scratch + off_sync, 0, off_part - off_sync, st));
  P.map_base = 0;
  P.scales[0] = s;
  P.zeros[0] = z;
  P.frag_in = scratch + off_rec;
  P.frag_cta_stride = rec_stride;
  P.partials = reinterpret_cast<float*>(scratch + off_part);
  P.counters = reinterpret_cast<unsigned*>(scratch + off_cnt);
  P.epi = kEpiStore;
  P.out = out;
  P.ldo = n;
  p.x = x;
  p.ldx = k;
  p.K0 = k;
  p.do_norm = 0;
  p.frag0 = scratch + off_rec;
  p.frag0_cta_stride = rec_stride;
  p.gs0 = gs;
  p.frag0_bytes = P.frag_bytes;
  TmapPack maps;
  std::memset(&maps, 0, sizeof(maps));
  int stt = noalloc_tmap(w, n, k / 2, (uint32_t)(gs / 2), &maps.map[0]);
  if (stt != TK_OK) return stt;
  stt = noalloc_tmap(w, n, k / 2, (uint32_t)kStepRows, &maps.map[1]);
  if (stt != TK_OK) return stt;
  p.tile_stage_bytes = (P.spg * kStepRows * kRowBytes + 127) & ~127;
  p.aux_stage_bytes = (kSlices * (kScaleBytes + kZeroBytes) + P.frag_bytes + 15) & ~15;
  int stages = 0, rec0_smem = 0;
  size_t smem = 0;
  if (!engine_plan_smem(p.tile_stage_bytes, p.aux_stage_bytes, P.groups * P.frag_bytes,
                        smem_optin - kStaticSmemReserve, &stages, &rec0_smem, &smem))
    return fail(TK_ERR_UNSUPPORTED, "engine ring does not fit in shared memory");
  p.stages = stages;
  p.rec0_smem = rec0_smem;
  p.trace = nullptr;
  p.sync = reinterpret_cast<SyncState*>(scratch + off_sync);
  p.err = reinterpret_cast<unsigned*>(scratch);
  p.timeout_ns = kDefaultTimeoutNs;
  int blocks = 0;
  TK_CUDA_TRY(engine_occupancy(mt, p.gs0, smem, &blocks));
  if (blocks < 1) return fail(TK_ERR_UNSUPPORTED, "engine kernel cannot be resident");
  TK_CUDA_TRY(engine_launch(mt, p.gs0, maps, p, sm_count, smem, st));
  return TK_OK;
}

}  // namespace

extern "C" int tk_qmatmul_int4_noalloc(const float* x, const uint8_t* w, const uint16_t* s,
                                       const uint8_t* z, float* out, uint32_t m, uint32_t k,
                                       uint32_t n, uint32_t gs, void* stream) {
  if (!x || !w || !s || !z || !out) return fail(TK_ERR_ARG, "NULL argument");
  int st = check_qshape(m, k, n, gs);
  if (st != TK_OK) return st;
  int ordinal = 0;
  TK_CUDA_TRY(cudaGetDevice(&ordinal));
  cudaStream_t cs = static_cast<cudaStream_t>(stream);
  const bool fast = engine_shape(k, n, gs) && aligned16(x) && aligned16(w) && aligned16(s) &&
                    aligned16(z) && aligned16(out);
  if (!fast) {
    // the CUDA-core kernel these shapes take uses no scratch at all
    TK_CUDA_TRY(launch_qmatmul_int4_generic(x, w, s, z, out, (int)m, (int)k, (int)n, (int)gs, cs));
    TK_CUDA_TRY(cudaStreamSynchronize(cs));
    return TK_OK;
  }
  unsigned char* scratch = nullptr;
  st = noalloc_scratch(ordinal, &scratch);
  if (st != TK_OK) return st;
  int sm_count = 0, smem_optin = 0, major = 0;
  TK_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, ordinal));
  if (major < 10) return fail(TK_ERR_UNSUPPORTED, "device %d is not sm_100a", ordinal);
  TK_CUDA_TRY(cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, ordinal));
  TK_CUDA_TRY(cudaDeviceGetAttribute(&smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, ordinal));
  // the error word (the array's first bytes) starts at zero once per call and collects the
  // error bits of every chunk
  TK_CUDA_TRY(cudaMemsetAsync(scratch, 0, kNoAllocErrBytes, cs));
  for (uint32_t r = 0; r < m; r += 4) {
    const uint32_t mm = std::min<uint32_t>(4, m - r);
    st = noalloc_engine_chunk(scratch, sm_count, smem_optin, x + (size_t)r * k, w, s, z,
                              out + (size_t)r * n, (int)mm, (int)k, (int)n, (int)gs, cs);
    if (st != TK_OK) return st;
  }
  TK_CUDA_TRY(cudaStreamSynchronize(cs));
  unsigned h = 0;
  TK_CUDA_TRY(cudaMemcpy(&h, scratch, sizeof(h), cudaMemcpyDeviceToHost));
  if (h != 0) return fail(TK_ERR_TIMEOUT, "device-side bounded wait gave up (error bits 0x%x)", h);
  return TK_OK;
}

// ---- tensor parallelism: NCCL resolved at first use ----------------------------------------

namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
};

std::once_flag g_nccl_once;
NcclApi g_nccl;

int nccl_api(const NcclApi** out) {
  // Which NCCL: TK_NCCL_LIB (a path) first, then a libnccl.so.2 the process already holds (a
  // framework's own), then the loader's search.  All other code in the process that links
  // libnccl.so.2 binds to whichever copy is loaded first, so an older system NCCL loaded here
  // ahead of a framework's newer one would leave the framework's symbols unresolved.
  std::call_once(g_nccl_once, [] {
    void* h = nullptr;
    if (const char* lib = getenv("TK_NCCL_LIB"); lib && *lib) h = dlopen(lib, RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    g_nccl.get_unique_id = reinterpret_cast<decltype(g_nccl.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    g_nccl.comm_init_rank = reinterpret_cast<decltype(g_nccl.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    g_nccl.all_reduce = reinterpret_cast<decltype(g_nccl.all_reduce)>(dlsym(h, "ncclAllReduce"));
    g_nccl.all_gather = reinterpret_cast<decltype(g_nccl.all_gather)>(dlsym(h, "ncclAllGather"));
    g_nccl.comm_destroy = reinterpret_cast<decltype(g_nccl.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    g_nccl.error_string = reinterpret_cast<decltype(g_nccl.error_string)>(dlsym(h, "ncclGetErrorString"));
    g_nccl.ok = g_nccl.get_unique_id && g_nccl.comm_init_rank && g_nccl.all_reduce &&
                g_nccl.all_gather && g_nccl.comm_destroy && g_nccl.error_string;
  });
  if (!g_nccl.ok) return fail(TK_ERR_NCCL, "NCCL (libnccl.so.2) could not be loaded");
  *out = &g_nccl;
  return TK_OK;
}

int nccl_fail(const NcclApi* n, const char* what, ncclResult_t r) {
  return fail(TK_ERR_NCCL, "%s failed: %s", what, n->error_string(r));
}

static_assert(sizeof(ncclUniqueId) == TK_TP_UNIQUE_ID_BYTES, "NCCL unique id size");

}  // namespace

struct tk_tp {
  tk_device* dev = nullptr;
  ncclComm_t comm = nullptr;
  int nranks = 0, rank = 0;
  // one-shot peer-memory all-reduce (tk_allreduce.cu); off when any rank could not map its peers
  bool p2p = false;
  void* p2p_base = nullptr;              // this rank's receive area + flags + chunk epochs
  void* p2p_peer[tk::kP2PMaxRanks] = {};  // peers' areas mapped here (CUDA IPC)
  tk::P2PParams p2p_params{};
  // the batch 1-2 FFN's exchange fused into the decode kernel (same mapped areas): launch
  // counters of this rank and every rank's tagged-word area
  TpFuse fuse{};
  bool fused = false;
  // the device's p2p_timeouts when the group was made: a wait of this group that ran out leaves
  // the ranks' chunk epochs out of step, so the group takes no further exchange after one
  unsigned p2p_timeouts_at_create = 0;
};

namespace {

// Sum of one int across the group (NCCL), for decisions every rank must take alike.
int tp_sum_int(tk_tp* tp, const NcclApi* n, int v, int* out) {
  int* dv = nullptr;
  TK_CUDA_TRY(cudaMalloc(&dv, sizeof(int)));
  cudaError_t e = cudaMemcpy(dv, &v, sizeof(int), cudaMemcpyHostToDevice);
  ncclResult_t r = e == cudaSuccess ? n->all_reduce(dv, dv, 1, ncclInt32, ncclSum, tp->comm, tp->dev->stream)
                                    : ncclSuccess;
  if (e == cudaSuccess && r == ncclSuccess) e = cudaStreamSynchronize(tp->dev->stream);
  if (e == cudaSuccess && r == ncclSuccess) e = cudaMemcpy(out, dv, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(dv);
  if (r != ncclSuccess) return nccl_fail(n, "ncclAllReduce", r);
  TK_CUDA_TRY(e);
  return TK_OK;
}

void tp_p2p_release(tk_tp* tp) {
  for (int r = 0; r < tk::kP2PMaxRanks; ++r)
    if (tp->p2p_peer[r]) {
      cudaIpcCloseMemHandle(tp->p2p_peer[r]);
      tp->p2p_peer[r] = nullptr;
    }
  if (tp->p2p_base) cudaFree(tp->p2p_base);
  tp->p2p_base = nullptr;
  tp->p2p = false;
}

// Receive areas for the peer-memory all-reduce: allocate, zero, exchange IPC handles (NCCL
// all-gather), map the peers; then every rank learns whether all ranks succeeded.
int tp_p2p_setup(tk_tp* tp, const NcclApi* n) {
  using namespace tk;
  const int R = tp->nranks;
  const size_t slot = kP2PMaxFloats;
  const size_t recv_bytes = 2 * (size_t)R * slot * sizeof(float);
  const size_t flag_bytes = (size_t)R * kP2PMaxChunks * sizeof(unsigned);
  const size_t counter_bytes = kP2PMaxChunks * sizeof(unsigned);
  const size_t fuse_epoch_off = recv_bytes + flag_bytes + counter_bytes;
  const size_t fuse_off = fuse_epoch_off + kDecEpochSlots * sizeof(unsigned);
  const size_t bytes = fuse_off + 2 * (size_t)R * kTpFuseWords * 8;
  int ok = 1;
  cudaIpcMemHandle_t mine{};
  if (cudaMalloc(&tp->p2p_base, bytes) != cudaSuccess || cudaMemset(tp->p2p_base, 0, bytes) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess || cudaIpcGetMemHandle(&mine, tp->p2p_base) != cudaSuccess)
    ok = 0;
  cudaGetLastError();
  // all ranks take part in the all-gather whatever happened above
  uint8_t* dh = nullptr;
  TK_CUDA_TRY(cudaMalloc(&dh, (size_t)R * sizeof(cudaIpcMemHandle_t)));
  std::vector<cudaIpcMemHandle_t> handles(R);
  cudaError_t e = cudaMemcpy(dh + (size_t)tp->rank * sizeof(mine), &mine, sizeof(mine), cudaMemcpyHostToDevice);
  ncclResult_t r = n->all_gather(dh + (size_t)tp->rank * sizeof(mine), dh, sizeof(mine), ncclUint8, tp->comm,
                                 tp->dev->stream);
  if (e == cudaSuccess && r == ncclSuccess) e = cudaStreamSynchronize(tp->dev->stream);
  if (e == cudaSuccess && r == ncclSuccess)
    e = cudaMemcpy(handles.data(), dh, (size_t)R * sizeof(mine), cudaMemcpyDeviceToHost);
  cudaFree(dh);
  if (r != ncclSuccess) return nccl_fail(n, "ncclAllGather", r);
  TK_CUDA_TRY(e);
  P2PParams& P = tp->p2p_params;
  std::memset(&P, 0, sizeof(P));
  for (int q = 0; q < R && ok; ++q) {
    void* base = tp->p2p_base;
    if (q != tp->rank) {
      if (cudaIpcOpenMemHandle(&tp->p2p_peer[q], handles[q], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        ok = 0;
        break;
      }
      base = tp->p2p_peer[q];
    }
    P.recv[q] = static_cast<float*>(base);
    P.flags[q] = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(base) + recv_bytes);
    tp->fuse.recv[q] = reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(base) + fuse_off);
  }
  int all = 0;
  int st = tp_sum_int(tp, n, ok, &all);
  if (st != TK_OK) return st;
  if (all != R) {
    tp_p2p_release(tp);
    return TK_OK;  // NCCL carries the exchange
  }
  P.chunk = kP2PChunkFloats;
  P.nranks = R;
  P.rank = tp->rank;
  P.slot_floats = slot;
  P.counters = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(tp->p2p_base) + recv_bytes + flag_bytes);
  P.err = tp->dev->err;
  P.timeout_ns = tp->dev->timeout_ns;
  tp->p2p = true;
  tp->fuse.n = R;
  tp->fuse.rank = tp->rank;
  tp->fuse.words = (int)kTpFuseWords;
  tp->fuse.epoch = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(tp->p2p_base) + fuse_epoch_off);
  const char* fused = std::getenv("TK_TP_FUSED");
  tp->fused = !(fused && !std::atoi(fused));
  return TK_OK;
}

}  // namespace

extern "C" {

int tk_tp_unique_id(uint8_t id[TK_TP_UNIQUE_ID_BYTES]) {
  if (!id) return fail(TK_ERR_ARG, "id is NULL");
  const NcclApi* n = nullptr;
  int st = nccl_api(&n);
  if (st != TK_OK) return st;
  ncclUniqueId u;
  ncclResult_t r = n->get_unique_id(&u);
  if (r != ncclSuccess) return nccl_fail(n, "ncclGetUniqueId", r);
  std::memcpy(id, &u, sizeof(u));
  return TK_OK;
}

int tk_tp_create(tk_device* d, int nranks, int rank, const uint8_t id[TK_TP_UNIQUE_ID_BYTES],
                 tk_tp** out) {
  if (!d || !id || !out) return fail(TK_ERR_ARG, "NULL argument");
  *out = nullptr;
  if (nranks < 1 || rank < 0 || rank >= nranks)
    return fail(TK_ERR_ARG, "rank %d of %d is out of range", rank, nranks);
  const NcclApi* n = nullptr;
  int st = nccl_api(&n);
  if (st != TK_OK) return st;
  if ((st = set_device(d)) != TK_OK) return st;
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  tk_tp* tp = new tk_tp();
  tp->dev = d;
  tp->nranks = nranks;
  tp->rank = rank;
  tp->p2p_timeouts_at_create = d->p2p_timeouts;
  ncclResult_t r = n->comm_init_rank(&tp->comm, nranks, u, rank);
  if (r != ncclSuccess) {
    delete tp;
    return nccl_fail(n, "ncclCommInitRank", r);
  }
  const char* force_nccl = std::getenv("TK_TP_NCCL");
  if (nranks > 1 && nranks <= tk::kP2PMaxRanks && !(force_nccl && std::atoi(force_nccl))) {
    st = tp_p2p_setup(tp, n);
    if (st != TK_OK) {
      tk_tp_destroy(tp);
      return st;
    }
  }
  *out = tp;
  return TK_OK;
}

int tk_tp_uses_p2p(tk_tp* tp) { return tp && tp->p2p ? 1 : 0; }

void tk_tp_destroy(tk_tp* tp) {
  if (!tp) return;
  const NcclApi* n = nullptr;
  if (tp->comm && nccl_api(&n) == TK_OK) {
    cudaSetDevice(tp->dev->ordinal);
    cudaStreamSynchronize(tp->dev->stream);
    if (tp->p2p_base) {
      // no peer may still be writing into this rank's area when it is freed
      int all = 0;
      tp_sum_int(tp, n, 1, &all);
    }
    tp_p2p_release(tp);
    n->comm_destroy(tp->comm);
  }
  delete tp;
}

int tk_tp_allreduce_sum_f32(tk_tp* tp, float* buf, size_t count, void* stream) {
  if (!tp || (!buf && count)) return fail(TK_ERR_ARG, "NULL argument");
  if (count == 0 || tp->nranks == 1) return TK_OK;
  if (tp->p2p && tp->dev->p2p_timeouts != tp->p2p_timeouts_at_create)
    return fail(TK_ERR_TIMEOUT,
                "a peer-memory exchange on this device timed out; the group's ranks are out of "
                "step: destroy it (tk_tp_destroy) and create a new one");
  int st = set_device(tp->dev);
  if (st != TK_OK) return st;
  if (tp->p2p && count <= tk::kP2PMaxFloats) {
    tk::P2PParams P = tp->p2p_params;
    P.buf = buf;
    P.count = (int)count;
    TK_LAUNCH(tp->dev, tk::launch_p2p_allreduce(P, pick_stream(tp->dev, stream)));
    return TK_OK;
  }
  const NcclApi* n = nullptr;
  if ((st = nccl_api(&n)) != TK_OK) return st;
  ncclResult_t r = n->all_reduce(buf, buf, count, ncclFloat32, ncclSum, tp->comm,
                                 pick_stream(tp->dev, stream));
  if (r != ncclSuccess) return nccl_fail(n, "ncclAllReduce", r);
  return TK_OK;
}

int tk_int4_ffn_tp_exchange(tk_tp* tp, uint32_t m, uint32_t hidden, uint32_t inter, uint32_t gs) {
  if (!tp) return fail(TK_ERR_ARG, "tp is NULL");
  if (tp->nranks == 1) return 0;
  if (!tp->p2p) return 0;
  if (tp->fused && (int)m <= kDecMaxRows && tp->dev->decode_enabled &&
      (size_t)m * hidden <= kTpFuseWords &&
      tk_int4_ffn_path(m, hidden, inter, gs) == 3)
    return 2;
  return (size_t)m * hidden <= tk::kP2PMaxFloats ? 1 : 0;
}

int tk_int4_ffn_tp_async(tk_tp* tp, const float* x, const float* norm_w, const tk_int4_matrix* gate,
                         const tk_int4_matrix* up, const tk_int4_matrix* down, float* out,
                         uint32_t m, uint32_t hidden, uint32_t inter, uint32_t gs, float eps,
                         uint32_t flags, void* stream) {
  if (!tp) return fail(TK_ERR_ARG, "tp is NULL");
  if (flags & TK_FFN_HOST_IO)
    return fail(TK_ERR_ARG, "TK_FFN_HOST_IO is not supported by the tensor-parallel FFN");
  if (tp->nranks > 1 && tk_int4_ffn_tp_exchange(tp, m, hidden, inter, gs) == 2) {
    // one decode launch per rank: its reduction stores this rank's partial y into every rank's
    // area and sums the ranks' words in rank order (the residual, if any, after the sum)
    if (!x || !norm_w || !gate || !up || !down || !out) return fail(TK_ERR_ARG, "NULL argument");
    for (const tk_int4_matrix* a : {gate, up, down})
      if (!a->w_packed || !a->scales || !a->zeros) return fail(TK_ERR_ARG, "NULL matrix pointer");
    if (flags & ~TK_FFN_RESIDUAL) return fail(TK_ERR_ARG, "unknown flags 0x%x", flags);
    if (tp->dev->p2p_timeouts != tp->p2p_timeouts_at_create)
      return fail(TK_ERR_TIMEOUT,
                  "a peer-memory exchange on this device timed out; the group's ranks are out of "
                  "step: destroy it (tk_tp_destroy) and create a new one");
    // (a rank taking another exchange than its peers would leave them waiting: buffers that
    // would send one rank elsewhere are an error)
    if (!(aligned16(x) && aligned16(norm_w) && aligned16(out) && matrix_aligned(gate) &&
          matrix_aligned(up) && matrix_aligned(down)))
      return fail(TK_ERR_ARG, "the fused exchange needs 16-byte aligned buffers");
    int st = set_device(tp->dev);
    if (st != TK_OK) return st;
    st = decode_run(tp->dev, x, norm_w, eps, gate, up, down, out, nullptr, (int)m, (int)hidden, 0,
                    (int)inter, (int)gs, (flags & TK_FFN_RESIDUAL) != 0,
                    pick_stream(tp->dev, stream), false, &tp->fuse);
    // unsupported is decided by the shapes and the device type, alike on every rank
    if (st != TK_ERR_UNSUPPORTED) return st;
  }
  // the residual is added once, by rank 0, before the sum
  const uint32_t f = tp->rank == 0 ? flags : (flags & ~TK_FFN_RESIDUAL);
  int st = tk_int4_ffn_async(tp->dev, x, norm_w, gate, up, down, out, nullptr, m, hidden, inter, gs,
                             eps, f, stream);
  if (st != TK_OK) return st;
  return tk_tp_allreduce_sum_f32(tp, out, (size_t)m * hidden, stream);
}

int tk_int4_ffn_tp(tk_tp* tp, const float* x, const float* norm_w, const tk_int4_matrix* gate,
                   const tk_int4_matrix* up, const tk_int4_matrix* down, float* out, uint32_t m,
                   uint32_t hidden, uint32_t inter, uint32_t gs, float eps, uint32_t flags) {
  int st = tk_int4_ffn_tp_async(tp, x, norm_w, gate, up, down, out, m, hidden, inter, gs, eps,
                                flags, nullptr);
  if (st != TK_OK) return st;
  return sync_and_check(tp->dev, tp->dev->stream);
}

}  // extern "C"
