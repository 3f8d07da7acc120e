// cpu_baseline.cpp -- multithreaded CPU transcription of the reference shader semantics
// (test / benchmark infrastructure: the timed CPU baseline and a second f32 checker).
//
// qmatmul_int4 follows src/kernels/shaders.zig:442-501 exactly per output column:
//   acc += (x[k] * scale[g][n]) * (float(q[k][n]) - float(zero[g][n])),  k ascending,
// in IEEE f32 with no FMA contraction (built with -ffp-contract=off), so each column's
// result is bit-identical to the shader's arithmetic.  Columns are split into blocks over
// std::threads; inside a block the loop runs k-outer / n-inner so the packed rows stream
// through the cache (the per-column operation order is unchanged).  Unlike the shader it
// accepts any K (the shader's shared_x[4096] caps K, shaders.zig:457) and all M rows.
// rmsnorm (shaders.zig:16-56), silu*up (shaders.zig:344-357, fast_silu :7-9) and the FFN
// composition (src/bench.zig:266-341 + the down projection, src/model/llama.zig:220-231)
// are single-pass f32 loops.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

float g_f16[65536];
bool g_f16_ready = false;

// IEEE binary16 -> binary32 decode (exact).
float half_bits_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  const int exp = (h >> 10) & 31;
  const uint32_t man = h & 1023u;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: value = man * 2^-24
      float v = std::ldexp((float)man, -24);
      std::memcpy(&bits, &v, 4);
      bits |= sign;
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((uint32_t)(exp - 15 + 127) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

void init_f16() {
  if (g_f16_ready) return;
  for (uint32_t i = 0; i < 65536; ++i) g_f16[i] = half_bits_to_float((uint16_t)i);
  g_f16_ready = true;
}

int pick_threads(int threads) {
  if (threads > 0) return threads;
  unsigned h = std::thread::hardware_concurrency();
  return h ? (int)h : 1;
}

template <typename F>
void parallel_blocks(int nblocks, int threads, F&& fn) {
  threads = std::min(threads, nblocks);
  if (threads <= 1) {
    for (int b = 0; b < nblocks; ++b) fn(b);
    return;
  }
  std::vector<std::thread> pool;
  pool.reserve(threads);
  for (int t = 0; t < threads; ++t)
    pool.emplace_back([&, t] {
      for (int b = t; b < nblocks; b += threads) fn(b);
    });
  for (auto& th : pool) th.join();
}

constexpr int kColBlock = 256;

void qmatmul_block(const float* x, const uint8_t* w, const uint16_t* s, const uint8_t* z, float* out,
                   int m, int k, int n, int gs, int c0, int c1) {
  const int nc = c1 - c0;
  float acc[kColBlock];
  float scale[kColBlock];
  float fz[kColBlock];
  for (int r = 0; r < m; ++r) {
    const float* xr = x + (size_t)r * k;
    for (int j = 0; j < nc; ++j) acc[j] = 0.0f;
    for (int g = 0; g < k / gs; ++g) {
      for (int j = 0; j < nc; ++j) {
        const int col = c0 + j;
        scale[j] = g_f16[s[(size_t)g * n + col]];
        fz[j] = (float)((z[(size_t)g * (n / 2) + col / 2] >> ((col & 1) * 4)) & 15);
      }
      for (int i = 0; i < gs; i += 2) {
        const int kk = g * gs + i;
        const uint8_t* row = w + (size_t)(kk / 2) * n + c0;
        const float x0 = xr[kk], x1 = xr[kk + 1];
        for (int j = 0; j < nc; ++j) {
          const uint32_t p = row[j];
          acc[j] = acc[j] + (x0 * scale[j]) * ((float)(p & 15u) - fz[j]);
          acc[j] = acc[j] + (x1 * scale[j]) * ((float)(p >> 4) - fz[j]);
        }
      }
    }
    for (int j = 0; j < nc; ++j) out[(size_t)r * n + c0 + j] = acc[j];
  }
}

}  // namespace

extern "C" {

int tkcpu_default_threads(void) { return pick_threads(0); }

// y[m][n] (see header comment). Returns 0, or -1 on an invalid shape.
int tkcpu_qmatmul_int4(const float* x, const uint8_t* w, const uint16_t* s, const uint8_t* z,
                       float* out, int m, int k, int n, int gs, int threads) {
  if (m <= 0 || k <= 0 || n <= 0 || gs <= 0 || gs % 2 || k % gs || n % 2) return -1;
  init_f16();
  const int nb = (n + kColBlock - 1) / kColBlock;
  parallel_blocks(nb, pick_threads(threads), [&](int b) {
    const int c0 = b * kColBlock, c1 = std::min(n, c0 + kColBlock);
    qmatmul_block(x, w, s, z, out, m, k, n, gs, c0, c1);
  });
  return 0;
}

// out = x * rsqrt(sum(x^2)/dim + eps) * w per row (f32, sequential sum).
int tkcpu_rmsnorm(const float* x, const float* w, float* out, int rows, int dim, float eps) {
  for (int r = 0; r < rows; ++r) {
    const float* xr = x + (size_t)r * dim;
    float ss = 0.0f;
    for (int i = 0; i < dim; ++i) ss = ss + xr[i] * xr[i];
    const float rms = 1.0f / std::sqrt(ss / (float)dim + eps);
    for (int i = 0; i < dim; ++i) out[(size_t)r * dim + i] = xr[i] * rms * w[i];
  }
  return 0;
}

int tkcpu_silu_mul(const float* g, const float* u, float* out, int n) {
  for (int i = 0; i < n; ++i) out[i] = g[i] / (1.0f + std::exp(-g[i])) * u[i];
  return 0;
}

// INT4 Llama FFN on m rows; scratch needs m*(hidden + 3*inter) floats.
int tkcpu_int4_ffn(const float* x, const float* norm_w, const uint8_t* gw, const uint16_t* gsc,
                   const uint8_t* gz, const uint8_t* uw, const uint16_t* usc, const uint8_t* uz,
                   const uint8_t* dw, const uint16_t* dsc, const uint8_t* dz, float* out, int m,
                   int hidden, int inter, int gs, float eps, int residual, float* scratch,
                   int threads) {
  float* normed = scratch;
  float* gate = normed + (size_t)m * hidden;
  float* up = gate + (size_t)m * inter;
  float* h = up + (size_t)m * inter;
  tkcpu_rmsnorm(x, norm_w, normed, m, hidden, eps);
  if (tkcpu_qmatmul_int4(normed, gw, gsc, gz, gate, m, hidden, inter, gs, threads)) return -1;
  if (tkcpu_qmatmul_int4(normed, uw, usc, uz, up, m, hidden, inter, gs, threads)) return -1;
  tkcpu_silu_mul(gate, up, h, m * inter);
  if (tkcpu_qmatmul_int4(h, dw, dsc, dz, out, m, inter, hidden, gs, threads)) return -1;
  if (residual)
    for (size_t i = 0; i < (size_t)m * hidden; ++i) out[i] = x[i] + out[i];
  return 0;
}

}  // extern "C"
