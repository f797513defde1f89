/*
 * ORACLE — test infrastructure, not product.
 *
 * C restatement of the reference's CPU arithmetic on the FFN path, used as a second
 * checker and as the timed CPU baseline:
 *   oracle_q80_quantize   quantize_q80      src/orchestrator/quantizer.py:11-26
 *   oracle_q80_dequantize dequantize_q80    src/orchestrator/quantizer.py:29-40
 *   oracle_matmul_f32     matmul_f32        src/kernels/mojo/pyre_kernels.mojo:133-146
 *                         (loop order i, j, k with an f32 accumulator, b read at k*N+j)
 *   oracle_silu_mul       silu_mul          src/kernels/mojo/pyre_kernels.mojo:121-129
 *   oracle_root_decode_ffn  the root's decode FFN, src/orchestrator/root_node.py:972-980:
 *                         matmul_f32 x3 + silu_mul on f32 weights, columns [c0, c1) only
 *                         (a bounded sample of the full shard for timing)
 * Build: make -C oracle   (gcc, no fast-math, no FP contraction: IEEE f32 division and
 * round-half-even rintf, matching numpy).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static float absf(float x) { return x < 0 ? -x : x; }

void oracle_q80_quantize(const float* x, int64_t n, int8_t* q, float* scales) {
  const int64_t nb = (n + 31) / 32;
  for (int64_t b = 0; b < nb; ++b) {
    float blk[32];
    for (int i = 0; i < 32; ++i) {
      const int64_t e = b * 32 + i;
      blk[i] = e < n ? x[e] : 0.0f;
    }
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) {
      const float a = absf(blk[i]);
      if (a > amax) amax = a;
    }
    if (amax == 0.0f) amax = 1.0f;
    const float s = amax / 127.0f;
    scales[b] = s;
    for (int i = 0; i < 32; ++i) {
      float r = rintf(blk[i] / s);
      if (r < -128.0f) r = -128.0f;
      if (r > 127.0f) r = 127.0f;
      q[b * 32 + i] = (int8_t)r;
    }
  }
}

void oracle_q80_dequantize(const int8_t* q, const float* scales, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = (float)q[i] * scales[i / 32];
}

void oracle_matmul_f32(const float* a, const float* b, float* r, int64_t M, int64_t K, int64_t N) {
  for (int64_t i = 0; i < M; ++i)
    for (int64_t j = 0; j < N; ++j) {
      float acc = 0.0f;
      for (int64_t k = 0; k < K; ++k) acc += a[i * K + k] * b[k * N + j];
      r[i * N + j] = acc;
    }
}

void oracle_silu_mul(const float* g, const float* u, float* r, int64_t n) {
  for (int64_t i = 0; i < n; ++i) r[i] = g[i] / (1.0f + expf(-g[i])) * u[i];
}

/* Root decode FFN restricted to intermediate columns [c0, c1): gate/up [H, W] and the
 * down rows [c0, c1) of [W, H]; out[H] += that slice's contribution. Scalar, one thread,
 * the Mojo loop order. */
void oracle_root_decode_ffn(const float* x, const float* gate, const float* up, const float* down,
                            int64_t H, int64_t W, int64_t c0, int64_t c1, float* out) {
  for (int64_t j = c0; j < c1; ++j) {
    float g = 0.0f, u = 0.0f;
    for (int64_t k = 0; k < H; ++k) g += x[k] * gate[k * W + j];
    for (int64_t k = 0; k < H; ++k) u += x[k] * up[k * W + j];
    const float h = g / (1.0f + expf(-g)) * u;
    for (int64_t n = 0; n < H; ++n) out[n] += h * down[j * H + n];
  }
}
