/*
 * C restatement of the reference's int8 row quantiser - TEST INFRASTRUCTURE (the oracle), never the product path.
 *
 * Int8Tensor.quantize (src/opendecider/quant.py:37-41) and the weight quantiser of Int8Linear.__init__
 * (quant.py:124-127), per row of K float32 values:
 *     s = max(max_k |x|, 1e-8f) / 127.0f        (IEEE float32 division)
 *     q = clamp(rint(x / s), -127, 127)          (round half to even: the default rounding mode)
 * Build with plain gcc and no fast-math (oracle/build.py). Loaded by tests/ through ctypes.
 */
#include <math.h>
#include <stdint.h>

void oq_quantize_rows_f32(const float* x, int64_t M, int64_t K, int8_t* q, float* s_out) {
  for (int64_t m = 0; m < M; ++m) {
    const float* r = x + m * K;
    float amax = 0.0f;
    for (int64_t k = 0; k < K; ++k) {
      const float a = fabsf(r[k]);
      if (a > amax) amax = a;
    }
    const float s = (amax > 1e-8f ? amax : 1e-8f) / 127.0f;
    for (int64_t k = 0; k < K; ++k) {
      float v = rintf(r[k] / s);
      if (v > 127.0f) v = 127.0f;
      if (v < -127.0f) v = -127.0f;
      q[m * K + k] = (int8_t)v;
    }
    s_out[m] = s;
  }
}

/* int32 accumulators of the W8A8 GEMM, acc[m, n] = sum_k a[m, k] * w[n, k] (exact in int64, stored as int32). */
void oq_gemm_i32(const int8_t* a, const int8_t* w, int64_t M, int64_t N, int64_t K, int32_t* acc) {
  for (int64_t m = 0; m < M; ++m)
    for (int64_t n = 0; n < N; ++n) {
      int64_t s = 0;
      const int8_t* ar = a + m * K;
      const int8_t* wr = w + n * K;
      for (int64_t k = 0; k < K; ++k) s += (int64_t)ar[k] * (int64_t)wr[k];
      acc[m * N + n] = (int32_t)s;
    }
}
