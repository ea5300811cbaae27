/*
 * C restatement of the AWQ W4A16 reference arithmetic -- TEST INFRASTRUCTURE ONLY.
 *
 * The checker and the timed CPU baseline ("port"), never the product. It follows
 * the reference's PyTorch code in ashqk/ref.py (MMMchou/ash-quant-kernels):
 *   - nibble extraction: column j of a word sits at bits 4*AWQ_REVERSE_ORDER[j]
 *     (ashqk/ref.py:20-21, unpack_awq at :49-55);
 *   - dequantisation W = (q - z) * s, computed in fp32 (ashqk/ref.py:78-86);
 *   - the GEMM y = x @ W (ashqk/ref.py:89-103), here with fp64 accumulation so it
 *     doubles as a high-precision truth.
 * Multi-threaded with OpenMP over output columns.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static const int kReverseOrder[8] = {0, 4, 1, 5, 2, 6, 3, 7};

/* IEEE binary16 -> binary32, exact (all fp16 values are representable in fp32). */
static float half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1F;
  uint32_t man = h & 0x3FF;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: renormalise */
      int e = -1;
      do { man <<= 1; ++e; } while (!(man & 0x400));
      man &= 0x3FF;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 0x1F) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

int awq_oracle_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

static inline int nibble_of(const int32_t* row, int64_t col) {
  uint32_t word = (uint32_t)row[col >> 3];
  return (int)((word >> (4 * kReverseOrder[col & 7])) & 0xF);
}

/* W[k, n] = (q - z) * s in fp32, row-major [K, N]. */
int awq_oracle_dequant_f32(const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                           float* out, int64_t K, int64_t N, int64_t G) {
  if (K <= 0 || N <= 0 || G <= 0 || K % G || N % 8) return 1;
  const int64_t W = N / 8;
#pragma omp parallel for schedule(static)
  for (int64_t k = 0; k < K; ++k) {
    const int32_t* qrow = qweight + k * W;
    const int32_t* zrow = qzeros + (k / G) * W;
    const uint16_t* srow = scales + (k / G) * N;
    float* orow = out + k * N;
    for (int64_t n = 0; n < N; ++n) {
      orow[n] = (float)(nibble_of(qrow, n) - nibble_of(zrow, n)) * half_to_float(srow[n]);
    }
  }
  return 0;
}

/*
 * y[m, n] = sum_k x[m, k] * W[k, n], W dequantised in fp32, accumulated in fp64.
 * y is fp64 [M, N]. threads <= 0 uses the OpenMP default.
 */
int awq_oracle_gemm(const uint16_t* x, const int32_t* qweight, const int32_t* qzeros,
                    const uint16_t* scales, double* y, int64_t M, int64_t N, int64_t K, int64_t G,
                    int threads) {
  if (M <= 0 || K <= 0 || N <= 0 || G <= 0 || K % G || N % 8) return 1;
  const int64_t W = N / 8;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
  float* xf = (float*)malloc(sizeof(float) * (size_t)(M * K));
  if (!xf) return 2;
  for (int64_t i = 0; i < M * K; ++i) xf[i] = half_to_float(x[i]);
  memset(y, 0, sizeof(double) * (size_t)(M * N));

  /* Parallel over 8-column blocks: each thread owns whole output columns. */
#pragma omp parallel
  {
    double acc[16][8];
    float wcol[8];
#pragma omp for schedule(static)
    for (int64_t wb = 0; wb < W; ++wb) {
      for (int64_t m0 = 0; m0 < M; m0 += 16) {
        int64_t mb = M - m0 < 16 ? M - m0 : 16;
        for (int64_t i = 0; i < mb; ++i)
          for (int j = 0; j < 8; ++j) acc[i][j] = 0.0;
        for (int64_t k = 0; k < K; ++k) {
          uint32_t q = (uint32_t)qweight[k * W + wb];
          uint32_t z = (uint32_t)qzeros[(k / G) * W + wb];
          const uint16_t* s = scales + (k / G) * N + wb * 8;
          for (int j = 0; j < 8; ++j) {
            int sh = 4 * kReverseOrder[j];
            int qv = (int)((q >> sh) & 0xF), zv = (int)((z >> sh) & 0xF);
            wcol[j] = (float)(qv - zv) * half_to_float(s[j]);
          }
          for (int64_t i = 0; i < mb; ++i) {
            double xv = (double)xf[(m0 + i) * K + k];
            for (int j = 0; j < 8; ++j) acc[i][j] += xv * (double)wcol[j];
          }
        }
        for (int64_t i = 0; i < mb; ++i)
          for (int j = 0; j < 8; ++j) y[(m0 + i) * N + wb * 8 + j] = acc[i][j];
      }
    }
  }
  free(xf);
  return 0;
}
