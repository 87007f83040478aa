/*
 * cpu_ref.c -- C restatement of tinygrad-dx12's packed decode + CPU matmul branch.
 *
 * TEST INFRASTRUCTURE ONLY (the checker and the timed CPU baseline): only tests/,
 * __graft_entry__.smoke() and bench.py's CPU legs load it. The product never does.
 *
 * Follows:
 *   src/tinygrad_dx12/codegen/decomp/dx12.py:69-77   word build + payload extraction
 *   src/tinygrad_dx12/codegen/decomp/dx12.py:93-100  INT4/UINT4 and FP4/FP6 values (float32)
 *   src/tinygrad_dx12/codegen/decomp/dx12.py:102-106 block scales, multiply in float32
 *   src/tinygrad_dx12/codegen/linalg.py:169-174      CPU branch: the packed operand is
 *       unpacked to float32 and materialised (.contiguous()), then an fp32-accumulated matmul.
 *
 * oref_linear() keeps that order per weight row: the row is decoded into a float32 buffer
 * (the materialised weight), then each output is a float32 dot product in k order.
 * Rows are distributed over OpenMP threads. Pinned by the same golden vectors as the numpy
 * restatement (tests/test_oracle_c.py).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* formats: 0 int4, 1 uint4, 2 fp4_e2m1, 3 fp6_e2m3, 4 fp6_e3m2 (dx12.py:10) */
static const int BITS[5] = {4, 4, 4, 6, 6};
static const int MBITS[5] = {0, 0, 1, 3, 2};
static const int EBITS[5] = {0, 0, 2, 2, 3};
static const int BIAS[5] = {0, 0, 1, 1, 3};

/* scale / activation dtypes: 12 f16, 13 bf16, 14 f32, 16 e8m0 (same codes as the C-ABI) */
static float half_to_float(uint16_t h) {
  uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1F, f = h & 0x3FF, bits;
  if (e == 0) {
    float v = ldexpf((float)f, -24);
    return s ? -v : v;
  } else if (e == 31) {
    bits = s | 0x7F800000u | (f << 13);
  } else {
    bits = s | ((e - 15 + 127) << 23) | (f << 13);
  }
  float out;
  memcpy(&out, &bits, 4);
  return out;
}

static float load_f32(const void *p, int64_t i, int dt) {
  uint32_t bits;
  float v;
  switch (dt) {
    case 12: return half_to_float(((const uint16_t *)p)[i]);
    case 13: bits = (uint32_t)((const uint16_t *)p)[i] << 16; memcpy(&v, &bits, 4); return v;
    case 14: return ((const float *)p)[i];
    case 16: {
      uint8_t b = ((const uint8_t *)p)[i];
      if (b == 0xFF) return NAN;
      bits = b == 0 ? 0x00400000u : (uint32_t)b << 23;
      memcpy(&v, &bits, 4);
      return v;
    }
  }
  return 0.f;
}

static uint32_t payload(const uint8_t *data, int64_t nbytes, int fmt, int64_t e) {
  const int bits = BITS[fmt], wb = bits / 2;
  const int64_t w = e >> 2;
  uint32_t word = 0;
  for (int i = 0; i < wb; ++i) {
    int64_t b = w * wb + i;
    if (b < nbytes) word |= (uint32_t)data[b] << (8 * i);
  }
  return (word >> ((e & 3) * bits)) & ((1u << bits) - 1u);
}

/* float32 value of a payload: dx12.py:93-100 (significand * exp2(...), sign after) */
static float value(int fmt, uint32_t p) {
  if (fmt == 0) return (float)((int)(p ^ 8u) - 8);
  if (fmt == 1) return (float)p;
  const int bits = BITS[fmt], m = MBITS[fmt], eb = EBITS[fmt], bias = BIAS[fmt];
  const float fraction = (float)(p & ((1u << m) - 1u));
  const int exponent = (int)((p >> m) & ((1u << eb) - 1u));
  const float sig = exponent == 0 ? fraction : fraction + (float)(1 << m);
  const float v = sig * exp2f((float)((exponent == 0 ? 1 : exponent) - bias - m));
  return (p & (1u << (bits - 1))) ? -v : v;
}

/* Decode rows [row0, row0+nrows) to float32 (dequant of dx12.py:49-106 with float32 scales). */
int oref_dequant_f32(const uint8_t *data, int64_t nbytes, int fmt, int64_t rows, int64_t cols, const void *scales,
                     int sdt, int64_t block, float *out) {
  const int64_t nblk = (cols + block - 1) / block;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t k = 0; k < cols; ++k) {
      float v = value(fmt, payload(data, nbytes, fmt, r * cols + k));
      if (scales) v = v * load_f32(scales, r * nblk + k / block, sdt);
      out[r * cols + k] = v;
    }
  }
  return 0;
}

/* y[m, n] = sum_k x[m, k] * W[n, k] in float32 (linalg.py:169-174 order), y float32 [M, N]. */
int oref_linear(const uint8_t *data, int64_t nbytes, int fmt, int64_t rows, int64_t cols, const void *scales, int sdt,
                int64_t block, const void *x, int xdt, int64_t M, float *y, int nthreads) {
  const int64_t nblk = (cols + block - 1) / block;
  float *xf = (float *)malloc(sizeof(float) * (size_t)(M * cols));
  if (!xf) return -1;
  for (int64_t i = 0; i < M * cols; ++i) xf[i] = load_f32(x, i, xdt);
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#endif
  int failed = 0;
#pragma omp parallel
  {
    float *wrow = (float *)malloc(sizeof(float) * (size_t)cols);
    if (!wrow) {
#pragma omp atomic write
      failed = 1;
    }
#pragma omp for schedule(static)
    for (int64_t n = 0; n < rows; ++n) {
      if (!wrow) continue;
      for (int64_t k = 0; k < cols; ++k) {
        float v = value(fmt, payload(data, nbytes, fmt, n * cols + k));
        if (scales) v = v * load_f32(scales, n * nblk + k / block, sdt);
        wrow[k] = v;
      }
      for (int64_t m = 0; m < M; ++m) {
        const float *xr = xf + m * cols;
        float acc = 0.f;
        for (int64_t k = 0; k < cols; ++k) acc += xr[k] * wrow[k];
        y[m * rows + n] = acc;
      }
    }
    free(wrow);
  }
  free(xf);
  return failed ? -1 : 0;
}

int oref_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
