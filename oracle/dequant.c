/* CPU oracle helper: weight dequantisation to fp32, the step of the reference's CPU GEMMs that
 * dominates the oracle's time at full layer sizes.
 *
 * TEST INFRASTRUCTURE ONLY (checker side): loaded by oracle/moe_oracle.py, which tests/, smoke() and
 * bench.py's CPU-baseline leg call. Nothing on the product path links or loads it.
 *
 * Restates, value for value, the dequantisation of the reference's CPU kernel stand-ins
 * (leyten/shard engines/deepseek_v4/v4_kernels_cpu.py:141-173: unpack_fp4 low nibble first, e2m1
 * table :61-62, then values x scale in fp32) for the three weight formats of the MoE stage:
 *   MXFP4  e2m1 x 2^(e8m0 - 127), one scale per 32 K
 *   NVFP4  (e2m1 x e4m3 scale per 16) x fp32 tensor scale, multiplied left to right in fp32
 *   FP8    e4m3 x fp32 scale per 128 x 128 block
 * The products are computed in fp32 exactly as numpy computes them in moe_oracle.dequant_weight. */
#include <math.h>
#include <stdint.h>

static const float E2M1[16] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                               -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

/* e4m3fn code -> fp32 (0x7f / 0xff are NaN) */
static float e4m3(uint8_t c) {
  const float s = (c & 0x80) ? -1.0f : 1.0f;
  const int e = (c >> 3) & 0xF, m = c & 0x7;
  if (e == 0xF && m == 0x7) return NAN;
  if (e == 0) return s * ldexpf((float)m / 8.0f, -6);
  return s * ldexpf(1.0f + (float)m / 8.0f, e - 7);
}

/* fp4 weights [n, k/2] (low nibble first) with scales -> out fp32 [n, k].
 * fmt 1 = NVFP4 (scale e4m3 [n, k/16], tensor scale ts), 2 = MXFP4 (scale e8m0 [n, k/32]). */
int oracle_dequant_fp4(int fmt, const uint8_t* packed, const uint8_t* scale, float ts, int64_t n, int64_t k,
                       float* out) {
  if (fmt != 1 && fmt != 2) return -1;
  float e4[256];
  for (int c = 0; c < 256; ++c) e4[c] = e4m3((uint8_t)c);
  const int64_t g = fmt == 1 ? 16 : 32;
  for (int64_t r = 0; r < n; ++r) {
    const uint8_t* p = packed + r * (k / 2);
    const uint8_t* s = scale + r * (k / g);
    float* o = out + r * k;
    for (int64_t j = 0; j < k / g; ++j) {
      const float sc = fmt == 1 ? e4[s[j]] : ldexpf(1.0f, (int)s[j] - 127);
      for (int64_t i = 0; i < g; i += 2) {
        const uint8_t b = p[(j * g + i) / 2];
        float v0 = E2M1[b & 0xF] * sc, v1 = E2M1[b >> 4] * sc;
        if (fmt == 1) {
          v0 = v0 * ts;
          v1 = v1 * ts;
        }
        o[j * g + i] = v0;
        o[j * g + i + 1] = v1;
      }
    }
  }
  return 0;
}

/* FP8 weights e4m3 [n, k] with fp32 block scales [ceil(n/128), ceil(k/128)] -> out fp32 [n, k]. */
int oracle_dequant_fp8(const uint8_t* q, const float* scale, int64_t n, int64_t k, float* out) {
  float e4[256];
  for (int c = 0; c < 256; ++c) e4[c] = e4m3((uint8_t)c);
  const int64_t kb = (k + 127) / 128;
  for (int64_t r = 0; r < n; ++r) {
    const float* srow = scale + (r / 128) * kb;
    for (int64_t i = 0; i < k; ++i) out[r * k + i] = e4[q[r * k + i]] * srow[i / 128];
  }
  return 0;
}

/* y [m, n] = xa [m, k] . dequant(W)^T for a quantised weight W [n, k] (fmt 1 NVFP4, 2 MXFP4, 3 FP8 with
 * `scale` fp32 block scales): row r of W is dequantised as above into `row` (k floats of scratch),
 * then dotted with every activation row in fp32 (eight interleaved partial sums, added pairwise at
 * the end). For activation batches of a few rows; the oracle takes BLAS for wide ones. */
int oracle_qgemm(int fmt, const uint8_t* w, const void* scale, float ts, int64_t n, int64_t k, const float* xa,
                 int64_t m, float* y, float* row) {
  if (fmt < 1 || fmt > 3) return -1;
  for (int64_t r = 0; r < n; ++r) {
    if (fmt == 3) {
      const int64_t kb = (k + 127) / 128;
      oracle_dequant_fp8(w + r * k, (const float*)scale + (r / 128) * kb, 1, k, row);
    } else {
      const int64_t g = fmt == 1 ? 16 : 32;
      oracle_dequant_fp4(fmt, w + r * (k / 2), (const uint8_t*)scale + r * (k / g), ts, 1, k, row);
    }
    for (int64_t t = 0; t < m; ++t) {
      const float* x = xa + t * k;
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      int64_t i = 0;
      for (; i + 8 <= k; i += 8)
        for (int j = 0; j < 8; ++j) acc[j] += x[i + j] * row[i + j];
      for (; i < k; ++i) acc[0] += x[i] * row[i];
      y[t * n + r] = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
    }
  }
  return 0;
}
