/*
 * Host-side builders for the synthetic BASELINE layers: a seeded normal
 * generator and the Swift MXFP4 quantizer, fast enough to build the experts a
 * CPU run touches (tens of experts of 44M values) on the host cores.
 *
 * TEST INFRASTRUCTURE ONLY: the product library never links this file.  It
 * feeds the timed CPU restatement (bench.py's reference arm) without the
 * device library, and the oracle's own tests.
 *
 *   oracle_normal_bf16: counter-based (splitmix64 of seed, stream, index)
 *     uniform pairs turned into N(0, 1) by Box-Muller in double precision,
 *     times std, rounded to the nearest bf16 value (returned as float32).
 *     Output i depends only on (seed, stream, i), so any thread count gives
 *     the same values.
 *   oracle_mxfp4_quantize: MXFP4.quantizeBF16 (Sources/DeepSeekRepack/
 *     MXFP4.swift:19-37, fp4Code :115-131) on float32 values: per 32-value
 *     group, amax == 0 gives scale byte 0 and codes 0; otherwise
 *     e = clamp(floor(log2 amax) - 2, -127, 128), scale byte e + 127, values
 *     times 2^-e rounded to the nearest e2m1 magnitude (ties to the even code
 *     index, saturating at 6), sign from the float's sign bit; two codes per
 *     byte, the even column in the low nibble (dequant.py:53-60).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static inline uint64_t splitmix64(uint64_t x) {
  x += 0x9e3779b97f4a7c15ULL;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ULL;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebULL;
  return x ^ (x >> 31);
}

static inline float round_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  u += 0x7fffu + ((u >> 16) & 1u);
  u &= 0xffff0000u;
  float r;
  memcpy(&r, &u, 4);
  return r;
}

void oracle_normal_bf16(uint64_t seed, uint64_t stream, int64_t n, float std, float *out) {
  const uint64_t key = splitmix64(seed * 0x100000001b3ULL ^ splitmix64(stream + 0x632be59bd9b4e019ULL));
  const int64_t pairs = (n + 1) / 2;
#pragma omp parallel for schedule(static)
  for (int64_t p = 0; p < pairs; ++p) {
    const uint64_t h1 = splitmix64(key ^ (uint64_t)(2 * p));
    const uint64_t h2 = splitmix64(key ^ (uint64_t)(2 * p + 1));
    const double u1 = ((double)(h1 >> 11) + 1.0) * 0x1p-53;   /* (0, 1] */
    const double u2 = (double)(h2 >> 11) * 0x1p-53;           /* [0, 1) */
    const double r = sqrt(-2.0 * log(u1));
    const double a = 6.283185307179586 * u2;
    out[2 * p] = round_bf16((float)(r * cos(a) * std));
    if (2 * p + 1 < n) out[2 * p + 1] = round_bf16((float)(r * sin(a) * std));
  }
}

/* nearest e2m1 magnitude index of |v| <= 6, ties to the even index */
static inline uint8_t e2m1_index(float mag) {
  return (uint8_t)((mag > 0.25f) + (mag >= 0.75f) + (mag > 1.25f) + (mag >= 1.75f) + (mag > 2.5f) +
                   (mag >= 3.5f) + (mag > 5.0f));
}

void oracle_mxfp4_quantize(const float *src, int64_t rows, int cols, uint8_t *packed, uint8_t *scales) {
  const int groups = cols / 32;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    for (int g = 0; g < groups; ++g) {
      const float *v = src + r * cols + g * 32;
      uint8_t *pk = packed + r * (cols / 2) + g * 16;
      float amax = 0.0f;
      for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
      if (amax == 0.0f) {
        scales[r * groups + g] = 0;
        memset(pk, 0, 16);
        continue;
      }
      int ex;
      frexpf(amax, &ex);                           /* amax = m * 2^ex, m in [0.5, 1): floor(log2) = ex - 1 */
      int e = ex - 1 - 2;
      if (e < -127) e = -127;
      if (e > 128) e = 128;
      scales[r * groups + g] = (uint8_t)(e + 127);
      const float f = ldexpf(1.0f, -e);
      uint8_t c[32];
      for (int i = 0; i < 32; ++i) {
        const float s = v[i] * f;
        uint32_t bits;
        memcpy(&bits, &s, 4);
        float mag = fabsf(s);
        if (mag > 6.0f) mag = 6.0f;
        c[i] = (uint8_t)(e2m1_index(mag) | ((bits >> 31) << 3));
      }
      for (int i = 0; i < 16; ++i) pk[i] = (uint8_t)(c[2 * i] | (c[2 * i + 1] << 4));
    }
  }
}
