/*
 * CPU restatement of the quantized expert matmuls (MLX quantized_matmul /
 * gather_qmm with transpose=True) used by the MoE-layer oracle and timed as
 * the CPU baseline.
 *
 * TEST INFRASTRUCTURE ONLY: the product library never links this file.
 *
 *   mxfp4:   W[r][c] = e2m1[code] * 2^(scale-127), group 32 along c,
 *            low nibble = even column        (deepseek_v41/dequant.py:24-66)
 *   affine4: W[r][c] = scale * q + bias, group `group` along c, 8 nibbles per
 *            uint32, element 0 in the low nibble (deepseek_v41/engram.py:207-221)
 *   y[t][r] = sum_c x[t][c] * W[r][c], float32 accumulation per 32-wide group,
 *   groups summed in order (model.py:462-471, qwen4_exp.py:588-597).
 *
 * Weights are dequantized group by group inside the loop, as the reference's
 * quantized_matmul does; nothing is pre-expanded.  Rows are split across
 * OpenMP threads.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static const float kE2M1[16] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                                0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

static inline float e8m0(uint8_t b) { return ldexpf(1.0f, (int)b - 127); }
static inline float bf16f(uint16_t b) { uint32_t u = ((uint32_t)b) << 16; float f; memcpy(&f, &u, 4); return f; }

/* x [n, K] f32, w [rows, K/2] u8, s [rows, K/32] u8 -> y [n, rows] f32 */
void oracle_mxfp4_matmul(const float *x, int n, const uint8_t *w, const uint8_t *s,
                         int rows, int K, float *y) {
  const int G = K / 32;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r) {
    float wv[32];
    const uint8_t *wr = w + (size_t)r * (K / 2);
    const uint8_t *sr = s + (size_t)r * G;
    float acc[64];
    for (int t0 = 0; t0 < n; t0 += 64) {
      int nt = n - t0 < 64 ? n - t0 : 64;
      for (int t = 0; t < nt; ++t) acc[t] = 0.0f;
      for (int g = 0; g < G; ++g) {
        float sc = e8m0(sr[g]);
        for (int i = 0; i < 16; ++i) {
          uint8_t b = wr[g * 16 + i];
          wv[2 * i] = kE2M1[b & 15] * sc;
          wv[2 * i + 1] = kE2M1[b >> 4] * sc;
        }
        for (int t = 0; t < nt; ++t) {
          const float *xt = x + (size_t)(t0 + t) * K + g * 32;
          float a = 0.0f;
          for (int i = 0; i < 32; ++i) a += xt[i] * wv[i];
          acc[t] += a;
        }
      }
      for (int t = 0; t < nt; ++t) y[(size_t)(t0 + t) * rows + r] = acc[t];
    }
  }
}

/* affine4: w [rows, K/8] u32, scales/biases [rows, K/group] bf16 bits */
void oracle_affine4_matmul(const float *x, int n, const uint32_t *w, const uint16_t *scales,
                           const uint16_t *biases, int group, int rows, int K, float *y) {
  const int G = K / group;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r) {
    float wv[256];
    const uint32_t *wr = w + (size_t)r * (K / 8);
    float acc[64];
    for (int t0 = 0; t0 < n; t0 += 64) {
      int nt = n - t0 < 64 ? n - t0 : 64;
      for (int t = 0; t < nt; ++t) acc[t] = 0.0f;
      for (int g = 0; g < G; ++g) {
        float sc = bf16f(scales[(size_t)r * G + g]);
        float bi = bf16f(biases[(size_t)r * G + g]);
        for (int i = 0; i < group / 8; ++i) {
          uint32_t word = wr[g * (group / 8) + i];
          for (int j = 0; j < 8; ++j) wv[8 * i + j] = sc * (float)((word >> (4 * j)) & 15u) + bi;
        }
        for (int t = 0; t < nt; ++t) {
          const float *xt = x + (size_t)(t0 + t) * K + g * group;
          float a = 0.0f;
          for (int i = 0; i < group; ++i) a += xt[i] * wv[i];
          acc[t] += a;
        }
      }
      for (int t = 0; t < nt; ++t) y[(size_t)(t0 + t) * rows + r] = acc[t];
    }
  }
}
