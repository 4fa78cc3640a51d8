/*
 * CPU restatement of the MoE router, evaluated in a fixed float32 order.
 *
 * TEST INFRASTRUCTURE ONLY: the product library never links this file.
 *
 * Reference semantics restated here:
 *   gate logits  x @ W^T in float32      deepseek_v41/moe.py:59, qwen4_exp.py:693
 *   score functions softmax / sigmoid / sqrt(softplus)   deepseek_v41/moe.py:60-65
 *   selection on score + bias, bias not in the weights   deepseek_v41/moe.py:67-70
 *   ties resolved by expert position                     model.py:548-560
 *   renormalise by (sum + eps), times route_scale        deepseek_v41/moe.py:71-73
 *   Qwen: renormalise by sum (eps 0), no scale           qwen4_exp.py:693-697
 *   Qwen gate dtypes (score function SOFTMAX_BF16): the gate is a bf16
 *     nn.Linear, so its logits are rounded to bf16          qwen4_exp.py:683
 *     softmax(precise=True): float32 math, bf16 result     qwen4_exp.py:693
 *     top-k on the bf16 probabilities                      qwen4_exp.py:694-695
 *     scores / scores.sum(): bf16 sum, bf16 quotient       qwen4_exp.py:696-697
 *     shared gate sigmoid(bf16 logit) in bf16              qwen4_exp.py:699
 *     (every rounding to nearest even; the sum is taken in float32 in
 *     selection order and rounded once)
 *
 * The reference computes these with MLX kernels whose reduction order is not
 * specified.  To compare routing indices exactly, this oracle and the device
 * kernel agree on one order:
 *   logit[t][e]: the 256-wide column blocks are split into 4 contiguous
 *     segments; in each, partial l accumulates with fmaf the elements
 *     h = 256*i + 8*l + j (i ascending, then j = 0..7); the 4 segment
 *     partials of l are added in segment order; then a butterfly over the 32
 *     partials with strides 16, 8, 4, 2, 1.
 *   softmax sum: partial l sums experts l, l+32, l+64, ... in order, then the
 *     same butterfly.
 *   exp / log: Cody-Waite argument reduction (ln 2 split in a high and a low
 *     part) with the Taylor series of exp truncated after r^7/7!, and
 *     log(m) = 2 atanh((m-1)/(m+1)) truncated after s^13/13; log1p uses
 *     Goldberg's log(1+y) = log(u) * y / (u-1) with u = 1+y.
 * Compile with -ffp-contract=off so that only the explicit fmaf calls fuse
 * (with -mfma they are single fused instructions, the same IEEE operation).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define LOG2E 0x1.715476p+0f
#define LN2_HI 0x1.62e430p-1f
#define LN2_LO -0x1.05c610p-29f
#define SQRT2 0x1.6a09e6p+0f

static inline float bits_f(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static inline uint32_t f_bits(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }
static inline float bf16f(uint16_t b) { return bits_f(((uint32_t)b) << 16); }

/* float32 -> nearest bf16 (ties to even), returned as float32 */
static inline float round_bf16(float f) {
  uint32_t u = f_bits(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return bits_f(0x7fc00000u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return bits_f(u & 0xffff0000u);
}

float oracle_exp(float x) {
  if (x != x) return x;
  if (!(x > -104.0f)) return 0.0f;
  if (x > 88.72283935546875f) return INFINITY;
  float n = rintf(x * LOG2E);
  float r = fmaf(-n, LN2_HI, x);
  r = fmaf(-n, LN2_LO, r);
  float p = 0x1.a01a02p-13f;          /* 1/7! */
  p = fmaf(p, r, 0x1.6c16c2p-10f);    /* 1/6! */
  p = fmaf(p, r, 0x1.111112p-7f);     /* 1/5! */
  p = fmaf(p, r, 0x1.555556p-5f);     /* 1/4! */
  p = fmaf(p, r, 0x1.555556p-3f);     /* 1/3! */
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  int ni = (int)n;
  if (ni > 127) { p = p * 2.0f; ni -= 1; }
  if (ni < -126) { p = p * 0x1p-64f; ni += 64; }
  return p * bits_f((uint32_t)(ni + 127) << 23);
}

/* natural log of a positive, normal, finite float */
float oracle_log(float u) {
  uint32_t b = f_bits(u);
  int e = (int)((b >> 23) & 255u) - 127;
  float m = bits_f((b & 0x7fffffu) | 0x3f800000u);
  if (m > SQRT2) { m = m * 0.5f; e += 1; }
  float s = (m - 1.0f) / (m + 1.0f);
  float s2 = s * s;
  float p = 0x1.3b13b2p-4f;           /* 1/13 */
  p = fmaf(p, s2, 0x1.745d18p-4f);    /* 1/11 */
  p = fmaf(p, s2, 0x1.c71c72p-4f);    /* 1/9 */
  p = fmaf(p, s2, 0x1.24924ap-3f);    /* 1/7 */
  p = fmaf(p, s2, 0x1.99999ap-3f);    /* 1/5 */
  p = fmaf(p, s2, 0x1.555556p-2f);    /* 1/3 */
  float t = s2 * p;
  float s2x = 2.0f * s;
  float lm = fmaf(s2x, t, s2x);
  float fe = (float)e;
  return fmaf(fe, LN2_HI, fmaf(fe, LN2_LO, lm));
}

float oracle_log1p(float y) {
  float u = 1.0f + y;
  if (u == 1.0f) return y;
  float q = y / (u - 1.0f);
  return oracle_log(u) * q;
}

float oracle_softplus(float v) {
  return fmaxf(v, 0.0f) + oracle_log1p(oracle_exp(-fabsf(v)));
}

static float butterfly32(float *p) {
  float a[32];
  memcpy(a, p, sizeof(a));
  for (int m = 16; m >= 1; m >>= 1) {
    float b[32];
    for (int l = 0; l < 32; ++l) b[l] = a[l] + a[l ^ m];
    memcpy(a, b, sizeof(a));
  }
  return a[0];
}

/* x.w in the device order: the 256-wide column blocks i = 0..n-1 (n = ceil(H/256))
 * are split into 4 contiguous segments [floor(s*n/4), floor((s+1)*n/4)); lane l
 * of segment s accumulates, with fmaf, the elements 256*i + 8*l + j (i ascending,
 * j = 0..7); the four segment partials of a lane are added in segment order;
 * the 32 lane sums are combined by the butterfly. */
float oracle_dot_bf16(const uint16_t *x, const uint16_t *w, int H) {
  const int n = (H + 255) / 256;
  float part[32];
  for (int l = 0; l < 32; ++l) {
    float seg[4];
    for (int sgi = 0; sgi < 4; ++sgi) {
      float acc = 0.0f;
      for (int i = (sgi * n) / 4; i < ((sgi + 1) * n) / 4; ++i) {
        const int base = 256 * i + 8 * l;
        if (base >= H) continue;
        for (int j = 0; j < 8; ++j) acc = fmaf(bf16f(x[base + j]), bf16f(w[base + j]), acc);
      }
      seg[sgi] = acc;
    }
    part[l] = ((seg[0] + seg[1]) + seg[2]) + seg[3];
  }
  return butterfly32(part);
}

enum { SCORE_SOFTMAX = 0, SCORE_SIGMOID = 1, SCORE_SQRTSOFTPLUS = 2, SCORE_NONE = 3, SCORE_SOFTMAX_BF16 = 4 };

/* Scores and top-k for one token from its E logits (already biased). */
static void topk_one(const float *logit, int E, int k, int score_fn, const float *select_bias,
                     float norm_eps, float route_scale, float *score, int32_t *idx, float *wout) {
  const int bf = score_fn == SCORE_SOFTMAX_BF16;
  if (score_fn == SCORE_SOFTMAX || bf) {
    float mx = -INFINITY;
    for (int e = 0; e < E; ++e) score[e] = bf ? round_bf16(logit[e]) : logit[e];
    for (int e = 0; e < E; ++e) mx = fmaxf(mx, score[e]);
    float part[32];
    for (int l = 0; l < 32; ++l) part[l] = 0.0f;
    for (int e = 0; e < E; ++e) score[e] = oracle_exp(score[e] - mx);
    for (int l = 0; l < 32; ++l)
      for (int e = l; e < E; e += 32) part[l] = part[l] + score[e];
    float sum = butterfly32(part);
    for (int e = 0; e < E; ++e) score[e] = bf ? round_bf16(score[e] / sum) : score[e] / sum;
  } else if (score_fn == SCORE_SIGMOID) {
    for (int e = 0; e < E; ++e) score[e] = 1.0f / (1.0f + oracle_exp(-logit[e]));
  } else if (score_fn == SCORE_SQRTSOFTPLUS) {
    for (int e = 0; e < E; ++e) score[e] = sqrtf(oracle_softplus(logit[e]));
  } else {
    for (int e = 0; e < E; ++e) score[e] = logit[e];
  }
  unsigned char taken[4096];
  memset(taken, 0, (size_t)E);
  for (int j = 0; j < k; ++j) {
    int best = -1;
    float bk = 0.0f;
    for (int e = 0; e < E; ++e) {
      if (taken[e]) continue;
      float key = select_bias ? score[e] + select_bias[e] : score[e];
      if (key != key) key = -INFINITY; /* NaN keys rank last */
      if (best < 0 || key > bk) { best = e; bk = key; }
    }
    taken[best] = 1;
    idx[j] = best;
    wout[j] = score[best];
  }
  if (norm_eps >= 0.0f) {
    float s = 0.0f;
    for (int j = 0; j < k; ++j) s = s + wout[j];
    s = s + norm_eps;
    if (bf) s = round_bf16(s);
    for (int j = 0; j < k; ++j) wout[j] = bf ? round_bf16(wout[j] / s) : wout[j] / s;
  }
  for (int j = 0; j < k; ++j) wout[j] = wout[j] * route_scale;
}

/*
 * x [T,H] bf16 bits, wg [E,H] bf16 bits, logit_bias/select_bias [E] or NULL.
 * Writes logits [T,E] (biased), idx [T,k], weights [T,k].
 * wg_shared [H] or NULL: shared-expert gate row, shared_w[t] = sigmoid(x.wg_shared)
 * (qwen4_exp.py:699).  Returns 0, or -1 for unsupported sizes.
 */
int oracle_router(const uint16_t *x, const uint16_t *wg, const float *logit_bias,
                  const float *select_bias, int T, int H, int E, int k, int score_fn,
                  float norm_eps, float route_scale, const uint16_t *wg_shared,
                  float *logits, int32_t *idx, float *weights, float *shared_w) {
  if (E > 4096 || k > E || k < 1 || H % 8) return -1;
  /* tokens are independent: split across OpenMP threads (each token's
   * arithmetic is unchanged) */
#pragma omp parallel for schedule(dynamic, 4)
  for (int t = 0; t < T; ++t) {
    float score[4096];
    const uint16_t *xt = x + (size_t)t * H;
    float *lt = logits + (size_t)t * E;
    for (int e = 0; e < E; ++e) {
      float l = oracle_dot_bf16(xt, wg + (size_t)e * H, H);
      lt[e] = logit_bias ? l + logit_bias[e] : l;
    }
    topk_one(lt, E, k, score_fn, select_bias, norm_eps, route_scale, score,
             idx + (size_t)t * k, weights + (size_t)t * k);
    if (wg_shared && shared_w) {
      float g = oracle_dot_bf16(xt, wg_shared, H);
      if (score_fn == SCORE_SOFTMAX_BF16)
        shared_w[t] = round_bf16(1.0f / (1.0f + oracle_exp(-round_bf16(g))));
      else
        shared_w[t] = 1.0f / (1.0f + oracle_exp(-g));
    }
  }
  return 0;
}

/* Vectorised entry points used by tests to pin the math helpers. */
void oracle_exp_n(const float *x, float *y, int n) { for (int i = 0; i < n; ++i) y[i] = oracle_exp(x[i]); }
void oracle_softplus_n(const float *x, float *y, int n) { for (int i = 0; i < n; ++i) y[i] = oracle_softplus(x[i]); }
