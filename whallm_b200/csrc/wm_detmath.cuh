// Deterministic float32 exp / log / softplus for the router.
//
// Routing indices are compared exactly against a CPU restatement, so the
// router cannot use library transcendentals whose last-bit behaviour differs
// between host and device.  These functions use only IEEE-exact operations
// (+, -, *, /, fmaf, sqrtf, rintf, bit moves), so any IEEE host evaluating
// the same sequence gets the same bits.  The translation unit that includes
// this header is compiled with -fmad=false, so only the explicit fmaf calls
// fuse.
//
// exp:   Cody-Waite reduction x = n ln2 + r (ln 2 split into a high and a low
//        float32 part), exp(r) by its Taylor series through r^7/7! in Horner
//        form, scaled by 2^n through the exponent bits.  |r| <= ln2/2 makes
//        the truncation error about 5e-9 relative.
// log:   m in [sqrt(1/2), sqrt(2)), log m = 2 atanh(s), s = (m-1)/(m+1), series
//        through s^13/13 (|s| <= 0.1716), plus e ln2.
// log1p: Goldberg's form log(u) * y / (u - 1), u = 1 + y.
#pragma once

#include <stdint.h>

#define WM_LOG2E 0x1.715476p+0f
#define WM_LN2_HI 0x1.62e430p-1f
#define WM_LN2_LO -0x1.05c610p-29f
#define WM_SQRT2 0x1.6a09e6p+0f

__device__ __forceinline__ float wm_exp(float x) {
  if (x != x) return x;
  if (!(x > -104.0f)) return 0.0f;
  if (x > 88.72283935546875f) return __int_as_float(0x7f800000);
  float n = rintf(x * WM_LOG2E);
  float r = fmaf(-n, WM_LN2_HI, x);
  r = fmaf(-n, WM_LN2_LO, r);
  float p = 0x1.a01a02p-13f;
  p = fmaf(p, r, 0x1.6c16c2p-10f);
  p = fmaf(p, r, 0x1.111112p-7f);
  p = fmaf(p, r, 0x1.555556p-5f);
  p = fmaf(p, r, 0x1.555556p-3f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  int ni = static_cast<int>(n);
  if (ni > 127) { p = p * 2.0f; ni -= 1; }
  if (ni < -126) { p = p * 0x1p-64f; ni += 64; }
  return p * __uint_as_float(static_cast<uint32_t>(ni + 127) << 23);
}

// log of a positive, normal, finite float
__device__ __forceinline__ float wm_log(float u) {
  uint32_t b = __float_as_uint(u);
  int e = static_cast<int>((b >> 23) & 255u) - 127;
  float m = __uint_as_float((b & 0x7fffffu) | 0x3f800000u);
  if (m > WM_SQRT2) { m = m * 0.5f; e += 1; }
  float s = __fdiv_rn(m - 1.0f, m + 1.0f);
  float s2 = s * s;
  float p = 0x1.3b13b2p-4f;
  p = fmaf(p, s2, 0x1.745d18p-4f);
  p = fmaf(p, s2, 0x1.c71c72p-4f);
  p = fmaf(p, s2, 0x1.24924ap-3f);
  p = fmaf(p, s2, 0x1.99999ap-3f);
  p = fmaf(p, s2, 0x1.555556p-2f);
  float t = s2 * p;
  float s2x = 2.0f * s;
  float lm = fmaf(s2x, t, s2x);
  float fe = static_cast<float>(e);
  return fmaf(fe, WM_LN2_HI, fmaf(fe, WM_LN2_LO, lm));
}

__device__ __forceinline__ float wm_log1p(float y) {
  float u = 1.0f + y;
  if (u == 1.0f) return y;
  float q = __fdiv_rn(y, u - 1.0f);
  return wm_log(u) * q;
}

__device__ __forceinline__ float wm_softplus(float v) {
  return fmaxf(v, 0.0f) + wm_log1p(wm_exp(-fabsf(v)));
}

__device__ __forceinline__ float wm_sigmoid(float v) { return __fdiv_rn(1.0f, 1.0f + wm_exp(-v)); }
