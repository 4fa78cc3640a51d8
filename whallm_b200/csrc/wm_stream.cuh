// Building blocks of the CUDA-core weight-stream kernels (moe_stream.cu,
// linear_stream.cu): weights are widened to exact f16 pairs and multiplied by
// token values held as f16 with a power-of-two scale per 32 values, each
// product rounded once into an f32 sum (fma.rn.f32.f16).
#pragma once

#include "wm_common.cuh"

namespace wm_stream {

// eight e2m1 values (one 32-bit word) -> four exact f16 pairs
__device__ __forceinline__ void e2m1x8_to_f16x2(uint32_t w, uint32_t (&h)[4]) {
  asm("{.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;}"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(w));
}

// four e4m3 values (one 32-bit word, value i in byte i) -> two exact f16
// pairs (every e4m3 value, subnormals included, is an f16 value); pair j
// holds values 2j (low half) and 2j + 1
__device__ __forceinline__ void e4m3x4_to_f16x2(uint32_t w, uint32_t (&h)[2]) {
  asm("{.reg .b16 p0, p1;\n\t"
      "mov.b32 {p0, p1}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, p0;\n\t"
      "cvt.rn.f16x2.e4m3x2 %1, p1;}"
      : "=r"(h[0]), "=r"(h[1])
      : "r"(w));
}

// lo += a.lo * b.lo, hi += a.hi * b.hi: exact f16 products, one f32 rounding each
__device__ __forceinline__ void fma_f16x2_f32(uint32_t a, uint32_t b, float &lo, float &hi) {
  asm("{.reg .b16 a0, a1, b0, b1;\n\t"
      "mov.b32 {a0, a1}, %2;\n\t"
      "mov.b32 {b0, b1}, %3;\n\t"
      "fma.rn.f32.f16 %0, a0, b0, %0;\n\t"
      "fma.rn.f32.f16 %1, a1, b1, %1;}"
      : "+f"(lo), "+f"(hi)
      : "r"(a), "r"(b));
}

__device__ __forceinline__ uint32_t f32x2_to_f16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ float pow2f(int e) {  // 2^e for e in [-126, 127]
  return __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "l"(pol)
               : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void *src, uint64_t pol) {
  asm volatile("cp.async.ca.shared.global.L2::cache_hint [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "l"(pol)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Sums of V lane-held values over the warp.  Each xor step halves the values
// a lane carries (a transposed butterfly); every sum is built from the same
// pairs as a full butterfly of that value alone.  Afterwards lane l holds
// value (l >> (5 - log2 V)) & (V - 1), as do all lanes equal to it in the low
// bits.
template <int V>
__device__ __forceinline__ float warp_sums(float (&v)[V], int lane) {
#pragma unroll
  for (int m = 16, h = V / 2; h >= 1; m >>= 1, h >>= 1) {
    const bool hi = (lane & m) != 0;
#pragma unroll
    for (int i = 0; i < h; ++i) {
      const float send = hi ? v[i] : v[i + h];
      const float keep = hi ? v[i + h] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
    }
  }
  constexpr int kLow = 32 / V;               // lanes still holding partial sums of one value
  float s = v[0];
#pragma unroll
  for (int m = kLow / 2; m >= 1; m >>= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
  return s;
}

// One 32-value group of bf16 (four 16-byte words) -> f16 at d (64 bytes) with
// a power of two 2^-k chosen so the group's largest magnitude lies in
// [2^14, 2^15): every bf16 value within 2^-32 of the group maximum is then
// exact in f16 and smaller ones are off by less than 2^-39 of it.  Returns
// the factor 2^k that undoes the scaling (0 for an all-zero group).
__device__ __forceinline__ float stage_group_f16(const uint4 (&v)[4], uint4 *d) {
  uint32_t mx = 0u;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    mx = __vmaxu2(mx, v[i].x & 0x7fff7fffu);
    mx = __vmaxu2(mx, v[i].y & 0x7fff7fffu);
    mx = __vmaxu2(mx, v[i].z & 0x7fff7fffu);
    mx = __vmaxu2(mx, v[i].w & 0x7fff7fffu);
  }
  mx = max(mx & 0xffffu, mx >> 16);
  // the group maximum's exponent e (bf16 bits >> 7); values scale by 2^-k, k = e - 127 - 14
  const int k = max(static_cast<int>(mx >> 7) - 141, -100);
  const float down = pow2f(-k);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 o;
    o.x = f32x2_to_f16x2(wm_bf16lo(v[i].x) * down, wm_bf16hi(v[i].x) * down);
    o.y = f32x2_to_f16x2(wm_bf16lo(v[i].y) * down, wm_bf16hi(v[i].y) * down);
    o.z = f32x2_to_f16x2(wm_bf16lo(v[i].z) * down, wm_bf16hi(v[i].z) * down);
    o.w = f32x2_to_f16x2(wm_bf16lo(v[i].w) * down, wm_bf16hi(v[i].w) * down);
    d[i] = o;
  }
  return mx == 0u ? 0.0f : pow2f(k);
}

}  // namespace wm_stream
