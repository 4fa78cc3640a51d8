// Shared helpers for the whallm_b200 kernels: error reporting, bf16 and
// number-format bit manipulation.  sm_100a only.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/whallm_b200.h"

namespace wm {

// Thread-local message for w_last_error(); defined in capi.cu.
void set_error(const std::string &msg);
void clear_error();

inline int fail(int code, const std::string &msg) {
  set_error(msg);
  return code;
}

inline int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(WM_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return WM_OK;
}

inline bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Grid size helper: a multiple of the SM count (148 on B200), capped by work.
int sm_count();


// Programmatic dependent launch for the kernels of the MoE path: they are
// launched with programmatic stream serialization, so a kernel's CTAs may be
// scheduled (and run their set-up) while the previous kernel on the stream is
// still finishing.  Each kernel executes WM_PDL_WAIT() before it reads what
// earlier kernels wrote (it returns once those grids have completed and their
// memory is visible; a no-op for an ordinary launch) and WM_PDL_LAUNCH() to
// let its own successor be scheduled.
#define WM_PDL_WAIT() asm volatile("griddepcontrol.wait;" ::: "memory")
#define WM_PDL_LAUNCH() asm volatile("griddepcontrol.launch_dependents;" ::: "memory")

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace wm

#define WM_REQUIRE(cond, msg)                                   \
  do {                                                          \
    if (!(cond)) return ::wm::fail(WM_ERR_INVALID, (msg));      \
  } while (0)

// ---------------------------------------------------------------- device ---

__device__ __forceinline__ float wm_bf16_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// float32 -> bf16 bits, round to nearest even (NaN -> 0x7FC0).
__device__ __forceinline__ uint16_t wm_f32_to_bf16(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7FC0;
  u += 0x7fffu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

// Two bf16 packed in a uint32 (element 0 low) -> floats.
// Two fp32 lanes per instruction (sm_100 packed FMA / add): each lane is
// rounded exactly like fmaf / a scalar add, so the results are the same bits.
__device__ __forceinline__ unsigned long long wm_f2_bits(float2 v) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(v.x), "f"(v.y));
  return r;
}
__device__ __forceinline__ float2 wm_f2_of(unsigned long long r) {
  float2 v;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(r));
  return v;
}
__device__ __forceinline__ float2 wm_fma2(float2 a, float2 b, float2 c) {
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(wm_f2_bits(a)), "l"(wm_f2_bits(b)), "l"(wm_f2_bits(c)));
  return wm_f2_of(r);
}
__device__ __forceinline__ float2 wm_mul2(float2 a, float2 b) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(wm_f2_bits(a)), "l"(wm_f2_bits(b)));
  return wm_f2_of(r);
}
__device__ __forceinline__ float2 wm_add2(float2 a, float2 b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(wm_f2_bits(a)), "l"(wm_f2_bits(b)));
  return wm_f2_of(r);
}

__device__ __forceinline__ float wm_bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float wm_bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// E8M0 byte -> 2^(b-127) exactly (b=0 -> 2^-127 subnormal, b=255 -> +inf).
__device__ __forceinline__ float wm_e8m0(uint32_t b) {
  return b == 0 ? __uint_as_float(0x00400000u) : __uint_as_float(b << 23);
}

// e2m1 code (4 bits) -> value * 2^-126 as a float bit pattern: the 3
// magnitude bits land on the low exponent bits and the top mantissa bit, so
// code 1 (0.5) becomes the subnormal 2^-127 and code 8 becomes -0.0.
// Multiplying by 2^126 (exact, denormals are preserved: -ftz=false) gives
// the value.
__device__ __forceinline__ float wm_e2m1_scaled(uint32_t n) {
  return __uint_as_float(((n & 8u) << 28) | ((n & 7u) << 22));
}

// Exact e2m1 value; code 8 -> +0.0 as in the reference table.
__device__ __forceinline__ float wm_e2m1(uint32_t n) {
  float v = wm_e2m1_scaled(n) * 0x1p126f;
  return v + 0.0f;  // -0.0 + 0.0 = +0.0
}

// e4m3fn byte -> float (exact).
__device__ __forceinline__ float wm_e4m3_to_f32(uint32_t c) {
  uint32_t s = (c & 0x80u) << 24;
  uint32_t e = (c >> 3) & 15u, m = c & 7u;
  float v;
  if (e == 0) {
    v = static_cast<float>(m) * 0x1p-9f;
  } else if (e == 15 && m == 7) {
    return __uint_as_float(0x7fc00000u);
  } else {
    v = __uint_as_float(((e + 120u) << 23) | (m << 20));
  }
  return __uint_as_float(__float_as_uint(v) | s);
}

// float -> e4m3fn byte, round to nearest even, saturating to +-448 (callers
// clip first).  Written from the format definition: normals have 3 mantissa
// bits and exponent bias 7, subnormals are multiples of 2^-9.
__device__ __forceinline__ uint32_t wm_f32_to_e4m3(float f) {
  uint32_t sign = (__float_as_uint(f) >> 24) & 0x80u;
  float a = fminf(fabsf(f), 448.0f);
  if (!(a >= 0.001953125f * 0.5f)) {
    // below half the smallest subnormal (2^-10): rounds to zero (a==2^-10 ties to 0)
    return sign;
  }
  uint32_t ua = __float_as_uint(a);
  int ex = static_cast<int>((ua >> 23) & 255u) - 127;  // floor(log2 a), a is normal here
  if (ex < -6) ex = -6;
  // quantum q = 2^(ex-3); n = rint(a / q) computed exactly by scaling
  float n = rintf(a * __uint_as_float(static_cast<uint32_t>(127 - (ex - 3)) << 23));
  uint32_t ni = static_cast<uint32_t>(n);  // 0..16
  uint32_t code;
  if (ex == -6 && ni < 8) {
    code = ni;  // subnormal (or zero)
  } else {
    if (ni == 16) { ni = 8; ex += 1; }
    code = (static_cast<uint32_t>(ex + 7) << 3) | (ni - 8);
    if (code > 0x7eu) code = 0x7eu;
  }
  return sign | code;
}

// Swift fp4Code: nearest e2m1 magnitude (ties to the even code), saturating
// at 6; sign from the float's sign bit.
__device__ __forceinline__ uint32_t wm_e2m1_code(float v) {
  uint32_t neg = __float_as_uint(v) >> 31;
  float m = fminf(fabsf(v), 6.0f);
  uint32_t idx = (m > 0.25f) + (m >= 0.75f) + (m > 1.25f) + (m >= 1.75f) + (m > 2.5f) + (m >= 3.5f) +
                 (m > 5.0f);
  return idx | (neg << 3);
}
