// Number-format kernels: MXFP4 and affine-4 weights, KV-cache row formats.
//
// All of these are HBM-bound elementwise passes.  One thread owns one scale
// group (16..64 values), reads it with 16-byte loads and writes its packed
// bytes and scale; consecutive threads own consecutive groups, so warps read
// and write contiguous spans.  Results are bit-exact against the CPU
// restatement: only IEEE-exact float32 operations are used and this file is
// compiled with -fmad=false.
#include <cuda_fp16.h>

#include <algorithm>

#include "wm_common.cuh"

namespace {

constexpr float kFp8MaxInv = 0x1.24924ap-9f;  // float32(1/448)  (fakequant.py:34)
constexpr float kFp4MaxInv = 0x1.555556p-3f;  // float32(1/6)    (fakequant.py:35)
constexpr float kFp8Floor = 0x1.a36e2ep-14f;  // float32(1e-4)   (packed_cache.py:34)
constexpr float kFp4UeFloor = 0x1.8p-124f;    // 6 * 2^-126      (packed_cache.py:35)
constexpr float kFp4E4Floor = 0x1.8p-7f;      // 6 * 2^-9        (packed_cache.py:29)

// floor(log2 a) for positive finite a (subnormals included) == Swift Float.exponent
__device__ __forceinline__ int floor_log2(float a) {
  uint32_t b = __float_as_uint(a);
  uint32_t ex = (b >> 23) & 255u;
  if (ex != 0) return static_cast<int>(ex) - 127;
  uint32_t m = b & 0x7fffffu;
  return (31 - __clz(static_cast<int>(m))) - 149;
}

// 2^k as float for k in [-149, 127], exact
__device__ __forceinline__ float pow2i(int k) {
  if (k >= -126) return __uint_as_float(static_cast<uint32_t>(k + 127) << 23);
  return __uint_as_float(1u << (k + 149));
}

// ceil(log2 x) via IEEE bits for positive normal x (fakequant.py:47-52)
__device__ __forceinline__ int ceil_log2_bits(float x) {
  uint32_t b = __float_as_uint(x);
  int e = static_cast<int>((b >> 23) & 255u) - 127;
  return e + ((b & 0x7fffffu) != 0 ? 1 : 0);
}

__device__ __forceinline__ void load_bf16x32(const uint16_t *p, float *v) {
  const uint4 *q = reinterpret_cast<const uint4 *>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 u = __ldg(q + i);
    uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[8 * i + 2 * j] = wm_bf16lo(w[j]);
      v[8 * i + 2 * j + 1] = wm_bf16hi(w[j]);
    }
  }
}

// Swift MXFP4.quantizeBF16 (MXFP4.swift:19-37) on 32 float32 values.
__device__ __forceinline__ void mxfp4_group(const float *v, uint8_t *out16, uint8_t *scale) {
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  uint32_t words[4] = {0u, 0u, 0u, 0u};
  if (amax == 0.0f) {
    *scale = 0;
  } else {
    int e = floor_log2(amax) - 2;
    e = max(-127, min(128, e));
    *scale = static_cast<uint8_t>(e + 127);
    float f = pow2i(-e);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      uint32_t c = wm_e2m1_code(v[i] * f);
      words[i >> 3] |= c << (4 * (i & 7));
    }
  }
  *reinterpret_cast<uint4 *>(out16) = make_uint4(words[0], words[1], words[2], words[3]);
}

__global__ void k_mxfp4_quantize(const uint16_t *__restrict__ src, int64_t groups,
                                 uint8_t *__restrict__ packed, uint8_t *__restrict__ scales) {
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < groups;
       g += (int64_t)gridDim.x * blockDim.x) {
    float v[32];
    load_bf16x32(src + g * 32, v);
    mxfp4_group(v, packed + g * 16, scales + g);
  }
}

template <typename OutT>
__device__ __forceinline__ void store32(OutT *dst, const float *v);

template <>
__device__ __forceinline__ void store32<float>(float *dst, const float *v) {
  float4 *d = reinterpret_cast<float4 *>(dst);
#pragma unroll
  for (int i = 0; i < 8; ++i) d[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

template <>
__device__ __forceinline__ void store32<uint16_t>(uint16_t *dst, const float *v) {
  uint4 *d = reinterpret_cast<uint4 *>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      w[j] = wm_f32_to_bf16(v[8 * i + 2 * j]) | (static_cast<uint32_t>(wm_f32_to_bf16(v[8 * i + 2 * j + 1])) << 16);
    d[i] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

template <typename OutT>
__global__ void k_mxfp4_dequantize(const uint8_t *__restrict__ packed, const uint8_t *__restrict__ scales,
                                   int64_t groups, OutT *__restrict__ out) {
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < groups;
       g += (int64_t)gridDim.x * blockDim.x) {
    uint4 u = __ldg(reinterpret_cast<const uint4 *>(packed) + g);
    float s = wm_e8m0(scales[g]);
    uint32_t w[4] = {u.x, u.y, u.z, u.w};
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = wm_e2m1((w[i >> 3] >> (4 * (i & 7))) & 15u) * s;
    store32<OutT>(out + g * 32, v);
  }
}

// ------------------------------------------------------------ affine 4 ----

__global__ void k_affine4_quantize(const uint16_t *__restrict__ src, int64_t groups, int group,
                                   uint32_t *__restrict__ packed, uint16_t *__restrict__ scales,
                                   uint16_t *__restrict__ biases) {
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < groups;
       g += (int64_t)gridDim.x * blockDim.x) {
    const uint16_t *p = src + g * group;
    float wmax = -__int_as_float(0x7f800000), wmin = __int_as_float(0x7f800000);
    for (int i = 0; i < group; i += 32) {
      float v[32];
      load_bf16x32(p + i, v);
#pragma unroll
      for (int j = 0; j < 32; ++j) { wmax = fmaxf(wmax, v[j]); wmin = fminf(wmin, v[j]); }
    }
    bool mask = fabsf(wmin) > fabsf(wmax);
    float scale = fmaxf(__fdiv_rn(wmax - wmin, 15.0f), 1e-7f);
    scale = mask ? scale : -scale;
    float edge = mask ? wmin : wmax;
    float q0 = rintf(__fdiv_rn(edge, scale));
    if (q0 != 0.0f) scale = __fdiv_rn(edge, q0);
    float bias = q0 == 0.0f ? 0.0f : edge;
    uint32_t *dst = packed + g * (group / 8);
    for (int i = 0; i < group; i += 32) {
      float v[32];
      load_bf16x32(p + i, v);
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        uint32_t word = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float q = rintf(__fdiv_rn(v[8 * w + j] - bias, scale));
          q = fminf(fmaxf(q, 0.0f), 15.0f);
          word |= static_cast<uint32_t>(q) << (4 * j);
        }
        dst[i / 8 + w] = word;
      }
    }
    scales[g] = wm_f32_to_bf16(scale);
    biases[g] = wm_f32_to_bf16(bias);
  }
}

template <typename OutT>
__global__ void k_affine4_dequantize(const uint32_t *__restrict__ packed, const uint16_t *__restrict__ scales,
                                     const uint16_t *__restrict__ biases, int64_t chunks, int group,
                                     OutT *__restrict__ out) {
  // one thread per 32 values (a quarter or half group)
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < chunks;
       c += (int64_t)gridDim.x * blockDim.x) {
    int64_t g = (c * 32) / group;
    float s = wm_bf16_to_f32(scales[g]);
    float b = wm_bf16_to_f32(biases[g]);
    uint4 u = __ldg(reinterpret_cast<const uint4 *>(packed) + c);
    uint32_t w[4] = {u.x, u.y, u.z, u.w};
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = s * static_cast<float>((w[i >> 3] >> (4 * (i & 7))) & 15u) + b;
    store32<OutT>(out + c * 32, v);
  }
}

// --------------------------------------------------- affine KV (QSA) ----
// mlx-lm QuantizedKVCache with group 32 and 4 or 8 bits, as the Qwen QSA
// cache configures it (qwen_quantized_cache.py:6-20).  The cache of one
// tensor (keys or values) is packed uint32 [n_seq, capacity, D*BITS/32]
// (element 0 in the lowest bits) with bf16 scales and biases
// [n_seq, capacity, D/32]; n_seq = batch * kv heads.  blockIdx.y selects
// keys (0) or values (1), so one launch serves both.
// Division of a uint32 n by an invariant d >= 1 with one multiply-high, add
// and shift (Granlund & Montgomery, "Division by invariant integers using
// multiplication", PLDI 1994, fig. 4.1): l = ceil(log2 d),
// m = floor(2^32 (2^l - d) / d) + 1, n / d = (mulhi(n, m) + n) >> l, the sum
// taken in 64 bits.  Exact for every n < 2^32.
struct DivU32 {
  uint32_t m, l, d;
};

DivU32 make_divu32(uint32_t d) {
  uint32_t l = 0;
  while ((uint64_t(1) << l) < d) ++l;
  uint64_t m = ((uint64_t(1) << 32) * ((uint64_t(1) << l) - d)) / d + 1;
  return DivU32{static_cast<uint32_t>(m), l, d};
}

__device__ __forceinline__ uint32_t divu32(uint32_t n, DivU32 q) {
  return static_cast<uint32_t>((static_cast<uint64_t>(__umulhi(n, q.m)) + n) >> q.l);
}

struct AffineKV {
  const uint16_t *src[2];
  uint32_t *q[2];
  uint16_t *s[2];
  uint16_t *b[2];
  uint16_t *out[2];
};

// Per-group scale and bias of the affine scheme (the endpoint with the larger
// magnitude is represented exactly; see k_affine4_quantize).
__device__ __forceinline__ void affine_params(float wmin, float wmax, float nbins, float &scale, float &bias) {
  bool mask = fabsf(wmin) > fabsf(wmax);
  scale = fmaxf(__fdiv_rn(wmax - wmin, nbins), 1e-7f);
  scale = mask ? scale : -scale;
  float edge = mask ? wmin : wmax;
  float q0 = rintf(__fdiv_rn(edge, scale));
  if (q0 != 0.0f) scale = __fdiv_rn(edge, q0);
  bias = q0 == 0.0f ? 0.0f : edge;
}

// Quantize n_seq x L new rows into cache rows [offset, offset + L) of each
// sequence.  A thread owns 8 consecutive values (one 16-byte load); the four
// lanes of a 32-value group agree on its min/max by shuffles, and a warp
// covers 256 consecutive values, so loads and stores are contiguous.  The
// loop runs per warp (every lane takes the same trip count) so that the
// shuffles always see the whole warp; lanes past the end compute on zeros
// and store nothing.
template <int BITS>
__global__ void k_affine_kv_append(AffineKV a, uint32_t chunks, DivU32 cpr, DivU32 L, int64_t capacity,
                                   int64_t offset) {
  constexpr float kBins = static_cast<float>((1 << BITS) - 1);
  const int t = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const uint16_t *src = a.src[t];
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t base = blockIdx.x * blockDim.x + (threadIdx.x & ~31u); base < chunks; base += stride) {
    const uint32_t c = base + lane;
    const bool ok = c < chunks;
    float v[8];
    uint4 u = ok ? __ldg(reinterpret_cast<const uint4 *>(src) + c) : make_uint4(0, 0, 0, 0);
    const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[2 * j] = wm_bf16lo(w4[j]);
      v[2 * j + 1] = wm_bf16hi(w4[j]);
    }
    float wmax = v[0], wmin = v[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) { wmax = fmaxf(wmax, v[j]); wmin = fminf(wmin, v[j]); }
#pragma unroll
    for (int m = 1; m < 4; m <<= 1) {
      wmax = fmaxf(wmax, __shfl_xor_sync(0xffffffffu, wmax, m));
      wmin = fminf(wmin, __shfl_xor_sync(0xffffffffu, wmin, m));
    }
    float scale, bias;
    affine_params(wmin, wmax, kBins, scale, bias);
    // q = clamp(rint(RN((v - bias) / scale)), 0, bins).  The quotient is taken
    // as (v - bias) * RN(1/scale), which differs from the correctly rounded
    // one by under 2^-14 for |quotient| < 2^9; it can only round to another
    // integer when it lies within that distance of a half-integer, so there
    // (a 2^-10 window) the exact IEEE division decides.  Beyond 2^9 both
    // clamp to the same end.
    const float rcp = __frcp_rn(scale);
    uint32_t q8[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float x = v[j] - bias;
      float y = x * rcp;
      const float f = y - floorf(y);
      if (fabsf(f - 0.5f) < 0x1p-10f) y = __fdiv_rn(x, scale);
      const float q = fminf(fmaxf(rintf(y), 0.0f), kBins);
      q8[j] = __float_as_uint(q + 8388608.0f) & 0xFFu;   // integer q in [0, 255], exactly
    }
    if (!ok) continue;
    const uint32_t r = divu32(c, cpr);
    const uint32_t col = c - r * cpr.d;                      // 8-value chunk within the row
    const uint32_t seq = divu32(r, L);
    const int64_t row = static_cast<int64_t>(seq) * capacity + offset + (r - seq * L.d);
    uint32_t *dst = a.q[t] + row * (int64_t)cpr.d * (BITS / 4) + col * (BITS / 4);
    if (BITS == 4) {
      uint32_t word = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) word |= q8[j] << (4 * j);
      *dst = word;
    } else {
      uint32_t lo = q8[0] | (q8[1] << 8) | (q8[2] << 16) | (q8[3] << 24);
      uint32_t hi = q8[4] | (q8[5] << 8) | (q8[6] << 16) | (q8[7] << 24);
      *reinterpret_cast<uint2 *>(dst) = make_uint2(lo, hi);
    }
    if ((col & 3) == 0) {
      const int64_t gi = row * (cpr.d / 4) + col / 4;
      a.s[t][gi] = wm_f32_to_bf16(scale);
      a.b[t][gi] = wm_f32_to_bf16(bias);
    }
  }
}

// 0x4B000000 | code i of w: the float 2^23 + code.  For 8 bits one byte
// permute; for 4 bits a shift and a mask.
template <int BITS>
__device__ __forceinline__ uint32_t code_bits(uint32_t w, int i) {
  if (BITS == 8) return __byte_perm(w, 0x4B000000u, 0x7440u | static_cast<uint32_t>(i));
  return ((w >> (4 * i)) & 15u) | 0x4B000000u;
}

// Two floats -> bf16x2 (lo in the low half), round to nearest even, one cvt.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// Dequantize cache rows [0, L) of each sequence to bf16 [n_seq, L, D]:
// w = float32(scale) * q + float32(bias), rounded once to bf16 (scale * q is
// exact: an 8-bit significand times an integer below 256).  A thread
// reads 8 packed bytes (8 values at 8 bits, 16 at 4 bits) and writes them as
// one or two 16-byte stores; consecutive threads cover consecutive values.
template <int BITS>
__global__ void k_affine_kv_fetch(AffineKV a, uint32_t chunks, DivU32 cpr, DivU32 L, int64_t capacity) {
  constexpr int kVals = 64 / BITS;   // values per thread
  constexpr int kPer = 32 / BITS;    // values per uint32
  constexpr int kCpg = 32 / kVals;   // threads per 32-value scale group
  const int t = blockIdx.y;
  for (uint32_t c = blockIdx.x * blockDim.x + threadIdx.x; c < chunks; c += gridDim.x * blockDim.x) {
    const uint32_t r = divu32(c, cpr);
    const uint32_t col = c - r * cpr.d;
    const uint32_t seq = divu32(r, L);
    const int64_t row = static_cast<int64_t>(seq) * capacity + (r - seq * L.d);
    const int64_t gi = row * (cpr.d / kCpg) + col / kCpg;
    const float s = wm_bf16_to_f32(__ldg(a.s[t] + gi));
    const float b = wm_bf16_to_f32(__ldg(a.b[t] + gi));
    // a row holds D*BITS/32 = 2*cpr words
    const uint2 u = __ldg(reinterpret_cast<const uint2 *>(a.q[t] + row * (int64_t)cpr.d * 2) + col);
    const uint32_t w[2] = {u.x, u.y};
    uint32_t o[kVals / 2];
#pragma unroll
    for (int j = 0; j < kVals / 2; ++j) {
      const int e = 2 * j;
      // q as float, exactly: the code in the low mantissa bits of 2^23, minus 2^23
      const float q0 = __uint_as_float(code_bits<BITS>(w[e / kPer], e % kPer)) - 8388608.0f;
      const float q1 = __uint_as_float(code_bits<BITS>(w[e / kPer], e % kPer + 1)) - 8388608.0f;
      o[j] = pack_bf16x2(s * q0 + b, s * q1 + b);
    }
    uint4 *dst = reinterpret_cast<uint4 *>(a.out[t]) + static_cast<int64_t>(c) * (kVals / 8);   // values c*kVals..
#pragma unroll
    for (int i = 0; i < kVals / 8; ++i) __stcs(dst + i, make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]));
  }
}

// ------------------------------------------------------------- KV rows ----

__device__ __forceinline__ int kv_block(int fmt) {
  return fmt == WKV_FP8_F32_B64 ? 64 : (fmt == WKV_FP4_E4M3_B16 ? 16 : 32);
}
__device__ __host__ __forceinline__ int kv_bits(int fmt) {
  return (fmt == WKV_FP8_F32_B64 || fmt == WKV_FP8_UE8M0_B32 || fmt == WKV_MXFP8_B32) ? 8 : 4;
}

// e2m1 code of _e2m1_round(v) with the packed-cache sign rule:
// sign only for a nonzero negative result (packed_cache.py:40-42).
__device__ __forceinline__ uint32_t packed_fp4_code(float v) {
  float m = fabsf(v);
  uint32_t idx = (m > 0.25f) + (m > 1.25f) + (m > 2.5f) + (m > 5.0f) + (m >= 0.75f) + (m >= 1.75f) + (m >= 3.5f);
  return idx | ((idx != 0u && v < 0.0f) ? 8u : 0u);
}

// quantize one block of `blk` values (blk = 16, 32 or 64) starting at x
__device__ void kv_quant_block(const uint16_t *x, int blk, int fmt, uint8_t *payload, void *scales, int64_t sidx) {
  float v[64];
  for (int i = 0; i < blk; i += 32) {
    if (blk == 16) {
      const uint4 *q = reinterpret_cast<const uint4 *>(x);
      for (int a = 0; a < 2; ++a) {
        uint4 u = __ldg(q + a);
        uint32_t w[4] = {u.x, u.y, u.z, u.w};
        for (int j = 0; j < 4; ++j) { v[8 * a + 2 * j] = wm_bf16lo(w[j]); v[8 * a + 2 * j + 1] = wm_bf16hi(w[j]); }
      }
    } else {
      load_bf16x32(x + i, v + i);
    }
  }
  float amax = 0.0f;
  for (int i = 0; i < blk; ++i) amax = fmaxf(amax, fabsf(v[i]));
  if (fmt == WKV_MXFP4_B32) {
    uint8_t sc;
    mxfp4_group(v, payload, &sc);
    static_cast<uint8_t *>(scales)[sidx] = sc;
    return;
  }
  if (fmt == WKV_FP8_F32_B64 || fmt == WKV_FP8_UE8M0_B32 || fmt == WKV_MXFP8_B32) {
    float s = 0.0f, f = 1.0f;
    bool zero = false;
    bool mul = false;
    if (fmt == WKV_FP8_F32_B64) {
      s = __fdiv_rn(amax, 448.0f);
      zero = !(s > 0.0f);
      static_cast<float *>(scales)[sidx] = s;
    } else if (fmt == WKV_FP8_UE8M0_B32) {
      int e = ceil_log2_bits(fmaxf(amax, kFp8Floor) * kFp8MaxInv);
      s = __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
      static_cast<uint8_t *>(scales)[sidx] = static_cast<uint8_t>(e + 127);
    } else {
      zero = amax == 0.0f;
      int e = zero ? 0 : max(-127, min(127, floor_log2(amax) - 8));
      f = pow2i(-e);
      mul = true;
      static_cast<uint8_t *>(scales)[sidx] = zero ? 0 : static_cast<uint8_t>(e + 127);
    }
    for (int i = 0; i < blk; i += 4) {
      uint32_t word = 0;
      for (int j = 0; j < 4; ++j) {
        float q = 0.0f;
        if (!zero) {
          q = mul ? v[i + j] * f : __fdiv_rn(v[i + j], s);
          q = fminf(fmaxf(q, -448.0f), 448.0f);
        }
        uint32_t c = zero ? (__float_as_uint(v[i + j]) >> 31 ? 0u : 0u) : wm_f32_to_e4m3(q);
        word |= c << (8 * j);
      }
      reinterpret_cast<uint32_t *>(payload)[i / 4] = word;
    }
    return;
  }
  // fp4 packed-cache formats
  float s;
  if (fmt == WKV_FP4_E4M3_B16) {
    uint32_t enc = wm_f32_to_e4m3(__fdiv_rn(fmaxf(amax, kFp4E4Floor), 6.0f));
    s = wm_e4m3_to_f32(enc);
    static_cast<uint8_t *>(scales)[sidx] = static_cast<uint8_t>(enc);
  } else {
    int e = ceil_log2_bits(fmaxf(amax, kFp4UeFloor) * kFp4MaxInv);
    s = __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
    static_cast<uint8_t *>(scales)[sidx] = static_cast<uint8_t>(e + 127);
  }
  for (int i = 0; i < blk; i += 8) {
    uint32_t word = 0;
    for (int j = 0; j < 8; ++j) {
      float q = fminf(fmaxf(__fdiv_rn(v[i + j], s), -6.0f), 6.0f);
      word |= packed_fp4_code(q) << (4 * j);
    }
    reinterpret_cast<uint32_t *>(payload)[i / 8] = word;
  }
}

__global__ void k_kv_quantize(const uint16_t *__restrict__ x, int64_t rows, int D, int fmt,
                              uint8_t *__restrict__ payload, void *__restrict__ scales) {
  const int blk = kv_block(fmt);
  const int nb = D / blk;
  const int bits = kv_bits(fmt);
  const int64_t total = rows * nb;
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < total;
       b += (int64_t)gridDim.x * blockDim.x) {
    kv_quant_block(x + b * blk, blk, fmt, payload + b * blk * bits / 8, scales, b);
  }
}

__device__ __forceinline__ float kv_scale(const void *scales, int64_t sidx, int fmt) {
  if (fmt == WKV_FP8_F32_B64) return static_cast<const float *>(scales)[sidx];
  uint32_t b = static_cast<const uint8_t *>(scales)[sidx];
  if (fmt == WKV_FP4_E4M3_B16) return wm_e4m3_to_f32(b);
  if (fmt == WKV_MXFP8_B32 || fmt == WKV_MXFP4_B32) return wm_e8m0(b);
  return __uint_as_float(b << 23);  // PackedRows: (scale << 23).view(float32)
}

__device__ void kv_dequant_block(const uint8_t *payload, float s, int blk, int fmt, uint16_t *out) {
  const int bits = kv_bits(fmt);
  for (int i = 0; i < blk; i += 8) {
    float v[8];
    if (bits == 8) {
      uint2 u = *reinterpret_cast<const uint2 *>(payload + i);
      uint32_t w[2] = {u.x, u.y};
      for (int j = 0; j < 8; ++j) v[j] = wm_e4m3_to_f32((w[j >> 2] >> (8 * (j & 3))) & 255u) * s;
    } else {
      uint32_t w = *reinterpret_cast<const uint32_t *>(payload + i / 2);
      for (int j = 0; j < 8; ++j) {
        uint32_t c = (w >> (4 * j)) & 15u;
        float q = fmt == WKV_MXFP4_B32 ? wm_e2m1(c) : wm_e2m1_scaled(c) * 0x1p126f;
        v[j] = q * s;
      }
    }
    uint4 o;
    o.x = wm_f32_to_bf16(v[0]) | (static_cast<uint32_t>(wm_f32_to_bf16(v[1])) << 16);
    o.y = wm_f32_to_bf16(v[2]) | (static_cast<uint32_t>(wm_f32_to_bf16(v[3])) << 16);
    o.z = wm_f32_to_bf16(v[4]) | (static_cast<uint32_t>(wm_f32_to_bf16(v[5])) << 16);
    o.w = wm_f32_to_bf16(v[6]) | (static_cast<uint32_t>(wm_f32_to_bf16(v[7])) << 16);
    *reinterpret_cast<uint4 *>(out + i) = o;
  }
}

__global__ void k_kv_dequantize(const uint8_t *__restrict__ payload, const void *__restrict__ scales,
                                int64_t rows, const int32_t *__restrict__ row_idx, int64_t n, int D, int fmt,
                                uint16_t *__restrict__ out) {
  const int blk = kv_block(fmt);
  const int nb = D / blk;
  const int bits = kv_bits(fmt);
  const int64_t total = n * nb;
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < total;
       b += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = b / nb, j = b % nb;
    int64_t src = r;
    if (row_idx) {
      int64_t q = row_idx[r];
      src = q < 0 ? 0 : (q >= rows ? rows - 1 : q);
    }
    int64_t sb = src * nb + j;
    float s = kv_scale(scales, sb, fmt);
    kv_dequant_block(payload + sb * blk * bits / 8, s, blk, fmt, out + r * D + j * blk);
  }
}

// ---------------------------------------------- e4m3 KV rows, vectorised ---
//
// The three e4m3 row formats (WKV_FP8_F32_B64: fp32 scale amax/448 per 64;
// WKV_FP8_UE8M0_B32: PackedRows ue8m0 per 32; WKV_MXFP8_B32: E8M0 per 32) as
// coalesced streaming passes.  A quantize thread owns 16 consecutive values
// (two 16-byte bf16 loads, one 16-byte e4m3 store), a dequantize thread 8 (an
// 8-byte load, one 16-byte store), so a warp moves contiguous bytes.  The
// block / 16 quantize threads of a scale block are adjacent lanes and take the
// block maximum with xor shuffles; the block's first lane writes the scale.  Bytes and scales equal
// kv_quant_block's (the per-block kernel kept for the 4-bit formats):
//   * the e4m3 encode is cvt.rn.satfinite.e4m3x2.f32 on values already
//     clamped to +-448, i.e. round to nearest even as wm_f32_to_e4m3;
//   * for the fp32-scale format the scale amax / 448 and the quotients v / s
//     are correctly rounded divisions done as a product and one fma
//     correction (Markstein), exact division for blocks below 2^-80;  The product differs from the quotient by less than 2 ulps, so
//     away from a midpoint both round to the same e4m3 value;
//   * the power-of-two scales divide exactly as multiplications by 2^-e.
// Dequantize decodes pairs with cvt.rn.f16x2.e4m3x2 (exact), multiplies by the
// scale in float32 and packs bf16 pairs with cvt.rn.bf16x2.f32; a group with
// a NaN code or a non-finite scale takes the scalar path, whose NaN pattern
// (0x7FC0) is the oracle's.

template <int FMT>
struct Fp8Fmt {
  static constexpr int kG = FMT == WKV_FP8_F32_B64 ? 8 : 4;   // threads per scale block
};

__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  uint16_t d;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(d) : "f"(hi), "f"(lo));
  return d;
}

__device__ __forceinline__ float clamp448(float q) { return fminf(fmaxf(q, -448.0f), 448.0f); }

// NV (8 or 16) consecutive values of one thread; i indexes NV-value chunks.
template <int FMT, int NV>
__device__ __forceinline__ void kv_fp8_quant(const uint4 (&u)[NV / 8], int64_t i, unsigned gmask, int lane,
                                             uint8_t *__restrict__ payload, void *__restrict__ scales) {
  constexpr int G = Fp8Fmt<FMT>::kG * 8 / NV;   // threads per scale block
  float v[NV];
#pragma unroll
  for (int k = 0; k < NV / 8; ++k) {
    v[8 * k + 0] = wm_bf16lo(u[k].x); v[8 * k + 1] = wm_bf16hi(u[k].x);
    v[8 * k + 2] = wm_bf16lo(u[k].y); v[8 * k + 3] = wm_bf16hi(u[k].y);
    v[8 * k + 4] = wm_bf16lo(u[k].z); v[8 * k + 5] = wm_bf16hi(u[k].z);
    v[8 * k + 6] = wm_bf16lo(u[k].w); v[8 * k + 7] = wm_bf16hi(u[k].w);
  }
  float amax = 0.0f;
#pragma unroll
  for (int j = 0; j < NV; ++j) amax = fmaxf(amax, fabsf(v[j]));
#pragma unroll
  for (int m = 1; m < G; m <<= 1) amax = fmaxf(amax, __shfl_xor_sync(gmask, amax, m));
  const bool first = (lane & (G - 1)) == 0;
  float q[NV];
  if (FMT == WKV_FP8_F32_B64) {
    // Quotients by Markstein's correction: with y = RN(1/b) and q0 = RN(a * y)
    // within an ulp of a / b, the remainder a - q0 * b is exact in one fma and
    // RN(q0 + rem * y) is the correctly rounded a / b, as long as the remainder
    // does not underflow -- true for blocks whose maximum is at least 2^-80
    // (quotients below 2^-10, the only ones whose remainders could, encode to
    // a signed zero either way).  Smaller blocks divide exactly.  The sign is
    // the value's (for +-0); .satfinite saturates as the clamp to +-448 did.
    if (amax >= 0x1p-80f) {
      const float s0 = amax * kFp8MaxInv;
      const float s = fmaf(fmaf(-s0, 448.0f, amax), kFp8MaxInv, s0);     // RN(amax / 448)
      if (first) static_cast<float *>(scales)[i / G] = s;
      const float r = __frcp_rn(s);
      // value pairs on packed f32x2 arithmetic: each lane rounds as the scalar mul / fma do
      const float2 r2 = make_float2(r, r), ns2 = make_float2(-s, -s);
#pragma unroll
      for (int j = 0; j < NV; j += 2) {
        const float2 vv = make_float2(v[j], v[j + 1]);
        const float2 q0 = wm_mul2(vv, r2);
        const float2 qq = wm_fma2(wm_fma2(q0, ns2, vv), r2, q0);
        q[j] = __uint_as_float((__float_as_uint(qq.x) & 0x7fffffffu) | (__float_as_uint(v[j]) & 0x80000000u));
        q[j + 1] = __uint_as_float((__float_as_uint(qq.y) & 0x7fffffffu) | (__float_as_uint(v[j + 1]) & 0x80000000u));
      }
    } else {
      const float s = __fdiv_rn(amax, 448.0f);
      if (first) static_cast<float *>(scales)[i / G] = s;
#pragma unroll
      for (int j = 0; j < NV; ++j) q[j] = s > 0.0f ? clamp448(__fdiv_rn(v[j], s)) : 0.0f;
    }
  } else if (FMT == WKV_FP8_UE8M0_B32) {
    const int e = ceil_log2_bits(fmaxf(amax, kFp8Floor) * kFp8MaxInv);
    if (first) static_cast<uint8_t *>(scales)[i / G] = static_cast<uint8_t>(e + 127);
    const float f = pow2i(-e);
#pragma unroll
    for (int j = 0; j < NV; ++j) q[j] = clamp448(v[j] * f);
  } else {
    const bool zero = amax == 0.0f;
    const int e = zero ? 0 : max(-127, min(127, floor_log2(amax) - 8));
    if (first) static_cast<uint8_t *>(scales)[i / G] = zero ? 0 : static_cast<uint8_t>(e + 127);
    const float f = pow2i(-e);
#pragma unroll
    for (int j = 0; j < NV; ++j) q[j] = zero ? 0.0f : clamp448(v[j] * f);
  }
  uint32_t w[NV / 4];
#pragma unroll
  for (int k = 0; k < NV / 4; ++k) w[k] = e4m3x2(q[4 * k], q[4 * k + 1]) | (e4m3x2(q[4 * k + 2], q[4 * k + 3]) << 16);
  if constexpr (NV == 16) __stcs(reinterpret_cast<uint4 *>(payload) + i, make_uint4(w[0], w[1], w[2], w[3]));
  else __stcs(reinterpret_cast<uint2 *>(payload) + i, make_uint2(w[0], w[1]));
}

// 16 consecutive values per thread (two 16-byte loads issued together, one
// 16-byte store): the block maximum's shuffles, the scale and its reciprocal
// are paid once per 16 values.
template <int FMT>
__global__ void __launch_bounds__(256) k_kv_fp8_quantize(const uint4 *__restrict__ x, int64_t n16,
                                                         uint8_t *__restrict__ payload, void *__restrict__ scales) {
  constexpr int G = Fp8Fmt<FMT>::kG / 2;
  const int lane = threadIdx.x & 31;
  const unsigned gmask = ((1u << G) - 1u) << (lane & ~(G - 1));
  // n16 is a multiple of G, G divides 32 and the stride is a multiple of 32, so
  // the lanes of a block take each branch together (the shuffles only involve them)
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x) {
    uint4 u[2];
    u[0] = __ldcs(x + 2 * i);
    u[1] = __ldcs(x + 2 * i + 1);
    kv_fp8_quant<FMT, 16>(u, i, gmask, lane, payload, scales);
  }
}

__device__ __forceinline__ float2 e4m3x2_to_f32x2(uint32_t pair) {
  uint32_t h2;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(static_cast<uint16_t>(pair)));
  return __half22float2(*reinterpret_cast<__half2 *>(&h2));
}

template <int FMT, bool GATHER>
__global__ void __launch_bounds__(256) k_kv_fp8_dequantize(const uint2 *__restrict__ payload,
                                                           const void *__restrict__ scales, int64_t rows,
                                                           const int32_t *__restrict__ row_idx, int64_t n8,
                                                           int per_row8, uint4 *__restrict__ out) {
  constexpr int G = Fp8Fmt<FMT>::kG;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t src = i;
    if (GATHER) {
      const int64_t r = i / per_row8;
      const int64_t q = row_idx[r];
      src = (q < 0 ? 0 : (q >= rows ? rows - 1 : q)) * per_row8 + (i - r * per_row8);
    }
    const uint2 p = __ldcs(payload + src);
    const float s = kv_scale(scales, src / G, FMT);
    const uint32_t w[2] = {p.x, p.y};
    const bool nan_code = (__vcmpeq4(w[0] & 0x7f7f7f7fu, 0x7f7f7f7fu) | __vcmpeq4(w[1] & 0x7f7f7f7fu, 0x7f7f7f7fu)) != 0;
    uint32_t o[4];
    if (!nan_code && fabsf(s) <= 3.4028234663852886e38f) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = wm_mul2(e4m3x2_to_f32x2(w[j >> 1] >> (16 * (j & 1))), make_float2(s, s));
        o[j] = pack_bf16x2(f.x, f.y);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t c = w[j >> 1] >> (16 * (j & 1));
        o[j] = wm_f32_to_bf16(wm_e4m3_to_f32(c & 255u) * s) |
               (static_cast<uint32_t>(wm_f32_to_bf16(wm_e4m3_to_f32((c >> 8) & 255u) * s)) << 16);
      }
    }
    __stcs(out + i, make_uint4(o[0], o[1], o[2], o[3]));
  }
}

bool is_fp8_fmt(int fmt) { return fmt == WKV_FP8_F32_B64 || fmt == WKV_FP8_UE8M0_B32 || fmt == WKV_MXFP8_B32; }

int grid_for(int64_t work, int threads) {
  int64_t blocks = (work + threads - 1) / threads;
  int64_t cap = static_cast<int64_t>(wm::sm_count()) * 16;
  return static_cast<int>(std::max<int64_t>(1, std::min(blocks, cap)));
}

// rows n of D values from payload rows (row_idx[r] clipped to [0, rows), or r)
int launch_fp8_dequantize(const uint8_t *payload, const void *scales, int64_t rows, const int32_t *row_idx,
                          int64_t n, int D, int fmt, wm_bf16 *out, cudaStream_t stream) {
  const int64_t n8 = n * (D / 8);
  const auto *pv = reinterpret_cast<const uint2 *>(payload);
  auto *ov = reinterpret_cast<uint4 *>(out);
  const int grid = grid_for(n8, 256);
#define WM_FP8_DQ(F)                                                                                            \
  do {                                                                                                          \
    if (row_idx)                                                                                                \
      k_kv_fp8_dequantize<F, true><<<grid, 256, 0, stream>>>(pv, scales, rows, row_idx, n8, D / 8, ov);        \
    else                                                                                                        \
      k_kv_fp8_dequantize<F, false><<<grid, 256, 0, stream>>>(pv, scales, rows, nullptr, n8, D / 8, ov);       \
  } while (0)
  if (fmt == WKV_FP8_F32_B64) WM_FP8_DQ(WKV_FP8_F32_B64);
  else if (fmt == WKV_FP8_UE8M0_B32) WM_FP8_DQ(WKV_FP8_UE8M0_B32);
  else WM_FP8_DQ(WKV_MXFP8_B32);
#undef WM_FP8_DQ
  return wm::check_launch(row_idx ? "wkv_gather_dequantize" : "wkv_dequantize");
}

int kv_check(int64_t rows, int D, int fmt) {
  if (fmt < 0 || fmt > 5) return wm::fail(WM_ERR_INVALID, "unknown KV format");
  int blk = fmt == WKV_FP8_F32_B64 ? 64 : (fmt == WKV_FP4_E4M3_B16 ? 16 : 32);
  if (rows < 0 || D <= 0 || D % blk) return wm::fail(WM_ERR_INVALID, "Invalid packed cache format or width");
  return WM_OK;
}

}  // namespace

extern "C" {

int wmxfp4_quantize(const wm_bf16 *src, int64_t rows, int64_t cols, uint8_t *packed, uint8_t *scales,
                    wm_stream_t stream) {
  wm::clear_error();
  WM_REQUIRE(rows > 0 && cols > 0 && cols % 32 == 0, "MXFP4 source must contain complete BF16 rows");
  WM_REQUIRE(wm::aligned(src, 16) && wm::aligned(packed, 16), "MXFP4 buffers must be 16-byte aligned");
  int64_t groups = rows * (cols / 32);
  k_mxfp4_quantize<<<grid_for(groups, 256), 256, 0, stream>>>(src, groups, packed, scales);
  return wm::check_launch("wmxfp4_quantize");
}

int wmxfp4_dequantize(const uint8_t *packed, const uint8_t *scales, int64_t rows, int64_t cols, int out_dtype,
                      void *out, wm_stream_t stream) {
  wm::clear_error();
  WM_REQUIRE(rows >= 0 && cols > 0 && cols % 32 == 0, "MXFP4 dequantize needs cols % 32 == 0");
  WM_REQUIRE(out_dtype == WM_OUT_F32 || out_dtype == WM_OUT_BF16, "out_dtype must be WM_OUT_F32 or WM_OUT_BF16");
  WM_REQUIRE(wm::aligned(packed, 16) && wm::aligned(out, 16), "MXFP4 buffers must be 16-byte aligned");
  int64_t groups = rows * (cols / 32);
  if (groups == 0) return WM_OK;
  if (out_dtype == WM_OUT_F32)
    k_mxfp4_dequantize<float><<<grid_for(groups, 256), 256, 0, stream>>>(packed, scales, groups, static_cast<float *>(out));
  else
    k_mxfp4_dequantize<uint16_t><<<grid_for(groups, 256), 256, 0, stream>>>(packed, scales, groups, static_cast<uint16_t *>(out));
  return wm::check_launch("wmxfp4_dequantize");
}

int waffine4_quantize(const wm_bf16 *src, int64_t rows, int64_t cols, int group, uint32_t *packed, wm_bf16 *scales,
                      wm_bf16 *biases, wm_stream_t stream) {
  wm::clear_error();
  WM_REQUIRE(group == 32 || group == 64 || group == 128, "affine4 group must be 32, 64 or 128");
  WM_REQUIRE(rows > 0 && cols > 0 && cols % group == 0, "affine4 needs cols % group == 0");
  WM_REQUIRE(wm::aligned(src, 16) && wm::aligned(packed, 16), "affine4 buffers must be 16-byte aligned");
  int64_t groups = rows * (cols / group);
  k_affine4_quantize<<<grid_for(groups, 128), 128, 0, stream>>>(src, groups, group, packed, scales, biases);
  return wm::check_launch("waffine4_quantize");
}

int waffine4_dequantize(const uint32_t *packed, const wm_bf16 *scales, const wm_bf16 *biases, int64_t rows,
                        int64_t cols, int group, int out_dtype, void *out, wm_stream_t stream) {
  wm::clear_error();
  WM_REQUIRE(group == 32 || group == 64 || group == 128, "affine4 group must be 32, 64 or 128");
  WM_REQUIRE(rows >= 0 && cols > 0 && cols % group == 0, "affine4 needs cols % group == 0");
  WM_REQUIRE(out_dtype == WM_OUT_F32 || out_dtype == WM_OUT_BF16, "out_dtype must be WM_OUT_F32 or WM_OUT_BF16");
  WM_REQUIRE(wm::aligned(packed, 16) && wm::aligned(out, 16), "affine4 buffers must be 16-byte aligned");
  int64_t chunks = rows * (cols / 32);
  if (chunks == 0) return WM_OK;
  if (out_dtype == WM_OUT_F32)
    k_affine4_dequantize<float><<<grid_for(chunks, 256), 256, 0, stream>>>(packed, scales, biases, chunks, group,
                                                                            static_cast<float *>(out));
  else
    k_affine4_dequantize<uint16_t><<<grid_for(chunks, 256), 256, 0, stream>>>(packed, scales, biases, chunks, group,
                                                                               static_cast<uint16_t *>(out));
  return wm::check_launch("waffine4_dequantize");
}

int wkv_affine_append(const wm_bf16 *keys, const wm_bf16 *values, int64_t n_seq, int64_t L, int D, int bits,
                      uint32_t *k_q, wm_bf16 *k_s, wm_bf16 *k_b, uint32_t *v_q, wm_bf16 *v_s, wm_bf16 *v_b,
                      int64_t capacity, int64_t offset, wm_stream_t stream) {
  wm::clear_error();
  WM_REQUIRE(bits == 4 || bits == 8, "QSA quantized cache requires 4 or 8 bits and a width divisible by 32");
  WM_REQUIRE(D > 0 && D % 32 == 0, "QSA quantized cache requires 4 or 8 bits and a width divisible by 32");
  WM_REQUIRE(n_seq >= 0 && L >= 0 && offset >= 0 && offset + L <= capacity, "QSA cache rows exceed its capacity");
  WM_REQUIRE(keys && k_q && k_s && k_b, "QSA cache append needs keys and their cache");
  WM_REQUIRE(!values || (v_q && v_s && v_b), "QSA cache append: values given without their cache");
  WM_REQUIRE(wm::aligned(keys, 16) && wm::aligned(k_q, 16) && (!values || (wm::aligned(values, 16) && wm::aligned(v_q, 16))),
             "QSA cache buffers must be 16-byte aligned");
  const int cpr = D / 8;
  const int64_t chunks = n_seq * L * cpr;
  WM_REQUIRE(chunks <= (int64_t(1) << 31), "QSA cache append: more than 2^34 values in one call");
  if (chunks == 0) return WM_OK;
  AffineKV a{};
  a.src[0] = keys;
  a.src[1] = values;
  a.q[0] = k_q;
  a.q[1] = v_q;
  a.s[0] = k_s;
  a.s[1] = v_s;
  a.b[0] = k_b;
  a.b[1] = v_b;
  dim3 grid(grid_for(chunks, 256), values ? 2 : 1);
  if (bits == 4)
    k_affine_kv_append<4><<<grid, 256, 0, stream>>>(a, static_cast<uint32_t>(chunks), make_divu32(cpr),
                                                    make_divu32(static_cast<uint32_t>(L)), capacity, offset);
  else
    k_affine_kv_append<8><<<grid, 256, 0, stream>>>(a, static_cast<uint32_t>(chunks), make_divu32(cpr),
                                                    make_divu32(static_cast<uint32_t>(L)), capacity, offset);
  return wm::check_launch("wkv_affine_append");
}

int wkv_affine_fetch(const uint32_t *k_q, const wm_bf16 *k_s, const wm_bf16 *k_b, const uint32_t *v_q,
                     const wm_bf16 *v_s, const wm_bf16 *v_b, int64_t n_seq, int64_t L, int64_t capacity, int D,
                     int bits, wm_bf16 *keys_out, wm_bf16 *values_out, wm_stream_t stream) {
  wm::clear_error();
  WM_REQUIRE(bits == 4 || bits == 8, "QSA quantized cache requires 4 or 8 bits and a width divisible by 32");
  WM_REQUIRE(D > 0 && D % 32 == 0, "QSA quantized cache requires 4 or 8 bits and a width divisible by 32");
  WM_REQUIRE(n_seq >= 0 && L >= 0 && L <= capacity, "QSA cache rows exceed its capacity");
  WM_REQUIRE(k_q && k_s && k_b && keys_out, "QSA cache fetch needs the key cache and an output");
  WM_REQUIRE(!values_out || (v_q && v_s && v_b), "QSA cache fetch: values output without their cache");
  WM_REQUIRE(wm::aligned(k_q, 16) && wm::aligned(keys_out, 16) &&
                 (!values_out || (wm::aligned(v_q, 16) && wm::aligned(values_out, 16))),
             "QSA cache buffers must be 16-byte aligned");
  const int cpr = D * bits / 64;   // threads per row: 8 packed bytes each
  const int64_t chunks = n_seq * L * cpr;
  WM_REQUIRE(chunks <= (int64_t(1) << 31), "QSA cache fetch: more than 2^34 values in one call");
  if (chunks == 0) return WM_OK;
  AffineKV a{};
  a.q[0] = const_cast<uint32_t *>(k_q);
  a.q[1] = const_cast<uint32_t *>(v_q);
  a.s[0] = const_cast<uint16_t *>(k_s);
  a.s[1] = const_cast<uint16_t *>(v_s);
  a.b[0] = const_cast<uint16_t *>(k_b);
  a.b[1] = const_cast<uint16_t *>(v_b);
  a.out[0] = keys_out;
  a.out[1] = values_out;
  dim3 grid(grid_for(chunks, 256), values_out ? 2 : 1);
  if (bits == 4)
    k_affine_kv_fetch<4><<<grid, 256, 0, stream>>>(a, static_cast<uint32_t>(chunks), make_divu32(cpr),
                                                   make_divu32(static_cast<uint32_t>(L)), capacity);
  else
    k_affine_kv_fetch<8><<<grid, 256, 0, stream>>>(a, static_cast<uint32_t>(chunks), make_divu32(cpr),
                                                   make_divu32(static_cast<uint32_t>(L)), capacity);
  return wm::check_launch("wkv_affine_fetch");
}

int wkv_quantize(const wm_bf16 *x, int64_t rows, int D, int fmt, uint8_t *payload, void *scales, wm_stream_t stream) {
  wm::clear_error();
  if (int rc = kv_check(rows, D, fmt)) return rc;
  WM_REQUIRE(wm::aligned(x, 16) && wm::aligned(payload, 16) && wm::aligned(scales, 4),
             "KV buffers must be 16-byte aligned (scales 4-byte)");
  int blk = fmt == WKV_FP8_F32_B64 ? 64 : (fmt == WKV_FP4_E4M3_B16 ? 16 : 32);
  int64_t total = rows * (D / blk);
  if (total == 0) return WM_OK;
  if (is_fp8_fmt(fmt)) {
    const int64_t n16 = rows * (D / 16);
    const auto *xv = reinterpret_cast<const uint4 *>(x);
    const int grid = grid_for(n16, 256);
    if (fmt == WKV_FP8_F32_B64) k_kv_fp8_quantize<WKV_FP8_F32_B64><<<grid, 256, 0, stream>>>(xv, n16, payload, scales);
    else if (fmt == WKV_FP8_UE8M0_B32)
      k_kv_fp8_quantize<WKV_FP8_UE8M0_B32><<<grid, 256, 0, stream>>>(xv, n16, payload, scales);
    else k_kv_fp8_quantize<WKV_MXFP8_B32><<<grid, 256, 0, stream>>>(xv, n16, payload, scales);
    return wm::check_launch("wkv_quantize");
  }
  k_kv_quantize<<<grid_for(total, 128), 128, 0, stream>>>(x, rows, D, fmt, payload, scales);
  return wm::check_launch("wkv_quantize");
}

// e4m3 KV formats by (block, scale format): 64 values with an fp32 scale
// (amax / 448), or 32 values with a ue8m0 byte.
static int fp8_kv_format(int block, int scale_fmt) {
  if (block == 64 && scale_fmt == WKV_SCALE_F32) return WKV_FP8_F32_B64;
  if (block == 32 && scale_fmt == WKV_SCALE_UE8M0) return WKV_FP8_UE8M0_B32;
  return -1;
}

int wkv_fp8_quantize(const wm_bf16 *x, int rows, int D, int block, int scale_fmt, uint8_t *payload, void *scales,
                     wm_stream_t stream) {
  wm::clear_error();
  const int fmt = fp8_kv_format(block, scale_fmt);
  if (fmt < 0) return wm::fail(WM_ERR_UNSUPPORTED, "fp8 KV: block 64 with fp32 scales or block 32 with ue8m0");
  return wkv_quantize(x, rows, D, fmt, payload, scales, stream);
}

int wkv_fp8_dequantize(const uint8_t *payload, const void *scales, int rows, int D, int block, int scale_fmt,
                       wm_bf16 *out, wm_stream_t stream) {
  wm::clear_error();
  const int fmt = fp8_kv_format(block, scale_fmt);
  if (fmt < 0) return wm::fail(WM_ERR_UNSUPPORTED, "fp8 KV: block 64 with fp32 scales or block 32 with ue8m0");
  return wkv_dequantize(payload, scales, rows, D, fmt, out, stream);
}

int wkv_dequantize(const uint8_t *payload, const void *scales, int64_t rows, int D, int fmt, wm_bf16 *out,
                   wm_stream_t stream) {
  wm::clear_error();
  if (int rc = kv_check(rows, D, fmt)) return rc;
  WM_REQUIRE(wm::aligned(payload, 16) && wm::aligned(out, 16) && wm::aligned(scales, 4),
             "KV buffers must be 16-byte aligned (scales 4-byte)");
  int blk = fmt == WKV_FP8_F32_B64 ? 64 : (fmt == WKV_FP4_E4M3_B16 ? 16 : 32);
  int64_t total = rows * (D / blk);
  if (total == 0) return WM_OK;
  if (is_fp8_fmt(fmt)) return launch_fp8_dequantize(payload, scales, rows, nullptr, rows, D, fmt, out, stream);
  k_kv_dequantize<<<grid_for(total, 128), 128, 0, stream>>>(payload, scales, rows, nullptr, rows, D, fmt, out);
  return wm::check_launch("wkv_dequantize");
}

int wkv_gather_dequantize(const uint8_t *payload, const void *scales, int64_t rows, const int32_t *row_idx,
                          int64_t n, int D, int fmt, wm_bf16 *out, wm_stream_t stream) {
  wm::clear_error();
  if (int rc = kv_check(rows, D, fmt)) return rc;
  WM_REQUIRE(rows > 0 && n >= 0 && row_idx != nullptr, "gather needs rows > 0 and an index array");
  WM_REQUIRE(wm::aligned(payload, 16) && wm::aligned(out, 16) && wm::aligned(scales, 4),
             "KV buffers must be 16-byte aligned (scales 4-byte)");
  int blk = fmt == WKV_FP8_F32_B64 ? 64 : (fmt == WKV_FP4_E4M3_B16 ? 16 : 32);
  int64_t total = n * (D / blk);
  if (total == 0) return WM_OK;
  if (is_fp8_fmt(fmt)) return launch_fp8_dequantize(payload, scales, rows, row_idx, n, D, fmt, out, stream);
  k_kv_dequantize<<<grid_for(total, 128), 128, 0, stream>>>(payload, scales, rows, row_idx, n, D, fmt, out);
  return wm::check_launch("wkv_gather_dequantize");
}

}  // extern "C"
