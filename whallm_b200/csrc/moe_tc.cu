// Grouped MXFP4 expert GEMM on the 5th-generation tensor cores (tcgen05).
//
// Reference: the MLX gather_qmm / quantized_matmul expert math
// (model.py:393-481, qwen4_exp.py:588-678): y = x @ dequant(W)^T per routed
// (token, expert) pair, W in MXFP4 (e2m1 + E8M0 per 32 along K).
//
// Orientation ("swap AB"): the MMA's M dimension is 128 weight rows, N is the
// tokens routed to the expert (16..128 per tile), K is the reduction.  Decode
// routes a handful of tokens to each expert, so N stays small while M spans
// the weight matrix; prefill tiles the tokens in N = 128 chunks.
//
//   A (weights)  TMEM, f16.  TMA brings packed e2m1 tiles (128 rows x 64 K =
//                4 KB) into shared memory; a dequant warpgroup converts each
//                row with cvt.rn.f16x2.e2m1x2 and one f16x2 multiply by the
//                block scale 2^(s-127) * 2^12, then tcgen05.st writes the
//                32 columns (64 f16) of its TMEM lane.  A never round-trips
//                through shared memory as f16, which keeps shared-memory
//                traffic near 1 byte per weight element at decode rates.
//   B (tokens)   shared memory, f16, K-major, 128-byte swizzle, loaded by TMA
//                in 16-row boxes from a token matrix already in expert order.
//   D            TMEM, f32, 128 lanes x N columns, double buffered.
//
// Scaling: A holds w * 2^12 (exact in f16 for |w| <= 12, block scales down to
// 2^-25 kept exactly), B holds x * 2^-4, so D = 2^8 * (x . w); the epilogue
// multiplies by 2^-8.
//
// MLX affine 4-bit weights (the tiny configuration; deepseek_v41/engram.py:
// 207-221 shapes) use the same packed layout -- eight 4-bit codes per uint32,
// element 0 in the low bits, i.e. two codes per byte, low nibble first -- so
// the same TMA tiles carry them.  Their dequant is w = scale * q + bias with
// one bf16 (scale, bias) per 64 values of a row: each code becomes the exact
// f16 (1024 + q) - 1024 and one fma.rn.f16x2 applies the group's f16 scale
// and bias (one rounding to f16, relative error <= 2^-11).  A holds w
// unscaled, so D = 2^-4 * (x . w) and the epilogue multiplies by 2^4; a scale
// or bias beyond +-32768 (outside what f16 carries safely) sets the error code.
//
// Warp roles (640 threads, one CTA per SM, persistent over work items):
//   warp 0      TMA producer              warp 1   MMA issuer (one thread)
//   warp 2      TMEM allocator            warp 3   second MMA issuer (decode)
//   warps 4-15  three dequant warpgroups, round-robin over A slots (TMEM lanes 0-127)
//   warps 16-19 epilogue (TMEM lanes 0-127): fused ClampedSwiGLU for the
//               up projection (lanes 2j / 2j+1 hold up_j / gate_j), f32 rows
//               of y for the down projection.
// Every mbarrier wait gives up after 2 s, records an error code and skips the
// remaining work, so a broken invariant cannot hang the GPU.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "wm_common.cuh"
#include "wm_moe.cuh"
#include "wm_tc.cuh"

namespace {

using namespace wm_tc;

constexpr int kM = 128;
constexpr int kSub = 64;                      // K per A slot / MMA group (4 x K16)
constexpr int kACols = 32;                    // TMEM columns per A slot (64 f16)
constexpr int kTmemCols = 512;
constexpr int kDqGroups = 3;                  // dequant warpgroups, round-robin over A slots
constexpr int kEpiWarp0 = 4 + 4 * kDqGroups;  // first epilogue warp
constexpr int kThreads = 32 * (kEpiWarp0 + 4);

// Pipeline shapes.  KC: K per TMA stage; NMAX: tokens per tile (MMA N);
// decode streams long row segments (KC 256 = 128 B of e2m1 per row, 64 KB of
// weights in flight per SM), prefill keeps small stages and wide N.
template <int KC, int NMAX, int STAGES, int ISSUERS>
struct Cfg {
  static constexpr int kKC = KC;
  static constexpr int kNMax = NMAX;
  static constexpr int kStages = STAGES;
  static constexpr int kIssuers = ISSUERS;                         // MMA-issuing threads, one accumulator each
  static constexpr int kSubs = KC / kSub;                          // A slots per stage
  static constexpr int kAStageBytes = kM * KC / 2;
  static constexpr int kBSubBytes = NMAX * kSub * 2;               // one 64-wide K sub-tile of B
  static constexpr int kBStageBytes = kBSubBytes * kSubs;
  static constexpr int kDCol0 = 0;                                 // D[issuer][buffer]: NMAX columns each
  static constexpr int kACol0 = 2 * ISSUERS * NMAX;
  static constexpr int kASlots = (kTmemCols - kACol0) / kACols;
  static constexpr bool kSwizzleA = (KC / 2) == 128;               // 128-byte rows: 128B swizzle
  static constexpr size_t kSmem =
      1024 + static_cast<size_t>(STAGES) * (kAStageBytes + kBStageBytes) + (2 * STAGES + 2 * kASlots + 4) * 8 + 16;
  static_assert(kAStageBytes % 1024 == 0 && kBSubBytes % 1024 == 0, "stage buffers must stay 1024-aligned");
  static_assert(kASlots >= 4, "too few A slots");
  static_assert(ISSUERS == 1 || (ISSUERS == 2 && (KC / 64) % 2 == 0), "two issuers need an even number of A slots per stage");
};
using DecodeCfg = Cfg<256, 64, 4, 2>;
using PrefillCfg = Cfg<64, 128, 6, 1>;

struct TcParams {
  int mode;              // 0: up projection (+SwiGLU -> h), 1: down projection (-> y)
  int K;                 // reduction length
  int rows;              // weight rows per expert
  int I;                 // intermediate size (up: row mapping; down: unused)
  int H;                 // output row stride for y (down)
  int order;             // WM_UP_GATE / WM_GATE_UP
  float limit;           // ClampedSwiGLU limit (0: none)
  int m_tiles;           // 128-row tiles per expert
  const uint8_t *scales; // [E*rows, K/32]
  const int4 *tiles;     // {expert, first slot, tokens, 0}
  const int32_t *n_tiles;
  __half *h_out;         // up: [S, I] f16, h * 2^-4
  uint16_t *y_out;       // down: [S, H] bf16
  int32_t *err;
  const uint16_t *af_sc; // affine: bf16 scales [E*rows, K/64]
  const uint16_t *af_bi; // affine: bf16 biases [E*rows, K/64]
  float d_scale;         // D -> x . w: 2^-8 (MXFP4, A = w * 2^12) or 2^4 (affine, A = w)
};

// 16 packed bytes (32 affine codes, element 0 in the low nibble) -> 16 f16x2
// words scale * q + bias (scale2, bias2: f16x2 with both halves equal)
__device__ __forceinline__ void dequant16_affine(uint4 v, uint32_t scale2, uint32_t bias2, uint32_t *out) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t x = w[i] >> (8 * j);              // codes 2j (bits 0-3) and 2j+1 (bits 4-7) of this word
      uint32_t q = (x & 0xFu) | ((x & 0xF0u) << 12) | 0x64006400u;   // f16x2 (1024 + lo, 1024 + hi)
      asm("sub.rn.f16x2 %0, %0, %1;" : "+r"(q) : "r"(0x64006400u));
      asm("fma.rn.f16x2 %0, %0, %1, %2;" : "+r"(q) : "r"(scale2), "r"(bias2));
      out[4 * i + j] = q;
    }
  }
}

// bf16 bits -> f16x2 (both halves); |v| > 32768 or NaN sets `bad`
__device__ __forceinline__ uint32_t affine_f16x2(uint16_t b, bool &bad) {
  const float f = wm_bf16_to_f32(b);
  if (!(fabsf(f) <= 32768.0f)) bad = true;
  const __half h = __float2half_rn(f);
  const uint32_t u = static_cast<uint32_t>(*reinterpret_cast<const uint16_t *>(&h));
  return u | (u << 16);
}

#define WM_TMEM_ST32(taddr, r)                                                                                        \
  asm volatile(                                                                                                       \
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "   \
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),       \
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), \
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),   \
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),   \
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])                                                                 \
      : "memory")

// Block scale 2^(s-127) * 2^12 as f16x2 (both halves); s > 128 overflows f16 -> error.
__device__ __forceinline__ uint32_t scale_f16x2(uint32_t s, bool &bad) {
  uint32_t h;
  if (s > 128u) {
    bad = true;
    h = 0x7800u;  // 2^15: result is garbage, the error flag reports it
  } else if (s >= 101u) {
    h = (s - 100u) << 10;
  } else if (s >= 91u) {
    h = 1u << (s - 91u);
  } else {
    h = 0u;
  }
  return h | (h << 16);
}

// 16 packed bytes (32 e2m1 values) -> 16 f16x2 words scaled by `sf`
__device__ __forceinline__ void dequant16(uint4 v, uint32_t sf, uint32_t *out) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t r0, r1, r2, r3;
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
        "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
        "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
        "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
        : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
        : "r"(w[i]));
    asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(r0) : "r"(sf));
    asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(r1) : "r"(sf));
    asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(r2) : "r"(sf));
    asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(r3) : "r"(sf));
    out[4 * i + 0] = r0;
    out[4 * i + 1] = r1;
    out[4 * i + 2] = r2;
    out[4 * i + 3] = r3;
  }
}

__device__ __forceinline__ float silu_f32(float g) { return g / (1.0f + expf(-g)); }

template <class C, bool AFFINE>
__global__ void __launch_bounds__(kThreads, 1)
    k_expert_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, TcParams p) {
  constexpr int S = C::kStages;
  constexpr int SUBS = C::kSubs;
  constexpr int SLOTS = C::kASlots;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sB = smem;                                   // S x kBStageBytes
  uint8_t *sA = smem + S * C::kBStageBytes;             // S x kAStageBytes
  uint64_t *bars = reinterpret_cast<uint64_t *>(sA + S * C::kAStageBytes);
  uint64_t *full = bars;                                // [S]
  uint64_t *empty = full + S;                           // [S]
  uint64_t *afull = empty + S;                          // [SLOTS]
  uint64_t *aempty = afull + SLOTS;                     // [SLOTS]
  uint64_t *dfull = aempty + SLOTS;                     // [2]
  uint64_t *dempty = dfull + 2;                         // [2]
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(dempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], C::kIssuers); }
    for (int i = 0; i < SLOTS; ++i) { mbar_init(&afull[i], 128); mbar_init(&aempty[i], 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(&dfull[i], C::kIssuers); mbar_init(&dempty[i], 128); }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  WM_PDL_WAIT();
  WM_PDL_LAUNCH();

  const int n_items = (*p.n_tiles) * p.m_tiles;
  const int kstages = p.K / C::kKC;
  const int ub = p.order == WM_UP_GATE ? 0 : p.I;
  const int gb = p.order == WM_UP_GATE ? p.I : 0;

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    // The whole warp runs the loop; one elected lane issues the TMA copies.
    uint32_t g = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
      const int4 tile = p.tiles[item / p.m_tiles];
      const int m = item % p.m_tiles;
      const int nb = (tile.z + 15) >> 4;
      int r_lo, r_hi;
      if (p.mode == 0) { r_lo = ub + m * 64; r_hi = gb + m * 64; }
      else { r_lo = m * kM; r_hi = m * kM + 64; }
      const int ebase = tile.x * p.rows;
      for (int kc = 0; kc < kstages; ++kc, ++g) {
        const int s = g % S;
        const uint32_t u = g / S;
        if (!(ok = mbar_wait(&empty[s], (u & 1) ^ 1, p.err, 1))) break;
        if (elect_one()) {
          mbar_expect_tx(&full[s], C::kAStageBytes + SUBS * nb * 16 * kSub * 2);
          uint8_t *a = sA + s * C::kAStageBytes;
          tma_load_2d(a, &tmA, kc * (C::kKC / 2), ebase + r_lo, &full[s]);
          tma_load_2d(a + C::kAStageBytes / 2, &tmA, kc * (C::kKC / 2), ebase + r_hi, &full[s]);
          uint8_t *b = sB + s * C::kBStageBytes;
          for (int q = 0; q < SUBS; ++q)
            for (int j = 0; j < nb; ++j)
              tma_load_2d(b + q * C::kBSubBytes + j * 16 * 128, &tmB, kc * C::kKC + q * kSub, tile.y + 16 * j,
                          &full[s]);
        }
        __syncwarp();
      }
    }
    // drain: every issued stage has been consumed (its empty barrier completed)
    for (uint32_t q = 0; q < S && q < g && ok; ++q) {
      const uint32_t gg = g - 1 - q;
      ok = mbar_wait(&empty[gg % S], (gg / S) & 1, p.err, 2);
    }
  } else if (warp == 1 || (C::kIssuers == 2 && warp == 3)) {
    // --------------------------------------------------------------- MMA
    // Issuer i (warp 1 -> 0, warp 3 -> 1) takes the A slots h with
    // h % kIssuers == i and accumulates into its own D; the epilogue adds the
    // accumulators.  Two issuing threads double the MMA issue rate, which is
    // what bounds decode (each M128 x N16 x K16 MMA covers 1 KB of weights).
    const int issuer = warp == 1 ? 0 : 1;
    uint32_t g = 0, h = 0, it = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++it) {
      const int4 tile = p.tiles[item / p.m_tiles];
      const int n_mma = max(16, (tile.z + 15) & ~15);
      const uint32_t idesc = idesc_f16(n_mma);
      const int db = it & 1;
      if (!(ok = mbar_wait(&dempty[db], ((it >> 1) & 1) ^ 1, p.err, 3))) break;
      tc_fence_after();
      const uint32_t d_addr = tmem + C::kDCol0 + (issuer * 2 + db) * C::kNMax;
      bool first = true;
      for (int kc = 0; kc < kstages && ok; ++kc, ++g) {
        const int s = g % S;
        if (!(ok = mbar_wait(&full[s], (g / S) & 1, p.err, 4))) break;
        const uint32_t b_base = smem_u32(sB + s * C::kBStageBytes);
        for (int q = 0; q < SUBS; ++q, ++h) {
          if (static_cast<int>(h % C::kIssuers) != issuer) continue;
          const int slot = h % SLOTS;
          if (!(ok = mbar_wait(&afull[slot], (h / SLOTS) & 1, p.err, 5))) break;
          tc_fence_after();
          const uint64_t b0 = bdesc_sw128(b_base + q * C::kBSubBytes);
          if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < kSub / 16; ++kk) {
              const uint32_t a_addr = tmem + C::kACol0 + slot * kACols + kk * 8;
              tc_mma_ts(d_addr, a_addr, b0 + static_cast<uint64_t>(kk * 2), idesc, (first && kk == 0) ? 0u : 1u);
            }
            tc_commit(&aempty[slot]);
          }
          __syncwarp();
          first = false;
        }
        if (elect_one()) tc_commit(&empty[s]);
        __syncwarp();
      }
      if (ok) {
        if (elect_one()) tc_commit(&dfull[db]);
        __syncwarp();
      }
    }
  } else if (warp >= 4 && warp < kEpiWarp0) {
    // ----------------------------------------------------------- dequant
    // kDqGroups warpgroups take alternate sub-chunks (A slots), so several
    // tcgen05.st -> wait::st chains overlap on every SM sub-partition.  Within
    // a group the loop is software-pipelined: sub-chunk h+kDqGroups is
    // converted while the TMEM store of h completes.
    const int wg = (warp - 4) >> 2;
    const int t = (threadIdx.x - 128) & 127;          // TMEM lane == tile row
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    uint32_t g = 0, h0 = 0;
    bool ok = true, bad = false;
    bool pending = false;                             // a store waiting for wait::st + arrive
    int pend_slot = 0;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
      const int4 tile = p.tiles[item / p.m_tiles];
      const int m = item % p.m_tiles;
      int srow, grow;
      if (p.mode == 0) {
        srow = (t >> 1) + ((t & 1) ? 64 : 0);         // even lanes: up rows, odd lanes: gate rows
        grow = ((t & 1) ? gb : ub) + m * 64 + (t >> 1);
      } else {
        srow = t;
        grow = m * kM + t;
      }
      // This row's E8M0 scales as 8-byte words (256 K values each), prefetched
      // four words ahead through a register shift queue so the global-load
      // latency never sits on the per-stage critical path.
      const uint2 *scw = AFFINE ? nullptr :
          reinterpret_cast<const uint2 *>(p.scales + (static_cast<int64_t>(tile.x) * p.rows + grow) * (p.K / 32));
      const int nwords = AFFINE ? 0 : p.K / 256;
      auto ldw = [&](int w) { return w < nwords ? __ldg(scw + w) : make_uint2(0u, 0u); };
      uint2 q0 = ldw(0), q1 = ldw(1), q2 = ldw(2), q3 = ldw(3);
      // affine: this row's (scale, bias) per 64 values, one pair per A slot
      const int64_t af_row = (static_cast<int64_t>(tile.x) * p.rows + grow) * (p.K / kSub);
      int wcur = 0;
      const uint32_t a_row = (srow >> 6) * (C::kAStageBytes / 2) + (srow & 63) * (C::kKC / 2);
      for (int kc = 0; kc < kstages && ok; ++kc, ++g, h0 += SUBS) {
        const int s = g % S;
        const int wneed = (kc * C::kKC) >> 8;
        while (wcur < wneed) {
          q0 = q1; q1 = q2; q2 = q3; q3 = ldw(wcur + 4);
          ++wcur;
        }
        // does this group own a sub-chunk of this stage?
        const int first = static_cast<int>((wg - static_cast<int>(h0 % kDqGroups) + kDqGroups) % kDqGroups);
        if (first >= SUBS) continue;
        uint32_t sbytes[SUBS * 2];
        uint16_t af_s[SUBS], af_b[SUBS];
        if constexpr (AFFINE) {
#pragma unroll
          for (int q = 0; q < SUBS; ++q) {
            af_s[q] = __ldg(p.af_sc + af_row + kc * SUBS + q);
            af_b[q] = __ldg(p.af_bi + af_row + kc * SUBS + q);
          }
        } else {
          const int boff = ((kc * C::kKC) >> 5) & 7;  // first scale byte of this stage within q0
#pragma unroll
          for (int q = 0; q < SUBS * 2; ++q) {
            const int b = boff + q;
            const uint32_t word = b < 4 ? q0.x : q0.y;
            sbytes[q] = (word >> (8 * (b & 3))) & 0xffu;
          }
        }
        if (!(ok = mbar_wait(&full[s], (g / S) & 1, p.err, 6))) break;
        const uint8_t *arow = sA + s * C::kAStageBytes + a_row;
#pragma unroll
        for (int q = 0; q < SUBS; ++q) {
          const uint32_t h = h0 + q;
          if (static_cast<int>(h % kDqGroups) != wg) continue;
          uint4 v0, v1;
          if (C::kSwizzleA) {
            const int sw = srow & 7;
            v0 = *reinterpret_cast<const uint4 *>(arow + (((2 * q) ^ sw) << 4));
            v1 = *reinterpret_cast<const uint4 *>(arow + (((2 * q + 1) ^ sw) << 4));
          } else {
            v0 = reinterpret_cast<const uint4 *>(arow)[2 * q];
            v1 = reinterpret_cast<const uint4 *>(arow)[2 * q + 1];
          }
          uint32_t nr[32];
          if constexpr (AFFINE) {
            const uint32_t s2 = affine_f16x2(af_s[q], bad), b2 = affine_f16x2(af_b[q], bad);
            dequant16_affine(v0, s2, b2, nr);
            dequant16_affine(v1, s2, b2, nr + 16);
          } else {
            dequant16(v0, scale_f16x2(sbytes[2 * q], bad), nr);
            dequant16(v1, scale_f16x2(sbytes[2 * q + 1], bad), nr + 16);
          }
          if (pending) {
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            mbar_arrive(&afull[pend_slot]);
            pending = false;
          }
          const int slot = h % SLOTS;
          if (!(ok = mbar_wait(&aempty[slot], ((h / SLOTS) & 1) ^ 1, p.err, 7))) break;
          // tcgen05.st reads its source registers at issue; only the TMEM write
          // is asynchronous (completed by the wait::st above, next round)
          WM_TMEM_ST32(tmem + lane_base + C::kACol0 + slot * kACols, nr);
          pending = true;
          pend_slot = slot;
        }
      }
    }
    if (pending && ok) {
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      mbar_arrive(&afull[pend_slot]);
    }
    if (bad) atomicCAS(p.err, 0, 100);
  } else if (warp >= kEpiWarp0) {
    // ---------------------------------------------------------- epilogue
    const int t = threadIdx.x - 32 * kEpiWarp0;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    uint32_t it = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++it) {
      const int4 tile = p.tiles[item / p.m_tiles];
      const int m = item % p.m_tiles;
      const int db = it & 1;
      if (!(ok = mbar_wait(&dfull[db], (it >> 1) & 1, p.err, 8))) break;
      tc_fence_after();
      const int n = tile.z;
      for (int c0 = 0; c0 < n; c0 += 16) {
        uint32_t r[16];
        WM_TMEM_LD16(tmem + lane_base + C::kDCol0 + db * C::kNMax + c0, r);
        if (C::kIssuers == 2) {
          uint32_t r2[16];
          WM_TMEM_LD16(tmem + lane_base + C::kDCol0 + (2 + db) * C::kNMax + c0, r2);
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
          for (int q = 0; q < 16; ++q) r[q] = __float_as_uint(__uint_as_float(r[q]) + __uint_as_float(r2[q]));
        } else {
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        }
        if (p.mode == 0) {
          const int j = m * 64 + (t >> 1);
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const float v = __uint_as_float(r[q]) * p.d_scale;
            const float o = __shfl_xor_sync(0xffffffffu, v, 1);
            if (!(t & 1) && c0 + q < n) {
              float up = v, gate = o;
              if (p.limit > 0.0f) {
                up = fminf(fmaxf(up, -p.limit), p.limit);
                gate = fminf(gate, p.limit);
              }
              p.h_out[static_cast<int64_t>(tile.y + c0 + q) * p.I + j] = __float2half_rn(silu_f32(gate) * up * 0x1p-4f);
            }
          }
        } else {
          const int row = m * kM + t;
#pragma unroll
          for (int q = 0; q < 16; ++q)
            if (c0 + q < n)
              p.y_out[static_cast<int64_t>(tile.y + c0 + q) * p.H + row] = wm_f32_to_bf16(__uint_as_float(r[q]) * p.d_scale);
        }
      }
      tc_fence_before();
      mbar_arrive(&dempty[db]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// x16[p, :] = f16(x[perm[p] / kk, :] * 2^-4): the up projection's B operand in expert order
// With plan.idx set (calls of at most kSmallRouteMax slots) every CTA groups
// the call's assignments itself and CTA 0 writes the grouping for the
// launches that follow: no permute launch.
__global__ void k_gather_f16(const uint16_t *__restrict__ x, const int32_t *__restrict__ perm,
                             const int32_t *__restrict__ count, int S, int kk, int H, __half *__restrict__ x16,
                             const wm::RoutePlan plan) {
  __shared__ wm::SmallRoute<wm::kSmallRouteMax> route;
  __shared__ int32_t route_key[wm::kSmallRouteMax];
  WM_PDL_WAIT();
  WM_PDL_LAUNCH();
  const int per = H / 8;
  int rows;
  if (plan.idx) {
    wm::small_route(plan.idx, plan.T, plan.k, plan.shared_expert, plan.E, route, route_key);
    if (blockIdx.x == 0)
      wm::publish_route(route, plan.T, plan.k, plan.shared_expert, plan.E, plan.offsets, plan.perm, plan.inv,
                        plan.active, plan.counters, plan.tiles, plan.tile_n, plan.done);
    perm = route.perm;
    rows = route.bad ? 0 : S;
  } else {
    rows = min(S, max(0, *count));             // kept assignments (all of them unless an expert range drops some)
  }
  const int64_t total = static_cast<int64_t>(rows) * per;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int pidx = static_cast<int>(i / per), c = static_cast<int>(i % per) * 8;
    const int tok = perm[pidx] / kk;
    const uint4 u = *reinterpret_cast<const uint4 *>(x + static_cast<int64_t>(tok) * H + c);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __half2 hv = __floats2half2_rn(wm_bf16lo(w[j]) * 0x1p-4f, wm_bf16hi(w[j]) * 0x1p-4f);
      o[j] = *reinterpret_cast<uint32_t *>(&hv);
    }
    *reinterpret_cast<uint4 *>(x16 + static_cast<int64_t>(pidx) * H + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ------------------------------------------------------------ host side

template <class C>
int launch_tc_cfg(int mode, const uint8_t *w, const uint8_t *scales, int E, int rows, int K, const __half *bmat,
                  int S_rows, int I, int H, int order, float limit, const int4 *tiles, const int32_t *n_tiles,
                  __half *h_out, uint16_t *y_out, int32_t *err, cudaStream_t stream,
                  const uint16_t *af_sc = nullptr, const uint16_t *af_bi = nullptr) {
  if (K % C::kKC) return wm::fail(WM_ERR_UNSUPPORTED, "expert tc: K must be a multiple of the stage depth");
  CUtensorMap tmA, tmB;
  if (int rc = make_map(&tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, K / 2, static_cast<uint64_t>(E) * rows, K / 2,
                        C::kKC / 2, 64, C::kSwizzleA ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE))
    return rc;
  if (int rc = make_map(&tmB, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, bmat, K, S_rows, static_cast<uint64_t>(K) * 2, kSub, 16,
                        CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  const bool affine = af_sc != nullptr;
  const auto kern = affine ? k_expert_tc<C, true> : k_expert_tc<C, false>;
  static std::mutex mu;
  static bool attr_set[2][64] = {{false}, {false}};
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && !attr_set[affine][dev]) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(C::kSmem));
      if (e != cudaSuccess) return wm::fail(WM_ERR_CUDA, std::string("tc smem attribute: ") + cudaGetErrorString(e));
      attr_set[affine][dev] = true;
    }
  }
  TcParams p{};
  p.mode = mode;
  p.K = K;
  p.rows = rows;
  p.I = I;
  p.H = H;
  p.order = order;
  p.limit = limit;
  p.m_tiles = mode == 0 ? I / 64 : rows / kM;
  p.scales = scales;
  p.tiles = tiles;
  p.n_tiles = n_tiles;
  p.h_out = h_out;
  p.y_out = y_out;
  p.err = err;
  p.af_sc = af_sc;
  p.af_bi = af_bi;
  p.d_scale = affine ? 0x1p4f : 0x1p-8f;
  if (cudaError_t e = wm::launch_pdl(kern, dim3(wm::sm_count()), dim3(kThreads), C::kSmem, stream, tmA, tmB, p))
    return wm::fail(WM_ERR_CUDA, std::string("expert tc: ") + cudaGetErrorString(e));
  return wm::check_launch("expert tc");
}

int launch_tc(bool decode, int mode, const uint8_t *w, const uint8_t *scales, int E, int rows, int K,
              const __half *bmat, int S_rows, int I, int H, int order, float limit, const int4 *tiles,
              const int32_t *n_tiles, __half *h_out, uint16_t *y_out, int32_t *err, cudaStream_t stream,
              const uint16_t *af_sc = nullptr, const uint16_t *af_bi = nullptr) {
  if (decode)
    return launch_tc_cfg<DecodeCfg>(mode, w, scales, E, rows, K, bmat, S_rows, I, H, order, limit, tiles, n_tiles,
                                    h_out, y_out, err, stream, af_sc, af_bi);
  return launch_tc_cfg<PrefillCfg>(mode, w, scales, E, rows, K, bmat, S_rows, I, H, order, limit, tiles, n_tiles,
                                   h_out, y_out, err, stream, af_sc, af_bi);
}

}  // namespace

namespace wm {

bool tc_supported(int H, int I) { return H % 256 == 0 && I % 256 == 0; }

int tc_tile_n(int T) { return T <= DecodeCfg::kNMax ? DecodeCfg::kNMax : PrefillCfg::kNMax; }

int launch_gather_f16(const uint16_t *x, const int32_t *perm, const int32_t *count, int S, int kk, int H, void *x16,
                      cudaStream_t stream, const RoutePlan &plan) {
  const int64_t work = static_cast<int64_t>(S) * (H / 8);
  const int grid = static_cast<int>(std::min<int64_t>((work + 255) / 256, sm_count() * 8));
  if (grid > 0)
    if (cudaError_t e = launch_pdl(k_gather_f16, dim3(grid), dim3(256), 0, stream, x, perm, count, S, kk, H,
                                   static_cast<__half *>(x16), plan))
      return fail(WM_ERR_CUDA, std::string("gather f16: ") + cudaGetErrorString(e));
  return check_launch("gather f16");
}

int launch_tc_up(const uint8_t *w13, const uint8_t *s13, int E, int H, int I, const void *x16, int S_rows, int order,
                 float limit, const int4 *tiles, const int32_t *n_tiles, void *h16, int32_t *err, int tile_n,
                 cudaStream_t stream, const uint16_t *af_sc, const uint16_t *af_bi) {
  return launch_tc(tile_n == DecodeCfg::kNMax, 0, w13, s13, E, 2 * I, H, static_cast<const __half *>(x16), S_rows, I, H, order, limit, tiles,
                   n_tiles, static_cast<__half *>(h16), nullptr, err, stream, af_sc, af_bi);
}

int launch_tc_down(const uint8_t *w2, const uint8_t *s2, int E, int H, int I, const void *h16, int S_rows,
                   const int4 *tiles, const int32_t *n_tiles, uint16_t *y, int32_t *err, int tile_n, cudaStream_t stream,
                   const uint16_t *af_sc, const uint16_t *af_bi) {
  return launch_tc(tile_n == DecodeCfg::kNMax, 1, w2, s2, E, H, I, static_cast<const __half *>(h16), S_rows, I, H, WM_UP_GATE, 0.0f, tiles,
                   n_tiles, nullptr, y, err, stream, af_sc, af_bi);
}

}  // namespace wm
