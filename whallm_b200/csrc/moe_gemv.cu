// Grouped expert GEMV for decode-shaped work (few tokens per expert).
//
// Reference: _StreamingSwitchGLU decode / _forward_with_resident / _gather_qmm
// (model.py:283-459), _mxfp4 / _mxfp4_swiglu (model.py:462-481), Qwen
// StreamingExperts (qwen4_exp.py:600-678), ClampedSwiGLU
// (deepseek_v41/moe.py:30-43), _route_reduce (model.py:502-504).
//
// Shape of the work: weights are the bulk of the bytes (23.4 MB per
// DeepSeek-class expert) and each is used by a handful of tokens, so the
// kernel streams every active expert's packed rows from HBM exactly once per
// token chunk and dequantizes them in registers.
//
//   * Work item = (active expert, block of rows).  A persistent grid walks the
//     items; the list of active experts comes from the permute kernel, so
//     idle experts cost nothing.
//   * Each warp owns 4 weight rows and takes 4 tokens per pass.  Lane l covers
//     one 32-value scale group of each row (rows under 1024 values: part of a
//     group), eight values at a time: the eight weights are decoded once for
//     the 4 tokens, and token pairs share packed f32x2 FMAs.
//   * Per-lane partial sums are reduced with a transposed warp butterfly.
//   * Phase "up": rows are (up_j, gate_j, up_j+1, gate_j+1) of w13, so the
//     fused ClampedSwiGLU runs in the epilogue and writes h (bf16) directly.
//   * Phase "down": rows of w2 over h; outputs y (f32) in sorted-slot order.
//   * Combine: per token, sum_j w_j * y_j (+ shared) in float32, fixed order.
#include <cstdlib>

#include "wm_common.cuh"
#include "wm_moe.cuh"
#include "wm_combine.cuh"

namespace {

constexpr int kFmtMxfp4 = 0;
constexpr int kFmtAffine4 = 1;
constexpr int kModeUp = 0;
constexpr int kModeDown = 1;
constexpr int kNT = 4;        // tokens per pass
constexpr int kWarps = 8;     // warps per CTA
constexpr int kRowsPerWarp = 4;

struct Weights {
  const uint8_t *w;      // packed rows, K/2 bytes per row
  const uint8_t *s;      // mxfp4 scales [rows, K/32]
  const uint16_t *sc;    // affine scales [rows, K/group]
  const uint16_t *bi;    // affine biases
  int group;             // affine group size
  int rows;              // rows per expert
  int K;                 // row length in elements
};

__device__ __forceinline__ float silu_f32(float g) { return g / (1.0f + expf(-g)); }

template <int FMT, int MODE>
__global__ void __launch_bounds__(kWarps * 32, 2)
    k_expert_gemv(const uint16_t *__restrict__ in, int kk, const int32_t *__restrict__ offsets,
                  const int32_t *__restrict__ perm, const int32_t *__restrict__ active,
                  const int32_t *__restrict__ counters, Weights W, int I, int order, float limit,
                  uint16_t *__restrict__ h_out, uint16_t *__restrict__ y_out) {
  WM_PDL_WAIT();
  WM_PDL_LAUNCH();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = W.K;
  const int rows_per_item = kWarps * kRowsPerWarp;  // 32
  // up: an item covers 16 intermediate indices (32 rows of w13); down: 32 rows of w2
  const int items_per_expert = (MODE == kModeUp) ? (I / 16) : (W.rows / rows_per_item);
  const int n_items = counters[0] * items_per_expert;
  const int groups = K / 32;
  const int64_t row_bytes = K / 2;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int a = item / items_per_expert, blk = item - a * items_per_expert;
    const int e = active[a];
    const int p0 = offsets[e], n = offsets[e + 1] - p0;
    int row[kRowsPerWarp];
    int j0 = 0;
    if (MODE == kModeUp) {
      j0 = blk * 16 + warp * 2;
      const int ub = order == WM_UP_GATE ? 0 : I, gb = order == WM_UP_GATE ? I : 0;
      row[0] = ub + j0; row[1] = gb + j0; row[2] = ub + j0 + 1; row[3] = gb + j0 + 1;
    } else {
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) row[r] = blk * rows_per_item + warp * kRowsPerWarp + r;
    }
    const int64_t erow0 = static_cast<int64_t>(e) * W.rows;
    for (int c = 0; c < n; c += kNT) {
      const int nt = min(kNT, n - c);
      const uint16_t *src[kNT];
#pragma unroll
      for (int t = 0; t < kNT; ++t) {
        int p = p0 + c + min(t, nt - 1);
        src[t] = (MODE == kModeUp) ? in + static_cast<int64_t>(perm[p] / kk) * K : in + static_cast<int64_t>(p) * K;
      }
      float acc[kRowsPerWarp][kNT];
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
        for (int t = 0; t < kNT; ++t) acc[r][t] = 0.0f;
      // Rows of at most 16 groups (K <= 512) give each group to lpg lanes,
      // each taking 32 / lpg of its values, so fewer lanes idle; the partial
      // sums meet in the warp reduction below.  lpg divides 4, so the lpg
      // segments of nseg 8-value steps cover the 32 values of a group exactly
      // (9 or 10 groups take 2 lanes each, not 32 / groups = 3).
      const int lpg = groups > 16 ? 1 : (groups > 8 ? 2 : 4);
      const int nseg = 4 / lpg;                            // 8-value steps per lane
      for (int qq = lane; qq < groups * lpg; qq += 32) {
        const int q = qq / lpg, seg = qq - q * lpg;
        // Eight values at a time: one 16-byte load of x per token, each row's
        // eight weights decoded once and used by every token of the pass, two
        // tokens per packed instruction (part2[r][tp] = {token 2 tp, 2 tp + 1}).
        // Per (row, token) the products are added in element order.
        constexpr int kNP = kNT / 2;
        static_assert(kNT % 2 == 0, "tokens go in pairs");
        float2 part2[kRowsPerWarp][kNP], sx2[kNP];
#pragma unroll
        for (int tp = 0; tp < kNP; ++tp) {
          sx2[tp] = make_float2(0.0f, 0.0f);
#pragma unroll
          for (int r = 0; r < kRowsPerWarp; ++r) part2[r][tp] = make_float2(0.0f, 0.0f);
        }
#pragma unroll
        for (int s8 = 0; s8 < 4; ++s8) {
          if (s8 >= nseg) break;
          const int i0 = seg * nseg + s8;
          float xv[kNT][8];
#pragma unroll
          for (int t = 0; t < kNT; ++t) {
            // rows past nt repeat the last token (src clamps), their sums are never stored
            const uint4 u = __ldg(reinterpret_cast<const uint4 *>(src[t] + q * 32) + i0);
            xv[t][0] = wm_bf16lo(u.x); xv[t][1] = wm_bf16hi(u.x);
            xv[t][2] = wm_bf16lo(u.y); xv[t][3] = wm_bf16hi(u.y);
            xv[t][4] = wm_bf16lo(u.z); xv[t][5] = wm_bf16hi(u.z);
            xv[t][6] = wm_bf16lo(u.w); xv[t][7] = wm_bf16hi(u.w);
          }
          if (FMT == kFmtAffine4) {
#pragma unroll
            for (int tp = 0; tp < kNP; ++tp)
#pragma unroll
              for (int i = 0; i < 8; ++i) sx2[tp] = wm_add2(sx2[tp], make_float2(xv[2 * tp][i], xv[2 * tp + 1][i]));
          }
#pragma unroll
          for (int r = 0; r < kRowsPerWarp; ++r) {
            // 4 bytes of the row's 16-byte group per step (the first load brings the group into L1)
            const uint32_t wd =
                __ldg(reinterpret_cast<const uint32_t *>(W.w + (erow0 + row[r]) * row_bytes) + q * 4 + i0);
            float wv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const uint32_t nib = (wd >> (4 * i)) & 15u;
              if (FMT == kFmtMxfp4) wv[i] = wm_e2m1_scaled(nib);
              else wv[i] = __uint_as_float(0x4B000000u | nib) - 8388608.0f;
            }
#pragma unroll
            for (int tp = 0; tp < kNP; ++tp)
#pragma unroll
              for (int i = 0; i < 8; ++i)
                part2[r][tp] = wm_fma2(make_float2(xv[2 * tp][i], xv[2 * tp + 1][i]), make_float2(wv[i], wv[i]),
                                    part2[r][tp]);
          }
        }
        float part[kRowsPerWarp][kNT], sx[kNT];
#pragma unroll
        for (int tp = 0; tp < kNP; ++tp) {
          sx[2 * tp] = sx2[tp].x;
          sx[2 * tp + 1] = sx2[tp].y;
#pragma unroll
          for (int r = 0; r < kRowsPerWarp; ++r) {
            part[r][2 * tp] = part2[r][tp].x;
            part[r][2 * tp + 1] = part2[r][tp].y;
          }
        }
        float sc[kRowsPerWarp], bi[kRowsPerWarp];
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; ++r) {
          const int64_t gr = erow0 + row[r];
          if (FMT == kFmtMxfp4) {
            sc[r] = wm_e8m0(W.s[gr * groups + q]);
            bi[r] = 0.0f;
          } else {
            const int ng = K / W.group;
            const int g = (q * 32) / W.group;
            sc[r] = wm_bf16_to_f32(W.sc[gr * ng + g]);
            bi[r] = wm_bf16_to_f32(W.bi[gr * ng + g]);
          }
        }
#pragma unroll
        for (int t = 0; t < kNT; ++t) {
          if (t < nt) {
#pragma unroll
            for (int r = 0; r < kRowsPerWarp; ++r) {
              if (FMT == kFmtMxfp4) acc[r][t] = fmaf(part[r][t] * 0x1p126f, sc[r], acc[r][t]);
              else acc[r][t] = fmaf(part[r][t], sc[r], fmaf(sx[t], bi[r], acc[r][t]));
            }
          }
        }
      }
      // Warp sums of the 16 (row, token) partials by a transposed butterfly:
      // each xor step halves the values a lane carries (16 shuffles instead of
      // 80), and every sum is built from the same pairs in the same order as a
      // full butterfly, so the results are the same bits.  Afterwards lanes l
      // and l ^ 1 hold the sum for row (l >> 3) & 3, token (l >> 1) & 3.
      static_assert(kRowsPerWarp * kNT == 16, "transposed reduction of 16 sums");
      float v[16];
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
        for (int t = 0; t < kNT; ++t) v[r * kNT + t] = acc[r][t];
#pragma unroll
      for (int m = 16, h = 8; m >= 2; m >>= 1, h >>= 1) {
        const bool hi = (lane & m) != 0;
#pragma unroll
        for (int i = 0; i < h; ++i) {
          const float send = hi ? v[i] : v[i + h];
          const float keep = hi ? v[i + h] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
        }
      }
      const float sum = v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
      const int r_l = (lane >> 3) & 3, t_l = (lane >> 1) & 3;
      if (MODE == kModeUp) {
        // rows are (up j0, gate j0, up j0+1, gate j0+1): the gate sum is 8 lanes up
        const float gate_sum = __shfl_xor_sync(0xffffffffu, sum, 8);
        if ((lane & 9) == 0 && t_l < nt) {
          const int jj = r_l >> 1;
          float up = sum, gate = gate_sum;
          if (limit > 0.0f) {
            up = fminf(fmaxf(up, -limit), limit);
            gate = fminf(gate, limit);
          }
          h_out[static_cast<int64_t>(p0 + c + t_l) * I + j0 + jj] = wm_f32_to_bf16(silu_f32(gate) * up);
        }
      } else {
        if ((lane & 1) == 0 && t_l < nt) {
          const int rw = r_l == 0 ? row[0] : r_l == 1 ? row[1] : r_l == 2 ? row[2] : row[3];
          y_out[static_cast<int64_t>(p0 + c + t_l) * W.rows + rw] = wm_f32_to_bf16(sum);
        }
      }
    }
  }
}

// out[t, :] = sum_j w[t,j] * y[inv[t*kk+j], :] (+ shared_w[t] * y[inv[t*kk+k], :]) over the bf16
// expert outputs y, accumulated in f32 in a fixed order and rounded once to bf16 (F32_OUT false)
// or kept in f32 (an expert-parallel partial sum); the arithmetic is wm::combine_groups.
// A set error flag (expert id out of range) yields zeros; slots are bounds-checked and
// dropped assignments (slot -1) contribute nothing.
template <bool F32_OUT>
__global__ void k_combine(const uint16_t *__restrict__ y, const int32_t *__restrict__ inv, const float *__restrict__ w,
                          const float *__restrict__ shared_w, const int32_t *__restrict__ err, int T, int k, int kk,
                          int H, void *__restrict__ out_v) {
  WM_PDL_WAIT();
  WM_PDL_LAUNCH();
  const wm::CombineArgs a{y, inv, w, shared_w, err, T, k, kk, H, out_v, F32_OUT};
  wm::combine_groups<F32_OUT>(a, blockIdx.x * (int64_t)blockDim.x + threadIdx.x, (int64_t)gridDim.x * blockDim.x,
                              false);
}

// out[t, :] = bf16(sum_j w[t, j] * y[slots[t, j], :] (+ add[t, :])): the fmaf
// chain of k_combine over caller-given row indices (slot < 0 or >= R: skipped),
// then the optional float32 addend, rounded once.
__global__ void k_route_reduce(const uint16_t *__restrict__ y, int64_t R, const int32_t *__restrict__ slots,
                               const float *__restrict__ w, int T, int k, int H, const float *__restrict__ add,
                               uint16_t *__restrict__ out) {
  WM_PDL_WAIT();
  WM_PDL_LAUNCH();
  const int per_row = H / 8;
  const int64_t total = static_cast<int64_t>(T) * per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int t = static_cast<int>(i / per_row), c8 = static_cast<int>(i % per_row) * 8;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int j0 = 0; j0 < k; j0 += 8) {
      int64_t sl[8];
      float wt[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = j0 + u;
        sl[u] = j < k ? slots[static_cast<int64_t>(t) * k + j] : -1;
        wt[u] = j < k ? w[static_cast<int64_t>(t) * k + j] : 0.0f;
      }
      uint4 a[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        a[u] = (sl[u] >= 0 && sl[u] < R) ? *reinterpret_cast<const uint4 *>(y + sl[u] * H + c8)
                                         : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (sl[u] < 0 || sl[u] >= R) continue;
        const float wv = wt[u];
        acc[0] = fmaf(wv, wm_bf16lo(a[u].x), acc[0]); acc[1] = fmaf(wv, wm_bf16hi(a[u].x), acc[1]);
        acc[2] = fmaf(wv, wm_bf16lo(a[u].y), acc[2]); acc[3] = fmaf(wv, wm_bf16hi(a[u].y), acc[3]);
        acc[4] = fmaf(wv, wm_bf16lo(a[u].z), acc[4]); acc[5] = fmaf(wv, wm_bf16hi(a[u].z), acc[5]);
        acc[6] = fmaf(wv, wm_bf16lo(a[u].w), acc[6]); acc[7] = fmaf(wv, wm_bf16hi(a[u].w), acc[7]);
      }
    }
    if (add) {
      const float4 *ap = reinterpret_cast<const float4 *>(add + static_cast<int64_t>(t) * H + c8);
      const float4 p0 = ap[0], p1 = ap[1];
      acc[0] = acc[0] + p0.x; acc[1] = acc[1] + p0.y; acc[2] = acc[2] + p0.z; acc[3] = acc[3] + p0.w;
      acc[4] = acc[4] + p1.x; acc[5] = acc[5] + p1.y; acc[6] = acc[6] + p1.z; acc[7] = acc[7] + p1.w;
    }
    uint4 o;
    o.x = wm_f32_to_bf16(acc[0]) | (static_cast<uint32_t>(wm_f32_to_bf16(acc[1])) << 16);
    o.y = wm_f32_to_bf16(acc[2]) | (static_cast<uint32_t>(wm_f32_to_bf16(acc[3])) << 16);
    o.z = wm_f32_to_bf16(acc[4]) | (static_cast<uint32_t>(wm_f32_to_bf16(acc[5])) << 16);
    o.w = wm_f32_to_bf16(acc[6]) | (static_cast<uint32_t>(wm_f32_to_bf16(acc[7])) << 16);
    *reinterpret_cast<uint4 *>(out + static_cast<int64_t>(t) * H + c8) = o;
  }
}

// out[t, j, :] = y[inv[t*k+j], :]  (un-reduced switch_mlp output, bf16)
__global__ void k_unsort(const uint16_t *__restrict__ y, const int32_t *__restrict__ inv,
                         const int32_t *__restrict__ err, int S, int H, uint16_t *__restrict__ out) {
  WM_PDL_WAIT();
  WM_PDL_LAUNCH();
  const int per_row = H / 8;
  const bool bad = *err != 0;
  const int64_t total = static_cast<int64_t>(S) * per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int a = static_cast<int>(i / per_row), c8 = static_cast<int>(i % per_row) * 8;
    const int slot = inv[a];
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (!bad && slot >= 0 && slot < S) v = *reinterpret_cast<const uint4 *>(y + static_cast<int64_t>(slot) * H + c8);
    *reinterpret_cast<uint4 *>(out + static_cast<int64_t>(a) * H + c8) = v;
  }
}

struct Args {
  const uint16_t *x;
  const int32_t *idx;
  const float *weights;
  int T, k, H, I, E;
  Weights w13, w2;
  int order;
  float limit;
  int shared_expert;
  const float *shared_w;
  uint16_t *out;
  bool reduce;
  void *ws;
  size_t ws_bytes;
  cudaStream_t stream;
  wm::RouteFilter rf{};      // expert-parallel share (count 0: the whole layer)
  float *out_f32 = nullptr;  // f32 partial output instead of bf16 `out`
};

int check_common(const Args &a) {
  WM_REQUIRE(a.T >= 0 && a.k >= 1 && a.E >= 1 && a.E <= 4096, "experts: need T >= 0, k >= 1, 1 <= E <= 4096");
  WM_REQUIRE(a.H > 0 && a.H % 32 == 0 && a.I > 0 && a.I % 32 == 0, "experts: H and I must be multiples of 32");
  WM_REQUIRE(a.I % 16 == 0 && a.H % 32 == 0, "experts: I % 16 == 0 and H % 32 == 0 required");
  WM_REQUIRE(a.order == WM_UP_GATE || a.order == WM_GATE_UP, "experts: gate_up_order must be WM_UP_GATE or WM_GATE_UP");
  WM_REQUIRE(a.shared_expert < a.E, "experts: shared_expert must be < E");
  WM_REQUIRE(a.x && a.idx && (a.out || a.out_f32) && a.w13.w && a.w2.w, "experts: null buffer");
  WM_REQUIRE(!a.reduce || a.weights, "moe_forward: null weights");
  WM_REQUIRE(wm::aligned(a.x, 16) && wm::aligned(a.out, 16) && wm::aligned(a.out_f32, 16) &&
                 wm::aligned(a.w13.w, 16) && wm::aligned(a.w2.w, 16),
             "experts: x, out and packed weights must be 16-byte aligned");
  WM_REQUIRE(wm::aligned(a.ws, 256), "experts: workspace must be 256-byte aligned");
  return WM_OK;
}

// WM_EXPERT_PATH selects the MXFP4 expert path for A/B checks: "simt" (the
// general CUDA-core kernel), "f16" (tcgen05 kind::f16 with in-kernel
// dequantization), "mma" (block-scaled tcgen05 at every call size), "stream"
// (the CUDA-core weight stream at every call size whose staged rows fit);
// default: the weight stream for calls of at most kStreamMaxTokens tokens on
// Qwen-class experts (H <= kStreamMaxH, I <= kStreamMaxI), the block-scaled
// tcgen05 path otherwise.
enum class MxPath { kAuto, kMma, kStream, kF16, kSimt };
MxPath mx_path() {
  const char *v = getenv("WM_EXPERT_PATH");
  if (v && v[0] == 's' && v[1] == 'i') return MxPath::kSimt;
  if (v && v[0] == 's' && v[1] == 't') return MxPath::kStream;
  if (v && v[0] == 'f') return MxPath::kF16;
  if (v && v[0] == 'm') return MxPath::kMma;
  return MxPath::kAuto;
}

// The call's path: which kernels run it, whether its first expert kernel
// groups the slots itself (small) and where the rows are combined.
struct Choice {
  bool stream, mx, tc, affine_tc, small, stream_rows, fuse_combine;
  int tile_n;
};

Choice choose(const Args &a, int fmt) {
  Choice c{};
  const int has_shared = a.shared_expert >= 0 ? 1 : 0;
  const int S = a.T * (a.k + has_shared);
  const MxPath path = mx_path();
  const bool small_call = a.T <= wm::kStreamMaxTokens && a.H <= wm::kStreamMaxH && a.I <= wm::kStreamMaxI;
  c.stream = fmt == kFmtMxfp4 && (path == MxPath::kStream || (path == MxPath::kAuto && small_call)) &&
             wm::stream_supported(a.T, a.k, has_shared, a.H, a.I) && wm::aligned(a.w13.s, 8) && wm::aligned(a.w2.s, 8);
  c.mx = !c.stream && fmt == kFmtMxfp4 && (path == MxPath::kAuto || path == MxPath::kMma || path == MxPath::kStream) &&
         wm::mx_supported(a.H, a.I);
  // affine-4 (group 64) runs on the f16 tensor-core kernel, dequantizing in
  // software; WM_EXPERT_PATH=simt keeps it on the CUDA-core kernel
  c.affine_tc = fmt == kFmtAffine4 && path != MxPath::kSimt && a.w13.group == 64 && a.w2.group == 64 &&
                wm::tc_supported(a.H, a.I);
  c.tc = (fmt == kFmtMxfp4 && path == MxPath::kF16 && wm::tc_supported(a.H, a.I)) || c.affine_tc;
  const int n_routed = a.rf.count > 0 ? a.rf.n_global : a.E - has_shared;
  c.tile_n = c.mx ? wm::mx_tile_n(a.T, a.k, n_routed) : wm::tc_tile_n(a.T);
  // small calls: the first expert kernel groups the assignments itself (no permute launch), and when
  // the output is at most 4096 values the last CTA of the down projection combines the rows (no combine
  // launch; for a 7168-wide DeepSeek-class row the serial passes of one CTA cost more than the launch)
  // (WM_FUSE=0 keeps the separate permute and combine launches, for A/B checks)
  const char *fuse_env = getenv("WM_FUSE");
  const bool fuse = !(fuse_env && fuse_env[0] == '0');
  c.small = fuse && a.rf.count == 0 && (c.stream || c.mx || c.tc) &&
            S <= (c.stream ? wm::kStreamRouteMax : wm::kSmallRouteMax);
  // one CTA combines the rows in about one pass over its threads (T * H / 8 output groups); the weight
  // stream's down projection splits the output rows over its CTAs and each combines its own
  c.stream_rows = c.small && c.stream && a.reduce && wm::stream_row_split(S, a.H, a.I);
  c.fuse_combine = c.stream_rows || (c.small && (c.stream || c.mx) && a.reduce && a.T * a.H <= 4096);
  return c;
}

int run(const Args &a, int fmt) {
  if (a.T == 0) return WM_OK;
  if (int rc = check_common(a)) return rc;
  const int has_shared = a.shared_expert >= 0 ? 1 : 0;
  wm::MoeWorkspace ws = wm::carve_workspace(a.ws, a.T, a.k, a.H, a.I, a.E, has_shared);
  if (a.ws_bytes < ws.bytes) return wm::fail(WM_ERR_WORKSPACE, "experts: workspace too small");
  const int kk = a.k + has_shared;
  const int S = a.T * kk;
  const Choice ch = choose(a, fmt);
  const bool stream = ch.stream, mx = ch.mx, tc = ch.tc, affine_tc = ch.affine_tc, small = ch.small;
  const bool stream_rows = ch.stream_rows, fuse_combine = ch.fuse_combine;
  const int tile_n = ch.tile_n;
  wm::RoutePlan plan{};
  const wm::CombineArgs comb{ws.y, ws.inv, a.weights, a.shared_w, ws.counters + 1, a.T, a.k, kk, a.H,
                             a.out_f32 ? static_cast<void *>(a.out_f32) : static_cast<void *>(a.out),
                             a.out_f32 != nullptr};
  int32_t *done = fuse_combine && !stream_rows ? ws.counters + 4 : nullptr;
  if (small) {
    plan.idx = a.idx; plan.T = a.T; plan.k = a.k; plan.shared_expert = a.shared_expert; plan.E = a.E;
    plan.offsets = ws.offsets; plan.perm = ws.perm; plan.inv = ws.inv; plan.active = ws.active;
    plan.counters = ws.counters; plan.tiles = (mx || tc) ? ws.tiles : nullptr; plan.tile_n = tile_n; plan.done = done;
  } else if (int rc = wm::launch_permute(a.idx, a.T, a.k, a.shared_expert, a.E, ws.offsets, ws.perm, ws.inv,
                                         ws.active, ws.counters, ws.counters + 1, (tc || mx) ? ws.tiles : nullptr,
                                         ws.counters + 2, tile_n, a.stream, a.rf, ws.counters + 3)) {
    return rc;
  }
  const int grid = wm::sm_count() * 2;
  if (stream) {
    if (int rc = wm::launch_stream_up(a.w13.w, a.w13.s, a.T, kk, a.H, a.I, a.order, a.limit, a.x, ws.offsets, ws.perm,
                                      ws.active, ws.counters, ws.h, a.stream, plan))
      return rc;
    if (int rc = wm::launch_stream_down(a.w2.w, a.w2.s, S, a.H, a.I, ws.h, ws.offsets, ws.active, ws.counters, ws.y,
                                        a.stream, &comb, done, stream_rows ? &plan : nullptr))
      return rc;
  } else if (mx) {
    const int32_t *count = ws.offsets + a.E;
    if (int rc = wm::launch_split_e4m3(a.x, ws.perm, count, S, kk, a.H, ws.x_hi, ws.x_lo, ws.x_sc, a.stream, nullptr,
                                       plan))
      return rc;
    if (int rc = wm::launch_mx_up(a.w13.w, a.w13.s, a.E, a.H, a.I, ws.x_hi, ws.x_lo, ws.x_sc, ws.s_pad, a.order,
                                  a.limit, ws.tiles, ws.counters + 2, ws.h_hi, ws.h_lo, ws.h_sc, ws.h,
                                  ws.counters + 3, tile_n, a.stream, a.T))
      return rc;
    if (!wm::mx_fused_split(tile_n))
      if (int rc = wm::launch_split_e4m3(ws.h, nullptr, count, S, 1, a.I, ws.h_hi, ws.h_lo, ws.h_sc, a.stream))
        return rc;
    if (int rc = wm::launch_mx_down(a.w2.w, a.w2.s, a.E, a.H, a.I, ws.h_hi, ws.h_lo, ws.h_sc, ws.s_pad, ws.tiles,
                                    ws.counters + 2, ws.y, ws.counters + 3, tile_n, a.stream, &comb, done))
      return rc;
  } else if (tc) {
    if (int rc = wm::launch_gather_f16(a.x, ws.perm, ws.offsets + a.E, S, kk, a.H, ws.x16, a.stream, plan)) return rc;
    if (int rc = wm::launch_tc_up(a.w13.w, a.w13.s, a.E, a.H, a.I, ws.x16, ws.s_pad, a.order, a.limit, ws.tiles,
                                  ws.counters + 2, ws.h, ws.counters + 3, tile_n, a.stream,
                                  affine_tc ? a.w13.sc : nullptr, affine_tc ? a.w13.bi : nullptr))
      return rc;
    if (int rc = wm::launch_tc_down(a.w2.w, a.w2.s, a.E, a.H, a.I, ws.h, ws.s_pad, ws.tiles, ws.counters + 2, ws.y,
                                    ws.counters + 3, tile_n, a.stream, affine_tc ? a.w2.sc : nullptr,
                                    affine_tc ? a.w2.bi : nullptr))
      return rc;
  } else {
    const uint16_t *x = a.x;
    const auto up = fmt == kFmtMxfp4 ? k_expert_gemv<kFmtMxfp4, kModeUp> : k_expert_gemv<kFmtAffine4, kModeUp>;
    const auto down = fmt == kFmtMxfp4 ? k_expert_gemv<kFmtMxfp4, kModeDown> : k_expert_gemv<kFmtAffine4, kModeDown>;
    cudaError_t e = wm::launch_pdl(up, dim3(grid), dim3(kWarps * 32), 0, a.stream, x, kk,
                                   static_cast<const int32_t *>(ws.offsets), static_cast<const int32_t *>(ws.perm),
                                   static_cast<const int32_t *>(ws.active), static_cast<const int32_t *>(ws.counters),
                                   a.w13, a.I, a.order, a.limit, ws.h, static_cast<uint16_t *>(nullptr));
    if (e == cudaSuccess)
      e = wm::launch_pdl(down, dim3(grid), dim3(kWarps * 32), 0, a.stream, static_cast<const uint16_t *>(ws.h), kk,
                         static_cast<const int32_t *>(ws.offsets), static_cast<const int32_t *>(ws.perm),
                         static_cast<const int32_t *>(ws.active), static_cast<const int32_t *>(ws.counters), a.w2,
                         a.I, a.order, a.limit, static_cast<uint16_t *>(nullptr), ws.y);
    if (e != cudaSuccess) return wm::fail(WM_ERR_CUDA, std::string("expert gemv: ") + cudaGetErrorString(e));
  }
  if (int rc = wm::check_launch("expert gemv")) return rc;
  if (fuse_combine) return WM_OK;                     // the down projection's last CTA combined the rows
  const int64_t cwork = static_cast<int64_t>(a.reduce ? a.T : S) * (a.H / 8);
  const int cgrid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((cwork + 255) / 256, wm::sm_count() * 8)));
  cudaError_t e;
  if (a.reduce && a.out_f32)
    e = wm::launch_pdl(k_combine<true>, dim3(cgrid), dim3(256), 0, a.stream, static_cast<const uint16_t *>(ws.y),
                       static_cast<const int32_t *>(ws.inv), a.weights, a.shared_w,
                       static_cast<const int32_t *>(ws.counters + 1), a.T, a.k, kk, a.H, static_cast<void *>(a.out_f32));
  else if (a.reduce)
    e = wm::launch_pdl(k_combine<false>, dim3(cgrid), dim3(256), 0, a.stream, static_cast<const uint16_t *>(ws.y),
                       static_cast<const int32_t *>(ws.inv), a.weights, a.shared_w,
                       static_cast<const int32_t *>(ws.counters + 1), a.T, a.k, kk, a.H, static_cast<void *>(a.out));
  else
    e = wm::launch_pdl(k_unsort, dim3(cgrid), dim3(256), 0, a.stream, static_cast<const uint16_t *>(ws.y),
                       static_cast<const int32_t *>(ws.inv), static_cast<const int32_t *>(ws.counters + 1), S, a.H,
                       a.out);
  if (e != cudaSuccess) return wm::fail(WM_ERR_CUDA, std::string("expert combine: ") + cudaGetErrorString(e));
  return wm::check_launch("expert combine");
}

Weights mx_view(const uint8_t *w, const uint8_t *s, int rows, int K) {
  Weights v{};
  v.w = w; v.s = s; v.rows = rows; v.K = K; v.group = 32;
  return v;
}

Weights af_view(const uint32_t *w, const uint16_t *sc, const uint16_t *bi, int group, int rows, int K) {
  Weights v{};
  v.w = reinterpret_cast<const uint8_t *>(w); v.sc = sc; v.bi = bi; v.group = group; v.rows = rows; v.K = K;
  return v;
}

}  // namespace

extern "C" {

int wmoe_route_reduce(const wm_bf16 *y, int64_t rows, const int32_t *slots, const float *weights, int T, int k,
                      int H, const float *add, wm_bf16 *out, wm_stream_t stream) {
  wm::clear_error();
  WM_REQUIRE(T >= 0 && k >= 1 && H > 0 && H % 8 == 0 && rows >= 0, "route_reduce: need T >= 0, k >= 1, H % 8 == 0");
  if (T == 0) return WM_OK;
  WM_REQUIRE(y && slots && weights && out, "route_reduce: null buffer");
  WM_REQUIRE(wm::aligned(y, 16) && wm::aligned(out, 16) && wm::aligned(add, 16),
             "route_reduce: y, out and add must be 16-byte aligned");
  const int64_t work = static_cast<int64_t>(T) * (H / 8);
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, wm::sm_count() * 8)));
  if (cudaError_t e = wm::launch_pdl(k_route_reduce, dim3(grid), dim3(256), 0, static_cast<cudaStream_t>(stream),
                                     reinterpret_cast<const uint16_t *>(y), rows, slots, weights, T, k, H, add,
                                     reinterpret_cast<uint16_t *>(out)))
    return wm::fail(WM_ERR_CUDA, std::string("route_reduce: ") + cudaGetErrorString(e));
  return wm::check_launch("route_reduce");
}

size_t wmoe_workspace_size(int T, int k, int H, int I, int E, int has_shared) {
  if (T < 0 || k < 1 || H <= 0 || I <= 0 || E < 1) return 0;
  return wm::carve_workspace(nullptr, T, k, H, I, E, has_shared).bytes;
}

int wmoe_mxfp4_experts(const wm_bf16 *x, const int32_t *idx, int T, int k, int H, int I, int E, const uint8_t *w13,
                       const uint8_t *s13, const uint8_t *w2, const uint8_t *s2, int gate_up_order, float swiglu_limit,
                       wm_bf16 *out, void *workspace, size_t ws_bytes, wm_stream_t stream) {
  wm::clear_error();
  Args a{x, idx, nullptr, T, k, H, I, E, mx_view(w13, s13, 2 * I, H), mx_view(w2, s2, H, I), gate_up_order,
         swiglu_limit, -1, nullptr, out, false, workspace, ws_bytes, stream};
  return run(a, kFmtMxfp4);
}

int wmoe_mxfp4_moe_forward(const wm_bf16 *x, const int32_t *idx, const float *weights, int T, int k, int H, int I,
                           int E, const uint8_t *w13, const uint8_t *s13, const uint8_t *w2, const uint8_t *s2,
                           int gate_up_order, float swiglu_limit, int shared_expert, const float *shared_w,
                           wm_bf16 *out, void *workspace, size_t ws_bytes, wm_stream_t stream) {
  wm::clear_error();
  Args a{x, idx, weights, T, k, H, I, E, mx_view(w13, s13, 2 * I, H), mx_view(w2, s2, H, I), gate_up_order,
         swiglu_limit, shared_expert, shared_w, out, true, workspace, ws_bytes, stream};
  return run(a, kFmtMxfp4);
}

int wmoe_mxfp4_moe_layer(const wm_bf16 *x, int T, int H, int I, const wm_bf16 *wg, const float *logit_bias,
                         const float *select_bias, const wm_bf16 *wg_shared, int n_routed, int k, int score_fn,
                         float norm_eps, float route_scale, const uint8_t *w13, const uint8_t *s13, const uint8_t *w2,
                         const uint8_t *s2, int gate_up_order, float swiglu_limit, int shared_expert, float *logits,
                         int32_t *idx, float *weights, float *shared_w, wm_bf16 *out, void *workspace,
                         size_t ws_bytes, wm_stream_t stream) {
  wm::clear_error();
  WM_REQUIRE(T >= 0 && H > 0 && H % 8 == 0, "layer: router needs H % 8 == 0");
  WM_REQUIRE(n_routed >= 1 && n_routed <= 1024, "layer: router supports 1 <= n_routed <= 1024 experts");
  WM_REQUIRE(k >= 1 && k <= 32 && k <= n_routed, "layer: router needs 1 <= k <= min(32, n_routed)");
  WM_REQUIRE(score_fn >= WM_SCORE_SOFTMAX && score_fn <= WM_SCORE_SOFTMAX_BF16, "layer: unknown score function");
  WM_REQUIRE(shared_expert < 0 || shared_expert == n_routed, "layer: the shared expert must be expert n_routed");
  if (T == 0) return WM_OK;
  WM_REQUIRE(x && wg && logits && idx && weights, "layer: null buffer");
  WM_REQUIRE(!wg_shared || shared_w, "layer: wg_shared needs a shared_w output");
  WM_REQUIRE(wm::aligned(x, 16) && wm::aligned(wg, 16) && (!wg_shared || wm::aligned(wg_shared, 16)),
             "layer: router inputs must be 16-byte aligned");
  const int E = n_routed + (shared_expert >= 0 ? 1 : 0);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  Args a{x, idx, weights, T, k, H, I, E, mx_view(w13, s13, 2 * I, H), mx_view(w2, s2, H, I), gate_up_order,
         swiglu_limit, shared_expert, wg_shared ? shared_w : nullptr, out, true, workspace, ws_bytes, st};
  if (int rc = check_common(a)) return rc;
  const wm::MoeWorkspace ws = wm::carve_workspace(workspace, T, k, H, I, E, shared_expert >= 0 ? 1 : 0);
  if (ws_bytes < ws.bytes) return wm::fail(WM_ERR_WORKSPACE, "layer: workspace too small");
  // (the router's top-k run inside every CTA of the first expert kernel instead of its own launch was
  // measured slower: the per-CTA top-k costs more than the launch it saves)
  if (int rc = wm::router_logits(reinterpret_cast<const uint16_t *>(x), reinterpret_cast<const uint16_t *>(wg),
                                 reinterpret_cast<const uint16_t *>(wg_shared), logit_bias, T, H, n_routed, logits,
                                 wg_shared ? shared_w : nullptr, st))
    return rc;
  if (int rc = wm::router_topk(logits, select_bias, T, n_routed, k, score_fn, norm_eps, route_scale, idx, weights,
                               wg_shared ? shared_w : nullptr, st))
    return rc;
  return run(a, kFmtMxfp4);
}

int wmoe_mxfp4_moe_forward_ep(const wm_bf16 *x, const int32_t *idx, const float *weights, int T, int k, int H, int I,
                              int E_local, int n_routed, int route_base, int route_count, const int32_t *placement,
                              const uint8_t *w13,
                              const uint8_t *s13, const uint8_t *w2, const uint8_t *s2, int gate_up_order,
                              float swiglu_limit, int shared_expert, const float *shared_w, int shared_lo,
                              int shared_hi, float *out, void *workspace, size_t ws_bytes, wm_stream_t stream) {
  wm::clear_error();
  WM_REQUIRE(route_count >= 1 && route_base >= 0 && route_base + route_count <= n_routed,
             "moe_forward_ep: need 1 <= route_count and [route_base, route_base + route_count) inside [0, n_routed)");
  WM_REQUIRE(route_count <= E_local && (shared_expert < 0 || shared_expert >= route_count),
             "moe_forward_ep: local experts are [0, route_count) routed, then the shared expert");
  WM_REQUIRE(shared_lo >= 0 && shared_lo <= shared_hi && shared_hi <= T, "moe_forward_ep: need 0 <= shared_lo <= shared_hi <= T");
  WM_REQUIRE(out != nullptr, "moe_forward_ep: null output");
  Args a{x, idx, weights, T, k, H, I, E_local, mx_view(w13, s13, 2 * I, H), mx_view(w2, s2, H, I), gate_up_order,
         swiglu_limit, shared_expert, shared_w, nullptr, true, workspace, ws_bytes, stream};
  a.rf = wm::RouteFilter{route_base, route_count, n_routed, shared_lo, shared_hi, placement};
  a.out_f32 = out;
  return run(a, kFmtMxfp4);
}

int wmoe_affine4_experts(const wm_bf16 *x, const int32_t *idx, int T, int k, int H, int I, int E, const uint32_t *w13,
                         const wm_bf16 *sc13, const wm_bf16 *bi13, const uint32_t *w2, const wm_bf16 *sc2,
                         const wm_bf16 *bi2, int group, int gate_up_order, float swiglu_limit, wm_bf16 *out,
                         void *workspace, size_t ws_bytes, wm_stream_t stream) {
  wm::clear_error();
  WM_REQUIRE(group == 32 || group == 64 || group == 128, "affine4 group must be 32, 64 or 128");
  WM_REQUIRE(H % group == 0 && I % group == 0, "affine4: H and I must be multiples of the group");
  Args a{x, idx, nullptr, T, k, H, I, E, af_view(w13, sc13, bi13, group, 2 * I, H), af_view(w2, sc2, bi2, group, H, I),
         gate_up_order, swiglu_limit, -1, nullptr, out, false, workspace, ws_bytes, stream};
  return run(a, kFmtAffine4);
}

int wmoe_affine4_moe_forward(const wm_bf16 *x, const int32_t *idx, const float *weights, int T, int k, int H, int I,
                             int E, const uint32_t *w13, const wm_bf16 *sc13, const wm_bf16 *bi13, const uint32_t *w2,
                             const wm_bf16 *sc2, const wm_bf16 *bi2, int group, int gate_up_order, float swiglu_limit,
                             int shared_expert, const float *shared_w, wm_bf16 *out, void *workspace, size_t ws_bytes,
                             wm_stream_t stream) {
  wm::clear_error();
  WM_REQUIRE(group == 32 || group == 64 || group == 128, "affine4 group must be 32, 64 or 128");
  WM_REQUIRE(H % group == 0 && I % group == 0, "affine4: H and I must be multiples of the group");
  Args a{x, idx, weights, T, k, H, I, E, af_view(w13, sc13, bi13, group, 2 * I, H),
         af_view(w2, sc2, bi2, group, H, I), gate_up_order, swiglu_limit, shared_expert, shared_w, out, true,
         workspace, ws_bytes, stream};
  return run(a, kFmtAffine4);
}

}  // extern "C"
