// Router: gate logits, score function, top-k, weight renormalisation.
//
// Reference: Gate.__call__ (deepseek_v41/moe.py:58-75), SparseMoE routing
// (qwen4_exp.py:692-699), tie rule _stable_topk_indices (model.py:548-560).
//
// Exactness contract with the CPU restatement (fixed float32 order):
//   logit[t][e]: lane l of a warp accumulates with fmaf the elements
//   h = 256*i + 8*l + j (i ascending, j = 0..7); the 32 partials are combined
//   by a shuffle butterfly with strides 16, 8, 4, 2, 1.  The softmax
//   denominator uses the same butterfly over lane partials of experts
//   l, l+32, l+64, ...  Compiled with -fmad=false.
//
// Kernel 1 (logits): one warp per (expert row, chunk of up to 8 tokens), two
//   warps per CTA so the rows spread over all SMs; the expert row is read once
//   per chunk with 16-byte loads, four in flight per lane.
// Kernel 2 (top-k): one warp per token; scores live in registers
//   (E <= 1024 -> 32 per lane); k rounds of a warp arg-max with ties to the
//   lower expert id.
#include "wm_common.cuh"
#include "wm_detmath.cuh"

namespace {

constexpr int kTokChunk = 8;
constexpr int kMaxE = 1024;
constexpr int kMaxK = 32;

__global__ void __launch_bounds__(64) k_router_logits(const uint16_t *__restrict__ x, const uint16_t *__restrict__ wg,
                                                       const uint16_t *__restrict__ wg_shared,
                                                       const float *__restrict__ logit_bias, int T, int H, int E,
                                                       float *__restrict__ logits, float *__restrict__ shared_raw) {
  const int lane = threadIdx.x & 31;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int rows = E + (wg_shared ? 1 : 0);
  const int chunks = (T + kTokChunk - 1) / kTokChunk;
  if (warp >= rows * chunks) return;
  const int e = warp % rows;
  const int t0 = (warp / rows) * kTokChunk;
  const int nt = min(kTokChunk, T - t0);
  const uint16_t *w = (e < E) ? wg + static_cast<int64_t>(e) * H : wg_shared;
  float acc[kTokChunk];
#pragma unroll
  for (int t = 0; t < kTokChunk; ++t) acc[t] = 0.0f;
#pragma unroll 4
  for (int base = 8 * lane; base < H; base += 256) {
    uint4 wu = __ldg(reinterpret_cast<const uint4 *>(w + base));
    float wv[8] = {wm_bf16lo(wu.x), wm_bf16hi(wu.x), wm_bf16lo(wu.y), wm_bf16hi(wu.y),
                   wm_bf16lo(wu.z), wm_bf16hi(wu.z), wm_bf16lo(wu.w), wm_bf16hi(wu.w)};
#pragma unroll
    for (int t = 0; t < kTokChunk; ++t) {
      if (t < nt) {
        uint4 xu = __ldg(reinterpret_cast<const uint4 *>(x + static_cast<int64_t>(t0 + t) * H + base));
        float xv[8] = {wm_bf16lo(xu.x), wm_bf16hi(xu.x), wm_bf16lo(xu.y), wm_bf16hi(xu.y),
                       wm_bf16lo(xu.z), wm_bf16hi(xu.z), wm_bf16lo(xu.w), wm_bf16hi(xu.w)};
        float a = acc[t];
#pragma unroll
        for (int j = 0; j < 8; ++j) a = fmaf(xv[j], wv[j], a);
        acc[t] = a;
      }
    }
  }
#pragma unroll
  for (int t = 0; t < kTokChunk; ++t) {
    float v = acc[t];
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) v = v + __shfl_xor_sync(0xffffffffu, v, m);
    acc[t] = v;
  }
  if (lane == 0) {
    for (int t = 0; t < nt; ++t) {
      if (e < E) {
        float v = acc[t];
        if (logit_bias) v = v + logit_bias[e];
        logits[static_cast<int64_t>(t0 + t) * E + e] = v;
      } else {
        shared_raw[t0 + t] = acc[t];
      }
    }
  }
}

__global__ void __launch_bounds__(256) k_router_topk(const float *__restrict__ logits, const float *__restrict__ select_bias,
                                                     int T, int E, int k, int score_fn, float norm_eps,
                                                     float route_scale, int32_t *__restrict__ idx,
                                                     float *__restrict__ weights, float *__restrict__ shared_w) {
  const int lane = threadIdx.x & 31;
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (t >= T) return;
  const float *lt = logits + static_cast<int64_t>(t) * E;
  const int per = (E + 31) / 32;
  float sc[kMaxE / 32];
  float key[kMaxE / 32];
  const float kNegInf = -__int_as_float(0x7f800000);
#pragma unroll
  for (int j = 0; j < kMaxE / 32; ++j) {
    int e = lane + 32 * j;
    sc[j] = (j < per && e < E) ? lt[e] : kNegInf;
  }
  if (score_fn == WM_SCORE_SOFTMAX) {
    float mx = kNegInf;
#pragma unroll
    for (int j = 0; j < kMaxE / 32; ++j)
      if (j < per && lane + 32 * j < E) mx = fmaxf(mx, sc[j]);
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, m));
    float part = 0.0f;
#pragma unroll
    for (int j = 0; j < kMaxE / 32; ++j) {
      if (j < per && lane + 32 * j < E) {
        sc[j] = wm_exp(sc[j] - mx);
        part = part + sc[j];
      }
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) part = part + __shfl_xor_sync(0xffffffffu, part, m);
#pragma unroll
    for (int j = 0; j < kMaxE / 32; ++j)
      if (j < per && lane + 32 * j < E) sc[j] = __fdiv_rn(sc[j], part);
  } else if (score_fn == WM_SCORE_SIGMOID) {
#pragma unroll
    for (int j = 0; j < kMaxE / 32; ++j)
      if (j < per && lane + 32 * j < E) sc[j] = wm_sigmoid(sc[j]);
  } else if (score_fn == WM_SCORE_SQRTSOFTPLUS) {
#pragma unroll
    for (int j = 0; j < kMaxE / 32; ++j)
      if (j < per && lane + 32 * j < E) sc[j] = __fsqrt_rn(wm_softplus(sc[j]));
  }
#pragma unroll
  for (int j = 0; j < kMaxE / 32; ++j) {
    int e = lane + 32 * j;
    float kv = (j < per && e < E) ? (select_bias ? sc[j] + select_bias[e] : sc[j]) : kNegInf;
    key[j] = (kv != kv) ? kNegInf : kv;
  }
  uint32_t taken = 0u;  // bit j: expert lane + 32 j selected
  float wsel[kMaxK];
  int32_t isel[kMaxK];
  for (int r = 0; r < k; ++r) {
    float bk = kNegInf;
    int be = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < kMaxE / 32; ++j) {
      int e = lane + 32 * j;
      if (j < per && e < E && !((taken >> j) & 1u)) {
        if (key[j] > bk || (key[j] == bk && e < be)) { bk = key[j]; be = e; }
      }
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
      float ok = __shfl_xor_sync(0xffffffffu, bk, m);
      int oe = __shfl_xor_sync(0xffffffffu, be, m);
      if (ok > bk || (ok == bk && oe < be)) { bk = ok; be = oe; }
    }
    // the owner marks it taken and broadcasts its score
    float s = 0.0f;
    if ((be & 31) == lane) {
      int j = be >> 5;
#pragma unroll
      for (int jj = 0; jj < kMaxE / 32; ++jj)
        if (jj == j) { s = sc[jj]; taken |= 1u << jj; }
    }
    s = __shfl_sync(0xffffffffu, s, be & 31);
    wsel[r] = s;
    isel[r] = be;
  }
  if (lane == 0) {
    float denom = 1.0f;
    bool norm = norm_eps >= 0.0f;
    if (norm) {
      float sum = 0.0f;
      for (int r = 0; r < k; ++r) sum = sum + wsel[r];
      denom = sum + norm_eps;
    }
    for (int r = 0; r < k; ++r) {
      float w = norm ? __fdiv_rn(wsel[r], denom) : wsel[r];
      idx[static_cast<int64_t>(t) * k + r] = isel[r];
      weights[static_cast<int64_t>(t) * k + r] = w * route_scale;
    }
    if (shared_w) shared_w[t] = wm_sigmoid(shared_w[t]);
  }
}

}  // namespace

extern "C" int wmoe_router_topk(const wm_bf16 *x, const wm_bf16 *wg, const float *logit_bias, const float *select_bias,
                                const wm_bf16 *wg_shared, int T, int H, int E, int k, int score_fn, float norm_eps,
                                float route_scale, float *logits, int32_t *idx, float *weights, float *shared_w,
                                wm_stream_t stream) {
  wm::clear_error();
  WM_REQUIRE(T >= 0 && H > 0 && H % 8 == 0, "router needs H % 8 == 0");
  WM_REQUIRE(E >= 1 && E <= kMaxE, "router supports 1 <= E <= 1024 experts");
  WM_REQUIRE(k >= 1 && k <= kMaxK && k <= E, "router needs 1 <= k <= min(32, E)");
  WM_REQUIRE(score_fn >= WM_SCORE_SOFTMAX && score_fn <= WM_SCORE_NONE, "unknown score function");
  if (T == 0) return WM_OK;
  WM_REQUIRE(x && wg && logits && idx && weights, "router: null buffer");
  WM_REQUIRE(!wg_shared || shared_w, "router: wg_shared needs a shared_w output");
  WM_REQUIRE(wm::aligned(x, 16) && wm::aligned(wg, 16) && (!wg_shared || wm::aligned(wg_shared, 16)),
             "router inputs must be 16-byte aligned");
  const int rows = E + (wg_shared ? 1 : 0);
  const int64_t warps = static_cast<int64_t>(rows) * ((T + kTokChunk - 1) / kTokChunk);
  k_router_logits<<<static_cast<int>((warps * 32 + 63) / 64), 64, 0, stream>>>(x, wg, wg_shared, logit_bias, T, H, E,
                                                                             logits, shared_w);
  const int threads = 256;
  if (int rc = wm::check_launch("wmoe_router_topk(logits)")) return rc;
  k_router_topk<<<(T * 32 + threads - 1) / threads, threads, 0, stream>>>(logits, select_bias, T, E, k, score_fn,
                                                                            norm_eps, route_scale, idx, weights,
                                                                            shared_w);
  return wm::check_launch("wmoe_router_topk(topk)");
}

extern "C" int wmoe_topk_scores(const float *logits, const float *select_bias, int T, int E, int k, int score_fn,
                                float norm_eps, float route_scale, int32_t *idx, float *weights, wm_stream_t stream) {
  wm::clear_error();
  WM_REQUIRE(T >= 0, "topk: T >= 0");
  WM_REQUIRE(E >= 1 && E <= kMaxE, "topk supports 1 <= E <= 1024");
  WM_REQUIRE(k >= 1 && k <= kMaxK && k <= E, "topk needs 1 <= k <= min(32, E)");
  WM_REQUIRE(score_fn >= WM_SCORE_SOFTMAX && score_fn <= WM_SCORE_NONE, "unknown score function");
  if (T == 0) return WM_OK;
  WM_REQUIRE(logits && idx && weights, "topk: null buffer");
  const int threads = 256;
  k_router_topk<<<(T * 32 + threads - 1) / threads, threads, 0, stream>>>(logits, select_bias, T, E, k, score_fn,
                                                                            norm_eps, route_scale, idx, weights,
                                                                            nullptr);
  return wm::check_launch("wmoe_topk_scores");
}
