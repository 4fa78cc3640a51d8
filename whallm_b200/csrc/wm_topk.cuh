// Router top-k of one token row by a whole CTA: scores, selection, weights.
//
// Reference: Gate.__call__ (deepseek_v41/moe.py:58-75) and the routing half
// of SparseMoE.__call__ (qwen4_exp.py:692-699); ties go to the lower expert
// id, as _stable_topk_indices (model.py:548-560) orders them.
//
// Arithmetic (bit-for-bit the warp-per-token kernel's and the CPU
// restatement's): scores per score function (bf16 rounding of the logits and
// of the probabilities for WM_SCORE_SOFTMAX_BF16); the softmax denominator is
// lane l's sum of experts l, l + 32, l + 64, ... in that order, then a
// shuffle butterfly with strides 16, 8, 4, 2, 1; the selection is the k
// largest keys (score plus selection bias; NaN as -inf, -0 as +0), larger
// key first, equal keys by lower expert id; the renormalising sum adds the
// selected scores in selection order.  Compile with -fmad=false.
//
// Selection in two parallel stages instead of k serial rounds over the whole
// row: every warp takes the k best of its own experts (k rounds of two warp
// reductions over at most 32 x PERT keys), then each of the NW * k
// candidates counts the candidates ahead of it; that count is its place in
// the overall order, since everything ahead of an overall winner is itself a
// winner of its warp.
#pragma once

#include "wm_common.cuh"
#include "wm_detmath.cuh"

namespace wm {

constexpr int kTopkMaxE = 1024;
constexpr int kTopkMaxK = 32;

__device__ __forceinline__ float topk_round_bf16(float v) { return wm_bf16_to_f32(wm_f32_to_bf16(v)); }

// Order-preserving unsigned key of a selection value: NaN sorts as -inf, -0
// as +0; every key of a real expert is >= 0x007fffff, so 0 marks "none".
__device__ __forceinline__ uint32_t topk_key(float kv) {
  const float kNegInf = -__int_as_float(0x7f800000);
  kv = (kv != kv) ? kNegInf : kv;
  const uint32_t b = __float_as_uint(kv == 0.0f ? 0.0f : kv);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

template <int NW>
struct TopkScratch {
  float sc[kTopkMaxE];              // scores by expert id
  float red[NW];
  uint2 cand[NW * kTopkMaxK];       // per-warp winners: (key, expert id); (0, 0x7fffffff) = none
  int32_t sel_id[kTopkMaxK];        // overall winners in selection order
  float sel_w[kTopkMaxK];           // their scores (without the selection bias)
};

// All threads of the CTA call this (threads of warps >= NW only meet the
// barriers); E <= 32 * NW * PERT, 1 <= k <= min(kTopkMaxK, E).  On return
// s.sel_id / s.sel_w hold the k winners of row `lt` in selection order and
// *denom the renormalising divisor (1 when norm_eps < 0).
template <int NW, int PERT>
__device__ __forceinline__ void cta_topk_row(const float *__restrict__ lt, const float *__restrict__ select_bias,
                                             int E, int k, int score_fn, float norm_eps, TopkScratch<NW> &s,
                                             float *denom) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool live = warp < NW;
  const float kNegInf = -__int_as_float(0x7f800000);
  const bool bf = score_fn == WM_SCORE_SOFTMAX_BF16;
  float sc[PERT];
#pragma unroll
  for (int i = 0; i < PERT; ++i) {
    const int e = lane + 32 * (warp + NW * i);
    sc[i] = (live && e < E) ? (bf ? topk_round_bf16(lt[e]) : lt[e]) : kNegInf;
  }
  if (score_fn == WM_SCORE_SOFTMAX || bf) {
    float mx = kNegInf;
#pragma unroll
    for (int i = 0; i < PERT; ++i) mx = fmaxf(mx, sc[i]);
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, m));
    if (live && lane == 0) s.red[warp] = mx;
    __syncthreads();
    mx = s.red[0];
#pragma unroll
    for (int w = 1; w < NW; ++w) mx = fmaxf(mx, s.red[w]);
#pragma unroll
    for (int i = 0; i < PERT; ++i) {
      const int e = lane + 32 * (warp + NW * i);
      if (live && e < E) {
        sc[i] = wm_exp(sc[i] - mx);
        s.sc[e] = sc[i];
      }
    }
    __syncthreads();                                  // every warp has read s.red
    if (warp == 0) {
      constexpr int J = NW * PERT;                    // E <= 32 J
      float v[J];
#pragma unroll
      for (int j = 0; j < J; ++j) v[j] = s.sc[min(lane + 32 * j, E - 1)];   // all loads first
      float part = 0.0f;
#pragma unroll
      for (int j = 0; j < J; ++j)
        if (lane + 32 * j < E) part = part + v[j];    // experts lane, lane + 32, ... in order
#pragma unroll
      for (int m = 16; m >= 1; m >>= 1) part = part + __shfl_xor_sync(0xffffffffu, part, m);
      if (lane == 0) s.red[0] = part;
    }
    __syncthreads();
    const float part = s.red[0];
#pragma unroll
    for (int i = 0; i < PERT; ++i) sc[i] = bf ? topk_round_bf16(__fdiv_rn(sc[i], part)) : __fdiv_rn(sc[i], part);
  } else if (score_fn == WM_SCORE_SIGMOID) {
#pragma unroll
    for (int i = 0; i < PERT; ++i) sc[i] = wm_sigmoid(sc[i]);
  } else if (score_fn == WM_SCORE_SQRTSOFTPLUS) {
#pragma unroll
    for (int i = 0; i < PERT; ++i) sc[i] = __fsqrt_rn(wm_softplus(sc[i]));
  }
  uint32_t kb[PERT];
#pragma unroll
  for (int i = 0; i < PERT; ++i) {
    const int e = lane + 32 * (warp + NW * i);
    kb[i] = 0u;
    if (live && e < E) {
      kb[i] = topk_key(select_bias ? sc[i] + select_bias[e] : sc[i]);
      s.sc[e] = sc[i];                                // scores by id, for the weights
    }
  }
  // stage 1: this warp's k best, in order (a lane's own keys are in id order,
  // so its best untaken key is its lowest-id one among equals; across lanes
  // the lowest (i, lane) pair holding the warp maximum is the lowest id)
  if (live) {
    uint32_t taken = 0u;
    for (int r = 0; r < k; ++r) {
      uint32_t best = 0u;
      int bi = 0;
#pragma unroll
      for (int i = 0; i < PERT; ++i)
        if (!((taken >> i) & 1u) && kb[i] > best) { best = kb[i]; bi = i; }
      const uint32_t wbest = __reduce_max_sync(0xffffffffu, best);
      const uint32_t code = (wbest != 0u && best == wbest) ? static_cast<uint32_t>(bi * 32 + lane) : 0xffffffffu;
      const uint32_t win = __reduce_min_sync(0xffffffffu, code);
      if (win != 0xffffffffu && lane == static_cast<int>(win & 31u)) taken |= 1u << (win >> 5);
      if (lane == 0)
        s.cand[warp * k + r] = win != 0xffffffffu
                                   ? make_uint2(wbest, static_cast<uint32_t>((win & 31u) + 32 * (warp + NW * (win >> 5))))
                                   : make_uint2(0u, 0x7fffffffu);
    }
  }
  __syncthreads();
  // stage 2: a candidate's place = the candidates ahead of it (larger key, or equal key and lower id)
  const int nc = NW * k;
  for (int c = threadIdx.x; c < nc; c += blockDim.x) {
    const uint2 me = s.cand[c];
    if (me.y == 0x7fffffffu) continue;
    int ahead = 0;
#pragma unroll 8
    for (int c2 = 0; c2 < nc; ++c2) {
      const uint2 o = s.cand[c2];
      ahead += (o.x > me.x || (o.x == me.x && o.y < me.y)) ? 1 : 0;
    }
    if (ahead < k) {
      s.sel_id[ahead] = static_cast<int32_t>(me.y);
      s.sel_w[ahead] = s.sc[me.y];
    }
  }
  __syncthreads();
  float d = 1.0f;
  if (norm_eps >= 0.0f) {
    float v[kTopkMaxK];
#pragma unroll
    for (int r = 0; r < kTopkMaxK; ++r) v[r] = r < k ? s.sel_w[r] : 0.0f;
    float sum = 0.0f;
#pragma unroll
    for (int r = 0; r < kTopkMaxK; ++r)
      if (r < k) sum = sum + v[r];
    d = sum + norm_eps;
    if (bf) d = topk_round_bf16(d);
  }
  *denom = d;
}

// Weight r of the row: (score / denom, bf16-rounded for WM_SCORE_SOFTMAX_BF16) * route_scale.
__device__ __forceinline__ float topk_weight(float score, float denom, bool norm, bool bf, float route_scale) {
  float w = norm ? __fdiv_rn(score, denom) : score;
  if (bf) w = topk_round_bf16(w);
  return w * route_scale;
}

// The shared-expert gate from its raw logit.
__device__ __forceinline__ float topk_shared_gate(float raw, bool bf) {
  return bf ? topk_round_bf16(wm_sigmoid(topk_round_bf16(raw))) : wm_sigmoid(raw);
}

}  // namespace wm
