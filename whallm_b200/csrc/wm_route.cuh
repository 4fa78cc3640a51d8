// Stable grouping of a small call's (token, slot) assignments by expert,
// computed inside the first kernel of the expert call instead of a separate
// permute launch.
//
// Reference: mlx-lm _gather_sort (called at model.py:404, qwen4_exp.py:622),
// the stable argsort of the flat expert ids; the result is the one k_permute
// produces: slot order = (expert id, flat assignment index) ascending, the
// active experts in ascending id order, the tensor-core work list with the
// shared expert's tiles first.
//
// For S = T * kk <= kSmallRouteMax every CTA of the kernel builds the grouping
// in shared memory (each thread ranks its assignments against all S keys), so
// no CTA waits for another; CTA 0 also writes it to the workspace for the
// launches that follow (offsets, perm, inv, active, counters, tiles).
#pragma once

#include "wm_common.cuh"

namespace wm {

// Every CTA of the first kernel repeats the ranking (S^2 / threads comparisons
// before its first row): measured, that beats a permute launch at 9-63 slots
// (DeepSeek-class B = 1: expert call 63.3 -> 60.4 us; B = 4: 106.8 -> 106.4)
// and loses above (256 slots, the tiny layer: 38.6 -> 41.6 us; 352, Qwen-class
// B = 32: 74.5 -> 89.1 us).
constexpr int kSmallRouteMax = 64;
constexpr int kStreamRouteMax = 64;

// Where a kernel that routes in-kernel finds the call's routing and writes the
// grouping (idx == nullptr: the grouping is already in the workspace).
struct RoutePlan {
  const int32_t *idx = nullptr;    // [T, k] expert ids
  int T = 0, k = 0, shared_expert = -1, E = 0;
  int32_t *offsets = nullptr, *perm = nullptr, *inv = nullptr, *active = nullptr, *counters = nullptr;
  int4 *tiles = nullptr;           // tensor-core work list (nullptr: none)
  int tile_n = 0;
  int32_t *done = nullptr;         // a counter later launches of the call use, zeroed here
};

template <int CAP>
struct SmallRoute {
  static constexpr int kCap = CAP;
  int32_t perm[CAP];               // sorted slot -> flat assignment t * kk + j
  int32_t inv[CAP];                // flat assignment -> sorted slot
  int32_t act_e[CAP];              // active experts, ascending
  int32_t act_p0[CAP];             // their first slot
  int32_t act_n[CAP];              // their slot count
  int32_t n_act;
  int32_t bad;                     // an expert id outside [0, E)
};

// Every thread of the calling CTA runs this (blockDim.x >= 64, a multiple of
// 32; three barriers inside); the result is in `r` when it returns.  `key` is
// CAP ints of shared scratch.  idx is [T, k]; slot j >= k of a token is the
// shared expert.  Each thread ranks its assignments against all S keys (the
// stable order of (expert, assignment)), then warp 0 finds and numbers the
// experts' first slots.  S <= CAP.
template <int CAP>
__device__ __forceinline__ void small_route(const int32_t *__restrict__ idx, int T, int k, int shared_expert, int E,
                                            SmallRoute<CAP> &r, int32_t *key) {
  const int kk = k + (shared_expert >= 0 ? 1 : 0);
  const int S = T * kk;
  int bad = 0;
  for (int a = threadIdx.x; a < S; a += blockDim.x) {
    const int t = a / kk, j = a - t * kk;
    const int e = j < k ? idx[t * k + j] : shared_expert;
    if (e < 0 || e >= E) bad = 1;
    key[a] = (e < 0 || e >= E ? 0 : e) * CAP + a;   // unique; orders by (expert, assignment)
  }
  const int bad_any = __syncthreads_or(bad);       // (also the barrier that publishes key[])
  for (int a = threadIdx.x; a < S; a += blockDim.x) {
    const int ka = key[a];
    int rank = 0;
    for (int b = 0; b < S; ++b) rank += key[b] < ka ? 1 : 0;
    r.perm[rank] = a;
    r.inv[a] = rank;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    // run starts in the sorted keys (the first slot of each expert), numbered by a warp scan
    const int lane = threadIdx.x;
    constexpr int kPer = CAP / 32;                     // slots per lane, in order
    bool first[kPer];
    int cnt = 0;
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int sl = lane * kPer + u;
      first[u] = sl < S && (sl == 0 || key[r.perm[sl]] / CAP != key[r.perm[sl - 1]] / CAP);
      cnt += first[u] ? 1 : 0;
    }
    int incl = cnt;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += o;
    }
    const int n_act = __shfl_sync(0xffffffffu, incl, 31);
    int ai = incl - cnt;
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int sl = lane * kPer + u;
      if (first[u]) {
        r.act_e[ai] = key[r.perm[sl]] / CAP;
        r.act_p0[ai] = sl;
        ++ai;
      }
    }
    __syncwarp();
    for (int q = lane; q < n_act; q += 32) r.act_n[q] = (q + 1 < n_act ? r.act_p0[q + 1] : S) - r.act_p0[q];
    if (lane == 0) {
      r.n_act = bad_any ? 0 : n_act;
      r.bad = bad_any;
    }
  }
  __syncthreads();
}

// CTA 0 writes the grouping where k_permute would have: offsets [E + 1]
// (offsets[E] = -1 and no active experts when an id was out of range), perm,
// inv, active, counters[0] = active experts, counters[1] = error flag,
// counters[3] = 0 (the tensor kernels' error word), *done = 0 (a counter the
// call's later launches use), and with tiles the tensor-core work list and
// counters[2].  All threads of the CTA call it after the __syncthreads that
// ends small_route.
template <int CAP>
__device__ __forceinline__ void publish_route(const SmallRoute<CAP> &r, int T, int k, int shared_expert, int E,
                                              int32_t *offsets, int32_t *perm, int32_t *inv, int32_t *active,
                                              int32_t *counters, int4 *tiles, int tile_n, int32_t *done) {
  const int kk = k + (shared_expert >= 0 ? 1 : 0);
  const int S = T * kk;
  for (int e = threadIdx.x; e <= E; e += blockDim.x) {
    int o = 0;
    if (r.bad) {
      o = e == E ? -1 : 0;
    } else {
      o = S;                                     // slots of experts < e: the first active expert >= e starts there
      for (int ai = 0; ai < r.n_act; ++ai)
        if (r.act_e[ai] >= e) { o = r.act_p0[ai]; break; }
    }
    offsets[e] = o;
  }
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    perm[s] = r.perm[s];
    inv[s] = r.inv[s];
  }
  for (int ai = threadIdx.x; ai < r.n_act; ai += blockDim.x) active[ai] = r.act_e[ai];
  if (threadIdx.x == 0) {
    counters[0] = r.n_act;
    counters[1] = r.bad;
    counters[3] = 0;
    if (done) *done = 0;
    if (tiles) {
      // the shared expert (the last id) first: its tiles are the widest
      int nt = 0;
      const int sh = (shared_expert == E - 1 && r.n_act > 0 && r.act_e[r.n_act - 1] == shared_expert) ? r.n_act - 1 : -1;
      if (sh >= 0)
        for (int q = 0; q < r.act_n[sh]; q += tile_n)
          tiles[nt++] = make_int4(shared_expert, r.act_p0[sh] + q, min(tile_n, r.act_n[sh] - q), 0);
      for (int ai = 0; ai < r.n_act; ++ai) {
        if (ai == sh) continue;
        for (int q = 0; q < r.act_n[ai]; q += tile_n)
          tiles[nt++] = make_int4(r.act_e[ai], r.act_p0[ai] + q, min(tile_n, r.act_n[ai] - q), 0);
      }
      counters[2] = nt;
    }
  }
}

}  // namespace wm
