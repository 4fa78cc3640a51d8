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
// in shared memory (warp 0: each lane ranks its assignments against all S
// keys), so no CTA waits for another; CTA 0 also writes it to the workspace
// for the launches that follow (offsets, perm, inv, active, counters, tiles).
#pragma once

#include "wm_common.cuh"

namespace wm {

constexpr int kSmallRouteMax = 64;

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

struct SmallRoute {
  int32_t perm[kSmallRouteMax];    // sorted slot -> flat assignment t * kk + j
  int32_t inv[kSmallRouteMax];     // flat assignment -> sorted slot
  int32_t act_e[kSmallRouteMax];   // active experts, ascending
  int32_t act_p0[kSmallRouteMax];  // their first slot
  int32_t act_n[kSmallRouteMax];   // their slot count
  int32_t n_act;
  int32_t bad;                     // an expert id outside [0, E)
};

// Warp 0 of the calling CTA runs this (all 32 lanes); the result is in `r`
// after the caller's next __syncthreads.  `key` is kSmallRouteMax ints of
// shared scratch.  idx is [T, k]; slot j >= k of a token is the shared expert.
__device__ __forceinline__ void small_route(const int32_t *__restrict__ idx, int T, int k, int shared_expert, int E,
                                            SmallRoute &r, int32_t *key) {
  const int lane = threadIdx.x & 31;
  const int kk = k + (shared_expert >= 0 ? 1 : 0);
  const int S = T * kk;
  int bad = 0;
  for (int a = lane; a < S; a += 32) {
    const int t = a / kk, j = a - t * kk;
    const int e = j < k ? idx[t * k + j] : shared_expert;
    if (e < 0 || e >= E) bad = 1;
    key[a] = (e < 0 || e >= E ? 0 : e) * kSmallRouteMax + a;   // unique; orders by (expert, assignment)
  }
  bad = __any_sync(0xffffffffu, bad);
  __syncwarp();
  for (int a = lane; a < S; a += 32) {
    const int ka = key[a];
    int rank = 0;
    for (int b = 0; b < S; ++b) rank += key[b] < ka ? 1 : 0;
    r.perm[rank] = a;
    r.inv[a] = rank;
  }
  __syncwarp();
  // first slot of each expert: a run start in the sorted keys
  int n_act = 0;
  for (int s0 = 0; s0 < S; s0 += 32) {
    const int s = s0 + lane;
    const int e = s < S ? key[r.perm[s]] / kSmallRouteMax : -1;
    const int e_prev = (s < S && s > 0) ? key[r.perm[s - 1]] / kSmallRouteMax : -2;
    const unsigned first = __ballot_sync(0xffffffffu, s < S && e != e_prev);
    if (s < S && e != e_prev) {
      const int ai = n_act + __popc(first & ((1u << lane) - 1u));
      r.act_e[ai] = e;
      r.act_p0[ai] = s;
    }
    n_act += __popc(first);
  }
  __syncwarp();
  for (int ai = lane; ai < n_act; ai += 32) r.act_n[ai] = (ai + 1 < n_act ? r.act_p0[ai + 1] : S) - r.act_p0[ai];
  if (lane == 0) {
    r.n_act = bad ? 0 : n_act;
    r.bad = bad;
  }
}

// CTA 0 writes the grouping where k_permute would have: offsets [E + 1]
// (offsets[E] = -1 and no active experts when an id was out of range), perm,
// inv, active, counters[0] = active experts, counters[1] = error flag,
// counters[3] = 0 (the tensor kernels' error word), *done = 0 (a counter the
// call's later launches use), and with tiles the tensor-core work list and
// counters[2].  All threads of the CTA call it after the __syncthreads that
// follows small_route.
__device__ __forceinline__ void publish_route(const SmallRoute &r, int T, int k, int shared_expert, int E,
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
