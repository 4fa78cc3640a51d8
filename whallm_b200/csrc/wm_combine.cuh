// Top-k combine of the bf16 expert outputs, shared by the combine kernel and
// by the last CTA of a small call's final expert launch (which then replaces
// the combine launch).
//
// Reference: _route_reduce (model.py:502-504) after switch_mlp returns the
// bf16 rows: out[t, :] = sum_j w[t, j] * y[slot(t, j), :] (+ the shared
// expert's row times its weight), accumulated in f32 in slot order j and
// rounded once to bf16 (or kept in f32: an expert-parallel partial sum).
#pragma once

#include "wm_common.cuh"

namespace wm {

struct CombineArgs {
  const uint16_t *y;        // [S, H] bf16 expert outputs in sorted-slot order
  const int32_t *inv;       // [T * kk] flat assignment -> sorted slot (-1: dropped)
  const float *w;           // [T, k] routing weights
  const float *shared_w;    // [T] shared-expert weights, or null (weight 1)
  const int32_t *err;       // error flag: set -> zeros
  int T, k, kk, H;
  void *out;                // bf16 [T, H], or f32 [T, H] when f32_out
  bool f32_out;
};

// Output groups i = begin, begin + stride, ... of 8 values each (T * H / 8 in all).
// `cg`: read y through L2 only (rows another CTA of the same launch wrote).
template <bool F32_OUT>
__device__ __forceinline__ void combine_groups(const CombineArgs &a, int64_t begin, int64_t stride, bool cg) {
  const int per_row = a.H / 8;
  const int S = a.T * a.kk;
  const bool bad = *a.err != 0;
  const int64_t total = static_cast<int64_t>(a.T) * per_row;
  for (int64_t i = begin; i < total; i += stride) {
    const int t = static_cast<int>(i / per_row), c8 = static_cast<int>(i % per_row) * 8;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    // slots and weights of 8 assignments, then their 8 rows in flight together, then the fmaf
    // chain in slot order
    for (int j0 = 0; j0 < a.kk && !bad; j0 += 8) {
      int sl[8];
      float wt[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = j0 + u;
        sl[u] = j < a.kk ? a.inv[static_cast<int64_t>(t) * a.kk + j] : -1;
        wt[u] = j < a.k ? a.w[static_cast<int64_t>(t) * a.k + j] : (j < a.kk && a.shared_w ? a.shared_w[t] : 1.0f);
      }
      uint4 r[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const uint4 *src = reinterpret_cast<const uint4 *>(a.y + static_cast<int64_t>(sl[u]) * a.H + c8);
        r[u] = (sl[u] >= 0 && sl[u] < S) ? (cg ? __ldcg(src) : *src) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (sl[u] < 0 || sl[u] >= S) continue;
        const float wv = wt[u];
        acc[0] = fmaf(wv, wm_bf16lo(r[u].x), acc[0]); acc[1] = fmaf(wv, wm_bf16hi(r[u].x), acc[1]);
        acc[2] = fmaf(wv, wm_bf16lo(r[u].y), acc[2]); acc[3] = fmaf(wv, wm_bf16hi(r[u].y), acc[3]);
        acc[4] = fmaf(wv, wm_bf16lo(r[u].z), acc[4]); acc[5] = fmaf(wv, wm_bf16hi(r[u].z), acc[5]);
        acc[6] = fmaf(wv, wm_bf16lo(r[u].w), acc[6]); acc[7] = fmaf(wv, wm_bf16hi(r[u].w), acc[7]);
      }
    }
    if constexpr (F32_OUT) {
      float4 *op = reinterpret_cast<float4 *>(static_cast<float *>(a.out) + static_cast<int64_t>(t) * a.H + c8);
      op[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      op[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    } else {
      uint4 o;
      o.x = wm_f32_to_bf16(acc[0]) | (static_cast<uint32_t>(wm_f32_to_bf16(acc[1])) << 16);
      o.y = wm_f32_to_bf16(acc[2]) | (static_cast<uint32_t>(wm_f32_to_bf16(acc[3])) << 16);
      o.z = wm_f32_to_bf16(acc[4]) | (static_cast<uint32_t>(wm_f32_to_bf16(acc[5])) << 16);
      o.w = wm_f32_to_bf16(acc[6]) | (static_cast<uint32_t>(wm_f32_to_bf16(acc[7])) << 16);
      *reinterpret_cast<uint4 *>(static_cast<uint16_t *>(a.out) + static_cast<int64_t>(t) * a.H + c8) = o;
    }
  }
}

// Called by every thread of every CTA of a launch as its last step (no early
// returns before it): the last CTA to get here combines the call's rows.
// Each thread's earlier writes are fenced before its CTA takes a ticket from
// `done` (zeroed before the launch), and the last CTA fences again before it
// reads, so it sees every other CTA's rows.  No CTA waits for another.
__device__ __forceinline__ void combine_if_last(const CombineArgs &a, int32_t *done) {
  __shared__ int is_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = atomicAdd(done, 1) == static_cast<int>(gridDim.x) - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  if (a.f32_out) combine_groups<true>(a, threadIdx.x, blockDim.x, true);
  else combine_groups<false>(a, threadIdx.x, blockDim.x, true);
}

}  // namespace wm
