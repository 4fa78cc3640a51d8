// Internal declarations shared by the MoE kernels (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "wm_common.cuh"

namespace wm {

// permute.cu
int launch_permute(const int32_t *idx, int T, int k, int shared_expert, int E, int32_t *offsets, int32_t *perm,
                   int32_t *inv, int32_t *active, int32_t *n_active, int32_t *error_flag, cudaStream_t stream);

// Workspace carved out of the caller's buffer for one expert-forward call.
// S = T * (k + has_shared) assignments.
struct MoeWorkspace {
  int32_t *offsets;    // [E+1]
  int32_t *perm;       // [S] sorted slot -> flat assignment
  int32_t *inv;        // [S] flat assignment -> sorted slot
  int32_t *active;     // [E] active expert ids, ascending
  int32_t *counters;   // [4]: n_active, error flag, spare
  uint16_t *h;         // [S, I] bf16 SwiGLU output in sorted-slot order
  float *y;            // [S, H] f32 expert outputs in sorted-slot order
  size_t bytes;
};

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

inline MoeWorkspace carve_workspace(void *base, int T, int k, int H, int I, int E, int has_shared) {
  MoeWorkspace w{};
  const size_t S = static_cast<size_t>(T) * (k + (has_shared ? 1 : 0));
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
  };
  size_t o_off = take((E + 1) * sizeof(int32_t));
  size_t o_perm = take(S * sizeof(int32_t));
  size_t o_inv = take(S * sizeof(int32_t));
  size_t o_act = take(E * sizeof(int32_t));
  size_t o_cnt = take(4 * sizeof(int32_t));
  size_t o_h = take(S * I * sizeof(uint16_t));
  size_t o_y = take(S * H * sizeof(float));
  w.bytes = off;
  if (base) {
    char *b = static_cast<char *>(base);
    w.offsets = reinterpret_cast<int32_t *>(b + o_off);
    w.perm = reinterpret_cast<int32_t *>(b + o_perm);
    w.inv = reinterpret_cast<int32_t *>(b + o_inv);
    w.active = reinterpret_cast<int32_t *>(b + o_act);
    w.counters = reinterpret_cast<int32_t *>(b + o_cnt);
    w.h = reinterpret_cast<uint16_t *>(b + o_h);
    w.y = reinterpret_cast<float *>(b + o_y);
  }
  return w;
}

}  // namespace wm
