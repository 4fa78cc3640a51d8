// Internal declarations shared by the MoE kernels (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "wm_common.cuh"
#include "wm_combine.cuh"
#include "wm_route.cuh"

namespace wm {

// Expert-parallel share of one rank: routed ids in [base, base + count) are
// this rank's local experts 0..count-1, other ids in [0, n_global) are
// dropped, and only tokens in [shared_lo, shared_hi) get a shared-expert
// slot.  count == 0 means no filter (the whole layer on one device).
struct RouteFilter {
  int base = 0, count = 0, n_global = 0, shared_lo = 0, shared_hi = 0;
  // expert placement: routed id e belongs to position remap[e] of the ranks'
  // contiguous ranges (nullptr: position e)
  const int32_t *remap = nullptr;
};

// permute.cu.  With tiles != nullptr it also emits the tensor-core work list:
// {expert, first slot, tokens (<= tile_n), 0} per tile, count in *n_tiles.
int launch_permute(const int32_t *idx, int T, int k, int shared_expert, int E, int32_t *offsets, int32_t *perm,
                   int32_t *inv, int32_t *active, int32_t *n_active, int32_t *error_flag, int4 *tiles,
                   int32_t *n_tiles, int tile_n, cudaStream_t stream, RouteFilter rf = RouteFilter{},
                   int32_t *clear = nullptr);  // clear: a flag the permute sets to 0 (the expert kernels' error code)

// moe_tc.cu
bool tc_supported(int H, int I);
int tc_tile_n(int T);  // tokens per tile: 64 for decode batches (T <= 64), else 128
// rows [0, *count) of the expert-ordered token matrix (count = offsets[E] on the device)
// plan.idx set: the kernel groups the call's assignments itself (no permute launch; perm unused)
int launch_gather_f16(const uint16_t *x, const int32_t *perm, const int32_t *count, int S, int kk, int H, void *x16,
                      cudaStream_t stream, const RoutePlan &plan = RoutePlan{});
// af_sc / af_bi (bf16 [E * rows, K / 64]): MLX affine 4-bit weights (group 64) instead of MXFP4 (s13 / s2 unused)
int launch_tc_up(const uint8_t *w13, const uint8_t *s13, int E, int H, int I, const void *x16, int S_rows, int order,
                 float limit, const int4 *tiles, const int32_t *n_tiles, void *h16, int32_t *err, int tile_n,
                 cudaStream_t stream, const uint16_t *af_sc = nullptr, const uint16_t *af_bi = nullptr);
int launch_tc_down(const uint8_t *w2, const uint8_t *s2, int E, int H, int I, const void *h16, int S_rows,
                   const int4 *tiles, const int32_t *n_tiles, uint16_t *y, int32_t *err, int tile_n, cudaStream_t stream,
                   const uint16_t *af_sc = nullptr, const uint16_t *af_bi = nullptr);

// router.cu: the two router launches of wmoe_router_topk (arguments checked by the caller); the logits
// launch writes the raw shared-gate logit into shared_raw[t], the top-k launch turns shared_w[t] (the same
// buffer, when given) into the gate
int router_logits(const uint16_t *x, const uint16_t *wg, const uint16_t *wg_shared, const float *logit_bias, int T,
                  int H, int E, float *logits, float *shared_raw, cudaStream_t stream);
int router_topk(const float *logits, const float *select_bias, int T, int E, int k, int score_fn, float norm_eps,
                float route_scale, int32_t *idx, float *weights, float *shared_w, cudaStream_t stream);

// moe_stream.cu: CUDA-core MXFP4 weight stream for calls of one or two tokens
constexpr size_t kStreamSmemMax = 216 * 1024;   // shared memory: staged f16 operand rows + copy rings (+ ~7 KB static)
constexpr int kStreamMaxTokens = 2;               // calls of at most this many tokens take the stream path
constexpr int kStreamMaxH = 4096, kStreamMaxI = 1024;   // ... when the experts are this small (Qwen-class)
// H and I multiples of 256, and the staged rows (T tokens of H, S slots of I) fit in shared memory
bool stream_supported(int T, int k, int has_shared, int H, int I);
// the down projection can split the output rows over its CTAs and combine in each (a small call of S slots)
bool stream_row_split(int S, int H, int I);
// plan.idx set: the kernel groups the call's assignments itself (no permute launch)
int launch_stream_up(const uint8_t *w13, const uint8_t *s13, int T, int kk, int H, int I, int order, float limit,
                     const uint16_t *x, const int32_t *offsets, const int32_t *perm, const int32_t *active,
                     const int32_t *counters, uint16_t *h, cudaStream_t stream, const RoutePlan &plan = RoutePlan{});
// comb + done: the launch's last CTA also combines the rows (done zeroed by the call's first kernel);
// comb + plan (plan->idx set): each CTA takes a range of output rows of every active expert, grouping the
// call itself before its dependency wait, and combines its own rows (y is not written)
int launch_stream_down(const uint8_t *w2, const uint8_t *s2, int S, int H, int I, const uint16_t *h,
                       const int32_t *offsets, const int32_t *active, const int32_t *counters, uint16_t *y,
                       cudaStream_t stream, const CombineArgs *comb = nullptr, int32_t *done = nullptr,
                       const RoutePlan *plan = nullptr);

// linear_stream.cu: dense block-scaled linear of one or two rows on CUDA cores (fmt 8: e4m3 weights, 4: e2m1)
constexpr int kLinearStreamMaxT = 2;
bool linear_stream_supported(int T, int K, int N, int fmt);
int launch_linear_stream(const uint16_t *x, int T, int K, const uint8_t *w, const uint8_t *sc, int N, int fmt,
                         uint16_t *y, cudaStream_t stream);

// moe_mx.cu: block-scaled tensor-core path (MXFP4 weights x two e4m3 token terms)
bool mx_supported(int H, int I);
// tokens per tile: 32 (decode configuration) while T * k / n_routed <= 32, else 112
int mx_tile_n(int T, int k, int n_routed);
// rows [0, min(S, *count)) (all S when count is null); GATHER when perm != null: row p = src[perm[p] / kk];
// *zero (if given) is set to 0 once the kernel's dependency wait has returned
// plan.idx set (GATHER only): the kernel groups the call's assignments itself (no permute launch; perm unused)
int launch_split_e4m3(const uint16_t *src, const int32_t *perm, const int32_t *count, int S, int kk, int K,
                      uint8_t *hi, uint8_t *lo, uint8_t *sc, cudaStream_t stream, int32_t *zero = nullptr,
                      const RoutePlan &plan = RoutePlan{});
// the up projection writes h's e4m3 terms itself (true) or bf16 h for launch_split_e4m3 (false)
bool mx_fused_split(int tile_n);
int launch_mx_up(const uint8_t *w13, const uint8_t *s13, int E, int H, int I, const uint8_t *x_hi,
                 const uint8_t *x_lo, const uint8_t *x_sc, int S_rows, int order, float limit, const int4 *tiles,
                 const int32_t *n_tiles, uint8_t *h_hi, uint8_t *h_lo, uint8_t *h_sc, uint16_t *h, int32_t *err,
                 int tile_n, cudaStream_t stream, int T);  // T: tokens of the call (tiles of more than 16 use two epilogue groups)
// comb + done: the launch's last CTA also combines the rows (done zeroed by the call's first kernel)
int launch_mx_down(const uint8_t *w2, const uint8_t *s2, int E, int H, int I, const uint8_t *h_hi,
                   const uint8_t *h_lo, const uint8_t *h_sc, int S_rows, const int4 *tiles, const int32_t *n_tiles,
                   uint16_t *y, int32_t *err, int tile_n, cudaStream_t stream, const CombineArgs *comb = nullptr,
                   int32_t *done = nullptr);

// Workspace carved out of the caller's buffer for one expert-forward call.
// S = T * (k + has_shared) assignments.
struct MoeWorkspace {
  int32_t *offsets;    // [E+1]
  int32_t *perm;       // [S] sorted slot -> flat assignment
  int32_t *inv;        // [S] flat assignment -> sorted slot
  int32_t *active;     // [E] active expert ids, ascending
  int32_t *counters;   // [8]: n_active, permute error flag, n_tiles, tensor-core error code, fused-combine ticket
  int4 *tiles;         // [E + S/16 + 2] tensor-core work list
  uint16_t *h;         // [S_pad, I] SwiGLU output in sorted-slot order (bf16; f16 on the f16 tensor path)
  uint16_t *x16;       // [S_pad, H] f16 tokens in sorted-slot order (f16 tensor path)
  uint8_t *x_hi, *x_lo;  // [S_pad, H] e4m3 token terms (block-scaled path; same bytes as x16)
  uint8_t *x_sc;       // [S_pad, H/32] E8M0 scale of x_hi
  uint8_t *h_hi, *h_lo;  // [S_pad, I] e4m3 terms of h
  uint8_t *h_sc;       // [S_pad, I/32]
  uint16_t *y;         // [S, H] bf16 expert outputs in sorted-slot order (the reference switch_mlp dtype)
  int s_pad;           // S rounded up to at least 16 rows (TMA box height)
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
  size_t o_cnt = take(8 * sizeof(int32_t));
  const size_t S_pad = S < 16 ? 16 : S;
  size_t o_tiles = take((E + S / 16 + 2) * sizeof(int4));
  size_t o_h = take(S_pad * I * sizeof(uint16_t));
  size_t o_x16 = take(S_pad * H * sizeof(uint16_t));
  size_t o_xsc = take(S_pad * (H / 32));
  size_t o_h8 = take(S_pad * I * 2);
  size_t o_hsc = take(S_pad * (I / 32));
  size_t o_y = take(S * H * sizeof(uint16_t));
  w.s_pad = static_cast<int>(S_pad);
  w.bytes = off;
  if (base) {
    char *b = static_cast<char *>(base);
    w.offsets = reinterpret_cast<int32_t *>(b + o_off);
    w.perm = reinterpret_cast<int32_t *>(b + o_perm);
    w.inv = reinterpret_cast<int32_t *>(b + o_inv);
    w.active = reinterpret_cast<int32_t *>(b + o_act);
    w.counters = reinterpret_cast<int32_t *>(b + o_cnt);
    w.tiles = reinterpret_cast<int4 *>(b + o_tiles);
    w.h = reinterpret_cast<uint16_t *>(b + o_h);
    w.x16 = reinterpret_cast<uint16_t *>(b + o_x16);
    w.x_hi = reinterpret_cast<uint8_t *>(b + o_x16);
    w.x_lo = w.x_hi + S_pad * H;
    w.x_sc = reinterpret_cast<uint8_t *>(b + o_xsc);
    w.h_hi = reinterpret_cast<uint8_t *>(b + o_h8);
    w.h_lo = w.h_hi + S_pad * I;
    w.h_sc = reinterpret_cast<uint8_t *>(b + o_hsc);
    w.y = reinterpret_cast<uint16_t *>(b + o_y);
  }
  return w;
}

}  // namespace wm
