// Router: gate logits, score function, top-k, weight renormalisation.
//
// Reference: Gate.__call__ (deepseek_v41/moe.py:58-75), SparseMoE routing
// (qwen4_exp.py:692-699), tie rule _stable_topk_indices (model.py:548-560).
//
// Exactness contract with the CPU restatement (fixed float32 order):
//   logit[t][e]: the 256-wide column blocks i = 0..n-1 are split into 4
//   contiguous segments [s*n/4, (s+1)*n/4); in each, lane l accumulates with
//   fmaf the elements h = 256*i + 8*l + j (i ascending, j = 0..7); a lane's 4
//   segment partials are added in segment order, and the 32 lane sums are
//   combined by a shuffle butterfly with strides 16, 8, 4, 2, 1.  The softmax
//   denominator uses the same butterfly over lane partials of experts
//   l, l+32, l+64, ...  Compiled with -fmad=false.
//
// Kernel 1 (logits): one 4-warp CTA per (expert-row group, token group);
//   each warp streams a quarter of the rows with 16-byte loads.
// Kernel 2 (top-k): one warp per token; scores in registers, then k rounds
//   of a warp arg-max with ties to the lower expert id.
//
// WM_SCORE_SOFTMAX_BF16 is the Qwen gate as the reference evaluates it: the
// bf16 nn.Linear rounds the logits to bf16 (qwen4_exp.py:683), softmax
// (precise=True) runs in float32 and returns bf16 probabilities
// (qwen4_exp.py:693), top-k selects on those bf16 values (:694-695), and the
// renormalisation divides bf16 by a bf16 sum, rounding the quotient to bf16
// (:696-697); the shared-expert gate is sigmoid of a bf16 logit, rounded to
// bf16 (:699).  Every rounding is round-to-nearest-even.
#include <mutex>

#include "wm_common.cuh"
#include "wm_detmath.cuh"
#include "wm_topk.cuh"

namespace {

constexpr int kMaxE = 1024;
constexpr int kMaxK = 32;
constexpr int kSegs = 4;          // warps per expert row

__device__ __forceinline__ float round_bf16(float v) { return wm_bf16_to_f32(wm_f32_to_bf16(v)); }

// One CTA (4 warps) per (group of ET expert rows, group of TT tokens).  Warp
// s takes the column blocks [s*n/4, (s+1)*n/4) (n = ceil(H/256)); lane l
// keeps one fmaf chain per (expert, token) pair of the tile over its 8-element
// pieces 256*i + 8*l .. +7, so every weight and token load feeds ET or TT
// chains.  Partials meet in shared memory; warp w reduces the pairs
// p = w, w+4, ... in the canonical order.
template <int ET, int TT>
__global__ void __launch_bounds__(128) k_router_logits(const uint16_t *__restrict__ x, const uint16_t *__restrict__ wg,
                                                       const uint16_t *__restrict__ wg_shared,
                                                       const float *__restrict__ logit_bias, int T, int H, int E,
                                                       float *__restrict__ logits, float *__restrict__ shared_raw) {
  __shared__ float part[kSegs][ET * TT][32];
  WM_PDL_WAIT();
  WM_PDL_LAUNCH();
  const int lane = threadIdx.x & 31, seg = threadIdx.x >> 5;
  const int rows = E + (wg_shared ? 1 : 0);
  const int egroups = (rows + ET - 1) / ET;
  const int e0 = (blockIdx.x % egroups) * ET;
  const int t0 = (blockIdx.x / egroups) * TT;
  const uint16_t *wrow[ET];
#pragma unroll
  for (int a = 0; a < ET; ++a) {
    const int e = min(e0 + a, rows - 1);              // clamped rows compute a discarded duplicate
    wrow[a] = e < E ? wg + static_cast<int64_t>(e) * H : wg_shared;
  }
  const uint16_t *xrow[TT];
#pragma unroll
  for (int b = 0; b < TT; ++b) xrow[b] = x + static_cast<int64_t>(min(t0 + b, T - 1)) * H;
  const int n = (H + 255) / 256;
  const int i0 = (seg * n) / kSegs, i1 = ((seg + 1) * n) / kSegs;
  float acc[ET][TT];
#pragma unroll
  for (int a = 0; a < ET; ++a)
#pragma unroll
    for (int b = 0; b < TT; ++b) acc[a][b] = 0.0f;
  // loads of D column blocks are issued before any of them is consumed: small
  // tiles (decode) keep a whole segment in flight, large tiles two blocks
  constexpr int D = (ET + TT <= 4) ? 8 : 2;
  for (int i0c = i0; i0c < i1; i0c += D) {
    uint4 wu[D][ET], xu[D][TT];
#pragma unroll
    for (int d = 0; d < D; ++d) {
      const int base = 256 * (i0c + d) + 8 * lane;
      const bool live = i0c + d < i1 && base < H;
#pragma unroll
      for (int a = 0; a < ET; ++a)
        wu[d][a] = live ? __ldg(reinterpret_cast<const uint4 *>(wrow[a] + base)) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int b = 0; b < TT; ++b)
        xu[d][b] = live ? __ldg(reinterpret_cast<const uint4 *>(xrow[b] + base)) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int d = 0; d < D; ++d) {
      const int base = 256 * (i0c + d) + 8 * lane;
      if (!(i0c + d < i1 && base < H)) continue;        // the chain skips absent pieces exactly as before
      float xv[TT][8];                                  // each token piece converted once per block
#pragma unroll
      for (int b = 0; b < TT; ++b) {
        xv[b][0] = wm_bf16lo(xu[d][b].x); xv[b][1] = wm_bf16hi(xu[d][b].x);
        xv[b][2] = wm_bf16lo(xu[d][b].y); xv[b][3] = wm_bf16hi(xu[d][b].y);
        xv[b][4] = wm_bf16lo(xu[d][b].z); xv[b][5] = wm_bf16hi(xu[d][b].z);
        xv[b][6] = wm_bf16lo(xu[d][b].w); xv[b][7] = wm_bf16hi(xu[d][b].w);
      }
#pragma unroll
      for (int a = 0; a < ET; ++a) {
        const float wv[8] = {wm_bf16lo(wu[d][a].x), wm_bf16hi(wu[d][a].x), wm_bf16lo(wu[d][a].y),
                             wm_bf16hi(wu[d][a].y), wm_bf16lo(wu[d][a].z), wm_bf16hi(wu[d][a].z),
                             wm_bf16lo(wu[d][a].w), wm_bf16hi(wu[d][a].w)};
#pragma unroll
        for (int b = 0; b < TT; ++b) {
          float v = acc[a][b];
#pragma unroll
          for (int j = 0; j < 8; ++j) v = fmaf(xv[b][j], wv[j], v);
          acc[a][b] = v;
        }
      }
    }
  }
#pragma unroll
  for (int a = 0; a < ET; ++a)
#pragma unroll
    for (int b = 0; b < TT; ++b) part[seg][a * TT + b][lane] = acc[a][b];
  __syncthreads();
  for (int pidx = seg; pidx < ET * TT; pidx += kSegs) {
    float v = ((part[0][pidx][lane] + part[1][pidx][lane]) + part[2][pidx][lane]) + part[3][pidx][lane];
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) v = v + __shfl_xor_sync(0xffffffffu, v, m);
    const int e = e0 + pidx / TT, t = t0 + pidx % TT;
    if (lane == 0 && e < rows && t < T) {
      if (e < E) logits[static_cast<int64_t>(t) * E + e] = logit_bias ? v + logit_bias[e] : v;
      else shared_raw[t] = v;
    }
  }
}

// Large-T variant: the same chains for an (ET experts x TT tokens) tile, with
// each lane's 8-element pieces of the next column block copied with cp.async
// into its own slots of a double-buffered shared-memory stage while the
// current block is computed (no registers held by loads in flight), so the
// tile can be large enough for the FMAs, not the loads, to set the pace.
template <int ET, int TT>
__global__ void __launch_bounds__(128) k_router_logits_staged(const uint16_t *__restrict__ x,
                                                              const uint16_t *__restrict__ wg,
                                                              const uint16_t *__restrict__ wg_shared,
                                                              const float *__restrict__ logit_bias, int T, int H,
                                                              int E, float *__restrict__ logits,
                                                              float *__restrict__ shared_raw) {
  extern __shared__ __align__(16) uint4 stage[];        // [4 warps][2 buffers][ET + TT rows][32 lanes]
  WM_PDL_WAIT();
  WM_PDL_LAUNCH();
  const int lane = threadIdx.x & 31, seg = threadIdx.x >> 5;
  const int rows = E + (wg_shared ? 1 : 0);
  const int egroups = (rows + ET - 1) / ET;
  const int e0 = (blockIdx.x % egroups) * ET;
  const int t0 = (blockIdx.x / egroups) * TT;
  const uint16_t *src[ET + TT];
#pragma unroll
  for (int a = 0; a < ET; ++a) {
    const int e = min(e0 + a, rows - 1);
    src[a] = e < E ? wg + static_cast<int64_t>(e) * H : wg_shared;
  }
#pragma unroll
  for (int b = 0; b < TT; ++b) src[ET + b] = x + static_cast<int64_t>(min(t0 + b, T - 1)) * H;
  const int n = (H + 255) / 256;
  const int i0 = (seg * n) / kSegs, i1 = ((seg + 1) * n) / kSegs;
  uint4 *mine = stage + seg * 2 * (ET + TT) * 32;
  auto issue = [&](int i, int buf) {
    const int base = 256 * i + 8 * lane;
    if (i < i1 && base < H) {
#pragma unroll
      for (int r = 0; r < ET + TT; ++r) {
        const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(mine + (buf * (ET + TT) + r) * 32 + lane));
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src[r] + base) : "memory");
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  float acc[ET][TT];
#pragma unroll
  for (int a = 0; a < ET; ++a)
#pragma unroll
    for (int b = 0; b < TT; ++b) acc[a][b] = 0.0f;
  issue(i0, 0);
  for (int i = i0; i < i1; ++i) {
    const int buf = (i - i0) & 1;
    issue(i + 1, buf ^ 1);
    asm volatile("cp.async.wait_group 1;" ::: "memory");
    if (256 * i + 8 * lane >= H) continue;            // the chain skips absent pieces exactly as before
    const uint4 *row = mine + buf * (ET + TT) * 32 + lane;
    float wv[ET][8];
#pragma unroll
    for (int a = 0; a < ET; ++a) {
      const uint4 u = row[a * 32];
      wv[a][0] = wm_bf16lo(u.x); wv[a][1] = wm_bf16hi(u.x); wv[a][2] = wm_bf16lo(u.y); wv[a][3] = wm_bf16hi(u.y);
      wv[a][4] = wm_bf16lo(u.z); wv[a][5] = wm_bf16hi(u.z); wv[a][6] = wm_bf16lo(u.w); wv[a][7] = wm_bf16hi(u.w);
    }
#pragma unroll
    for (int b = 0; b < TT; ++b) {
      const uint4 u = row[(ET + b) * 32];
      const float xv[8] = {wm_bf16lo(u.x), wm_bf16hi(u.x), wm_bf16lo(u.y), wm_bf16hi(u.y),
                           wm_bf16lo(u.z), wm_bf16hi(u.z), wm_bf16lo(u.w), wm_bf16hi(u.w)};
#pragma unroll
      for (int a = 0; a < ET; ++a) {
        float v = acc[a][b];
#pragma unroll
        for (int j = 0; j < 8; ++j) v = fmaf(xv[j], wv[a][j], v);
        acc[a][b] = v;
      }
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();                                      // the stage is reused for the partials below
  float *part = reinterpret_cast<float *>(stage);       // [kSegs][ET * TT][32]
#pragma unroll
  for (int a = 0; a < ET; ++a)
#pragma unroll
    for (int b = 0; b < TT; ++b) part[(seg * ET * TT + a * TT + b) * 32 + lane] = acc[a][b];
  __syncthreads();
  for (int pidx = seg; pidx < ET * TT; pidx += kSegs) {
    float v = ((part[(0 * ET * TT + pidx) * 32 + lane] + part[(1 * ET * TT + pidx) * 32 + lane]) +
               part[(2 * ET * TT + pidx) * 32 + lane]) +
              part[(3 * ET * TT + pidx) * 32 + lane];
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) v = v + __shfl_xor_sync(0xffffffffu, v, m);
    const int e = e0 + pidx / TT, t = t0 + pidx % TT;
    if (lane == 0 && e < rows && t < T) {
      if (e < E) logits[static_cast<int64_t>(t) * E + e] = logit_bias ? v + logit_bias[e] : v;
      else shared_raw[t] = v;
    }
  }
}

// Many tokens, short rows (T > 64, H <= 4096): the per-warp segments of the
// kernels above hold only a few column blocks, so their shared-memory partial
// reduction outweighs the multiply-adds.  Here one thread owns a TE x TT tile
// of (expert, token) outputs and evaluates each output's whole canonical sum
// itself: the 32 lane partials l (each the four segment chains, added in
// segment order) are produced in bit-reversed lane order 0, 16, 8, 24, 4, ...,
// which turns the butterfly (strides 16, 8, 4, 2, 1) into a five-level binary
// counter of running sums -- the same additions in the same tree, so the
// bits equal k_router_logits'.  A CTA (256 threads) covers 16 TE experts x
// 16 TT tokens; leaf l's 16-byte pieces 256 i + 8 l of its rows are staged
// with cp.async, double buffered; token pairs share packed f32x2 FMAs; the
// last merge lands in the tree's top level, which then holds the output.
// 8 x 4 tiles (half the token staging per multiply-add; a few registers
// spill) measured 10 % faster than 4 x 4 from one and a half waves of CTAs up
// (512-row gate: 1730 -> 1551 us at 16384 tokens, 492 -> 441 at 4096) and
// slower below (127 -> 217 us at 1024).

__device__ __forceinline__ int bitrev5(int k) { return static_cast<int>(__brev(static_cast<unsigned>(k)) >> 27); }

// The CTA's tile: rows [e0, e0 + 16 TE) x tokens [t0, t0 + 16 TT).
template <int TE, int TT>
__device__ __forceinline__ void tree_tile(const uint16_t *__restrict__ x, const uint16_t *__restrict__ wg,
                                          const uint16_t *__restrict__ wg_shared,
                                          const float *__restrict__ logit_bias, int T, int H, int E, int e0, int t0,
                                          float *__restrict__ logits, float *__restrict__ shared_raw,
                                          uint4 *tstage) {                // [2][(16 * (TE + TT))][pitch]
  const int n = (H + 255) / 256;
  const int pitch = n + ((9 - n % 8) % 8);               // pitch % 8 == 1: 16 consecutive rows hit distinct banks
  const int rows = E + (wg_shared ? 1 : 0);
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  // staged row r: r < 16 TE gate row e0 + r (clamped; row E is the shared gate), else token t0 + r - 16 TE
  auto row_ptr = [&](int r) -> const uint16_t * {
    if (r < 16 * TE) {
      const int e = min(e0 + r, rows - 1);
      return e < E ? wg + static_cast<int64_t>(e) * H : wg_shared;
    }
    return x + static_cast<int64_t>(min(t0 + r - 16 * TE, T - 1)) * H;
  };
  auto issue = [&](int leaf, int buf) {
    uint4 *dst = tstage + buf * (16 * (TE + TT)) * pitch;
    for (int c = threadIdx.x; c < (16 * (TE + TT)) * n; c += 256) {
      const int r = c / n, i = c - r * n;
      const int base = 256 * i + 8 * leaf;
      const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst + r * pitch + i));
      const uint16_t *src = row_ptr(r) + (base < H ? base : 0);
      const int sz = base < H ? 16 : 0;                  // out-of-row pieces are zero-filled (and skipped)
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(sz) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  float lv[5][TE][TT];                         // running sums of the butterfly tree, by level
  issue(0, 0);
  for (int k = 0; k < 32; ++k) {
    const int leaf = bitrev5(k);
    if (k + 1 < 32) {
      issue(bitrev5(k + 1), (k + 1) & 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const uint4 *st = tstage + (k & 1) * (16 * (TE + TT)) * pitch;
    float ls[TE][TT];                          // lane partial of this leaf: segments in order
#pragma unroll
    for (int a = 0; a < TE; ++a)
#pragma unroll
      for (int b = 0; b < TT; ++b) ls[a][b] = 0.0f;
    for (int sg = 0; sg < 4; ++sg) {
      const int i0 = (sg * n) / 4, i1 = ((sg + 1) * n) / 4;
      float2 acc[TE][TT / 2];                  // {token 2 bp, token 2 bp + 1}
#pragma unroll
      for (int a = 0; a < TE; ++a)
#pragma unroll
        for (int bp = 0; bp < TT / 2; ++bp) acc[a][bp] = make_float2(0.0f, 0.0f);
      for (int i = i0; i < i1; ++i) {
        if (256 * i + 8 * leaf >= H) continue;           // the chain skips absent pieces, as k_router_logits
        uint4 wu[TE], xu[TT];
#pragma unroll
        for (int a = 0; a < TE; ++a) wu[a] = st[(ty + 16 * a) * pitch + i];
#pragma unroll
        for (int b = 0; b < TT; ++b) xu[b] = st[(16 * TE + tx + 16 * b) * pitch + i];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int wd = j >> 1;
          float xv[TT];
#pragma unroll
          for (int b = 0; b < TT; ++b) {
            const uint32_t u = wd == 0 ? xu[b].x : wd == 1 ? xu[b].y : wd == 2 ? xu[b].z : xu[b].w;
            xv[b] = (j & 1) ? wm_bf16hi(u) : wm_bf16lo(u);
          }
#pragma unroll
          for (int a = 0; a < TE; ++a) {
            const uint32_t u = wd == 0 ? wu[a].x : wd == 1 ? wu[a].y : wd == 2 ? wu[a].z : wu[a].w;
            const float wv = (j & 1) ? wm_bf16hi(u) : wm_bf16lo(u);
#pragma unroll
            for (int bp = 0; bp < TT / 2; ++bp)
              acc[a][bp] = wm_fma2(make_float2(xv[2 * bp], xv[2 * bp + 1]), make_float2(wv, wv), acc[a][bp]);
          }
        }
      }
#pragma unroll
      for (int a = 0; a < TE; ++a)
#pragma unroll
        for (int bp = 0; bp < TT / 2; ++bp) {
          ls[a][2 * bp] = ls[a][2 * bp] + acc[a][bp].x;   // ((seg0 + seg1) + seg2) + seg3 (0 + seg0 exact)
          ls[a][2 * bp + 1] = ls[a][2 * bp + 1] + acc[a][bp].y;
        }
    }
    // insert the leaf into the tree: k's trailing ones are the merges
#pragma unroll
    for (int a = 0; a < TE; ++a)
#pragma unroll
      for (int b = 0; b < TT; ++b) {
        float v = ls[a][b];
        if (!(k & 1)) { lv[0][a][b] = v; continue; }
        v = lv[0][a][b] + v;
        if (!(k & 2)) { lv[1][a][b] = v; continue; }
        v = lv[1][a][b] + v;
        if (!(k & 4)) { lv[2][a][b] = v; continue; }
        v = lv[2][a][b] + v;
        if (!(k & 8)) { lv[3][a][b] = v; continue; }
        v = lv[3][a][b] + v;
        if (!(k & 16)) { lv[4][a][b] = v; continue; }
        lv[4][a][b] = lv[4][a][b] + v;
      }
    __syncthreads();                                     // buffer k & 1 is refilled by the next iteration's issue
  }
#pragma unroll
  for (int a = 0; a < TE; ++a) {
    const int e = e0 + ty + 16 * a;
#pragma unroll
    for (int b = 0; b < TT; ++b) {
      const int t = t0 + tx + 16 * b;
      if (e < rows && t < T) {
        if (e < E) logits[static_cast<int64_t>(t) * E + e] = logit_bias ? lv[4][a][b] + logit_bias[e] : lv[4][a][b];
        else shared_raw[t] = lv[4][a][b];
      }
    }
  }
}


// Rows [0, main_rows) in TE x TT tiles (main_rows a multiple of 16 TE), then
// the few rows left over (the shared gate after 512 experts) in TE2 x TT tiles,
// so that a ragged last row group does not cost a whole wide tile.
template <int TE, int TT, int TE2>
__global__ void __launch_bounds__(256, 1) k_router_logits_tree(const uint16_t *__restrict__ x,
                                                               const uint16_t *__restrict__ wg,
                                                               const uint16_t *__restrict__ wg_shared,
                                                               const float *__restrict__ logit_bias, int T, int H,
                                                               int E, float *__restrict__ logits,
                                                               float *__restrict__ shared_raw, int main_rows) {
  extern __shared__ __align__(16) uint4 tstage[];
  WM_PDL_WAIT();
  WM_PDL_LAUNCH();
  const int eg = main_rows / (16 * TE);
  const int main_ctas = eg * ((T + 16 * TT - 1) / (16 * TT));
  const int b = static_cast<int>(blockIdx.x);
  if (b < main_ctas) {
    tree_tile<TE, TT>(x, wg, wg_shared, logit_bias, T, H, E, (b % eg) * 16 * TE, (b / eg) * 16 * TT, logits,
                      shared_raw, tstage);
  } else {
    const int rows = E + (wg_shared ? 1 : 0);
    const int eg2 = (rows - main_rows + 16 * TE2 - 1) / (16 * TE2);
    const int r = b - main_ctas;
    tree_tile<TE2, TT>(x, wg, wg_shared, logit_bias, T, H, E, main_rows + (r % eg2) * 16 * TE2,
                       (r / eg2) * 16 * TT, logits, shared_raw, tstage);
  }
}

// Tile shape by batch: enough CTAs to stream the gate matrix at small T, and
// register-resident reuse of every load (ET x TT chains) at large T.
int launch_router_logits(const uint16_t *x, const uint16_t *wg, const uint16_t *wg_shared, const float *logit_bias,
                         int T, int H, int E, float *logits, float *shared_raw, cudaStream_t stream) {
  const int rows = E + (wg_shared ? 1 : 0);
  auto go = [&](auto kern, int et, int tt) {
    const int64_t ctas = static_cast<int64_t>((rows + et - 1) / et) * ((T + tt - 1) / tt);
    if (ctas >= (1LL << 31)) return wm::fail(WM_ERR_INVALID, "router: too many tokens");
    if (cudaError_t e = wm::launch_pdl(kern, dim3(static_cast<unsigned>(ctas)), dim3(128), 0, stream, x, wg, wg_shared,
                                       logit_bias, T, H, E, logits, shared_raw))
      return wm::fail(WM_ERR_CUDA, std::string("router logits: ") + cudaGetErrorString(e));
    return wm::check_launch("router logits");
  };
  if (T <= 1) return go(k_router_logits<2, 1>, 2, 1);
  if (T <= 16) return go(k_router_logits<2, 4>, 2, 4);
  if (T <= 64) {
    // 4 x 8 tiles with the loads staged through shared memory (no registers held by loads in flight):
    // measured against the register-held form, router 19.7 -> 16.1 us at 64 tokens (DeepSeek-class gate),
    // 13.8 -> 10.8 us at 32 (Qwen-class); 2 x 4 register tiles are the faster form at 16 tokens and fewer
    constexpr int ET = 4, TT = 8;
    constexpr size_t smem = static_cast<size_t>(kSegs) * 2 * (ET + TT) * 32 * sizeof(uint4);
    static_assert(smem >= static_cast<size_t>(kSegs) * ET * TT * 32 * sizeof(float), "stage must hold the partials");
    static std::mutex smu;
    static bool sattr[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return wm::fail(WM_ERR_CUDA, "router: no device");
    {
      std::lock_guard<std::mutex> lock(smu);
      if (!sattr[dev]) {
        if (cudaError_t e = cudaFuncSetAttribute(k_router_logits_staged<ET, TT>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)))
          return wm::fail(WM_ERR_CUDA, std::string("router logits smem: ") + cudaGetErrorString(e));
        sattr[dev] = true;
      }
    }
    const int64_t ctas = static_cast<int64_t>((rows + ET - 1) / ET) * ((T + TT - 1) / TT);
    if (cudaError_t e = wm::launch_pdl(k_router_logits_staged<ET, TT>, dim3(static_cast<unsigned>(ctas)), dim3(128),
                                       smem, stream, x, wg, wg_shared, logit_bias, T, H, E, logits, shared_raw))
      return wm::fail(WM_ERR_CUDA, std::string("router logits: ") + cudaGetErrorString(e));
    return wm::check_launch("router logits");
  }
  if (H <= 4096) {
    const int n = (H + 255) / 256;
    const size_t pitch = n + ((9 - n % 8) % 8);
    static std::mutex tmu;
    static bool tattr[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return wm::fail(WM_ERR_CUDA, "router: no device");
    {
      std::lock_guard<std::mutex> lock(tmu);
      if (!tattr[dev]) {
        // H <= 4096: at most 2 buffers x 192 rows x 17 pieces x 16 B = 104 KB
        for (auto kern : {k_router_logits_tree<4, 4, 1>, k_router_logits_tree<8, 4, 1>})
          if (cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(112 * 1024)))
            return wm::fail(WM_ERR_CUDA, std::string("router logits smem: ") + cudaGetErrorString(e));
        tattr[dev] = true;
      }
    }
    const int tg = (T + 63) / 64;
    auto tree = [&](auto kern, int te) {
      const int main_rows = rows / (16 * te) * (16 * te);
      const int64_t ctas = static_cast<int64_t>(main_rows / (16 * te) + (rows - main_rows + 15) / 16) * tg;
      const size_t smem = static_cast<size_t>(2) * 16 * (te + 4) * pitch * sizeof(uint4);
      if (ctas >= (1LL << 31)) return wm::fail(WM_ERR_INVALID, "router: too many tokens");
      if (cudaError_t e = wm::launch_pdl(kern, dim3(static_cast<unsigned>(ctas)), dim3(256), smem, stream, x, wg,
                                         wg_shared, logit_bias, T, H, E, logits, shared_raw, main_rows))
        return wm::fail(WM_ERR_CUDA, std::string("router logits: ") + cudaGetErrorString(e));
      return wm::check_launch("router logits");
    };
    if (2 * static_cast<int64_t>(rows / 128) * tg >= 3LL * wm::sm_count()) return tree(k_router_logits_tree<8, 4, 1>, 8);
    return tree(k_router_logits_tree<4, 4, 1>, 4);
  }
  // large T: staged 8 x 16 tiles; stage = 4 warps x 2 buffers x 24 rows x 512 B = 96 KB, which also holds the
  // 4 x 128 x 32 partial sums (64 KB) afterwards
  constexpr int ET = 8, TT = 16;
  constexpr size_t smem = static_cast<size_t>(kSegs) * 2 * (ET + TT) * 32 * sizeof(uint4);
  static_assert(smem >= static_cast<size_t>(kSegs) * ET * TT * 32 * sizeof(float), "stage must hold the partials");
  static std::mutex mu;
  static bool attr_set[64] = {false};                    // per device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return wm::fail(WM_ERR_CUDA, "router: no device");
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!attr_set[dev]) {
      if (cudaError_t e = cudaFuncSetAttribute(k_router_logits_staged<ET, TT>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)))
        return wm::fail(WM_ERR_CUDA, std::string("router logits smem: ") + cudaGetErrorString(e));
      attr_set[dev] = true;
    }
  }
  const int64_t ctas = static_cast<int64_t>((rows + ET - 1) / ET) * ((T + TT - 1) / TT);
  if (ctas >= (1LL << 31)) return wm::fail(WM_ERR_INVALID, "router: too many tokens");
  if (cudaError_t e = wm::launch_pdl(k_router_logits_staged<ET, TT>, dim3(static_cast<unsigned>(ctas)), dim3(128),
                                     smem, stream, x, wg, wg_shared, logit_bias, T, H, E, logits, shared_raw))
    return wm::fail(WM_ERR_CUDA, std::string("router logits: ") + cudaGetErrorString(e));
  return wm::check_launch("router logits");
}

// One warp per token (4 tokens per CTA): lane l holds the scores of experts
// l, l+32, ...; the softmax denominator sums them in that order and then
// across lanes with the butterfly; k rounds of a warp arg-max (ties to the
// lower expert id, NaN keys last) carry the winner's score along, and lane r
// keeps the r-th selection.  The renormalising sum runs over r in order.
template <int PER>
__global__ void __launch_bounds__(128) k_router_topk(const float *__restrict__ logits,
                                                     const float *__restrict__ select_bias, int T, int E, int k,
                                                     int score_fn, float norm_eps, float route_scale,
                                                     int32_t *__restrict__ idx, float *__restrict__ weights,
                                                     float *__restrict__ shared_w) {
  WM_PDL_WAIT();
  WM_PDL_LAUNCH();
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 4 + (threadIdx.x >> 5);
  if (t >= T) return;
  const float kNegInf = -__int_as_float(0x7f800000);
  const float *lt = logits + static_cast<int64_t>(t) * E;
  const bool bf = score_fn == WM_SCORE_SOFTMAX_BF16;
  float sc[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = lane + 32 * j;
    sc[j] = e < E ? (bf ? round_bf16(lt[e]) : lt[e]) : kNegInf;
  }
  if (score_fn == WM_SCORE_SOFTMAX || bf) {
    float mx = kNegInf;
#pragma unroll
    for (int j = 0; j < PER; ++j) mx = fmaxf(mx, sc[j]);
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, m));
    float part = 0.0f;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      if (lane + 32 * j < E) {
        sc[j] = wm_exp(sc[j] - mx);
        part = part + sc[j];
      }
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) part = part + __shfl_xor_sync(0xffffffffu, part, m);
#pragma unroll
    for (int j = 0; j < PER; ++j) sc[j] = bf ? round_bf16(__fdiv_rn(sc[j], part)) : __fdiv_rn(sc[j], part);
  } else if (score_fn == WM_SCORE_SIGMOID) {
#pragma unroll
    for (int j = 0; j < PER; ++j) sc[j] = wm_sigmoid(sc[j]);
  } else if (score_fn == WM_SCORE_SQRTSOFTPLUS) {
#pragma unroll
    for (int j = 0; j < PER; ++j) sc[j] = __fsqrt_rn(wm_softplus(sc[j]));
  }
  float key[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = lane + 32 * j;
    float kv = kNegInf;
    if (e < E) kv = select_bias ? sc[j] + select_bias[e] : sc[j];
    key[j] = (kv != kv) ? kNegInf : kv;
  }
  // Keys as order-preserving unsigned bits (-0 folded into +0, so equal
  // floats stay equal); each round takes the warp maximum of the lanes' best
  // untaken keys, then the lowest expert id among the lanes holding it.
  uint32_t kb[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const uint32_t b = __float_as_uint(key[j] == 0.0f ? 0.0f : key[j]);
    kb[j] = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  }
  uint32_t taken = 0u;                                // bit j: expert lane + 32 j selected
  float my_w = 0.0f;
  int32_t my_i = 0;
  for (int r = 0; r < k; ++r) {
    uint32_t best = 0u;                               // below every key (-inf maps to 0x007fffff)
    int bj = -1;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      if (lane + 32 * j < E && !((taken >> j) & 1u) && (bj < 0 || kb[j] > best)) {
        best = kb[j];
        bj = j;
      }
    }
    const uint32_t wbest = __reduce_max_sync(0xffffffffu, bj < 0 ? 0u : best);
    const int cand = (bj >= 0 && best == wbest) ? lane + 32 * bj : 0x7fffffff;
    const int be = static_cast<int>(__reduce_min_sync(0xffffffffu, static_cast<uint32_t>(cand)));
    float bs = 0.0f;
#pragma unroll
    for (int j = 0; j < PER; ++j)
      if (lane + 32 * j == be) bs = sc[j];
    bs = __shfl_sync(0xffffffffu, bs, be & 31);
    if ((be & 31) == lane) taken |= 1u << (be >> 5);
    if (lane == r) { my_w = bs; my_i = be; }
  }
  const bool norm = norm_eps >= 0.0f;
  float denom = 1.0f;
  if (norm) {
    float sum = 0.0f;
    for (int r = 0; r < k; ++r) sum = sum + __shfl_sync(0xffffffffu, my_w, r);
    denom = sum + norm_eps;
    if (bf) denom = round_bf16(denom);
  }
  if (lane < k) {
    float w = norm ? __fdiv_rn(my_w, denom) : my_w;
    if (bf) w = round_bf16(w);
    idx[static_cast<int64_t>(t) * k + lane] = my_i;
    weights[static_cast<int64_t>(t) * k + lane] = w * route_scale;
  }
  if (lane == 0 && shared_w)
    shared_w[t] = bf ? round_bf16(wm_sigmoid(round_bf16(shared_w[t]))) : wm_sigmoid(shared_w[t]);
}

// Wide routers (E > 128): one 256-thread CTA per token (wm::cta_topk_row:
// per-warp winners, then each candidate's place by counting the candidates
// ahead of it), so no single warp walks hundreds of experts in k serial
// rounds.  Same arithmetic and order as k_router_topk.
template <int PERT>
__global__ void __launch_bounds__(256) k_router_topk_cta(const float *__restrict__ logits,
                                                         const float *__restrict__ select_bias, int T, int E, int k,
                                                         int score_fn, float norm_eps, float route_scale,
                                                         int32_t *__restrict__ idx, float *__restrict__ weights,
                                                         float *__restrict__ shared_w) {
  constexpr int kWarpsCta = 8;
  __shared__ wm::TopkScratch<kWarpsCta> s;
  WM_PDL_WAIT();
  WM_PDL_LAUNCH();
  const int t = blockIdx.x;
  if (t >= T) return;
  float denom = 1.0f;
  wm::cta_topk_row<kWarpsCta, PERT>(logits + static_cast<int64_t>(t) * E, select_bias, E, k, score_fn, norm_eps, s,
                                    &denom);
  const bool bf = score_fn == WM_SCORE_SOFTMAX_BF16;
  const int r = threadIdx.x;
  if (r < k) {
    idx[static_cast<int64_t>(t) * k + r] = s.sel_id[r];
    weights[static_cast<int64_t>(t) * k + r] = wm::topk_weight(s.sel_w[r], denom, norm_eps >= 0.0f, bf, route_scale);
  }
  if (r == 0 && shared_w) shared_w[t] = wm::topk_shared_gate(shared_w[t], bf);
}

int launch_router_topk(const float *logits, const float *select_bias, int T, int E, int k, int score_fn,
                       float norm_eps, float route_scale, int32_t *idx, float *weights, float *shared_w,
                       cudaStream_t stream) {
  if (E > 128) {
    // one CTA per token; PERT experts per thread
    const int pert = (E + 255) / 256;
    cudaError_t e2 = cudaSuccess;
#define WM_TOPK_CTA(P)                                                                                          \
  e2 = wm::launch_pdl(k_router_topk_cta<P>, dim3(T), dim3(256), 0, stream, logits, select_bias, T, E, k, score_fn, \
                      norm_eps, route_scale, idx, weights, shared_w)
    if (pert <= 1) WM_TOPK_CTA(1);
    else if (pert <= 2) WM_TOPK_CTA(2);
    else WM_TOPK_CTA(4);
#undef WM_TOPK_CTA
    if (e2 != cudaSuccess) return wm::fail(WM_ERR_CUDA, std::string("router topk: ") + cudaGetErrorString(e2));
    return wm::check_launch("router topk");
  }
  const int grid = (T + 3) / 4;
  const int per = (E + 31) / 32;
#define WM_TOPK(P)                                                                                              \
  err = wm::launch_pdl(k_router_topk<P>, dim3(grid), dim3(128), 0, stream, logits, select_bias, T, E, k, score_fn, \
                       norm_eps, route_scale, idx, weights, shared_w)
  cudaError_t err = cudaSuccess;
  if (per <= 1) WM_TOPK(1);
  else if (per <= 2) WM_TOPK(2);
  else if (per <= 4) WM_TOPK(4);
  else if (per <= 8) WM_TOPK(8);
  else if (per <= 16) WM_TOPK(16);
  else WM_TOPK(32);
#undef WM_TOPK
  if (err != cudaSuccess) return wm::fail(WM_ERR_CUDA, std::string("router topk: ") + cudaGetErrorString(err));
  return wm::check_launch("router topk");
}

}  // namespace

namespace wm {

int router_logits(const uint16_t *x, const uint16_t *wg, const uint16_t *wg_shared, const float *logit_bias, int T,
                  int H, int E, float *logits, float *shared_raw, cudaStream_t stream) {
  return launch_router_logits(x, wg, wg_shared, logit_bias, T, H, E, logits, shared_raw, stream);
}

int router_topk(const float *logits, const float *select_bias, int T, int E, int k, int score_fn, float norm_eps,
                float route_scale, int32_t *idx, float *weights, float *shared_w, cudaStream_t stream) {
  return launch_router_topk(logits, select_bias, T, E, k, score_fn, norm_eps, route_scale, idx, weights, shared_w,
                            stream);
}

}  // namespace wm

extern "C" int wmoe_router_topk(const wm_bf16 *x, const wm_bf16 *wg, const float *logit_bias, const float *select_bias,
                                const wm_bf16 *wg_shared, int T, int H, int E, int k, int score_fn, float norm_eps,
                                float route_scale, float *logits, int32_t *idx, float *weights, float *shared_w,
                                wm_stream_t stream) {
  wm::clear_error();
  WM_REQUIRE(T >= 0 && H > 0 && H % 8 == 0, "router needs H % 8 == 0");
  WM_REQUIRE(E >= 1 && E <= kMaxE, "router supports 1 <= E <= 1024 experts");
  WM_REQUIRE(k >= 1 && k <= kMaxK && k <= E, "router needs 1 <= k <= min(32, E)");
  WM_REQUIRE(score_fn >= WM_SCORE_SOFTMAX && score_fn <= WM_SCORE_SOFTMAX_BF16, "unknown score function");
  if (T == 0) return WM_OK;
  WM_REQUIRE(x && wg && logits && idx && weights, "router: null buffer");
  WM_REQUIRE(!wg_shared || shared_w, "router: wg_shared needs a shared_w output");
  WM_REQUIRE(wm::aligned(x, 16) && wm::aligned(wg, 16) && (!wg_shared || wm::aligned(wg_shared, 16)),
             "router inputs must be 16-byte aligned");
  if (int rc = launch_router_logits(reinterpret_cast<const uint16_t *>(x), reinterpret_cast<const uint16_t *>(wg),
                                    reinterpret_cast<const uint16_t *>(wg_shared), logit_bias, T, H, E, logits,
                                    shared_w, stream))
    return rc;
  return launch_router_topk(logits, select_bias, T, E, k, score_fn, norm_eps, route_scale, idx, weights, shared_w,
                            stream);
}

extern "C" int wmoe_topk_scores(const float *logits, const float *select_bias, int T, int E, int k, int score_fn,
                                float norm_eps, float route_scale, int32_t *idx, float *weights, wm_stream_t stream) {
  wm::clear_error();
  WM_REQUIRE(T >= 0, "topk: T >= 0");
  WM_REQUIRE(E >= 1 && E <= kMaxE, "topk supports 1 <= E <= 1024");
  WM_REQUIRE(k >= 1 && k <= kMaxK && k <= E, "topk needs 1 <= k <= min(32, E)");
  WM_REQUIRE(score_fn >= WM_SCORE_SOFTMAX && score_fn <= WM_SCORE_SOFTMAX_BF16, "unknown score function");
  if (T == 0) return WM_OK;
  WM_REQUIRE(logits && idx && weights, "topk: null buffer");
  return launch_router_topk(logits, select_bias, T, E, k, score_fn, norm_eps, route_scale, idx, weights, nullptr,
                            stream);
}

// ------------------------------------------------------------------------
// Allocation-free variant of wmoe_router_topk.
//
// Some callers cannot call cudaMalloc at the point where they route: serving
// loops that must never take the device-synchronising allocation path, and
// hosts whose device memory is owned by another framework's allocator with no
// hook to borrow scratch.  This entry point takes the same inputs and outputs
// as wmoe_router_topk but keeps the [T, E] logits scratch in a fixed
// file-scope device array instead of a caller buffer.
//
// Limits and contract:
//   * the array holds kStaticLogits = 262,144 floats (1 MiB); every GPU that
//     loads this library reserves it until the process exits; T * E beyond it
//     is rejected with WM_ERR_INVALID;
//   * the array's device address is looked up once per device, on the first
//     call made with that device current (cudaGetSymbolAddress), and kept;
//     make that first call before any stream capture.  The kept address is
//     the one of the context current then: it does not survive
//     cudaDeviceReset;
//   * all calls share the one array and it keeps the last call's contents:
//     every element the kernels read is written earlier in the same call, so
//     nothing has to be cleared, but calls whose kernels overlap on the GPU
//     (different streams, no ordering between them) race on it.
// ------------------------------------------------------------------------
namespace {

constexpr int64_t kStaticLogits = 262144;
__device__ __align__(256) float g_router_logits_scratch[kStaticLogits];

std::mutex g_scratch_mu;
float *g_scratch_ptr[64] = {nullptr};

}  // namespace

extern "C" int wmoe_router_topk_static(const wm_bf16 *x, const wm_bf16 *wg, const float *logit_bias,
                                       const float *select_bias, const wm_bf16 *wg_shared, int T, int H, int E, int k,
                                       int score_fn, float norm_eps, float route_scale, int32_t *idx, float *weights,
                                       float *shared_w, wm_stream_t stream) {
  wm::clear_error();
  WM_REQUIRE(T >= 0 && H > 0 && H % 8 == 0, "router needs H % 8 == 0");
  WM_REQUIRE(E >= 1 && E <= kMaxE, "router supports 1 <= E <= 1024 experts");
  WM_REQUIRE(k >= 1 && k <= kMaxK && k <= E, "router needs 1 <= k <= min(32, E)");
  WM_REQUIRE(score_fn >= WM_SCORE_SOFTMAX && score_fn <= WM_SCORE_SOFTMAX_BF16, "unknown score function");
  WM_REQUIRE(static_cast<int64_t>(T) * E <= kStaticLogits,
             "wmoe_router_topk_static: T*E exceeds the 262144-float (1 MiB) static scratch; use wmoe_router_topk");
  if (T == 0) return WM_OK;
  WM_REQUIRE(x && wg && idx && weights, "router: null buffer");
  WM_REQUIRE(!wg_shared || shared_w, "router: wg_shared needs a shared_w output");
  WM_REQUIRE(wm::aligned(x, 16) && wm::aligned(wg, 16) && (!wg_shared || wm::aligned(wg_shared, 16)),
             "router inputs must be 16-byte aligned");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return wm::fail(WM_ERR_CUDA, "wmoe_router_topk_static: no current CUDA device");
  float *scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
      void *p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_router_logits_scratch);
      if (e != cudaSuccess || !p)
        return wm::fail(WM_ERR_CUDA, std::string("wmoe_router_topk_static: cudaGetSymbolAddress failed: ") +
                                         cudaGetErrorString(e));
      g_scratch_ptr[dev] = static_cast<float *>(p);
    }
    scratch = g_scratch_ptr[dev];
  }
  if (int rc = launch_router_logits(reinterpret_cast<const uint16_t *>(x), reinterpret_cast<const uint16_t *>(wg),
                                    reinterpret_cast<const uint16_t *>(wg_shared), logit_bias, T, H, E, scratch,
                                    shared_w, stream))
    return rc;
  return launch_router_topk(scratch, select_bias, T, E, k, score_fn, norm_eps, route_scale, idx, weights, shared_w,
                            stream);
}
