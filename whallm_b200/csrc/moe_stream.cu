// Decode-size MXFP4 expert FFN on CUDA cores: calls of one or two tokens.
//
// Reference: the MLX gather_qmm decode path (model.py:393-481,
// qwen4_exp.py:613-678): y = x @ dequant(W)^T per routed (token, expert)
// pair, ClampedSwiGLU (deepseek_v41/moe.py:30-43) between the projections.
//
// At one or two tokens a layer is a weight stream and each weight byte meets
// at most two token values, so for Qwen-class experts (1.6 MB each, 17 MB per
// token) the tensor-core kernels' fixed cost (TMEM and barrier set-up,
// pipeline fill, a split launch) is most of the call.  Here the weights go
// from HBM through shared memory straight to CUDA-core arithmetic:
//
//   * A chunk is 8 weight rows of one active expert (up projection: up_j..j+3
//     and gate_j..j+3, so the SwiGLU runs in the epilogue).  The chunks of
//     all active experts are cut into one contiguous range per CTA and one
//     per warp, so every SM streams the same number of bytes.
//   * Lane l takes piece l + 32 s of each row: 16 bytes (one whole 32-value
//     scale group), or 8 bytes (half a group) for rows of fewer than 1024
//     values, so each row's step is one coalesced 512-byte (256-byte) read.
//     The pieces travel by cp.async through a 3-stage ring per warp in shared
//     memory, two steps ahead of the arithmetic (12 warps x 2 x 4 KB, about
//     96 KB in flight per SM, none of it in registers; a register double
//     buffer stalled on loads at 28 % of the HBM peak).
//   * cvt.rn.f16x2.e2m1x2 turns each weight byte into two exact f16 values;
//     fma.rn.f32.f16 multiplies them by the token values exactly and rounds
//     once into an f32 sum.  The token operand is held as f16 with a power of
//     two per 32-value group, chosen so the group's largest magnitude lies in
//     [2^14, 2^15): every bf16 value within 2^-32 of its group maximum is then
//     exact in f16, and smaller ones are off by less than 2^-39 of it.  The
//     operand rows (up: the call's tokens; down: the SwiGLU rows of the
//     CTA's experts, bf16 as the reference rounds them) are converted into
//     shared memory once per CTA.
//   * Per (row, token): two f32 chains (even and odd values) per piece, their
//     sum times the group's token scale, then fmaf with the row's E8M0 scale
//     into the lane's sum; the 32 lane sums meet in a butterfly whose tree
//     does not depend on how many (row, token) sums it carries, so a token's
//     result is the same alone or beside another.
//
// Measured (one B200, expert call with permute and combine, eager launches):
// Qwen-class one token 23.3 us against 28.4 us on the block-scaled tensor
// cores, two tokens 32.7 against 33.1 us; DeepSeek-class one token 67 us
// against 59 us -- about 2.3 issued instructions per weight value (the
// conversion and one FMA per value and token) keep a 23 MB expert below the
// HBM rate, so the dispatch sends only small experts here.
//
// Three launch forms (MODE): 0 the up projection (+ ClampedSwiGLU, and for
// a small call the grouping of its slots, CTA 0 writing it for the later
// launches); 1 the down projection over a contiguous share of (expert, chunk)
// pairs per CTA, y (bf16, slot order) combined by k_combine or the last CTA;
// 2 the down projection of a small call split by output rows: CTA b takes
// chunks [b n, b n + n) of every active expert, groups the call and issues its
// first weight copies before its dependency wait (the routing was complete
// before the up projection's own wait returned), and combines its own rows
// with k_combine's arithmetic -- y never leaves shared memory.
#include <mutex>

#include "wm_common.cuh"
#include "wm_combine.cuh"
#include "wm_moe.cuh"
#include "wm_tc.cuh"
#include "wm_stream.cuh"

namespace {

using namespace wm_stream;

constexpr int kWarps = 12;
constexpr int kThreads = kWarps * 32;
constexpr int kRows = 8;    // weight rows per chunk (up: 4 up/gate pairs)
constexpr int kNT = 2;      // tokens per pass over a chunk

struct StreamParams {
  const uint8_t *w;          // packed e2m1 rows [E * rows, K / 2]
  const uint8_t *sc;         // E8M0 [E * rows, K / 32]
  const uint16_t *src;       // up: tokens [T, K] bf16; down: h [S, K] bf16 in slot order
  const int32_t *offsets;    // [E + 1] first slot of each expert
  const int32_t *perm;       // [S] slot -> flat assignment t * kk + j
  const int32_t *active;     // active expert ids, ascending
  const int32_t *counters;   // [0] active experts, [1] error flag (an expert id out of range)
  int kk;                    // slots per token
  int K;                     // row length (values)
  int rows;                  // weight rows per expert (up: 2 I, down: H)
  int I;
  int up_base, gate_base;    // up projection: first up row, first gate row
  float limit;
  int stage_rows;            // rows the shared-memory operand buffer holds
  int ring_offset;           // shared-memory offset of the warps' copy rings
  wm::RoutePlan plan;        // up projection: plan.idx set -> group the assignments in-kernel
  wm::CombineArgs comb;      // down projection: with `done` set, the last CTA combines the rows
  int32_t *done;
  uint16_t *out;             // up: h [S, I]; down: y [S, H] (bf16, slot order)
  int row_chunks;            // MODE 2: 8-row chunks of every active expert per CTA
  int y_offset;              // MODE 2: shared-memory offset of the CTA's y rows [S][row_chunks * 8] (bf16)
};

// Each warp streams its weight pieces through a ring of kDepth stages in
// shared memory (cp.async: the bytes in flight are not held in registers);
// a stage holds every lane's piece of the chunk's 4 rows and the rows' E8M0
// bytes of the step (8-byte copies by the first 16 lanes).
constexpr int kDepth = 3;
template <int PB>
struct Ring {
  static constexpr int kW = kRows * 32 * PB;      // weight bytes per stage
  static constexpr int kS = kRows * 32;           // scale bytes per stage (2 PB per row used)
  static constexpr int kStage = kW + kS;
  static constexpr int kWarpBytes = kDepth * kStage;
};

constexpr int kMaxCtaExperts = 32;
constexpr int kRowChunksMax = 8;     // MODE 2: 8-row chunks per CTA (H <= 9472 on 148 SMs)   // experts one CTA's chunk range can span: at most E / grid + 2

template <int MODE, int PB>
__device__ __forceinline__ void stream_body(const StreamParams &p) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ int m_e[kMaxCtaExperts], m_p0[kMaxCtaExperts], m_n[kMaxCtaExperts];
  __shared__ wm::SmallRoute<wm::kStreamRouteMax> route;
  __shared__ int32_t route_key[wm::kStreamRouteMax];
  __shared__ float comb_w[wm::kStreamRouteMax];   // MODE 2: the weight of flat assignment t * kk + j
  constexpr int VPP = 2 * PB;                 // values per piece
  // MODE 2 reads only what was complete before the previous launch started (the routing, the weights)
  // until its copies are in flight, then waits for that launch (the up projection's h)
  if (MODE != 2) {
    WM_PDL_WAIT();
    WM_PDL_LAUNCH();
  }
  const int K = p.K, G = K / 32;
  // up projection: this thread's first 32-value group of the token rows is loaded now, so that its latency
  // overlaps the grouping below (the rows do not depend on it)
  uint4 pre[4];
  if (MODE == 0 && static_cast<int>(threadIdx.x) < p.stage_rows * G) {
    const uint4 *s = reinterpret_cast<const uint4 *>(p.src + static_cast<int64_t>(threadIdx.x / G) * K +
                                                     (threadIdx.x % G) * 32);
#pragma unroll
    for (int i = 0; i < 4; ++i) pre[i] = __ldcg(s + i);
  }
  if (MODE == 2)                              // the combine's weights (inputs of the call, complete before it)
    for (int a = threadIdx.x; a < p.comb.T * p.comb.kk; a += kThreads) {
      const int t = a / p.comb.kk, j = a - t * p.comb.kk;
      comb_w[a] = j < p.comb.k ? p.comb.w[static_cast<int64_t>(t) * p.comb.k + j]
                               : (p.comb.shared_w ? p.comb.shared_w[t] : 1.0f);
    }
  // small calls: group the assignments here (every CTA); in the up projection CTA 0 writes the grouping
  const bool in_kernel = (MODE == 0 || MODE == 2) && p.plan.idx != nullptr;
  int n_active;
  if (in_kernel) {
    wm::small_route(p.plan.idx, p.plan.T, p.plan.k, p.plan.shared_expert, p.plan.E, route, route_key);
    if (MODE == 0 && blockIdx.x == 0)
      wm::publish_route(route, p.plan.T, p.plan.k, p.plan.shared_expert, p.plan.E, p.plan.offsets, p.plan.perm,
                        p.plan.inv, p.plan.active, p.plan.counters, nullptr, 0, p.plan.done);
    if (MODE == 0 && route.bad) return;       // bad expert id: the combine writes zeros
    n_active = route.bad ? 0 : route.n_act;
  } else {
    if (p.counters[1] != 0) return;
    n_active = p.counters[0];
  }
  const int cpe = p.rows / kRows;
  // the CTA's chunks: MODE 0 / 1 a contiguous share of all (expert, row chunk) pairs; MODE 2 the row chunks
  // [mb, mb + lc) of every active expert, so the CTA holds every slot's rows there and combines them itself
  // chunk indices fit 32 bits (at most 4096 experts x 1024 chunks), and 32-bit divisions are a few
  // instructions where 64-bit ones are a subroutine
  int c0, c1;
  int lc = cpe, mb = 0;
  if (MODE == 2) {
    mb = blockIdx.x * p.row_chunks;
    lc = max(0, min(p.row_chunks, cpe - mb));
    c0 = 0;
    c1 = n_active * lc;
  } else {
    const int n_chunks = n_active * cpe;
    c0 = n_chunks * blockIdx.x / gridDim.x;
    c1 = n_chunks * (blockIdx.x + 1) / gridDim.x;
    if (c0 >= c1) return;
  }
  const int a_first = MODE == 2 ? 0 : c0 / cpe;
  const int a_last = MODE == 2 ? n_active - 1 : (c1 - 1) / cpe;

  // ------------------------------ the CTA's experts
  if (!in_kernel) {
    for (int i = threadIdx.x; i <= a_last - a_first && i < kMaxCtaExperts; i += kThreads) {
      const int e = p.active[a_first + i];
      const int o = p.offsets[e];
      m_e[i] = e; m_p0[i] = o; m_n[i] = p.offsets[e + 1] - o;
    }
    __syncthreads();                          // the warps' copies below read them
  }
  int p_lo = 0, p_hi = 0;
  if (MODE != 2) {
    p_lo = in_kernel ? route.act_p0[a_first] : p.offsets[p.active[a_first]];
    p_hi = in_kernel ? route.act_p0[a_last] + route.act_n[a_last] : p.offsets[p.active[a_last] + 1];
  }
  int base_row = 0, n_rows;
  if (MODE != 1) {
    n_rows = p.stage_rows;                    // every token (up) or every slot (MODE 2) of the call
  } else {
    base_row = p_lo;                          // the slots of the CTA's experts
    n_rows = p_hi - p_lo;
  }
  uint16_t *xs = reinterpret_cast<uint16_t *>(smem);                                        // [n_rows][K]
  float *xk = reinterpret_cast<float *>(smem + static_cast<size_t>(p.stage_rows) * K * 2);  // [n_rows][G]
  int *tok = reinterpret_cast<int *>(xk + static_cast<size_t>(p.stage_rows) * G);           // up: slot -> token
  const int rows_cta = p.row_chunks * kRows;
  uint16_t *ysm = reinterpret_cast<uint16_t *>(smem + p.y_offset);                            // MODE 2: [S][rows_cta]
  // operand rows -> f16 with a power-of-two scale per 32 values (all threads; run after the first weight
  // copies are issued, so the two latencies overlap)
  auto stage_operands = [&]() {
  if (MODE == 0)
    for (int i = threadIdx.x; i < p_hi - p_lo; i += kThreads)
      tok[i] = (in_kernel ? route.perm[p_lo + i] : p.perm[p_lo + i]) / p.kk;
  for (int g = threadIdx.x; g < n_rows * G; g += kThreads) {
    const int r = g / G, q = g - r * G;
    const uint4 *s = reinterpret_cast<const uint4 *>(p.src + static_cast<int64_t>(base_row + r) * K + q * 32);
    uint4 v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = (MODE == 0 && g == static_cast<int>(threadIdx.x)) ? pre[i] : __ldcg(s + i);
    xk[r * G + q] = stage_group_f16(v, reinterpret_cast<uint4 *>(xs + static_cast<int64_t>(r) * K + q * 32));
  }
  };

  // ------------------------------------------------------------ stream
  // Each warp walks its chunks as one stream of (chunk, pass, step) with the
  // loads one step ahead of the arithmetic, across chunk boundaries too.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nc = c1 - c0;
  const int w0 = c0 + nc * warp / kWarps, w1 = c0 + nc * (warp + 1) / kWarps;
  const bool has_work = w0 < w1;
  const int pieces = K / VPP;
  const int steps = (pieces + 31) / 32;
  const int64_t row_bytes = K / 2;
  const int rstep = MODE == 0 ? 1 : 2;        // row distance between rows r and r + 2
  const uint64_t pol = wm_tc::l2_evict_first_policy();
  auto meta = [&](int a, int &e, int &p0, int &n) {
    const int i = a - a_first;
    if (in_kernel) {
      e = route.act_e[a]; p0 = route.act_p0[a]; n = route.act_n[a];
    } else if (i < kMaxCtaExperts) {
      e = m_e[i]; p0 = m_p0[i]; n = m_n[i];
    } else {
      e = p.active[a]; p0 = p.offsets[e]; n = p.offsets[e + 1] - p0;
    }
  };
  // first weight rows of chunk m (r = 0, 1); row r is row r & 1 plus (r >> 1) * rstep
  auto first_rows = [&](int m, int &r0, int &r1) {
    if (MODE == 0) { r0 = p.up_base + (kRows / 2) * m; r1 = p.gate_base + (kRows / 2) * m; }
    else { r0 = kRows * m; r1 = kRows * m + 1; }
  };
  struct Cursor {
    int c;            // chunk
    int a, m;         // active expert, chunk within it
    int t0, s;        // first slot of the pass, step
    int n;            // slots of the expert
  };
  auto start = [&](Cursor &u) {
    u.c = w0; u.a = w0 / lc; u.m = mb + (w0 - u.a * lc);
    u.t0 = 0; u.s = 0;
    int e, p0;
    meta(u.a, e, p0, u.n);
  };
  auto advance = [&](Cursor &u) {
    if (++u.s < steps) return;
    u.s = 0;
    u.t0 += kNT;
    if (u.t0 < u.n) return;
    u.t0 = 0;
    ++u.c;
    if (++u.m == mb + lc) {
      u.m = mb;
      ++u.a;
    }
    if (u.c < w1) {
      int e, p0;
      meta(u.a, e, p0, u.n);
    }
  };

  // ---- copies (cursor L, kDepth - 1 steps ahead)
  using RG = Ring<PB>;
  constexpr int kGps = 2 * PB;                // scale groups per step
  uint8_t *ring = smem + p.ring_offset + static_cast<size_t>(warp) * RG::kWarpBytes;
  const uint32_t ring_s = static_cast<uint32_t>(__cvta_generic_to_shared(ring));
  Cursor L{};
  if (has_work) start(L);
  const uint8_t *wb0 = nullptr, *wb1 = nullptr, *sb0 = nullptr, *sb1 = nullptr;
  int l_chunk = -1;
  auto issue = [&](int slot) {
    if (L.c < w1) {
      if (L.c != l_chunk) {
        l_chunk = L.c;
        int e, p0, n, r0, r1;
        meta(L.a, e, p0, n);
        first_rows(L.m, r0, r1);
        const int64_t e_row = static_cast<int64_t>(e) * p.rows;
        wb0 = p.w + (e_row + r0) * row_bytes; wb1 = p.w + (e_row + r1) * row_bytes;
        sb0 = p.sc + (e_row + r0) * G; sb1 = p.sc + (e_row + r1) * G;
      }
      const int q = lane + 32 * L.s;
      const uint32_t st = ring_s + slot * RG::kStage;
      if (q < pieces) {
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
          const uint8_t *wr = ((r & 1) ? wb1 : wb0) + static_cast<int64_t>((r >> 1) * rstep) * row_bytes;
          if (PB == 16) cp_async16(st + r * 32 * PB + lane * PB, wr + q * PB, pol);
          else cp_async8(st + r * 32 * PB + lane * PB, wr + q * PB, pol);
        }
      }
      if (lane < 4 * kRows) {                 // row r = lane / 4, bytes [8 j, 8 j + 8) of the step's groups
        const int r = lane >> 2, j = lane & 3;
        const int g0 = L.s * kGps + 8 * j;
        if (8 * j < kGps && g0 < G) {
          const uint8_t *sr = ((r & 1) ? sb1 : sb0) + static_cast<int64_t>((r >> 1) * rstep) * G;
          cp_async8(st + RG::kW + r * 32 + 8 * j, sr + g0, pol);
        }
      }
      advance(L);
    }
    cp_async_commit();
  };

  // ---- arithmetic (cursor C) and the per-pass epilogue
  Cursor C{};
  if (has_work) start(C);
  int c_p0 = 0, nt = 1;
  int xr[kNT];
  float acc[kRows][kNT];
  auto begin_pass = [&]() {
    int e, n;
    meta(C.a, e, c_p0, n);
    nt = min(kNT, n - C.t0);
#pragma unroll
    for (int t = 0; t < kNT; ++t) {
      const int pp = c_p0 + C.t0 + min(t, nt - 1);
      xr[t] = MODE == 0 ? tok[pp - p_lo] : pp - base_row;
    }
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int t = 0; t < kNT; ++t) acc[r][t] = 0.0f;
  };
  auto compute = [&](int slot, auto ntok_c) {
    constexpr int NTOK = decltype(ntok_c)::value;
    const int q = lane + 32 * C.s;
    if (q >= pieces) return;
    const int grp = (q * VPP) / 32;
    const uint8_t *st = ring + slot * RG::kStage;
    uint32_t xv[NTOK][PB];
    float xsc[NTOK];
#pragma unroll
    for (int t = 0; t < NTOK; ++t) {
      const uint4 *src = reinterpret_cast<const uint4 *>(xs + static_cast<int64_t>(xr[t]) * K + q * VPP);
#pragma unroll
      for (int i = 0; i < PB / 4; ++i) {
        const uint4 u = src[i];
        xv[t][4 * i] = u.x; xv[t][4 * i + 1] = u.y; xv[t][4 * i + 2] = u.z; xv[t][4 * i + 3] = u.w;
      }
      xsc[t] = xk[xr[t] * G + grp];
    }
    // two rows at a time: four independent f32 chains per token (each row's
    // lo and hi chains keep their own order)
#pragma unroll
    for (int r = 0; r < kRows; r += 2) {
      uint32_t h[2][PB];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        uint32_t wv[PB / 4];
        if constexpr (PB == 16) {
          const uint4 v = *reinterpret_cast<const uint4 *>(st + (r + u) * 32 * PB + lane * PB);
          wv[0] = v.x; wv[1] = v.y; wv[2] = v.z; wv[3] = v.w;
        } else {
          const uint2 v = *reinterpret_cast<const uint2 *>(st + (r + u) * 32 * PB + lane * PB);
          wv[0] = v.x; wv[1] = v.y;
        }
#pragma unroll
        for (int i = 0; i < PB / 4; ++i) {
          uint32_t hh[4];
          e2m1x8_to_f16x2(wv[i], hh);
          h[u][4 * i] = hh[0]; h[u][4 * i + 1] = hh[1]; h[u][4 * i + 2] = hh[2]; h[u][4 * i + 3] = hh[3];
        }
      }
      const float sw0 = wm_e8m0(st[RG::kW + r * 32 + grp - C.s * kGps]);
      const float sw1 = wm_e8m0(st[RG::kW + (r + 1) * 32 + grp - C.s * kGps]);
#pragma unroll
      for (int t = 0; t < NTOK; ++t) {
        float lo0 = 0.0f, hi0 = 0.0f, lo1 = 0.0f, hi1 = 0.0f;
#pragma unroll
        for (int i = 0; i < PB; ++i) {
          fma_f16x2_f32(h[0][i], xv[t][i], lo0, hi0);
          fma_f16x2_f32(h[1][i], xv[t][i], lo1, hi1);
        }
        acc[r][t] = fmaf((lo0 + hi0) * xsc[t], sw0, acc[r][t]);
        acc[r + 1][t] = fmaf((lo1 + hi1) * xsc[t], sw1, acc[r + 1][t]);
      }
    }
  };
  // warp sums, then the epilogue: value r * NTOK + t is (row r, token t)
  auto epilogue = [&](auto ntok_c) {
    constexpr int NTOK = decltype(ntok_c)::value;
    constexpr int V = kRows * NTOK;
    constexpr int kShift = V == 16 ? 1 : V == 8 ? 2 : 3;   // lane bits below the value index
    float v[V];
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int t = 0; t < NTOK; ++t) v[r * NTOK + t] = acc[r][t];
    const float sum = warp_sums<V>(v, lane);
    const int vi = (lane >> kShift) & (V - 1);
    const int r = vi / NTOK, t = vi - r * NTOK;
    const bool writer = (lane & ((1 << kShift) - 1)) == 0;
    const int64_t slot = c_p0 + C.t0 + t;
    if (MODE == 0) {
      // rows (up, gate, up, gate, ...): the gate sum of row r is value r + 1, 32 / kRows lanes over
      const float gate_sum = __shfl_xor_sync(0xffffffffu, sum, 32 / kRows);
      if (writer && (r & 1) == 0) {
        float up = sum, gate = gate_sum;
        if (p.limit > 0.0f) {
          up = fminf(fmaxf(up, -p.limit), p.limit);
          gate = fminf(gate, p.limit);
        }
        const float silu = gate / (1.0f + expf(-gate));
        p.out[slot * p.I + (kRows / 2) * C.m + (r >> 1)] = wm_f32_to_bf16(silu * up);
      }
    } else if (MODE == 2) {
      if (writer) ysm[slot * rows_cta + kRows * (C.m - mb) + r] = wm_f32_to_bf16(sum);
    } else if (writer) {
      p.out[slot * p.rows + kRows * C.m + r] = wm_f32_to_bf16(sum);
    }
  };
  // one step of cursor C on piece b; false once the warp's chunks are done
  auto step = [&](int slot) -> bool {
    if (nt == 1) compute(slot, std::integral_constant<int, 1>{});
    else compute(slot, std::integral_constant<int, 2>{});
    if (C.s == steps - 1) {
      if (nt == 1) epilogue(std::integral_constant<int, 1>{});
      else epilogue(std::integral_constant<int, 2>{});
    }
    advance(C);
    if (C.c >= w1) return false;
    if (C.s == 0) begin_pass();
    return true;
  };

  if (has_work)
    for (int i = 0; i < kDepth - 1; ++i) issue(i);
  if (MODE == 2) {
    WM_PDL_WAIT();                            // h of the up projection from here on
    WM_PDL_LAUNCH();
  }
  stage_operands();
  __syncthreads();
  if (MODE != 2 && !has_work) return;
  if (has_work) {
    begin_pass();
    for (int use = 0, fill = kDepth - 1;;) {
      issue(fill);                            // the slot the previous step used
      cp_async_wait<kDepth - 1>();            // this lane's copies of this step have landed
      __syncwarp();                           // and every lane's (the scale bytes)
      const bool more = step(use);
      __syncwarp();                           // the slot is read before a later step refills it
      if (!more) break;
      fill = use;
      use = use + 1 == kDepth ? 0 : use + 1;
    }
    cp_async_wait<0>();
  }
  if constexpr (MODE == 2) {
    // the combine of rows [8 mb, 8 (mb + lc)): out[t, h] = sum_j w[t, j] * y[slot(t, j), h] (+ the shared
    // expert's row times its weight), f32 fmaf chain in assignment order j, rounded once -- the arithmetic
    // of wm::combine_groups, on the CTA's own y rows
    __syncthreads();
    const wm::CombineArgs &a = p.comb;
    const int S = a.T * a.kk;
    const bool bad = route.bad != 0;
    for (int i = threadIdx.x; i < a.T * lc; i += kThreads) {
      const int t = i / lc, q = i - t * lc;   // rows 8 (mb + q) .. + 7 of token t
      float acc[kRows] = {0, 0, 0, 0, 0, 0, 0, 0};
      // eight assignments at a time: their slots, weights and rows loaded together, then the chain
      for (int j0 = 0; j0 < a.kk && !bad; j0 += 8) {
        int sl[8];
        float wv[8];
        uint4 y[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int j = j0 + u;
          sl[u] = j < a.kk ? route.inv[t * a.kk + j] : -1;
          wv[u] = j < a.kk ? comb_w[t * a.kk + j] : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
          y[u] = (sl[u] >= 0 && sl[u] < S) ? *reinterpret_cast<const uint4 *>(ysm + sl[u] * rows_cta + kRows * q)
                                           : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (sl[u] < 0 || sl[u] >= S) continue;
          acc[0] = fmaf(wv[u], wm_bf16lo(y[u].x), acc[0]); acc[1] = fmaf(wv[u], wm_bf16hi(y[u].x), acc[1]);
          acc[2] = fmaf(wv[u], wm_bf16lo(y[u].y), acc[2]); acc[3] = fmaf(wv[u], wm_bf16hi(y[u].y), acc[3]);
          acc[4] = fmaf(wv[u], wm_bf16lo(y[u].z), acc[4]); acc[5] = fmaf(wv[u], wm_bf16hi(y[u].z), acc[5]);
          acc[6] = fmaf(wv[u], wm_bf16lo(y[u].w), acc[6]); acc[7] = fmaf(wv[u], wm_bf16hi(y[u].w), acc[7]);
        }
      }
      const int64_t o = static_cast<int64_t>(t) * a.H + kRows * (mb + q);
      if (a.f32_out) {
        float4 *op = reinterpret_cast<float4 *>(static_cast<float *>(a.out) + o);
        op[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        op[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
      } else {
        uint4 ob;
        ob.x = wm_f32_to_bf16(acc[0]) | (static_cast<uint32_t>(wm_f32_to_bf16(acc[1])) << 16);
        ob.y = wm_f32_to_bf16(acc[2]) | (static_cast<uint32_t>(wm_f32_to_bf16(acc[3])) << 16);
        ob.z = wm_f32_to_bf16(acc[4]) | (static_cast<uint32_t>(wm_f32_to_bf16(acc[5])) << 16);
        ob.w = wm_f32_to_bf16(acc[6]) | (static_cast<uint32_t>(wm_f32_to_bf16(acc[7])) << 16);
        *reinterpret_cast<uint4 *>(static_cast<uint16_t *>(a.out) + o) = ob;
      }
    }
  }
}

// The body may return early (CTAs or warps without chunks); the down
// projection of a small call then combines the call's rows in its last CTA.
template <int MODE, int PB>
__global__ void __launch_bounds__(kThreads, 1) k_expert_stream(const __grid_constant__ StreamParams p) {
  stream_body<MODE, PB>(p);
  if (MODE == 1 && p.done) wm::combine_if_last(p.comb, p.done);
}

// operand rows (f16 + one f32 scale per 32 values) and, for the up projection, a token index per slot
size_t stage_bytes(int rows, int K, int slots = 0) {
  return static_cast<size_t>(rows) * K * 2 + static_cast<size_t>(rows) * (K / 32) * 4 + static_cast<size_t>(slots) * 4;
}

// shared memory of a launch over rows of K values: the staged operand rows, then the copy rings
size_t launch_smem(size_t stage, int K, size_t *ring_offset) {
  *ring_offset = (stage + 15) / 16 * 16;
  const size_t ring = static_cast<size_t>(kWarps) * (K >= 1024 ? Ring<16>::kWarpBytes : Ring<8>::kWarpBytes);
  return *ring_offset + ring;
}

template <int MODE, int PB>
cudaError_t launch_one(const StreamParams &p, size_t smem, cudaStream_t stream, int grid = 0) {
  // the attribute is per function and device: set once per template instance on each device
  static std::mutex mu;
  static bool attr_done[64] = {false};
  int dev = 0;
  if (cudaError_t e = cudaGetDevice(&dev)) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!attr_done[dev]) {
      cudaError_t e = cudaFuncSetAttribute(k_expert_stream<MODE, PB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(wm::kStreamSmemMax));
      if (e != cudaSuccess) return e;
      attr_done[dev] = true;
    }
  }
  return wm::launch_pdl(k_expert_stream<MODE, PB>, dim3(grid > 0 ? grid : wm::sm_count()), dim3(kThreads), smem,
                        stream, p);
}

}  // namespace

namespace wm {

bool stream_supported(int T, int k, int has_shared, int H, int I) {
  const int S = T * (k + has_shared);
  size_t o;
  return T >= 1 && H % 256 == 0 && I % 256 == 0 && launch_smem(stage_bytes(T, H, S), H, &o) <= kStreamSmemMax &&
         launch_smem(stage_bytes(S, I), I, &o) <= kStreamSmemMax;
}

int stream_row_chunks(int H) {
  const int cpe = H / kRows, nsm = sm_count();
  return (cpe + nsm - 1) / nsm;
}

bool stream_row_split(int S, int H, int I) {
  size_t o;
  const int rc = stream_row_chunks(H);
  return S <= kStreamRouteMax && rc <= kRowChunksMax &&
         launch_smem(stage_bytes(S, I), I, &o) + 16 + static_cast<size_t>(S) * rc * kRows * 2 <= kStreamSmemMax;
}

int launch_stream_up(const uint8_t *w13, const uint8_t *s13, int T, int kk, int H, int I, int order, float limit,
                     const uint16_t *x, const int32_t *offsets, const int32_t *perm, const int32_t *active,
                     const int32_t *counters, uint16_t *h, cudaStream_t stream, const RoutePlan &plan) {
  StreamParams p{};
  p.plan = plan;
  p.w = w13; p.sc = s13; p.src = x; p.offsets = offsets; p.perm = perm; p.active = active; p.counters = counters;
  p.kk = kk; p.K = H; p.rows = 2 * I; p.I = I;
  p.up_base = order == WM_UP_GATE ? 0 : I;
  p.gate_base = order == WM_UP_GATE ? I : 0;
  p.limit = limit; p.stage_rows = T; p.out = h;
  size_t ring_offset;
  const size_t smem = launch_smem(stage_bytes(T, H, T * kk), H, &ring_offset);
  p.ring_offset = static_cast<int>(ring_offset);
  cudaError_t e = H >= 1024 ? launch_one<0, 16>(p, smem, stream) : launch_one<0, 8>(p, smem, stream);
  if (e != cudaSuccess) return fail(WM_ERR_CUDA, std::string("expert stream up: ") + cudaGetErrorString(e));
  return check_launch("expert stream up");
}

int launch_stream_down(const uint8_t *w2, const uint8_t *s2, int S, int H, int I, const uint16_t *h,
                       const int32_t *offsets, const int32_t *active, const int32_t *counters, uint16_t *y,
                       cudaStream_t stream, const CombineArgs *comb, int32_t *done, const RoutePlan *plan) {
  StreamParams p{};
  const bool rows = plan && plan->idx && comb;
  if (rows) {
    p.plan = *plan;
    p.comb = *comb;
  } else if (comb && done) {
    p.comb = *comb;
    p.done = done;
  }
  p.w = w2; p.sc = s2; p.src = h; p.offsets = offsets; p.active = active; p.counters = counters;
  p.kk = 1; p.K = I; p.rows = H; p.I = I; p.stage_rows = S; p.out = y;
  size_t ring_offset;
  size_t smem = launch_smem(stage_bytes(S, I), I, &ring_offset);
  p.ring_offset = static_cast<int>(ring_offset);
  cudaError_t e;
  if (rows) {
    // row chunks per CTA: the fewest that cover H / 8 chunks with at most one CTA per SM
    if (!stream_row_split(S, H, I)) return fail(WM_ERR_INVALID, "expert stream down: no row split for this shape");
    const int cpe = H / kRows;
    p.row_chunks = stream_row_chunks(H);
    const int grid = (cpe + p.row_chunks - 1) / p.row_chunks;
    p.y_offset = static_cast<int>((smem + 15) / 16 * 16);
    smem = p.y_offset + static_cast<size_t>(S) * p.row_chunks * kRows * 2;
    e = I >= 1024 ? launch_one<2, 16>(p, smem, stream, grid) : launch_one<2, 8>(p, smem, stream, grid);
  } else {
    e = I >= 1024 ? launch_one<1, 16>(p, smem, stream) : launch_one<1, 8>(p, smem, stream);
  }
  if (e != cudaSuccess) return fail(WM_ERR_CUDA, std::string("expert stream down: ") + cudaGetErrorString(e));
  return check_launch("expert stream down");
}

}  // namespace wm
