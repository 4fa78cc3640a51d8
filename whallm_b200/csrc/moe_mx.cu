// Grouped MXFP4 expert GEMM on block-scaled tcgen05 tensor cores.
//
// Reference: the MLX gather_qmm / quantized_matmul expert math
// (model.py:393-481, qwen4_exp.py:588-678): y = x @ dequant(W)^T per routed
// (token, expert) pair, W in MXFP4 (e2m1 + E8M0 per 32 along K).
//
// The weights go to the tensor core as they are stored: TMA expands each
// 128-value e2m1 row segment into the padded shared-memory form the MMA reads
// (CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B) and the MXFP4 E8M0 bytes become the
// MMA's A scale factors, so nothing dequantizes the weights in software.
//
//   tcgen05.mma.kind::mxf8f6f4.block_scale  D[f32, TMEM] += (A * sa) x (B * sb)
//   A  e2m1 weights, 128 rows x 32 K per instruction, scale sa per 32 K (the
//      weight's own E8M0 byte)
//   B  the tokens as two e4m3 terms, x = sb_hi * hi + sb_hi * 2^-5 * lo, with
//      one E8M0 scale per (token, 32 K) chosen so the block maximum lands in
//      [128, 256).  For bf16 inputs the two terms are exact for every element
//      within 2^-14 of its block maximum (8 significant bits = 4 + 4) and off
//      by at most 2^-22 of the block maximum below that, so the product is the
//      bf16 x MXFP4 product of the reference up to f32 accumulation order.
//      The terms are stacked along N (hi rows [0, n16), lo rows [n16, 2 n16),
//      n16 = tokens rounded up to 16, each row with its own scale), so one
//      MMA per K-block reads the weight tile once and D = [D_hi | D_lo]; the
//      epilogue adds the halves.  Shared-memory traffic, not the tensor core,
//      bounds a skinny MMA: the padded e2m1 tile is 4 KB per 32 K, read once.
//
// Orientation ("swap AB"): M = 128 weight rows, N = the tokens routed to one
// expert (16..NMAX per tile), K = reduction.  The up projection's 128 rows
// are 64 up and 64 gate rows interleaved in groups of 8 by a 4-D tensor map,
// so lanes m and m ^ 8 of one warp hold up_j and gate_j for the fused
// ClampedSwiGLU epilogue, which rounds h to bf16 and (decode configuration)
// writes its two e4m3 terms and scales, the down projection's token operand,
// directly; the prefill configuration writes bf16 h for a split kernel.
//
// Warp roles (384 threads for decode, 768 for prefill; one CTA per SM,
// persistent over (tile, 128-row) work items):
//   warp 0      TMA producer (weights, token terms)
//   warp 1      MMA issuer: tcgen05.cp of the stage's scale factors into
//               TMEM, then KC/32 MMAs (the copies and the MMAs of one thread
//               execute in issue order)
//   warp 2      TMEM allocator
//   warps 4-7   scale warps: they read the rows' E8M0 bytes from global
//               memory a chunk (up to 32 bytes per row) ahead and write each
//               stage's bytes in the 32 x 16-byte layout that
//               tcgen05.cp.32x128b.warpx4 takes
//   warps 8-11  epilogue (TMEM lanes 0-127); prefill adds warps 12-23, four
//               epilogue groups in all, taking a work item's 16-token chunks
//               in turn
// Every mbarrier wait is bounded and records an error code instead of hanging.
#include "wm_common.cuh"
#include "wm_combine.cuh"
#include "wm_moe.cuh"
#include "wm_route.cuh"
#include "wm_tc.cuh"

namespace {

using namespace wm_tc;

constexpr int kM = 128;
constexpr int kKH = 128;                 // K values per TMA box row and per scale-factor group
constexpr int kLoShift = 5;              // lo term scale = hi scale * 2^-5
constexpr uint32_t kLoSub = 0x01010101u * kLoShift;   // E8M0 bytes of the lo term, four at a time

template <int KC, int NMAX, int STAGES, bool FUSE_SPLIT, int EPI = 1, bool PAIR = false>
struct MxCfg {
  // PAIR: a cluster of two CTAs on two SMs runs each work item as one
  // cta_group::2 MMA of M = 256 weight rows: CTA r holds rows [128 r, 128 r +
  // 128) of A and one token term of B (r = 0: hi rows, r = 1: lo rows), so a
  // CTA stages half the token tile and the stage count grows; CTA 0 issues
  // the MMAs into both CTAs' tensor memory.
  static constexpr bool kPair = PAIR;
  // EPI: epilogue warp groups (4 warps each, one per TMEM lane quadrant);
  // the groups take 16-token chunks of a work item in turn, for short-K items
  // whose epilogue would otherwise outlast their mainloop (prefill: 4 groups,
  // 768 threads; Qwen-class prefill 2.86M -> 3.53M tok/s).
  static constexpr int kEpi = EPI;
  static constexpr int kThreads = 256 + 128 * EPI;
  // FUSE_SPLIT: the up projection's epilogue writes the e4m3 terms of h
  // (decode: at most two 16-column chunks per item, hidden behind the
  // mainloop); otherwise it writes bf16 h and a split kernel follows.
  static constexpr bool kFuseSplit = FUSE_SPLIT;
  static constexpr int kKC = KC;
  static constexpr int kNMax = NMAX;
  static constexpr int kStages = STAGES;
  static constexpr int kHalves = KC / kKH;                   // 128-K groups per stage
  static constexpr int kABox = kM * kKH;                     // 16 KB: 128 rows x 128 padded bytes
  static constexpr int kAStage = kHalves * kABox;
  static constexpr int kBBox = (PAIR ? 1 : 2) * NMAX * kKH;  // hi + lo rows (a pair CTA: its term) x 128 B, one K group
  static constexpr int kBStage = kHalves * kBBox;
  static constexpr int kBAtoms = (2 * NMAX + 127) / 128;     // 128-row scale atoms of B per K group
  static constexpr int kSFStage = (((1 + kBAtoms) * kHalves * 512 + 1023) / 1024) * 1024;  // A and B atoms
  static constexpr int kDCols = 2 * NMAX;                    // one accumulator: [D_hi | D_lo]
  static constexpr int kSfCol0 = 2 * kDCols;                 // after the two accumulators
  static constexpr int kSfbCols = 4 * kBAtoms;               // TMEM columns of B scales per K group
  static constexpr int kSfCols = kHalves * (4 + kSfbCols);
  static constexpr int kColsUsed = kSfCol0 + kSfCols;
  static constexpr int kTmemCols = kColsUsed <= 32 ? 32 : kColsUsed <= 64 ? 64 : kColsUsed <= 128 ? 128
                                 : kColsUsed <= 256 ? 256 : 512;
  static constexpr size_t kSmem =
      1024 + static_cast<size_t>(STAGES) * (kAStage + kBStage + kSFStage) + (3 * STAGES + 6 + 4 * EPI) * 8 + 16;
  static_assert(KC % kKH == 0, "stage depth must be a multiple of 128");
  static_assert(NMAX % 16 == 0 && 2 * NMAX <= 256, "tile width: MMA N = 2 x tokens <= 256");
  static_assert(kBBox % 1024 == 0, "B boxes must stay 1024-aligned");
  static_assert(kSmem <= 232448, "shared memory");
  static_assert(kColsUsed <= 512, "TMEM columns");
  static_assert(EPI >= 1 && EPI <= 4 && (EPI <= 2 || !FUSE_SPLIT),
                "1-4 epilogue groups; the fused split's column-max exchange buffers are for two");
  static_assert(!PAIR || !FUSE_SPLIT, "the CTA pair runs the prefill configuration (bf16 h, separate split)");
};
using MxDecode = MxCfg<256, 32, 4, true>;
// A decode up projection whose tiles can hold more than 16 tokens (T > 16: the
// shared expert's tile holds every token) has two epilogue groups, so a
// 32-token tile's two 16-token chunks (ClampedSwiGLU, the e4m3 split of h) run
// side by side and a short-K item (Qwen-class: K = 2048, 8 stages) is not held
// up by its epilogue (Qwen-class B = 32 expert call 59.5 -> 56.5 us).  With at
// most 16 tokens per tile the second group would idle (DeepSeek-class B = 1:
// 63.2 -> 64.9 us), so smaller batches keep one.
using MxDecodeUp = MxCfg<256, 32, 4, true, 2>;
using MxPrefill = MxCfg<128, 112, 4, false, 4>;
// The prefill configuration on CTA pairs: 32 KB stages (16 KB weights, 14 KB
// of one token term, scale atoms), six of them.  Opt-in (WM_MX_PAIR=1): it
// matches the single-CTA results within the tolerance but measured 2.2x
// slower on the 4096-token DeepSeek-class layer (9.1 vs 4.1 ms): per-stage
// stamps show the stage period doubling (0.45 -> 0.9 us) with ~4.4 us from a
// stage's copy issue to its ready barrier, unchanged by the wait mode, the
// stage count, the epilogue width or removing the MMAs altogether.
using MxPrefillPair = MxCfg<128, 112, 6, false, 4, true>;

struct MxParams {
  int mode;                  // 0: up projection (+ClampedSwiGLU -> h bf16), 1: down projection (-> y f32)
  int K;                     // reduction length
  int rows;                  // weight rows per expert
  int I, H;
  int order;                 // WM_UP_GATE / WM_GATE_UP
  float limit;
  int m_tiles;               // work items per tile: 128-row blocks x k_splits
  int k_splits;              // K ranges per 128-row block (down form only); > 1: f32 partial sums to y_part
  int a_fp8;                 // A operand e4m3 (MXFP8: one byte per value) instead of e2m1
  const uint8_t *a_scales;   // [E * rows, K/32] E8M0 (the MXFP4 scales)
  const uint8_t *b_scales;   // [S_pad, K/32] hi-term E8M0 in slot order
  const int4 *tiles;         // {expert, first slot, tokens, 0}
  const int32_t *n_tiles;
  uint8_t *h_hi, *h_lo;     // up, fused split: [S_pad, I] e4m3 terms of the bf16 SwiGLU output
  uint8_t *h_sc;             // up, fused split: [S_pad, I/32] E8M0 scale of h_hi
  uint16_t *h_out;           // up, separate split: [S_pad, I] bf16
  uint16_t *y_out;           // down: [S, H] bf16
  float *y_part;             // down, k_splits > 1: [k_splits][part_stride] f32, summed by k_sum_splits
  int64_t part_stride;
  // Dense tiles (score and linear launches): d_tiles > 0 tiles computed from
  // their index instead of read from `tiles`: tile i = {b, b * d_lq + j * d_nmax,
  // min(d_nmax, d_lq - j * d_nmax)} for b = i / d_per, j = i % d_per.
  int d_tiles, d_per, d_lq, d_nmax;
  int32_t *err;
  // down projection of a small call: with done set, the last CTA to finish combines the rows
  wm::CombineArgs comb;
  int32_t *done;
};

__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, int x, int y, int z, int w,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_4d_hint(void *dst, const CUtensorMap *map, int x, int y, int z, int w,
                                                 uint64_t *bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
      "%3, %4, %5}], [%6], %7;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// ------------------------------------------------ CTA-pair (cta_group::2)

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_idx() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// shared::cluster address of this CTA's shared variable at `saddr` in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t peer_addr(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// arrive on an mbarrier of any CTA of the cluster, releasing this thread's earlier writes at cluster scope
__device__ __forceinline__ void mbar_arrive_at(uint32_t cl_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cl_addr) : "memory");
}
// bounded wait that acquires at cluster scope (arrivals and copies from the peer CTA)
__device__ __forceinline__ bool mbar_try_cl(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(100000u)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cl(uint64_t *bar, uint32_t parity, int32_t *err, int code) {
  if (mbar_try_cl(bar, parity)) return true;
  const unsigned long long t0 = gtimer();
  while (true) {
    for (int i = 0; i < 8; ++i)
      if (mbar_try_cl(bar, parity)) return true;
    if (gtimer() - t0 > kWaitNs) {
      atomicCAS(err, 0, code);
      return false;
    }
  }
}
// completion of this thread's earlier tcgen05 operations (both CTAs' tensor
// memory) signalled on an mbarrier of either CTA
__device__ __forceinline__ void tc_commit_pair(uint32_t cl_bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cl_bar) : "memory");
}
__device__ __forceinline__ void tc_mma_mx_pair(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t sfa,
                                               uint32_t sfb, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb)
      : "memory");
}
// each CTA's scale atom (same shared-memory offset) into its own tensor memory
__device__ __forceinline__ void tc_cp_sf_pair(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Block-scaled instruction descriptor: A e2m1, B e4m3, E8M0 scales, f32 D,
// K-major A and B, M = 128, N = n, scale-factor byte ids for A and B = j.
__device__ __forceinline__ uint32_t idesc_mx(int n, uint32_t j, int m = kM) {
  return (j << 4) | (5u << 7) | (0u << 10) | (static_cast<uint32_t>(n >> 3) << 17) | (1u << 23) |
         (static_cast<uint32_t>(m >> 4) << 24) | (j << 29);
}

__device__ __forceinline__ void tc_mma_mx(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t sfa,
                                          uint32_t sfb, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb)
      : "memory");
}

// 512-byte scale-factor atom (32 rows of 16 bytes, no swizzle) as the source
// descriptor of tcgen05.cp: 8-row core matrices 128 B apart.
__device__ __forceinline__ uint64_t sdesc_atom(uint32_t saddr) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | (static_cast<uint64_t>(128 >> 4) << 32) |
         (1ull << 46);
}

// Atom -> TMEM: source row i (16 bytes) goes to lane i of every 32-lane
// quadrant, columns +0..+3; column a then holds the 4 K-block scales of
// matrix row 32a + i.
__device__ __forceinline__ void tc_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

__device__ __forceinline__ uint32_t e4m3x2(float first, float second) {  // first -> low byte
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(second), "f"(first));
  return r;
}

__device__ __forceinline__ float2 e4m3x2_to_f32(uint32_t v) {  // .x <- low byte
  uint32_t h2;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(static_cast<uint16_t>(v)));
  return __half22float2(*reinterpret_cast<__half2 *>(&h2));
}

__device__ __forceinline__ float silu_mx(float g) { return g / (1.0f + expf(-g)); }

// Work items blockIdx.x, +gridDim.x, ... with the tile of the next item loaded
// one item ahead, so no role waits on a tile-list load between items.
struct TileCursor {
  const int4 *tiles;
  int m_tiles, n_items, item;
  int d_per, d_lq, d_nmax;                    // dense tiles when d_per > 0
  int4 cur, nxt;
  __device__ __forceinline__ int4 load(int i) const {
    if (i >= n_items) return make_int4(0, 0, 0, 0);
    const int t = i / m_tiles;
    if (d_per == 0) return tiles[t];
    const int b = t / d_per, j = t - b * d_per;
    return make_int4(b, b * d_lq + j * d_nmax, min(d_nmax, d_lq - j * d_nmax), 0);
  }
  int step;                                   // CTAs (CTA pairs) walking the items
  __device__ __forceinline__ TileCursor(const MxParams &p, int n, int first, int stride)
      : tiles(p.tiles), m_tiles(p.m_tiles), n_items(n), d_per(p.d_tiles > 0 ? p.d_per : 0), d_lq(p.d_lq),
        d_nmax(p.d_nmax), step(stride) {
    item = first;
    cur = load(item);
    nxt = load(item + step);
  }
  __device__ __forceinline__ bool valid() const { return item < n_items; }
  __device__ __forceinline__ int m() const { return item % m_tiles; }
  __device__ __forceinline__ void advance() {
    item += step;
    cur = nxt;
    nxt = load(item + step);
  }
};

template <class C>
__global__ void __launch_bounds__(C::kThreads, 1)
    k_expert_mx(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmBh,
                const __grid_constant__ CUtensorMap tmBl, const __grid_constant__ MxParams p) {
  constexpr int S = C::kStages;
  constexpr int HV = C::kHalves;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sA = smem;                                   // S x kAStage
  uint8_t *sB = sA + S * C::kAStage;                    // S x kBStage: [group][hi rows | lo rows]
  uint8_t *sF = sB + S * C::kBStage;                    // S x kSFStage: [A | B][group] atoms
  uint64_t *bars = reinterpret_cast<uint64_t *>(sF + S * C::kSFStage);
  uint64_t *full = bars;                                // [S]: TMA bytes + 128 scale-thread arrivals
  uint64_t *empty = full + S;                           // [S]: MMA commit
  uint64_t *dfull = empty + S;                          // [2]
  uint64_t *dempty = dfull + 2;                         // [2]
  uint64_t *xbar = dempty + 2;                          // [group][2 warp pairs][2 buffers]: column-max exchange
  uint64_t *pfull = xbar + 4 * C::kEpi;                 // [S] pair, rank 1: its scale threads' arrivals
  uint64_t *pempty = pfull + S;                         // [2] pair, rank 1: its epilogue threads' arrivals
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(pempty + 2);

  const int warp = threadIdx.x >> 5;
  // CTA pair: rank 0 issues the MMAs and owns the barriers they wait on (full,
  // dempty).  Rank 1's scale and epilogue threads arrive on barriers of their
  // own CTA (pfull, pempty) as cheaply as on a single CTA, and one of its idle
  // warps forwards each completed phase with a single cluster-scope arrival:
  // a cluster-scope release from the busy threads themselves would wait for
  // their outstanding loads and stores (ncu: the pair ran at half speed).
  const uint32_t rank = C::kPair ? cluster_rank() : 0u;
  if (threadIdx.x == 0) {
    // full: the producer's expect_tx + every scale thread (+ the peer's forwarded arrival);
    // dempty: every epilogue thread (+ the peer's forwarded arrival)
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], C::kPair ? 1 + 128 + 1 : 1 + 128);
      mbar_init(&empty[i], 1);
      mbar_init(&pfull[i], 128 + 1);                   // rank 1: its scale threads + its producer's expect_tx
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&dfull[i], 1);
      mbar_init(&dempty[i], C::kPair ? 128 * C::kEpi + 1 : 128 * C::kEpi);
      mbar_init(&pempty[i], 128 * C::kEpi);
    }
    for (int i = 0; i < 4 * C::kEpi; ++i) mbar_init(&xbar[i], 64);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if constexpr (C::kPair) cluster_sync();              // the peer's barriers exist before anything reaches them
  if (warp == 2) {
    if constexpr (C::kPair) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                   "r"(C::kTmemCols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                   "r"(C::kTmemCols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // work items: CTA (pair) c takes items c, c + count, ...; a pair CTA's weight rows are block 2 m + rank
  const int first_item = C::kPair ? static_cast<int>(cluster_idx()) : static_cast<int>(blockIdx.x);
  const int item_step = C::kPair ? static_cast<int>(cluster_count()) : static_cast<int>(gridDim.x);
  // the leader's barriers as shared::cluster addresses (the pair's reports go there)
  const uint32_t full_l = C::kPair ? peer_addr(smem_u32(full), 0) : 0u;
  const uint32_t dempty_l = C::kPair ? peer_addr(smem_u32(dempty), 0) : 0u;
  const uint32_t tmem = *tmem_slot;
  // set-up above overlaps the previous kernel's tail; its results are read below
  WM_PDL_WAIT();
  WM_PDL_LAUNCH();

  const int n_items = (p.d_tiles > 0 ? p.d_tiles : *p.n_tiles) * p.m_tiles;
  const int kstages = p.K / C::kKC / p.k_splits;      // stages per work item
  const int ks32 = p.K / 32;

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    uint32_t g = 0;
    bool ok = true;
    // decode: each weight box is read by one tile per launch, so it streams
    // through L2 evict-first; prefill tiles of one expert share its boxes
    const uint64_t stream_once = l2_evict_first_policy();
    for (TileCursor tc(p, n_items, first_item, item_step); tc.valid() && ok; tc.advance()) {
      const int4 tile = tc.cur;
      const int mi = tc.m() / p.k_splits;
      const int k0 = (tc.m() - mi * p.k_splits) * kstages * C::kKC;   // this item's K range
      const int m = C::kPair ? 2 * mi + static_cast<int>(rank) : mi;  // this CTA's 128-row block
      const int nb = (tile.z + 15) >> 4;                // 16-row token boxes per term
      for (int kc = 0; kc < kstages; ++kc, ++g) {
        const int s = g % S;
        if (!(ok = mbar_wait(&empty[s], ((g / S) & 1) ^ 1, p.err, 1))) break;
        if (C::kPair && elect_one()) {
          // this CTA's 128 weight rows and its own token term (rank 0: hi, rank 1: lo), counted on a
          // barrier of its own CTA: rank 0's full, rank 1's pfull (which its forwarding warp relays
          // to rank 0 with the scale rows; copies completing on the other SM's barrier made the
          // pair slower than one CTA)
          uint64_t *fb = rank == 0 ? &full[s] : &pfull[s];
          mbar_expect_tx(fb, HV * kM * kKH / 2 + HV * nb * 16 * kKH);
          for (int q = 0; q < HV; ++q) {
            const int x = k0 + kc * C::kKC + q * kKH;
            uint8_t *a = sA + s * C::kAStage + q * C::kABox;
            if (p.mode == 0)
              tma_load_4d(a, &tmA, x, 0, 0, tile.x * (p.I / 4) + m * 8, fb);
            else
              tma_load_2d(a, &tmA, x, tile.x * p.rows + m * kM, fb);
            uint8_t *b = sB + s * C::kBStage + q * C::kBBox;
            for (int j = 0; j < nb; ++j) tma_load_2d(b + j * 16 * kKH, rank == 0 ? &tmBh : &tmBl, x, tile.y + 16 * j, fb);
          }
        } else if (!C::kPair && elect_one()) {
          // transaction bytes count the packed global bytes of the weights
          mbar_expect_tx(&full[s], HV * (p.a_fp8 ? kM * kKH : kM * kKH / 2) + 2 * HV * nb * 16 * kKH);
          for (int q = 0; q < HV; ++q) {
            const int x = k0 + kc * C::kKC + q * kKH;
            uint8_t *a = sA + s * C::kAStage + q * C::kABox;
            if constexpr (C::kNMax == 32) {
              if (p.mode == 0)
                tma_load_4d_hint(a, &tmA, x, 0, 0, tile.x * (p.I / 4) + m * 8, &full[s], stream_once);
              else
                tma_load_2d_hint(a, &tmA, x, tile.x * p.rows + m * kM, &full[s], stream_once);
            } else {
              if (p.mode == 0)
                tma_load_4d(a, &tmA, x, 0, 0, tile.x * (p.I / 4) + m * 8, &full[s]);
              else
                tma_load_2d(a, &tmA, x, tile.x * p.rows + m * kM, &full[s]);
            }
            uint8_t *b = sB + s * C::kBStage + q * C::kBBox;
            for (int j = 0; j < nb; ++j) {
              tma_load_2d(b + j * 16 * kKH, &tmBh, x, tile.y + 16 * j, &full[s]);
              tma_load_2d(b + (nb + j) * 16 * kKH, &tmBl, x, tile.y + 16 * j, &full[s]);
            }
          }
        }
        __syncwarp();
      }
    }
    for (uint32_t q = 0; q < S && q < g && ok; ++q) {
      const uint32_t gg = g - 1 - q;
      ok = mbar_wait(&empty[gg % S], (gg / S) & 1, p.err, 2);
    }
  } else if (C::kPair && rank != 0 && (warp == 1 || warp == 3)) {
    // ------------------------------------- pair, rank 1: forward to rank 0
    // warp 1: each stage's copies and scale rows (pfull) -> the leader's full barrier;
    // warp 3: each work item's released accumulator (pempty) -> its dempty
    uint32_t g = 0, it = 0;
    bool ok = true;
    for (TileCursor tc(p, n_items, first_item, item_step); tc.valid() && ok; tc.advance(), ++it) {
      if (warp == 1) {
        for (int kc = 0; kc < kstages && ok; ++kc, ++g) {
          const int s = g % S;
          if (!(ok = mbar_wait(&pfull[s], (g / S) & 1, p.err, 11))) break;
          if ((threadIdx.x & 31) == 0) mbar_arrive_at(full_l + 8u * s);
          __syncwarp();
        }
      } else {
        const int db = it & 1;
        if (!(ok = mbar_wait(&pempty[db], (it >> 1) & 1, p.err, 12))) break;
        if ((threadIdx.x & 31) == 0) mbar_arrive_at(dempty_l + 8u * db);
        __syncwarp();
      }
    }
  } else if (warp == 1 && C::kPair) {
    // ------------------------------------------- MMA, CTA pair (rank 0 only)
    // M = 256: rows [0, 128) from this CTA's A stage, [128, 256) from the
    // peer's; N = hi rows (this CTA's B stage) then lo rows (the peer's); D
    // lands in both CTAs' tensor memory, each CTA's scale atoms in its own
    if (rank == 0) {
      const uint32_t sfa = tmem + C::kSfCol0;
      const uint32_t sfb = sfa + HV * 4;
      uint32_t g = 0, it = 0;
      bool ok = true;
      for (TileCursor tc(p, n_items, first_item, item_step); tc.valid() && ok; tc.advance(), ++it) {
        const int4 tile = tc.cur;
        const int n_mma = 2 * max(16, (tile.z + 15) & ~15);
        const int db = it & 1;
        if (!(ok = mbar_wait_cl(&dempty[db], ((it >> 1) & 1) ^ 1, p.err, 3))) break;
        tc_fence_after();
        const uint32_t d_addr = tmem + db * C::kDCols;
        for (int kc = 0; kc < kstages && ok; ++kc, ++g) {
          const int s = g % S;
          if (!(ok = mbar_wait_cl(&full[s], (g / S) & 1, p.err, 4))) break;
          tc_fence_after();
          if (elect_one()) {
            const uint32_t f0 = smem_u32(sF + s * C::kSFStage);
#pragma unroll
            for (int q = 0; q < HV; ++q) {
              tc_cp_sf_pair(sfa + 4 * q, sdesc_atom(f0 + q * 512));
#pragma unroll
              for (int a = 0; a < C::kBAtoms; ++a)
                tc_cp_sf_pair(sfb + C::kSfbCols * q + 4 * a, sdesc_atom(f0 + (HV + q * C::kBAtoms + a) * 512));
            }
            const uint32_t a0 = smem_u32(sA + s * C::kAStage);
            const uint32_t b0 = smem_u32(sB + s * C::kBStage);
#pragma unroll
            for (int kb = 0; kb < C::kKC / 32; ++kb) {
              const int q = kb >> 2;
              const uint32_t j = kb & 3;
              tc_mma_mx_pair(d_addr, bdesc_sw128(a0 + q * C::kABox) + 2 * j, bdesc_sw128(b0 + q * C::kBBox) + 2 * j,
                             idesc_mx(n_mma, j, 2 * kM), (j << 30) | (sfa + 4 * q), (j << 30) | (sfb + C::kSfbCols * q),
                             (kc == 0 && kb == 0) ? 0u : 1u);
            }
            tc_commit_pair(peer_addr(smem_u32(&empty[s]), 0));
            tc_commit_pair(peer_addr(smem_u32(&empty[s]), 1));
          }
          __syncwarp();
        }
        if (ok) {
          if (elect_one()) {
            tc_commit_pair(peer_addr(smem_u32(&dfull[db]), 0));
            tc_commit_pair(peer_addr(smem_u32(&dfull[db]), 1));
          }
          __syncwarp();
        }
      }
    }
  } else if (warp == 1) {
    // --------------------------------------------------------------- MMA
    const uint32_t sfa = tmem + C::kSfCol0;
    const uint32_t sfb = sfa + HV * 4;
    const uint32_t a_fmt_mask = p.a_fp8 ? ~(7u << 7) : ~0u;   // A format field: e2m1 (5) or e4m3 (0)
    uint32_t g = 0, it = 0;
    bool ok = true;
    for (TileCursor tc(p, n_items, first_item, item_step); tc.valid() && ok; tc.advance(), ++it) {
      const int4 tile = tc.cur;
      const int n_mma = 2 * max(16, (tile.z + 15) & ~15);   // hi and lo rows
      const int db = it & 1;
      if (!(ok = mbar_wait(&dempty[db], ((it >> 1) & 1) ^ 1, p.err, 3))) break;
      tc_fence_after();
      const uint32_t d_addr = tmem + db * C::kDCols;
      for (int kc = 0; kc < kstages && ok; ++kc, ++g) {
        const int s = g % S;
        if (!(ok = mbar_wait(&full[s], (g / S) & 1, p.err, 4))) break;
        tc_fence_after();
        if (elect_one()) {
          const uint32_t f0 = smem_u32(sF + s * C::kSFStage);
#pragma unroll
          for (int q = 0; q < HV; ++q) {
            tc_cp_sf(sfa + 4 * q, sdesc_atom(f0 + q * 512));
#pragma unroll
            for (int a = 0; a < C::kBAtoms; ++a)
              tc_cp_sf(sfb + C::kSfbCols * q + 4 * a, sdesc_atom(f0 + (HV + q * C::kBAtoms + a) * 512));
          }
          const uint32_t a0 = smem_u32(sA + s * C::kAStage);
          const uint32_t b0 = smem_u32(sB + s * C::kBStage);
#pragma unroll
          for (int kb = 0; kb < C::kKC / 32; ++kb) {
            const int q = kb >> 2;
            const uint32_t j = kb & 3;
            tc_mma_mx(d_addr, bdesc_sw128(a0 + q * C::kABox) + 2 * j, bdesc_sw128(b0 + q * C::kBBox) + 2 * j,
                      idesc_mx(n_mma, j) & a_fmt_mask, (j << 30) | (sfa + 4 * q), (j << 30) | (sfb + C::kSfbCols * q),
                      (kc == 0 && kb == 0) ? 0u : 1u);
          }
          tc_commit(&empty[s]);
        }
        __syncwarp();
      }
      if (ok) {
        if (elect_one()) tc_commit(&dfull[db]);
        __syncwarp();
      }
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------- scale warps
    // Thread t owns row t of the A atom (weight row of the work item) and row
    // t (+128) of the B atoms: the hi scale of token r for r < n16, the lo
    // scale of token r - n16 for n16 <= r < 2 n16, zero past the tile's
    // tokens.  Scales are read in chunks of CW 32-bit words per row (up to 32
    // bytes, one vector load, covering CW / HV stages) into a two-chunk
    // register ring, so the loads need no L1 reuse (the shared-memory
    // carve-out leaves L1 small) and run a chunk ahead of their use.
    const int t = threadIdx.x - 128;
    const int o = (t & 31) * 4 + (t >> 5);              // 32-bit word of row t inside an atom
    constexpr int BA = C::kBAtoms;
    const int kb = ks32 / p.k_splits;                   // scale bytes per row of one work item
    const int CW = (kb % 32 == 0) ? 8 : (kb % 16 == 0) ? 4 : 2;   // words per row per chunk
    const int SPC = CW / HV;                            // stages per chunk (K range % 256 == 0: kb % 8 == 0)
    const int n_ch = kb / (4 * CW);                     // chunks per work item
    struct Chunk {
      uint32_t a[8];
      uint32_t b[BA][8];
      uint32_t sub[BA];                                 // kLoSub for a lo-term row, else 0
    };
    TileCursor cur(p, n_items, first_item, item_step);   // prefetch cursor
    int c_ch = 0;
    auto load_words = [&](const uint8_t *src, uint32_t *dst) {
      if (CW == 8) {
        const uint4 u0 = __ldg(reinterpret_cast<const uint4 *>(src));
        const uint4 u1 = __ldg(reinterpret_cast<const uint4 *>(src) + 1);
        dst[0] = u0.x; dst[1] = u0.y; dst[2] = u0.z; dst[3] = u0.w;
        dst[4] = u1.x; dst[5] = u1.y; dst[6] = u1.z; dst[7] = u1.w;
      } else if (CW == 4) {
        const uint4 u0 = __ldg(reinterpret_cast<const uint4 *>(src));
        dst[0] = u0.x; dst[1] = u0.y; dst[2] = u0.z; dst[3] = u0.w;
      } else {
        const uint2 u0 = __ldg(reinterpret_cast<const uint2 *>(src));
        dst[0] = u0.x; dst[1] = u0.y;
      }
    };
    auto fetch = [&](Chunk &e) {
#pragma unroll
      for (int w = 0; w < 8; ++w) e.a[w] = 0u;
#pragma unroll
      for (int a = 0; a < BA; ++a) {
        e.sub[a] = 0u;
#pragma unroll
        for (int w = 0; w < 8; ++w) e.b[a][w] = 0u;
      }
      if (!cur.valid()) return;
      const int4 tile = cur.cur;
      const int mi = cur.m() / p.k_splits;
      const int kofs = (cur.m() - mi * p.k_splits) * kb + c_ch * 4 * CW;   // first scale byte of the chunk
      const int m = C::kPair ? 2 * mi + static_cast<int>(rank) : mi;    // this CTA's 128-row block
      const int grow = p.mode == 0 ? ((t >> 3) & 1) * p.I + m * 64 + (t >> 4) * 8 + (t & 7) : m * kM + t;
      if (grow < p.rows)                                // a last partial 128-row tile (score rows): zero scales
        load_words(p.a_scales + (static_cast<int64_t>(tile.x) * p.rows + grow) * ks32 + kofs, e.a);
      const int n16 = max(16, (tile.z + 15) & ~15);
#pragma unroll
      for (int a = 0; a < BA; ++a) {
        const int r = t + 128 * a;                      // B atom row: hi term of token r, or lo of r - n16
        const bool lo_row = r >= n16;
        const int tok = lo_row ? r - n16 : r;
        if (tok < tile.z && r < 2 * n16) {
          load_words(p.b_scales + static_cast<int64_t>(tile.y + tok) * ks32 + kofs, e.b[a]);
          e.sub[a] = lo_row ? kLoSub : 0u;
        }
      }
      if (++c_ch == n_ch) {
        c_ch = 0;
        cur.advance();
      }
    };
    const int my_items = first_item < n_items ? (n_items - 1 - first_item) / item_step + 1 : 0;
    const uint32_t total = static_cast<uint32_t>(my_items) * kstages;
    Chunk ring[2];
    fetch(ring[0]);
    fetch(ring[1]);
    bool ok = true;
    uint32_t g = 0;
    while (g < total && ok) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        for (int si = 0; si < SPC && g < total && ok; ++si, ++g) {
          const int s = g % S;
          ok = mbar_wait(&empty[s], ((g / S) & 1) ^ 1, p.err, 9);
          if (!ok) break;
          uint32_t *f = reinterpret_cast<uint32_t *>(sF + s * C::kSFStage);
#pragma unroll
          for (int q = 0; q < HV; ++q) {
            const int want = si * HV + q;                 // word of this stage within the chunk
            uint32_t va = 0u, vb[BA];
#pragma unroll
            for (int a = 0; a < BA; ++a) vb[a] = 0u;
#pragma unroll
            for (int w = 0; w < 8; ++w) {
              if (w == want) {
                va = ring[u].a[w];
#pragma unroll
                for (int a = 0; a < BA; ++a) vb[a] = ring[u].b[a][w];
              }
            }
            f[q * 128 + o] = va;
#pragma unroll
            for (int a = 0; a < BA; ++a) f[(HV + q * BA + a) * 128 + o] = vb[a] - ring[u].sub[a];
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          mbar_arrive(C::kPair && rank != 0 ? &pfull[s] : &full[s]);
        }
        if (!ok || g >= total) break;
        fetch(ring[u]);
      }
    }
  } else if (warp >= 8) {
    // ---------------------------------------------------------- epilogue
    const int t = (threadIdx.x - 256) & 127;            // TMEM lane = tile row
    const int grp = (threadIdx.x - 256) >> 7;           // epilogue group: chunks grp, grp + kEpi, ...
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int up_half = p.order == WM_UP_GATE ? 0 : 1;
    const bool is_up = ((t >> 3) & 1) == up_half;
    const int lane = threadIdx.x & 31;
    __shared__ uint32_t xchg[2][2][4][16];              // [group][buffer][warp] column maxima
    uint32_t xchg_n = 0;
    uint32_t it = 0;
    bool ok = true;
    for (TileCursor tc(p, n_items, first_item, item_step); tc.valid() && ok; tc.advance(), ++it) {
      const int4 tile = tc.cur;
      const int m = C::kPair ? 2 * (tc.m() / p.k_splits) + static_cast<int>(rank) : tc.m() / p.k_splits;
      const int db = it & 1;
      if (!(ok = C::kPair ? mbar_wait_cl(&dfull[db], (it >> 1) & 1, p.err, 8)
                          : mbar_wait(&dfull[db], (it >> 1) & 1, p.err, 8)))
        break;
      tc_fence_after();
      const int n = tile.z;
      const int n16 = max(16, (n + 15) & ~15);
      for (int c0 = 16 * grp; c0 < n; c0 += 16 * C::kEpi) {
        uint32_t r[16], rl[16];
        WM_TMEM_LD16(tmem + lane_base + db * C::kDCols + c0, r);
        WM_TMEM_LD16(tmem + lane_base + db * C::kDCols + n16 + c0, rl);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int q = 0; q < 16; ++q) r[q] = __float_as_uint(__uint_as_float(r[q]) + __uint_as_float(rl[q]));
        if (p.mode == 0 && !C::kFuseSplit) {
          const int jj = m * 64 + (t >> 4) * 8 + (t & 7);
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const float v = __uint_as_float(r[q]);
            const float o = __shfl_xor_sync(0xffffffffu, v, 8);
            if (is_up && c0 + q < n) {
              float up = v, gate = o;
              if (p.limit > 0.0f) {
                up = fminf(fmaxf(up, -p.limit), p.limit);
                gate = fminf(gate, p.limit);
              }
              p.h_out[static_cast<int64_t>(tile.y + c0 + q) * p.I + jj] = wm_f32_to_bf16(silu_mx(gate) * up);
            }
          }
        } else if (p.mode == 0) {
          // h = ClampedSwiGLU(up, gate) rounded to bf16, then its two e4m3
          // terms: the item's 64 intermediate columns are two whole 32-column
          // scale blocks, block b held by the up lanes of warps 2b and 2b+1
          const int jj = m * 64 + (t >> 4) * 8 + (t & 7);
          uint32_t hb[16];                                // h as f32 bits of its bf16 value (0: not this lane's)
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const float v = __uint_as_float(r[q]);
            const float o = __shfl_xor_sync(0xffffffffu, v, 8);
            hb[q] = 0u;
            if (is_up && c0 + q < n) {
              float up = v, gate = o;
              if (p.limit > 0.0f) {
                up = fminf(fmaxf(up, -p.limit), p.limit);
                gate = fminf(gate, p.limit);
              }
              hb[q] = static_cast<uint32_t>(wm_f32_to_bf16(silu_mx(gate) * up)) << 16;
            }
          }
          const int wq = warp & 3, buf = xchg_n & 1;
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const uint32_t am = __reduce_max_sync(0xffffffffu, hb[q] & 0x7fffffffu);
            if (lane == 0) xchg[grp & 1][buf][wq][q] = am;
          }
          mbar_arrive(&xbar[grp * 4 + (wq >> 1) * 2 + buf]);
          if (!(ok = mbar_wait(&xbar[grp * 4 + (wq >> 1) * 2 + buf], (xchg_n >> 1) & 1, p.err, 10))) break;
          ++xchg_n;
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            if (!(is_up && c0 + q < n)) continue;
            const uint32_t am = max(xchg[grp & 1][buf][wq][q], xchg[grp & 1][buf][wq ^ 1][q]);
            const int sh = max(static_cast<int>(min(am >> 23, 255u)) - 134, -122);
            const float xs = __uint_as_float(hb[q]) * __uint_as_float(static_cast<uint32_t>(127 - sh) << 23);
            const uint32_t hi = e4m3x2(xs, 0.0f) & 0xffu;
            const float hf = e4m3x2_to_f32(hi).x;
            const uint32_t lo = e4m3x2((xs - hf) * static_cast<float>(1 << kLoShift), 0.0f) & 0xffu;
            const int64_t off = static_cast<int64_t>(tile.y + c0 + q) * p.I + jj;
            p.h_hi[off] = static_cast<uint8_t>(hi);
            p.h_lo[off] = static_cast<uint8_t>(lo);
            if (!(wq & 1) && (t & 7) == 0 && ((t >> 4) & 1) == 0)  // first up lane of the block
              p.h_sc[static_cast<int64_t>(tile.y + c0 + q) * (p.I / 32) + (jj >> 5)] = static_cast<uint8_t>(sh + 127);
          }
        } else if (p.k_splits > 1) {
          const int row = m * kM + t;
          float *part = p.y_part + static_cast<int64_t>(tc.m() - m * p.k_splits) * p.part_stride;
#pragma unroll
          for (int q = 0; q < 16; ++q)
            if (c0 + q < n && row < p.rows)
              part[static_cast<int64_t>(tile.y + c0 + q) * p.H + row] = __uint_as_float(r[q]);
        } else {
          const int row = m * kM + t;
#pragma unroll
          for (int q = 0; q < 16; ++q)
            if (c0 + q < n && row < p.rows)
              p.y_out[static_cast<int64_t>(tile.y + c0 + q) * p.H + row] = wm_f32_to_bf16(__uint_as_float(r[q]));
        }
      }
      tc_fence_before();
      mbar_arrive(C::kPair && rank != 0 ? &pempty[db] : &dempty[db]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (C::kPair) cluster_sync();              // both CTAs done with the pair's tensor memory and barriers
  if (warp == 2) {
    tc_fence_after();
    if constexpr (C::kPair)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kTmemCols));
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kTmemCols));
  }
  if (p.done) wm::combine_if_last(p.comb, p.done);
}

// --------------------------------------------------------- two-term split

// Rows [0, rows) of a bf16 matrix (GATHER: row p is x[perm[p] / kk]) ->
// hi, lo e4m3 bytes and the hi term's E8M0 scale per 32 columns.  Four
// threads per 32-value block, eight values each.  `zero`, if set, is a word
// the following tensor-core launch reports errors in, cleared here.
// With plan.idx set (GATHER, calls of at most kSmallRouteMax slots) every CTA
// groups the call's assignments by expert itself (small_route) and CTA 0
// writes the grouping for the launches that follow: no permute launch.
template <bool GATHER>
__global__ void k_split_e4m3(const uint16_t *__restrict__ src, const int32_t *__restrict__ perm,
                             const int32_t *__restrict__ count, int S, int kk, int K, uint8_t *__restrict__ hi,
                             uint8_t *__restrict__ lo, uint8_t *__restrict__ sc, int32_t *__restrict__ zero,
                             const wm::RoutePlan plan) {
  __shared__ wm::SmallRoute<wm::kSmallRouteMax> route;
  __shared__ int32_t route_key[wm::kSmallRouteMax];
  WM_PDL_WAIT();
  WM_PDL_LAUNCH();
  int rows;
  if (GATHER && plan.idx) {
    wm::small_route(plan.idx, plan.T, plan.k, plan.shared_expert, plan.E, route, route_key);
    if (blockIdx.x == 0)
      wm::publish_route(route, plan.T, plan.k, plan.shared_expert, plan.E, plan.offsets, plan.perm, plan.inv,
                        plan.active, plan.counters, plan.tiles, plan.tile_n, plan.done);
    perm = route.perm;
    rows = route.bad ? 0 : S;
  } else {
    if (zero && blockIdx.x == 0 && threadIdx.x == 0) *zero = 0;
    rows = count ? min(S, max(0, *count)) : S;
  }
  const int per_row = K / 8;
  const int64_t total = static_cast<int64_t>(rows) * per_row;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;   // a multiple of 32
  const int64_t span = (total + 31) / 32 * 32;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < span; i += stride) {
    const bool live = i < total;
    const int p = live ? static_cast<int>(i / per_row) : 0;
    const int c = live ? static_cast<int>(i % per_row) : 0;
    uint4 u = make_uint4(0u, 0u, 0u, 0u);
    if (live) {
      const int64_t srow = GATHER ? perm[p] / kk : p;
      u = *reinterpret_cast<const uint4 *>(src + srow * K + c * 8);
    }
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    float v[8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      v[2 * q] = wm_bf16lo(w[q]);
      v[2 * q + 1] = wm_bf16hi(w[q]);
    }
    uint32_t amax = 0u;                                   // |v| bit patterns compare like the values
#pragma unroll
    for (int q = 0; q < 8; ++q) amax = max(amax, __float_as_uint(v[q]) & 0x7fffffffu);
    amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const int ebits = static_cast<int>(min(amax >> 23, 255u));
    const int sh = max(ebits - 134, -122);               // block max / 2^sh in [128, 256)
    const float inv = __uint_as_float(static_cast<uint32_t>(127 - sh) << 23);
    uint32_t hb[4], lb[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float x0 = v[2 * q] * inv, x1 = v[2 * q + 1] * inv;
      hb[q] = e4m3x2(x0, x1);
      const float2 hf = e4m3x2_to_f32(hb[q]);
      lb[q] = e4m3x2((x0 - hf.x) * static_cast<float>(1 << kLoShift), (x1 - hf.y) * static_cast<float>(1 << kLoShift));
    }
    if (live) {
      const int64_t off = static_cast<int64_t>(p) * K + c * 8;
      *reinterpret_cast<uint2 *>(hi + off) = make_uint2(hb[0] | (hb[1] << 16), hb[2] | (hb[3] << 16));
      *reinterpret_cast<uint2 *>(lo + off) = make_uint2(lb[0] | (lb[1] << 16), lb[2] | (lb[3] << 16));
      if ((c & 3) == 0) sc[static_cast<int64_t>(p) * (K / 32) + (c >> 2)] = static_cast<uint8_t>(sh + 127);
    }
  }
}

// out[i] = bf16(part[0][i] + part[1][i] + ... + part[splits-1][i]), added in
// split order so the result does not depend on which CTA finished first.
__global__ void k_sum_splits(const float *__restrict__ part, int64_t n, int64_t stride, int splits,
                             uint16_t *__restrict__ out) {
  WM_PDL_WAIT();
  WM_PDL_LAUNCH();
  const int64_t groups = (n + 3) / 4;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < groups;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = 4 * i;
    if (e + 4 <= n) {
      float4 acc = *reinterpret_cast<const float4 *>(part + e);
      for (int s0 = 1; s0 < splits; s0 += 8) {       // eight loads in flight, then the adds in split order
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (s0 + u < splits) v[u] = *reinterpret_cast<const float4 *>(part + (s0 + u) * stride + e);
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (s0 + u < splits) {
            acc.x += v[u].x;
            acc.y += v[u].y;
            acc.z += v[u].z;
            acc.w += v[u].w;
          }
      }
      *reinterpret_cast<uint2 *>(out + e) =
          make_uint2(static_cast<uint32_t>(wm_f32_to_bf16(acc.x)) | (static_cast<uint32_t>(wm_f32_to_bf16(acc.y)) << 16),
                     static_cast<uint32_t>(wm_f32_to_bf16(acc.z)) | (static_cast<uint32_t>(wm_f32_to_bf16(acc.w)) << 16));
    } else {
      for (int64_t j = e; j < n; ++j) {
        float acc = part[j];
        for (int s = 1; s < splits; ++s) acc += part[s * stride + j];
        out[j] = wm_f32_to_bf16(acc);
      }
    }
  }
}

// ------------------------------------------------------------ host side

int make_map_nd(CUtensorMap *map, CUtensorMapDataType dt, int rank, const void *base, const cuuint64_t *dims,
                const cuuint64_t *strides, const cuuint32_t *box, CUtensorMapSwizzle sw) {
  auto fn = encode_fn();
  if (!fn) return wm::fail(WM_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, dt, rank, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return wm::fail(WM_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  return WM_OK;
}

template <class C>
int launch_mx_cfg(int mode, const uint8_t *w, const uint8_t *a_scales, int E, int rows, int K, const uint8_t *b_hi,
                  const uint8_t *b_lo, const uint8_t *b_sc, int S_rows, int I, int H, int order, float limit,
                  const int4 *tiles, const int32_t *n_tiles, uint8_t *h_hi, uint8_t *h_lo, uint8_t *h_sc,
                  uint16_t *h_out, uint16_t *y_out, int32_t *err, cudaStream_t stream, bool a_fp8 = false,
                  int k_splits = 1, float *y_part = nullptr, int64_t part_stride = 0, int4 dense = int4{0, 0, 0, 0},
                  const wm::CombineArgs *comb = nullptr, int32_t *done = nullptr) {
  if (K % C::kKC) return wm::fail(WM_ERR_UNSUPPORTED, "expert mx: K must be a multiple of the stage depth");
  if (k_splits < 1 || (K / C::kKC) % k_splits || (k_splits > 1 && (mode != 1 || !y_part)))
    return wm::fail(WM_ERR_INVALID, "expert mx: bad K split");
  if (dense.x > 0 && (mode != 1 || dense.y < 1 || dense.w < 1 || dense.w > C::kNMax))
    return wm::fail(WM_ERR_INVALID, "expert mx: bad dense tiles");
  if (!wm::aligned(w, a_fp8 ? 16 : 32)) return wm::fail(WM_ERR_INVALID, "expert mx: packed A operand misaligned");
  if (!wm::aligned(a_scales, 16) || !wm::aligned(b_sc, 16))
    return wm::fail(WM_ERR_INVALID, "expert mx: scales must be 16-byte aligned");
  CUtensorMap tmA, tmBh, tmBl;
  const cuuint64_t rb = static_cast<cuuint64_t>(K) / 2;   // packed bytes per weight row
  if (mode == 0) {
    // (K, row in group of 8, half [first I rows | second I rows], group of 8 rows over all experts):
    // one box = 8 groups x (8 rows of each half) = 64 up + 64 gate rows, interleaved by 8
    const cuuint64_t dims[4] = {static_cast<cuuint64_t>(K), 8, 2, static_cast<cuuint64_t>(E) * (I / 4)};
    const cuuint64_t strides[3] = {rb, rb * I, rb * 8};
    const cuuint32_t box[4] = {kKH, 8, 2, 8};
    if (int rc = make_map_nd(&tmA, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 4, w, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  } else if (a_fp8) {
    // e4m3 rows, one byte per value: plain byte boxes of 128 rows x 128 values
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(E) * rows};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K)};
    const cuuint32_t box[2] = {kKH, kM};
    if (int rc = make_map_nd(&tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  } else {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(E) * rows};
    const cuuint64_t strides[1] = {rb};
    const cuuint32_t box[2] = {kKH, kM};
    if (int rc = make_map_nd(&tmA, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 2, w, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  }
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(S_rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K)};
    const cuuint32_t box[2] = {kKH, 16};
    if (int rc = make_map_nd(&tmBh, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, b_hi, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
    if (int rc = make_map_nd(&tmBl, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, b_lo, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  }
  static std::mutex mu;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
      cudaError_t e = cudaFuncSetAttribute(k_expert_mx<C>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(C::kSmem));
      if (e != cudaSuccess) return wm::fail(WM_ERR_CUDA, std::string("mx smem attribute: ") + cudaGetErrorString(e));
      attr_set[dev] = true;
    }
  }
  MxParams p{};
  p.mode = mode;
  p.K = K;
  p.rows = rows;
  p.I = I;
  p.H = H;
  p.order = order;
  p.limit = limit;
  p.m_tiles = C::kPair ? (mode == 0 ? I / 128 : rows / (2 * kM)) : (mode == 0 ? I / 64 : (rows + kM - 1) / kM) * k_splits;
  if (C::kPair && (k_splits != 1 || a_fp8 || dense.x > 0 || (mode == 0 ? I % 128 : rows % (2 * kM)) != 0))
    return wm::fail(WM_ERR_INVALID, "expert mx: the CTA-pair configuration takes whole 256-row blocks, no K split");
  p.k_splits = k_splits;
  p.y_part = y_part;
  p.part_stride = part_stride;
  p.d_tiles = dense.x;                                  // {tiles, tiles per batch, rows per batch, rows per tile}
  p.d_per = dense.y;
  p.d_lq = dense.z;
  p.d_nmax = dense.w;
  p.a_fp8 = a_fp8 ? 1 : 0;
  p.a_scales = a_scales;
  p.b_scales = b_sc;
  p.tiles = tiles;
  p.n_tiles = n_tiles;
  p.h_hi = h_hi;
  p.h_lo = h_lo;
  p.h_sc = h_sc;
  p.h_out = h_out;
  p.y_out = y_out;
  p.err = err;
  if (comb && done) {
    p.comb = *comb;
    p.done = done;
  }
  cudaError_t e;
  if constexpr (C::kPair) {
    // clusters of two CTAs (the pair), programmatic dependent launch as for every launch of the path
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(wm::sm_count() & ~1);
    cfg.blockDim = dim3(C::kThreads);
    // a persistent grid must be resident all at once: clusters of two need both CTAs on one
    // TPC's pair of SMs, and not every SM can be part of a pair, so the grid is the number of
    // pairs that fit, not the SM count
    static int max_clusters[64] = {0};
    if (dev >= 0 && dev < 64 && max_clusters[dev] == 0) {
      cudaLaunchConfig_t q = cfg;
      q.dynamicSmemBytes = C::kSmem;
      cudaLaunchAttribute qa[1];
      qa[0].id = cudaLaunchAttributeClusterDimension;
      qa[0].val.clusterDim.x = 2;
      qa[0].val.clusterDim.y = 1;
      qa[0].val.clusterDim.z = 1;
      q.attrs = qa;
      q.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, k_expert_mx<C>, &q) != cudaSuccess || n < 1)
        return wm::fail(WM_ERR_CUDA, "expert mx: no resident CTA pair");
      max_clusters[dev] = std::min(n, wm::sm_count() / 2);
      if (getenv("WM_MX_PAIR_VERBOSE")) fprintf(stderr, "expert mx: %d resident CTA pairs\n", max_clusters[dev]);
    }
    cfg.gridDim = dim3(2 * max_clusters[dev]);
    cfg.dynamicSmemBytes = C::kSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    e = cudaLaunchKernelEx(&cfg, k_expert_mx<C>, tmA, tmBh, tmBl, p);
  } else {
    e = wm::launch_pdl(k_expert_mx<C>, dim3(wm::sm_count()), dim3(C::kThreads), C::kSmem, stream, tmA, tmBh, tmBl, p);
  }
  if (e != cudaSuccess) return wm::fail(WM_ERR_CUDA, std::string("expert mx: ") + cudaGetErrorString(e));
  return wm::check_launch("expert mx");
}

// WM_MX_PAIR=1: the prefill configuration runs on CTA pairs (cta_group::2)
bool mx_pair_enabled() {
  const char *v = getenv("WM_MX_PAIR");
  return v && v[0] == '1';
}

int launch_mx(bool decode, int mode, const uint8_t *w, const uint8_t *a_scales, int E, int rows, int K,
              const uint8_t *b_hi, const uint8_t *b_lo, const uint8_t *b_sc, int S_rows, int I, int H, int order,
              float limit, const int4 *tiles, const int32_t *n_tiles, uint8_t *h_hi, uint8_t *h_lo, uint8_t *h_sc,
              uint16_t *h_out, uint16_t *y_out, int32_t *err, cudaStream_t stream, bool wide_up = false,
              const wm::CombineArgs *comb = nullptr, int32_t *done = nullptr) {
  const int4 nd{0, 0, 0, 0};
  if (decode && mode == 0 && wide_up)
    return launch_mx_cfg<MxDecodeUp>(mode, w, a_scales, E, rows, K, b_hi, b_lo, b_sc, S_rows, I, H, order, limit,
                                     tiles, n_tiles, h_hi, h_lo, h_sc, h_out, y_out, err, stream);
  if (decode)
    return launch_mx_cfg<MxDecode>(mode, w, a_scales, E, rows, K, b_hi, b_lo, b_sc, S_rows, I, H, order, limit, tiles,
                                   n_tiles, h_hi, h_lo, h_sc, h_out, y_out, err, stream, false, 1, nullptr, 0, nd,
                                   comb, done);
  if (mx_pair_enabled() && (mode == 0 ? I % 128 : rows % (2 * kM)) == 0)
    return launch_mx_cfg<MxPrefillPair>(mode, w, a_scales, E, rows, K, b_hi, b_lo, b_sc, S_rows, I, H, order, limit,
                                        tiles, n_tiles, h_hi, h_lo, h_sc, h_out, y_out, err, stream, false, 1, nullptr,
                                        0, nd, comb, done);
  return launch_mx_cfg<MxPrefill>(mode, w, a_scales, E, rows, K, b_hi, b_lo, b_sc, S_rows, I, H, order, limit, tiles,
                                  n_tiles, h_hi, h_lo, h_sc, h_out, y_out, err, stream, false, 1, nullptr, 0, nd,
                                  comb, done);
}

}  // namespace

namespace wm {

bool mx_supported(int H, int I) { return H % 256 == 0 && I % 256 == 0; }

int mx_tile_n(int T, int k, int n_routed) {
  // expected tokens per routed expert under uniform routing
  const int64_t per_expert = static_cast<int64_t>(T) * k / std::max(1, n_routed);
  return per_expert <= MxDecode::kNMax ? MxDecode::kNMax : MxPrefill::kNMax;
}

int launch_split_e4m3(const uint16_t *src, const int32_t *perm, const int32_t *count, int S, int kk, int K,
                      uint8_t *hi, uint8_t *lo, uint8_t *sc, cudaStream_t stream, int32_t *zero, const RoutePlan &plan) {
  const int64_t work = static_cast<int64_t>(S) * (K / 8);
  const int grid = static_cast<int>(std::min<int64_t>((work + 255) / 256, sm_count() * 8));
  if (grid > 0) {
    const cudaError_t e =
        perm ? launch_pdl(k_split_e4m3<true>, dim3(grid), dim3(256), 0, stream, src, perm, count, S, kk, K, hi, lo, sc,
                          zero, plan)
             : launch_pdl(k_split_e4m3<false>, dim3(grid), dim3(256), 0, stream, src, static_cast<const int32_t *>(nullptr),
                          count, S, 1, K, hi, lo, sc, zero, RoutePlan{});
    if (e != cudaSuccess) return fail(WM_ERR_CUDA, std::string("split e4m3: ") + cudaGetErrorString(e));
  }
  return check_launch("split e4m3");
}

bool mx_fused_split(int tile_n) { return tile_n == MxDecode::kNMax ? MxDecode::kFuseSplit : MxPrefill::kFuseSplit; }

int launch_mx_up(const uint8_t *w13, const uint8_t *s13, int E, int H, int I, const uint8_t *x_hi,
                 const uint8_t *x_lo, const uint8_t *x_sc, int S_rows, int order, float limit, const int4 *tiles,
                 const int32_t *n_tiles, uint8_t *h_hi, uint8_t *h_lo, uint8_t *h_sc, uint16_t *h, int32_t *err,
                 int tile_n, cudaStream_t stream, int T) {
  return launch_mx(tile_n == MxDecode::kNMax, 0, w13, s13, E, 2 * I, H, x_hi, x_lo, x_sc, S_rows, I, H, order, limit,
                   tiles, n_tiles, h_hi, h_lo, h_sc, h, nullptr, err, stream, T > 16);
}

int launch_mx_down(const uint8_t *w2, const uint8_t *s2, int E, int H, int I, const uint8_t *h_hi,
                   const uint8_t *h_lo, const uint8_t *h_sc, int S_rows, const int4 *tiles, const int32_t *n_tiles,
                   uint16_t *y, int32_t *err, int tile_n, cudaStream_t stream, const CombineArgs *comb,
                   int32_t *done) {
  return launch_mx(tile_n == MxDecode::kNMax, 1, w2, s2, E, H, I, h_hi, h_lo, h_sc, S_rows, I, H, WM_UP_GATE, 0.0f,
                   tiles, n_tiles, nullptr, nullptr, nullptr, nullptr, y, err, stream, false, comb, done);
}

}  // namespace wm

namespace {

struct ScoreWorkspace {
  uint8_t *q_hi, *q_lo, *q_sc;
  int32_t *counters;  // [1] the tensor-core kernel's error code (cleared by the token split)
  float *part;        // [splits][part_stride] f32 partial scores
  int64_t part_stride;
  size_t bytes;
};

constexpr int kB200Sms = 148;

// K ranges per work item for a decode-configuration score launch whose
// (tile, 128-row) items do not fill the GPU: the divisor s of the stage count
// that minimises the busiest CTA's stages, counting one stage of per-item
// overhead, ceil(items * s / sm) * (stages / s + 1).  s = 1 for launches that
// already fill every SM, and always for the prefill configuration.
int choose_splits(int64_t items, int stages, int nmax, int sm) {
  if (nmax != MxDecode::kNMax || items <= 0 || items >= sm) return 1;
  int best = 1;
  int64_t best_cost = (items + sm - 1) / sm * (stages + 1);
  for (int s = 2; s <= stages && s <= 32; ++s) {
    if (stages % s) continue;
    const int64_t cost = (items * s + sm - 1) / sm * (stages / s + 1);
    if (cost < best_cost) {
      best = s;
      best_cost = cost;
    }
  }
  return best;
}

int score_nmax(int Lq) { return Lq <= 32 ? MxDecode::kNMax : MxPrefill::kNMax; }

int score_splits(int B, int Lq, int D, int L, int sm) {
  const int nmax = score_nmax(Lq);
  const int64_t items = static_cast<int64_t>(B) * ((Lq + nmax - 1) / nmax) * ((L + kM - 1) / kM);
  return choose_splits(items, D / MxDecode::kKC, nmax, sm);
}

ScoreWorkspace carve_scores(void *base, int B, int Lq, int D, int L, int splits) {
  ScoreWorkspace w{};
  const size_t rows = static_cast<size_t>(std::max(B * Lq, 16));
  size_t off = 0;
  auto take = [&](size_t n) {
    const size_t o = off;
    off = wm::align_up(off + n, 256);
    return o;
  };
  const size_t o_hi = take(rows * D), o_lo = take(rows * D), o_sc = take(rows * (D / 32));
  const size_t o_c = take(16);
  w.part_stride = splits > 1 ? static_cast<int64_t>(wm::align_up(static_cast<size_t>(B) * Lq * L, 64)) : 0;
  const size_t o_p = take(static_cast<size_t>(splits > 1 ? splits : 0) * w.part_stride * sizeof(float));
  w.bytes = off;
  if (base) {
    char *b = static_cast<char *>(base);
    w.q_hi = reinterpret_cast<uint8_t *>(b + o_hi);
    w.q_lo = reinterpret_cast<uint8_t *>(b + o_lo);
    w.q_sc = reinterpret_cast<uint8_t *>(b + o_sc);
    w.counters = reinterpret_cast<int32_t *>(b + o_c);
    w.part = reinterpret_cast<float *>(b + o_p);
  }
  return w;
}

}  // namespace

extern "C" size_t wkv_scores_workspace_size(int B, int Lq, int D, int L) {
  if (B < 1 || Lq < 1 || D < 32 || L < 1) return 0;
  return carve_scores(nullptr, B, Lq, D, L, D % 256 ? 1 : score_splits(B, Lq, D, L, kB200Sms)).bytes;
}

extern "C" int wkv_mx_scores(const wm_bf16 *query, int B, int Lq, int D, const uint8_t *payload,
                             const uint8_t *scales, int L, int fmt, wm_bf16 *scores, void *workspace,
                             size_t ws_bytes, wm_stream_t stream) {
  wm::clear_error();
  WM_REQUIRE(B >= 1 && Lq >= 1 && L >= 1, "kv scores: need B, Lq, L >= 1");
  WM_REQUIRE(fmt == WKV_MXFP8_B32 || fmt == WKV_MXFP4_B32, "kv scores: fmt must be WKV_MXFP8_B32 or WKV_MXFP4_B32");
  WM_REQUIRE(D % 256 == 0, "kv scores: the tensor-core path needs D % 256 == 0");
  WM_REQUIRE(query && payload && scales && scores && workspace, "kv scores: null buffer");
  WM_REQUIRE(wm::aligned(query, 16) && wm::aligned(scores, 16) && wm::aligned(workspace, 256),
             "kv scores: query/scores 16-byte, workspace 256-byte aligned");
  // K splits for an under-filled launch, fewer if the workspace was sized for fewer
  int splits = score_splits(B, Lq, D, L, wm::sm_count());
  ScoreWorkspace ws = carve_scores(workspace, B, Lq, D, L, splits);
  while (splits > 1 && ws_bytes < ws.bytes) {
    do --splits; while ((D / MxDecode::kKC) % splits);
    ws = carve_scores(workspace, B, Lq, D, L, splits);
  }
  if (ws_bytes < ws.bytes) return wm::fail(WM_ERR_WORKSPACE, "kv scores: workspace too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int nmax = score_nmax(Lq);
  const int per = (Lq + nmax - 1) / nmax;
  // tiles {batch, first query row, queries}: ceil(Lq / nmax) per batch, computed in the kernel
  const int4 dense = make_int4(B * per, per, Lq, nmax);
  if (int rc = wm::launch_split_e4m3(reinterpret_cast<const uint16_t *>(query), nullptr, nullptr, B * Lq, 1, D,
                                     ws.q_hi, ws.q_lo, ws.q_sc, st, ws.counters + 1))
    return rc;
  // scores[b, q, l] = D[l, q] of the "down projection" form: rows = L cache rows of batch b, output row stride L
  const int s_rows = std::max(B * Lq, 16);
  if (nmax == MxDecode::kNMax) {
    if (int rc = launch_mx_cfg<MxDecode>(1, payload, scales, B, L, D, ws.q_hi, ws.q_lo, ws.q_sc, s_rows, 0, L,
                                         WM_UP_GATE, 0.0f, nullptr, ws.counters, nullptr, nullptr, nullptr, nullptr,
                                         reinterpret_cast<uint16_t *>(scores), ws.counters + 1, st,
                                         fmt == WKV_MXFP8_B32, splits, ws.part, ws.part_stride, dense))
      return rc;
    if (splits == 1) return WM_OK;
    const int64_t n = static_cast<int64_t>(B) * Lq * L;
    const int grid = static_cast<int>(std::min<int64_t>(((n + 3) / 4 + 255) / 256, wm::sm_count() * 8));
    if (cudaError_t e = wm::launch_pdl(k_sum_splits, dim3(grid), dim3(256), 0, st, static_cast<const float *>(ws.part),
                                       n, ws.part_stride, splits, reinterpret_cast<uint16_t *>(scores)))
      return wm::fail(WM_ERR_CUDA, std::string("kv scores split sum: ") + cudaGetErrorString(e));
    return wm::check_launch("kv scores split sum");
  }
  return launch_mx_cfg<MxPrefill>(1, payload, scales, B, L, D, ws.q_hi, ws.q_lo, ws.q_sc, s_rows, 0, L, WM_UP_GATE,
                                  0.0f, nullptr, ws.counters, nullptr, nullptr, nullptr, nullptr,
                                  reinterpret_cast<uint16_t *>(scores), ws.counters + 1, st, fmt == WKV_MXFP8_B32, 1,
                                  nullptr, 0, dense);
}

extern "C" size_t wmx_linear_workspace_size(int T, int K, int N) { return wkv_scores_workspace_size(1, T, K, N); }

// A dense block-scaled linear is the score kernel with one "sequence" whose N
// cached rows are the weight rows and whose T queries are the tokens.  Calls
// of one or two rows stream the weights on CUDA cores instead (one launch,
// linear_stream.cu); WM_LINEAR_PATH=tc keeps them on the tensor path.
extern "C" int wmx_linear(const wm_bf16 *x, int T, int K, const uint8_t *w, const uint8_t *scales, int N, int fmt,
                          wm_bf16 *y, void *workspace, size_t ws_bytes, wm_stream_t stream) {
  wm::clear_error();
  if (T == 0) return WM_OK;
  const char *path = getenv("WM_LINEAR_PATH");
  const int bits = fmt == WKV_MXFP8_B32 ? 8 : fmt == WKV_MXFP4_B32 ? 4 : 0;
  if (!(path && path[0] == 't') && T >= 1 && N >= 1 && bits && x && w && scales && y && wm::aligned(x, 16) &&
      wm::aligned(w, 16) && wm::aligned(scales, 8) && wm::linear_stream_supported(T, K, N, bits))
    return wm::launch_linear_stream(reinterpret_cast<const uint16_t *>(x), T, K, w, scales, N, bits,
                                    reinterpret_cast<uint16_t *>(y), static_cast<cudaStream_t>(stream));
  return wkv_mx_scores(x, 1, T, K, w, scales, N, fmt, y, workspace, ws_bytes, stream);
}

extern "C" int wmx_split_e4m3(const wm_bf16 *x, int rows, int cols, uint8_t *hi, uint8_t *lo, uint8_t *scales,
                              wm_stream_t stream) {
  wm::clear_error();
  WM_REQUIRE(rows >= 0 && cols > 0 && cols % 32 == 0, "split_e4m3: need rows >= 0 and cols a multiple of 32");
  if (rows == 0) return WM_OK;
  WM_REQUIRE(x && hi && lo && scales, "split_e4m3: null buffer");
  WM_REQUIRE(wm::aligned(x, 16) && wm::aligned(hi, 8) && wm::aligned(lo, 8), "split_e4m3: misaligned buffer");
  return wm::launch_split_e4m3(reinterpret_cast<const uint16_t *>(x), nullptr, nullptr, rows, 1, cols, hi, lo, scales,
                               static_cast<cudaStream_t>(stream));
}
