// Permute: stable sort of (token, slot) assignments by expert.
//
// Reference: mlx-lm switch_layers._gather_sort / _scatter_unsort, called at
// model.py:404/455 and qwen4_exp.py:622/649; the per-expert grouping by a
// stable argsort in _forward_with_resident (model.py:371-385).
//
// One CTA.  The S assignments are cut into W contiguous segments, one per
// warp.  Pass 1 builds a per-warp histogram in shared memory; a scan over
// (expert, warp) gives every warp its starting cursor for every expert; pass
// 2 walks each segment in order 32 assignments at a time, ranking equal
// experts inside the 32 with __match_any_sync.  The result is the stable
// order (ties by flat assignment index), independent of scheduling.
//
// Besides offsets/perm/inv the kernel emits the compact list of active
// experts (count > 0) that the expert kernels iterate over.
#include "wm_common.cuh"
#include "wm_moe.cuh"

namespace {

__global__ void __launch_bounds__(1024) k_permute(const int32_t *__restrict__ idx, int T, int k, int shared_expert,
                                                  wm::RouteFilter rf, int E, int32_t *__restrict__ offsets, int32_t *__restrict__ perm,
                                                  int32_t *__restrict__ inv, int32_t *__restrict__ active,
                                                  int32_t *__restrict__ n_active, int32_t *__restrict__ error_flag,
                                                  int4 *__restrict__ tiles, int32_t *__restrict__ n_tiles, int tile_n,
                                                  int32_t *__restrict__ clear) {
  extern __shared__ int32_t sm[];
  WM_PDL_WAIT();
  WM_PDL_LAUNCH();

  const int nw = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kk = k + (shared_expert >= 0 ? 1 : 0);
  const int S = T * kk;
  int32_t *hist = sm;                 // [nw][E]
  int32_t *tot = sm + nw * E;         // [E+1]
  __shared__ int32_t bad;
  if (threadIdx.x == 0) {
    bad = 0;
    if (clear) *clear = 0;
  }
  for (int i = threadIdx.x; i < nw * E; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int seg = (S + nw - 1) / nw;
  const int s0 = warp * seg, s1 = min(S, s0 + seg);
  // expert of assignment a, kBad for an id outside the layer's experts.  With
  // a route filter (rf.count > 0, an expert-parallel rank's share) routed ids
  // whose placement position (rf.remap[id], or id) lies in [rf.base, rf.base +
  // rf.count) are kept as position - rf.base; other ids in [0, rf.n_global),
  // and shared slots of tokens outside [rf.shared_lo, rf.shared_hi), are
  // kDropped.
  constexpr int kBad = -1, kDropped = -2;
  auto expert_of = [&](int a) -> int {
    int t = a / kk, j = a - t * kk;
    if (j >= k) return (rf.count > 0 && (t < rf.shared_lo || t >= rf.shared_hi)) ? kDropped : shared_expert;
    int e = idx[static_cast<int64_t>(t) * k + j];
    if (rf.count > 0) {
      if (e < 0 || e >= rf.n_global) return kBad;
      if (rf.remap) e = rf.remap[e];                 // placement position (any value outside the range is dropped)
      return (e >= rf.base && e < rf.base + rf.count) ? e - rf.base : kDropped;
    }
    return (e < 0 || e >= E) ? kBad : e;
  };
  for (int a = s0 + lane; a < s1; a += 32) {
    int e = expert_of(a);
    if (e == kDropped) continue;
    if (e == kBad) {
      bad = 1;
      continue;
    }
    atomicAdd(&hist[warp * E + e], 1);
  }
  __syncthreads();
  if (bad) {
    if (threadIdx.x == 0) {
      if (error_flag) *error_flag = 1;
      if (n_active) *n_active = 0;
      if (n_tiles) *n_tiles = 0;
      for (int e = 0; e < E; ++e) offsets[e] = 0;
      offsets[E] = -1;  // sentinel: an expert id was outside [0, E)
    }
    return;
  }
  // totals per expert, then a block-wide exclusive scan of (tokens, active
  // experts, tiles): thread i owns the contiguous experts [i*cpt, (i+1)*cpt)
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int c = 0;
    for (int w = 0; w < nw; ++w) c += hist[w * E + e];
    tot[e] = c;
  }
  __syncthreads();
  {
    __shared__ int3 wsum[32];
    const int cpt = (E + blockDim.x - 1) / blockDim.x;
    const int e0 = min(E, static_cast<int>(threadIdx.x) * cpt), e1 = min(E, e0 + cpt);
    int3 mine = make_int3(0, 0, 0);
    for (int e = e0; e < e1; ++e) {
      const int c = tot[e];
      mine.x += c;
      mine.y += c > 0 ? 1 : 0;
      mine.z += tiles ? (c + tile_n - 1) / tile_n : 0;
    }
    int3 inc = mine;  // inclusive warp scan
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int ax = __shfl_up_sync(0xffffffffu, inc.x, d);
      const int ay = __shfl_up_sync(0xffffffffu, inc.y, d);
      const int az = __shfl_up_sync(0xffffffffu, inc.z, d);
      if (lane >= d) { inc.x += ax; inc.y += ay; inc.z += az; }
    }
    if (lane == 31) wsum[warp] = inc;
    __syncthreads();
    int3 base = make_int3(0, 0, 0);
    for (int w = 0; w < warp; ++w) { base.x += wsum[w].x; base.y += wsum[w].y; base.z += wsum[w].z; }
    int run = base.x + inc.x - mine.x, na = base.y + inc.y - mine.y, nt = base.z + inc.z - mine.z;
    // The shared expert (the last id) has a slot for every token, so its tiles are
    // the widest: they go first in the work list, where their longer epilogues
    // overlap other tiles' work instead of ending the launch.  Only the order of
    // the list changes; every tile is computed the same way wherever it sits.
    const int sh_tiles = (tiles && shared_expert == E - 1) ? (tot[E - 1] + tile_n - 1) / tile_n : 0;
    __syncthreads();  // every thread has read tot[] for its experts before it is overwritten below
    for (int e = e0; e < e1; ++e) {
      const int c = tot[e];
      offsets[e] = run;
      tot[e] = run;
      if (c > 0) {
        if (active) active[na] = e;
        ++na;
      }
      if (tiles) {
        if (e == shared_expert && sh_tiles > 0) {      // the last expert: nt counts every other tile
          int at = 0;
          for (int q = 0; q < c; q += tile_n) tiles[at++] = make_int4(e, run + q, min(tile_n, c - q), 0);
          nt += sh_tiles;
        } else {
          for (int q = 0; q < c; q += tile_n) tiles[sh_tiles + nt++] = make_int4(e, run + q, min(tile_n, c - q), 0);
        }
      }
      run += c;
    }
    if (threadIdx.x == blockDim.x - 1) {
      offsets[E] = run;
      tot[E] = run;
      if (n_active) *n_active = na;
      if (n_tiles) *n_tiles = nt;
      if (error_flag) *error_flag = 0;
    }
  }
  __syncthreads();
  // per-warp cursors: base of expert e for warp w = tot[e] + sum_{w'<w} hist[w'][e]
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = tot[e];
    for (int w = 0; w < nw; ++w) {
      int c = hist[w * E + e];
      hist[w * E + e] = run;
      run += c;
    }
  }
  __syncthreads();
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int a0 = s0; a0 < s1; a0 += 32) {
    int a = a0 + lane;
    int e = a < s1 ? expert_of(a) : -1;
    if (a < s1 && e == kDropped) inv[a] = -1;
    const bool valid = a < s1 && e >= 0;
    unsigned peers = __match_any_sync(0xffffffffu, e);
    int rank = __popc(peers & lt_mask);
    int base = valid ? hist[warp * E + e] : 0;
    __syncwarp();
    if (valid) {
      int slot = base + rank;
      perm[slot] = a;
      inv[a] = slot;
      // the highest lane of each peer group advances the cursor
      if ((peers >> lane) == 1u) hist[warp * E + e] = base + __popc(peers);
    }
    __syncwarp();
  }
}

}  // namespace

namespace wm {

size_t permute_smem_bytes(int E, int nw) { return (static_cast<size_t>(nw) * E + E + 1) * sizeof(int32_t); }

int permute_warps(int E) {
  int nw = 32;
  while (nw > 1 && permute_smem_bytes(E, nw) > 200 * 1024) nw >>= 1;
  return nw;
}

int launch_permute(const int32_t *idx, int T, int k, int shared_expert, int E, int32_t *offsets, int32_t *perm,
                   int32_t *inv, int32_t *active, int32_t *n_active, int32_t *error_flag, int4 *tiles,
                   int32_t *n_tiles, int tile_n, cudaStream_t stream, RouteFilter rf, int32_t *clear) {
  // warps: one per 32 assignments (at least 4, for the per-expert loops), up
  // to what the per-warp histograms leave room for
  const int64_t S = static_cast<int64_t>(T) * (k + (shared_expert >= 0 ? 1 : 0));
  int nw = 4;
  while (nw < 32 && nw * 32 < S) nw <<= 1;
  nw = std::min(nw, permute_warps(E));
  const size_t smem = permute_smem_bytes(E, nw);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(k_permute, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return fail(WM_ERR_CUDA, std::string("permute smem: ") + cudaGetErrorString(e));
  }
  if (cudaError_t e = launch_pdl(k_permute, dim3(1), dim3(nw * 32), smem, stream, idx, T, k, shared_expert, rf, E,
                                 offsets, perm, inv, active, n_active, error_flag, tiles, n_tiles, tile_n, clear))
    return fail(WM_ERR_CUDA, std::string("permute: ") + cudaGetErrorString(e));
  return check_launch("permute");
}

}  // namespace wm

extern "C" int wmoe_permute(const int32_t *idx, int T, int k, int E, int32_t *offsets, int32_t *perm, int32_t *inv,
                            wm_stream_t stream) {
  wm::clear_error();
  WM_REQUIRE(T >= 0 && k >= 1 && E >= 1 && E <= 4096, "permute needs T >= 0, k >= 1, 1 <= E <= 4096");
  WM_REQUIRE(static_cast<int64_t>(T) * k < (1LL << 30), "permute: too many assignments");
  WM_REQUIRE(idx && offsets && perm && inv, "permute: null buffer");
  return wm::launch_permute(idx, T, k, -1, E, offsets, perm, inv, nullptr, nullptr, nullptr, nullptr, nullptr, 0,
                            stream);
}
