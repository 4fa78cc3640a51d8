// Dense block-scaled linear for calls of one or two rows, on CUDA cores:
// y [T, N] bf16 = x [T, K] bf16 @ dequant(w)^T for w stored as MXFP8 (e4m3
// [N, K]) or MXFP4 (e2m1 [N, K/2]) with one E8M0 scale per 32 values.
//
// Reference: the MXFP8 QuantizedLinear layers V4.1 installs over its native
// FP8 weights (runtime/deepseek_v4_ssd/deepseek_v41_ssd.py:232-261, 353-360:
// mx.quantized_matmul, transpose=True, group 32).
//
// At one or two rows every weight byte meets one or two token values: the
// call is a weight stream, and on the tensor-core path the fixed cost of its
// three launches (token split, GEMM, K-split sum) and of the GEMM's set-up is
// most of it.  Here one launch streams the weights to CUDA-core arithmetic:
//
//   * A chunk is 4 weight rows; step s of a chunk covers the rows' values
//     [1024 s, 1024 s + 1024), lane l the 32-value scale group 32 s + l of
//     each row (32 bytes of e4m3 or 16 of e2m1: one coalesced 1 KB / 512 B
//     read per row and step).  A chunk's steps are cut into `parts` runs;
//     the (chunk, part) units of a CTA's contiguous chunk range are cut into
//     one contiguous range per warp, so every warp gets a few units.
//   * Weights and scale bytes travel by cp.async through a 3-stage ring per
//     warp (two steps in flight, about 100 KB per SM), evict-first in L2.
//     A copy warp issuing 1D bulk copies (cp.async.bulk) into a deep ring
//     streamed at 1.2-3.3 TB/s against 5.9 TB/s for these per-lane copies
//     (one to eight copies per stage): a bulk copy's bytes arrive at a limited
//     rate per copy, and a few large copies do not keep HBM busy.  Each thread loads its token values before its first weight
//     copy, so they do not queue behind the weight stream.
//   * Each weight pair becomes two exact f16 values (cvt.rn.f16x2.e4m3x2 /
//     e2m1x2) and fma.rn.f32.f16 multiplies them by the token values exactly,
//     one f32 rounding per product.  The token rows are held as f16 with a
//     power of two per 32 values (every bf16 value within 2^-32 of its group
//     maximum exact).  A lane walks its group in four 8-value pieces starting
//     at piece ((l >> 1) + (l >> 3)) & 3, which makes its 16-byte token reads
//     and 8- / 4-byte weight reads free of bank conflicts.
//   * Per (row, token): the group's two f32 chains (even and odd values) are
//     added, multiplied by the token group's power of two and fmaf'ed with
//     the row's E8M0 scale into the lane's sum; a unit's lane sums meet in a
//     warp butterfly.  One part per chunk: the warp writes y.  Several: the
//     warps write f32 partial sums into shared memory and the CTA adds a
//     row's parts in part order.  Results do not depend on which warp ran
//     what, and a row's result is the same with one token or two.
#include <mutex>

#include "wm_common.cuh"
#include "wm_moe.cuh"
#include "wm_tc.cuh"
#include "wm_stream.cuh"

namespace {

using namespace wm_stream;

constexpr int kLWarps = 12;
constexpr int kLThreads = kLWarps * 32;
constexpr int kLRows = 4;           // weight rows per chunk: one token-piece load serves 4 rows
constexpr int kLDepth = 3;          // ring stages per warp (two steps in flight)
constexpr int kLUnitsPerWarp = 3;   // the parts per chunk aim for at least this many units per warp

template <int FMT>
struct LRing {
  static constexpr int kPB = FMT == 8 ? 32 : 16;    // bytes of one 32-value group
  static constexpr int kW = kLRows * 32 * kPB;      // weight bytes per stage
  static constexpr int kS = kLRows * 32;            // scale bytes per stage
  static constexpr int kStage = kW + kS;
  static constexpr int kWarpBytes = kLDepth * kStage;
};

struct LinearStreamParams {
  const uint16_t *x;     // [T, K] bf16
  const uint8_t *w;      // e4m3 [N, K] or e2m1 [N, K / 2]
  const uint8_t *sc;     // E8M0 [N, K / 32]
  uint16_t *y;           // [T, N] bf16
  int T, K, N;
  int parts;             // runs of whole steps per chunk
  int part_offset;       // shared memory: f32 partial sums [chunks of the CTA][parts][4 rows x NT]
  int ring_offset;       // shared memory: the warps' copy rings
};

template <int FMT, int NT>
__global__ void __launch_bounds__(kLThreads, 1) k_linear_stream(const __grid_constant__ LinearStreamParams p) {
  using RG = LRing<FMT>;
  constexpr int PB = RG::kPB;
  constexpr int V = kLRows * NT;                         // sums per unit
  constexpr int kShift = V == 16 ? 1 : V == 8 ? 2 : 3;   // lane bits below the value index after warp_sums
  extern __shared__ __align__(16) uint8_t smem[];
  const int K = p.K, G = K / 32, N = p.N, T = p.T, P = p.parts;
  const int steps = (G + 31) / 32;
  const int nc = (N + kLRows - 1) / kLRows;
  const int c0 = static_cast<int>(static_cast<int64_t>(nc) * blockIdx.x / gridDim.x);
  const int c1 = static_cast<int>(static_cast<int64_t>(nc) * (blockIdx.x + 1) / gridDim.x);
  const int units = (c1 - c0) * P;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int u0 = static_cast<int>(static_cast<int64_t>(units) * warp / kLWarps);
  const int u1 = static_cast<int>(static_cast<int64_t>(units) * (warp + 1) / kLWarps);
  const bool has_work = u0 < u1;
  const int64_t row_bytes = FMT == 8 ? K : K / 2;
  uint16_t *xs = reinterpret_cast<uint16_t *>(smem);                                  // [T][K] f16
  float *xk = reinterpret_cast<float *>(smem + static_cast<size_t>(T) * K * 2);       // [T][G]
  float *part = reinterpret_cast<float *>(smem + p.part_offset);
  uint8_t *ring = smem + p.ring_offset + static_cast<size_t>(warp) * RG::kWarpBytes;
  const uint32_t ring_s = static_cast<uint32_t>(__cvta_generic_to_shared(ring));

  // cursor over the warp's (unit, step) sequence; unit u is local chunk u / P, part u % P
  struct Cur {
    int u, s, se;
  };
  auto begin_unit = [&](Cur &c) {
    const int j = c.u % P;
    c.s = j * steps / P;
    c.se = (j + 1) * steps / P;
  };
  auto advance = [&](Cur &c) {
    if (++c.s < c.se) return;
    if (++c.u < u1) begin_unit(c);
  };

  // the token rows (and nothing else) may come from the previous launch
  WM_PDL_WAIT();
  WM_PDL_LAUNCH();

  // this thread's first token group is requested before any weight copy
  uint4 xv0[4];
  if (static_cast<int>(threadIdx.x) < T * G) {
    const int t = threadIdx.x / G, q = threadIdx.x - t * G;
    const uint4 *src = reinterpret_cast<const uint4 *>(p.x + static_cast<int64_t>(t) * K + q * 32);
#pragma unroll
    for (int i = 0; i < 4; ++i) xv0[i] = __ldcg(src + i);
  }

  const uint64_t pol = wm_tc::l2_evict_first_policy();
  Cur L{u0, 0, 0};
  if (has_work) begin_unit(L);
  auto issue = [&](int slot) {
    if (L.u < u1) {
      const int row0 = (c0 + L.u / P) * kLRows;
      const int q = L.s * 32 + lane;
      const uint32_t st = ring_s + slot * RG::kStage;
      if (q < G) {
#pragma unroll
        for (int r = 0; r < kLRows; ++r) {
          if (row0 + r >= N) break;
          const uint8_t *src = p.w + static_cast<int64_t>(row0 + r) * row_bytes + static_cast<int64_t>(q) * PB;
          cp_async16(st + r * 32 * PB + lane * PB, src, pol);
          if (PB == 32) cp_async16(st + r * 32 * PB + lane * PB + 16, src + 16, pol);
        }
      }
      if (lane < 4 * kLRows) {               // row lane / 4, scale bytes [8 j, 8 j + 8) of the step's 32 groups
        const int r = lane >> 2, j = lane & 3;
        const int g0 = L.s * 32 + 8 * j;
        if (g0 < G && row0 + r < N)
          cp_async8(st + RG::kW + r * 32 + 8 * j, p.sc + static_cast<int64_t>(row0 + r) * G + g0, pol);
      }
      advance(L);
    }
    cp_async_commit();
  };
  if (has_work)
    for (int i = 0; i < kLDepth - 1; ++i) issue(i);

  // token rows -> f16 with a power of two per 32 values (while the first weight copies are in flight)
  for (int g = threadIdx.x; g < T * G; g += kLThreads) {
    const int t = g / G, q = g - t * G;
    if (g != static_cast<int>(threadIdx.x)) {
      const uint4 *src = reinterpret_cast<const uint4 *>(p.x + static_cast<int64_t>(t) * K + q * 32);
#pragma unroll
      for (int i = 0; i < 4; ++i) xv0[i] = __ldcg(src + i);
    }
    xk[t * G + q] = stage_group_f16(xv0, reinterpret_cast<uint4 *>(xs + static_cast<int64_t>(t) * K + q * 32));
  }
  __syncthreads();

  if (has_work) {
    Cur C{u0, 0, 0};
    begin_unit(C);
    int xr[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) xr[t] = min(t, T - 1);
    const int rot = ((lane >> 1) + (lane >> 3)) & 3;   // first 8-value piece of the lane's group
    float acc[kLRows][NT];
#pragma unroll
    for (int r = 0; r < kLRows; ++r)
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[r][t] = 0.0f;

    auto compute = [&](int slot) {
      const int q = C.s * 32 + lane;
      if (q >= G) return;
      const uint8_t *st = ring + slot * RG::kStage;
      float lo[kLRows][NT], hi[kLRows][NT];
#pragma unroll
      for (int r = 0; r < kLRows; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) lo[r][t] = hi[r][t] = 0.0f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int pc = (i + rot) & 3;                   // values [8 pc, 8 pc + 8) of the group
        uint32_t xv[NT][4];
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const uint4 u = *reinterpret_cast<const uint4 *>(xs + static_cast<int64_t>(xr[t]) * K + q * 32 + 8 * pc);
          xv[t][0] = u.x; xv[t][1] = u.y; xv[t][2] = u.z; xv[t][3] = u.w;
        }
#pragma unroll
        for (int r = 0; r < kLRows; ++r) {
          uint32_t h[4];
          if constexpr (FMT == 8) {
            const uint2 wv = *reinterpret_cast<const uint2 *>(st + r * 32 * PB + lane * PB + 8 * pc);
            uint32_t a[2], b[2];
            e4m3x4_to_f16x2(wv.x, a);
            e4m3x4_to_f16x2(wv.y, b);
            h[0] = a[0]; h[1] = a[1]; h[2] = b[0]; h[3] = b[1];
          } else {
            e2m1x8_to_f16x2(*reinterpret_cast<const uint32_t *>(st + r * 32 * PB + lane * PB + 4 * pc), h);
          }
#pragma unroll
          for (int t = 0; t < NT; ++t)
#pragma unroll
            for (int j = 0; j < 4; ++j) fma_f16x2_f32(h[j], xv[t][j], lo[r][t], hi[r][t]);
        }
      }
#pragma unroll
      for (int r = 0; r < kLRows; ++r) {
        const float sw = wm_e8m0(st[RG::kW + r * 32 + lane]);
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[r][t] = fmaf((lo[r][t] + hi[r][t]) * xk[xr[t] * G + q], sw, acc[r][t]);
      }
    };
    // the unit's sums: value r * NT + t is (row r, token t)
    auto flush = [&]() {
      float v[V];
#pragma unroll
      for (int r = 0; r < kLRows; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          v[r * NT + t] = acc[r][t];
          acc[r][t] = 0.0f;
        }
      const float sum = warp_sums<V>(v, lane);
      if ((lane & ((1 << kShift) - 1)) != 0) return;
      const int vi = (lane >> kShift) & (V - 1);
      if (P == 1) {
        const int r = vi / NT, t = vi - r * NT;
        const int row = (c0 + C.u) * kLRows + r;
        if (row < N && t < T) p.y[static_cast<int64_t>(t) * N + row] = wm_f32_to_bf16(sum);
      } else {
        part[C.u * V + vi] = sum;
      }
    };

    for (int use = 0, fill = kLDepth - 1;;) {
      issue(fill);                           // the slot the previous step used
      cp_async_wait<kLDepth - 1>();          // this lane's copies of this step have landed
      __syncwarp();                          // and every lane's (the scale bytes)
      compute(use);
      if (C.s + 1 == C.se) flush();
      advance(C);
      __syncwarp();                          // the slot is read before a later step refills it
      if (C.u >= u1) break;
      fill = use;
      use = use + 1 == kLDepth ? 0 : use + 1;
    }
    cp_async_wait<0>();
  }
  if (P > 1) {
    // a row's parts added in part order
    __syncthreads();
    const int n_out = (c1 - c0) * V;
    for (int i = threadIdx.x; i < n_out; i += kLThreads) {
      const int lc = i / V, vi = i - lc * V;
      const int r = vi / NT, t = vi - r * NT;
      const int row = (c0 + lc) * kLRows + r;
      if (row >= N || t >= T) continue;
      float s = part[(lc * P) * V + vi];
      for (int j = 1; j < P; ++j) s += part[(lc * P + j) * V + vi];
      p.y[static_cast<int64_t>(t) * N + row] = wm_f32_to_bf16(s);
    }
  }
}

struct LinearPlan {
  int grid, parts;
  size_t part_offset, ring_offset, smem;
};

LinearPlan plan_linear(int T, int K, int N, int fmt, int sm) {
  LinearPlan lp{};
  const int G = K / 32, steps = (G + 31) / 32;
  const int nc = (N + kLRows - 1) / kLRows;
  lp.grid = std::min(sm, nc);
  const int64_t want = static_cast<int64_t>(kLUnitsPerWarp) * kLWarps * lp.grid;
  lp.parts = static_cast<int>(std::min<int64_t>(steps, std::max<int64_t>(1, (want + nc - 1) / nc)));
  const int nt = T <= 1 ? 1 : 2;
  const int cta_chunks = (nc + lp.grid - 1) / lp.grid;
  const size_t stage = static_cast<size_t>(T) * K * 2 + static_cast<size_t>(T) * G * 4;
  lp.part_offset = wm::align_up(stage, 16);
  const size_t parts = lp.parts > 1 ? static_cast<size_t>(cta_chunks) * lp.parts * kLRows * nt * 4 : 0;
  lp.ring_offset = wm::align_up(lp.part_offset + parts, 16);
  lp.smem = lp.ring_offset + static_cast<size_t>(kLWarps) * (fmt == 8 ? LRing<8>::kWarpBytes : LRing<4>::kWarpBytes);
  return lp;
}

template <int FMT, int NT>
cudaError_t launch_linear(const LinearStreamParams &p, const LinearPlan &lp, cudaStream_t stream) {
  // the attribute is per function and device: set once per template instance on each device
  static std::mutex mu;
  static bool attr_done[64] = {false};
  int dev = 0;
  if (cudaError_t e = cudaGetDevice(&dev)) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!attr_done[dev]) {
      cudaError_t e = cudaFuncSetAttribute(k_linear_stream<FMT, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(wm::kStreamSmemMax));
      if (e != cudaSuccess) return e;
      attr_done[dev] = true;
    }
  }
  return wm::launch_pdl(k_linear_stream<FMT, NT>, dim3(lp.grid), dim3(kLThreads), lp.smem, stream, p);
}

}  // namespace

namespace wm {

bool linear_stream_supported(int T, int K, int N, int fmt) {
  if (T < 1 || T > kLinearStreamMaxT || K < 256 || K % 256 != 0 || N < 1 || (fmt != 8 && fmt != 4)) return false;
  // two rows double the arithmetic per byte: on one B200 the stream then holds ~4.5 TB/s, so matrices
  // beyond 48 MB (the tensor path's fixed cost amortised) stay on the tensor path (7168 x 18432 MXFP8:
  // 30.0 against 24.4 us; 5120 x 5120: 10.5 against 11.5 us)
  if (T == 2 && static_cast<int64_t>(N) * (fmt == 8 ? K : K / 2) > (int64_t{48} << 20)) return false;
  return plan_linear(T, K, N, fmt, sm_count()).smem <= kStreamSmemMax;
}

int launch_linear_stream(const uint16_t *x, int T, int K, const uint8_t *w, const uint8_t *sc, int N, int fmt,
                         uint16_t *y, cudaStream_t stream) {
  if (!linear_stream_supported(T, K, N, fmt)) return fail(WM_ERR_INVALID, "linear stream: unsupported shape");
  if (!aligned(w, 16) || !aligned(sc, 8) || !aligned(x, 16))
    return fail(WM_ERR_INVALID, "linear stream: rows and weights 16-byte, scales 8-byte aligned");
  const LinearPlan lp = plan_linear(T, K, N, fmt, sm_count());
  LinearStreamParams p{};
  p.x = x; p.w = w; p.sc = sc; p.y = y;
  p.T = T; p.K = K; p.N = N;
  p.parts = lp.parts;
  p.part_offset = static_cast<int>(lp.part_offset);
  p.ring_offset = static_cast<int>(lp.ring_offset);
  cudaError_t e;
  if (fmt == 8) e = T == 1 ? launch_linear<8, 1>(p, lp, stream) : launch_linear<8, 2>(p, lp, stream);
  else e = T == 1 ? launch_linear<4, 1>(p, lp, stream) : launch_linear<4, 2>(p, lp, stream);
  if (e != cudaSuccess) return fail(WM_ERR_CUDA, std::string("linear stream: ") + cudaGetErrorString(e));
  return check_launch("linear stream");
}

}  // namespace wm
