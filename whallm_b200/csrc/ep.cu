// Expert-parallel exchange over peer memory (NVLink / NVSwitch, CUDA IPC).
//
// The decode form of the expert-parallel layer moves a few rows per rank per
// layer call: every rank's tokens and routes to every rank, then every rank's
// partial sums back to the tokens' owner.  Collective libraries spend tens of
// microseconds per call on such small messages; here the rows are written
// straight into the peers' receive buffers with plain stores over NVLink and
// a per-rank flag is raised in every peer's flag array afterwards:
//
//   wep_put_rows   rows of up to four regions -> region offset rank * rows of
//                  every peer's buffer (optionally a different source block
//                  per peer), then flags[q][rank] = ++epoch on every peer q
//                  (the last CTA to finish raises them, after a system-scope
//                  fence, with release stores);
//   wep_wait       one thread spins (acquire loads, bounded to 2 s, then an
//                  error code) until every flags[q] >= epoch;
//   wep_sum_rows   out[b] = bf16(sum over q = 0..W-1 of part[q][b]), f32 in
//                  rank order (deterministic).
//
// Epochs live in device memory, so the calls replay from a CUDA graph; each
// rank makes the same sequence of calls, so epochs agree.  A buffer slot is
// overwritten only after its reader has signalled a later step (the protocol
// of the layer guarantees it), so single buffering is enough.  No TMA or
// library kernel touches peer memory: only these kernels' loads and stores.
#include <cuda_runtime.h>

#include <cstring>

#include "wm_common.cuh"

namespace {

constexpr int kMaxWorld = 8;
constexpr int kMaxRegions = 4;
constexpr unsigned long long kWaitNs = 2000000000ull;

struct Region {
  const uint8_t *src;      // rows x row_bytes (per-peer blocks src_peer_stride apart)
  size_t row_bytes;        // a multiple of 4
  size_t src_peer_stride;  // 0: the same rows go to every peer
  size_t dst_offset;       // byte offset of the region in each peer buffer
  int wide;                // 16-byte copies (every address and block size 16-aligned), else 4-byte copies
};

struct PutArgs {
  Region reg[kMaxRegions];
  int n_regions;
  int rows;
  int rank, world;
  uint8_t *dst[kMaxWorld];       // peer q's buffer (q == rank: the local one)
  uint32_t *flags[kMaxWorld];    // peer q's flag array for this exchange
  uint32_t *epoch;               // local epoch counter of this exchange
  int32_t *counter;              // local CTA-arrival counter (left at 0)
};

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__global__ void __launch_bounds__(256) k_put_rows(PutArgs a) {
  WM_PDL_WAIT();
  WM_PDL_LAUNCH();
  // grid-stride over (peer, region, 16-byte chunk)
  for (int r = 0; r < a.n_regions; ++r) {
    const Region &g = a.reg[r];
    const size_t block = static_cast<size_t>(a.rows) * g.row_bytes;   // bytes this rank sends each peer
    const size_t chunks = block / (g.wide ? 16 : 4);
    const size_t total = chunks * a.world;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
      const int q = static_cast<int>(i / chunks);
      const size_t c = i % chunks;
      const uint8_t *sp = g.src + q * g.src_peer_stride;
      uint8_t *dp = a.dst[q] + g.dst_offset + static_cast<size_t>(a.rank) * block;
      if (g.wide)
        reinterpret_cast<uint4 *>(dp)[c] = reinterpret_cast<const uint4 *>(sp)[c];
      else
        reinterpret_cast<uint32_t *>(dp)[c] = reinterpret_cast<const uint32_t *>(sp)[c];
    }
  }
  // the last CTA raises this rank's flag on every peer once every CTA's stores are visible system-wide
  __threadfence_system();
  __syncthreads();
  __shared__ int last;
  if (threadIdx.x == 0) last = atomicAdd(a.counter, 1) == static_cast<int>(gridDim.x) - 1;
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence_system();
    const uint32_t e = *a.epoch + 1;
    *a.epoch = e;
    *a.counter = 0;
    for (int q = 0; q < a.world; ++q) st_release_sys(a.flags[q] + a.rank, e);
  }
}

__global__ void k_wait(const uint32_t *flags, int world, const uint32_t *epoch, int32_t *err, int code) {
  WM_PDL_WAIT();
  WM_PDL_LAUNCH();
  if (threadIdx.x != 0) return;
  const uint32_t e = *epoch;
  const unsigned long long t0 = gtimer();
  for (int q = 0; q < world; ++q) {
    while (static_cast<int32_t>(ld_acquire_sys(flags + q) - e) < 0) {
      if (gtimer() - t0 > kWaitNs) {
        atomicCAS(err, 0, code);
        return;
      }
      __nanosleep(200);
    }
  }
}

// out[b, :] = bf16(sum_q part[q][b, :]) in q order; zeros if *err is set
__global__ void k_sum_rows(const float *__restrict__ part, int world, int rows, int H, const int32_t *__restrict__ err,
                           uint16_t *__restrict__ out) {
  WM_PDL_WAIT();
  WM_PDL_LAUNCH();
  const bool bad = err && *err != 0;
  const int64_t per = H / 4;
  const int64_t total = static_cast<int64_t>(rows) * per;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < world && !bad; ++q) {
      const float4 v = reinterpret_cast<const float4 *>(part + static_cast<int64_t>(q) * rows * H)[i];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    uint2 o;
    o.x = wm_f32_to_bf16(acc.x) | (static_cast<uint32_t>(wm_f32_to_bf16(acc.y)) << 16);
    o.y = wm_f32_to_bf16(acc.z) | (static_cast<uint32_t>(wm_f32_to_bf16(acc.w)) << 16);
    reinterpret_cast<uint2 *>(out)[i] = o;
  }
}

}  // namespace

extern "C" {

int wep_ipc_alloc(size_t bytes, void **ptr, unsigned char *handle) {
  wm::clear_error();
  WM_REQUIRE(bytes > 0 && ptr && handle, "wep_ipc_alloc: need bytes > 0 and output pointers");
  void *p = nullptr;
  if (cudaError_t e = cudaMalloc(&p, bytes)) return wm::fail(WM_ERR_CUDA, std::string("wep_ipc_alloc: ") + cudaGetErrorString(e));
  if (cudaError_t e = cudaMemset(p, 0, bytes)) {
    cudaFree(p);
    return wm::fail(WM_ERR_CUDA, std::string("wep_ipc_alloc memset: ") + cudaGetErrorString(e));
  }
  cudaIpcMemHandle_t h;
  if (cudaError_t e = cudaIpcGetMemHandle(&h, p)) {
    cudaFree(p);
    return wm::fail(WM_ERR_CUDA, std::string("wep_ipc_alloc handle: ") + cudaGetErrorString(e));
  }
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return WM_OK;
}

int wep_ipc_open(const unsigned char *handle, void **ptr) {
  wm::clear_error();
  WM_REQUIRE(handle && ptr, "wep_ipc_open: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void *p = nullptr;
  if (cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess))
    return wm::fail(WM_ERR_CUDA, std::string("wep_ipc_open: ") + cudaGetErrorString(e));
  *ptr = p;
  return WM_OK;
}

int wep_ipc_close(void *ptr) {
  wm::clear_error();
  if (!ptr) return WM_OK;
  if (cudaError_t e = cudaIpcCloseMemHandle(ptr))
    return wm::fail(WM_ERR_CUDA, std::string("wep_ipc_close: ") + cudaGetErrorString(e));
  return WM_OK;
}

int wep_ipc_free(void *ptr) {
  wm::clear_error();
  if (!ptr) return WM_OK;
  if (cudaError_t e = cudaFree(ptr)) return wm::fail(WM_ERR_CUDA, std::string("wep_ipc_free: ") + cudaGetErrorString(e));
  return WM_OK;
}

int wep_put_rows(int n_regions, const void *const *srcs, const size_t *row_bytes, const size_t *src_peer_stride,
                 const size_t *dst_offsets, int rows, void *const *peer_dst, int rank, int world,
                 uint32_t *const *peer_flags, uint32_t *epoch, int32_t *counter, wm_stream_t stream) {
  wm::clear_error();
  WM_REQUIRE(world >= 1 && world <= kMaxWorld && rank >= 0 && rank < world, "wep_put_rows: need 0 <= rank < world <= 8");
  WM_REQUIRE(n_regions >= 1 && n_regions <= kMaxRegions && rows >= 0, "wep_put_rows: 1..4 regions, rows >= 0");
  WM_REQUIRE(srcs && row_bytes && dst_offsets && peer_dst && peer_flags && epoch && counter, "wep_put_rows: null argument");
  PutArgs a{};
  a.n_regions = n_regions;
  a.rows = rows;
  a.rank = rank;
  a.world = world;
  a.epoch = epoch;
  a.counter = counter;
  for (int r = 0; r < n_regions; ++r) {
    const size_t stride = src_peer_stride ? src_peer_stride[r] : 0;
    WM_REQUIRE(row_bytes[r] % 4 == 0 && dst_offsets[r] % 4 == 0 && wm::aligned(srcs[r], 4) && stride % 4 == 0,
               "wep_put_rows: row bytes, offsets, strides and sources must be 4-byte multiples / aligned");
    const size_t block = static_cast<size_t>(rows) * row_bytes[r];
    const int wide = (block % 16 == 0 && dst_offsets[r] % 16 == 0 && wm::aligned(srcs[r], 16) && stride % 16 == 0) ? 1 : 0;
    a.reg[r] = Region{static_cast<const uint8_t *>(srcs[r]), row_bytes[r], stride, dst_offsets[r], wide};
  }
  for (int q = 0; q < world; ++q) {
    WM_REQUIRE(peer_dst[q] && peer_flags[q] && wm::aligned(peer_dst[q], 16), "wep_put_rows: null or misaligned peer");
    a.dst[q] = static_cast<uint8_t *>(peer_dst[q]);
    a.flags[q] = peer_flags[q];
  }
  size_t work = 0;
  for (int r = 0; r < n_regions; ++r)
    work += static_cast<size_t>(rows) * row_bytes[r] / (a.reg[r].wide ? 16 : 4) * world;
  const int grid = static_cast<int>(std::max<size_t>(1, std::min<size_t>((work + 255) / 256, wm::sm_count() * 2)));
  if (cudaError_t e = wm::launch_pdl(k_put_rows, dim3(grid), dim3(256), 0, static_cast<cudaStream_t>(stream), a))
    return wm::fail(WM_ERR_CUDA, std::string("wep_put_rows: ") + cudaGetErrorString(e));
  return wm::check_launch("wep_put_rows");
}

int wep_wait(const uint32_t *flags, int world, const uint32_t *epoch, int32_t *err, wm_stream_t stream) {
  wm::clear_error();
  WM_REQUIRE(flags && epoch && err && world >= 1 && world <= kMaxWorld, "wep_wait: bad arguments");
  if (cudaError_t e = wm::launch_pdl(k_wait, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), flags, world,
                                     epoch, err, 1))
    return wm::fail(WM_ERR_CUDA, std::string("wep_wait: ") + cudaGetErrorString(e));
  return wm::check_launch("wep_wait");
}

int wep_sum_rows(const float *part, int world, int rows, int H, const int32_t *err, wm_bf16 *out, wm_stream_t stream) {
  wm::clear_error();
  WM_REQUIRE(part && out && world >= 1 && rows >= 0 && H % 4 == 0, "wep_sum_rows: bad arguments");
  // the kernel reads part as float4 and writes out as 4 bf16 (8 bytes) at a time
  WM_REQUIRE(wm::aligned(part, 16) && wm::aligned(out, 8),
             "wep_sum_rows: part must be 16-byte and out 8-byte aligned");
  if (rows == 0) return WM_OK;
  const int64_t work = static_cast<int64_t>(rows) * (H / 4);
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, wm::sm_count() * 4)));
  if (cudaError_t e = wm::launch_pdl(k_sum_rows, dim3(grid), dim3(256), 0, static_cast<cudaStream_t>(stream), part,
                                     world, rows, H, err, reinterpret_cast<uint16_t *>(out)))
    return wm::fail(WM_ERR_CUDA, std::string("wep_sum_rows: ") + cudaGetErrorString(e));
  return wm::check_launch("wep_sum_rows");
}

}  // extern "C"
