// Installed-model expert layer -> device-resident expert tensors.
//
// An installed layer file holds n_blobs expert blobs of blob_size bytes; each
// blob carries the regions the manifest lists at fixed byte offsets
// (runtime/deepseek_v4_ssd/manifest.py:14-47, 170-175).  The reference's
// expert cache copies those regions, one blob at a time, into a cache slot in
// its fused layout (expert_cache.py:416-428, expert_layout.py:8-80).  Here the
// whole layer is made resident in one pass: the file is read in chunks of
// whole blobs into two pinned host buffers, and each region of every blob in a
// chunk goes to its destination with a single pitched host-to-device copy
// (source pitch = blob_size, destination pitch = one expert), so the copy
// engine performs the re-layout while the next chunk is being read (by
// several reader threads on disjoint slices).
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "wm_common.cuh"

namespace {

// Pinned staging, kept across calls (allocating hundreds of MB of pinned
// memory costs more than reading it); grown when a call needs more.  Loads
// are serialised by the mutex that guards it.
struct Staging {
  std::mutex mu;
  void *p[2] = {nullptr, nullptr};
  size_t bytes = 0;
  cudaError_t reserve(size_t n) {
    if (n <= bytes) return cudaSuccess;
    for (int i = 0; i < 2; ++i) {
      if (p[i]) cudaFreeHost(p[i]);
      p[i] = nullptr;
    }
    bytes = 0;
    for (int i = 0; i < 2; ++i) {
      cudaError_t e = cudaHostAlloc(&p[i], n, cudaHostAllocDefault);
      if (e != cudaSuccess) return e;
    }
    bytes = n;
    return cudaSuccess;
  }
};
Staging g_staging;

struct Fd {
  int fd = -1;
  ~Fd() {
    if (fd >= 0) close(fd);
  }
};

struct Ev {
  cudaEvent_t e = nullptr;
  bool live = false;
  ~Ev() {
    if (e) cudaEventDestroy(e);
  }
};

// Read n bytes at `at`; 0 on success, else the errno (or -1 at end of file).
int read_span(int fd, uint8_t *dst, size_t n, off_t at) {
  size_t got = 0;
  while (got < n) {
    ssize_t k = pread(fd, dst + got, n - got, at + static_cast<off_t>(got));
    if (k < 0 && errno == EINTR) continue;
    if (k <= 0) return k < 0 ? errno : -1;
    got += static_cast<size_t>(k);
  }
  return 0;
}

// Read a chunk with up to kReaders threads on disjoint slices (page-cache
// copies and NVMe queues both scale with concurrent readers).
constexpr int kReaders = 8;
constexpr size_t kMinSlice = 8u << 20;

int read_full(int fd, uint8_t *dst, size_t n, off_t at, const char *path) {
  int t = static_cast<int>(std::min<size_t>(kReaders, std::max<size_t>(1, n / kMinSlice)));
  size_t slice = (n + t - 1) / t;
  slice = (slice + 4095) & ~size_t(4095);
  std::vector<int> err(t, 0);
  std::vector<std::thread> pool;
  for (int i = 1; i < t; ++i) {
    size_t lo = i * slice;
    if (lo >= n) break;
    size_t len = std::min(slice, n - lo);
    pool.emplace_back([&, i, lo, len] { err[i] = read_span(fd, dst + lo, len, at + static_cast<off_t>(lo)); });
  }
  err[0] = read_span(fd, dst, std::min(slice, n), at);
  for (auto &th : pool) th.join();
  for (int e : err)
    if (e != 0)
      return wm::fail(WM_ERR_INVALID, std::string("short read from ") + path + ": " +
                                          (e > 0 ? std::strerror(e) : "end of file"));
  return WM_OK;
}

int cuda_fail(cudaError_t e, const char *what) {
  return wm::fail(WM_ERR_CUDA, std::string("wld_load_expert_layer: ") + what + ": " + cudaGetErrorString(e));
}

}  // namespace

extern "C" {

WM_API int wld_load_expert_layer(const char *path, size_t blob_size, int n_blobs, int n_regions,
                                 const size_t *src_offsets, const size_t *lengths, void *const *dst_bases,
                                 const size_t *dst_pitches, size_t chunk_bytes, wm_stream_t stream) {
  if (!path || blob_size == 0 || n_blobs <= 0 || n_regions <= 0 || !src_offsets || !lengths || !dst_bases ||
      !dst_pitches)
    return wm::fail(WM_ERR_INVALID, "wld_load_expert_layer: bad arguments");
  for (int r = 0; r < n_regions; ++r) {
    if (lengths[r] == 0 || src_offsets[r] > blob_size || lengths[r] > blob_size - src_offsets[r])
      return wm::fail(WM_ERR_INVALID,
                      "wld_load_expert_layer: region " + std::to_string(r) + " lies outside the blob");
    if (!dst_bases[r] || dst_pitches[r] < lengths[r])
      return wm::fail(WM_ERR_INVALID, "wld_load_expert_layer: region " + std::to_string(r) +
                                          " has no destination or its pitch is shorter than the region");
  }
  Fd f;
  f.fd = open(path, O_RDONLY | O_CLOEXEC);
  if (f.fd < 0) return wm::fail(WM_ERR_INVALID, std::string("cannot open ") + path + ": " + std::strerror(errno));
  struct stat st;
  if (fstat(f.fd, &st) != 0) return wm::fail(WM_ERR_INVALID, std::string("cannot stat ") + path);
  if (static_cast<size_t>(st.st_size) != blob_size * static_cast<size_t>(n_blobs))
    return wm::fail(WM_ERR_INVALID, std::string("installed expert layer has an invalid size: ") + path);

  size_t per = chunk_bytes / blob_size;
  if (per < 1) per = 1;
  if (per > static_cast<size_t>(n_blobs)) per = static_cast<size_t>(n_blobs);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  std::lock_guard<std::mutex> lock(g_staging.mu);
  {
    cudaError_t e = g_staging.reserve(per * blob_size);
    if (e != cudaSuccess) return cuda_fail(e, "pinned staging");
  }
  Ev done[2];
  for (int i = 0; i < 2; ++i) {
    cudaError_t e = cudaEventCreateWithFlags(&done[i].e, cudaEventDisableTiming);
    if (e != cudaSuccess) return cuda_fail(e, "event");
  }
  int ci = 0;
  int rc = WM_OK;
  for (size_t e0 = 0; e0 < static_cast<size_t>(n_blobs) && rc == WM_OK; e0 += per, ++ci) {
    const size_t n = (e0 + per <= static_cast<size_t>(n_blobs)) ? per : static_cast<size_t>(n_blobs) - e0;
    const int b = ci & 1;
    // The copies out of this staging buffer (issued two chunks ago) must have finished.
    if (done[b].live) {
      cudaError_t e = cudaEventSynchronize(done[b].e);
      if (e != cudaSuccess) return cuda_fail(e, "staging wait");
    }
    uint8_t *buf = static_cast<uint8_t *>(g_staging.p[b]);
    rc = read_full(f.fd, buf, n * blob_size, static_cast<off_t>(e0 * blob_size), path);
    for (int r = 0; r < n_regions && rc == WM_OK; ++r) {
      uint8_t *dst = static_cast<uint8_t *>(dst_bases[r]) + e0 * dst_pitches[r];
      cudaError_t e = cudaMemcpy2DAsync(dst, dst_pitches[r], buf + src_offsets[r], blob_size, lengths[r], n,
                                        cudaMemcpyHostToDevice, s);
      if (e != cudaSuccess) rc = cuda_fail(e, "region copy");
    }
    if (rc == WM_OK) {
      cudaError_t e = cudaEventRecord(done[b].e, s);
      if (e != cudaSuccess) rc = cuda_fail(e, "event record");
      done[b].live = true;
    }
  }
  // The staging buffers are reused by the next call: every copy out of them must be done.
  cudaError_t e = cudaStreamSynchronize(s);
  if (rc == WM_OK && e != cudaSuccess) rc = cuda_fail(e, "final wait");
  return rc;
}

}  // extern "C"
