// akv_lib.cu — library-level entry points: version, last error, status reset.
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstring>
#include <thread>
#include <vector>

#include "akv_common.cuh"

namespace {
thread_local char g_last_error[512] = {0};
}

void akv_set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int akv_cuda_fail(cudaError_t err, const char* what) {
  akv_set_error("%s: %s (%s)", what, cudaGetErrorString(err), cudaGetErrorName(err));
  return AKV_ERR_CUDA;
}

extern "C" int akv_version(void) { return (AKV_VERSION_MAJOR << 16) | AKV_VERSION_MINOR; }

extern "C" int akv_last_error(char* buf, int len) {
  if (buf == nullptr || len <= 0) return AKV_ERR_INVALID_ARG;
  strncpy(buf, g_last_error, static_cast<size_t>(len) - 1);
  buf[len - 1] = '\0';
  return AKV_OK;
}

extern "C" int akv_status_clear(AkvStatus* status, void* stream) {
  AKV_ARG_CHECK(status != nullptr, "akv_status_clear: status is NULL");
  cudaError_t e = cudaMemsetAsync(status, 0, sizeof(AkvStatus), akv_stream(stream));
  if (e != cudaSuccess) return akv_cuda_fail(e, "akv_status_clear");
  return AKV_OK;
}

extern "C" int akv_copy_wait(void* dst, const void* src, int64_t bytes, int32_t to_host, int32_t wait,
                             void* stream) {
  AKV_ARG_CHECK(bytes >= 0 && (bytes == 0 || (dst != nullptr && src != nullptr)), "akv_copy_wait: bad arguments");
  cudaStream_t s = akv_stream(stream);
  if (bytes > 0) {
    const cudaError_t e = cudaMemcpyAsync(dst, src, static_cast<size_t>(bytes),
                                          to_host ? cudaMemcpyDeviceToHost : cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return akv_cuda_fail(e, "akv_copy_wait: copy");
  }
  if (wait) {
    const cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return akv_cuda_fail(e, "akv_copy_wait: wait");
  }
  return AKV_OK;
}

extern "C" int akv_gather_upload(const uint64_t* src, const int64_t* lens, int32_t n, int32_t* dst,
                                 int32_t* d_dst, int32_t threads, void* stream) {
  AKV_ARG_CHECK(n >= 0 && (n == 0 || (src != nullptr && lens != nullptr && dst != nullptr)),
                "akv_gather_upload: bad arguments");
  AKV_ARG_CHECK(threads >= 1 && threads <= 64, "akv_gather_upload: threads=%d not in [1, 64]", threads);
  std::vector<int64_t> off(static_cast<size_t>(n) + 1, 0);
  for (int32_t i = 0; i < n; ++i) {
    AKV_ARG_CHECK(lens[i] >= 0 && (lens[i] == 0 || src[i] != 0), "akv_gather_upload: array %d: %lld tokens at %p", i,
                  static_cast<long long>(lens[i]), reinterpret_cast<const void*>(src[i]));
    off[i + 1] = off[i] + lens[i];
  }
  const int64_t total = off[n];
  // Tokens [lo, hi) of the packing, from whichever arrays cover them.
  auto copy_range = [&](int64_t lo, int64_t hi) {
    if (lo >= hi) return;
    int32_t i = static_cast<int32_t>(std::upper_bound(off.begin(), off.end(), lo) - off.begin()) - 1;
    for (i = std::max(i, 0); i < n && off[i] < hi; ++i) {
      const int64_t a = std::max(off[i], lo), b = std::min(off[i + 1], hi);
      if (b > a)
        std::memcpy(dst + a, reinterpret_cast<const int32_t*>(src[i]) + (a - off[i]), 4 * static_cast<size_t>(b - a));
    }
  };
  // With an upload, the packing goes in slices: slice k's copy to the device
  // is enqueued as soon as every thread has written its share of it, so the
  // transfer of one slice overlaps the gather of the next.
  const int32_t parts = total < (1 << 16) ? 1 : threads;
  const int32_t slices = (d_dst != nullptr && total >= (1 << 20)) ? 4 : 1;
  std::vector<std::atomic<int32_t>> done(static_cast<size_t>(slices));
  for (auto& d : done) d.store(0);
  auto worker = [&](int32_t t) {
    for (int32_t k = 0; k < slices; ++k) {
      const int64_t lo = total * k / slices, hi = total * (k + 1) / slices;
      copy_range(lo + (hi - lo) * t / parts, lo + (hi - lo) * (t + 1) / parts);
      done[k].fetch_add(1, std::memory_order_release);
    }
  };
  std::vector<std::thread> pool;
  pool.reserve(parts - 1);
  for (int32_t t = 1; t < parts; ++t) pool.emplace_back(worker, t);
  // The calling thread copies share 0 of each slice, waits for the others'
  // shares of it and enqueues its upload.
  cudaError_t err = cudaSuccess;
  for (int32_t k = 0; k < slices; ++k) {
    const int64_t lo = total * k / slices, hi = total * (k + 1) / slices;
    copy_range(lo, lo + (hi - lo) / parts);
    done[k].fetch_add(1, std::memory_order_release);
    while (done[k].load(std::memory_order_acquire) < parts) std::this_thread::yield();
    if (d_dst != nullptr && hi > lo && err == cudaSuccess)
      err = cudaMemcpyAsync(d_dst + lo, dst + lo, 4 * static_cast<size_t>(hi - lo), cudaMemcpyHostToDevice,
                            akv_stream(stream));
  }
  for (auto& th : pool) th.join();
  if (err != cudaSuccess) return akv_cuda_fail(err, "akv_gather_upload: copy");
  return AKV_OK;
}

extern "C" int akv_prepare(void) {
  if (int rc = akv_blocks_prepare()) return rc;
  if (int rc = akv_alloc_prepare()) return rc;
  if (int rc = akv_tree_prepare()) return rc;
  if (int rc = akv_kvio_prepare()) return rc;
  if (int rc = akv_agents_prepare()) return rc;
  return akv_fanout_prepare();
}
