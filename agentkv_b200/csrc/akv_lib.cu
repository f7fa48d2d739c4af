// akv_lib.cu — library-level entry points: version, last error, status reset.
#include <algorithm>
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
  // each thread copies whole arrays, about total / threads tokens in all
  auto work = [&](int32_t t, int32_t parts) {
    const int64_t lo_tok = total * t / parts, hi_tok = total * (t + 1) / parts;
    const int32_t a = static_cast<int32_t>(std::upper_bound(off.begin(), off.end(), lo_tok) - off.begin()) - 1;
    for (int32_t i = std::max(a, 0); i < n && off[i] < hi_tok; ++i) {
      if (off[i] < lo_tok) continue;  // starts in the previous thread's share
      if (lens[i]) std::memcpy(dst + off[i], reinterpret_cast<const int32_t*>(src[i]), 4 * static_cast<size_t>(lens[i]));
    }
  };
  const int32_t parts = total < (1 << 16) ? 1 : threads;
  if (parts == 1) {
    work(0, 1);
  } else {
    std::vector<std::thread> pool;
    pool.reserve(parts - 1);
    for (int32_t t = 1; t < parts; ++t) pool.emplace_back(work, t, parts);
    work(0, parts);
    for (auto& th : pool) th.join();
  }
  if (d_dst != nullptr && total > 0) {
    const cudaError_t e = cudaMemcpyAsync(d_dst, dst, 4 * static_cast<size_t>(total), cudaMemcpyHostToDevice,
                                          akv_stream(stream));
    if (e != cudaSuccess) return akv_cuda_fail(e, "akv_gather_upload: copy");
  }
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
