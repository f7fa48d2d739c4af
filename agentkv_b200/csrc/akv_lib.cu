// akv_lib.cu — library-level entry points: version, last error, status reset.
#include <cstdarg>
#include <cstring>

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

extern "C" int akv_prepare(void) {
  if (int rc = akv_blocks_prepare()) return rc;
  if (int rc = akv_alloc_prepare()) return rc;
  if (int rc = akv_tree_prepare()) return rc;
  if (int rc = akv_kvio_prepare()) return rc;
  if (int rc = akv_agents_prepare()) return rc;
  return akv_fanout_prepare();
}
