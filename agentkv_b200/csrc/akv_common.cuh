// akv_common.cuh — shared helpers for the sm_100a kernels behind the C ABI.
#pragma once

#include <cstdint>
#include <cstdio>
#include <cuda_runtime.h>

#include "agentkv_b200.h"

#define AKV_VERSION_MAJOR 0
#define AKV_VERSION_MINOR 3

#define AKV_DEV __device__ __forceinline__
#define AKV_HD __host__ __device__ __forceinline__

constexpr int kAkvMaxFanoutLevels = AKV_MAX_FANOUT_LEVELS;

// Number of SMs on a B200; grids are sized in multiples of it.
constexpr int kAkvSMs = 148;

// Upper bound for any bounded device wait, in nanoseconds of %globaltimer.
constexpr uint64_t kAkvWaitLimitNs = 2000000000ull;  // 2 s

// ── device status ──────────────────────────────────────────────────────────
// The first error wins the CAS; its details are written by the winner only.
AKV_DEV void akv_fail(AkvStatus* st, int32_t code, int32_t index, int32_t id,
                      int32_t observed, int64_t aux = 0) {
  if (st == nullptr) return;
  if (atomicCAS(&st->code, 0, code) == 0) {
    st->index = index;
    st->id = id;
    st->observed = observed;
    st->aux = aux;
  }
}

// True when an earlier kernel (or this one) recorded an error.
AKV_DEV bool akv_failed(const AkvStatus* st) {
  if (st == nullptr) return false;
  return *reinterpret_cast<const volatile int32_t*>(&st->code) != 0;
}

AKV_DEV uint64_t akv_globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ── host side error plumbing ───────────────────────────────────────────────
void akv_set_error(const char* fmt, ...);
int akv_cuda_fail(cudaError_t err, const char* what);

// Loads a kernel into the current device's context now rather than at its
// first launch (CUDA 12 loads kernels lazily by default); used by
// akv_prepare so that no first launch happens inside a stream capture.
inline int akv_load_kernel(const void* fn, const char* name) {
  cudaFuncAttributes attr;
  const cudaError_t e = cudaFuncGetAttributes(&attr, fn);
  if (e != cudaSuccess) return akv_cuda_fail(e, name);
  return 0;
}

// Per-file halves of akv_prepare: load every kernel, set attributes.
int akv_blocks_prepare();
int akv_alloc_prepare();
int akv_tree_prepare();
int akv_fanout_prepare();
int akv_kvio_prepare();
int akv_agents_prepare();

#define AKV_ARG_CHECK(cond, ...)              \
  do {                                        \
    if (!(cond)) {                            \
      akv_set_error(__VA_ARGS__);             \
      return AKV_ERR_INVALID_ARG;             \
    }                                         \
  } while (0)

// Checks the launch that was just enqueued.
#define AKV_LAUNCH_CHECK(what)                                   \
  do {                                                           \
    cudaError_t _e = cudaGetLastError();                         \
    if (_e != cudaSuccess) return akv_cuda_fail(_e, (what));     \
  } while (0)

inline cudaStream_t akv_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline int akv_ceil_div(int64_t a, int64_t b) { return static_cast<int>((a + b - 1) / b); }
