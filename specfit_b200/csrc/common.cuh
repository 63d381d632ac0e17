// Shared helpers for the specfit_b200 CUDA library (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdlib>
#include <string>
#include <utility>

#include "specfit_b200.h"

namespace sf {

// Records a message for sf_last_error() and returns the status unchanged.
int set_error(int status, const char* fmt, ...);
inline int ok() { return SF_OK; }

#define SF_CHECK_ARG(cond, ...)                                   \
  do {                                                            \
    if (!(cond)) return ::sf::set_error(SF_ERR_INVALID_ARGUMENT, __VA_ARGS__); \
  } while (0)

#define SF_CHECK_CUDA(expr)                                                        \
  do {                                                                             \
    cudaError_t _e = (expr);                                                       \
    if (_e != cudaSuccess)                                                         \
      return ::sf::set_error(SF_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,          \
                             cudaGetErrorString(_e), __FILE__, __LINE__);          \
  } while (0)

#define SF_CHECK_LAUNCH() SF_CHECK_CUDA(cudaGetLastError())

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int num_sms();  // cached SM count of the current device

// Runs f() once per device (per `done` flag word); later calls on that device
// return SF_OK without calling f.  f must be idempotent: two threads may race
// to run it the first time.
template <typename F>
int once_per_device(std::atomic<unsigned long long>& done, F&& f) {
  int dev = 0;
  SF_CHECK_CUDA(cudaGetDevice(&dev));
  const unsigned long long bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return SF_OK;
  const int rc = f();
  if (rc == SF_OK) done.fetch_or(bit, std::memory_order_release);
  return rc;
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch.
//
// The kernels of a verify pass run back to back on one stream, most of them
// for a few microseconds.  Launched with programmatic stream serialization,
// a kernel's CTAs are scheduled while its predecessor is still running and
// block in pdl_wait() until the predecessor has completed and its writes
// are visible, so launch and rasterisation overlap the predecessor's tail.
// Every kernel launched this way calls pdl_wait() before its first global
// memory access (and before any early return), which also keeps the chain
// transitive: a kernel's completion implies its predecessors'.  Each calls
// pdl_trigger() right after, letting its own successor be scheduled once
// all of its CTAs are resident.  Without the launch attribute both are
// no-ops.  SF_PDL=0 in the environment launches everything plainly.

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

inline bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("SF_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

// cudaLaunchKernelEx with programmatic stream serialization (when enabled)
// and, if cluster_x > 0, a (cluster_x, cluster_y, 1) cluster shape.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                               cudaStream_t stream, unsigned cluster_x, unsigned cluster_y,
                               Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_x > 0) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = cluster_y;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster3(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                cudaStream_t stream, dim3 cluster, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  attr[n].id = cudaLaunchAttributeClusterDimension;
  attr[n].val.clusterDim.x = cluster.x;
  attr[n].val.clusterDim.y = cluster.y;
  attr[n].val.clusterDim.z = cluster.z;
  ++n;
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
  return launch_pdl_cluster(kernel, grid, block, smem, stream, 0u, 0u, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------
// dtype helpers shared by kernels

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// Round an fp32 value to the model dtype and back (identity for fp32).
template <typename T>
__device__ __forceinline__ float round_to(float v) {
  return to_f32(from_f32<T>(v));
}

// SiLU in fp32: v * sigmoid(v) = v / (1 + exp(-v)).
__device__ __forceinline__ float silu_f32(float v) { return v / (1.0f + expf(-v)); }

}  // namespace sf
