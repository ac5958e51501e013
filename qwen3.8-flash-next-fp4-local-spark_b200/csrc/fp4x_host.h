// Host-side helpers shared by the fp4x translation units: status reporting, device facts, PDL launches.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <string>

#include "fp4x.h"

namespace fp4x {

// thread-local message of the last failing call (read through fp4x_last_error_message)
void set_error_message(const std::string& msg);
int fail(int code, const std::string& msg);

struct DeviceFacts {
  int sms;
  int smem_optin;  // max dynamic shared memory per block (opt-in)
  int smem_sm;     // shared memory per multiprocessor
};
const DeviceFacts& device_facts();

// kernels launched (or recorded into a graph under capture) by this library; read by fp4x_launch_count
extern std::atomic<int64_t> g_launches;
// the timeline record of the next launch (kTlWords words), or null when no timeline buffer is installed / it is full
unsigned long long* timeline_next();

// launch with programmatic stream serialization (the kernel may begin while its predecessor drains)
template <typename Kernel, typename... Args>
cudaError_t launch_pdl(Kernel kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
  if (e == cudaSuccess) g_launches.fetch_add(1, std::memory_order_relaxed);
  return e;
}

// the same with a thread-block cluster of (1, cluster_y, 1) CTAs
template <typename Kernel, typename... Args>
cudaError_t launch_pdl_cluster(Kernel kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, int cluster_y,
                               Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = (unsigned)cluster_y;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
  if (e == cudaSuccess) g_launches.fetch_add(1, std::memory_order_relaxed);
  return e;
}

// the same with a thread-block cluster of (cluster_x, 1, 1) CTAs
template <typename Kernel, typename... Args>
cudaError_t launch_pdl_cluster_x(Kernel kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                 int cluster_x, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = (unsigned)cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
  if (e == cudaSuccess) g_launches.fetch_add(1, std::memory_order_relaxed);
  return e;
}

// address of the device error word on the current device (cudaGetSymbolAddress, cached per device)
int* dev_error_ptr();

// raise a kernel's dynamic shared-memory limit once per device
cudaError_t ensure_smem_attr(const void* kernel, int bytes);

inline int check_launch(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return fail(FP4X_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return FP4X_OK;
}

inline bool aligned(const void* p, uintptr_t a) { return ((uintptr_t)p % a) == 0; }

}  // namespace fp4x
