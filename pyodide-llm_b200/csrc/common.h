// common.h — host-side plumbing shared by the kernels and the engine: the thread's last error message, CUDA status
// checks that turn into B200FWD_E* codes, and the count of kernels launched.
#pragma once

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <string>
#include <utility>

#include <cuda_runtime.h>

#include "../../include/b200fwd.h"

namespace b200 {

// the message b200fwd_last_error() returns (one per calling thread)
std::string &last_error();
int fail(int code, const std::string &message);
// a CUDA status as a B200FWD code with the call named in the message
int cuda_fail(cudaError_t e, const char *what);
// every kernel this library launches is counted here (graph replays add their node counts)
extern std::atomic<uint64_t> launches;

inline cudaStream_t as_stream(b200fwd_stream s) { return reinterpret_cast<cudaStream_t>(s); }

// Programmatic dependent launch: a kernel launched by launch() may be scheduled while the kernel before it in the
// stream is still running; it waits (griddepcontrol.wait, in pdl_begin / pdl_wait) for that kernel to complete and
// its writes to be visible before it touches memory another kernel writes. The environment variable B200FWD_PDL=0
// turns the attribute off (plain stream order; the waits then return at once).
bool pdl_on();

// kernel<<<grid, block, smem, stream>>>(args...) with the programmatic-serialization attribute; a bad configuration
// is left in cudaGetLastError() for B200_LAUNCHED
template <typename... KArgs, typename... Args>
inline void launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                   Args &&...args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_on() ? 1 : 0;
  (void)cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace b200

#ifdef __CUDACC__
// the next kernel in the stream may be scheduled once every block of this one has started
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// until the kernel before this one in the stream has completed and its writes are visible
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// the first statement of every kernel launched by launch(): nothing before it reads or writes global memory
__device__ __forceinline__ void pdl_begin() {
  pdl_launch_dependents();
  pdl_wait();
}
#endif

#define B200_CUDA(call)                                                   \
  do {                                                                    \
    cudaError_t e_ = (call);                                              \
    if (e_ != cudaSuccess) return ::b200::cuda_fail(e_, #call);           \
  } while (0)

// after a launch: the launch's own error (a bad configuration), counted when it went
#define B200_LAUNCHED(what)                                                 \
  do {                                                                      \
    cudaError_t e_ = cudaGetLastError();                                    \
    if (e_ != cudaSuccess) return ::b200::cuda_fail(e_, what);              \
    ::b200::launches.fetch_add(1, std::memory_order_relaxed);               \
  } while (0)
