// common.h — host-side plumbing shared by the kernels and the engine: the thread's last error message, CUDA status
// checks that turn into B200FWD_E* codes, and the count of kernels launched.
#pragma once

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <string>

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

}  // namespace b200

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
