// attention_static.cu — b200k_attention_static: kernel.ts:365-373's attention for one query token, with its
// scratch in this file's own device array instead of memory the caller hands over.
//
// For callers that cannot allocate device memory at the point of the call. cudaMalloc is forbidden while a stream
// is being captured into a graph, it can synchronize the whole device (a stall a latency-bound caller cannot
// afford), and some embedders own a fixed device budget that a library must not grow. Such a caller still passes
// its inputs and outputs; the softmax weights live in STATIC_SCRATCH_FLOATS floats reserved here.
//
// Costs and rules:
//  - every GPU that loads this library holds the array (4 MiB) until the process exits;
//  - the first call on a device looks the array's device address up (cudaGetSymbolAddress) with that device
//    current, so make that first call before any stream capture;
//  - every call shares the one array: calls that overlap on the GPU (other streams, other threads) race, so
//    serialize them;
//  - nothing in the array must start at zero (each call writes every weight it reads first), and it keeps the last
//    call's weights afterwards;
//  - nh * (pos + 1) above STATIC_SCRATCH_FLOATS is refused with B200FWD_EINVAL, and so is pos + 1 above
//    MAX_POSITIONS (51200: the softmax of one head holds a row of weights in a block's shared memory);
//  - the array's address is kept for the life of the process: a host that calls cudaDeviceReset after using this
//    entry must not call it again in that process (the address it kept may no longer be the array's).
#include <mutex>
#include <string>

#include "common.h"
#include "kernels.h"

namespace {

constexpr int64_t STATIC_SCRATCH_FLOATS = 1 << 20;  // 4 MiB: e.g. 32 heads at 32768 positions
constexpr int64_t MAX_POSITIONS = 51200;             // 200 KiB of one block's shared memory, 4 bytes a weight

// the scratch, one per device; its name in host code is not a device address (see scratch_on_current_device)
static __device__ __align__(256) float static_scratch[STATIC_SCRATCH_FLOATS];

constexpr int MAX_DEVICES = 64;
float *scratch_address[MAX_DEVICES];
std::mutex scratch_mutex;

// the array's address on the current device, looked up once per device
int scratch_on_current_device(float **out) {
  int device = 0;
  B200_CUDA(cudaGetDevice(&device));
  if (device < 0 || device >= MAX_DEVICES) return b200::fail(B200FWD_EINVAL, "attention_static: device ordinal past 63");
  std::lock_guard<std::mutex> lock(scratch_mutex);
  if (!scratch_address[device]) {
    float *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void **>(&p), static_scratch);
    if (e != cudaSuccess) return b200::cuda_fail(e, "cudaGetSymbolAddress(static_scratch)");
    scratch_address[device] = p;
  }
  *out = scratch_address[device];
  return 0;
}

}  // namespace

extern "C" int b200k_attention_static(float *out, const float *q, const void *kc, const void *vc, int32_t pos,
                                      int32_t nh, int32_t nkv, int32_t hs, int32_t h0, int32_t h1, int32_t half,
                                      b200fwd_stream stream) {
  try {
    if (!out || !q || !kc || !vc) return b200::fail(B200FWD_EINVAL, "attention_static: null pointer");
    if (pos < 0 || nh < 1 || nkv < 1 || nh % nkv || hs < 1 || h0 < 0 || h1 > nh || h0 > h1)
      return b200::fail(B200FWD_EINVAL, "attention_static: bad sizes");
    const int64_t count = (int64_t)pos + 1;
    if (count > MAX_POSITIONS)
      return b200::fail(B200FWD_EINVAL, "attention_static: pos + 1 = " + std::to_string(count) + " positions, above " +
                                            std::to_string(MAX_POSITIONS) + " (a softmax row in one block)");
    if ((int64_t)nh * count > STATIC_SCRATCH_FLOATS)
      return b200::fail(B200FWD_EINVAL, "attention_static: nh * (pos + 1) = " + std::to_string((int64_t)nh * count) +
                                            " floats of scratch, above this entry's fixed " +
                                            std::to_string(STATIC_SCRATCH_FLOATS) +
                                            " (use b200k_attention with scratch of your own)");
    if (h0 == h1) return 0;
    float *att = nullptr;
    const int rc = scratch_on_current_device(&att);
    if (rc) return rc;
    return b200::launch_attention(out, nh * hs, q, nh * hs, kc, vc, att, nullptr, nullptr, pos, nullptr, 1, 1, 0,
                                  pos + 1, pos + 1, nh, nkv, hs, h0, h1, half ? 1 : 0, b200::as_stream(stream));
  } catch (...) {
    return b200::fail(B200FWD_EINVAL, "attention_static: exception");
  }
}
