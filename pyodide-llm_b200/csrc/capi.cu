// capi.cu — the kernel entry points of include/b200fwd.h (b200k_*): the exports of kernels/kernel.ts and
// kernels/kernel_relaxed.ts (public/jobs.js:56-62 lists them), as sm_100a kernels on device pointers.
#include <cmath>
#include <string>

#include "common.h"
#include "gemm_tc.h"
#include "kernels.h"

namespace {
// the tensor-core kernel's wait-gave-up word for the kernel entry points
__device__ int capi_tc_error;
}  // namespace

using namespace b200;

namespace {

template <typename F>
int guarded(F &&f) {
  try {
    return f();
  } catch (...) {
    return fail(B200FWD_EINVAL, "exception in a kernel entry");
  }
}

int matmul(float *xout, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws, const int32_t *wc,
           int32_t n, int32_t r0, int32_t r1, int32_t count, int64_t out_stride, int64_t q_stride, int64_t s_stride,
           bool relaxed, b200fwd_stream stream) {
  if (!xout || !xq || !xs || !wq || !ws) return fail(B200FWD_EINVAL, "matmul: null pointer");
  if (n <= 0 || n % 32) return fail(B200FWD_EINVAL, "matmul: n must be whole groups of 32");
  if (r0 < 0 || r1 < r0 || count < 1) return fail(B200FWD_EINVAL, "matmul: bad rows or count");
  if (r1 == r0) return 0;
  if (q_stride % 16 || (reinterpret_cast<uintptr_t>(xq) % 16) || (reinterpret_cast<uintptr_t>(wq) % 16))
    return fail(B200FWD_EINVAL, "matmul: weights and activations must be 16-byte aligned (16-byte loads)");
  MatJobs jobs{};
  const int ng = n / 32;
  jobs.job[0] = {wq + (int64_t)r0 * n, ws + (int64_t)r0 * ng, wc ? wc + (int64_t)r0 * ng : nullptr, xout + r0, r1 - r0,
                 0, out_stride};
  jobs.njobs = 1;
  jobs.n = n;
  jobs.total_rows = r1 - r0;
  return launch_matvec(jobs, xq, xs, q_stride, s_stride, 1, count, relaxed, as_stream(stream));
}

}  // namespace

extern "C" {

int b200k_quantize_x(int8_t *xq, float *xs, const float *x, int32_t n, int32_t bias, int32_t count, int64_t x_stride,
                     int64_t q_stride, int64_t s_stride, b200fwd_stream stream) {
  return guarded([&] {
    if (bias != 0 && bias != 64) return fail(B200FWD_EINVAL, "quantize_x: bias must be 0 or 64");
    return launch_quantize(x, x_stride, n, bias, count, xq, q_stride, xs, s_stride, 1, as_stream(stream));
  });
}

int b200k_int8_sums(int32_t *out, const int8_t *w, int64_t groups, b200fwd_stream stream) {
  return guarded([&] { return launch_int8_sums(out, w, groups, as_stream(stream)); });
}

int b200k_matmul_q8r(float *xout, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws,
                     const int32_t *wc, int32_t n, int32_t r0, int32_t r1, int32_t count, int64_t out_stride,
                     int64_t q_stride, int64_t s_stride, b200fwd_stream stream) {
  return guarded([&] {
    return matmul(xout, xq, xs, wq, ws, wc, n, r0, r1, count, out_stride, q_stride, s_stride, true, stream);
  });
}

int b200k_matmul_q8s(float *xout, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws,
                     int64_t ws_stride, int32_t n, int32_t rows, int32_t count, int64_t out_stride, int64_t q_stride,
                     int64_t s_stride, b200fwd_stream stream) {
  return guarded([&] {
    if (!xout || !xq || !xs || !wq || !ws) return fail(B200FWD_EINVAL, "matmul_q8s: null pointer");
    if (n <= 0 || n % 32 || rows < 0 || count < 0) return fail(B200FWD_EINVAL, "matmul_q8s: bad sizes");
    if (rows == 0 || count == 0) return 0;
    if (q_stride % 16 || (reinterpret_cast<uintptr_t>(xq) % 16) || (reinterpret_cast<uintptr_t>(wq) % 16))
      return fail(B200FWD_EINVAL, "matmul_q8s: weights and activations must be 16-byte aligned");
    if (ws_stride == 0) ws_stride = n / 32;
    if (ws_stride < n / 32) return fail(B200FWD_EINVAL, "matmul_q8s: ws_stride below n / 32");
    cudaStream_t st = as_stream(stream);
    // the tensor cores need whole TMA boxes and scale rows of whole 16 bytes: else the CUDA cores
    if (count < 16 || n < 128 || rows < 128 || ws_stride % 4 || (reinterpret_cast<uintptr_t>(ws) % 16)) {
      MatJobs jobs{};
      jobs.job[0] = {wq, ws, nullptr, xout, rows, 0, out_stride, (int)ws_stride};
      jobs.njobs = 1;
      jobs.n = n;
      jobs.total_rows = rows;
      jobs.signed_input = 1;
      return launch_matvec(jobs, xq, xs, q_stride, s_stride, 1, count, true, st);
    }
    int *err = nullptr;
    B200_CUDA(cudaGetSymbolAddress((void **)&err, capi_tc_error));
    const int sms = gemm_sms();
    if (sms < 0) return sms;
    // the token maps hold exactly `count` rows: tiles no wider than the tokens (past 16)
    const int widest = count >= 64 ? 64 : count >= 32 ? 32 : 16;
    const int bn = choose_gemm_bn(rows, count, sms, widest);
    // the kernel reads the activation scales one row per group: a stream-ordered copy in that layout
    const int64_t tstride = (count + 3) / 4 * 4;
    float *xs_g = nullptr;
    B200_CUDA(cudaMallocAsync((void **)&xs_g, (size_t)tstride * (n / 32) * 4, st));
    struct Free {
      float *p;
      cudaStream_t s;
      ~Free() { cudaFreeAsync(p, s); }
    } free_xs{xs_g, st};
    // the error word starts this call at 0, in stream order (calls that overlap on the GPU share it: see the header)
    B200_CUDA(cudaMemsetAsync(err, 0, 4, st));
    int rc = launch_scales_by_group(xs_g, tstride, xs, s_stride, count, n / 32, st);
    GemmArgs a{};
    a.out = xout;
    a.error = err;
    a.n = n;
    a.rows = rows;
    a.count = count;
    a.w_row0 = 0;
    a.out_stride = out_stride;
    a.accumulate = 0;
    GemmMaps maps;
    if (!rc && gemm_lanes_enabled() && gemm_lanes_fits(n, rows, count) &&
        gemm_lanes_pays(rows, count, n, sms, widest)) {
      // n a multiple of 128 and few row tiles: the lane-split kernel (a cluster of four CTAs per tile)
      const int lbn = choose_lanes_bn(count, widest);
      rc = make_lane_weight_maps(&maps.w, &maps.ws, wq, ws, n, rows, ws_stride);
      if (!rc) rc = make_lane_token_maps(&maps.x, &maps.xs, xq, xs_g, count, q_stride, n, tstride, lbn);
      if (!rc) rc = launch_gemm_lanes(maps, a, lbn, st);
    } else {
      if (!rc) rc = make_i8_map(&maps.w, wq, n, rows, n, 128);
      if (!rc) rc = make_i8_map(&maps.x, xq, n, count, q_stride, bn);
      if (!rc) rc = make_scale_map(&maps.ws, ws, ws_stride, rows, ws_stride, 128);
      if (!rc) rc = make_token_scale_map(&maps.xs, xs_g, count, n / 32, tstride, bn);
      if (!rc) rc = launch_gemm_tc(maps, a, bn, st);
    }
    if (rc) return rc;
    int32_t e = 0;
    B200_CUDA(cudaMemcpyAsync(&e, err, 4, cudaMemcpyDeviceToHost, st));
    B200_CUDA(cudaStreamSynchronize(st));
    if (e) return fail(B200FWD_ETIMEOUT, "matmul_q8s: a tensor-core pipeline wait gave up (code " + std::to_string(e) + ")");
    return 0;
  });
}

int b200k_matmul_q8(float *xout, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws, int32_t n,
                    int32_t r0, int32_t r1, int32_t count, int64_t out_stride, int64_t q_stride, int64_t s_stride,
                    b200fwd_stream stream) {
  return guarded([&] {
    return matmul(xout, xq, xs, wq, ws, nullptr, n, r0, r1, count, out_stride, q_stride, s_stride, false, stream);
  });
}

int b200k_rmsnorm(float *out, const float *x, const float *w, int32_t n, float eps, int32_t count, int64_t stride,
                  b200fwd_stream stream) {
  return guarded([&] { return launch_rmsnorm(out, x, w, n, eps, count, stride, as_stream(stream)); });
}

int b200k_rope(float *v, const float *fcr, const float *fci, int32_t nh, int32_t hs, int32_t rot,
               b200fwd_stream stream) {
  return guarded([&] {
    if (hs % 2) return fail(B200FWD_EINVAL, "rope: the head size must be even");
    return launch_rope(v, fcr, fci, nh, hs, rot, as_stream(stream));
  });
}

int b200k_attention(float *out, const float *q, const void *kc, const void *vc, float *att, int32_t pos, int32_t nh,
                    int32_t nkv, int32_t hs, int32_t h0, int32_t h1, int32_t half, b200fwd_stream stream) {
  return guarded([&] {
    if (pos < 0 || nh < 1 || nkv < 1 || nh % nkv || hs < 1 || h0 < 0 || h1 > nh || h0 > h1)
      return fail(B200FWD_EINVAL, "attention: bad sizes");
    if (h0 == h1) return 0;
    return launch_attention(out, nh * hs, q, nh * hs, kc, vc, att, nullptr, nullptr, pos, nullptr, 1, 1, 0, pos + 1,
                            pos + 1, nh, nkv, hs, h0, h1, half ? 1 : 0, as_stream(stream));
  });
}

int b200k_matmul_plan(int32_t rows, int32_t n, int32_t count, int32_t sms, int32_t widest, int32_t *lane_split,
                      int32_t *tile_tokens) {
  return guarded([&] {
    if (rows < 1 || n < 32 || n % 32 || count < 2 || sms < 1 || !(widest == 16 || widest == 32 || widest == 64) ||
        !lane_split || !tile_tokens)
      return fail(B200FWD_EINVAL, "matmul_plan: bad arguments");
    // the engine's rule (engine.cu matmul): the lane split where it fits and its estimate is the lower
    const bool lanes = widest == 64 && gemm_lanes_enabled() && gemm_lanes_fits(n, rows, count) &&
                       gemm_lanes_pays(rows, count, n, sms, widest);
    *lane_split = lanes ? 1 : 0;
    *tile_tokens = lanes ? choose_lanes_bn(count, widest) : choose_gemm_bn(rows, count, sms, widest);
    return 0;
  });
}

int b200k_attention_batch(float *out, const float *q, const void *kc, const void *vc, float *att, const int32_t *seq,
                          const int32_t *pos, int32_t n, int64_t seq_stride, int32_t scratch_positions, int32_t nh,
                          int32_t nkv, int32_t hs, int32_t half, b200fwd_stream stream) {
  return guarded([&] {
    if (!seq || !pos || n < 0 || nh < 1 || nkv < 1 || nh % nkv || scratch_positions < 1)
      return fail(B200FWD_EINVAL, "attention_batch: bad arguments");
    return launch_attention(out, nh * hs, q, nh * hs, kc, vc, att, seq, pos, 0, nullptr, n, n, seq_stride,
                            scratch_positions, scratch_positions, nh, nkv, hs, 0, nh, half ? 1 : 0, as_stream(stream));
  });
}

int b200k_to_f16(uint16_t *out, const float *x, int64_t n, b200fwd_stream stream) {
  return guarded([&] { return launch_to_f16(out, x, n, as_stream(stream)); });
}

int b200k_from_f16(float *out, const uint16_t *x, int64_t n, b200fwd_stream stream) {
  return guarded([&] { return launch_from_f16(out, x, n, as_stream(stream)); });
}

int b200k_swiglu(float *out, const float *h1, const float *h3, int64_t n, b200fwd_stream stream) {
  return guarded([&] { return launch_swiglu(out, h1, h3, n, as_stream(stream)); });
}

int b200k_add_inplace(float *x, const float *y, int64_t n, b200fwd_stream stream) {
  return guarded([&] { return launch_add_inplace(x, y, n, as_stream(stream)); });
}

int b200k_add_columns(float *y, const float *rows, const float *a, int32_t count, int32_t n, b200fwd_stream stream) {
  return guarded([&] { return launch_add_columns(y, n, rows, a, count, count, n, 1, as_stream(stream)); });
}

int b200k_penalize(float *logits, const int32_t *tokens, int32_t count, float penalty, b200fwd_stream stream) {
  return guarded([&] {
    if (count < 0 || (count && (!logits || !tokens))) return fail(B200FWD_EINVAL, "penalize: bad arguments");
    if (count == 0) return 0;
    return launch_penalize(logits, 0, tokens, count, nullptr, penalty, nullptr, 1, as_stream(stream));
  });
}

int b200k_sample_scratch(int32_t n, uint64_t *bytes) {
  if (n < 1 || !bytes) return fail(B200FWD_EINVAL, "sample_scratch: bad arguments");
  *bytes = sample_scratch_words(n) * 4 + sample_stack_words() * 4;
  return 0;
}

int b200k_sample(int32_t *out, const float *logits, int32_t n, float temperature, float topp, double random,
                 void *scratch, b200fwd_stream stream) {
  return guarded([&] {
    if (!out || !logits || !scratch || n < 1) return fail(B200FWD_EINVAL, "sample: bad arguments");
    if (reinterpret_cast<uintptr_t>(scratch) % 8) return fail(B200FWD_EINVAL, "sample: scratch must be 8-byte aligned");
    float *probs = reinterpret_cast<float *>(scratch);
    int32_t *stack = reinterpret_cast<int32_t *>(probs + sample_scratch_words(n));
    return launch_sample(out, logits, 0, n, temperature, topp, nullptr, random, 0, nullptr, probs, stack, nullptr, 1,
                         as_stream(stream));
  });
}

int b200k_prefill_attention_scratch(int32_t batch, int32_t seq, int32_t heads, int32_t kv_heads, int32_t head_size,
                                    uint64_t *bytes) {
  if (!bytes || batch < 1 || seq < 1 || heads < 1 || kv_heads < 1 || head_size < 1)
    return fail(B200FWD_EINVAL, "prefill_attention_scratch: bad arguments");
  *bytes = prefill_attention_scratch(batch, seq, heads, kv_heads, head_size);
  return 0;
}

int b200k_prefill_attention(float *out, const float *q, const float *k, const float *v, const float *fcr,
                            const float *fci, int32_t batch, int32_t seq, int32_t heads, int32_t kv_heads,
                            int32_t head_size, void *scratch, b200fwd_stream stream) {
  return guarded([&] {
    if (!out || !q || !k || !v || !fcr || !fci || !scratch) return fail(B200FWD_EINVAL, "prefill_attention: null");
    // kernel.ts:454 isq = 1 / sqrt(hs), in float32
    const float isq = 1.0f / sqrtf((float)head_size);
    return launch_prefill_attention(out, q, k, v, fcr, fci, batch, seq, heads, kv_heads, head_size, isq, scratch,
                                    as_stream(stream));
  });
}

int b200k_prefill_attention_check(const void *scratch, int32_t batch, int32_t seq, int32_t heads, int32_t kv_heads,
                                  int32_t head_size, b200fwd_stream stream) {
  return guarded([&] {
    if (!scratch) return fail(B200FWD_EINVAL, "prefill_attention_check: null scratch");
    return check_prefill_attention(scratch, batch, seq, heads, kv_heads, head_size, as_stream(stream));
  });
}

int b200k_argmax(int32_t *out, const float *x, int32_t n, b200fwd_stream stream) {
  return guarded([&] {
    if (n < 1) return fail(B200FWD_EINVAL, "argmax: no values");
    return launch_argmax(out, x, n, n, 1, 0, as_stream(stream));
  });
}

}  // extern "C"
