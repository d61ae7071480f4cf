// kernels.cu — the hot-path kernels of the forward pass for sm_100a, each the number of its reference kernel to the
// bit (kernels/kernel.ts, kernels/kernel_relaxed.ts), and their launchers.
//
// Built with --fmad=false; every float step is written with the rounding intrinsics of exact.cuh.
#include <algorithm>
#include <cfloat>
#include <cstdint>

#include "common.h"
#include "exact.cuh"
#include "kernels.h"

namespace b200 {

namespace {

constexpr unsigned FULL = 0xffffffffu;
constexpr int MV_WARPS = 8;

__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c) { return __dp4a((int)a, (int)b, c); }

// the exact integer of one group's 32 products
__device__ __forceinline__ int dot_group(const uint4 &wa, const uint4 &wb, const uint4 &xa, const uint4 &xb, int c) {
  c = dp4a(wa.x, xa.x, c);
  c = dp4a(wa.y, xa.y, c);
  c = dp4a(wa.z, xa.z, c);
  c = dp4a(wa.w, xa.w, c);
  c = dp4a(wb.x, xb.x, c);
  c = dp4a(wb.y, xb.y, c);
  c = dp4a(wb.z, xb.z, c);
  return dp4a(wb.w, xb.w, c);
}

// kernel.ts:222-226 dot32's lanes: lane k holds products 2k, 2k+1, 2k+8, 2k+9 of each half of 16
__device__ __forceinline__ void dot32_lanes(const uint4 &wa, const uint4 &wb, const uint4 &xa, const uint4 &xb,
                                            int L[4]) {
  const uint32_t w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
  const uint32_t x[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const int lo = k >> 1;                      // words 0/2 (k = 0, 1) or 1/3 (k = 2, 3) of a half
    const uint32_t sel = (k & 1) ? 0x7632u : 0x5410u;  // the low or high two bytes of each word
    int s = 0;
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const uint32_t ww = __byte_perm(w[4 * h + lo], w[4 * h + lo + 2], sel);
      const uint32_t xx = __byte_perm(x[4 * h + lo], x[4 * h + lo + 2], sel);
      s = dp4a(ww, xx, s);
    }
    L[k] = s;
  }
}

template <typename T>
__device__ __forceinline__ T pick3(int j, T a, T b, T c) { return j == 0 ? a : (j == 1 ? b : c); }

// The int8 matmul of count tokens (MT at a time), one warp a row. Each lane takes groups lane, lane+32, ...: their
// exact integers, each times (weight scale x activation scale) rounded once, go to shared memory; then lanes
// 4t..4t+3 add token t's chains in the reference's order:
//  relaxed (kernel_relaxed.ts:34-67): lane k the groups 4j+k below the last four, the lanes ((0+1)+2)+3, then the
//    groups past the fours one at a time;
//  8-bit (kernel.ts:231-251): lane k dot32's lane k of every group, then ((0+1)+2)+3.
template <int MT, bool RELAXED>
__global__ void __launch_bounds__(MV_WARPS * 32)
    matvec_kernel(MatJobs jobs, const int8_t *__restrict__ xq, const float *__restrict__ xs, int64_t q_stride,
                  int64_t s_stride, int64_t g_stride, int count) {
  pdl_begin();
  constexpr int LANES = RELAXED ? 1 : 4;
  __shared__ float buf[MV_WARPS][MT][LANES][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n = jobs.n, ng = n >> 5, ng4 = ng & ~3;
  const int ct = lane >> 2, ck = lane & 3;
  for (int row = blockIdx.x * MV_WARPS + warp; row < jobs.total_rows; row += gridDim.x * MV_WARPS) {
    int j = 0, r = row;
    if (jobs.njobs > 1 && r >= jobs.job[0].rows) {
      r -= jobs.job[0].rows;
      j = 1;
      if (jobs.njobs > 2 && r >= jobs.job[1].rows) {
        r -= jobs.job[1].rows;
        j = 2;
      }
    }
    const int8_t *wrow = pick3(j, jobs.job[0].w, jobs.job[1].w, jobs.job[2].w) + (int64_t)r * n;
    const int ss = pick3(j, jobs.job[0].sstride, jobs.job[1].sstride, jobs.job[2].sstride);
    const int64_t sstride = ss ? ss : ng;
    const float *srow = pick3(j, jobs.job[0].s, jobs.job[1].s, jobs.job[2].s) + (int64_t)r * sstride;
    const int32_t *cbase = pick3(j, jobs.job[0].c, jobs.job[1].c, jobs.job[2].c);
    const int32_t *crow = cbase ? cbase + (int64_t)r * sstride : nullptr;
    float *out = pick3(j, jobs.job[0].out, jobs.job[1].out, jobs.job[2].out) + r;
    const int64_t ostride = pick3(j, jobs.job[0].out_stride, jobs.job[1].out_stride, jobs.job[2].out_stride);
    const int accumulate = pick3(j, jobs.job[0].accumulate, jobs.job[1].accumulate, jobs.job[2].accumulate);
    for (int t0 = 0; t0 < count; t0 += MT) {
      const int mt = min(MT, count - t0);
      float acc = 0.0f;
      for (int g0 = 0; g0 < ng; g0 += 32) {
        const int g = g0 + lane;
        if (g < ng) {
          const uint4 wa = __ldg(reinterpret_cast<const uint4 *>(wrow + (int64_t)g * 32));
          const uint4 wb = __ldg(reinterpret_cast<const uint4 *>(wrow + (int64_t)g * 32 + 16));
          const float sw = __ldg(srow + g);
          int corr = 0;
          if (RELAXED && !jobs.signed_input) {
            if (crow) {
              corr = __ldg(crow + g);
            } else {
              // -64 times the group's sum (int8_sums, kernel.ts:204-212): dot(w, q) + corr = dot(w, q - 64)
              const uint4 ones = make_uint4(0x01010101u, 0x01010101u, 0x01010101u, 0x01010101u);
              corr = -64 * dot_group(wa, wb, ones, ones, 0);
            }
          }
#pragma unroll
          for (int t = 0; t < MT; t++) {
            if (t < mt) {
              const int8_t *xrow = xq + (int64_t)(t0 + t) * q_stride + (int64_t)g * 32;
              const uint4 xa = *reinterpret_cast<const uint4 *>(xrow);
              const uint4 xb = *reinterpret_cast<const uint4 *>(xrow + 16);
              const float sc = fmul(sw, xs[(int64_t)(t0 + t) * s_stride + (int64_t)g * g_stride]);
              if (RELAXED) {
                const int S = dot_group(wa, wb, xa, xb, corr);
                buf[warp][t][0][lane] = fmul(__int2float_rn(S), sc);
              } else {
                int L[4];
                dot32_lanes(wa, wb, xa, xb, L);
#pragma unroll
                for (int k = 0; k < 4; k++) buf[warp][t][k % LANES][lane] = fmul(__int2float_rn(L[k]), sc);
              }
            }
          }
        }
        __syncwarp();
        if (ct < mt) {
          if (RELAXED) {
#pragma unroll
            for (int i = 0; i < 8; i++)
              if (g0 + ck + 4 * i < ng4) acc = fadd(acc, buf[warp][ct][0][ck + 4 * i]);
          } else {
            for (int i = 0; i < 32 && g0 + i < ng; i++) acc = fadd(acc, buf[warp][ct][ck % LANES][i]);
          }
        }
        __syncwarp();
      }
      const float a1 = __shfl_down_sync(FULL, acc, 1);
      const float a2 = __shfl_down_sync(FULL, acc, 2);
      const float a3 = __shfl_down_sync(FULL, acc, 3);
      if (ck == 0 && ct < mt) {
        float sum = fadd(fadd(fadd(acc, a1), a2), a3);
        if (RELAXED) {
          const int last = ((ng - 1) >> 5) << 5;  // the last round's first group; the tail groups are in it
          for (int g = ng4; g < ng; g++) sum = fadd(sum, buf[warp][ct][0][g - last]);
        }
        float *o = out + (int64_t)(t0 + ct) * ostride;
        *o = accumulate ? fadd(*o, sum) : sum;
      }
      __syncwarp();
    }
  }
}

// one group of 32 values (a lane each) quantized as kernel.ts:129-156: groupMax's lane-class maxima, then the
// scalar comparisons; the scale, its inverse, and each value's rounding
__device__ __forceinline__ void quantize_group(float v, int lane, int bias, int8_t *xq, float *xs, int shift) {
  float m = fabsf(v);
  m = wmax(m, __shfl_xor_sync(FULL, m, 4));
  m = wmax(m, __shfl_xor_sync(FULL, m, 8));
  m = wmax(m, __shfl_xor_sync(FULL, m, 16));
  const float m0 = __shfl_sync(FULL, m, 0), m1 = __shfl_sync(FULL, m, 1);
  const float m2 = __shfl_sync(FULL, m, 2), m3 = __shfl_sync(FULL, m, 3);
  float amax = m0;
  if (m1 > amax) amax = m1;
  if (m2 > amax) amax = m2;
  if (m3 > amax) amax = m3;
  const float scale = fdiv(amax, bias == 0 ? 127.0f : 63.0f);
  const float inv = scale > 0 ? fdiv(1.0f, scale) : 0.0f;
  xq[lane] = (int8_t)(quantize_one(v, inv, bias) - shift);
  if (lane == 0) *xs = scale;
}

// kernel.ts:330-342 rmsnorm's scale: four lane chains over the fours, ((0+1)+2)+3, the rest one by one. The whole
// block squares the vector into shared memory (sq: n floats, each square rounded once as the reference rounds it),
// then four lanes of warp 0 run the lane chains (the chains' adds are the only serial part: each lane reads its next
// sixteen squares while it adds the sixteen before, so the adds follow one another at the add's latency).
constexpr int NORM_MAX = 12288;  // the longest vector a block normalizes (its squares fill 48 KB of shared memory)
__device__ __forceinline__ float norm_scale(const float *x, int n, float eps, float *sq, float *part) {
  if ((reinterpret_cast<uintptr_t>(x) & 15) == 0 && n % 4 == 0) {
    for (int j = threadIdx.x; j < n / 4; j += blockDim.x) {
      const float4 v = reinterpret_cast<const float4 *>(x)[j];
      reinterpret_cast<float4 *>(sq)[j] = make_float4(fmul(v.x, v.x), fmul(v.y, v.y), fmul(v.z, v.z), fmul(v.w, v.w));
    }
  } else {
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
      const float v = x[j];
      sq[j] = fmul(v, v);
    }
  }
  __syncthreads();
  const int n4 = n & ~3;
  if (threadIdx.x < 4) {
    float acc = 0.0f;
    int j = threadIdx.x;
    if (j + 60 < n4) {
      float cur[16];
#pragma unroll
      for (int u = 0; u < 16; u++) cur[u] = sq[j + 4 * u];
      for (; j + 124 < n4; j += 64) {
        float nxt[16];
#pragma unroll
        for (int u = 0; u < 16; u++) nxt[u] = sq[j + 64 + 4 * u];
#pragma unroll
        for (int u = 0; u < 16; u++) acc = fadd(acc, cur[u]);
#pragma unroll
        for (int u = 0; u < 16; u++) cur[u] = nxt[u];
      }
#pragma unroll
      for (int u = 0; u < 16; u++) acc = fadd(acc, cur[u]);
      j += 64;
    }
    for (; j < n4; j += 4) acc = fadd(acc, sq[j]);
    part[threadIdx.x] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float ss = fadd(fadd(fadd(part[0], part[1]), part[2]), part[3]);
    for (int j = n4; j < n; j++) ss = fadd(ss, sq[j]);
    part[4] = fdiv(1.0f, __fsqrt_rn(fadd(fdiv(ss, (float)n), eps)));
  }
  __syncthreads();
  return part[4];
}

__global__ void norm_quantize_kernel(const float *x, int64_t x_stride, const float *w, int n, float eps, int bias,
                                     int8_t *xq, int64_t q_stride, float *xs, int64_t s_stride, int64_t g_stride,
                                     const int32_t *channels, int nch, float *picked, float *out_f,
                                     int64_t out_stride, int shift) {
  pdl_begin();
  __shared__ float part[5];
  extern __shared__ float sq[];
  const int tok = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
  const float *xr = x + (int64_t)tok * x_stride;
  const int ng = n >> 5;
  // this warp's first NQ_PRE groups' values and weights, read before the norm's serial chain (they do not depend on
  // it), so that the quantization after it waits on no memory
  constexpr int NQ_PRE = 4;
  float xv[NQ_PRE], wv[NQ_PRE];
#pragma unroll
  for (int u = 0; u < NQ_PRE; u++) {
    const int g = warp + u * warps;
    xv[u] = g < ng ? xr[g * 32 + lane] : 0.0f;
    wv[u] = g < ng ? w[g * 32 + lane] : 0.0f;
  }
  const float s = norm_scale(xr, n, eps, sq, part);
  auto group = [&](int g, float xj, float wj) {
    const int j = g * 32 + lane;
    float v = fmul(wj, fmul(s, xj));
    if (out_f) out_f[(int64_t)tok * out_stride + j] = v;
    for (int c = 0; c < nch; c++) {
      if (channels[c] == j) {
        picked[(int64_t)tok * nch + c] = v;
        v = 0.0f;
      }
    }
    quantize_group(v, lane, bias, xq + (int64_t)tok * q_stride + g * 32,
                   xs + (int64_t)tok * s_stride + (int64_t)g * g_stride, shift);
  };
#pragma unroll
  for (int u = 0; u < NQ_PRE; u++) {
    const int g = warp + u * warps;
    if (g < ng) group(g, xv[u], wv[u]);
  }
  for (int g = warp + NQ_PRE * warps; g < ng; g += warps) group(g, xr[g * 32 + lane], w[g * 32 + lane]);
}

__global__ void rmsnorm_kernel(float *out, const float *x, const float *w, int n, float eps, int64_t stride) {
  pdl_begin();
  __shared__ float part[5];
  extern __shared__ float sq[];
  const float *xr = x + (int64_t)blockIdx.x * stride;
  const float s = norm_scale(xr, n, eps, sq, part);
  for (int j = threadIdx.x; j < n; j += blockDim.x) out[(int64_t)blockIdx.x * stride + j] = fmul(w[j], fmul(s, xr[j]));
}

__global__ void rope_kernel(float *v, const float *fcr, const float *fci, int nh, int hs, int rot) {
  pdl_begin();
  const int turned = rot > 0 && rot < hs ? rot : hs;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  const int h = idx / (turned / 2), i = 2 * (idx % (turned / 2));
  if (h >= nh) return;
  float *base = v + h * hs + i;
  const float v0 = base[0], v1 = base[1], c = fcr[i >> 1], s = fci[i >> 1];
  base[0] = fsub(fmul(v0, c), fmul(v1, s));
  base[1] = fadd(fmul(v0, s), fmul(v1, c));
}

// grid (groups / 8 rounded up, tokens): a warp a group of 32
__global__ void quantize_kernel(const float *x, int64_t x_stride, int n, int bias, int count, int8_t *xq,
                                int64_t q_stride, float *xs, int64_t s_stride, int64_t g_stride, int shift) {
  pdl_begin();
  const int lane = threadIdx.x & 31;
  const int g = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), tok = blockIdx.y;
  if (g >= (n >> 5)) return;
  const float v = x[(int64_t)tok * x_stride + g * 32 + lane];
  quantize_group(v, lane, bias, xq + (int64_t)tok * q_stride + g * 32,
                 xs + (int64_t)tok * s_stride + (int64_t)g * g_stride, shift);
}

// kernel.ts:654-667 swiglu (vexp on the fours, fexp after them) feeding quantize_x; grid as quantize_kernel's
__global__ void swiglu_quantize_kernel(const float *h1, const float *h3, int64_t stride, int n, int bias, int count,
                                       int8_t *xq, int64_t q_stride, float *xs, int64_t s_stride, int64_t g_stride, int shift) {
  pdl_begin();
  const int lane = threadIdx.x & 31;
  const int n4 = n & ~3;
  const int g = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), tok = blockIdx.y;
  if (g >= (n >> 5)) return;
  const int j = g * 32 + lane;
  const float v = h1[(int64_t)tok * stride + j];
  const float e = j < n4 ? vexp(-v) : fexp(-v);
  const float o = fmul(fdiv(v, fadd(1.0f, e)), h3[(int64_t)tok * stride + j]);
  quantize_group(o, lane, bias, xq + (int64_t)tok * q_stride + g * 32,
                 xs + (int64_t)tok * s_stride + (int64_t)g * g_stride, shift);
}

// quantize_x of a group of 32 values held four a lane by eight consecutive lanes (lane l % 8 holding values
// 4(l % 8) .. + 3): each of a lane's four values is one of quantize_x's lane classes (index mod 4), so each class's
// largest |value| is a max over the eight lanes (kernel.ts:129-156 groupMax); then the same scalar comparisons,
// scale and rounding as quantize_group. Every lane of the warp calls it (the shuffles); live lanes store their four
// bytes at xq (4-byte aligned) and the group's first lane the scale at *xs.
__device__ __forceinline__ void quantize_four(const float (&o)[4], bool live, int lane, int bias, int shift,
                                              int8_t *xq, float *xs) {
  float m[4];
#pragma unroll
  for (int c = 0; c < 4; c++) {
    m[c] = fabsf(o[c]);
    m[c] = wmax(m[c], __shfl_xor_sync(FULL, m[c], 1));
    m[c] = wmax(m[c], __shfl_xor_sync(FULL, m[c], 2));
    m[c] = wmax(m[c], __shfl_xor_sync(FULL, m[c], 4));
  }
  if (!live) return;
  float amax = m[0];
  if (m[1] > amax) amax = m[1];
  if (m[2] > amax) amax = m[2];
  if (m[3] > amax) amax = m[3];
  const float scale = fdiv(amax, bias == 0 ? 127.0f : 63.0f);
  const float inv = scale > 0 ? fdiv(1.0f, scale) : 0.0f;
  uint32_t packed = 0;
#pragma unroll
  for (int c = 0; c < 4; c++) packed |= (uint32_t)(uint8_t)(int8_t)(quantize_one(o[c], inv, bias) - shift) << (8 * c);
  *reinterpret_cast<uint32_t *>(xq) = packed;
  if ((lane & 7) == 0) *xs = scale;
}

// rmsnorm + quantize_x with four consecutive values a thread (16-byte loads): the norm's scale as
// norm_quantize_kernel computes it, then each thread's values w * (s * x) (and the outlier columns taken out as it
// takes them) quantized by quantize_four, a group on eight lanes, so that a block of 1024 threads quantizes 128
// groups in one pass. One block per token; x rows and w 16-byte aligned, xq rows 4-byte aligned.
__global__ void norm_quantize_v4_kernel(const float *x, int64_t x_stride, const float *w, int n, float eps, int bias,
                                        int8_t *xq, int64_t q_stride, float *xs, int64_t s_stride, int64_t g_stride,
                                        const int32_t *channels, int nch, float *picked, float *out_f,
                                        int64_t out_stride, int shift) {
  pdl_begin();
  __shared__ float part[5];
  extern __shared__ float sq[];
  const int tok = blockIdx.x, lane = threadIdx.x & 31, n4 = n >> 2;
  const float *xr = x + (int64_t)tok * x_stride;
  // the first pass's values and weights, read before the norm's serial chain (they do not depend on it)
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  const bool live0 = (int)threadIdx.x < n4;
  const float4 x0 = live0 ? reinterpret_cast<const float4 *>(xr)[threadIdx.x] : zero;
  const float4 w0 = live0 ? reinterpret_cast<const float4 *>(w)[threadIdx.x] : zero;
  const float s = norm_scale(xr, n, eps, sq, part);
  for (int base = 0; base < n4; base += blockDim.x) {
    const int j4 = base + threadIdx.x;
    const bool live = j4 < n4;
    const float4 xv = base == 0 ? x0 : live ? reinterpret_cast<const float4 *>(xr)[j4] : zero;
    const float4 wv = base == 0 ? w0 : live ? reinterpret_cast<const float4 *>(w)[j4] : zero;
    const float xa[4] = {xv.x, xv.y, xv.z, xv.w}, wa[4] = {wv.x, wv.y, wv.z, wv.w};
    float o[4];
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const int j = 4 * j4 + c;
      float v = fmul(wa[c], fmul(s, xa[c]));
      if (live && out_f) out_f[(int64_t)tok * out_stride + j] = v;
      for (int k = 0; k < nch; k++) {
        if (live && channels[k] == j) {
          picked[(int64_t)tok * nch + k] = v;
          v = 0.0f;
        }
      }
      o[c] = v;
    }
    quantize_four(o, live, lane, bias, shift, xq + (int64_t)tok * q_stride + 4 * j4,
                  xs + (int64_t)tok * s_stride + (int64_t)(j4 >> 3) * g_stride);
  }
}

// quantize_kernel (SWIGLU false: x = h1) and swiglu_quantize_kernel (true) with four consecutive values a thread
// (16-byte loads): eight lanes a group, four groups a warp. A thread's four values are one of each of quantize_x's
// lane classes (index mod 4), so each class's largest |value| is a max over the group's eight lanes; then the same
// scalar comparisons, scale and rounding as quantize_group. grid (groups / 32 rounded up, tokens), 256 threads;
// the input rows 16-byte aligned, the xq rows 4-byte aligned.
template <bool SWIGLU>
__global__ void quantize_v4_kernel(const float *h1, const float *h3, int64_t stride, int n, int bias, int8_t *xq,
                                   int64_t q_stride, float *xs, int64_t s_stride, int64_t g_stride, int shift) {
  pdl_begin();
  const int lane = threadIdx.x & 31, sub = lane & 7;
  const int n4 = n & ~3;
  const int g = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 4 + (lane >> 3), tok = blockIdx.y;
  const bool live = g < (n >> 5);
  const int j = g * 32 + sub * 4;
  float o[4] = {0.f, 0.f, 0.f, 0.f};
  if (live) {
    const float4 a = *reinterpret_cast<const float4 *>(h1 + (int64_t)tok * stride + j);
    const float va[4] = {a.x, a.y, a.z, a.w};
    if (SWIGLU) {
      // kernel.ts:654-667 swiglu (vexp on the fours, fexp after them)
      const float4 b = *reinterpret_cast<const float4 *>(h3 + (int64_t)tok * stride + j);
      const float vb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int c = 0; c < 4; c++) {
        const float e = j + c < n4 ? vexp(-va[c]) : fexp(-va[c]);
        o[c] = fmul(fdiv(va[c], fadd(1.0f, e)), vb[c]);
      }
    } else {
#pragma unroll
      for (int c = 0; c < 4; c++) o[c] = va[c];
    }
  }
  quantize_four(o, live, lane, bias, shift, xq + (int64_t)tok * q_stride + j,
                xs + (int64_t)tok * s_stride + (int64_t)g * g_stride);
}

__global__ void embed_kernel(const int8_t *w, const float *s, int sstride, const int32_t *tokens, int count, int dim,
                             float *x, int64_t x_stride) {
  pdl_begin();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)count * dim) return;
  const int t = (int)(i / dim), j = (int)(i % dim);
  const int64_t row = tokens[t];
  x[(int64_t)t * x_stride + j] = fmul((float)w[row * dim + j], s[row * sstride + j / 32]);
}

__global__ void rope_cache_kernel(float *q, int64_t q_stride, const float *k, const float *v, int64_t kv_stride,
                                  const float *cos, const float *sin, const int32_t *pos, const int32_t *seq,
                                  uint8_t *kc, uint8_t *vc, int64_t seq_stride, int half, int nh, int nkv, int hs,
                                  int rot) {
  pdl_begin();
  const int tok = blockIdx.y;
  const int p = pos[tok];
  const int64_t sq = seq[tok];
  const int hp = hs / 2, kvDim = nkv * hs;
  const int turned = rot > 0 && rot < hs ? rot : hs;
  const float *cr = cos + (int64_t)p * hp, *sr = sin + (int64_t)p * hp;
  const int esize = half ? 2 : 4;
  const int64_t cache_at = (sq * seq_stride + (int64_t)p * kvDim) * esize;
  const int total = (nh + nkv) * hp + kvDim;
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += gridDim.x * blockDim.x) {
    if (idx < (nh + nkv) * hp) {
      const bool isq = idx < nh * hp;
      const int local = isq ? idx : idx - nh * hp;
      const int h = local / hp, i = 2 * (local % hp);
      float v0, v1;
      if (isq) {
        float *base = q + (int64_t)tok * q_stride + h * hs + i;
        v0 = base[0];
        v1 = base[1];
        if (i < turned) {
          const float c = cr[i >> 1], s = sr[i >> 1];
          base[0] = fsub(fmul(v0, c), fmul(v1, s));
          base[1] = fadd(fmul(v0, s), fmul(v1, c));
        }
      } else {
        const float *base = k + (int64_t)tok * kv_stride + h * hs + i;
        v0 = base[0];
        v1 = base[1];
        float o0 = v0, o1 = v1;
        if (i < turned) {
          const float c = cr[i >> 1], s = sr[i >> 1];
          o0 = fsub(fmul(v0, c), fmul(v1, s));
          o1 = fadd(fmul(v0, s), fmul(v1, c));
        }
        const int64_t e = cache_at + (int64_t)(h * hs + i) * esize;
        if (half) {
          reinterpret_cast<uint16_t *>(kc + e)[0] = float_to_half(o0);
          reinterpret_cast<uint16_t *>(kc + e)[1] = float_to_half(o1);
        } else {
          reinterpret_cast<float *>(kc + e)[0] = o0;
          reinterpret_cast<float *>(kc + e)[1] = o1;
        }
      }
    } else {
      const int j = idx - (nh + nkv) * hp;
      const float val = v[(int64_t)tok * kv_stride + j];
      const int64_t e = cache_at + (int64_t)j * esize;
      if (half)
        *reinterpret_cast<uint16_t *>(vc + e) = float_to_half(val);
      else
        *reinterpret_cast<float *>(vc + e) = val;
    }
  }
}

__global__ void add_columns_kernel(float *y, int64_t y_stride, const float *rows, const float *a, int64_t a_stride,
                                   int nc, int n, int count) {
  pdl_begin();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)n * count) return;
  const int tok = (int)(i / n), j = (int)(i % n);
  float v = y[(int64_t)tok * y_stride + j];
  for (int c = 0; c < nc; c++) v = fadd(v, fmul(a[(int64_t)tok * a_stride + c], rows[(int64_t)c * n + j]));
  y[(int64_t)tok * y_stride + j] = v;
}

// (value, index) better than (value2, index2) for argmax: mode 0 kernel.ts's `>` scan (NaN never taken), mode 1
// numpy's (the first NaN wins); ties to the lower index
__device__ __forceinline__ bool better(float a, int ia, float b, int ib, int mode) {
  const bool na = a != a, nb = b != b;
  if (mode == 1) {
    if (na != nb) return na;
    if (na && nb) return ia < ib;
  } else {
    if (na != nb) return nb;
    if (na && nb) return ia < ib;
  }
  if (a != b) return a > b;
  return ia < ib;
}

__global__ void argmax_kernel(int32_t *out, const float *x, int64_t stride, int n, int mode) {
  pdl_begin();
  __shared__ float sv[32];
  __shared__ int si[32];
  const int tok = blockIdx.x;
  const float *r = x + (int64_t)tok * stride;
  float bv = 0.0f;
  int bi = -1;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const float v = r[j];
    if (bi < 0 || better(v, j, bv, bi, mode)) { bv = v; bi = j; }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(FULL, bv, o);
    const int oi = __shfl_xor_sync(FULL, bi, o);
    if (oi >= 0 && (bi < 0 || better(ov, oi, bv, bi, mode))) { bv = ov; bi = oi; }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); w++)
      if (si[w] >= 0 && (bi < 0 || better(sv[w], si[w], bv, bi, mode))) { bv = sv[w]; bi = si[w]; }
    // kernel.ts's scan starts from x[0]: a NaN there is never replaced
    if (mode == 0 && r[0] != r[0]) bi = 0;
    out[tok] = bi;
  }
}

__global__ void gather_rows_kernel(float *dst, int64_t dst_stride, const float *src, int64_t src_stride,
                                   const int32_t *idx, int count, int dim) {
  pdl_begin();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)count * dim) return;
  const int t = (int)(i / dim), j = (int)(i % dim);
  dst[(int64_t)t * dst_stride + j] = src[(int64_t)idx[t] * src_stride + j];
}

// scales of count tokens, one row per token (s_stride apart), into one row per group (t_stride apart)
__global__ void scales_by_group_kernel(float *dst, int64_t t_stride, const float *src, int64_t s_stride, int count,
                                       int groups) {
  pdl_begin();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)count * groups) return;
  const int g = (int)(i / count), t = (int)(i % count);
  dst[(int64_t)g * t_stride + t] = src[(int64_t)t * s_stride + g];
}

__global__ void outlier_columns_kernel(float *cols, const int8_t *w, const float *s, int sstride, int dim, int vocab,
                                       const int32_t *channels, int nch) {
  pdl_begin();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)vocab * nch) return;
  const int c = (int)(i / vocab), v = (int)(i % vocab);
  const int ch = channels[c];
  cols[i] = fmul((float)w[(int64_t)v * dim + ch], s[(int64_t)v * sstride + ch / 32]);
}

__global__ void to_f16_kernel(uint16_t *out, const float *x, int64_t n) {
  pdl_begin();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = float_to_half(x[i]);
}
__global__ void from_f16_kernel(float *out, const uint16_t *x, int64_t n) {
  pdl_begin();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = half_to_float(x[i]);
}
__global__ void add_inplace_kernel(float *x, const float *y, int64_t n) {
  pdl_begin();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) x[i] = fadd(x[i], y[i]);
}
__global__ void swiglu_kernel(float *out, const float *h1, const float *h3, int64_t n) {
  pdl_begin();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = h1[i];
  const float e = i < (n & ~(int64_t)3) ? vexp(-v) : fexp(-v);
  out[i] = fmul(fdiv(v, fadd(1.0f, e)), h3[i]);
}
__global__ void int8_sums_kernel(int32_t *out, const int8_t *w, int64_t groups) {
  pdl_begin();
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= groups) return;
  int s = 0;
  for (int j = 0; j < 32; j++) s += w[g * 32 + j];
  out[g] = -64 * s;
}
__global__ void advance_kernel(int32_t *tokens, int32_t *pos, const int32_t *ids, int32_t *history, int steps,
                               int32_t *step, int count, const float *logits, int64_t vocab, int32_t *bad) {
  pdl_begin();
  const int i = threadIdx.x;
  const int at = *step;
  __syncthreads();
  if (i < count) {
    const int32_t id = ids[i];
    const float v = logits[(int64_t)i * vocab + id];
    // llama2_numpy.greedy (public/llama2_numpy.py:1521-1527): a largest logit that is no finite number stops
    if (!(v == v) || v == INFINITY || v == -INFINITY) atomicExch(bad, 1);
    tokens[i] = id;
    pos[i] += 1;
    if (at < steps) history[(int64_t)i * steps + at] = id;
  }
  if (i == 0) *step = at + 1;
}

#define CHECK_RC(expr)      \
  do {                      \
    int rc_ = (expr);       \
    if (rc_) return rc_;    \
  } while (0)

inline unsigned blocks_for(int64_t n, int threads) { return (unsigned)((n + threads - 1) / threads); }

}  // namespace

int launch_matvec(const MatJobs &jobs, const int8_t *xq, const float *xs, int64_t q_stride, int64_t s_stride,
                  int64_t g_stride, int count, bool relaxed, cudaStream_t stream) {
  if (count <= 0 || jobs.total_rows <= 0) return 0;
  if (jobs.n % 32) return fail(B200FWD_EINVAL, "matvec: n must be whole groups of 32");
  const unsigned grid = std::min<unsigned>(blocks_for(jobs.total_rows, MV_WARPS), 148u * 32u);
  const int mt = count >= 8 ? 8 : count >= 4 ? 4 : count >= 2 ? 2 : 1;
#define B200_MV(MT, R) \
  launch(matvec_kernel<MT, R>, grid, MV_WARPS * 32, 0, stream, jobs, xq, xs, q_stride, s_stride, g_stride, count)
  if (relaxed) {
    switch (mt) {
      case 8: B200_MV(8, true); break;
      case 4: B200_MV(4, true); break;
      case 2: B200_MV(2, true); break;
      default: B200_MV(1, true); break;
    }
  } else {
    switch (mt) {
      case 8: B200_MV(8, false); break;
      case 4: B200_MV(4, false); break;
      case 2: B200_MV(2, false); break;
      default: B200_MV(1, false); break;
    }
  }
#undef B200_MV
  B200_LAUNCHED("matvec_kernel");
  return 0;
}

int launch_norm_quantize(const float *x, int64_t x_stride, const float *w, int n, float eps, int bias, int count,
                         int8_t *xq, int64_t q_stride, float *xs, int64_t s_stride, int64_t g_stride,
                         const int32_t *channels, int nch, float *picked, float *out_f, int64_t out_stride,
                         cudaStream_t stream, int shift) {
  if (count <= 0) return 0;
  if (n % 32) return fail(B200FWD_EINVAL, "rmsnorm+quantize: n must be whole groups of 32");
  if (n > NORM_MAX) return fail(B200FWD_EUNSUPPORTED, "rmsnorm+quantize: vectors above 12288 values");
  // a block per token: the squares and the groups' quantization spread over the block (only the four lane chains of
  // the norm are serial); 1024 threads while the tokens leave SMs free, 256 (more tokens' chains at once) past that
  const int threads = count <= 148 ? 1024 : 256;
  if (reinterpret_cast<uintptr_t>(x) % 16 == 0 && x_stride % 4 == 0 && reinterpret_cast<uintptr_t>(w) % 16 == 0 &&
      reinterpret_cast<uintptr_t>(xq) % 4 == 0 && q_stride % 4 == 0) {
    launch(norm_quantize_v4_kernel, count, threads, (size_t)n * 4, stream, x, x_stride, w, n, eps, bias, xq, q_stride,
           xs, s_stride, g_stride, channels, nch, picked, out_f, out_stride, shift);
    B200_LAUNCHED("norm_quantize_v4_kernel");
    return 0;
  }
  launch(norm_quantize_kernel, count, threads, (size_t)n * 4, stream, x, x_stride, w, n, eps, bias, xq, q_stride, xs,
         s_stride, g_stride, channels, nch, picked, out_f, out_stride, shift);
  B200_LAUNCHED("norm_quantize_kernel");
  return 0;
}

int launch_quantize(const float *x, int64_t x_stride, int n, int bias, int count, int8_t *xq, int64_t q_stride,
                    float *xs, int64_t s_stride, int64_t g_stride, cudaStream_t stream, int shift) {
  if (count <= 0) return 0;
  if (n % 32) return fail(B200FWD_EINVAL, "quantize_x: n must be whole groups of 32");
  if (count > 65535) return fail(B200FWD_EINVAL, "quantize_x: more than 65535 tokens");
  if (reinterpret_cast<uintptr_t>(x) % 16 == 0 && x_stride % 4 == 0 && reinterpret_cast<uintptr_t>(xq) % 4 == 0 &&
      q_stride % 4 == 0) {
    launch(quantize_v4_kernel<false>, dim3(blocks_for(n / 32, 32), count), 256, 0, stream, x, nullptr, x_stride, n,
           bias, xq, q_stride, xs, s_stride, g_stride, shift);
    B200_LAUNCHED("quantize_v4_kernel");
    return 0;
  }
  launch(quantize_kernel, dim3(blocks_for(n / 32, 8), count), 256, 0, stream, x, x_stride, n, bias, count, xq, q_stride,
         xs, s_stride, g_stride, shift);
  B200_LAUNCHED("quantize_kernel");
  return 0;
}

int launch_swiglu_quantize(const float *h1, const float *h3, int64_t stride, int n, int bias, int count, int8_t *xq,
                           int64_t q_stride, float *xs, int64_t s_stride, int64_t g_stride,
                           cudaStream_t stream, int shift) {
  if (count <= 0) return 0;
  if (n % 32) return fail(B200FWD_EINVAL, "swiglu+quantize: n must be whole groups of 32");
  if (count > 65535) return fail(B200FWD_EINVAL, "swiglu+quantize: more than 65535 tokens");
  const bool v4 = reinterpret_cast<uintptr_t>(h1) % 16 == 0 && reinterpret_cast<uintptr_t>(h3) % 16 == 0 &&
                  stride % 4 == 0 && reinterpret_cast<uintptr_t>(xq) % 4 == 0 && q_stride % 4 == 0;
  if (v4) {
    launch(quantize_v4_kernel<true>, dim3(blocks_for(n / 32, 32), count), 256, 0, stream, h1, h3, stride, n, bias, xq,
           q_stride, xs, s_stride, g_stride, shift);
    B200_LAUNCHED("quantize_v4_kernel<swiglu>");
    return 0;
  }
  launch(swiglu_quantize_kernel, dim3(blocks_for(n / 32, 8), count), 256, 0, stream, h1, h3, stride, n, bias, count, xq,
         q_stride, xs, s_stride, g_stride, shift);
  B200_LAUNCHED("swiglu_quantize_kernel");
  return 0;
}

int launch_embed(const int8_t *w, const float *s, int sstride, const int32_t *tokens, int count, int dim, float *x,
                 int64_t x_stride, cudaStream_t stream) {
  if (count <= 0) return 0;
  launch(embed_kernel, blocks_for((int64_t)count * dim, 256), 256, 0, stream, w, s, sstride, tokens, count, dim, x,
         x_stride);
  B200_LAUNCHED("embed_kernel");
  return 0;
}

int launch_rope_cache(float *q, int64_t q_stride, const float *k, const float *v, int64_t kv_stride, const float *cos,
                      const float *sin, const int32_t *pos, const int32_t *seq, int count, void *kc, void *vc,
                      int64_t seq_stride, int half, int nh, int nkv, int hs, int rot, cudaStream_t stream) {
  if (count <= 0) return 0;
  if (hs % 2) return fail(B200FWD_EINVAL, "rope: the head size must be even");
  const int total = (nh + nkv) * (hs / 2) + nkv * hs;
  dim3 grid(blocks_for(total, 256), count);
  launch(rope_cache_kernel, grid, 256, 0, stream, q, q_stride, k, v, kv_stride, cos, sin, pos, seq,
         reinterpret_cast<uint8_t *>(kc), reinterpret_cast<uint8_t *>(vc), seq_stride, half, nh, nkv, hs, rot);
  B200_LAUNCHED("rope_cache_kernel");
  return 0;
}

int launch_rmsnorm(float *out, const float *x, const float *w, int n, float eps, int count, int64_t stride,
                   cudaStream_t stream) {
  if (count <= 0) return 0;
  if (n > NORM_MAX) return fail(B200FWD_EUNSUPPORTED, "rmsnorm: vectors above 12288 values");
  launch(rmsnorm_kernel, count, 256, (size_t)n * 4, stream, out, x, w, n, eps, stride);
  B200_LAUNCHED("rmsnorm_kernel");
  return 0;
}

int launch_rope(float *v, const float *fcr, const float *fci, int nh, int hs, int rot, cudaStream_t stream) {
  const int turned = rot > 0 && rot < hs ? rot : hs;
  const int pairs = nh * (turned / 2);
  if (pairs <= 0) return 0;
  launch(rope_kernel, blocks_for(pairs, 128), 128, 0, stream, v, fcr, fci, nh, hs, rot);
  B200_LAUNCHED("rope_kernel");
  return 0;
}

int launch_add_columns(float *y, int64_t y_stride, const float *rows, const float *a, int64_t a_stride, int nc,
                       int n, int count, cudaStream_t stream) {
  if (count <= 0 || nc <= 0) return 0;
  launch(add_columns_kernel, blocks_for((int64_t)n * count, 256), 256, 0, stream, y, y_stride, rows, a, a_stride, nc, n,
         count);
  B200_LAUNCHED("add_columns_kernel");
  return 0;
}

int launch_argmax(int32_t *out, const float *x, int64_t stride, int n, int count, int mode, cudaStream_t stream) {
  if (count <= 0) return 0;
  launch(argmax_kernel, count, 1024, 0, stream, out, x, stride, n, mode);
  B200_LAUNCHED("argmax_kernel");
  return 0;
}

int launch_gather_rows(float *dst, int64_t dst_stride, const float *src, int64_t src_stride, const int32_t *idx,
                       int count, int dim, cudaStream_t stream) {
  if (count <= 0) return 0;
  launch(gather_rows_kernel, blocks_for((int64_t)count * dim, 256), 256, 0, stream, dst, dst_stride, src, src_stride,
         idx, count, dim);
  B200_LAUNCHED("gather_rows_kernel");
  return 0;
}

int launch_scales_by_group(float *dst, int64_t t_stride, const float *src, int64_t s_stride, int count, int groups,
                           cudaStream_t stream) {
  if (count <= 0 || groups <= 0) return 0;
  launch(scales_by_group_kernel, blocks_for((int64_t)count * groups, 256), 256, 0, stream, dst, t_stride, src, s_stride,
         count, groups);
  B200_LAUNCHED("scales_by_group_kernel");
  return 0;
}

int launch_outlier_columns(float *cols, const int8_t *w, const float *s, int sstride, int dim, int vocab,
                           const int32_t *channels, int nch, cudaStream_t stream) {
  if (nch <= 0) return 0;
  launch(outlier_columns_kernel, blocks_for((int64_t)vocab * nch, 256), 256, 0, stream, cols, w, s, sstride, dim, vocab,
         channels, nch);
  B200_LAUNCHED("outlier_columns_kernel");
  return 0;
}

int launch_to_f16(uint16_t *out, const float *x, int64_t n, cudaStream_t stream) {
  if (n <= 0) return 0;
  launch(to_f16_kernel, blocks_for(n, 256), 256, 0, stream, out, x, n);
  B200_LAUNCHED("to_f16_kernel");
  return 0;
}
int launch_from_f16(float *out, const uint16_t *x, int64_t n, cudaStream_t stream) {
  if (n <= 0) return 0;
  launch(from_f16_kernel, blocks_for(n, 256), 256, 0, stream, out, x, n);
  B200_LAUNCHED("from_f16_kernel");
  return 0;
}
int launch_add_inplace(float *x, const float *y, int64_t n, cudaStream_t stream) {
  if (n <= 0) return 0;
  launch(add_inplace_kernel, blocks_for(n, 256), 256, 0, stream, x, y, n);
  B200_LAUNCHED("add_inplace_kernel");
  return 0;
}
int launch_swiglu(float *out, const float *h1, const float *h3, int64_t n, cudaStream_t stream) {
  if (n <= 0) return 0;
  launch(swiglu_kernel, blocks_for(n, 256), 256, 0, stream, out, h1, h3, n);
  B200_LAUNCHED("swiglu_kernel");
  return 0;
}
int launch_int8_sums(int32_t *out, const int8_t *w, int64_t groups, cudaStream_t stream) {
  if (groups <= 0) return 0;
  launch(int8_sums_kernel, blocks_for(groups, 256), 256, 0, stream, out, w, groups);
  B200_LAUNCHED("int8_sums_kernel");
  return 0;
}
int launch_advance(int32_t *tokens, int32_t *pos, const int32_t *ids, int32_t *history, int steps, int32_t *step,
                   int count, const float *logits, int64_t vocab, int32_t *bad, cudaStream_t stream) {
  if (count <= 0) return 0;
  if (count > 1024) return fail(B200FWD_EINVAL, "advance: more than 1024 sequences");
  launch(advance_kernel, 1, ((count + 31) / 32) * 32, 0, stream, tokens, pos, ids, history, steps, step, count, logits,
         vocab, bad);
  B200_LAUNCHED("advance_kernel");
  return 0;
}

}  // namespace b200
