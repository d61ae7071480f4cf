// oracle.cpp — TEST INFRASTRUCTURE, not the product.
//
// A plain C++ restatement of the reference's CPU forward path: the WASM-SIMD kernels of kernels/kernel.ts and
// kernels/kernel_relaxed.ts, and the layer loop of public/forward.js run(), in the same float32 operation order
// with no fused multiply-add (built with -ffp-contract=off). Four-lane SIMD steps are written out lane by lane.
// It is the checker of the CUDA engine (tests/, __graft_entry__.smoke) and the timed CPU baseline of bench.py; the
// product never calls it. Its multithreading follows public/jobs.js / forward.js phase(): the rows of a matmul in
// chunks taken from an atomic counter, attention by head; every row is computed whole by one thread, so the numbers
// do not depend on the thread count (public/forward.js:291-295).
//
// Each function cites the reference lines it restates.

#include <algorithm>
#include <atomic>
#include <cfloat>
#include <cmath>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <functional>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../include/b200fwd.h"

namespace {

constexpr int GS = 32;  // kernel.ts:7

inline float bits_f(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }
inline uint32_t f_bits(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }

// WASM f32.max / f32x4.max: a NaN in either gives NaN, and -0 is below +0 (kernel.ts:416-417)
inline float wmax(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == b) return std::signbit(a) ? b : a;
  return a > b ? a : b;
}
inline float wmin(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == b) return std::signbit(a) ? a : b;
  return a < b ? a : b;
}
// f32x4.nearest / nearest<f32>: round half to even
inline float nearest(float x) { return std::nearbyint(x); }
// i32x4.trunc_sat_f32x4_s: NaN -> 0, saturated
inline int32_t trunc_sat(float x) {
  if (x != x) return 0;
  if (x >= 2147483648.0f) return INT32_MAX;
  if (x <= -2147483648.0f) return INT32_MIN;
  return (int32_t)x;
}

// kernel.ts:15-28 fexp: table-free Cephes expf
float fexp(float x) {
  if (x < -87.0f) return 0;
  if (x > 88.0f) x = 88.0f;
  const float k = nearest(x * 1.44269504088896341f);
  const float r = x - k * 0.693359375f - k * -2.12194440e-4f;
  float p = 1.9875691500e-4f;
  p = p * r + 1.3981999507e-3f;
  p = p * r + 8.3334519073e-3f;
  p = p * r + 4.1665795894e-2f;
  p = p * r + 1.6666665459e-1f;
  p = p * r + 5.0000001201e-1f;
  const float e = p * (r * r) + r + 1.0f;
  return e * bits_f((uint32_t)((int32_t)k + 127) << 23);
}
// kernel.ts:32-45 vexp, one lane: fexp except that below -87 it is exp(-87)
float vexp(float x) {
  x = wmin(wmax(x, -87.0f), 88.0f);
  const float k = nearest(x * 1.44269504088896341f);
  const float r = (x - k * 0.693359375f) - k * -2.12194440e-4f;
  float p = 1.9875691500e-4f;
  p = p * r + 1.3981999507e-3f;
  p = p * r + 8.3334519073e-3f;
  p = p * r + 4.1665795894e-2f;
  p = p * r + 1.6666665459e-1f;
  p = p * r + 5.0000001201e-1f;
  const float e = (p * (r * r) + r) + 1.0f;
  const float scale = bits_f((uint32_t)(trunc_sat(k) + 127) << 23);
  return e * scale;
}

// kernel.ts:383-392 half / halves4: a float16's bits to float32 by one multiply by 2^112
inline float half_to_float(uint16_t h) {
  const int32_t v = (int32_t)(int16_t)h;
  return bits_f((uint32_t)((v << 13) & (int32_t)0x8fffffff)) * 5.192296858534828e33f;
}

template <typename T> inline float kv(const T *p);
template <> inline float kv<float>(const float *p) { return *p; }
template <> inline float kv<uint16_t>(const uint16_t *p) { return half_to_float(*p); }

// kernel.ts:10-12 hsum: ((l0 + l1) + l2) + l3
inline float hsum(const float a[4]) { return ((a[0] + a[1]) + a[2]) + a[3]; }
// kernel.ts:406-414 sums4 / sum4: (l0 + l2) + (l1 + l3)
inline float sum4(const float a[4]) { return (a[0] + a[2]) + (a[1] + a[3]); }

}  // namespace

extern "C" {

// kernel.ts:129-156 quantize_x
void oracle_quantize_x(int8_t *xq, float *xs, const float *x, int n, int bias) {
  const float qmax = bias == 0 ? 127.0f : 63.0f;
  for (int g = 0; g < n; g += GS) {
    const float *p = x + g;
    // groupMax (kernel.ts:72-81): a tree of f32x4.max of |v|, then the lanes by scalar comparison
    float m[4];
    for (int l = 0; l < 4; l++) {
      float a[8];
      for (int v = 0; v < 8; v++) a[v] = std::fabs(p[4 * v + l]);
      m[l] = wmax(wmax(wmax(a[0], a[1]), wmax(a[2], a[3])), wmax(wmax(a[4], a[5]), wmax(a[6], a[7])));
    }
    float amax = m[0];
    if (m[1] > amax) amax = m[1];
    if (m[2] > amax) amax = m[2];
    if (m[3] > amax) amax = m[3];
    const float scale = amax / qmax;
    xs[g / GS] = scale;
    const float inv = scale > 0 ? 1.0f / scale : 0.0f;
    for (int j = 0; j < GS; j++) {
      // i32x4.add wraps; the two narrowing steps saturate
      int32_t q = (int32_t)((uint32_t)trunc_sat(nearest(p[j] * inv)) + (uint32_t)bias);
      q = std::min(std::max(q, -32768), 32767);
      q = std::min(std::max(q, -128), 127);
      xq[g + j] = (int8_t)q;
    }
  }
}

// kernel.ts:204-212 int8_sums
void oracle_int8_sums(int32_t *out, const int8_t *w, int64_t groups) {
  for (int64_t g = 0; g < groups; g++) {
    int32_t s = 0;
    for (int j = 0; j < GS; j++) s += w[g * GS + j];
    out[g] = -64 * s;
  }
}

// kernel.ts:222-226,255-258 dot32 / groupQ8: lane k holds products 2k, 2k+1, 2k+8, 2k+9 of each half of 16
static inline void group_q8(const int8_t *row, const int8_t *xq, int g, int32_t lanes[4]) {
  const int o = g * GS;
  for (int k = 0; k < 4; k++) {
    int32_t s = 0;
    for (int h = 0; h < 2; h++) {
      const int b = o + 16 * h;
      for (int j : {2 * k, 2 * k + 1, 2 * k + 8, 2 * k + 9}) s += (int32_t)row[b + j] * (int32_t)xq[b + j];
    }
    lanes[k] = s;
  }
}

// kernel.ts:231-251 matmul_q8
void oracle_matmul_q8(float *xout, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws, int n,
                      int r0, int r1) {
  const int ng = n / GS;
  for (int i = r0; i < r1; i++) {
    const int8_t *row = wq + (int64_t)i * n;
    const float *srow = ws + (int64_t)i * ng;
    float facc[4] = {0, 0, 0, 0};
    for (int g = 0; g < ng; g++) {
      const float s = srow[g] * xs[g];
      int32_t l[4];
      group_q8(row, xq, g, l);
      for (int k = 0; k < 4; k++) facc[k] = facc[k] + (float)l[k] * s;
    }
    xout[i] = hsum(facc);
  }
}

// the exact integer of one group of kernel_relaxed.ts's dot products (the lanes' sum; integers, any order)
static inline int32_t group_dot(const int8_t *row, const int8_t *xq, int g) {
  int32_t s = 0;
  for (int j = 0; j < GS; j++) s += (int32_t)row[g * GS + j] * (int32_t)xq[g * GS + j];
  return s;
}

// kernel_relaxed.ts:34-67 matmul_q8r
void oracle_matmul_q8r(float *xout, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws,
                       const int32_t *wc, int n, int r0, int r1) {
  const int ng = n / GS, ng4 = ng & ~3;
  for (int i = r0; i < r1; i++) {
    const int8_t *row = wq + (int64_t)i * n;
    const float *srow = ws + (int64_t)i * ng;
    const int32_t *crow = wc + (int64_t)i * ng;
    float facc[4] = {0, 0, 0, 0};
    int g = 0;
    for (; g < ng4; g += 4) {
      for (int k = 0; k < 4; k++) {
        const float scale = srow[g + k] * xs[g + k];
        const int32_t sum = group_dot(row, xq, g + k) + crow[g + k];
        facc[k] = facc[k] + (float)sum * scale;
      }
    }
    float sum = ((facc[0] + facc[1]) + facc[2]) + facc[3];
    for (; g < ng; g++) {
      const int32_t whole = group_dot(row, xq, g) + crow[g];
      sum += (float)whole * (srow[g] * xs[g]);
    }
    xout[i] = sum;
  }
}

// kernel_relaxed.ts:106-152 tile: rows i..i+3 by four tokens `frame` bytes apart (xq) / apart (xs), outputs os
// floats apart. Lane passes: pass k takes the groups 4j+k, the passes are added in order, then the groups past the
// fours one at a time.
static void tile(float *xout, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws,
                 const int32_t *wc, int n, int i, int64_t os, int64_t qframe, int64_t sframe) {
  const int ng = n / GS, ng4 = ng & ~3;
  float f[4][4];  // f[row][token]
  for (int lane = 0; lane < 4; lane++) {
    float a[4][4] = {{0}};
    for (int g = lane; g < ng4; g += 4) {
      for (int r = 0; r < 4; r++) {
        const int8_t *w = wq + (int64_t)(i + r) * n;
        for (int t = 0; t < 4; t++) {
          const float sum = (float)(group_dot(w, xq + t * qframe, g) + wc[(int64_t)(i + r) * ng + g]);
          a[r][t] = a[r][t] + sum * (ws[(int64_t)(i + r) * ng + g] * xs[t * sframe + g]);
        }
      }
    }
    for (int r = 0; r < 4; r++)
      for (int t = 0; t < 4; t++) f[r][t] = lane == 0 ? a[r][t] : f[r][t] + a[r][t];
  }
  for (int g = ng4; g < ng; g++) {
    for (int r = 0; r < 4; r++) {
      const int8_t *w = wq + (int64_t)(i + r) * n;
      for (int t = 0; t < 4; t++) {
        const float sum = (float)(group_dot(w, xq + t * qframe, g) + wc[(int64_t)(i + r) * ng + g]);
        f[r][t] = f[r][t] + sum * (ws[(int64_t)(i + r) * ng + g] * xs[t * sframe + g]);
      }
    }
  }
  for (int t = 0; t < 4; t++)
    for (int r = 0; r < 4; r++) xout[t * os + i + r] = f[r][t];
}

// kernel_relaxed.ts:164-183 matmul_q8r_tile: count tokens, rows r0..r1. q_frame: bytes between tokens' xq,
// s_frame: floats between tokens' xs, os: floats between tokens' outputs (the reference keeps xq and xs one frame
// apart; here the two strides are separate).
void oracle_matmul_q8r_tile(float *xout, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws,
                            const int32_t *wc, int n, int r0, int r1, int count, int64_t os, int64_t q_frame,
                            int64_t s_frame) {
  const int rows4 = r0 + ((r1 - r0) & ~3), count4 = count & ~3;
  for (int i = r0; i < rows4; i += 4) {
    int t = 0;
    for (; t < count4; t += 4)
      tile(xout + t * os, xq + t * q_frame, xs + t * s_frame, wq, ws, wc, n, i, os, q_frame, s_frame);
    for (; t < count; t++)
      oracle_matmul_q8r(xout + t * os, xq + t * q_frame, xs + t * s_frame, wq, ws, wc, n, i, i + 4);
  }
  if (rows4 < r1) {
    for (int t = 0; t < count; t++)
      oracle_matmul_q8r(xout + t * os, xq + t * q_frame, xs + t * s_frame, wq, ws, wc, n, rows4, r1);
  }
}

// kernel.ts:48-68 matmul_f32
void oracle_matmul_f32(float *xout, const float *x, const float *w, int n, int r0, int r1) {
  const int n16 = n & ~15;
  for (int i = r0; i < r1; i++) {
    const float *row = w + (int64_t)i * n;
    float a[4][4] = {{0}};
    int j = 0;
    for (; j < n16; j += 16)
      for (int v = 0; v < 4; v++)
        for (int l = 0; l < 4; l++) a[v][l] = a[v][l] + row[j + 4 * v + l] * x[j + 4 * v + l];
    float s[4];
    for (int l = 0; l < 4; l++) s[l] = (a[0][l] + a[1][l]) + (a[2][l] + a[3][l]);
    float val = hsum(s);
    for (; j < n; j++) val += row[j] * x[j];
    xout[i] = val;
  }
}

// kernel.ts:330-342 rmsnorm
void oracle_rmsnorm(float *out, const float *x, const float *w, int n, float eps) {
  float acc[4] = {0, 0, 0, 0};
  int j = 0;
  const int n4 = n & ~3;
  for (; j < n4; j += 4)
    for (int l = 0; l < 4; l++) acc[l] = acc[l] + x[j + l] * x[j + l];
  float ss = hsum(acc);
  for (; j < n; j++) ss += x[j] * x[j];
  const float s = 1.0f / std::sqrt(ss / (float)n + eps);
  for (j = 0; j < n; j++) out[j] = w[j] * (s * x[j]);
}

// kernel.ts:344-357 rope
void oracle_rope(float *v, const float *fcr, const float *fci, int nh, int hs, int rot) {
  const int turned = rot > 0 && rot < hs ? rot : hs;
  for (int h = 0; h < nh; h++) {
    float *base = v + h * hs;
    for (int i = 0; i < turned; i += 2) {
      const float c = fcr[i >> 1], s = fci[i >> 1];
      const float v0 = base[i], v1 = base[i + 1];
      base[i] = v0 * c - v1 * s;
      base[i + 1] = v0 * s + v1 * c;
    }
  }
}

}  // extern "C"

// kernel.ts:447-566 attentionOf<T>
template <typename T>
static void attention_of(float *out, const float *q, const T *kc, const T *vc, float *att, int pos, int nh, int nkv,
                         int hs, int h0, int h1) {
  const int kvDim = nkv * hs, kvMul = nh / nkv, hs4 = hs & ~3;
  const int count = pos + 1, count4 = count & ~3;
  const float isq = 1.0f / std::sqrt((float)hs);
  int t = 0;
  // 1. scores: four positions at a time with an accumulator each; the tail position with one; same sums
  for (; t < count4; t += 4) {
    for (int h = h0; h < h1; h++) {
      const float *qh = q + h * hs;
      const T *k[4];
      for (int p = 0; p < 4; p++) k[p] = kc + (int64_t)(t + p) * kvDim + (h / kvMul) * hs;
      float a[4][4] = {{0}};
      int j = 0;
      for (; j < hs4; j += 4)
        for (int p = 0; p < 4; p++)
          for (int l = 0; l < 4; l++) a[p][l] = a[p][l] + qh[j + l] * kv<T>(k[p] + j + l);
      float sc[4];
      for (int p = 0; p < 4; p++) sc[p] = sum4(a[p]);
      for (; j < hs; j++) {
        const float x = qh[j];
        for (int p = 0; p < 4; p++) sc[p] = sc[p] + x * kv<T>(k[p] + j);
      }
      for (int p = 0; p < 4; p++) att[h * count + t + p] = sc[p] * isq;
    }
  }
  for (; t < count; t++) {
    for (int h = h0; h < h1; h++) {
      const float *qh = q + h * hs;
      const T *kt = kc + (int64_t)t * kvDim + (h / kvMul) * hs;
      float a[4] = {0, 0, 0, 0};
      int j = 0;
      for (; j < hs4; j += 4)
        for (int l = 0; l < 4; l++) a[l] = a[l] + qh[j + l] * kv<T>(kt + j + l);
      float sc = sum4(a);
      for (; j < hs; j++) sc += qh[j] * kv<T>(kt + j);
      att[h * count + t] = sc * isq;
    }
  }
  // 2. softmax, head by head: the largest from -FLT_MAX (kernel.ts:423-445, order-free), vexp on fours, fexp after
  for (int h = h0; h < h1; h++) {
    float *scores = att + h * count;
    float mx = -3.4028234663852886e38f;
    for (int i = 0; i < count; i++) mx = wmax(mx, scores[i]);
    float sums[4] = {0, 0, 0, 0};
    int u = 0;
    for (; u < count4; u += 4)
      for (int l = 0; l < 4; l++) {
        const float e = vexp(scores[u + l] - mx);
        scores[u + l] = e;
        sums[l] = sums[l] + e;
      }
    float sum = hsum(sums);
    for (; u < count; u++) {
      const float e = fexp(scores[u] - mx);
      scores[u] = e;
      sum += e;
    }
    const float inv = 1.0f / sum;
    for (u = 0; u < count; u++) scores[u] = scores[u] * inv;
  }
  // 3. the weighted sum of the values, four positions at a time ((w0 v0 + w1 v1) + (w2 v2 + w3 v3)), then one by one
  for (int j = h0 * hs; j < h1 * hs; j++) out[j] = 0;
  for (t = 0; t < count4; t += 4) {
    for (int h = h0; h < h1; h++) {
      const float *w = att + h * count + t;
      float *oh = out + h * hs;
      const T *v[4];
      for (int p = 0; p < 4; p++) v[p] = vc + (int64_t)(t + p) * kvDim + (h / kvMul) * hs;
      int j = 0;
      for (; j < hs4; j++) {
        const float pair0 = w[0] * kv<T>(v[0] + j) + w[1] * kv<T>(v[1] + j);
        const float pair1 = w[2] * kv<T>(v[2] + j) + w[3] * kv<T>(v[3] + j);
        oh[j] = oh[j] + (pair0 + pair1);
      }
      for (; j < hs; j++)
        oh[j] = oh[j] + w[0] * kv<T>(v[0] + j) + w[1] * kv<T>(v[1] + j) + w[2] * kv<T>(v[2] + j) +
                w[3] * kv<T>(v[3] + j);
    }
  }
  for (; t < count; t++) {
    for (int h = h0; h < h1; h++) {
      const float weight = att[h * count + t];
      float *oh = out + h * hs;
      const T *vt = vc + (int64_t)t * kvDim + (h / kvMul) * hs;
      for (int j = 0; j < hs; j++) oh[j] = oh[j] + weight * kv<T>(vt + j);
    }
  }
}

extern "C" {

// kernel.ts:365-373 attention / attention_f16
void oracle_attention(float *out, const float *q, const void *kc, const void *vc, float *att, int pos, int nh, int nkv,
                      int hs, int h0, int h1, int half) {
  if (half)
    attention_of<uint16_t>(out, q, (const uint16_t *)kc, (const uint16_t *)vc, att, pos, nh, nkv, hs, h0, h1);
  else
    attention_of<float>(out, q, (const float *)kc, (const float *)vc, att, pos, nh, nkv, hs, h0, h1);
}

// kernel.ts:570-599 to_f16
void oracle_to_f16(uint16_t *out, const float *x, int64_t n) {
  for (int64_t i = 0; i < n; i++) {
    const uint32_t bits = f_bits(x[i]);
    const uint32_t sign = (bits >> 16) & 0x8000;
    const int32_t exponent = (int32_t)((bits >> 23) & 0xff) - 112;
    uint32_t mantissa = bits & 0x7fffff;
    uint32_t result;
    if (exponent >= 31) {
      result = sign | 0x7c00;
    } else if (exponent <= 0) {
      if (exponent < -10) {
        result = sign;
      } else {
        mantissa |= 0x800000;
        const uint32_t shift = (uint32_t)(14 - exponent);
        const uint32_t rest = mantissa & ((1u << shift) - 1), middle = 1u << (shift - 1);
        uint32_t value = mantissa >> shift;
        if (rest > middle || (rest == middle && (value & 1))) value++;
        result = sign | value;
      }
    } else {
      const uint32_t rest = mantissa & 0x1fff;
      uint32_t value = ((uint32_t)exponent << 10) | (mantissa >> 13);
      if (rest > 0x1000 || (rest == 0x1000 && (value & 1))) value++;
      result = sign | value;
    }
    out[i] = (uint16_t)result;
  }
}

// kernel.ts:604-608 from_f16
void oracle_from_f16(float *out, const uint16_t *x, int64_t n) {
  for (int64_t i = 0; i < n; i++) out[i] = half_to_float(x[i]);
}

// kernel.ts:654-667 swiglu (vexp on fours, fexp on the rest)
void oracle_swiglu(float *out, const float *h1, const float *h3, int64_t n) {
  int64_t j = 0;
  for (; j + 4 <= n; j += 4)
    for (int l = 0; l < 4; l++) {
      const float v = h1[j + l];
      out[j + l] = v / (1.0f + vexp(-v)) * h3[j + l];
    }
  for (; j < n; j++) {
    const float v = h1[j];
    out[j] = v / (1.0f + fexp(-v)) * h3[j];
  }
}

// kernel.ts:671-689 add_columns
void oracle_add_columns(float *y, const float *rows, const float *a, int count, int n) {
  for (int j = 0; j < n; j++) {
    float v = y[j];
    for (int c = 0; c < count; c++) v = v + a[c] * rows[(int64_t)c * n + j];
    y[j] = v;
  }
}

// kernel.ts:691-693 add_inplace
void oracle_add_inplace(float *x, const float *y, int64_t n) {
  for (int64_t j = 0; j < n; j++) x[j] = x[j] + y[j];
}

// kernel.ts:695-699 argmax
int oracle_argmax(const float *x, int n) {
  int mi = 0;
  float mv = x[0];
  for (int j = 1; j < n; j++)
    if (x[j] > mv) { mv = x[j]; mi = j; }
  return mi;
}

// kernel.ts:15-45, one value each (tests)
float oracle_fexp(float x) { return fexp(x); }
float oracle_vexp(float x) { return vexp(x); }

// kernel.ts:705-719 penalize: each of the count recent tokens made less likely once, however often it occurs
void oracle_penalize(float *logits, const int32_t *tokens, int count, float penalty) {
  for (int i = 0; i < count; i++) {
    const int32_t token = tokens[i];
    bool seen = false;
    for (int j = 0; j < i; j++)
      if (tokens[j] == token) {
        seen = true;
        break;
      }
    if (seen) continue;
    const float value = logits[token];
    logits[token] = value > 0 ? value / penalty : value * penalty;
  }
}

}  // extern "C"

namespace {

// kernel.ts:721-775 sortNucleus / intoNucleus: the nucleus's running mass (float64), its limit and its last index
struct Nucleus {
  double mass = 0, limit = 0;
  int last = -1;
};

bool into_nucleus(Nucleus &nu, const float *probs, int lo, int hi) {
  for (int k = lo; k <= hi; k++) {
    nu.mass += (double)probs[k];
    if (nu.mass >= nu.limit) {
      nu.last = k;
      return true;
    }
  }
  return false;
}

// probs[lo..hi] in descending order (index along), from the left and only as far as the nucleus reaches: quicksort
// with a median of three, insertion sort for ranges of 13 or fewer
void sort_nucleus(Nucleus &nu, float *probs, int32_t *index, int lo, int hi) {
  while (hi - lo > 12) {
    const int mid = lo + ((hi - lo) >> 1);
    float a = probs[lo], b = probs[mid];
    const float c = probs[hi];
    if (a < b) std::swap(a, b);
    if (b < c) {
      b = c;
      if (a < b) b = a;
    }
    const float pivot = b;
    int i = lo, j = hi;
    while (i <= j) {
      while (probs[i] > pivot) i++;
      while (probs[j] < pivot) j--;
      if (i <= j) {
        std::swap(probs[i], probs[j]);
        std::swap(index[i], index[j]);
        i++;
        j--;
      }
    }
    sort_nucleus(nu, probs, index, lo, j);
    if (nu.last >= 0) return;
    if (into_nucleus(nu, probs, j + 1, i - 1)) return;  // equal to the pivot
    lo = i;
  }
  for (int i = lo + 1; i <= hi; i++) {
    const float p = probs[i];
    const int32_t x = index[i];
    int j = i - 1;
    while (j >= lo && probs[j] < p) {
      probs[j + 1] = probs[j];
      index[j + 1] = index[j];
      j--;
    }
    probs[j + 1] = p;
    index[j + 1] = x;
  }
  into_nucleus(nu, probs, lo, hi);
}

}  // namespace

extern "C" {

// kernel.ts:808-868 sample: a token of softmax(logits / temperature), restricted to the nucleus when 0 < topp < 1,
// drawn with `random` in [0, 1); -1 when the largest logit is no finite number. probs, index: scratch of n each.
int oracle_sample(const float *logits, int n, float temperature, float topp, double random, float *probs,
                  int32_t *index) {
  float best = logits[0];
  for (int i = 0; i < n; i++) best = wmax(best, logits[i]);  // largest(): a NaN anywhere, order-free
  if (!std::isfinite(best)) return -1;
  const bool nucleus = topp > 0 && topp < 1;
  const float floor = nucleus ? best - temperature * 16.118095f : -FLT_MAX;
  int count = 0;
  for (int i = 0; i < n; i++) {
    const float v = logits[i];
    probs[count] = v - best;
    index[count] = i;
    count += v >= floor ? 1 : 0;
  }
  const float inverse = 1.0f / temperature;
  int i = 0;
  for (; i + 4 <= count; i += 4)
    for (int k = 0; k < 4; k++) probs[i + k] = vexp(probs[i + k] * inverse);
  for (; i < count; i++) probs[i] = fexp(probs[i] / temperature);
  double total = 0;
  float top = 0;
  for (i = 0; i < count; i++) {
    total += (double)probs[i];
    top = wmax(top, probs[i]);
  }
  int last = count - 1;
  double mass = total;
  if (nucleus) {
    const double spread = (1.0 - (double)topp) / (double)(count > 1 ? count - 1 : 1) * total;
    const double cutoff = spread < (double)top ? spread : (double)top;
    int likely = 0;
    for (int k = 0; k < count; k++) {
      const float p = probs[k];
      probs[likely] = p;
      index[likely] = index[k];
      likely += (double)p >= cutoff ? 1 : 0;
    }
    Nucleus nu;
    nu.limit = (double)topp * total;
    sort_nucleus(nu, probs, index, 0, likely - 1);
    last = nu.last >= 0 ? nu.last : likely - 1;
    mass = nu.mass;
  }
  const double target = random * mass;
  double cumulative = 0;
  for (int k = 0; k <= last; k++) {
    cumulative += (double)probs[k];
    if (cumulative > target) return index[k];
  }
  return index[last];
}

}  // extern "C"

// ------------------------------------------------------------------------------------------- the layer loop
namespace {

// public/jobs.js + helper.js: a persistent pool; a phase's jobs are cut into chunks taken from an atomic counter.
// Each phase has its own counters, so a helper that wakes late only ever takes chunks of the phase it saw.
class Pool {
 public:
  explicit Pool(int threads) : threads_(std::max(1, threads)) {
    for (int i = 1; i < threads_; i++) workers_.emplace_back([this] { loop(); });
  }
  ~Pool() {
    {
      std::lock_guard<std::mutex> g(m_);
      quit_ = true;
      gen_++;
    }
    cv_.notify_all();
    for (auto &w : workers_) w.join();
  }
  int threads() const { return threads_; }
  // run(chunk) for chunk in [0, total), on every thread
  void run(int total, const std::function<void(int)> &body) {
    if (threads_ == 1 || total <= 1) {
      for (int c = 0; c < total; c++) body(c);
      return;
    }
    auto phase = std::make_shared<Phase>();
    phase->body = &body;
    phase->total = total;
    {
      std::lock_guard<std::mutex> g(m_);
      current_ = phase;
      gen_++;
    }
    cv_.notify_all();
    work(*phase);
    std::unique_lock<std::mutex> g(m_);
    done_cv_.wait(g, [&] { return phase->done.load() == phase->total; });
    current_.reset();
  }

 private:
  struct Phase {
    const std::function<void(int)> *body = nullptr;
    int total = 0;
    std::atomic<int> next{0}, done{0};
  };
  void work(Phase &p) {
    for (int c = p.next.fetch_add(1); c < p.total; c = p.next.fetch_add(1)) {
      (*p.body)(c);
      if (p.done.fetch_add(1) + 1 == p.total) {
        std::lock_guard<std::mutex> g(m_);
        done_cv_.notify_all();
      }
    }
  }
  void loop() {
    uint64_t seen = 0;
    for (;;) {
      std::shared_ptr<Phase> phase;
      {
        std::unique_lock<std::mutex> g(m_);
        cv_.wait(g, [&] { return gen_ != seen; });
        seen = gen_;
        if (quit_) return;
        phase = current_;
      }
      if (phase) work(*phase);
    }
  }
  int threads_;
  std::vector<std::thread> workers_;
  std::mutex m_;
  std::condition_variable cv_, done_cv_;
  std::shared_ptr<Phase> current_;
  uint64_t gen_ = 0;
  bool quit_ = false;
};

struct Matrix {
  int rows = 0, n = 0, group = 32;
  const int8_t *values = nullptr;
  const float *scales = nullptr;
  std::vector<int32_t> corrections;  // forward.js:176-184 (relaxed): int8_sums
  int64_t layer_values(int l) const { return (int64_t)l * rows * n; }
  int64_t layer_groups(int l) const { return (int64_t)l * rows * (n / 32); }
};

}  // namespace

struct oracle_engine {
  b200fwd_plan plan{};
  std::vector<uint8_t> ckpt;
  int dim, hidden, layers, heads, kvHeads, hs, vocab, seqLen, kvDim, qDim;
  bool relaxed, halfKV;
  int bias;
  float eps;
  Matrix wq, wk, wv, wo, w1, w2, w3, wcls;
  const float *attW, *ffnW, *finalW;
  std::vector<float> cosT, sinT;
  b200fwd_tensor emb;
  std::vector<int> channels;
  std::vector<float> columns;
  // frames: BATCH tokens, arrays side by side per token (forward.js:192-208)
  static constexpr int BATCH = 16;
  std::vector<float> x, xb, xb2, q, kNow, vNow, hb, hb2, att, logits;
  std::vector<int8_t> xq;
  std::vector<float> xs;
  int XQ;
  int capacity;
  std::vector<std::vector<uint8_t>> keys, values;  // per layer [capacity][kvDim] of float or half
  Pool *pool;
  std::string error;
};

static Matrix make_matrix(oracle_engine *e, const b200fwd_tensor &t) {
  Matrix m;
  m.rows = (int)t.shape[t.ndim - 2];
  m.n = (int)t.shape[t.ndim - 1];
  m.group = t.group;
  m.values = (const int8_t *)(e->ckpt.data() + t.offset);
  m.scales = (const float *)(e->ckpt.data() + t.scales);
  if (e->relaxed) {
    int64_t count = 1;
    for (int i = 0; i < t.ndim; i++) count *= t.shape[i];
    m.corrections.resize(count / 32);
    oracle_int8_sums(m.corrections.data(), m.values, count / 32);
  }
  return m;
}

extern "C" {

oracle_engine *oracle_create(const void *checkpoint, size_t size, const b200fwd_plan *plan, int half_keys,
                             int threads) {
  auto *e = new oracle_engine();
  e->plan = *plan;
  e->ckpt.assign((const uint8_t *)checkpoint, (const uint8_t *)checkpoint + size);
  const b200fwd_plan &p = *plan;
  e->dim = p.dim; e->hidden = p.hidden_dim; e->layers = p.n_layers; e->heads = p.n_heads;
  e->kvHeads = p.n_kv_heads; e->hs = p.head_size; e->vocab = p.vocab_size; e->seqLen = p.seq_len;
  e->kvDim = e->kvHeads * e->hs; e->qDim = e->heads * e->hs;
  e->relaxed = p.relaxed != 0;
  e->bias = e->relaxed ? 64 : 0;
  e->eps = p.rms_norm_eps;
  // forward.js:203: float16 keys and values where the plan allows and halfKeys (or kvHeads >= heads) says so
  const bool hk = half_keys < 0 ? (e->kvHeads >= e->heads) : half_keys != 0;
  e->halfKV = p.half_kv && hk;
  e->wq = make_matrix(e, p.wq); e->wk = make_matrix(e, p.wk); e->wv = make_matrix(e, p.wv);
  e->wo = make_matrix(e, p.wo); e->w1 = make_matrix(e, p.w1); e->w2 = make_matrix(e, p.w2);
  e->w3 = make_matrix(e, p.w3);
  e->wcls = make_matrix(e, p.shared_classifier ? p.token_embedding_table : p.wcls);
  e->emb = p.token_embedding_table;
  e->attW = (const float *)(e->ckpt.data() + p.rms_att_weight.offset);
  e->ffnW = (const float *)(e->ckpt.data() + p.rms_ffn_weight.offset);
  e->finalW = (const float *)(e->ckpt.data() + p.rms_final_weight.offset);
  const size_t table = (size_t)e->seqLen * (e->hs / 2);
  e->cosT.assign(p.freq_cis_real, p.freq_cis_real + table);
  e->sinT.assign(p.freq_cis_imag, p.freq_cis_imag + table);
  // forward.js:799-813: the outlier channels' columns of the classifier in float32
  for (int i = 0; i < p.n_outliers; i++) e->channels.push_back(p.outliers[i]);
  if (!e->channels.empty()) {
    const b200fwd_tensor &t = p.shared_classifier ? p.token_embedding_table : p.wcls;
    const int8_t *w = (const int8_t *)(e->ckpt.data() + t.offset);
    const float *s = (const float *)(e->ckpt.data() + t.scales);
    const int groups = e->dim / t.group;
    e->columns.resize(e->channels.size() * (size_t)e->vocab);
    for (size_t i = 0; i < e->channels.size(); i++) {
      const int c = e->channels[i];
      for (int v = 0; v < e->vocab; v++)
        e->columns[i * e->vocab + v] = (float)w[(int64_t)v * e->dim + c] * s[(int64_t)v * groups + c / t.group];
    }
  }
  const int B = oracle_engine::BATCH;
  e->x.resize((size_t)B * e->dim); e->xb.resize((size_t)B * std::max(e->dim, e->qDim));
  e->xb2.resize((size_t)B * e->dim); e->q.resize((size_t)B * e->qDim);
  e->kNow.resize((size_t)B * e->kvDim); e->vNow.resize((size_t)B * e->kvDim);
  e->hb.resize((size_t)B * e->hidden); e->hb2.resize((size_t)B * e->hidden);
  e->XQ = std::max(std::max(e->dim, e->hidden), e->qDim);
  e->xq.resize((size_t)B * e->XQ); e->xs.resize((size_t)B * (e->XQ / 32));
  e->att.resize((size_t)B * e->seqLen * e->heads);
  e->logits.resize(e->vocab);
  e->capacity = std::min(p.kv_start, e->seqLen);
  const size_t KV = (size_t)e->kvDim * (e->halfKV ? 2 : 4);
  e->keys.assign(e->layers, std::vector<uint8_t>(e->capacity * KV));
  e->values.assign(e->layers, std::vector<uint8_t>(e->capacity * KV));
  e->pool = new Pool(threads);
  return e;
}

void oracle_destroy(oracle_engine *e) {
  if (!e) return;
  delete e->pool;
  delete e;
}

int oracle_half_kv(oracle_engine *e) { return e->halfKV ? 1 : 0; }

}  // extern "C"

// forward.js:274-289 grow: larger capacity, values unchanged
static void grow(oracle_engine *e, int pos) {
  const int larger = std::min(std::max(2 * e->capacity, pos + 1), e->seqLen);
  const size_t KV = (size_t)e->kvDim * (e->halfKV ? 2 : 4);
  for (int l = 0; l < e->layers; l++) {
    e->keys[l].resize(larger * KV);
    e->values[l].resize(larger * KV);
  }
  e->capacity = larger;
}

// forward.js:395-400 matmuls + forward.js:350-393 phase: quantize each token's input once, then the rows of every
// matrix in chunks (count > 1: fours of rows, the tiles of matmul_q8r_tile)
struct MatJob {
  const Matrix *m;
  float *out;  // token t's at out + t * ostride
  int64_t ostride;
  int layer;
};

static void matmuls(oracle_engine *e, const float *input, int64_t istride, int count,
                    const std::vector<MatJob> &jobs) {
  const int n = jobs[0].m->n;
  for (int t = 0; t < count; t++)
    oracle_quantize_x(e->xq.data() + (size_t)t * e->XQ, e->xs.data() + (size_t)t * (e->XQ / 32),
                      input + t * istride, n, e->bias);
  const int threads = e->pool->threads();
  struct Chunked { const MatJob *job; int size, first, rows; };
  std::vector<Chunked> cj;
  int total = 0;
  for (const MatJob &j : jobs) {
    const int rows = j.m->rows;
    const int quad = count > 1 ? 4 : 1;
    const int size = quad * (int)std::ceil(rows / (double)(threads * 4 * quad));
    cj.push_back({&j, size, total, rows});
    total += (rows + size - 1) / size;
  }
  e->pool->run(total, [&](int c) {
    int k = (int)cj.size() - 1;
    while (cj[k].first > c) k--;
    const MatJob &j = *cj[k].job;
    const int r0 = (c - cj[k].first) * cj[k].size, r1 = std::min(r0 + cj[k].size, cj[k].rows);
    const Matrix &m = *j.m;
    const int8_t *w = m.values + m.layer_values(j.layer);
    const float *s = m.scales + m.layer_groups(j.layer);
    if (e->relaxed) {
      const int32_t *wc = m.corrections.data() + m.layer_groups(j.layer);
      if (count == 1)
        oracle_matmul_q8r(j.out, e->xq.data(), e->xs.data(), w, s, wc, m.n, r0, r1);
      else
        oracle_matmul_q8r_tile(j.out, e->xq.data(), e->xs.data(), w, s, wc, m.n, r0, r1, count, j.ostride, e->XQ,
                               e->XQ / 32);
    } else {
      for (int t = 0; t < count; t++)
        oracle_matmul_q8(j.out + t * j.ostride, e->xq.data() + (size_t)t * e->XQ,
                         e->xs.data() + (size_t)t * (e->XQ / 32), w, s, m.n, r0, r1);
    }
  });
}

// forward.js:403-414 embed: an int8 row times its group's scale (Math.fround of the product)
static void embed(oracle_engine *e, const int32_t *tokens, int count) {
  const b200fwd_tensor &t = e->emb;
  const int8_t *w = (const int8_t *)(e->ckpt.data() + t.offset);
  const float *s = (const float *)(e->ckpt.data() + t.scales);
  for (int i = 0; i < count; i++) {
    const int64_t row = (int64_t)tokens[i] * e->dim;
    for (int j = 0; j < e->dim; j++) e->x[(size_t)i * e->dim + j] = (float)w[row + j] * s[(row + j) / t.group];
  }
}

// forward.js:452-531 run
static int run(oracle_engine *e, const int32_t *tokens, int count, int pos0, bool needLogits) {
  if (count < 1 || count > oracle_engine::BATCH || pos0 < 0 || pos0 + count > e->seqLen) {
    e->error = "oracle run: bad count or position";
    return -1;
  }
  if (pos0 + count - 1 >= e->capacity) grow(e, pos0 + count - 1);
  embed(e, tokens, count);
  const int D = e->dim, KVD = e->kvDim, QD = e->qDim, HID = e->hidden;
  const size_t KV = (size_t)KVD * (e->halfKV ? 2 : 4);
  for (int l = 0; l < e->layers; l++) {
    for (int t = 0; t < count; t++)
      oracle_rmsnorm(&e->xb[(size_t)t * D], &e->x[(size_t)t * D], e->attW + (size_t)l * D, D, e->eps);
    matmuls(e, e->xb.data(), D, count,
            {{&e->wq, e->q.data(), QD, l}, {&e->wk, e->kNow.data(), KVD, l}, {&e->wv, e->vNow.data(), KVD, l}});
    for (int t = 0; t < count; t++) {
      const int pos = pos0 + t;
      const float *cs = e->cosT.data() + (size_t)pos * (e->hs / 2), *sn = e->sinT.data() + (size_t)pos * (e->hs / 2);
      oracle_rope(&e->q[(size_t)t * QD], cs, sn, e->heads, e->hs, e->plan.rotary);
      oracle_rope(&e->kNow[(size_t)t * KVD], cs, sn, e->kvHeads, e->hs, e->plan.rotary);
      // forward.js:439-447 cache
      uint8_t *kp = e->keys[l].data() + (size_t)pos * KV, *vp = e->values[l].data() + (size_t)pos * KV;
      if (e->halfKV) {
        oracle_to_f16((uint16_t *)kp, &e->kNow[(size_t)t * KVD], KVD);
        oracle_to_f16((uint16_t *)vp, &e->vNow[(size_t)t * KVD], KVD);
      } else {
        std::memcpy(kp, &e->kNow[(size_t)t * KVD], KV);
        std::memcpy(vp, &e->vNow[(size_t)t * KVD], KV);
      }
    }
    // forward.js:498 the heads of every token as one phase (jobs.js kind 3/4: rows = heads)
    {
      const int threads = e->pool->threads();
      const int size = (int)std::ceil(e->heads / (double)(threads * 4));
      const int per = (e->heads + size - 1) / size;
      e->pool->run(per * count, [&](int c) {
        const int t = c / per, h0 = (c % per) * size, h1 = std::min(h0 + size, e->heads);
        oracle_attention(&e->xb[(size_t)t * std::max(D, QD)], &e->q[(size_t)t * QD], e->keys[l].data(),
                         e->values[l].data(), &e->att[(size_t)t * e->seqLen * e->heads], pos0 + t, e->heads,
                         e->kvHeads, e->hs, h0, h1, e->halfKV ? 1 : 0);
      });
    }
    matmuls(e, e->xb.data(), std::max(D, QD), count, {{&e->wo, e->xb2.data(), D, l}});
    for (int t = 0; t < count; t++) oracle_add_inplace(&e->x[(size_t)t * D], &e->xb2[(size_t)t * D], D);
    for (int t = 0; t < count; t++)
      oracle_rmsnorm(&e->xb[(size_t)t * std::max(D, QD)], &e->x[(size_t)t * D], e->ffnW + (size_t)l * D, D, e->eps);
    matmuls(e, e->xb.data(), std::max(D, QD), count,
            {{&e->w1, e->hb.data(), HID, l}, {&e->w3, e->hb2.data(), HID, l}});
    for (int t = 0; t < count; t++)
      oracle_swiglu(&e->hb[(size_t)t * HID], &e->hb[(size_t)t * HID], &e->hb2[(size_t)t * HID], HID);
    matmuls(e, e->hb.data(), HID, count, {{&e->w2, e->xb2.data(), D, l}});
    for (int t = 0; t < count; t++) oracle_add_inplace(&e->x[(size_t)t * D], &e->xb2[(size_t)t * D], D);
  }
  if (!needLogits) return 0;
  const float *last = &e->x[(size_t)(count - 1) * D];
  oracle_rmsnorm(e->xb.data(), last, e->finalW, D, e->eps);
  std::vector<float> picked(e->channels.size());
  for (size_t i = 0; i < e->channels.size(); i++) {
    picked[i] = e->xb[e->channels[i]];
    e->xb[e->channels[i]] = 0;
  }
  matmuls(e, e->xb.data(), D, 1, {{&e->wcls, e->logits.data(), 0, 0}});
  if (!e->channels.empty())
    oracle_add_columns(e->logits.data(), e->columns.data(), picked.data(), (int)e->channels.size(), e->vocab);
  return 0;
}

extern "C" {

// forward.js:532 forward(token, pos, needLogits); logits copied out when asked
int oracle_forward(oracle_engine *e, int32_t token, int32_t pos, int32_t need_logits, float *logits) {
  const int rc = run(e, &token, 1, pos, need_logits != 0);
  if (rc == 0 && need_logits && logits) std::memcpy(logits, e->logits.data(), sizeof(float) * e->vocab);
  return rc;
}

// forward.js:1755-1769 forwardMany on the CPU: BATCH at a time
int oracle_forward_many(oracle_engine *e, const int32_t *tokens, int32_t count, int32_t pos) {
  for (int at = 0; at < count; at += oracle_engine::BATCH) {
    const int n = std::min(oracle_engine::BATCH, count - at);
    const int rc = run(e, tokens + at, n, pos + at, false);
    if (rc) return rc;
  }
  return 0;
}

// forward.js:1939-1953 keysAndValues
int oracle_keys_values(oracle_engine *e, int32_t from, int32_t count, float *keys, float *values) {
  if (from < 0 || from + count > e->capacity) return -1;
  const size_t KV = (size_t)e->kvDim * (e->halfKV ? 2 : 4);
  for (int l = 0; l < e->layers; l++)
    for (int t = 0; t < count; t++) {
      float *ko = keys + ((size_t)l * count + t) * e->kvDim, *vo = values + ((size_t)l * count + t) * e->kvDim;
      const uint8_t *ka = e->keys[l].data() + (size_t)(from + t) * KV, *va = e->values[l].data() + (size_t)(from + t) * KV;
      if (e->halfKV) {
        oracle_from_f16(ko, (const uint16_t *)ka, e->kvDim);
        oracle_from_f16(vo, (const uint16_t *)va, e->kvDim);
      } else {
        std::memcpy(ko, ka, sizeof(float) * e->kvDim);
        std::memcpy(vo, va, sizeof(float) * e->kvDim);
      }
    }
  return 0;
}

int oracle_threads(oracle_engine *e) { return e->pool->threads(); }

}  // extern "C"
