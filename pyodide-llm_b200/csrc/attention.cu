// attention.cu — kernel.ts:447-566 attentionOf (attention / attention_f16) for many query tokens at once, each to the
// bit as the reference computes it alone, with the keys and values staged through shared memory.
//
// Query tokens come in tiles: up to ATT_TT consecutive tokens of one sequence at consecutive positions (a prompt
// block), or a single token (decode). A tile shares its sequence's keys and values, so every block loads a chunk of
// ATT_CH positions once with coalesced 16-byte loads, widens it exactly to float32 (the reference's half(), the
// 2^112 multiply) in shared memory, and serves every token and every query head of the kv head from it.
//
//   scores  grid (chunks, kv heads, tiles), a thread a position: per token and head four lane accumulators over
//           the head's fours, (l0+l2)+(l1+l3), the rest after, times 1/sqrt(hs) (kernel.ts:462-498);
//   softmax grid (heads, tokens): the largest, exp (vexp on the fours, fexp after), four lane sums then the rest,
//           times 1/sum (kernel.ts:499-521);
//   values  grid (kv heads, tiles), a thread two neighbouring values of one head for every token of the tile: the
//           positions in fours ((w0 v0 + w1 v1) + (w2 v2 + w3 v3)) added in order, then the positions past the
//           fours one by one (kernel.ts:522-565); values past the fours of a head add their four products one after
//           another.
//
// Single query tokens (decode; the whole-head rows 16-byte aligned) take attn_scores_decode and, for float16 caches
// with heads of a multiple of 64 values, attn_values_decode_h (else attn_values_decode) instead: key chunks of
// DEC_POS positions and value chunks come to shared memory by cp.async several chunks ahead, and the lane sums and
// the fours of positions run on paired float32 operations (fma with a run-time one for the adds, so that every
// product and sum keeps the reference's own rounding).
#include <algorithm>
#include <cfloat>
#include <cstdint>
#include <cstdlib>

#include "common.h"
#include "exact.cuh"
#include "kernels.h"

namespace b200 {
namespace {

constexpr unsigned FULL = 0xffffffffu;
constexpr int ATT_CH = 64;   // positions of a chunk
constexpr int ATT_TT = 16;   // tokens of a tile at most
constexpr size_t MAX_SOFTMAX_SMEM = 200 * 1024;
constexpr size_t MAX_TILE_SMEM = 200 * 1024;

#define CHECK_ATT(expr)  \
  do {                   \
    int rc_ = (expr);    \
    if (rc_) return rc_; \
  } while (0)

struct Tile {
  int first, count;
};

__device__ __forceinline__ Tile tile_of(const int32_t *tiles, int i) {
  if (tiles) return Tile{tiles[2 * i], tiles[2 * i + 1]};
  return Tile{i, 1};
}
__device__ __forceinline__ int pos_of(const int32_t *pos, int pos0, int tok) { return pos ? pos[tok] : pos0; }

// Two float32 lanes at once (PTX .f32x2), each rounded on its own. A paired multiply feeding a paired add can be
// fused into one fma below PTX; a product that is an operand of fma(one, a, b), `one` = 1.0f handed over at run
// time, cannot, and one * a + b is a + b rounded once.
__device__ __forceinline__ uint64_t pk(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ float lo(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float hi(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)), "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// positions c0..c0+rows-1 of one kv head of one sequence's cache, as float32, into dst rows `pitch` floats apart
template <bool HALF>
__device__ __forceinline__ void stage_rows(float *dst, int pitch, const void *cache, int64_t row0, int64_t kvDim,
                                           int hs, int rows, bool vec) {
  if (vec) {
    constexpr int per = HALF ? 8 : 4;  // values a 16-byte load holds
    const int pieces = hs / per;
    for (int idx = threadIdx.x; idx < rows * pieces; idx += blockDim.x) {
      const int r = idx / pieces, p = idx % pieces;
      const int64_t at = row0 + (int64_t)r * kvDim + p * per;
      float *d = dst + r * pitch + p * per;
      if (HALF) {
        const uint4 u = *reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(cache) + at);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int k = 0; k < 4; k++) {
          d[2 * k] = half_to_float((uint16_t)(w[k] & 0xffff));
          d[2 * k + 1] = half_to_float((uint16_t)(w[k] >> 16));
        }
      } else {
        const float4 f = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(cache) + at);
        d[0] = f.x;
        d[1] = f.y;
        d[2] = f.z;
        d[3] = f.w;
      }
    }
  } else {
    for (int idx = threadIdx.x; idx < rows * hs; idx += blockDim.x) {
      const int r = idx / hs, j = idx % hs;
      const int64_t at = row0 + (int64_t)r * kvDim + j;
      dst[r * pitch + j] = HALF ? half_to_float(reinterpret_cast<const uint16_t *>(cache)[at])
                                : reinterpret_cast<const float *>(cache)[at];
    }
  }
}

template <bool HALF, int G>
__global__ void __launch_bounds__(ATT_CH)
    attn_scores_tiled(const float *q, int64_t q_stride, const void *kc, float *att, const int32_t *seq,
                      const int32_t *pos, int pos0, const int32_t *tiles, int64_t seq_stride, int P, int nh, int nkv,
                      int hs, int h0, int h1, int vec, float one) {
  pdl_begin();
  extern __shared__ float sm[];
  const int kvh = blockIdx.y, chunk = blockIdx.x;
  const Tile tl = tile_of(tiles, blockIdx.z);
  const int last = pos_of(pos, pos0, tl.first + tl.count - 1);
  const int c0 = chunk * ATT_CH;
  if (c0 > last) return;
  const int rows = min(ATT_CH, last + 1 - c0);
  const int kvDim = nkv * hs, hs4 = hs & ~3, hsp = (hs + 3) & ~3, pitch = hsp + 4;
  float *kf = sm;                        // [ATT_CH][pitch]: rows on 16 bytes, banks apart
  float *qs = sm + ATT_CH * pitch;       // [count][G][hsp]
  const int64_t sq = seq ? seq[tl.first] : 0;
  stage_rows<HALF>(kf, pitch, kc, sq * seq_stride + (int64_t)c0 * kvDim + (int64_t)kvh * hs, kvDim, hs, rows, vec);
  if (hsp == hs && (G * hs) % 4 == 0 && q_stride % 4 == 0 && (reinterpret_cast<uintptr_t>(q) & 15) == 0) {
    // each token's G heads are one contiguous run of G * hs floats: 16-byte copies, no division
    for (int i = 0; i < tl.count; i++) {
      const float4 *src = reinterpret_cast<const float4 *>(q + (int64_t)(tl.first + i) * q_stride + (int64_t)kvh * G * hs);
      float4 *dst = reinterpret_cast<float4 *>(qs + i * G * hs);
      for (int r = threadIdx.x; r < G * hs / 4; r += blockDim.x) dst[r] = src[r];
    }
  } else {
    for (int idx = threadIdx.x; idx < tl.count * G * hs; idx += blockDim.x) {
      const int i = idx / (G * hs), r = idx % (G * hs), gg = r / hs, d = r % hs;
      qs[(i * G + gg) * hsp + d] = q[(int64_t)(tl.first + i) * q_stride + (int64_t)kvh * G * hs + r];
    }
  }
  __syncthreads();
  const int t = threadIdx.x, p = c0 + t;
  if (t >= rows) return;
  const float isq = fdiv(1.0f, __fsqrt_rn((float)hs));
  const float *krow = kf + t * pitch;
  const uint64_t one2 = pk(one, one);
  for (int i = 0; i < tl.count; i++) {
    const int tok = tl.first + i;
    if (p > pos_of(pos, pos0, tok)) continue;  // causal: a token reads the positions up to its own
    // lane accumulators (0, 1) and (2, 3) of each head, paired (each lane rounded on its own): lane k takes the
    // dims 4i + k
    uint64_t a01[G], a23[G];
#pragma unroll
    for (int g = 0; g < G; g++) a01[g] = a23[g] = 0;
    const float *qi = qs + i * G * hsp;
    for (int j = 0; j < hs4; j += 4) {
      const ulonglong2 k4 = *reinterpret_cast<const ulonglong2 *>(krow + j);
#pragma unroll
      for (int g = 0; g < G; g++) {
        const ulonglong2 q4 = *reinterpret_cast<const ulonglong2 *>(qi + g * hsp + j);
        a01[g] = fma2(one2, a01[g], mul2(q4.x, k4.x));
        a23[g] = fma2(one2, a23[g], mul2(q4.y, k4.y));
      }
    }
#pragma unroll
    for (int g = 0; g < G; g++) {
      const int h = kvh * G + g;
      if (h < h0 || h >= h1) continue;
      float s = fadd(fadd(lo(a01[g]), lo(a23[g])), fadd(hi(a01[g]), hi(a23[g])));  // (l0+l2)+(l1+l3)
      for (int j = hs4; j < hs; j++) s = fadd(s, fmul(qi[g * hsp + j], krow[j]));
      att[((int64_t)tok * nh + h) * P + p] = fmul(s, isq);
    }
  }
}

__global__ void attn_softmax_tiled(float *att, const int32_t *pos, int pos0, int P, int nh, int h0, int h1) {
  pdl_begin();
  extern __shared__ float e[];
  __shared__ float part[5];
  __shared__ float wm[32];
  const int tok = blockIdx.y, h = blockIdx.x;
  if (h < h0 || h >= h1) return;
  const int count = pos_of(pos, pos0, tok) + 1, count4 = count & ~3;
  float *row = att + ((int64_t)tok * nh + h) * P;
  // the largest from -FLT_MAX, a NaN kept (kernel.ts:423-445: the order does not matter)
  float mx = -FLT_MAX;
  for (int t = threadIdx.x; t < count; t += blockDim.x) {
    const float v = row[t];
    e[t] = v;  // the row stays in shared memory for the exponentials
    mx = wmax(mx, v);
  }
  for (int o = 16; o > 0; o >>= 1) mx = wmax(mx, __shfl_xor_sync(FULL, mx, o));
  if ((threadIdx.x & 31) == 0) wm[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = -FLT_MAX;
  for (int w = 0; w < (int)(blockDim.x >> 5); w++) mx = wmax(mx, wm[w]);
  for (int t = threadIdx.x; t < count; t += blockDim.x) {
    const float d = fsub(e[t], mx);  // this thread's own entry of the row
    e[t] = t < count4 ? vexp(d) : fexp(d);
  }
  __syncthreads();
  if (threadIdx.x < 4) {
    // the lane's chain, its next sixteen terms read while the sixteen before are added
    float acc = 0.0f;
    int t = threadIdx.x;
    if (t + 60 < count4) {
      float cur[16];
#pragma unroll
      for (int u = 0; u < 16; u++) cur[u] = e[t + 4 * u];
      for (; t + 124 < count4; t += 64) {
        float nxt[16];
#pragma unroll
        for (int u = 0; u < 16; u++) nxt[u] = e[t + 64 + 4 * u];
#pragma unroll
        for (int u = 0; u < 16; u++) acc = fadd(acc, cur[u]);
#pragma unroll
        for (int u = 0; u < 16; u++) cur[u] = nxt[u];
      }
#pragma unroll
      for (int u = 0; u < 16; u++) acc = fadd(acc, cur[u]);
      t += 64;
    }
    for (; t < count4; t += 4) acc = fadd(acc, e[t]);
    part[threadIdx.x] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float sum = fadd(fadd(fadd(part[0], part[1]), part[2]), part[3]);
    for (int t = count4; t < count; t++) sum = fadd(sum, e[t]);
    part[4] = fdiv(1.0f, sum);
  }
  __syncthreads();
  const float inv = part[4];
  for (int t = threadIdx.x; t < count; t += blockDim.x) row[t] = fmul(e[t], inv);
}

// attn_softmax_tiled for rows of at most SOFTMAX_ROW_MAX positions: one warp a (token, head) row, SOFTMAX_ROWS rows a
// block, each warp's row in its own part of shared memory. The same steps in the same order: the largest (any order),
// the exponentials (vexp on the fours, fexp after), four lane chains over the fours then hsum and the rest, times
// 1/sum. grid (ceil(count * nh / SOFTMAX_ROWS)), 32 * SOFTMAX_ROWS threads.
constexpr int SOFTMAX_ROWS = 8;
constexpr int SOFTMAX_ROW_MAX = 1024;
__global__ void __launch_bounds__(32 * SOFTMAX_ROWS)
    attn_softmax_rows(float *att, const int32_t *pos, int pos0, int P, int nh, int h0, int h1, int count_tokens) {
  pdl_begin();
  __shared__ float rows[SOFTMAX_ROWS][SOFTMAX_ROW_MAX];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int r = blockIdx.x * SOFTMAX_ROWS + w;
  if (r >= count_tokens * nh) return;
  const int tok = r / nh, h = r % nh;
  if (h < h0 || h >= h1) return;
  const int count = pos_of(pos, pos0, tok) + 1, count4 = count & ~3;
  float *row = att + ((int64_t)tok * nh + h) * P;
  float *e = rows[w];
  float mx = -FLT_MAX;
  for (int t = lane; t < count; t += 32) {
    const float v = row[t];
    e[t] = v;
    mx = wmax(mx, v);
  }
  for (int o = 16; o > 0; o >>= 1) mx = wmax(mx, __shfl_xor_sync(FULL, mx, o));
  for (int t = lane; t < count; t += 32) {
    const float d = fsub(e[t], mx);
    e[t] = t < count4 ? vexp(d) : fexp(d);
  }
  __syncwarp();
  float acc = 0.0f;
  if (lane < 4) {
    int t = lane;
    if (t + 60 < count4) {
      float cur[16];
#pragma unroll
      for (int u = 0; u < 16; u++) cur[u] = e[t + 4 * u];
      for (; t + 124 < count4; t += 64) {
        float nxt[16];
#pragma unroll
        for (int u = 0; u < 16; u++) nxt[u] = e[t + 64 + 4 * u];
#pragma unroll
        for (int u = 0; u < 16; u++) acc = fadd(acc, cur[u]);
#pragma unroll
        for (int u = 0; u < 16; u++) cur[u] = nxt[u];
      }
#pragma unroll
      for (int u = 0; u < 16; u++) acc = fadd(acc, cur[u]);
      t += 64;
    }
    for (; t < count4; t += 4) acc = fadd(acc, e[t]);
  }
  const float p0 = __shfl_sync(FULL, acc, 0), p1 = __shfl_sync(FULL, acc, 1);
  const float p2 = __shfl_sync(FULL, acc, 2), p3 = __shfl_sync(FULL, acc, 3);
  float sum = fadd(fadd(fadd(p0, p1), p2), p3);
  for (int t = count4; t < count; t++) sum = fadd(sum, e[t]);
  const float inv = fdiv(1.0f, sum);
  for (int t = lane; t < count; t += 32) row[t] = fmul(e[t], inv);
}

// one output value's step over four positions (kernel.ts:535-545): below the head's fours the products in pairs,
// past them one after another
__device__ __forceinline__ float four(float o, float w0, float w1, float w2, float w3, float v0, float v1, float v2,
                                      float v3, bool in_fours) {
  if (in_fours) return fadd(o, fadd(fadd(fmul(w0, v0), fmul(w1, v1)), fadd(fmul(w2, v2), fmul(w3, v3))));
  return fadd(fadd(fadd(fadd(o, fmul(w0, v0)), fmul(w1, v1)), fmul(w2, v2)), fmul(w3, v3));
}

template <bool HALF, int G>
__global__ void attn_values_tiled(float *out, int64_t out_stride, const void *vc, const float *att,
                                  const int32_t *seq, const int32_t *pos, int pos0, const int32_t *tiles,
                                  int64_t seq_stride, int P, int nh, int nkv, int hs, int h0, int h1, int vec,
                                  float one) {
  pdl_begin();
  extern __shared__ float sm[];
  const int kvh = blockIdx.x;
  const Tile tl = tile_of(tiles, blockIdx.y);
  const int kvDim = nkv * hs, hs4 = hs & ~3, hp = (hs + 1) / 2;
  float *vs = sm;                      // [ATT_CH][hs]
  float *wsm = sm + ATT_CH * hs;       // [count][G][ATT_CH]
  const int g = threadIdx.x / hp, jp = threadIdx.x % hp;
  const int h = kvh * G + g;
  const bool active = g < G && h >= h0 && h < h1;
  const int j0 = 2 * jp, j1 = j0 + 1;
  const bool has1 = j1 < hs;
  const int last = pos_of(pos, pos0, tl.first + tl.count - 1);
  const int64_t sq = seq ? seq[tl.first] : 0;
  // the two values' sums of each token, paired (value j0 low, j1 high; each rounded on its own)
  uint64_t o[ATT_TT];
#pragma unroll
  for (int i = 0; i < ATT_TT; i++) o[i] = 0;
  const uint64_t one2 = pk(one, one);
  const bool pair4 = has1 && j1 < hs4;  // both values in the head's fours: the paired step
  for (int c0 = 0; c0 <= last; c0 += ATT_CH) {
    const int rows = min(ATT_CH, last + 1 - c0);
    __syncthreads();  // the previous chunk is done with
    stage_rows<HALF>(vs, hs, vc, sq * seq_stride + (int64_t)c0 * kvDim + (int64_t)kvh * hs, kvDim, hs, rows, vec);
    for (int idx = threadIdx.x; idx < tl.count * G * ATT_CH; idx += blockDim.x) {
      const int i = idx / (G * ATT_CH), r = idx % (G * ATT_CH), gg = r / ATT_CH, p = r % ATT_CH;
      const int tok = tl.first + i, hh = kvh * G + gg;
      float w = 0.0f;
      if (p < rows && c0 + p <= pos_of(pos, pos0, tok) && hh >= h0 && hh < h1)
        w = att[((int64_t)tok * nh + hh) * P + c0 + p];
      wsm[idx] = w;
    }
    __syncthreads();
    if (!active) continue;
    for (int p = 0; p < rows; p += 4) {
      const int P0 = c0 + p;
      const int n4 = min(4, rows - p);
      float v0[4], v1[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        v0[u] = u < n4 ? vs[(p + u) * hs + j0] : 0.0f;
        v1[u] = (u < n4 && has1) ? vs[(p + u) * hs + j1] : 0.0f;
      }
#pragma unroll
      for (int i = 0; i < ATT_TT; i++) {
        if (i >= tl.count) break;
        const int count = pos_of(pos, pos0, tl.first + i) + 1, count4 = count & ~3;
        const float *w = wsm + (i * G + g) * ATT_CH + p;
        if (P0 + 4 <= count4) {
          const float4 w4 = *reinterpret_cast<const float4 *>(w);
          if (pair4) {
            // ((w0 v0 + w1 v1) + (w2 v2 + w3 v3)) for both values at once, then added to the sums
            const uint64_t s01 = fma2(one2, mul2(pk(w4.x, w4.x), pk(v0[0], v1[0])), mul2(pk(w4.y, w4.y), pk(v0[1], v1[1])));
            const uint64_t s23 = fma2(one2, mul2(pk(w4.z, w4.z), pk(v0[2], v1[2])), mul2(pk(w4.w, w4.w), pk(v0[3], v1[3])));
            o[i] = fma2(one2, o[i], fma2(one2, s01, s23));
          } else {
            const float a0 = four(lo(o[i]), w4.x, w4.y, w4.z, w4.w, v0[0], v0[1], v0[2], v0[3], j0 < hs4);
            const float a1 = has1 ? four(hi(o[i]), w4.x, w4.y, w4.z, w4.w, v1[0], v1[1], v1[2], v1[3], j1 < hs4) : 0.0f;
            o[i] = pk(a0, a1);
          }
        } else if (P0 < count) {
          // the positions past the fours, one at a time (kernel.ts:548-564)
          float a0 = lo(o[i]), a1 = hi(o[i]);
          for (int u = 0; u < 4 && P0 + u < count; u++) {
            a0 = fadd(a0, fmul(w[u], v0[u]));
            if (has1) a1 = fadd(a1, fmul(w[u], v1[u]));
          }
          o[i] = pk(a0, a1);
        }
      }
    }
  }
  if (!active) return;
#pragma unroll
  for (int i = 0; i < ATT_TT; i++) {
    if (i >= tl.count) break;
    float *dst = out + (int64_t)(tl.first + i) * out_stride + h * hs;
    dst[j0] = lo(o[i]);
    if (has1) dst[j1] = hi(o[i]);
  }
}

// ---- prompt blocks, register-blocked (heads of a multiple of 64 values, 16-byte rows). The block stages its rows
// once and each thread keeps a 4 x 4 tile of outputs in registers: every 16-byte shared-memory read then serves four
// outputs' sums (one with a thread an output), the limit of the kernels above. The arithmetic of each output and its
// order are those of attn_scores_tiled and attn_values_tiled.
constexpr int RB_POS = 64;  // positions of a scores block and of a values chunk
constexpr int RB_VAL = 64;  // values of a head a values block takes

// grid (chunks of RB_POS positions, kv heads, tiles), 64G threads: thread (ty, tx) takes rows 4ty .. 4ty + 3 of the
// tile (row r: token r / G, head r % G of the kv head) and positions tx, tx + 16, tx + 32, tx + 48 of the chunk; per
// output the four lane accumulators over the head's dims (lane k takes the dims 4i + k), paired (0, 1) and (2, 3),
// then (l0+l2)+(l1+l3) times 1/sqrt(hs). q rows start on 16 bytes (q_stride a multiple of 4).
template <bool HALF, int G>
__global__ void __launch_bounds__(64 * G, G <= 4 ? 2 : 1)
    attn_scores_rb(const float *q, int64_t q_stride, const void *kc, float *att, const int32_t *seq,
                   const int32_t *pos, int pos0, const int32_t *tiles, int64_t seq_stride, int P, int nh, int nkv,
                   int hs, int h0, int h1, float one) {
  pdl_begin();
  extern __shared__ __align__(16) float sm[];
  const int kvh = blockIdx.y, chunk = blockIdx.x;
  const Tile tl = tile_of(tiles, blockIdx.z);
  const int last = pos_of(pos, pos0, tl.first + tl.count - 1);
  const int c0 = chunk * RB_POS;
  if (c0 > last) return;
  const int rows = min(RB_POS, last + 1 - c0);
  const int kvDim = nkv * hs, pitch = hs + 4;  // rows 16 bytes apart in the banks
  float *ks = sm;                             // [RB_POS][pitch]
  float *qs = sm + RB_POS * pitch;            // [ATT_TT * G][pitch]
  const int64_t sq = seq ? seq[tl.first] : 0;
  stage_rows<HALF>(ks, pitch, kc, sq * seq_stride + (int64_t)c0 * kvDim + (int64_t)kvh * hs, kvDim, hs, rows, true);
  // the tile's tokens' G heads of this kv head: each token's G * hs floats are contiguous
  const int h4 = hs / 4;
  for (int idx = threadIdx.x; idx < tl.count * G * h4; idx += blockDim.x) {
    const int r = idx / h4, d4 = idx % h4;
    const float4 v = *reinterpret_cast<const float4 *>(q + (int64_t)(tl.first + r / G) * q_stride +
                                                      (int64_t)(kvh * G + r % G) * hs + 4 * d4);
    *reinterpret_cast<float4 *>(qs + r * pitch + 4 * d4) = v;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, tx = lane & 15, ty = (threadIdx.x >> 5) * 2 + (lane >> 4);
  const float *qrow = qs + 4 * ty * pitch, *krow = ks + tx * pitch;
  const uint64_t one2 = pk(one, one);
  uint64_t a01[4][4], a23[4][4];  // [row][position]: lanes 0, 1 and 2, 3
#pragma unroll
  for (int e = 0; e < 4; e++)
#pragma unroll
    for (int f = 0; f < 4; f++) a01[e][f] = a23[e][f] = 0;
  for (int d = 0; d < hs; d += 4) {
    ulonglong2 qv[4], kv[4];
#pragma unroll
    for (int e = 0; e < 4; e++) qv[e] = *reinterpret_cast<const ulonglong2 *>(qrow + e * pitch + d);
#pragma unroll
    for (int f = 0; f < 4; f++) kv[f] = *reinterpret_cast<const ulonglong2 *>(krow + 16 * f * pitch + d);
#pragma unroll
    for (int e = 0; e < 4; e++)
#pragma unroll
      for (int f = 0; f < 4; f++) {
        a01[e][f] = fma2(one2, a01[e][f], mul2(qv[e].x, kv[f].x));
        a23[e][f] = fma2(one2, a23[e][f], mul2(qv[e].y, kv[f].y));
      }
  }
  const float isq = fdiv(1.0f, __fsqrt_rn((float)hs));
#pragma unroll
  for (int e = 0; e < 4; e++) {
    const int r = 4 * ty + e, i = r / G, h = kvh * G + r % G;
    if (i >= tl.count || h < h0 || h >= h1) continue;
    const int tok = tl.first + i, ptok = pos_of(pos, pos0, tok);
    float *dst = att + ((int64_t)tok * nh + h) * P;
#pragma unroll
    for (int f = 0; f < 4; f++) {
      const int p = c0 + tx + 16 * f;
      if (p > ptok) continue;  // causal: a token reads the positions up to its own
      const float s4 = fadd(fadd(lo(a01[e][f]), lo(a23[e][f])), fadd(hi(a01[e][f]), hi(a23[e][f])));
      dst[p] = fmul(s4, isq);
    }
  }
}

// grid (kv heads, tiles, hs / RB_VAL), 64G threads: thread (ty, tx) takes rows 4ty .. 4ty + 3 of the tile and the
// values z * RB_VAL + 4tx .. + 3 of their heads, summed as attn_values_tiled sums them (the positions in fours,
// ((w0 v0 + w1 v1) + (w2 v2 + w3 v3)) then added, on the values in pairs; the positions past the fours one by one).
// The chunk's values and the tile's weights come to shared memory chunk by chunk, each loaded into registers while
// the chunk before is summed. out rows start on 16 bytes; att rows too (P a multiple of four).
template <bool HALF, int G>
__global__ void __launch_bounds__(64 * G, G <= 4 ? 3 : 1)
    attn_values_rb(float *out, int64_t out_stride, const void *vc, const float *att, const int32_t *seq,
                   const int32_t *pos, int pos0, const int32_t *tiles, int64_t seq_stride, int P, int nh, int nkv,
                   int hs, int h0, int h1, float one) {
  pdl_begin();
  extern __shared__ __align__(16) float sm[];
  constexpr int ROWS = ATT_TT * G, VP = RB_VAL + 4, WP = RB_POS + 4;
  const int kvh = blockIdx.x, v0 = blockIdx.z * RB_VAL;
  const Tile tl = tile_of(tiles, blockIdx.y);
  const int kvDim = nkv * hs;
  float *vs = sm;                  // [RB_POS][VP]: the chunk's positions' values v0 .. v0 + RB_VAL
  float *wsm = sm + RB_POS * VP;   // [ROWS][WP]: the rows' weights of the chunk's positions (0 past a token's own)
  const int lane = threadIdx.x & 31, tx = lane & 15, ty = (threadIdx.x >> 5) * 2 + (lane >> 4);
  const int last = pos_of(pos, pos0, tl.first + tl.count - 1);
  const int64_t sq = seq ? seq[tl.first] : 0;
  // each row's positions (its token's own + 1; 0: no such row), then the chunks: chunk c + 1's values and weights
  // are loaded into registers while chunk c is summed, and stored to shared memory after it
  constexpr int ES = HALF ? 2 : 4, PR = RB_VAL * ES / 16;          // 16-byte pieces of a position's values
  constexpr int NV = (RB_POS * PR + 64 * G - 1) / (64 * G), NW = 4;  // pieces and weight fours a thread moves
  __shared__ int rcount[ROWS];
  for (int r = threadIdx.x; r < ROWS; r += blockDim.x) {
    const int i = r / G, h = kvh * G + r % G;
    rcount[r] = i < tl.count && h >= h0 && h < h1 ? pos_of(pos, pos0, tl.first + i) + 1 : 0;
  }
  __syncthreads();
  int count[4];
#pragma unroll
  for (int e = 0; e < 4; e++) count[e] = rcount[4 * ty + e];
  const uint8_t *vbase = reinterpret_cast<const uint8_t *>(vc) + (sq * seq_stride + (int64_t)kvh * hs + v0) * ES;
  uint4 vreg[NV];
  float4 wreg[NW];
  auto fetch = [&](int c0) {
    const int rows = min(RB_POS, last + 1 - c0);
#pragma unroll
    for (int k = 0; k < NV; k++) {
      const int idx = threadIdx.x + k * 64 * G, r = idx / PR;
      vreg[k] = make_uint4(0, 0, 0, 0);
      if (idx < RB_POS * PR && r < rows)
        vreg[k] = *reinterpret_cast<const uint4 *>(vbase + (int64_t)(c0 + r) * kvDim * ES + (idx % PR) * 16);
    }
#pragma unroll
    for (int k = 0; k < NW; k++) {
      const int idx = threadIdx.x + k * 64 * G, r = idx / (RB_POS / 4), p = c0 + 4 * (idx % (RB_POS / 4));
      const int cnt = rcount[r];
      float4 w = make_float4(0.f, 0.f, 0.f, 0.f);
      if (p < cnt) {  // P a multiple of four: the whole four lies in the row
        w = *reinterpret_cast<const float4 *>(att + ((int64_t)(tl.first + r / G) * nh + kvh * G + r % G) * P + p);
        if (p + 1 >= cnt) w.y = 0.f;
        if (p + 2 >= cnt) w.z = 0.f;
        if (p + 3 >= cnt) w.w = 0.f;
      }
      wreg[k] = w;
    }
  };
  auto store = [&]() {
#pragma unroll
    for (int k = 0; k < NV; k++) {
      const int idx = threadIdx.x + k * 64 * G, r = idx / PR, piece = idx % PR;
      if (idx >= RB_POS * PR) continue;
      float *d = vs + r * VP + piece * (16 / ES);
      if (HALF) {
        const uint32_t w[4] = {vreg[k].x, vreg[k].y, vreg[k].z, vreg[k].w};
        float f[8];
#pragma unroll
        for (int u = 0; u < 4; u++) {
          f[2 * u] = half_to_float((uint16_t)(w[u] & 0xffff));
          f[2 * u + 1] = half_to_float((uint16_t)(w[u] >> 16));
        }
        *reinterpret_cast<float4 *>(d) = make_float4(f[0], f[1], f[2], f[3]);
        *reinterpret_cast<float4 *>(d + 4) = make_float4(f[4], f[5], f[6], f[7]);
      } else {
        *reinterpret_cast<uint4 *>(d) = vreg[k];
      }
    }
#pragma unroll
    for (int k = 0; k < NW; k++) {
      const int idx = threadIdx.x + k * 64 * G;
      *reinterpret_cast<float4 *>(wsm + (idx / (RB_POS / 4)) * WP + 4 * (idx % (RB_POS / 4))) = wreg[k];
    }
  };
  const uint64_t one2 = pk(one, one);
  uint64_t o[4][2];  // [row][value pair]: values 4tx, +1 and 4tx + 2, +3
#pragma unroll
  for (int e = 0; e < 4; e++) o[e][0] = o[e][1] = 0;
  fetch(0);
  for (int c0 = 0; c0 <= last; c0 += RB_POS) {
    const int rows = min(RB_POS, last + 1 - c0);
    __syncthreads();  // the previous chunk is done with
    store();
    __syncthreads();
    if (c0 + RB_POS <= last) fetch(c0 + RB_POS);
    for (int p = 0; p < rows; p += 4) {
      const int P0 = c0 + p;
      float4 vv[4];
#pragma unroll
      for (int u = 0; u < 4; u++) vv[u] = *reinterpret_cast<const float4 *>(vs + (p + u) * VP + 4 * tx);
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const float4 w = *reinterpret_cast<const float4 *>(wsm + (4 * ty + e) * WP + p);
        if (P0 + 4 <= (count[e] & ~3)) {
          // ((w0 v0 + w1 v1) + (w2 v2 + w3 v3)) for both values of each pair at once, then added to the sums
          const uint64_t w0 = pk(w.x, w.x), w1 = pk(w.y, w.y), w2 = pk(w.z, w.z), w3 = pk(w.w, w.w);
          const uint64_t s01a = fma2(one2, mul2(w0, pk(vv[0].x, vv[0].y)), mul2(w1, pk(vv[1].x, vv[1].y)));
          const uint64_t s23a = fma2(one2, mul2(w2, pk(vv[2].x, vv[2].y)), mul2(w3, pk(vv[3].x, vv[3].y)));
          o[e][0] = fma2(one2, o[e][0], fma2(one2, s01a, s23a));
          const uint64_t s01b = fma2(one2, mul2(w0, pk(vv[0].z, vv[0].w)), mul2(w1, pk(vv[1].z, vv[1].w)));
          const uint64_t s23b = fma2(one2, mul2(w2, pk(vv[2].z, vv[2].w)), mul2(w3, pk(vv[3].z, vv[3].w)));
          o[e][1] = fma2(one2, o[e][1], fma2(one2, s01b, s23b));
        } else if (P0 < count[e]) {
          // the positions past the fours, one at a time (kernel.ts:548-564)
          const float wu[4] = {w.x, w.y, w.z, w.w};
          float a[4] = {lo(o[e][0]), hi(o[e][0]), lo(o[e][1]), hi(o[e][1])};
          for (int u = 0; u < 4 && P0 + u < count[e]; u++) {
            a[0] = fadd(a[0], fmul(wu[u], vv[u].x));
            a[1] = fadd(a[1], fmul(wu[u], vv[u].y));
            a[2] = fadd(a[2], fmul(wu[u], vv[u].z));
            a[3] = fadd(a[3], fmul(wu[u], vv[u].w));
          }
          o[e][0] = pk(a[0], a[1]);
          o[e][1] = pk(a[2], a[3]);
        }
      }
    }
  }
#pragma unroll
  for (int e = 0; e < 4; e++) {
    if (!count[e]) continue;
    const int r = 4 * ty + e, h = kvh * G + r % G;
    float *dst = out + (int64_t)(tl.first + r / G) * out_stride + (int64_t)h * hs + v0 + 4 * tx;
    *reinterpret_cast<float4 *>(dst) = make_float4(lo(o[e][0]), hi(o[e][0]), lo(o[e][1]), hi(o[e][1]));
  }
}

// ---- single query tokens (decode): no tile shares the keys and values, so each thread loads its own straight from
// the cache (16-byte loads of its position's row for the scores; a pair of values per position for the weighted
// sum), with no shared-memory staging and no block-wide waits in the loops.
constexpr int DEC_POS = 128;  // positions of a scores block

// grid (position blocks of DEC_POS, kv heads, tokens), a thread a position: the same sums as attn_scores_tiled
// (four lane accumulators over the head's dims, (l0+l2)+(l1+l3), times 1/sqrt(hs)); hs a multiple of the values a
// 16-byte load holds, so the head has no dims past its fours
template <bool HALF, int G>
__global__ void __launch_bounds__(DEC_POS)
    attn_scores_decode(const float *q, int64_t q_stride, const void *kc, float *att, const int32_t *seq,
                       const int32_t *pos, int pos0, int64_t seq_stride, int P, int nh, int nkv, int hs, int h0,
                       int h1, float one) {
  pdl_begin();
  extern __shared__ __align__(16) float qs[];  // [G][hs], then the chunk's keys: DEC_POS rows of hs * ES + 16 bytes
  constexpr int PER = HALF ? 8 : 4, ES = HALF ? 2 : 4;
  const int kvh = blockIdx.y, tok = blockIdx.z;
  const int last = pos_of(pos, pos0, tok);
  const int c0 = blockIdx.x * DEC_POS;
  if (c0 > last) return;
  const int rows = min(DEC_POS, last + 1 - c0);
  const int64_t kvDim = (int64_t)nkv * hs;
  const int row_bytes = hs * ES, pitch = row_bytes + 16, pieces = row_bytes / 16;  // pitch: rows 4 banks apart
  uint8_t *ks = reinterpret_cast<uint8_t *>(qs + G * hs);
  const uint8_t *kbase = reinterpret_cast<const uint8_t *>(kc) +
                         ((seq ? (int64_t)seq[tok] : 0) * seq_stride + (int64_t)c0 * kvDim + (int64_t)kvh * hs) * ES;
  for (int i = threadIdx.x; i < rows * pieces; i += blockDim.x) {
    const int r = i / pieces, c = i % pieces;
    cp_async16(ks + r * pitch + c * 16, kbase + (int64_t)r * kvDim * ES + c * 16);
  }
  cp_async_commit();
  for (int idx = threadIdx.x; idx < G * hs; idx += blockDim.x)
    qs[idx] = q[(int64_t)tok * q_stride + (int64_t)kvh * G * hs + idx];
  cp_async_wait<0>();
  __syncthreads();
  const int p = c0 + threadIdx.x;
  if (p > last) return;
  const uint8_t *krow = ks + threadIdx.x * pitch;
  const uint64_t one2 = pk(one, one);
  // lane accumulators (0, 1) and (2, 3) of each head, paired: lane k takes the dims 4i + k
  uint64_t a01[G], a23[G];
#pragma unroll
  for (int g = 0; g < G; g++) a01[g] = a23[g] = 0;
#pragma unroll 4
  for (int j = 0; j < hs; j += PER) {
    uint64_t k2[PER / 2];  // this position's keys j .. j + PER - 1 in pairs
    if (HALF) {
      const uint4 u = *reinterpret_cast<const uint4 *>(krow + j * 2);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
      const uint64_t big = pk(5.192296858534828e33f, 5.192296858534828e33f);  // 2^112: the reference's half()
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int32_t lo16 = (((int32_t)(int16_t)(w[i] & 0xffff)) << 13) & (int32_t)0x8fffffff;
        const int32_t hi16 = (((int32_t)(int16_t)(w[i] >> 16)) << 13) & (int32_t)0x8fffffff;
        k2[i] = mul2(pk(__int_as_float(lo16), __int_as_float(hi16)), big);
      }
    } else {
      const ulonglong2 f = *reinterpret_cast<const ulonglong2 *>(krow + j * 4);
      k2[0] = f.x;
      k2[1] = f.y;
    }
#pragma unroll
    for (int g = 0; g < G; g++) {
#pragma unroll
      for (int u = 0; u < PER; u += 4) {
        const ulonglong2 q4 = *reinterpret_cast<const ulonglong2 *>(qs + g * hs + j + u);
        a01[g] = fma2(one2, a01[g], mul2(q4.x, k2[u / 2]));
        a23[g] = fma2(one2, a23[g], mul2(q4.y, k2[u / 2 + 1]));
      }
    }
  }
  const float isq = fdiv(1.0f, __fsqrt_rn((float)hs));
#pragma unroll
  for (int g = 0; g < G; g++) {
    const int h = kvh * G + g;
    if (h < h0 || h >= h1) continue;
    const float s4 = fadd(fadd(lo(a01[g]), lo(a23[g])), fadd(hi(a01[g]), hi(a23[g])));  // (l0+l2)+(l1+l3)
    att[((int64_t)tok * nh + h) * P + p] = fmul(s4, isq);
  }
}

constexpr int VCH = 32;  // positions of a value chunk
constexpr int VNB = 4;   // value chunks in flight (shared-memory buffers)

// shared memory of attn_values_decode for `dims` values of a head: VNB raw chunks, the widened chunk (float16
// caches), VNB chunks of weights
inline size_t values_smem(int dims, int G, bool half) {
  return (size_t)VNB * VCH * dims * (half ? 2 : 4) + (half ? (size_t)VCH * dims * 4 : 0) + (size_t)VNB * G * VCH * 4;
}

// grid (kv heads, tokens, parts), part z of gridDim.z taking the head's values z * dims .. + dims (dims even); a
// thread two neighbouring values of one head: the same chain as
// attn_values_tiled, the positions in fours then one by one. The head's values come in chunks of VCH positions,
// copied to shared memory asynchronously (cp.async, the next chunk on its way while this one is used), widened to
// float32 once per block (the reference's half()), then read by the G heads' threads; the chunk's softmax weights
// of the G heads come along the same way, VNB - 1 chunks ahead. A four of positions of two neighbouring values is
// one paired step: ((w0 v0 + w1 v1) + (w2 v2 + w3 v3)), then added to the sum. wvec: the weight rows start on 16
// bytes. Shared memory: values_smem(hs, G, HALF).
template <bool HALF, int G>
__global__ void __launch_bounds__(1024)
    attn_values_decode(float *out, int64_t out_stride, const void *vc, const float *att, const int32_t *seq,
                       const int32_t *pos, int pos0, int64_t seq_stride, int P, int nh, int nkv, int hs, int h0,
                       int h1, int wvec, float one) {
  pdl_begin();
  extern __shared__ __align__(16) uint8_t vsm[];
  constexpr int ES = HALF ? 2 : 4;
  const int kvh = blockIdx.x, tok = blockIdx.y;
  const int dims = hs / gridDim.z, dim0 = blockIdx.z * dims;  // this block's part of the head
  const int hp = dims / 2, hs4 = hs & ~3;
  const int g = threadIdx.x / hp, jp = threadIdx.x % hp;
  const int h = kvh * G + g;
  const bool active = g < G && h >= h0 && h < h1;
  const int count = pos_of(pos, pos0, tok) + 1, count4 = count & ~3;
  const int chunks = (count + VCH - 1) / VCH;
  const int64_t kvDim = (int64_t)nkv * hs;
  const uint8_t *vbase = reinterpret_cast<const uint8_t *>(vc) +
                         ((seq ? (int64_t)seq[tok] : 0) * seq_stride + (int64_t)kvh * hs + dim0) * ES;
  const int row_bytes = dims * ES, pieces = row_bytes / 16;
  float *wide = reinterpret_cast<float *>(vsm + VNB * VCH * row_bytes);  // the chunk in float32 (HALF)
  float *wts = reinterpret_cast<float *>(vsm + VNB * VCH * row_bytes + (HALF ? VCH * dims * 4 : 0));  // [VNB][G][VCH]
  const float *watt = att + ((int64_t)tok * nh + (int64_t)kvh * G) * P;  // head kvh * G + gg's row at gg * P
  // chunk c's values and weights into buffer c % VNB, one commit group per call (empty past the last chunk)
  auto issue = [&](int c) {
    const int r0 = c * VCH, rows = max(0, min(VCH, count - r0));
    uint8_t *dst = vsm + (c % VNB) * VCH * row_bytes;
    for (int i = threadIdx.x; i < rows * pieces; i += blockDim.x) {
      const int r = i / pieces, q = i % pieces;
      cp_async16(dst + r * row_bytes + q * 16, vbase + (int64_t)(r0 + r) * kvDim * ES + q * 16);
    }
    float *wd = wts + (c % VNB) * G * VCH;
    if (wvec && rows % 4 == 0) {
      for (int i = threadIdx.x; i < G * rows / 4; i += blockDim.x) {
        const int gg = i / (rows / 4), r = 4 * (i % (rows / 4));
        cp_async16(wd + gg * VCH + r, watt + (int64_t)gg * P + r0 + r);
      }
    } else {
      for (int i = threadIdx.x; i < G * rows; i += blockDim.x) {
        const int gg = i / rows, r = i % rows;
        wd[gg * VCH + r] = watt[(int64_t)gg * P + r0 + r];
      }
    }
    cp_async_commit();
  };
  const int j0 = 2 * jp;                // within the part; the head's value dim0 + j0
  const bool fours = dim0 + j0 < hs4;   // both of the thread's values lie in the head's fours (hs4, dim0, j0 even)
  const uint64_t one2 = pk(one, one);
  uint64_t o = 0;  // the two values' sums
  for (int c = 0; c + 1 < VNB; c++) issue(c);
  for (int c = 0; c < chunks; c++) {
    issue(c + VNB - 1);
    cp_async_wait<VNB - 1>();
    __syncthreads();  // chunk c is in shared memory, every thread's copies of it
    const int r0 = c * VCH, rows = min(VCH, count - r0);
    const float *vf;
    if (HALF) {
      const uint32_t *src = reinterpret_cast<const uint32_t *>(vsm + (c % VNB) * VCH * row_bytes);
      const uint64_t big = pk(5.192296858534828e33f, 5.192296858534828e33f);  // 2^112
      for (int i = threadIdx.x; i < rows * hp; i += blockDim.x) {
        const uint32_t u = src[i];
        const int32_t a = (((int32_t)(int16_t)(u & 0xffff)) << 13) & (int32_t)0x8fffffff;
        const int32_t b = (((int32_t)(int16_t)(u >> 16)) << 13) & (int32_t)0x8fffffff;
        reinterpret_cast<uint64_t *>(wide)[i] = mul2(pk(__int_as_float(a), __int_as_float(b)), big);
      }
      __syncthreads();
      vf = wide;
    } else {
      vf = reinterpret_cast<const float *>(vsm + (c % VNB) * VCH * row_bytes);
    }
    if (active) {
      const float *w = wts + (c % VNB) * G * VCH + g * VCH;  // this head's weights of the chunk
      for (int i = 0; i < rows; i += 4) {
        const int p = r0 + i;
        if (p + 4 <= count4) {
          const float4 w4 = *reinterpret_cast<const float4 *>(w + i);
          const float w0 = w4.x, w1 = w4.y, w2 = w4.z, w3 = w4.w;
          const uint64_t v0 = *reinterpret_cast<const uint64_t *>(vf + (i + 0) * dims + j0);
          const uint64_t v1 = *reinterpret_cast<const uint64_t *>(vf + (i + 1) * dims + j0);
          const uint64_t v2 = *reinterpret_cast<const uint64_t *>(vf + (i + 2) * dims + j0);
          const uint64_t v3 = *reinterpret_cast<const uint64_t *>(vf + (i + 3) * dims + j0);
          if (fours) {
            const uint64_t s01 = fma2(one2, mul2(pk(w0, w0), v0), mul2(pk(w1, w1), v1));
            const uint64_t s23 = fma2(one2, mul2(pk(w2, w2), v2), mul2(pk(w3, w3), v3));
            o = fma2(one2, o, fma2(one2, s01, s23));
          } else {
            const float a0 = four(lo(o), w0, w1, w2, w3, lo(v0), lo(v1), lo(v2), lo(v3), false);
            const float a1 = four(hi(o), w0, w1, w2, w3, hi(v0), hi(v1), hi(v2), hi(v3), false);
            o = pk(a0, a1);
          }
        } else {
          // the positions past the fours, one at a time (kernel.ts:548-564)
          float a0 = lo(o), a1 = hi(o);
          for (int u = 0; u < 4 && p + u < count; u++) {
            const float2 v = *reinterpret_cast<const float2 *>(vf + (i + u) * dims + j0);
            a0 = fadd(a0, fmul(w[i + u], v.x));
            a1 = fadd(a1, fmul(w[i + u], v.y));
          }
          o = pk(a0, a1);
        }
      }
    }
    __syncthreads();  // chunk c's buffers are free for chunk c + VNB
  }
  if (active) {
    float *dst = out + (int64_t)tok * out_stride + (int64_t)h * hs + dim0 + j0;
    dst[0] = lo(o);
    dst[1] = hi(o);
  }
}

constexpr int HCH = 32;  // positions of a value chunk (attn_values_decode_h)
constexpr int HNB = 6;   // value chunks in flight

// the reference's half() of two float16 values (kernel.ts half: bits << 13 with the sign kept, times 2^112), less the
// factor 2^112: the float32 whose bits are the half's shifted into place. The caller multiplies the weights by 2^112
// instead: w * 2^112 is exact (a power of two; the weights lie in [0, 1]) and the product with the shifted bits is
// the same real number as w * half(v), so it rounds to the same float.
__device__ __forceinline__ uint64_t half2_bits(uint32_t u) {
  const uint32_t lo = (uint32_t)((int32_t)(u << 16) >> 3) & 0x8fffe000u;
  const uint32_t hi = (uint32_t)((int32_t)u >> 3) & 0x8fffe000u;
  return (uint64_t)lo | ((uint64_t)hi << 32);
}

// Decode values over a float16 cache, heads a multiple of 64 values: grid (kv heads x hs / 64, tokens), one warp a
// block; lane l takes the values dim0 + 2l and dim0 + 2l + 1 (dim0 = 64 x the block's part) of all G query heads of
// the kv head, so every float16 pair is widened once for G heads. The same chain as attn_values_tiled: per head and
// value the positions in fours ((w0 v0 + w1 v1) + (w2 v2 + w3 v3)) added in order, then the positions past the fours
// one by one (kernel.ts:522-565). The values come in chunks of HCH positions by cp.async, HNB - 1 chunks ahead; the
// chunk's weights (times 2^112, each twice for the paired multiplies) are read one chunk ahead into registers and
// stored to shared memory after the chunk before is done.
// QUANT: also write the rows quantized (xq, xs); the instance without it keeps the registers of the sums alone.
template <int G, bool QUANT>
__global__ void __launch_bounds__(32)
    attn_values_decode_h(float *out, int64_t out_stride, const uint16_t *vc, const float *att, const int32_t *seq,
                         const int32_t *pos, int pos0, int64_t seq_stride, int P, int nh, int nkv, int hs, int h0,
                         int h1, float one, int8_t *xq, int64_t q_stride, float *xs, int64_t s_stride,
                         int64_t g_stride, int bias, int shift) {
  pdl_begin();
  __shared__ __align__(16) uint32_t vbuf[HNB][HCH][32];  // raw float16 pairs: [chunk][position][lane]
  __shared__ __align__(16) uint64_t wbuf[2][G][HCH];     // the weights x 2^112, twice: [chunk & 1][head][position]
  const int parts = hs >> 6;
  const int kvh = blockIdx.x / parts, dim0 = (blockIdx.x % parts) * 64, tok = blockIdx.y;
  const int lane = threadIdx.x;
  const int count = pos_of(pos, pos0, tok) + 1, count4 = count & ~3;
  const int chunks = (count + HCH - 1) / HCH;
  const int64_t kvDim = (int64_t)nkv * hs;
  const uint16_t *vbase = vc + (seq ? (int64_t)seq[tok] : 0) * seq_stride + (int64_t)kvh * hs + dim0;
  const float *watt = att + ((int64_t)tok * nh + (int64_t)kvh * G) * P;  // head kvh * G + g's row at g * P
  const float big = 5.192296858534828e33f;                                // 2^112
  // chunk c's values into buffer c % HNB: 16-byte piece lane % 8 of the rows lane / 8 + 4 i (one commit group per
  // call, empty past the last chunk)
  auto issue = [&](int c) {
    if (c < chunks) {
      const int r0 = c * HCH, rows = min(HCH, count - r0);
      uint32_t(*dst)[32] = vbuf[c % HNB];
      const int piece = lane & 7;
#pragma unroll
      for (int i = 0; i < HCH / 4; i++) {
        const int r = (lane >> 3) + 4 * i;
        if (r < rows) cp_async16(&dst[r][4 * piece], vbase + (int64_t)(r0 + r) * kvDim + 8 * piece);
      }
    }
    cp_async_commit();
  };
  auto load_weights = [&](int c, float (&w)[G]) {
    const int p = c * HCH + lane;
#pragma unroll
    for (int g = 0; g < G; g++) w[g] = c < chunks && p < count ? watt[(int64_t)g * P + p] : 0.0f;
  };
  auto store_weights = [&](int c, const float (&w)[G]) {
#pragma unroll
    for (int g = 0; g < G; g++) {
      const float s = fmul(w[g], big);
      wbuf[c & 1][g][lane] = pk(s, s);
    }
  };
  const uint64_t one2 = pk(one, one);
  uint64_t o[G];
#pragma unroll
  for (int g = 0; g < G; g++) o[g] = 0;
  for (int c = 0; c + 1 < HNB; c++) issue(c);
  {
    float w[G];
    load_weights(0, w);
    store_weights(0, w);
  }
  for (int c = 0; c < chunks; c++) {
    issue(c + HNB - 1);
    float wn[G];
    load_weights(c + 1, wn);
    cp_async_wait<HNB - 1>();
    __syncwarp();  // chunk c's values (every lane's copies) and weights are in shared memory
    const uint32_t(*vb)[32] = vbuf[c % HNB];
    const uint64_t(*wb)[HCH] = wbuf[c & 1];
    const int r0 = c * HCH, rows = min(HCH, count - r0);
    const int rows4 = max(0, min(rows, count4 - r0));  // a multiple of four (r0 is)
#pragma unroll 2
    for (int i = 0; i < rows4; i += 4) {
      const uint64_t v0 = half2_bits(vb[i][lane]), v1 = half2_bits(vb[i + 1][lane]);
      const uint64_t v2 = half2_bits(vb[i + 2][lane]), v3 = half2_bits(vb[i + 3][lane]);
#pragma unroll
      for (int g = 0; g < G; g++) {
        const ulonglong2 w01 = *reinterpret_cast<const ulonglong2 *>(&wb[g][i]);
        const ulonglong2 w23 = *reinterpret_cast<const ulonglong2 *>(&wb[g][i + 2]);
        const uint64_t s01 = fma2(one2, mul2(w01.x, v0), mul2(w01.y, v1));
        const uint64_t s23 = fma2(one2, mul2(w23.x, v2), mul2(w23.y, v3));
        o[g] = fma2(one2, o[g], fma2(one2, s01, s23));
      }
    }
    // the positions past the fours, one at a time (kernel.ts:548-564)
    for (int i = rows4; i < rows; i++) {
      const uint64_t v = half2_bits(vb[i][lane]);
#pragma unroll
      for (int g = 0; g < G; g++) o[g] = fma2(one2, o[g], mul2(wb[g][i], v));
    }
    // chunk c + 1's weights into the buffer chunk c - 1's used; then every lane is done with chunk c (its values'
    // buffer is the next one refilled) and the weights are in place
    store_weights(c + 1, wn);
    __syncwarp();
  }
#pragma unroll
  for (int g = 0; g < G; g++) {
    const int h = kvh * G + g;
    if (h < h0 || h >= h1) continue;
    float *dst = out + (int64_t)tok * out_stride + (int64_t)h * hs + dim0 + 2 * lane;
    dst[0] = lo(o[g]);
    dst[1] = hi(o[g]);
    if (QUANT) {
      // quantize_x (kernel.ts:129-156) of the head's values dim0 .. + 63: two groups of 32, on lanes 0-15 and 16-31,
      // value 2(l % 16) + e of its group on lane l. Class (index mod 4) 0 and 1 are the even lanes' two values, 2
      // and 3 the odd lanes': each class's largest |value| over the eight lanes of its parity, then the scalar
      // comparisons, scale and rounding of quantize_group.
      float ma = fabsf(lo(o[g])), mb = fabsf(hi(o[g]));
#pragma unroll
      for (int x = 2; x <= 8; x <<= 1) {
        ma = wmax(ma, __shfl_xor_sync(FULL, ma, x));
        mb = wmax(mb, __shfl_xor_sync(FULL, mb, x));
      }
      const float oa = __shfl_xor_sync(FULL, ma, 1), ob = __shfl_xor_sync(FULL, mb, 1);
      const bool even = (lane & 1) == 0;
      float amax = even ? ma : oa;
      const float m1 = even ? mb : ob, m2 = even ? oa : ma, m3 = even ? ob : mb;
      if (m1 > amax) amax = m1;
      if (m2 > amax) amax = m2;
      if (m3 > amax) amax = m3;
      const float scale = fdiv(amax, bias == 0 ? 127.0f : 63.0f);
      const float inv = scale > 0 ? fdiv(1.0f, scale) : 0.0f;
      const uint32_t q0 = (uint8_t)(int8_t)(quantize_one(lo(o[g]), inv, bias) - shift);
      const uint32_t q1 = (uint8_t)(int8_t)(quantize_one(hi(o[g]), inv, bias) - shift);
      const int64_t j = (int64_t)h * hs + dim0 + 2 * lane;
      *reinterpret_cast<uint16_t *>(xq + (int64_t)tok * q_stride + j) = (uint16_t)(q0 | (q1 << 8));
      if ((lane & 15) == 0) xs[(int64_t)tok * s_stride + (j >> 5) * g_stride] = scale;
    }
  }
}

// the softmax of count tokens' rows: a warp a row where the longest fits SOFTMAX_ROW_MAX, else a block a row
int launch_softmax(float *att, const int32_t *pos, int pos0, int P, int nh, int h0, int h1, int count, int max_count,
                   size_t smem_soft, cudaStream_t stream) {
  if (max_count <= SOFTMAX_ROW_MAX) {
    const int64_t rows = (int64_t)count * nh;
    launch(attn_softmax_rows, (unsigned)((rows + SOFTMAX_ROWS - 1) / SOFTMAX_ROWS), 32 * SOFTMAX_ROWS, 0, stream, att,
           pos, pos0, P, nh, h0, h1, count);
    B200_LAUNCHED("attn_softmax_rows");
    return 0;
  }
  launch(attn_softmax_tiled, dim3(nh, count), 256, smem_soft, stream, att, pos, pos0, P, nh, h0, h1);
  B200_LAUNCHED("attn_softmax_tiled");
  return 0;
}

template <bool HALF, int G>
int launch_tiled(float *out, int64_t out_stride, const float *q, int64_t q_stride, const void *kc, const void *vc,
                 float *att, const int32_t *seq, const int32_t *pos, int pos0, const int32_t *tiles, int ntiles,
                 int count, int64_t seq_stride, int P, int max_count, int nh, int nkv, int hs, int h0, int h1, int vec,
                 cudaStream_t stream, AttentionQuant *quant) {
  const size_t smem_soft = (size_t)max_count * sizeof(float);
  if (smem_soft > MAX_SOFTMAX_SMEM) return fail(B200FWD_EINVAL, "attention: more positions than one block's shared memory");
  if (!tiles && vec && hs % 2 == 0 && G * (hs / 2) <= 1024) {
    // one query token a tile: the decode kernels
    const size_t smem_scores = (size_t)G * hs * sizeof(float) + (size_t)DEC_POS * (hs * (HALF ? 2 : 4) + 16);
    if (smem_scores > MAX_TILE_SMEM) return fail(B200FWD_EUNSUPPORTED, "attention: heads too wide for a key chunk");
    B200_CUDA(cudaFuncSetAttribute(attn_scores_decode<HALF, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)MAX_TILE_SMEM));
    launch(attn_scores_decode<HALF, G>, dim3((max_count + DEC_POS - 1) / DEC_POS, nkv, count), DEC_POS, smem_scores,
           stream, q, q_stride, kc, att, seq, pos, pos0, seq_stride, P, nh, nkv, hs, h0, h1, 1.0f);
    B200_LAUNCHED("attn_scores_decode");
    CHECK_ATT(launch_softmax(att, pos, pos0, P, nh, h0, h1, count, max_count, smem_soft, stream));
    // the head's values split over `parts` blocks per token (more blocks streaming at once; the positions stay in
    // one chain per value): the most parts, up to two (measured best at 64 sequences of 512 to 8192 positions: 4 as
    // fast, 8 slower), whose rows are whole 16-byte pieces of an even number of values and that leave a block at
    // least one warp (B200FWD_ATT_PARTS sets the cap, a tuning knob for measurements)
    static const int cap = [] {
      const char *v = getenv("B200FWD_ATT_PARTS");
      const int c = v ? atoi(v) : 0;
      return c == 1 || c == 2 || c == 4 || c == 8 ? c : 2;
    }();
    if (HALF && hs % 64 == 0) {
      // every head written: quantize_x of the rows in the same kernel (2-byte stores of a lane's two values)
      const bool fold = quant && h0 == 0 && h1 == nh && reinterpret_cast<uintptr_t>(quant->xq) % 2 == 0 &&
                        quant->q_stride % 2 == 0;
      if (fold)
        launch(attn_values_decode_h<G, true>, dim3(nkv * (hs / 64), count), 32, 0, stream, out, out_stride,
               static_cast<const uint16_t *>(vc), att, seq, pos, pos0, seq_stride, P, nh, nkv, hs, h0, h1, 1.0f,
               quant->xq, quant->q_stride, quant->xs, quant->s_stride, quant->g_stride, quant->bias, quant->shift);
      else
        launch(attn_values_decode_h<G, false>, dim3(nkv * (hs / 64), count), 32, 0, stream, out, out_stride,
               static_cast<const uint16_t *>(vc), att, seq, pos, pos0, seq_stride, P, nh, nkv, hs, h0, h1, 1.0f,
               nullptr, 0, nullptr, 0, 0, 0, 0);
      B200_LAUNCHED("attn_values_decode_h");
      if (fold) quant->done = 1;
      return 0;
    }
    int parts = 1;
    for (int p = cap; p > 1; p /= 2) {
      const int dims = hs / p;
      if (hs % p == 0 && dims % 2 == 0 && (dims * (HALF ? 2 : 4)) % 16 == 0 && G * dims / 2 >= 32) {
        parts = p;
        break;
      }
    }
    const int threads = ((G * (hs / parts / 2) + 31) / 32) * 32;
    const size_t smem_values = values_smem(hs / parts, G, HALF);
    if (smem_values > MAX_TILE_SMEM) return fail(B200FWD_EUNSUPPORTED, "attention: heads too wide for a value chunk");
    B200_CUDA(cudaFuncSetAttribute(attn_values_decode<HALF, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)MAX_TILE_SMEM));
    launch(attn_values_decode<HALF, G>, dim3(nkv, count, parts), threads, smem_values, stream, out, out_stride, vc, att,
           seq, pos, pos0, seq_stride, P, nh, nkv, hs, h0, h1,
           P % 4 == 0 && reinterpret_cast<uintptr_t>(att) % 16 == 0 ? 1 : 0, 1.0f);
    B200_LAUNCHED("attn_values_decode");
    return 0;
  }
  const int chunks = (max_count + ATT_CH - 1) / ATT_CH;
  if (tiles && vec && hs % RB_VAL == 0 && q_stride % 4 == 0 && out_stride % 4 == 0 && P % 4 == 0 &&
      reinterpret_cast<uintptr_t>(q) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
      reinterpret_cast<uintptr_t>(att) % 16 == 0) {
    // prompt blocks: the register-blocked kernels
    const size_t smem_s = (size_t)(RB_POS + ATT_TT * G) * (hs + 4) * sizeof(float);
    const size_t smem_v = (size_t)(RB_POS * (RB_VAL + 4) + ATT_TT * G * (RB_POS + 4)) * sizeof(float);
    if (smem_s <= MAX_TILE_SMEM && smem_v <= MAX_TILE_SMEM) {
      B200_CUDA(cudaFuncSetAttribute(attn_scores_rb<HALF, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)MAX_TILE_SMEM));
      B200_CUDA(cudaFuncSetAttribute(attn_values_rb<HALF, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)MAX_TILE_SMEM));
      launch(attn_scores_rb<HALF, G>, dim3((max_count + RB_POS - 1) / RB_POS, nkv, ntiles), 64 * G, smem_s, stream, q,
             q_stride, kc, att, seq, pos, pos0, tiles, seq_stride, P, nh, nkv, hs, h0, h1, 1.0f);
      B200_LAUNCHED("attn_scores_rb");
      CHECK_ATT(launch_softmax(att, pos, pos0, P, nh, h0, h1, count, max_count, smem_soft, stream));
      launch(attn_values_rb<HALF, G>, dim3(nkv, ntiles, hs / RB_VAL), 64 * G, smem_v, stream, out, out_stride, vc, att,
             seq, pos, pos0, tiles, seq_stride, P, nh, nkv, hs, h0, h1, 1.0f);
      B200_LAUNCHED("attn_values_rb");
      return 0;
    }
  }
  const int tt = tiles ? ATT_TT : 1;
  const int hsp = (hs + 3) & ~3;
  const size_t smem_scores = (size_t)(ATT_CH * (hsp + 4) + tt * G * hsp) * sizeof(float);
  const size_t smem_values = (size_t)(ATT_CH * hs + tt * G * ATT_CH) * sizeof(float);
  if (smem_scores > MAX_TILE_SMEM || smem_values > MAX_TILE_SMEM)
    return fail(B200FWD_EUNSUPPORTED, "attention: heads too wide for a tile in shared memory");
  B200_CUDA(cudaFuncSetAttribute(attn_scores_tiled<HALF, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)MAX_TILE_SMEM));
  B200_CUDA(cudaFuncSetAttribute(attn_values_tiled<HALF, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)MAX_TILE_SMEM));
  launch(attn_scores_tiled<HALF, G>, dim3(chunks, nkv, ntiles), ATT_CH, smem_scores, stream, q, q_stride, kc, att, seq,
         pos, pos0, tiles, seq_stride, P, nh, nkv, hs, h0, h1, vec, 1.0f);
  B200_LAUNCHED("attn_scores_tiled");
  CHECK_ATT(launch_softmax(att, pos, pos0, P, nh, h0, h1, count, max_count, smem_soft, stream));
  const int threads = ((G * ((hs + 1) / 2) + 31) / 32) * 32;
  launch(attn_values_tiled<HALF, G>, dim3(nkv, ntiles), threads, smem_values, stream, out, out_stride, vc, att, seq,
         pos, pos0, tiles, seq_stride, P, nh, nkv, hs, h0, h1, vec, 1.0f);
  B200_LAUNCHED("attn_values_tiled");
  return 0;
}

}  // namespace

int prepare_attention() {
  int device = 0;
  B200_CUDA(cudaGetDevice(&device));
  static std::atomic<uint64_t> opted{0};
  if (device >= 64 || !(opted.load() & (1ull << device))) {
    B200_CUDA(cudaFuncSetAttribute(attn_softmax_tiled, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)MAX_SOFTMAX_SMEM));
    if (device < 64) opted.fetch_or(1ull << device);
  }
  return 0;
}

int launch_attention(float *out, int64_t out_stride, const float *q, int64_t q_stride, const void *kc, const void *vc,
                     float *att, const int32_t *seq, const int32_t *pos, int pos0, const int32_t *tiles, int ntiles,
                     int count, int64_t seq_stride, int P, int max_count, int nh, int nkv, int hs, int h0, int h1,
                     int half, cudaStream_t stream, AttentionQuant *quant) {
  if (quant) quant->done = 0;
  if (count <= 0) return 0;
  if (nkv <= 0 || nh % nkv) return fail(B200FWD_EINVAL, "attention: heads must be a multiple of the kv heads");
  if (max_count > P) return fail(B200FWD_EINVAL, "attention: a position past the scratch");
  if (!tiles) ntiles = count;
  CHECK_ATT(prepare_attention());
  // 16-byte loads where every row of the head starts on 16 bytes
  const int esize = half ? 2 : 4, per = half ? 8 : 4;
  const int vec = hs % per == 0 && (nkv * hs * esize) % 16 == 0 && reinterpret_cast<uintptr_t>(kc) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(vc) % 16 == 0 && (seq_stride * esize) % 16 == 0;
  const int G = nh / nkv;
#define B200_ATT(H, GG)                                                                                            \
  return launch_tiled<H, GG>(out, out_stride, q, q_stride, kc, vc, att, seq, pos, pos0, tiles, ntiles, count,     \
                             seq_stride, P, max_count, nh, nkv, hs, h0, h1, vec, stream, quant)
  if (half) {
    switch (G) {
      case 1: B200_ATT(true, 1);
      case 2: B200_ATT(true, 2);
      case 4: B200_ATT(true, 4);
      case 8: B200_ATT(true, 8);
    }
  } else {
    switch (G) {
      case 1: B200_ATT(false, 1);
      case 2: B200_ATT(false, 2);
      case 4: B200_ATT(false, 4);
      case 8: B200_ATT(false, 8);
    }
  }
#undef B200_ATT
  return fail(B200FWD_EUNSUPPORTED, "attention: query heads per kv head must be 1, 2, 4 or 8");
}

}  // namespace b200
