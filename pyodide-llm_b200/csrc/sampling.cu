// sampling.cu — kernel.ts:705-868 penalize and sample on the device, for many sequences at once (one block each),
// each to the bit as the reference's WASM computes it alone, and the bookkeeping of one sampled step.
//
// sample() (kernel.ts:808-868), block-parallel where the reference's order does not matter and sequential (one
// thread) where it does:
//   - the largest logit (a NaN anywhere wins; order-free): block reduction;
//   - the tokens at or above the nucleus floor, in vocabulary order, as (logit - best, id): an ordered compaction
//     (each thread a contiguous range, a block-wide prefix sum of the counts);
//   - the exponentials: vexp of (value * (1 / temperature)) for the fours of the list, fexp of (value / temperature)
//     past them, each independent;
//   - the float64 total (a chain in list order: one thread), the largest probability (order-free);
//   - with a nucleus: the tokens at or above the cutoff, ordered compaction again; the reference's partial quicksort
//     (median of three, insertion sort for 13 or fewer, stopping once the nucleus is complete), one thread, with an
//     explicit stack in global memory (bounded: past it the token is -2 and the host reports it);
//   - the cumulative float64 walk to the drawn number: one thread.
// The sequential parts run on one thread per sequence; for a peaked distribution they are short, for a flat one over
// a large vocabulary they take milliseconds.
#include <cfloat>
#include <cstdint>

#include "common.h"
#include "exact.cuh"
#include "kernels.h"

namespace b200 {
namespace {

constexpr unsigned FULL = 0xffffffffu;
constexpr int ST = 1024;            // threads of a sampling block
constexpr int STACK_FRAMES = 4096;  // the quicksort's pending frames at most (three int32 each)

__device__ __forceinline__ bool finite(float v) { return v == v && v != INFINITY && v != -INFINITY; }

// block-wide reduction of wmax (shared scratch of 32)
__device__ float block_max(float v, float *red) {
  for (int o = 16; o > 0; o >>= 1) v = wmax(v, __shfl_xor_sync(FULL, v, o));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < (int)(blockDim.x >> 5) ? red[lane] : red[0];
    for (int o = 16; o > 0; o >>= 1) v = wmax(v, __shfl_xor_sync(FULL, v, o));
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

// exclusive prefix sum of one int per thread; returns this thread's offset, *total the sum (shared scratch of 33)
__device__ int block_scan(int c, int *red, int *total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = c;
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(FULL, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) red[warp] = x;
  __syncthreads();
  if (warp == 0) {
    const int nw = (int)(blockDim.x >> 5);
    int w = lane < nw ? red[lane] : 0;
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(FULL, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) red[lane] = w;  // inclusive
    if (lane == nw - 1) red[32] = w;
  }
  __syncthreads();
  const int before = (warp ? red[warp - 1] : 0) + x - c;
  *total = red[32];
  return before;
}

// kernel.ts:723-730 intoNucleus
__device__ bool into_nucleus(double &mass, double limit, int &last, const float *probs, int lo, int hi) {
  for (int k = lo; k <= hi; k++) {
    mass += (double)probs[k];
    if (mass >= limit) {
      last = k;
      return true;
    }
  }
  return false;
}

// kernel.ts:732-775 sortNucleus on one thread, its recursion on an explicit stack of (i, j, hi) frames: after the
// left part (lo..j) is done, the pivot's equals (j+1..i-1) join the nucleus and the loop goes on from i. Returns
// false when the stack would overflow.
__device__ bool sort_nucleus(float *probs, int32_t *index, int lo, int hi, double &mass, double limit, int &last,
                             int32_t *stack) {
  int sp = 0;
  for (;;) {
    if (hi - lo > 12) {
      const int mid = lo + ((hi - lo) >> 1);
      float a = probs[lo], b = probs[mid];
      const float c = probs[hi];
      if (a < b) {
        const float t = a;
        a = b;
        b = t;
      }
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
          const float p = probs[i];
          probs[i] = probs[j];
          probs[j] = p;
          const int32_t x = index[i];
          index[i] = index[j];
          index[j] = x;
          i++;
          j--;
        }
      }
      if (sp >= STACK_FRAMES) return false;
      stack[3 * sp] = i;
      stack[3 * sp + 1] = j;
      stack[3 * sp + 2] = hi;
      sp++;
      hi = j;  // the left part first (the reference's recursive call)
      continue;
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
    into_nucleus(mass, limit, last, probs, lo, hi);
    // back in the callers: each returns as soon as the nucleus is complete
    for (;;) {
      if (last >= 0 || sp == 0) return true;
      sp--;
      const int i = stack[3 * sp], j = stack[3 * sp + 1], h = stack[3 * sp + 2];
      if (into_nucleus(mass, limit, last, probs, j + 1, i - 1)) return true;
      lo = i;
      hi = h;
      break;
    }
  }
}

// kernel.ts:705-719 penalize, one block per sequence: recent[s][0..count) (a ring of the last tokens, any order),
// each token made less likely once. Sequences with done[s] are left alone.
__global__ void penalize_kernel(float *logits, int64_t stride, const int32_t *recent, int window,
                                const int32_t *recent_count, float penalty, const int32_t *done) {
  pdl_begin();
  const int s = blockIdx.x;
  if (done && done[s]) return;
  const int count = recent_count ? min(recent_count[s], window) : window;
  const int32_t *t = recent + (int64_t)s * window;
  for (int i = threadIdx.x; i < count; i += blockDim.x) {
    const int32_t token = t[i];
    bool seen = false;
    for (int j = 0; j < i; j++)
      if (t[j] == token) {
        seen = true;
        break;
      }
    if (seen) continue;
    float *at = logits + (int64_t)s * stride + token;
    const float v = *at;
    *at = v > 0 ? fdiv(v, penalty) : fmul(v, penalty);
  }
}

// kernel.ts:808-868 sample, one block per sequence s: logits row s, random[s * rstride + *step] (step null: 0),
// scratch (4 n words: two lists of (probability, id)) and stack at s's own offsets; the drawn id into out[s], -1
// where the largest logit is not finite, -2 where the quicksort's stack ran out. Sequences with done[s] are skipped.
__global__ void __launch_bounds__(ST)
    sample_kernel(int32_t *out, const float *logits, int64_t stride, int n, float temperature, float topp,
                  const double *random, double random0, int64_t rstride, const int32_t *step, float *scratch,
                  int32_t *stacks, const int32_t *done) {
  pdl_begin();
  __shared__ float fred[32];
  __shared__ int ired[33];
  __shared__ double shared_total;
  const int s = blockIdx.x;
  if (done && done[s]) return;
  const float *x = logits + (int64_t)s * stride;
  float *probs = scratch + (int64_t)s * 4 * n;
  int32_t *index = reinterpret_cast<int32_t *>(probs + n);
  float *probs2 = probs + 2 * n;
  int32_t *index2 = reinterpret_cast<int32_t *>(probs + 3 * n);
  // the largest logit (kernel.ts:423-445 largest: from x[0], a NaN anywhere, order-free)
  float m = x[0];
  for (int i = threadIdx.x; i < n; i += blockDim.x) m = wmax(m, x[i]);
  const float best = block_max(m, fred);
  if (!finite(best)) {
    if (threadIdx.x == 0) out[s] = -1;
    return;
  }
  const bool nucleus = topp > 0 && topp < 1;
  const float floor = nucleus ? fsub(best, fmul(temperature, 16.118095f)) : -FLT_MAX;
  // the tokens at or above the floor in vocabulary order: (logit - best, id)
  const int per = (n + blockDim.x - 1) / blockDim.x;
  const int a = min(n, (int)threadIdx.x * per), b = min(n, a + per);
  int c = 0;
  for (int i = a; i < b; i++) c += x[i] >= floor ? 1 : 0;
  int count;
  int at = block_scan(c, ired, &count);
  for (int i = a; i < b; i++) {
    const float v = x[i];
    if (v >= floor) {
      probs[at] = fsub(v, best);
      index[at] = i;
      at++;
    }
  }
  __syncthreads();
  // the exponentials: the list's fours times 1/temperature through vexp, the rest over temperature through fexp
  const float inverse = fdiv(1.0f, temperature);
  const int count4 = count & ~3;
  for (int k = threadIdx.x; k < count; k += blockDim.x)
    probs[k] = k < count4 ? vexp(fmul(probs[k], inverse)) : fexp(fdiv(probs[k], temperature));
  float t = 0.0f;
  for (int k = threadIdx.x; k < count; k += blockDim.x) t = wmax(t, probs[k]);
  const float top = block_max(t, fred);
  if (threadIdx.x == 0) {
    double total = 0;
    for (int k = 0; k < count; k++) total += (double)probs[k];
    shared_total = total;
  }
  __syncthreads();
  const double total = shared_total;
  const double r = random ? random[(int64_t)s * rstride + (step ? *step : 0)] : random0;
  if (!nucleus) {
    if (threadIdx.x == 0) {
      const double target = r * total;
      double cumulative = 0;
      int32_t chosen = index[count - 1];
      for (int k = 0; k < count; k++) {
        cumulative += (double)probs[k];
        if (cumulative > target) {
          chosen = index[k];
          break;
        }
      }
      out[s] = chosen;
    }
    return;
  }
  // the tokens at or above the cutoff, in the list's order (kernel.ts:846-852)
  const double spread = (1.0 - (double)topp) / (double)(count > 1 ? count - 1 : 1) * total;
  const double cutoff = spread < (double)top ? spread : (double)top;
  const int pa = min(count, (int)threadIdx.x * ((count + blockDim.x - 1) / blockDim.x));
  const int pb = min(count, pa + (count + blockDim.x - 1) / blockDim.x);
  c = 0;
  for (int k = pa; k < pb; k++) c += (double)probs[k] >= cutoff ? 1 : 0;
  int likely;
  at = block_scan(c, ired, &likely);
  for (int k = pa; k < pb; k++) {
    const float p = probs[k];
    if ((double)p >= cutoff) {
      probs2[at] = p;
      index2[at] = index[k];
      at++;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double mass = 0;
    int last = -1;
    const bool ok = sort_nucleus(probs2, index2, 0, likely - 1, mass, (double)topp * total, last,
                                 stacks + (int64_t)s * 3 * STACK_FRAMES);
    if (!ok) {
      out[s] = -2;
    } else {
      if (last < 0) last = likely - 1;
      const double target = r * mass;
      double cumulative = 0;
      int32_t chosen = index2[last];
      for (int k = 0; k <= last; k++) {
        cumulative += (double)probs2[k];
        if (cumulative > target) {
          chosen = index2[k];
          break;
        }
      }
      out[s] = chosen;
    }
  }
}

// one sampled step of count sequences: the id into history[s][*step] (ids: the sampled ones, -1/-2 as sample gives
// them; greedy: the chosen logit not finite is -1 too), the ring of recent tokens, the next token and position; a
// stop token ends the sequence (done, no further position); *bad the first failure's code (1 not finite, 2 stack).
__global__ void advance_sampled_kernel(int32_t *tokens, int32_t *pos, const int32_t *ids, int32_t *history,
                                       int steps, int32_t *step, int count, const float *logits, int64_t vocab,
                                       int greedy, int32_t *recent, int window, int32_t *recent_count,
                                       const int32_t *stops, int nstops, int32_t *done, int32_t *made, int32_t *bad) {
  pdl_begin();
  const int i = threadIdx.x;
  const int atstep = *step;
  __syncthreads();
  if (i < count && !done[i]) {
    int32_t id = ids[i];
    if (greedy && id >= 0) {
      const float v = logits[(int64_t)i * vocab + id];
      if (!finite(v)) id = -1;  // llama2_numpy.greedy's NOT_FINITE (public/llama2_numpy.py:1521-1527)
    }
    if (id < 0) {
      atomicCAS(bad, 0, id == -1 ? 1 : 2);
      done[i] = 1;
    } else {
      if (atstep < steps) history[(int64_t)i * steps + atstep] = id;
      made[i] = atstep + 1;
      recent[(int64_t)i * window + recent_count[i] % window] = id;
      recent_count[i] += 1;
      bool stop = false;
      for (int k = 0; k < nstops; k++) stop |= stops[k] == id;
      if (stop) {
        done[i] = 1;  // the stop token is the last id; nothing is fed after it
      } else {
        tokens[i] = id;
        pos[i] += 1;
      }
    }
  }
  if (i == 0) *step = atstep + 1;
}

}  // namespace

size_t sample_scratch_words(int n) { return (size_t)4 * n; }
size_t sample_stack_words() { return (size_t)3 * STACK_FRAMES; }

int launch_penalize(float *logits, int64_t stride, const int32_t *recent, int window, const int32_t *recent_count,
                    float penalty, const int32_t *done, int count, cudaStream_t stream) {
  if (count <= 0) return 0;
  launch(penalize_kernel, count, 64, 0, stream, logits, stride, recent, window, recent_count, penalty, done);
  B200_LAUNCHED("penalize_kernel");
  return 0;
}

int launch_sample(int32_t *out, const float *logits, int64_t stride, int n, float temperature, float topp,
                  const double *random, double random0, int64_t rstride, const int32_t *step, float *scratch,
                  int32_t *stacks, const int32_t *done, int count, cudaStream_t stream) {
  if (count <= 0) return 0;
  if (n < 1) return fail(B200FWD_EINVAL, "sample: no logits");
  if (!(temperature > 0)) return fail(B200FWD_EINVAL, "sample: the temperature must be above 0 (0 is greedy)");
  launch(sample_kernel, count, ST, 0, stream, out, logits, stride, n, temperature, topp, random, random0, rstride, step,
         scratch, stacks, done);
  B200_LAUNCHED("sample_kernel");
  return 0;
}

int launch_advance_sampled(int32_t *tokens, int32_t *pos, const int32_t *ids, int32_t *history, int steps,
                           int32_t *step, int count, const float *logits, int64_t vocab, int greedy, int32_t *recent,
                           int window, int32_t *recent_count, const int32_t *stops, int nstops, int32_t *done,
                           int32_t *made, int32_t *bad, cudaStream_t stream) {
  if (count > 1024) return fail(B200FWD_EINVAL, "sampled steps: at most 1024 sequences at once");
  launch(advance_sampled_kernel, 1, ((count + 31) / 32) * 32, 0, stream, tokens, pos, ids, history, steps, step, count,
         logits, vocab, greedy, recent, window, recent_count, stops, nstops, done, made, bad);
  B200_LAUNCHED("advance_sampled_kernel");
  return 0;
}

}  // namespace b200
