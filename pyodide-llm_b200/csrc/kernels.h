// kernels.h — the launchers of the hot-path kernels (kernels.cu), for the engine and the C ABI.
//
// Every launcher computes the reference's numbers to the bit (exact.cuh) and returns 0 or a B200FWD_E* code.
// Token rows sit `*_stride` elements apart; all pointers are device pointers.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace b200 {

// up to three matrices that read the same activations (q, k and v; w1 and w3), run as one launch: forward.js puts
// them in one phase (forward.js:476,516). Rows of the jobs follow each other.
struct MatJob {
  const int8_t *w;    // [rows][n]
  const float *s;     // [rows][n/32]
  const int32_t *c;   // int8_sums corrections [rows][n/32], or null: dot(w, q - 64) taken directly
  float *out;         // token t's row at out + t * out_stride
  int rows;
  int accumulate;     // out += the result (the residual add of forward.js:500,519), else out = the result
  int64_t out_stride;
  int sstride;        // scales (and corrections) per row; 0: n / 32
};
struct MatJobs {
  MatJob job[3];
  int njobs;
  int n;
  int total_rows;
  int signed_input;   // the activations are already less the bias (q - 64): a group's integer is dot(w, x)
};

// Activation scales: token t's group g at xs[t * s_stride + g * g_stride] (one row per token: g_stride 1; the
// engine's layout, one row per group, which the tensor-core matmul reads: s_stride 1).
// kernel_relaxed.ts:34-67/164-183 (relaxed) or kernel.ts:231-251 (8-bit): count tokens of activations
int launch_matvec(const MatJobs &jobs, const int8_t *xq, const float *xs, int64_t q_stride, int64_t s_stride,
                  int64_t g_stride, int count, bool relaxed, cudaStream_t stream);

// The quantizing kernels below store each int8 less `shift` (0: the reference's bytes; 64 with bias 64: q - 64,
// the signed values whose dot products with the weights are the reference's corrected group integers).
// kernel.ts:330-342 rmsnorm then kernel.ts:129-156 quantize_x of its output, per token; channels (nch of them,
// device) are taken out of the normalized vector first (forward.js:525-528: picked[c] = value, value = 0).
// out_f (nullable) also gets the normalized floats.
int launch_norm_quantize(const float *x, int64_t x_stride, const float *w, int n, float eps, int bias, int count,
                         int8_t *xq, int64_t q_stride, float *xs, int64_t s_stride, int64_t g_stride,
                         const int32_t *channels, int nch, float *picked, float *out_f, int64_t out_stride,
                         cudaStream_t stream, int shift = 0);
// kernel.ts:129-156 quantize_x, per token
int launch_quantize(const float *x, int64_t x_stride, int n, int bias, int count, int8_t *xq, int64_t q_stride,
                    float *xs, int64_t s_stride, int64_t g_stride, cudaStream_t stream, int shift = 0);
// kernel.ts:654-667 swiglu then quantize_x of its output, per token
int launch_swiglu_quantize(const float *h1, const float *h3, int64_t stride, int n, int bias, int count, int8_t *xq,
                           int64_t q_stride, float *xs, int64_t s_stride, int64_t g_stride, cudaStream_t stream,
                           int shift = 0);
// forward.js:403-414 embed of int8 rows: x[t][i] = w[token*dim+i] * s[token*sstride + i/32]; tokens on the device
int launch_embed(const int8_t *w, const float *s, int sstride, const int32_t *tokens, int count, int dim, float *x,
                 int64_t x_stride, cudaStream_t stream);
// forward.js:489-494: rope (kernel.ts:344-357) on q and k of each token at its position, and k, v into its
// sequence's cache (to_f16 when half). cache of sequence s: kc + s * seq_stride elements, [pos][nkv*hs]
int launch_rope_cache(float *q, int64_t q_stride, const float *k, const float *v, int64_t kv_stride, const float *cos,
                      const float *sin, const int32_t *pos, const int32_t *seq, int count, void *kc, void *vc,
                      int64_t seq_stride, int half, int nh, int nkv, int hs, int rot, cudaStream_t stream);
// kernel.ts:447-566 attentionOf for count tokens (attention.cu), each against its sequence's cache up to its
// position: device arrays seq and pos, or, with pos null, every token at pos0 of sequence 0. tiles: ntiles pairs
// (first token, count) of up to 16 consecutive tokens of one sequence at consecutive positions, sharing the keys and
// values they read; null: every token its own tile. att: [count][nh][P] scratch (P >= max position + 1), left
// holding the softmax weights; max_count bounds pos + 1 for the grid. Heads h0..h1.
// quant (may be null): where the kernels may also write out's rows as quantize_x writes them (launch_quantize's
// arguments); done = 1 when they did, so the caller's own quantize_x of out is not needed.
struct AttentionQuant {
  int8_t *xq;
  int64_t q_stride;
  float *xs;
  int64_t s_stride, g_stride;
  int bias, shift;
  int done;
};
int launch_attention(float *out, int64_t out_stride, const float *q, int64_t q_stride, const void *kc, const void *vc,
                     float *att, const int32_t *seq, const int32_t *pos, int pos0, const int32_t *tiles, int ntiles,
                     int count, int64_t seq_stride, int P, int max_count, int nh, int nkv, int hs, int h0, int h1,
                     int half, cudaStream_t stream, AttentionQuant *quant = nullptr);
constexpr int ATTN_TILE = 16;  // tokens of a tile at most
// the attention kernels' shared-memory opt-in on the current device (once; before any graph capture)
int prepare_attention();
// kernel.ts:671-689 add_columns for count tokens (y rows y_stride apart, a rows a_stride apart)
int launch_add_columns(float *y, int64_t y_stride, const float *rows, const float *a, int64_t a_stride, int nc,
                       int n, int count, cudaStream_t stream);
// argmax of count rows: mode 0 kernel.ts:695-699 (first index with `>`), mode 1 numpy.argmax (a NaN wins)
int launch_argmax(int32_t *out, const float *x, int64_t stride, int n, int count, int mode, cudaStream_t stream);
// dst[i] = src[idx[i]] (rows of dim floats)
// activation scales of count tokens from one row per token (s_stride apart) to one row per group (t_stride apart)
int launch_scales_by_group(float *dst, int64_t t_stride, const float *src, int64_t s_stride, int count, int groups,
                           cudaStream_t stream);
int launch_gather_rows(float *dst, int64_t dst_stride, const float *src, int64_t src_stride, const int32_t *idx,
                       int count, int dim, cudaStream_t stream);
// forward.js:799-813 the outlier channels' float32 columns: cols[i][v] = w[v*dim+c_i] * s[v*sstride + c_i/32]
int launch_outlier_columns(float *cols, const int8_t *w, const float *s, int sstride, int dim, int vocab,
                           const int32_t *channels, int nch, cudaStream_t stream);
int launch_to_f16(uint16_t *out, const float *x, int64_t n, cudaStream_t stream);
int launch_from_f16(float *out, const uint16_t *x, int64_t n, cudaStream_t stream);
int launch_add_inplace(float *x, const float *y, int64_t n, cudaStream_t stream);
int launch_swiglu(float *out, const float *h1, const float *h3, int64_t n, cudaStream_t stream);
int launch_int8_sums(int32_t *out, const int8_t *w, int64_t groups, cudaStream_t stream);
// greedy bookkeeping on the device: tokens[i] = ids[i]; pos[i] += 1; history[i * steps + *step] = ids[i]; ++*step;
// *bad = 1 where the chosen logit (logits[i * vocab + id]) is not finite
int launch_advance(int32_t *tokens, int32_t *pos, const int32_t *ids, int32_t *history, int steps, int32_t *step,
                   int count, const float *logits, int64_t vocab, int32_t *bad, cudaStream_t stream);
// kernel.ts:705-719 penalize for count sequences (logits rows stride apart): recent [count][window] tokens, the first
// min(recent_count[s], window) of row s used (recent_count null: all window); rows with done[s] (nullable) left alone
int launch_penalize(float *logits, int64_t stride, const int32_t *recent, int window, const int32_t *recent_count,
                    float penalty, const int32_t *done, int count, cudaStream_t stream);
// kernel.ts:808-868 sample for count sequences: out[s] the id drawn from logits row s with random[s * rstride + *step]
// (step nullable: 0; random null: random0), -1 where the largest logit is not finite, -2 where the nucleus sort's
// stack ran out; scratch sample_scratch_words(n) floats and stacks sample_stack_words() int32 per sequence; done[s]
// (nullable) skips s
int launch_sample(int32_t *out, const float *logits, int64_t stride, int n, float temperature, float topp,
                  const double *random, double random0, int64_t rstride, const int32_t *step, float *scratch,
                  int32_t *stacks, const int32_t *done, int count, cudaStream_t stream);
size_t sample_scratch_words(int n);
size_t sample_stack_words();
// the bookkeeping of one sampled step (sampling.cu advance_sampled_kernel)
int launch_advance_sampled(int32_t *tokens, int32_t *pos, const int32_t *ids, int32_t *history, int steps,
                           int32_t *step, int count, const float *logits, int64_t vocab, int greedy, int32_t *recent,
                           int window, int32_t *recent_count, const int32_t *stops, int nstops, int32_t *done,
                           int32_t *made, int32_t *bad, cudaStream_t stream);
// causal attention of whole sequences on the tensor cores (attention_tc.cu): q [B][S][H][D], k and v [B][S][KV][D]
// float32, RoPE tables [S][D/2]; out [B][S][H][D]; scratch prefill_attention_scratch() bytes (256-byte aligned)
size_t prefill_attention_scratch(int B, int S, int H, int KV, int D);
int launch_prefill_attention(float *out, const float *q, const float *k, const float *v, const float *cos_t,
                             const float *sin_t, int B, int S, int H, int KV, int D, float scale, void *scratch,
                             cudaStream_t stream);
// after the kernel: its pipeline-wait error word (in the scratch) as a status (synchronizes the stream)
int check_prefill_attention(const void *scratch, int B, int S, int H, int KV, int D, cudaStream_t stream);
// kernel.ts:330-342 rmsnorm of count rows (stride floats apart)
int launch_rmsnorm(float *out, const float *x, const float *w, int n, float eps, int count, int64_t stride,
                   cudaStream_t stream);
// kernel.ts:344-357 rope of one vector
int launch_rope(float *v, const float *fcr, const float *fci, int nh, int hs, int rot, cudaStream_t stream);

}  // namespace b200
