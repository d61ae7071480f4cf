/* b200fwd.h — the C ABI of the B200 forward engine and of its kernels.
 *
 * Two layers, both plain C (no torch types, no C++ in the signatures):
 *
 *  1. The ENGINE: what `public/forward.js` `createForward()` returns to `llama2_numpy.Llama(external=...)`.
 *     A handle owns the checkpoint's tensors in HBM, the KV cache and the logits; the caller owns its logits
 *     array (bind). Every entry returns 0 on success or a negative B200FWD_E* code, never aborts, and leaves a
 *     message for b200fwd_last_error(). Calls on one handle are synchronous and not re-entrant, as forward.js's.
 *
 *  2. The KERNELS: the exports of `kernels/kernel.ts` and `kernels/kernel_relaxed.ts` that forward.js calls (the
 *     table `public/jobs.js:56-62` lists them), as sm_100a CUDA kernels on DEVICE pointers with a CUDA stream.
 *     Each one computes the same numbers as its WASM counterpart to the bit (same float operation order, no
 *     fused multiply-add), so a host that drove the WASM kernels can drive these.
 *
 * Reference citations are `path:line` inside the ssig33/pyodide-llm project.
 */
#ifndef B200FWD_H
#define B200FWD_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200FWD_ABI_VERSION 1

/* status codes */
#define B200FWD_OK 0
#define B200FWD_EINVAL (-1)     /* an argument or the plan is wrong */
#define B200FWD_ECUDA (-2)      /* a CUDA call failed (message says which) */
#define B200FWD_ENOMEM (-3)     /* device memory could not be had */
#define B200FWD_EUNSUPPORTED (-4) /* a model form this engine does not run (message says which) */
#define B200FWD_ENOTFINITE (-5) /* logits that are not finite numbers (llama2_numpy.py:548 NOT_FINITE) */
#define B200FWD_ETIMEOUT (-6)   /* a bounded host wait gave up */

typedef void *b200fwd_stream; /* a cudaStream_t; NULL = the legacy default stream */

/* ---------------------------------------------------------------------------------------------- the plan
 * The plan dict `Llama.external_forward` hands to `external.start(plan)` (public/llama2_numpy.py:1261-1270),
 * as a C struct. Tensor offsets are byte offsets into the checkpoint (public/llama2_numpy.py:740-775,
 * `Tensor.plan()` / `Places.take`). Only the llama arch with int8 matrices is run (the scope of this engine). */
#define B200FWD_TENSOR_ABSENT 0
#define B200FWD_TENSOR_INT8 1 /* int8 values at offset, then one fp32 scale per group of the last dim at scales */
#define B200FWD_TENSOR_F32 2
#define B200FWD_TENSOR_F16 3

typedef struct b200fwd_tensor {
  int32_t kind;      /* B200FWD_TENSOR_* */
  int32_t group;     /* int8: values per scale (quantize.py: 32, halved until it divides the row) */
  int64_t offset;    /* byte offset of the values in the checkpoint */
  int64_t scales;    /* int8: byte offset of the fp32 scales */
  int32_t ndim;
  int32_t pad_;
  int64_t shape[4];
} b200fwd_tensor;

#define B200FWD_MAX_OUTLIERS 16

typedef struct b200fwd_plan {
  int32_t dim, hidden_dim, n_layers, n_heads, n_kv_heads, head_size, vocab_size, seq_len;
  int32_t rotary;            /* values of a head RoPE turns (head_size: all) */
  int32_t kv_start;          /* KV_START: the cache's first capacity, doubled as it fills (llama2_numpy.py:549) */
  float rms_norm_eps;
  int32_t shared_classifier; /* wcls is the embedding table */
  int32_t int8;              /* the int8 kernels compute on the int8 weights */
  int32_t relaxed;           /* 7-bit activations + bias 64 (matmul_q8r) rather than 8-bit (matmul_q8) */
  int32_t half_kv;           /* the keys and values may be float16 (plan.half_kv) */
  int32_t n_outliers;        /* outlier channels of the classifier input (plan.outliers, T92) */
  int32_t outliers[B200FWD_MAX_OUTLIERS];
  b200fwd_tensor token_embedding_table, rms_att_weight, wq, wk, wv, wo, rms_ffn_weight, w1, w2, w3,
      rms_final_weight, wcls;
  /* plan.derived: the fp32 RoPE tables [seq_len][head_size/2] that Python computes (llama2_numpy.py:1250-1254) */
  const float *freq_cis_real;
  const float *freq_cis_imag;
} b200fwd_plan;

/* What forward.js learns from the page rather than from the plan. */
typedef struct b200fwd_options {
  int32_t half_keys;   /* -1: forward.js's default (float16 where every head has keys of its own, forward.js:
                          203 `halfKeys ?? kvHeads >= heads`); 0: float32; 1: float16 (keysInHalf said so) */
  int32_t slots;       /* independent sequences the engine holds (1 = forward.js; >1 = the batched extension) */
  int32_t device;      /* CUDA device ordinal */
  int32_t max_tokens;  /* the most tokens one run() takes (a prompt block times slots); 0 = max(512, 16 * slots) */
  int32_t capacity;    /* first KV capacity per slot; 0 = plan.kv_start (then doubled as forward.js grow()) */
  int32_t checkpoint_on_device; /* 1: `checkpoint` is a DEVICE pointer, whose tensors create() copies into the
                                   engine's own layout (the caller may free it afterwards); 0: host memory */
  int32_t reserved[6];
} b200fwd_options;

typedef struct b200fwd_engine b200fwd_engine;

/* ---------------------------------------------------------------------------------------------- the engine */

/* public/forward.js:571-590 `external({...}).start(plan)` -> createForward (forward.js:626-...): uploads the
 * checkpoint bytes (host memory, `size` bytes) to HBM, makes the outlier columns (forward.js:799-813) and the KV
 * cache (forward.js:828-833). `options` may be NULL. */
int b200fwd_create(const void *checkpoint, size_t size, const b200fwd_plan *plan, const b200fwd_options *options,
                   b200fwd_engine **out);
/* forward.js:1745 `bind(array)`: where forward() writes the vocab_size logits (host memory, Python's array). */
int b200fwd_bind_logits(b200fwd_engine *engine, float *logits);
/* forward.js:1891-1912 `forward(token, pos, needLogits)`: one token of slot 0 through the layers, its key and value
 * into the cache at pos; the logits into the bound array when need_logits. */
int b200fwd_forward(b200fwd_engine *engine, int32_t token, int32_t pos, int32_t need_logits);
/* forward.js:1755-1769 `forwardMany(tokens, pos)`: a prompt's tokens of slot 0 at pos, pos+1, ..., no logits,
 * bit-identical to forward() token by token (tests/forward-check.mjs:440-451). */
int b200fwd_forward_many(b200fwd_engine *engine, const int32_t *tokens, int32_t count, int32_t pos);
/* forward.js:1773-1778 `promptBlock`: how many prompt tokens Python should hand forwardMany at once. */
int b200fwd_prompt_block(b200fwd_engine *engine, int32_t *out);
/* forward.js:1939-1953 `keysAndValues(from, count)`: slot's cache at positions from..from+count-1 as float32,
 * [layers][count][kvDim] each, into host arrays. */
int b200fwd_keys_values(b200fwd_engine *engine, int32_t slot, int32_t from, int32_t count, float *keys,
                        float *values);
/* forward.js:1936 `logits()`: the last logits (vocab_size floats) into a host array. */
int b200fwd_logits(b200fwd_engine *engine, float *out);
/* forward.js:1673-1675 `backend`: the line that names what runs. */
int b200fwd_backend(b200fwd_engine *engine, char *buffer, size_t size);
/* forward.js:1954 `memoryBytes()`: device bytes this engine holds. */
int b200fwd_memory_bytes(b200fwd_engine *engine, uint64_t *out);
/* forward.js:1915-1934 `release()`. NULL is accepted. */
int b200fwd_destroy(b200fwd_engine *engine);
/* The message of the last failed call on this thread (forward.js throws an Error with it). */
int b200fwd_last_error(char *buffer, size_t size);
/* The ABI version this library was built with (B200FWD_ABI_VERSION). */
int b200fwd_abi_version(void);

/* ---- the batched extension (no counterpart in forward.js, which holds one sequence): `slots` independent
 * sequences with a KV cache each, so that the matmuls of a step read the weights once for all of them. Each
 * (slot, token) computes the numbers forward()/forwardMany() compute for it alone, to the bit. */

/* One run of n tokens: token i belongs to slots[i] at position pos[i]. Tokens of one slot must be consecutive
 * positions in order (a prompt block). Every key and value goes into its slot's cache before any attention (as
 * forward.js run() does, forward.js:1043-1057). Logits of the tokens whose want[i] != 0 go, in order, to `logits`
 * (host, want-count x vocab) if non-NULL, and their first-index argmax (np.argmax) to `argmax` (host) if non-NULL.
 * want may be NULL (no logits). */
int b200fwd_run(b200fwd_engine *engine, int32_t n, const int32_t *slots, const int32_t *tokens, const int32_t *pos,
                const uint8_t *want, float *logits, int32_t *argmax);
/* Greedy decoding on the device: for each of the n slots, `steps` steps starting from token first[i] at
 * position pos0[i]; each step's argmax is the next step's token. out (host, n x steps) gets the sampled ids.
 * The logits never leave the device; one CUDA graph per step. Returns B200FWD_ENOTFINITE where a step's largest
 * logit is not finite (what llama2_numpy.greedy raises, llama2_numpy.py:1521-1527). */
int b200fwd_generate_greedy(b200fwd_engine *engine, int32_t n, const int32_t *slots, const int32_t *first,
                            const int32_t *pos0, int32_t steps, int32_t *out);
/* forward.js:1837-1890 `generateMany(token, pos, history, length, count, temperature, topp, penalty, randoms,
 * stops)`, for n slots at once: from token first[i] at position pos0[i], up to `steps` steps of generate()'s loop
 * (public/llama2_numpy.py:1612-1650) on the device: the forward pass, the repetition penalty over the slot's last
 * B200FWD_REPETITION_WINDOW tokens (kernel.ts:705-719 penalize; none where penalty == 1), then greedy argmax
 * (temperature 0, numpy's argmax) or kernel.ts:808-868 sample with randoms[i * steps + step] (temperature, topp),
 * the id fed back as the next token. recent: [n][B200FWD_REPETITION_WINDOW] the last min(recent_count[i], window)
 * tokens of slot i's history, oldest first; recent_count[i]: the history's length. A slot ends after a stop token
 * (stops: nstops ids, host), which is its last id. out: [n][steps] the ids (host), made[i]: how many of them slot i
 * has. The logits never leave the device; one CUDA graph per step. B200FWD_ENOTFINITE where a step's logits have
 * no finite largest value (llama2_numpy.py:548 NOT_FINITE). */
#define B200FWD_REPETITION_WINDOW 64
int b200fwd_generate_many(b200fwd_engine *engine, int32_t n, const int32_t *slots, const int32_t *first,
                          const int32_t *pos0, int32_t steps, float temperature, float topp, float penalty,
                          const int32_t *recent, const int32_t *recent_count, const double *randoms,
                          const int32_t *stops, int32_t nstops, int32_t *out, int32_t *made);
/* Forget a slot's sequence (its cache is written over from position 0 by the next run). */
int b200fwd_reset_slot(b200fwd_engine *engine, int32_t slot);
/* The stream the engine launches on (a cudaStream_t), for callers that time it with CUDA events. */
int b200fwd_stream_of(b200fwd_engine *engine, b200fwd_stream *out);
/* The number of kernels the engine launched since it was made (counted on the host at every launch). */
int b200fwd_launch_count(b200fwd_engine *engine, uint64_t *out);
/* No counterpart in the reference: a measurement aid. One pass = the int8 matmul of every weight matrix at `count`
 * tokens, as the forward pass launches it (each layer's q|k|v, o, w1|w3, w2, then the classifier), on the engine's
 * current activations, into a buffer of its own (the engine's state is left as it was). Runs one
 * warm-up pass and `reps` timed ones back to back; gives the GPU time of one pass (CUDA events on the engine's
 * stream), its algorithmic bytes (weights + scales + activations read once, outputs written once) and its launches. */
int b200fwd_time_matmuls(b200fwd_engine *engine, int32_t count, int32_t reps, float *ms_per_pass,
                         double *bytes_per_pass, int32_t *launches_per_pass);

/* No counterpart in the reference: a measurement aid. The int8 matmul of each weight-matrix kind at `count` tokens,
 * as the forward pass launches it: [0] q|k|v (qDim + 2 kvDim rows), [1] o (dim rows), [2] w1|w3 (2 hidden rows),
 * [3] w2 (dim rows, n = hidden), [4] the classifier (vocab rows). Each kind runs over every layer's copy in turn (so
 * no launch finds its weights in L2), one warm-up pass then `reps` timed passes, CUDA events on the engine's stream.
 * Gives the average GPU time of one launch of each kind (microseconds) and its algorithmic bytes (weights + scales
 * + activations read once, outputs written once). The engine's state is left as it was. */
int b200fwd_time_matmul_kinds(b200fwd_engine *engine, int32_t count, int32_t reps, float *us_per_launch,
                              double *bytes_per_launch);

/* ---------------------------------------------------------------------------------------------- the kernels
 * Device pointers, a stream, and the reference's arguments. `count` tokens of a prompt (T108) sit `*_stride`
 * elements apart where the reference keeps them a frame apart. Return 0 or B200FWD_E*. */

/* kernel.ts:129-156 quantize_x, for count tokens: x [count][n] (x_stride floats apart) -> xq [count][n] int8
 * (q_stride bytes apart), xs [count][n/32] (s_stride floats apart). bias 0: 8-bit; 64: 7-bit + 64. n % 32 == 0. */
int b200k_quantize_x(int8_t *xq, float *xs, const float *x, int32_t n, int32_t bias, int32_t count,
                     int64_t x_stride, int64_t q_stride, int64_t s_stride, b200fwd_stream stream);
/* kernel.ts:204-212 int8_sums: out[g] = -64 * sum of group g's 32 int8 values. */
int b200k_int8_sums(int32_t *out, const int8_t *w, int64_t groups, b200fwd_stream stream);
/* kernel_relaxed.ts:34-67 matmul_q8r (count == 1) and kernel_relaxed.ts:164-183 matmul_q8r_tile (count > 1):
 * rows r0..r1 of W (int8 [rows][n], scales ws [rows][n/32]) times count tokens' activations of
 * quantize_x(bias 64) (xq, xs: a_stride bytes / a_stride/... see below). wc: the int8_sums corrections, or NULL,
 * in which case each group's integer is taken as dot(w, q - 64) directly (the same integer). Token t's outputs at
 * xout + t * out_stride (floats). xq of token t at xq + t * q_stride (bytes), xs at xs + t * s_stride (floats). */
int b200k_matmul_q8r(float *xout, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws,
                     const int32_t *wc, int32_t n, int32_t r0, int32_t r1, int32_t count, int64_t out_stride,
                     int64_t q_stride, int64_t s_stride, b200fwd_stream stream);
/* kernel_relaxed.ts:34-67 / 164-183 on activations already less the bias (xq[i] = q[i] - 64, signed; the engine
 * keeps them so): all `rows` rows of W for `count` tokens, the same numbers to the bit. The tensor-core path reports
 * a pipeline wait that gave up through one device word of the library's: calls that overlap on the GPU (other
 * streams or threads) share it and must be serialized. From 16 tokens on (with
 * n >= 128, rows >= 128, and ws_stride a multiple of 4 floats: TMA rows of whole 16 bytes) it runs on the tensor
 * cores (tcgen05.mma kind::i8, one MMA per group of 32), else on the CUDA cores. ws: row r's scales at
 * ws + r * ws_stride (0: n / 32). xq, wq, ws 16-byte aligned; q_stride a multiple of 16. */
int b200k_matmul_q8s(float *xout, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws,
                     int64_t ws_stride, int32_t n, int32_t rows, int32_t count, int64_t out_stride, int64_t q_stride,
                     int64_t s_stride, b200fwd_stream stream);
/* No counterpart in the reference: the tensor-core matmul the engine launches for one rows x n matrix of its layers
 * at count tokens (count >= 2) on a GPU of `sms` SMs, with token tiles of at most `widest` (16, 32 or 64): *lane_split
 * 1 for q8_gemm_lanes (a cluster of four CTAs per tile, one per chain lane), 0 for q8_gemm_tc; *tile_tokens the
 * tile's tokens. The choice of least estimated time from measured stage times; host arithmetic only (no device). */
int b200k_matmul_plan(int32_t rows, int32_t n, int32_t count, int32_t sms, int32_t widest, int32_t *lane_split,
                      int32_t *tile_tokens);
/* kernel.ts:231-258 matmul_q8: the same on quantize_x(bias 0) activations, lane order of dot32. */
int b200k_matmul_q8(float *xout, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws, int32_t n,
                    int32_t r0, int32_t r1, int32_t count, int64_t out_stride, int64_t q_stride, int64_t s_stride,
                    b200fwd_stream stream);
/* kernel.ts:330-342 rmsnorm, for count rows `stride` floats apart (out and x alike). */
int b200k_rmsnorm(float *out, const float *x, const float *w, int32_t n, float eps, int32_t count, int64_t stride,
                  b200fwd_stream stream);
/* kernel.ts:344-357 rope: nh heads of hs at v, tables fcr/fci (hs/2 floats each, this position's row). */
int b200k_rope(float *v, const float *fcr, const float *fci, int32_t nh, int32_t hs, int32_t rot,
               b200fwd_stream stream);
/* kernel.ts:365-373 attention / attention_f16: one query token at position pos against a cache laid out
 * [position][nkv*hs] (float32, or float16 bits when half != 0), heads h0..h1; att: scratch of nh*(pos+1) floats
 * (device), which ends up holding the softmax weights as the reference's does. */
int b200k_attention(float *out, const float *q, const void *kc, const void *vc, float *att, int32_t pos, int32_t nh,
                    int32_t nkv, int32_t hs, int32_t h0, int32_t h1, int32_t half, b200fwd_stream stream);
/* No counterpart in the reference. b200k_attention for callers that cannot allocate device memory where they call
 * (inside a stream capture, where cudaMalloc is not allowed; on a latency path that must not stall the device the
 * way cudaMalloc can; under a fixed device budget): the same numbers, with the softmax scratch in a 4 MiB array of
 * the library's own, which every GPU that loads the library holds until exit. nh * (pos + 1) may be at most
 * 1048576 and pos + 1 at most 51200 (else B200FWD_EINVAL). The first call on a device looks the array up, so make it
 * before any capture; the address is kept for the process's life, so do not call it again after a
 * cudaDeviceReset. Every call shares the array: calls that overlap on the GPU race. Nothing needs zeroing; it keeps
 * the last call's softmax weights. */
int b200k_attention_static(float *out, const float *q, const void *kc, const void *vc, int32_t pos, int32_t nh,
                           int32_t nkv, int32_t hs, int32_t h0, int32_t h1, int32_t half, b200fwd_stream stream);
/* kernel.ts:570-599 to_f16 (round to nearest even, NumPy's astype(float16)) and kernel.ts:604-608 from_f16. */
int b200k_to_f16(uint16_t *out, const float *x, int64_t n, b200fwd_stream stream);
int b200k_from_f16(float *out, const uint16_t *x, int64_t n, b200fwd_stream stream);
/* kernel.ts:654-667 swiglu: out = h1 / (1 + exp(-h1)) * h3, n values. */
int b200k_swiglu(float *out, const float *h1, const float *h3, int64_t n, b200fwd_stream stream);
/* kernel.ts:691-693 add_inplace: x += y. */
int b200k_add_inplace(float *x, const float *y, int64_t n, b200fwd_stream stream);
/* kernel.ts:671-689 add_columns: y[j] += sum over c of a[c] * rows[c][j], c in order. */
int b200k_add_columns(float *y, const float *rows, const float *a, int32_t count, int32_t n, b200fwd_stream stream);
/* kernel.ts:705-719 penalize: each of the count tokens (device int32) made less likely once in logits (device):
 * value / penalty where it is above 0, else value * penalty. */
int b200k_penalize(float *logits, const int32_t *tokens, int32_t count, float penalty, b200fwd_stream stream);
/* kernel.ts:808-868 sample: the token drawn from softmax(logits / temperature) over n logits (device), restricted to
 * the nucleus where 0 < topp < 1, with the random number `random` in [0, 1), into *out (device int32): -1 where the
 * largest logit is no finite number, -2 where the nucleus sort's bounded stack ran out. scratch: a device buffer of
 * b200k_sample_scratch(n) bytes (the reference takes two arrays of n; this one also holds the sort's stack). */
int b200k_sample(int32_t *out, const float *logits, int32_t n, float temperature, float topp, double random,
                 void *scratch, b200fwd_stream stream);
int b200k_sample_scratch(int32_t n, uint64_t *bytes);
/* Causal attention of whole prompts on the tensor cores: what public/forward.js:1055-1057 computes one query token
 * at a time (kernel.ts:344-357 rope on the query and the keys, then kernel.ts:447-566 attentionOf over positions
 * 0..t), for every token of `batch` sequences of `seq` tokens at once. q [batch][seq][heads][head_size], k and v
 * [batch][seq][kv_heads][head_size] float32 (before RoPE; device), the RoPE tables fcr, fci [seq][head_size / 2]
 * (device); out [batch][seq][heads][head_size] float32. Float16 operands on the tensor cores with float32
 * accumulation: within 1e-3 of the exact result relative to its largest value (not bit-exact). head_size 64, seq a
 * multiple of 256. scratch: b200k_prefill_attention_scratch() bytes of device memory, 256-byte aligned. */
int b200k_prefill_attention(float *out, const float *q, const float *k, const float *v, const float *fcr,
                            const float *fci, int32_t batch, int32_t seq, int32_t heads, int32_t kv_heads,
                            int32_t head_size, void *scratch, b200fwd_stream stream);
int b200k_prefill_attention_scratch(int32_t batch, int32_t seq, int32_t heads, int32_t kv_heads, int32_t head_size,
                                    uint64_t *bytes);
/* b200k_prefill_attention only enqueues its kernels; this waits for them and gives B200FWD_ETIMEOUT where one of the
 * kernel's bounded pipeline waits gave up (the word it leaves in the scratch), else 0. */
int b200k_prefill_attention_check(const void *scratch, int32_t batch, int32_t seq, int32_t heads, int32_t kv_heads,
                                  int32_t head_size, b200fwd_stream stream);
/* kernel.ts:695-699 argmax (first index of the largest, `>`), into *out (device int32). */
int b200k_argmax(int32_t *out, const float *x, int32_t n, b200fwd_stream stream);

/* ---- batched attention for many sequences at once (configs of the B200 build; no single WASM counterpart):
 * token i (of n) attends to its sequence's cache. Cache of sequence s: K at kc + s * seq_stride elements, the
 * same layout as b200k_attention's ([position][nkv*hs]), V likewise. q [n][nh*hs], out [n][nh*hs].
 * Exact: every output is the number b200k_attention computes for that token alone, to the bit.
 * att: device scratch of n * nh * scratch_positions floats (scratch_positions >= max pos + 1). */
int b200k_attention_batch(float *out, const float *q, const void *kc, const void *vc, float *att,
                          const int32_t *seq, const int32_t *pos, int32_t n, int64_t seq_stride,
                          int32_t scratch_positions, int32_t nh, int32_t nkv, int32_t hs, int32_t half,
                          b200fwd_stream stream);

#ifdef __cplusplus
}
#endif

#endif /* B200FWD_H */
