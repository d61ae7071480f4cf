// engine.cu — the forward engine of include/b200fwd.h: what public/forward.js createForward() is to
// llama2_numpy.Llama(external=...), on one B200.
//
// HBM layout:
//  - each int8 matrix in its own 256-byte-aligned block: values [layers][rows][n], then scales [layers][rows][n/32]
//    (the checkpoint's order, moved off the file's unaligned offsets so that rows load as 16-byte vectors);
//  - the norm weights and the RoPE tables as float32;
//  - the KV cache of every slot: [slot][layer][keys|values][capacity][kvDim] in float16 or float32, the layout of
//    forward.js:269-273 per slot, its capacity doubled as forward.js grow() does (forward.js:274-289);
//  - the activations of up to max_tokens tokens, one row each (forward.js keeps them a frame apart, :192-208).
// run() is forward.js run() (forward.js:452-531) over tokens that may belong to different slots.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <initializer_list>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "common.h"
#include "gemm_tc.h"
#include "kernels.h"

namespace b200 {

std::atomic<uint64_t> launches{0};

std::string &last_error() {
  thread_local std::string message;
  return message;
}

int fail(int code, const std::string &message) {
  last_error() = message;
  return code;
}

int cuda_fail(cudaError_t e, const char *what) {
  return fail(e == cudaErrorMemoryAllocation ? B200FWD_ENOMEM : B200FWD_ECUDA,
              std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}

bool pdl_on() {
  static const bool on = [] {
    const char *v = std::getenv("B200FWD_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

namespace {

// an int8 matrix of every layer (rows x n each): values, and scales in rows of sstride floats (the row's n/32
// groups, padded to a multiple of four so that a TMA row is whole 16 bytes); its TMA maps over all layers' rows
struct Matrix {
  int8_t *w = nullptr;
  float *s = nullptr;
  int rows = 0, n = 0, layers = 1, sstride = 0;
  bool mapped = false, lane_mapped = false;
  CUtensorMap wmap, smap;
  CUtensorMap lwmap, lsmap;  // the lane-split matmul's (gemm_lanes.cu)
  const int8_t *layer_w(int l) const { return w + (int64_t)l * rows * n; }
  const float *layer_s(int l) const { return s + (int64_t)l * rows * sstride; }
};

inline int padded_groups(int n) { return ((n / 32 + 3) / 4) * 4; }

// kernel.ts:383-392 half on the host, for keysAndValues
float half_bits_to_float(uint16_t h) {
  const int32_t v = (int32_t)(int16_t)h;
  uint32_t u = (uint32_t)((v << 13) & (int32_t)0x8fffffff);
  float f;
  std::memcpy(&f, &u, 4);
  return f * 5.192296858534828e33f;
}

}  // namespace
}  // namespace b200

using namespace b200;

struct b200fwd_engine {
  int device = 0;
  cudaStream_t stream = nullptr;
  b200fwd_plan plan{};
  int dim, hidden, layers, heads, kvHeads, hs, vocab, seqLen, kvDim, qDim, XQ;
  bool relaxed, half;
  int bias;
  float eps;
  // q, k and v of a layer as one matrix of qDim + 2 kvDim rows, w1 and w3 as one of 2 hidden rows (forward.js puts
  // each set in one phase: forward.js:476,516)
  Matrix emb, wqkv, wo, w13, w2, wcls;
  float *attW = nullptr, *ffnW = nullptr, *finalW = nullptr, *cosT = nullptr, *sinT = nullptr;
  int nch = 0;
  int32_t *channels = nullptr;
  float *columns = nullptr;
  // the cache
  int slots = 1, capacity = 0;
  uint8_t *cache = nullptr;
  // activations
  int T = 0;
  int TP = 0;  // T rounded up to 32: the activation scales are [XQ/32 groups][TP tokens]
  int QKV = 0;
  float *x = nullptr, *xb = nullptr, *qkv = nullptr, *h13 = nullptr;
  float *att = nullptr;
  int8_t *xq = nullptr;
  float *xs = nullptr;
  float *xl = nullptr, *picked = nullptr, *logits = nullptr;
  int logit_rows = 0;
  int32_t *argmax = nullptr;
  int32_t *meta = nullptr;      // device: tokens[T], seq[T], pos[T], want[T], step, bad, tc error, -, tiles[2T]
  CUtensorMap xmap[3], xsmap[3]; // the activations and their scales, for tiles of 16, 32 and 64 tokens
  int widest_tile = 0;           // the widest of those tiles the activations have room for
  CUtensorMap lxmap[3], lxsmap[3];  // the same for the lane-split matmul
  bool lanes = false;
  bool tensor_cores = true;
  int sms = 148;
  int32_t *meta_h = nullptr;    // pinned host copy
  int32_t *history = nullptr;   // greedy ids [slots][steps]
  int history_len = 0;
  // generate_many's device state: one block of int32 words and one of doubles / floats, grown as needed
  int32_t *gm_words = nullptr;
  size_t gm_words_len = 0;
  double *gm_randoms = nullptr;
  size_t gm_randoms_len = 0;
  float *gm_scratch = nullptr;
  size_t gm_scratch_len = 0;
  float *bound = nullptr;       // Python's logits array (host)
  std::vector<float> last_logits;
  uint64_t bytes = 0;
  std::vector<void *> allocations;
  uint64_t launches_at_create = 0;
  std::string backend;

  int32_t *tokens_d() { return meta; }
  int32_t *seq_d() { return meta + T; }
  int32_t *pos_d() { return meta + 2 * T; }
  int32_t *want_d() { return meta + 3 * T; }
  int32_t *step_d() { return meta + 4 * T; }
  int32_t *bad_d() { return meta + 4 * T + 1; }
  int32_t *tc_error_d() { return meta + 4 * T + 2; }
  int32_t *tiles_d() { return meta + 4 * T + 4; }
  int esize() const { return half ? 2 : 4; }
  int64_t seq_stride() const { return (int64_t)layers * 2 * capacity * kvDim; }
  uint8_t *layer_keys(int l) { return cache + (int64_t)(l * 2) * capacity * kvDim * esize(); }
  uint8_t *layer_values(int l) { return cache + (int64_t)(l * 2 + 1) * capacity * kvDim * esize(); }
};

namespace {

int alloc(b200fwd_engine *e, void **p, size_t bytes) {
  if (bytes == 0) bytes = 16;
  cudaError_t err = cudaMalloc(p, bytes);
  if (err != cudaSuccess) return cuda_fail(err, "cudaMalloc");
  e->allocations.push_back(*p);
  e->bytes += bytes;
  return 0;
}

void release(b200fwd_engine *e, void *p, size_t bytes) {
  if (!p) return;
  cudaFree(p);
  auto it = std::find(e->allocations.begin(), e->allocations.end(), p);
  if (it != e->allocations.end()) e->allocations.erase(it);
  e->bytes -= bytes;
}

#define CHECK(expr)              \
  do {                           \
    int rc_ = (expr);            \
    if (rc_) return rc_;         \
  } while (0)

int64_t elements(const b200fwd_tensor &t) {
  int64_t c = 1;
  for (int i = 0; i < t.ndim; i++) c *= t.shape[i];
  return c;
}

cudaMemcpyKind copy_kind(bool on_device) { return on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice; }

int upload_matrix(b200fwd_engine *e, const uint8_t *ckpt, size_t size, bool on_device, const b200fwd_tensor &t,
                  const char *name, Matrix &m) {
  if (t.kind != B200FWD_TENSOR_INT8)
    return fail(B200FWD_EUNSUPPORTED, std::string("tensor ") + name + " is not int8 (this engine runs int8 only)");
  if (t.ndim < 2 || t.ndim > 3) return fail(B200FWD_EINVAL, std::string("tensor ") + name + " has a bad shape");
  m.rows = (int)t.shape[t.ndim - 2];
  m.n = (int)t.shape[t.ndim - 1];
  m.layers = t.ndim == 3 ? (int)t.shape[0] : 1;
  if (t.group != 32 || m.n % 32)
    return fail(B200FWD_EUNSUPPORTED, std::string("tensor ") + name + ": the int8 kernels take groups of 32");
  const int64_t count = elements(t);
  if (t.offset < 0 || t.scales < 0 || (size_t)(t.offset + count) > size || (size_t)(t.scales + count / 8) > size)
    return fail(B200FWD_EINVAL, std::string("tensor ") + name + " lies outside the checkpoint");
  m.sstride = padded_groups(m.n);
  const int64_t rows_all = count / m.n;
  CHECK(alloc(e, (void **)&m.w, count));
  CHECK(alloc(e, (void **)&m.s, rows_all * m.sstride * 4));
  B200_CUDA(cudaMemsetAsync(m.s, 0, rows_all * m.sstride * 4, e->stream));
  B200_CUDA(cudaMemcpyAsync(m.w, ckpt + t.offset, count, copy_kind(on_device), e->stream));
  B200_CUDA(cudaMemcpy2DAsync(m.s, (size_t)m.sstride * 4, ckpt + t.scales, (size_t)(m.n / 32) * 4,
                              (size_t)(m.n / 32) * 4, rows_all, copy_kind(on_device), e->stream));
  return 0;
}

// several tensors of the same layers and row length as one matrix per layer, their rows one after another
int upload_fused(b200fwd_engine *e, const uint8_t *ckpt, size_t size, bool on_device,
                 std::initializer_list<std::pair<const b200fwd_tensor *, const char *>> parts, Matrix &m) {
  m = Matrix();
  int n = -1, layers = -1, rows = 0;
  for (auto &pt : parts) {
    const b200fwd_tensor &t = *pt.first;
    if (t.kind != B200FWD_TENSOR_INT8)
      return fail(B200FWD_EUNSUPPORTED, std::string("tensor ") + pt.second + " is not int8 (this engine runs int8 only)");
    if (t.ndim != 3 || t.group != 32 || t.shape[2] % 32)
      return fail(B200FWD_EUNSUPPORTED, std::string("tensor ") + pt.second + ": layers of rows of whole groups of 32");
    if (n >= 0 && (t.shape[2] != n || t.shape[0] != layers))
      return fail(B200FWD_EINVAL, std::string("tensor ") + pt.second + " does not match the others of its phase");
    n = (int)t.shape[2];
    layers = (int)t.shape[0];
    const int64_t count = elements(t);
    if (t.offset < 0 || t.scales < 0 || (size_t)(t.offset + count) > size || (size_t)(t.scales + count / 8) > size)
      return fail(B200FWD_EINVAL, std::string("tensor ") + pt.second + " lies outside the checkpoint");
    rows += (int)t.shape[1];
  }
  m.rows = rows;
  m.n = n;
  m.layers = layers;
  m.sstride = padded_groups(n);
  const int64_t count = (int64_t)layers * rows * n;
  const int ng = n / 32;
  CHECK(alloc(e, (void **)&m.w, count));
  CHECK(alloc(e, (void **)&m.s, (int64_t)layers * rows * m.sstride * 4));
  B200_CUDA(cudaMemsetAsync(m.s, 0, (int64_t)layers * rows * m.sstride * 4, e->stream));
  int at = 0;
  for (auto &pt : parts) {
    const b200fwd_tensor &t = *pt.first;
    const int r = (int)t.shape[1];
    B200_CUDA(cudaMemcpy2DAsync(m.w + (int64_t)at * n, (size_t)rows * n, ckpt + t.offset, (size_t)r * n, (size_t)r * n,
                                layers, copy_kind(on_device), e->stream));
    for (int l = 0; l < layers; l++)
      B200_CUDA(cudaMemcpy2DAsync(m.s + ((int64_t)l * rows + at) * m.sstride, (size_t)m.sstride * 4,
                                  ckpt + t.scales + (int64_t)l * r * ng * 4, (size_t)ng * 4, (size_t)ng * 4, r,
                                  copy_kind(on_device), e->stream));
    at += r;
  }
  return 0;
}

int upload_floats(b200fwd_engine *e, const uint8_t *ckpt, size_t size, bool on_device, const b200fwd_tensor &t,
                  const char *name, int64_t want, float **out) {
  if (t.kind != B200FWD_TENSOR_F32)
    return fail(B200FWD_EUNSUPPORTED, std::string("tensor ") + name + " is not float32");
  const int64_t count = elements(t);
  if (count != want) return fail(B200FWD_EINVAL, std::string("tensor ") + name + " has the wrong size");
  if (t.offset < 0 || (size_t)(t.offset + 4 * count) > size)
    return fail(B200FWD_EINVAL, std::string("tensor ") + name + " lies outside the checkpoint");
  CHECK(alloc(e, (void **)out, count * 4));
  B200_CUDA(cudaMemcpyAsync(*out, ckpt + t.offset, count * 4, copy_kind(on_device), e->stream));
  return 0;
}

// the activations and scratch of T tokens against a cache of `capacity` positions
int alloc_activations(b200fwd_engine *e) {
  const int T = e->T;
  CHECK(alloc(e, (void **)&e->x, (size_t)T * e->dim * 4));
  CHECK(alloc(e, (void **)&e->xb, (size_t)T * e->qDim * 4));
  CHECK(alloc(e, (void **)&e->qkv, (size_t)T * e->QKV * 4));
  CHECK(alloc(e, (void **)&e->h13, (size_t)T * 2 * e->hidden * 4));
  CHECK(alloc(e, (void **)&e->xq, (size_t)T * e->XQ));
  CHECK(alloc(e, (void **)&e->xs, (size_t)e->TP * (e->XQ / 32) * 4));
  CHECK(alloc(e, (void **)&e->xl, (size_t)T * e->dim * 4));
  CHECK(alloc(e, (void **)&e->picked, (size_t)T * std::max(1, e->nch) * 4));
  CHECK(alloc(e, (void **)&e->argmax, (size_t)T * 4));
  CHECK(alloc(e, (void **)&e->meta, (size_t)(6 * T + 4) * 4));
  B200_CUDA(cudaMemsetAsync(e->meta, 0, (size_t)(6 * T + 4) * 4, e->stream));
  B200_CUDA(cudaMallocHost((void **)&e->meta_h, (size_t)(6 * T + 4) * 4));
  // the activations' TMA maps (rows of XQ bytes, one per token) and their scales' (rows of TP floats, one per group),
  // for tiles of 16, 32 and 64 tokens (as many as T holds)
  e->tensor_cores = e->tensor_cores && T >= 32 && e->XQ >= 128;
  if (e->tensor_cores)
    for (int i = 0, bn = 16; i < 3 && bn <= T; i++, bn *= 2) {
      CHECK(make_i8_map(&e->xmap[i], e->xq, e->XQ, T, e->XQ, bn));
      CHECK(make_token_scale_map(&e->xsmap[i], e->xs, T, e->XQ / 32, e->TP, bn));
      e->widest_tile = bn;
    }
  e->lanes = e->tensor_cores && e->widest_tile == 64 && e->XQ % 128 == 0 && e->XQ >= 2048 && gemm_lanes_enabled();
  if (e->lanes) {
    for (int i = 0, bn = 16; i < 3; i++, bn *= 2)
      CHECK(make_lane_token_maps(&e->lxmap[i], &e->lxsmap[i], e->xq, e->xs, T, e->XQ, e->XQ, e->TP, bn));
    CHECK(prepare_gemm_lanes());
  }
  return 0;
}

int ensure_logit_rows(b200fwd_engine *e, int rows) {
  if (rows <= e->logit_rows) return 0;
  B200_CUDA(cudaStreamSynchronize(e->stream));
  release(e, e->logits, (size_t)e->logit_rows * e->vocab * 4);
  e->logits = nullptr;
  const int want = std::max(rows, std::min(e->T, e->slots));
  CHECK(alloc(e, (void **)&e->logits, (size_t)want * e->vocab * 4));
  e->logit_rows = want;
  return 0;
}

// forward.js:274-289 grow: the capacity doubled (at least to pos + 1, at most seq_len), every slot's keys and values
// copied to the larger blocks (their values do not change)
int grow(b200fwd_engine *e, int pos) {
  const int larger = std::min(std::max(2 * e->capacity, pos + 1), e->seqLen);
  if (larger <= e->capacity) return 0;
  const size_t old_block = (size_t)e->capacity * e->kvDim * e->esize();
  const size_t new_block = (size_t)larger * e->kvDim * e->esize();
  const size_t blocks = (size_t)e->slots * e->layers * 2;
  uint8_t *cache = nullptr;
  CHECK(alloc(e, (void **)&cache, blocks * new_block));
  if (e->cache && e->capacity > 0)
    B200_CUDA(cudaMemcpy2DAsync(cache, new_block, e->cache, old_block, old_block, blocks, cudaMemcpyDeviceToDevice,
                                e->stream));
  B200_CUDA(cudaStreamSynchronize(e->stream));
  release(e, e->cache, blocks * old_block);
  release(e, e->att, (size_t)e->T * e->heads * e->capacity * 4);
  e->cache = cache;
  e->capacity = larger;
  e->att = nullptr;
  CHECK(alloc(e, (void **)&e->att, (size_t)e->T * e->heads * e->capacity * 4));
  return 0;
}

// one matrix of one layer times the quantized activations of count tokens (in e->xq, less the bias): the tensor
// cores from TC_MIN_TOKENS tokens on (gemm_tc.cu; a tile of 16 token columns whose columns past count read rows of the
// activation buffer that no output uses), the CUDA cores for one token (kernels.cu); the same numbers either way
constexpr int TC_MIN_TOKENS = 2;
int matmul(b200fwd_engine *e, const Matrix &m, int layer, float *out, int64_t out_stride, int accumulate, int count) {
  // (the TMA boxes are 128 bytes of K by 128 weight rows and by up to 64 tokens: never past the tensors' extents)
  if (count >= TC_MIN_TOKENS && e->relaxed && e->tensor_cores && m.mapped) {
    GemmArgs a{};
    a.out = out;
    a.error = e->tc_error_d();
    a.n = m.n;
    a.rows = m.rows;
    a.count = count;
    a.w_row0 = layer * m.rows;
    a.out_stride = out_stride;
    a.accumulate = accumulate;
    if (e->lanes && m.lane_mapped && gemm_lanes_fits(m.n, m.rows, count) &&
        gemm_lanes_pays(m.rows, count, m.n, e->sms, e->widest_tile)) {
      const int bn = choose_lanes_bn(count, 64);
      const int which = bn == 16 ? 0 : bn == 32 ? 1 : 2;
      GemmMaps maps{m.lwmap, e->lxmap[which], m.lsmap, e->lxsmap[which]};
      return launch_gemm_lanes(maps, a, bn, e->stream);
    }
    const int bn = choose_gemm_bn(m.rows, count, e->sms, e->widest_tile);
    const int which = bn == 16 ? 0 : bn == 32 ? 1 : 2;
    GemmMaps maps{m.wmap, e->xmap[which], m.smap, e->xsmap[which]};
    return launch_gemm_tc(maps, a, bn, e->stream);
  }
  MatJobs jobs{};
  jobs.job[0] = {m.layer_w(layer), m.layer_s(layer), nullptr, out, m.rows, accumulate, out_stride, m.sstride};
  jobs.njobs = 1;
  jobs.n = m.n;
  jobs.total_rows = m.rows;
  jobs.signed_input = 1;
  return launch_matvec(jobs, e->xq, e->xs, e->XQ, 1, e->TP, count, e->relaxed, e->stream);
}

// the layers over n tokens whose ids, slots and positions are in meta (device); the logits of the `want` tokens
// (their indices in want_d) into logits rows 0..want-1, and their argmax. ntiles > 0: the attention's token tiles
// are in tiles_d; 0: every token its own. Enqueues only (graph-capturable).
int forward_device(b200fwd_engine *e, int n, int want, int max_count, int ntiles, bool argmax = true) {
  cudaStream_t st = e->stream;
  const int D = e->dim, QD = e->qDim, KVD = e->kvDim, HID = e->hidden, XQ = e->XQ, TP = e->TP, QKV = e->QKV;
  const int shift = e->bias;  // activations stored less the bias
  float *q = e->qkv, *k = e->qkv + QD, *v = e->qkv + QD + KVD;
  CHECK(launch_embed(e->emb.w, e->emb.s, e->emb.sstride, e->tokens_d(), n, D, e->x, D, st));
  for (int l = 0; l < e->layers; l++) {
    CHECK(launch_norm_quantize(e->x, D, e->attW + (int64_t)l * D, D, e->eps, e->bias, n, e->xq, XQ, e->xs, 1, TP,
                               nullptr, 0, nullptr, nullptr, 0, st, shift));
    CHECK(matmul(e, e->wqkv, l, e->qkv, QKV, 0, n));
    CHECK(launch_rope_cache(q, QKV, k, v, QKV, e->cosT, e->sinT, e->pos_d(), e->seq_d(), n, e->layer_keys(l),
                            e->layer_values(l), e->seq_stride(), e->half ? 1 : 0, e->heads, e->kvHeads, e->hs,
                            e->plan.rotary, st));
    // the attention kernels quantize their rows themselves where they can (single tokens); else quantize_x after
    AttentionQuant aq{e->xq, XQ, e->xs, 1, TP, e->bias, shift, 0};
    CHECK(launch_attention(e->xb, QD, q, QKV, e->layer_keys(l), e->layer_values(l), e->att, e->seq_d(), e->pos_d(), 0,
                           ntiles ? e->tiles_d() : nullptr, ntiles, n, e->seq_stride(), e->capacity, max_count,
                           e->heads, e->kvHeads, e->hs, 0, e->heads, e->half ? 1 : 0, st, &aq));
    if (!aq.done) CHECK(launch_quantize(e->xb, QD, QD, e->bias, n, e->xq, XQ, e->xs, 1, TP, st, shift));
    CHECK(matmul(e, e->wo, l, e->x, D, 1, n));
    CHECK(launch_norm_quantize(e->x, D, e->ffnW + (int64_t)l * D, D, e->eps, e->bias, n, e->xq, XQ, e->xs, 1, TP,
                               nullptr, 0, nullptr, nullptr, 0, st, shift));
    CHECK(matmul(e, e->w13, l, e->h13, 2 * HID, 0, n));
    CHECK(launch_swiglu_quantize(e->h13, e->h13 + HID, 2 * HID, HID, e->bias, n, e->xq, XQ, e->xs, 1, TP, st, shift));
    CHECK(matmul(e, e->w2, l, e->x, D, 1, n));
  }
  if (want <= 0) return 0;
  // forward.js:521-530: the final norm of the wanted tokens, the outlier channels apart, the classifier, the columns
  CHECK(launch_gather_rows(e->xl, D, e->x, D, e->want_d(), want, D, st));
  CHECK(launch_norm_quantize(e->xl, D, e->finalW, D, e->eps, e->bias, want, e->xq, XQ, e->xs, 1, TP, e->channels, e->nch,
                             e->picked, nullptr, 0, st, shift));
  CHECK(matmul(e, e->wcls, 0, e->logits, e->vocab, 0, want));
  CHECK(launch_add_columns(e->logits, e->vocab, e->columns, e->picked, e->nch, e->nch, e->vocab, want, st));
  if (argmax) CHECK(launch_argmax(e->argmax, e->logits, e->vocab, e->vocab, want, 1, st));
  return 0;
}

// after a run: a tensor-core wait that gave up (it would leave the numbers unfinished) is an error
int check_tc(b200fwd_engine *e) {
  int32_t err = 0;
  B200_CUDA(cudaMemcpy(&err, e->tc_error_d(), 4, cudaMemcpyDeviceToHost));
  if (err) {
    B200_CUDA(cudaMemset(e->tc_error_d(), 0, 4));
    return fail(B200FWD_ETIMEOUT, "a tensor-core pipeline wait gave up (code " + std::to_string(err) + ")");
  }
  return 0;
}

int run(b200fwd_engine *e, int n, const int32_t *slots, const int32_t *tokens, const int32_t *pos,
        const uint8_t *want, float *logits_out, int32_t *argmax_out) {
  if (n < 1 || n > e->T) return fail(B200FWD_EINVAL, "run: " + std::to_string(n) + " tokens, at most " + std::to_string(e->T));
  int maxpos = 0, W = 0;
  for (int i = 0; i < n; i++) {
    const int s = slots ? slots[i] : 0;
    if (s < 0 || s >= e->slots) return fail(B200FWD_EINVAL, "run: slot " + std::to_string(s) + " out of range");
    if (tokens[i] < 0 || tokens[i] >= e->vocab)
      return fail(B200FWD_EINVAL, "run: token " + std::to_string(tokens[i]) + " outside the vocabulary");
    if (pos[i] < 0 || pos[i] >= e->seqLen)
      return fail(B200FWD_EINVAL, "run: position " + std::to_string(pos[i]) + " outside the context of " +
                                      std::to_string(e->seqLen));
    for (int j = 0; j < i; j++) {
      const int sj = slots ? slots[j] : 0;
      if (sj == s && pos[j] >= pos[i])
        return fail(B200FWD_EINVAL, "run: the tokens of a slot must come in order of their positions");
    }
    maxpos = std::max(maxpos, pos[i]);
    if (want && want[i]) W++;
  }
  if (maxpos >= e->capacity) CHECK(grow(e, maxpos));
  if (W) CHECK(ensure_logit_rows(e, W));
  const int T = e->T;
  int32_t *m = e->meta_h;
  B200_CUDA(cudaStreamSynchronize(e->stream));  // meta_h is free again
  for (int i = 0; i < n; i++) {
    m[i] = tokens[i];
    m[T + i] = slots ? slots[i] : 0;
    m[2 * T + i] = pos[i];
  }
  for (int i = 0, w = 0; i < n; i++)
    if (want && want[i]) m[3 * T + w++] = i;
  // the attention's tiles: runs of up to ATTN_TILE tokens of one slot at consecutive positions
  int ntiles = 0;
  for (int i = 0; i < n;) {
    int j = i + 1;
    const int si = slots ? slots[i] : 0;
    while (j < n && j - i < ATTN_TILE && (slots ? slots[j] : 0) == si && pos[j] == pos[j - 1] + 1) j++;
    m[4 * T + 4 + 2 * ntiles] = i;
    m[4 * T + 4 + 2 * ntiles + 1] = j - i;
    ntiles++;
    i = j;
  }
  B200_CUDA(cudaMemcpyAsync(e->meta, m, (size_t)(4 * T) * 4, cudaMemcpyHostToDevice, e->stream));
  B200_CUDA(cudaMemcpyAsync(e->tiles_d(), m + 4 * T + 4, (size_t)(2 * ntiles) * 4, cudaMemcpyHostToDevice, e->stream));
  CHECK(forward_device(e, n, W, maxpos + 1, ntiles));
  if (W) {
    if (logits_out)
      B200_CUDA(cudaMemcpyAsync(logits_out, e->logits, (size_t)W * e->vocab * 4, cudaMemcpyDeviceToHost, e->stream));
    if (argmax_out) B200_CUDA(cudaMemcpyAsync(argmax_out, e->argmax, (size_t)W * 4, cudaMemcpyDeviceToHost, e->stream));
  }
  B200_CUDA(cudaStreamSynchronize(e->stream));
  return check_tc(e);
}

int make_engine(const void *checkpoint, size_t size, const b200fwd_plan *plan, const b200fwd_options *options,
                b200fwd_engine *e) {
  const b200fwd_plan &p = *plan;
  b200fwd_options opt{};
  opt.half_keys = -1;
  opt.slots = 1;
  if (options) opt = *options;
  if (opt.slots < 1) opt.slots = 1;
  e->plan = p;
  e->plan.freq_cis_real = e->plan.freq_cis_imag = nullptr;
  e->dim = p.dim; e->hidden = p.hidden_dim; e->layers = p.n_layers; e->heads = p.n_heads; e->kvHeads = p.n_kv_heads;
  e->hs = p.head_size; e->vocab = p.vocab_size; e->seqLen = p.seq_len;
  if (e->dim <= 0 || e->hidden <= 0 || e->layers <= 0 || e->heads <= 0 || e->kvHeads <= 0 || e->hs <= 0 ||
      e->vocab <= 0 || e->seqLen <= 0)
    return fail(B200FWD_EINVAL, "the plan's sizes must be positive");
  if (e->heads % e->kvHeads) return fail(B200FWD_EINVAL, "n_heads must be a multiple of n_kv_heads");
  if (e->hs % 2) return fail(B200FWD_EINVAL, "head_size must be even");
  e->kvDim = e->kvHeads * e->hs;
  e->qDim = e->heads * e->hs;
  if (!p.int8) return fail(B200FWD_EUNSUPPORTED, "the plan does not run on the int8 kernels (plan.int8 is false)");
  if (e->dim % 32 || e->qDim % 32 || e->kvDim % 32 || e->hidden % 32)
    return fail(B200FWD_EUNSUPPORTED, "the int8 kernels take rows of whole groups of 32");
  if (p.n_outliers < 0 || p.n_outliers > B200FWD_MAX_OUTLIERS) return fail(B200FWD_EINVAL, "bad outlier count");
  if (!p.freq_cis_real || !p.freq_cis_imag) return fail(B200FWD_EINVAL, "the plan has no RoPE tables");
  // the activation rows: the widest input, rounded up to 128 bytes (whole TMA boxes; scale rows of whole 16 bytes)
  e->XQ = (std::max(std::max(e->dim, e->hidden), e->qDim) + 127) / 128 * 128;
  e->QKV = e->qDim + 2 * e->kvDim;
  e->relaxed = p.relaxed != 0;
  e->bias = e->relaxed ? 64 : 0;
  e->eps = p.rms_norm_eps;
  // forward.js:203: float16 keys and values where the plan allows it and halfKeys (default: every head has keys of
  // its own) says so. (forward.js also asks for a shared memory, which every multi-threaded page has.)
  const bool halfKeys = opt.half_keys < 0 ? (e->kvHeads >= e->heads) : opt.half_keys != 0;
  e->half = p.half_kv && halfKeys;
  e->slots = opt.slots;
  e->T = opt.max_tokens > 0 ? opt.max_tokens : std::max(512, 16 * e->slots);
  if (e->T > 65535) return fail(B200FWD_EINVAL, "max_tokens above 65535");
  e->TP = (e->T + 31) / 32 * 32;
  e->device = opt.device;
  B200_CUDA(cudaSetDevice(e->device));
  B200_CUDA(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
  CHECK(prepare_attention());
  CHECK(prepare_gemm());
  e->sms = gemm_sms();
  if (e->sms <= 0) return fail(B200FWD_ECUDA, "no SM count");
  const uint8_t *ck = (const uint8_t *)checkpoint;
  const bool dev = opt.checkpoint_on_device != 0;
  CHECK(upload_matrix(e, ck, size, dev, p.token_embedding_table, "token_embedding_table", e->emb));
  if (p.wq.shape[1] != e->qDim || p.wk.shape[1] != e->kvDim || p.wv.shape[1] != e->kvDim ||
      p.w1.shape[1] != e->hidden || p.w3.shape[1] != e->hidden || p.wo.shape[2] != e->qDim ||
      p.w2.shape[2] != e->hidden)
    return fail(B200FWD_EINVAL, "a layer matrix's shape does not match the plan's sizes");
  CHECK(upload_fused(e, ck, size, dev, {{&p.wq, "wq"}, {&p.wk, "wk"}, {&p.wv, "wv"}}, e->wqkv));
  CHECK(upload_fused(e, ck, size, dev, {{&p.wo, "wo"}}, e->wo));
  CHECK(upload_fused(e, ck, size, dev, {{&p.w1, "w1"}, {&p.w3, "w3"}}, e->w13));
  CHECK(upload_fused(e, ck, size, dev, {{&p.w2, "w2"}}, e->w2));
  if (p.shared_classifier)
    e->wcls = e->emb;
  else
    CHECK(upload_matrix(e, ck, size, dev, p.wcls, "wcls", e->wcls));
  const Matrix *shapes[] = {&e->wqkv, &e->wo, &e->w13, &e->w2};
  const int want_rows[] = {e->qDim + 2 * e->kvDim, e->dim, 2 * e->hidden, e->dim};
  const int want_n[] = {e->dim, e->qDim, e->dim, e->hidden};
  for (int i = 0; i < 4; i++)
    if (shapes[i]->rows != want_rows[i] || shapes[i]->n != want_n[i] || shapes[i]->layers != e->layers)
      return fail(B200FWD_EINVAL, "a layer matrix's shape does not match the plan's sizes");
  Matrix *maps[] = {&e->wqkv, &e->wo, &e->w13, &e->w2, &e->wcls};
  for (Matrix *m : maps)
    if (m->n >= 128 && (int64_t)m->layers * m->rows >= 128) {
      CHECK(make_i8_map(&m->wmap, m->w, m->n, (int64_t)m->layers * m->rows, m->n, 128));
      CHECK(make_scale_map(&m->smap, m->s, m->sstride, (int64_t)m->layers * m->rows, m->sstride, 128));
      m->mapped = true;
      if (gemm_lanes_enabled() && gemm_lanes_fits(m->n, (int)std::min<int64_t>((int64_t)m->layers * m->rows, 1 << 30), 1)) {
        CHECK(make_lane_weight_maps(&m->lwmap, &m->lsmap, m->w, m->s, m->n, (int64_t)m->layers * m->rows,
                                    m->sstride));
        m->lane_mapped = true;
      }
    }

  if (e->emb.rows != e->vocab || e->emb.n != e->dim || e->wcls.rows != e->vocab || e->wcls.n != e->dim)
    return fail(B200FWD_EINVAL, "the embedding or classifier does not match the plan's sizes");
  CHECK(upload_floats(e, ck, size, dev, p.rms_att_weight, "rms_att_weight", (int64_t)e->layers * e->dim, &e->attW));
  CHECK(upload_floats(e, ck, size, dev, p.rms_ffn_weight, "rms_ffn_weight", (int64_t)e->layers * e->dim, &e->ffnW));
  CHECK(upload_floats(e, ck, size, dev, p.rms_final_weight, "rms_final_weight", e->dim, &e->finalW));
  const size_t table = (size_t)e->seqLen * (e->hs / 2) * 4;
  CHECK(alloc(e, (void **)&e->cosT, table));
  CHECK(alloc(e, (void **)&e->sinT, table));
  B200_CUDA(cudaMemcpyAsync(e->cosT, p.freq_cis_real, table, cudaMemcpyHostToDevice, e->stream));
  B200_CUDA(cudaMemcpyAsync(e->sinT, p.freq_cis_imag, table, cudaMemcpyHostToDevice, e->stream));
  e->nch = p.n_outliers;
  for (int i = 0; i < e->nch; i++)
    if (p.outliers[i] < 0 || p.outliers[i] >= e->dim) return fail(B200FWD_EINVAL, "an outlier channel past dim");
  CHECK(alloc(e, (void **)&e->channels, sizeof(int32_t) * std::max(1, e->nch)));
  CHECK(alloc(e, (void **)&e->columns, (size_t)std::max(1, e->nch) * e->vocab * 4));
  if (e->nch) {
    B200_CUDA(cudaMemcpyAsync(e->channels, p.outliers, sizeof(int32_t) * e->nch, cudaMemcpyHostToDevice, e->stream));
    CHECK(launch_outlier_columns(e->columns, e->wcls.w, e->wcls.s, e->wcls.sstride, e->dim, e->vocab, e->channels,
                                 e->nch, e->stream));
  }
  CHECK(alloc_activations(e));
  // forward.js:272-273: the cache from kv_start positions (or the caller's first capacity)
  const int first = opt.capacity > 0 ? opt.capacity : p.kv_start;
  e->capacity = 0;
  CHECK(grow(e, std::max(1, std::min(first, e->seqLen)) - 1));
  B200_CUDA(cudaStreamSynchronize(e->stream));
  e->backend = std::string("B200 CUDA kernels (sm_100a), int8, ") +
               (e->relaxed ? "7-bit activations (relaxed)" : "8-bit activations") + ", " +
               (e->half ? "float16" : "float32") + " keys and values, exact float order" +
               (e->slots > 1 ? ", " + std::to_string(e->slots) + " slots" : "");
  e->launches_at_create = launches.load();
  return 0;
}

void destroy(b200fwd_engine *e) {
  if (!e) return;
  cudaSetDevice(e->device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  for (void *p : e->allocations) cudaFree(p);
  if (e->meta_h) cudaFreeHost(e->meta_h);
  if (e->stream) cudaStreamDestroy(e->stream);
  delete e;
}

template <typename F>
int guarded(F &&f) {
  try {
    return f();
  } catch (const std::exception &ex) {
    return fail(B200FWD_EINVAL, std::string("exception: ") + ex.what());
  } catch (...) {
    return fail(B200FWD_EINVAL, "unknown exception");
  }
}

int set_device(b200fwd_engine *e) {
  if (!e) return fail(B200FWD_EINVAL, "no engine");
  B200_CUDA(cudaSetDevice(e->device));
  return 0;
}

// a device buffer of at least `want` elements, reallocated (larger) when it is not
template <typename T>
int ensure(b200fwd_engine *e, T **p, size_t *len, size_t want) {
  if (*len >= want) return 0;
  B200_CUDA(cudaStreamSynchronize(e->stream));
  release(e, *p, *len * sizeof(T));
  *p = nullptr;
  *len = 0;
  CHECK(alloc(e, (void **)p, want * sizeof(T)));
  *len = want;
  return 0;
}

}  // namespace

extern "C" {

int b200fwd_abi_version(void) { return B200FWD_ABI_VERSION; }

int b200fwd_last_error(char *buffer, size_t size) {
  if (!buffer || size == 0) return B200FWD_EINVAL;
  const std::string &m = last_error();
  const size_t n = std::min(size - 1, m.size());
  std::memcpy(buffer, m.data(), n);
  buffer[n] = 0;
  return 0;
}

int b200fwd_create(const void *checkpoint, size_t size, const b200fwd_plan *plan, const b200fwd_options *options,
                   b200fwd_engine **out) {
  return guarded([&] {
    if (!checkpoint || !plan || !out) return fail(B200FWD_EINVAL, "create: null argument");
    *out = nullptr;
    auto *e = new b200fwd_engine();
    const int rc = make_engine(checkpoint, size, plan, options, e);
    if (rc) {
      const std::string keep = last_error();
      destroy(e);
      last_error() = keep;
      return rc;
    }
    *out = e;
    return 0;
  });
}

int b200fwd_destroy(b200fwd_engine *engine) {
  destroy(engine);
  return 0;
}

int b200fwd_bind_logits(b200fwd_engine *e, float *logits) {
  if (!e) return fail(B200FWD_EINVAL, "no engine");
  e->bound = logits;
  return 0;
}

int b200fwd_forward(b200fwd_engine *e, int32_t token, int32_t pos, int32_t need_logits) {
  return guarded([&] {
    CHECK(set_device(e));
    const int32_t slot = 0;
    const uint8_t want = need_logits ? 1 : 0;
    e->last_logits.resize(e->vocab);
    CHECK(run(e, 1, &slot, &token, &pos, &want, need_logits ? e->last_logits.data() : nullptr, nullptr));
    if (need_logits && e->bound) std::memcpy(e->bound, e->last_logits.data(), sizeof(float) * e->vocab);
    return 0;
  });
}

int b200fwd_forward_many(b200fwd_engine *e, const int32_t *tokens, int32_t count, int32_t pos) {
  return guarded([&] {
    CHECK(set_device(e));
    if (count < 0 || (count > 0 && !tokens)) return fail(B200FWD_EINVAL, "forward_many: bad tokens");
    std::vector<int32_t> slots(e->T, 0), p(e->T);
    for (int at = 0; at < count; at += e->T) {
      const int n = std::min(e->T, count - at);
      for (int i = 0; i < n; i++) p[i] = pos + at + i;
      CHECK(run(e, n, slots.data(), tokens + at, p.data(), nullptr, nullptr, nullptr));
    }
    return 0;
  });
}

int b200fwd_prompt_block(b200fwd_engine *e, int32_t *out) {
  if (!e || !out) return fail(B200FWD_EINVAL, "prompt_block: null argument");
  *out = e->T;
  return 0;
}

int b200fwd_keys_values(b200fwd_engine *e, int32_t slot, int32_t from, int32_t count, float *keys, float *values) {
  return guarded([&] {
    CHECK(set_device(e));
    if (slot < 0 || slot >= e->slots || from < 0 || count < 0 || from + count > e->capacity || !keys || !values)
      return fail(B200FWD_EINVAL, "keys_values: out of range");
    const size_t row = (size_t)e->kvDim * e->esize();
    std::vector<uint8_t> raw((size_t)count * row);
    for (int l = 0; l < e->layers; l++) {
      for (int kv = 0; kv < 2; kv++) {
        const uint8_t *src = e->cache + ((((int64_t)slot * e->layers + l) * 2 + kv) * e->capacity + from) * row;
        B200_CUDA(cudaMemcpy(raw.data(), src, raw.size(), cudaMemcpyDeviceToHost));
        float *dst = (kv ? values : keys) + (size_t)l * count * e->kvDim;
        const size_t total = (size_t)count * e->kvDim;
        if (e->half) {
          const uint16_t *h = reinterpret_cast<const uint16_t *>(raw.data());
          for (size_t i = 0; i < total; i++) dst[i] = half_bits_to_float(h[i]);
        } else {
          std::memcpy(dst, raw.data(), total * 4);
        }
      }
    }
    return 0;
  });
}

int b200fwd_logits(b200fwd_engine *e, float *out) {
  if (!e || !out) return fail(B200FWD_EINVAL, "logits: null argument");
  if (e->last_logits.empty()) std::memset(out, 0, sizeof(float) * e->vocab);
  else std::memcpy(out, e->last_logits.data(), sizeof(float) * e->vocab);
  return 0;
}

int b200fwd_backend(b200fwd_engine *e, char *buffer, size_t size) {
  if (!e || !buffer || !size) return fail(B200FWD_EINVAL, "backend: null argument");
  const size_t n = std::min(size - 1, e->backend.size());
  std::memcpy(buffer, e->backend.data(), n);
  buffer[n] = 0;
  return 0;
}

int b200fwd_memory_bytes(b200fwd_engine *e, uint64_t *out) {
  if (!e || !out) return fail(B200FWD_EINVAL, "memory_bytes: null argument");
  *out = e->bytes;
  return 0;
}

int b200fwd_run(b200fwd_engine *e, int32_t n, const int32_t *slots, const int32_t *tokens, const int32_t *pos,
                const uint8_t *want, float *logits, int32_t *argmax) {
  return guarded([&] {
    CHECK(set_device(e));
    if (!tokens || !pos) return fail(B200FWD_EINVAL, "run: null tokens or positions");
    return run(e, n, slots, tokens, pos, want, logits, argmax);
  });
}

int b200fwd_reset_slot(b200fwd_engine *e, int32_t slot) {
  if (!e || slot < 0 || slot >= e->slots) return fail(B200FWD_EINVAL, "reset_slot: out of range");
  return 0;  // positions are the caller's: the next run at position 0 writes over the cache
}

int b200fwd_stream_of(b200fwd_engine *e, b200fwd_stream *out) {
  if (!e || !out) return fail(B200FWD_EINVAL, "stream_of: null argument");
  *out = reinterpret_cast<b200fwd_stream>(e->stream);
  return 0;
}

int b200fwd_launch_count(b200fwd_engine *e, uint64_t *out) {
  if (!e || !out) return fail(B200FWD_EINVAL, "launch_count: null argument");
  *out = launches.load() - e->launches_at_create;
  return 0;
}

int b200fwd_time_matmuls(b200fwd_engine *e, int32_t count, int32_t reps, float *ms_per_pass, double *bytes_per_pass,
                          int32_t *launches_per_pass) {
  return guarded([&] {
    CHECK(set_device(e));
    if (count < 1 || count > e->T || reps < 1 || !ms_per_pass || !bytes_per_pass || !launches_per_pass)
      return fail(B200FWD_EINVAL, "time_matmuls: bad arguments");
    const Matrix *mats[4] = {&e->wqkv, &e->wo, &e->w13, &e->w2};
    // every output goes to a buffer of its own, count x the most rows of any matrix
    int most = e->wcls.rows;
    for (const Matrix *m : mats) most = std::max(most, m->rows);
    float *out = nullptr;
    B200_CUDA(cudaMallocAsync((void **)&out, (size_t)count * most * 4, e->stream));
    struct Free {
      float *p;
      cudaStream_t s;
      ~Free() { cudaFreeAsync(p, s); }
    } free_out{out, e->stream};
    auto bytes = [&](const Matrix &m) {
      return (double)m.rows * m.n * (1.0 + 4.0 / 32) + (double)count * m.n * (1.0 + 4.0 / 32) + 4.0 * count * m.rows;
    };
    double total = 0;
    for (const Matrix *m : mats) total += e->layers * bytes(*m);
    total += bytes(e->wcls);
    cudaEvent_t t0, t1;
    B200_CUDA(cudaEventCreate(&t0));
    B200_CUDA(cudaEventCreate(&t1));
    struct Drop {
      cudaEvent_t a, b;
      ~Drop() {
        cudaEventDestroy(a);
        cudaEventDestroy(b);
      }
    } drop{t0, t1};
    auto pass = [&]() -> int {
      for (int l = 0; l < e->layers; l++)
        for (const Matrix *m : mats) CHECK(matmul(e, *m, l, out, m->rows, 0, count));
      return matmul(e, e->wcls, 0, out, e->wcls.rows, 0, count);
    };
    CHECK(pass());  // warm-up
    B200_CUDA(cudaEventRecord(t0, e->stream));
    for (int r = 0; r < reps; r++) CHECK(pass());
    B200_CUDA(cudaEventRecord(t1, e->stream));
    B200_CUDA(cudaEventSynchronize(t1));
    float ms = 0;
    B200_CUDA(cudaEventElapsedTime(&ms, t0, t1));
    CHECK(check_tc(e));
    *ms_per_pass = ms / reps;
    *bytes_per_pass = total;
    *launches_per_pass = 4 * e->layers + 1;
    return 0;
  });
}

int b200fwd_time_matmul_kinds(b200fwd_engine *e, int32_t count, int32_t reps, float *us_per_launch,
                              double *bytes_per_launch) {
  return guarded([&] {
    CHECK(set_device(e));
    if (count < 1 || count > e->T || reps < 1 || !us_per_launch || !bytes_per_launch)
      return fail(B200FWD_EINVAL, "time_matmul_kinds: bad arguments");
    const Matrix *mats[5] = {&e->wqkv, &e->wo, &e->w13, &e->w2, &e->wcls};
    int most = 0;
    for (const Matrix *m : mats) most = std::max(most, m->rows);
    float *out = nullptr;
    B200_CUDA(cudaMallocAsync((void **)&out, (size_t)count * most * 4, e->stream));
    struct Free {
      float *p;
      cudaStream_t s;
      ~Free() { cudaFreeAsync(p, s); }
    } free_out{out, e->stream};
    cudaEvent_t t0, t1;
    B200_CUDA(cudaEventCreate(&t0));
    B200_CUDA(cudaEventCreate(&t1));
    struct Drop {
      cudaEvent_t a, b;
      ~Drop() {
        cudaEventDestroy(a);
        cudaEventDestroy(b);
      }
    } drop{t0, t1};
    for (int k = 0; k < 5; k++) {
      const Matrix &m = *mats[k];
      const int layers = k == 4 ? 1 : e->layers;
      // every layer's copy of the matrix in turn (distinct memory: a layer's weights are out of L2 again by the time
      // its turn comes back); the classifier alone is larger than L2
      auto pass = [&]() -> int {
        for (int l = 0; l < layers; l++) CHECK(matmul(e, m, l, out, m.rows, 0, count));
        return 0;
      };
      CHECK(pass());  // warm-up
      B200_CUDA(cudaEventRecord(t0, e->stream));
      for (int r = 0; r < reps; r++) CHECK(pass());
      B200_CUDA(cudaEventRecord(t1, e->stream));
      B200_CUDA(cudaEventSynchronize(t1));
      float ms = 0;
      B200_CUDA(cudaEventElapsedTime(&ms, t0, t1));
      us_per_launch[k] = ms * 1000.0f / (float)(reps * layers);
      bytes_per_launch[k] =
          (double)m.rows * m.n * (1.0 + 4.0 / 32) + (double)count * m.n * (1.0 + 4.0 / 32) + 4.0 * count * m.rows;
    }
    return check_tc(e);
  });
}

int b200fwd_generate_many(b200fwd_engine *e, int32_t n, const int32_t *slots, const int32_t *first,
                          const int32_t *pos0, int32_t steps, float temperature, float topp, float penalty,
                          const int32_t *recent, const int32_t *recent_count, const double *randoms,
                          const int32_t *stops, int32_t nstops, int32_t *out, int32_t *made) {
  return guarded([&] {
    CHECK(set_device(e));
    constexpr int W = B200FWD_REPETITION_WINDOW;
    if (n < 1 || n > std::min(e->T, 1024) || steps < 1 || !slots || !first || !pos0 || !out || !made ||
        nstops < 0 || (nstops && !stops) || (n && !recent_count) || !(temperature >= 0) || !(penalty > 0))
      return fail(B200FWD_EINVAL, "generate_many: bad arguments");
    if (temperature > 0 && !randoms) return fail(B200FWD_EINVAL, "generate_many: no random numbers");
    int maxpos = 0;
    for (int i = 0; i < n; i++) {
      if (slots[i] < 0 || slots[i] >= e->slots) return fail(B200FWD_EINVAL, "generate_many: slot out of range");
      for (int j = 0; j < i; j++)
        if (slots[j] == slots[i]) return fail(B200FWD_EINVAL, "generate_many: a slot given twice");
      if (first[i] < 0 || first[i] >= e->vocab) return fail(B200FWD_EINVAL, "generate_many: token out of range");
      if (pos0[i] < 0 || pos0[i] + steps > e->seqLen)
        return fail(B200FWD_EINVAL, "generate_many: the steps run past the context");
      if (recent_count[i] < 0) return fail(B200FWD_EINVAL, "generate_many: a negative history length");
      for (int k = 0; k < std::min(recent_count[i], W); k++)
        if (!recent || recent[(int64_t)i * W + k] < 0 || recent[(int64_t)i * W + k] >= e->vocab)
          return fail(B200FWD_EINVAL, "generate_many: a history token out of range");
      maxpos = std::max(maxpos, pos0[i] + steps - 1);
    }
    for (int k = 0; k < nstops; k++)
      if (stops[k] < 0 || stops[k] >= e->vocab) return fail(B200FWD_EINVAL, "generate_many: a stop token out of range");
    if (maxpos >= e->capacity) CHECK(grow(e, maxpos));
    CHECK(ensure_logit_rows(e, n));
    // the int32 state: ids [n][steps], ring [n][W], ring counts [n], done [n], made [n], stops, sampled ids [n]
    const size_t words = (size_t)n * steps + (size_t)n * W + 4 * (size_t)n + nstops + 1 +
                         (size_t)n * sample_stack_words();
    CHECK(ensure(e, &e->gm_words, &e->gm_words_len, words));
    const bool greedy = temperature == 0;
    if (!greedy) {
      CHECK(ensure(e, &e->gm_randoms, &e->gm_randoms_len, (size_t)n * steps));
      CHECK(ensure(e, &e->gm_scratch, &e->gm_scratch_len, (size_t)n * sample_scratch_words(e->vocab)));
    }
    int32_t *ids_all = e->gm_words, *ring = ids_all + (size_t)n * steps, *ring_count = ring + (size_t)n * W;
    int32_t *done = ring_count + n, *made_d = done + n, *stops_d = made_d + n, *chosen = stops_d + nstops + 1;
    int32_t *stacks = chosen + n;
    // the rings as the reference keeps them (position p of the history at p % W), from the last W tokens given
    std::vector<int32_t> hring((size_t)n * W, 0), hcount(n), zeros(2 * (size_t)n, 0);
    for (int i = 0; i < n; i++) {
      const int len = recent_count[i], m = std::min(len, W);
      for (int k = 0; k < m; k++) hring[(size_t)i * W + (len - m + k) % W] = recent[(size_t)i * W + k];
      hcount[i] = len;
    }
    B200_CUDA(cudaMemcpyAsync(ring, hring.data(), hring.size() * 4, cudaMemcpyHostToDevice, e->stream));
    B200_CUDA(cudaMemcpyAsync(ring_count, hcount.data(), (size_t)n * 4, cudaMemcpyHostToDevice, e->stream));
    B200_CUDA(cudaMemcpyAsync(done, zeros.data(), 2 * (size_t)n * 4, cudaMemcpyHostToDevice, e->stream));
    if (nstops) B200_CUDA(cudaMemcpyAsync(stops_d, stops, (size_t)nstops * 4, cudaMemcpyHostToDevice, e->stream));
    if (!greedy)
      B200_CUDA(cudaMemcpyAsync(e->gm_randoms, randoms, (size_t)n * steps * 8, cudaMemcpyHostToDevice, e->stream));
    const int T = e->T;
    int32_t *m = e->meta_h;
    B200_CUDA(cudaStreamSynchronize(e->stream));
    for (int i = 0; i < n; i++) {
      m[i] = first[i];
      m[T + i] = slots[i];
      m[2 * T + i] = pos0[i];
      m[3 * T + i] = i;
    }
    m[4 * T] = 0;
    m[4 * T + 1] = 0;
    m[4 * T + 2] = 0;
    B200_CUDA(cudaMemcpyAsync(e->meta, m, (size_t)(4 * T + 3) * 4, cudaMemcpyHostToDevice, e->stream));
    // one step, captured once and replayed: every slot's forward pass, the penalty over its recent tokens, the draw
    // (or the argmax), then the bookkeeping (a stop token or a failure ends a slot: its token and position stay, so
    // the passes after it write its last position's keys and values again, the same numbers)
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    const uint64_t before = launches.load();
    B200_CUDA(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
    int rc = forward_device(e, n, n, e->capacity, 0, false);
    if (!rc && penalty != 1.0f)
      rc = launch_penalize(e->logits, e->vocab, ring, W, ring_count, penalty, done, n, e->stream);
    if (!rc)
      rc = greedy ? launch_argmax(chosen, e->logits, e->vocab, e->vocab, n, 1, e->stream)
                  : launch_sample(chosen, e->logits, e->vocab, e->vocab, temperature, topp, e->gm_randoms, 0.0, steps,
                                  e->step_d(), e->gm_scratch, stacks, done, n, e->stream);
    if (!rc)
      rc = launch_advance_sampled(e->tokens_d(), e->pos_d(), chosen, ids_all, steps, e->step_d(), n, e->logits,
                                  e->vocab, greedy ? 1 : 0, ring, W, ring_count, stops_d, nstops, done, made_d,
                                  e->bad_d(), e->stream);
    cudaError_t ce = cudaStreamEndCapture(e->stream, &graph);
    const uint64_t per_step = launches.load() - before;
    launches.fetch_sub(per_step);
    if (rc) {
      if (graph) cudaGraphDestroy(graph);
      return rc;
    }
    if (ce != cudaSuccess) return cuda_fail(ce, "cudaStreamEndCapture");
    ce = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ce != cudaSuccess) return cuda_fail(ce, "cudaGraphInstantiate");
    for (int s = 0; s < steps; s++) {
      ce = cudaGraphLaunch(exec, e->stream);
      if (ce != cudaSuccess) break;
      launches.fetch_add(per_step);
    }
    cudaError_t se = cudaStreamSynchronize(e->stream);
    cudaGraphExecDestroy(exec);
    if (ce != cudaSuccess) return cuda_fail(ce, "cudaGraphLaunch");
    if (se != cudaSuccess) return cuda_fail(se, "cudaStreamSynchronize");
    B200_CUDA(cudaMemcpy(out, ids_all, (size_t)n * steps * 4, cudaMemcpyDeviceToHost));
    B200_CUDA(cudaMemcpy(made, made_d, (size_t)n * 4, cudaMemcpyDeviceToHost));
    CHECK(check_tc(e));
    int32_t bad = 0;
    B200_CUDA(cudaMemcpy(&bad, e->bad_d(), 4, cudaMemcpyDeviceToHost));
    if (bad == 1)
      return fail(B200FWD_ENOTFINITE,
                  "The model computed logits that are not finite numbers (NaN or infinity), so no token can be drawn.");
    if (bad == 2) return fail(B200FWD_EUNSUPPORTED, "generate_many: the nucleus sort ran past its stack");
    return 0;
  });
}

int b200fwd_generate_greedy(b200fwd_engine *e, int32_t n, const int32_t *slots, const int32_t *first,
                            const int32_t *pos0, int32_t steps, int32_t *out) {
  return guarded([&] {
    CHECK(set_device(e));
    if (n < 1 || n > std::min(e->T, 1024) || steps < 1 || !slots || !first || !pos0 || !out)
      return fail(B200FWD_EINVAL, "generate_greedy: bad arguments");
    int maxpos = 0;
    for (int i = 0; i < n; i++) {
      if (slots[i] < 0 || slots[i] >= e->slots) return fail(B200FWD_EINVAL, "generate_greedy: slot out of range");
      for (int j = 0; j < i; j++)
        if (slots[j] == slots[i]) return fail(B200FWD_EINVAL, "generate_greedy: a slot given twice");
      if (first[i] < 0 || first[i] >= e->vocab) return fail(B200FWD_EINVAL, "generate_greedy: token out of range");
      if (pos0[i] < 0 || pos0[i] + steps > e->seqLen)
        return fail(B200FWD_EINVAL, "generate_greedy: the steps run past the context");
      maxpos = std::max(maxpos, pos0[i] + steps - 1);
    }
    if (maxpos >= e->capacity) CHECK(grow(e, maxpos));
    CHECK(ensure_logit_rows(e, n));
    if (e->history_len < n * steps) {
      B200_CUDA(cudaStreamSynchronize(e->stream));
      release(e, e->history, (size_t)e->history_len * 4);
      e->history = nullptr;
      CHECK(alloc(e, (void **)&e->history, (size_t)n * steps * 4));
      e->history_len = n * steps;
    }
    const int T = e->T;
    int32_t *m = e->meta_h;
    B200_CUDA(cudaStreamSynchronize(e->stream));
    for (int i = 0; i < n; i++) {
      m[i] = first[i];
      m[T + i] = slots[i];
      m[2 * T + i] = pos0[i];
      m[3 * T + i] = i;
    }
    m[4 * T] = 0;
    m[4 * T + 1] = 0;
    m[4 * T + 2] = 0;
    B200_CUDA(cudaMemcpyAsync(e->meta, m, (size_t)(4 * T + 3) * 4, cudaMemcpyHostToDevice, e->stream));
    // one step, captured once and replayed: the forward pass of every slot's token, the argmax, and the step's
    // bookkeeping (the argmax becomes the next token, the positions move on), with no host in between
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    const uint64_t before = launches.load();
    B200_CUDA(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
    int rc = forward_device(e, n, n, e->capacity, 0);
    if (!rc)
      rc = launch_advance(e->tokens_d(), e->pos_d(), e->argmax, e->history, steps, e->step_d(), n, e->logits, e->vocab,
                          e->bad_d(), e->stream);
    cudaError_t ce = cudaStreamEndCapture(e->stream, &graph);
    const uint64_t per_step = launches.load() - before;
    launches.fetch_sub(per_step);  // counted below as they replay
    if (rc) {
      if (graph) cudaGraphDestroy(graph);
      return rc;
    }
    if (ce != cudaSuccess) return cuda_fail(ce, "cudaStreamEndCapture");
    ce = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ce != cudaSuccess) return cuda_fail(ce, "cudaGraphInstantiate");
    for (int s = 0; s < steps; s++) {
      ce = cudaGraphLaunch(exec, e->stream);
      if (ce != cudaSuccess) break;
      launches.fetch_add(per_step);
    }
    cudaError_t se = cudaStreamSynchronize(e->stream);
    cudaGraphExecDestroy(exec);
    if (ce != cudaSuccess) return cuda_fail(ce, "cudaGraphLaunch");
    if (se != cudaSuccess) return cuda_fail(se, "cudaStreamSynchronize");
    B200_CUDA(cudaMemcpy(out, e->history, (size_t)n * steps * 4, cudaMemcpyDeviceToHost));
    CHECK(check_tc(e));
    int32_t bad = 0;
    B200_CUDA(cudaMemcpy(&bad, e->bad_d(), 4, cudaMemcpyDeviceToHost));
    if (bad)
      return fail(B200FWD_ENOTFINITE,
                  "The model computed logits that are not finite numbers (NaN or infinity), so no token can be drawn.");
    return 0;
  });
}

}  // extern "C"
