// attention_tc.cu — causal attention of a whole prompt on the 5th-generation tensor cores (flash attention with an
// online softmax): the computation the reference does one query token at a time (public/forward.js:1055-1057 ->
// kernels/kernel.ts:447-566 attentionOf over the cache, after kernel.ts:344-357 rope on the query and the keys), for
// every token of every sequence and head at once. Not bit-exact (the reference's own tolerance line for float
// attention is 1e-3 relative): float16 operands, float32 accumulation and softmax.
//
//   rope_prologue: the reference's rope (one rounding per operation) on q and k, then float16: Qh, Kh [b][h][s][d];
//   values_transposed: the values as float16, Vt [b][kv][d][s] (the tensor cores' B operand of P V wants the keys
//     contiguous).
//   flash_attn_tc: one block per (sequence, head, pair of neighbouring tiles of 128 queries), the heaviest pairs
//     first; 384 threads:
//     warp 0 TMA: both query tiles once, then each 64-key tile of K and of V^T (four buffers each, 128-byte swizzle),
//       shared by the two query tiles;
//     warp 1 MMA: per query tile t and key tile j, S_t(j) = Q_t K_j^T (kind::f16, M = 128, N = 64, four K = 16
//       steps) into one of the tile's two TMEM buffers, and O_t += P_t(j) V_j with P read from TMEM (the A operand)
//       and V^T from shared memory (M = 128, N = head size, four K = 16 steps); S_t(j + 2) is issued as soon as
//       P V_t(j) is done, so a softmax finds its next scores waiting;
//     warps 4..7 and 8..11 the softmax of each tile, a thread per query row (TMEM lane): the row's largest score,
//       exp2 of the scaled scores (ex2.approx) against a running maximum that moves only when a row's largest rises
//       by more than 2^8 (then O is rescaled in TMEM first), the row sum in float32, P as float16 pairs into TMEM
//       over the scores it read; at the end O / sum into the output.
// TMEM (512 columns): tile t's two S buffers at t * 128 + {0, 64}, its O at 256 + t * 64. One block an SM.
// Every mbarrier wait is bounded: past it the kernel records an error and runs to its end.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <cstdint>
#include <string>

#include "common.h"
#include "exact.cuh"
#include "gemm_tc.h"
#include "kernels.h"

namespace b200 {
namespace {

constexpr int QT = 128;       // queries of a tile (TMEM lanes)
constexpr int KT = 64;        // keys of a tile
constexpr int HD = 64;        // head size this kernel takes
constexpr int THREADS = 384;  // warps 0..3: TMA, MMA, two idle; 4..7 and 8..11: softmax of the two tiles
constexpr uint32_t WAIT_HINT_NS = 1000000;
constexpr uint32_t WAIT_TRIES = 2000;
constexpr float RESCALE = 8.0f;  // log2 of how far P may rise above 1 before the running maximum moves

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *error, int code) {
  const uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0;; i++) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity), "r"(WAIT_HINT_NS)
        : "memory");
    if (done) return true;
    if (*(volatile int *)error) return false;
    if (i >= WAIT_TRIES) {
      atomicCAS(error, 0, code);
      return false;
    }
  }
}
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
// K-major, 128-byte swizzle, 8-row atoms 1024 bytes apart
__device__ __forceinline__ uint64_t smem_desc(const void *p) {
  const uint64_t addr = smem_u32(p);
  return ((addr >> 4) & 0x3fff) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
         ((uint64_t)2 << 61);
}
// kind::f16, D float32, A and B float16, K-major, M = 128, N = n
__host__ __device__ constexpr uint32_t idesc_f16(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(QT >> 4) << 24);
}
__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, int acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// A from TMEM (P, float16 pairs along K), B from shared memory
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, int acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&r)[32]) {
  uint32_t u[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]), "=r"(u[7]), "=r"(u[8]),
        "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]), "=r"(u[14]), "=r"(u[15]), "=r"(u[16]),
        "=r"(u[17]), "=r"(u[18]), "=r"(u[19]), "=r"(u[20]), "=r"(u[21]), "=r"(u[22]), "=r"(u[23]), "=r"(u[24]),
        "=r"(u[25]), "=r"(u[26]), "=r"(u[27]), "=r"(u[28]), "=r"(u[29]), "=r"(u[30]), "=r"(u[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; i++) r[i] = __uint_as_float(u[i]);
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&u)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(u[0]), "r"(u[1]), "r"(u[2]), "r"(u[3]), "r"(u[4]), "r"(u[5]), "r"(u[6]), "r"(u[7]), "r"(u[8]), "r"(u[9]),
      "r"(u[10]), "r"(u[11]), "r"(u[12]), "r"(u[13]), "r"(u[14]), "r"(u[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(__float_as_uint(r[0])), "r"(__float_as_uint(r[1])), "r"(__float_as_uint(r[2])), "r"(__float_as_uint(r[3])),
      "r"(__float_as_uint(r[4])), "r"(__float_as_uint(r[5])), "r"(__float_as_uint(r[6])), "r"(__float_as_uint(r[7])),
      "r"(__float_as_uint(r[8])), "r"(__float_as_uint(r[9])), "r"(__float_as_uint(r[10])),
      "r"(__float_as_uint(r[11])), "r"(__float_as_uint(r[12])), "r"(__float_as_uint(r[13])),
      "r"(__float_as_uint(r[14])), "r"(__float_as_uint(r[15])), "r"(__float_as_uint(r[16])),
      "r"(__float_as_uint(r[17])), "r"(__float_as_uint(r[18])), "r"(__float_as_uint(r[19])),
      "r"(__float_as_uint(r[20])), "r"(__float_as_uint(r[21])), "r"(__float_as_uint(r[22])),
      "r"(__float_as_uint(r[23])), "r"(__float_as_uint(r[24])), "r"(__float_as_uint(r[25])),
      "r"(__float_as_uint(r[26])), "r"(__float_as_uint(r[27])), "r"(__float_as_uint(r[28])),
      "r"(__float_as_uint(r[29])), "r"(__float_as_uint(r[30])), "r"(__float_as_uint(r[31]))
      : "memory");
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ uint64_t fma_2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add_2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float lo_of(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float hi_of(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
// 32 consecutive TMEM columns of this thread's lane, not waited for (tcgen05.wait::ld before use)
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, float *r) {
  uint32_t *u = reinterpret_cast<uint32_t *>(r);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]), "=r"(u[7]), "=r"(u[8]),
        "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]), "=r"(u[14]), "=r"(u[15]), "=r"(u[16]),
        "=r"(u[17]), "=r"(u[18]), "=r"(u[19]), "=r"(u[20]), "=r"(u[21]), "=r"(u[22]), "=r"(u[23]), "=r"(u[24]),
        "=r"(u[25]), "=r"(u[26]), "=r"(u[27]), "=r"(u[28]), "=r"(u[29]), "=r"(u[30]), "=r"(u[31])
      : "r"(taddr));
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// two floats as float16 (round to nearest even): lo in the low half
__device__ __forceinline__ uint32_t pack_f16(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// one tile of scores of this thread's query row r (TMEM lane): its largest (keys past the row masked on the diagonal
// tile), the running maximum m moved (and O and the sum l scaled) only where the largest rises more than RESCALE,
// then P = 2^(s c - m) as float16 pairs over the scores' first half, the sum in float32
template <bool DIAG>
__device__ __forceinline__ void softmax_tile(uint32_t tS, uint32_t tO, int r, int off, float c, int j, float &m,
                                             float &l, uint64_t (*pv_done)[2], int *error) {
  float x[KT];
#pragma unroll
  for (int ch = 0; ch < KT / 32; ch++) tmem_ld32_nowait(tS + ch * 32, x + ch * 32);
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
  if (DIAG) {
#pragma unroll
    for (int i = 0; i < KT; i++)
      if (i + off > r) x[i] = -INFINITY;  // a key after the query (off: the key tile's start past the query tile's)
  }
  float mx = x[0];
#pragma unroll
  for (int i = 1; i + 1 < KT; i += 2) mx = max3(mx, x[i], x[i + 1]);
  mx = fmaxf(mx, x[KT - 1]);
  const float mnew = fmaxf(m, mx * c);  // (a row whose keys are all after it keeps m: -inf * c is -inf)
  if (j == 0) {
    m = mnew;
  } else if (mnew > m + RESCALE) {
    // O holds the steps so far: once the last P V is done, scale it (and the sum) to the new maximum
    mbar_wait(&(*pv_done)[(j - 1) & 1], ((j - 1) >> 1) & 1, error, 9);
    fence_after();
    const float f = ex2(m - mnew);
#pragma unroll
    for (int ch = 0; ch < HD / 32; ch++) {
      float o[32];
      tmem_ld32(tO + ch * 32, o);
#pragma unroll
      for (int i = 0; i < 32; i++) o[i] *= f;
      tmem_st32(tO + ch * 32, o);
    }
    l *= f;
    m = mnew;
  }
  const uint64_t c2 = f2(c, c), nm2 = f2(-m, -m);
  uint64_t sum = f2(0.0f, 0.0f);
  uint32_t pk[KT / 2];
#pragma unroll
  for (int i = 0; i < KT; i += 2) {
    const uint64_t e = fma_2(f2(x[i], x[i + 1]), c2, nm2);
    const float p0 = ex2(lo_of(e)), p1 = ex2(hi_of(e));
    sum = add_2(sum, f2(p0, p1));
    pk[i / 2] = pack_f16(p0, p1);
  }
  l += lo_of(sum) + hi_of(sum);
#pragma unroll
  for (int ch = 0; ch < KT / 32; ch++) tmem_st16(tS + ch * 16, *reinterpret_cast<const uint32_t(*)[16]>(pk + ch * 16));
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

constexpr int KSTAGES = 4;  // K and V^T tiles in flight

struct Smem {
  alignas(1024) uint8_t q[2][QT * HD * 2];             // two query tiles: 128 queries x 64 float16 each
  alignas(1024) uint8_t k[KSTAGES][KT * HD * 2];       // 64 keys x 64
  alignas(1024) uint8_t v[KSTAGES][HD * KT * 2];       // V^T: 64 dims x 64 keys
  uint64_t q_full, k_full[KSTAGES], k_empty[KSTAGES], v_full[KSTAGES], v_empty[KSTAGES];
  // [query tile][S buffer]: a barrier per buffer, so that no waiter is ever two phases behind (a softmax runs up to
  // two key tiles ahead of its P V)
  uint64_t s_full[2][2], p_full[2][2], pv_done[2][2], mma_done;
  uint32_t tmem_base;
};

// the reference's rope (kernel.ts:344-357, every product and sum rounded on its own) on q and k of each token, then
// float16 (round to nearest even): Qh [b][h][s][d], Kh [b][kv][s][d], Vt [b][kv][d][s]; tables [s][d/2]
__global__ void rope_prologue(__half *qh, __half *kh, const float *q, const float *k, const float *cos_t,
                              const float *sin_t, int B, int S, int H, int KV, int D) {
  // block (b, s) of gridDim.x = B * S; thread (head of H + KV, pair)
  const int pairs = D / 2, hh = threadIdx.x / pairs, p = threadIdx.x % pairs;
  const int bs = blockIdx.x, s = bs % S, b = bs / S;
  if (hh >= H + KV) return;
  const float c = cos_t[(int64_t)s * pairs + p], sn = sin_t[(int64_t)s * pairs + p];
  const bool isq = hh < H;
  const int h = isq ? hh : hh - H;
  const float2 v = *reinterpret_cast<const float2 *>((isq ? q : k) + ((int64_t)bs * (isq ? H : KV) + h) * D + 2 * p);
  const float r0 = fsub(fmul(v.x, c), fmul(v.y, sn)), r1 = fadd(fmul(v.x, sn), fmul(v.y, c));
  __half *dst = (isq ? qh : kh) + (((int64_t)b * (isq ? H : KV) + h) * S + s) * D + 2 * p;
  *reinterpret_cast<__half2 *>(dst) = __halves2half2(__float2half_rn(r0), __float2half_rn(r1));
}

// the values as float16, transposed per head through shared memory: Vt [b][kv][d][s] from v [b][s][kv][d]; a block a
// tile of 32 positions x 32 dims (both sides' accesses coalesced)
__global__ void values_transposed(__half *vt, const float *v, int S, int KV, int D) {
  __shared__ float tile[32][33];
  const int s0 = blockIdx.x * 32, d0 = blockIdx.z * 32, bk = blockIdx.y, b = bk / KV, h = bk % KV;
  for (int i = threadIdx.y; i < 32; i += blockDim.y)
    tile[i][threadIdx.x] = v[(((int64_t)b * S + s0 + i) * KV + h) * D + d0 + threadIdx.x];
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y)
    vt[(((int64_t)b * KV + h) * D + d0 + i) * S + s0 + threadIdx.x] = __float2half_rn(tile[threadIdx.x][i]);
}

__global__ void __launch_bounds__(THREADS, 1)
    flash_attn_tc(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                  const __grid_constant__ CUtensorMap vmap, float *out, int B, int S, int H, int KV, float scale,
                  int *error) {
  extern __shared__ uint8_t raw[];
  Smem &s = *reinterpret_cast<Smem *>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pairs = S / (2 * QT), bh_count = B * H;
  // the heaviest pairs of query tiles (the last queries, which see every key) first
  const int pair = pairs - 1 - (int)(blockIdx.x / bh_count);
  const int bh = (int)(blockIdx.x % bh_count), b = bh / H, h = bh % H, kvh = h / (H / KV);
  const int qt[2] = {2 * pair, 2 * pair + 1};
  const int per = QT / KT;  // key tiles of a query tile's width
  const int nkv_t[2] = {(qt[0] + 1) * per, (qt[1] + 1) * per};  // causal: the keys up to the tile's last query
  const int nkv = nkv_t[1];
  if (threadIdx.x == 0) {
    mbar_init(&s.q_full, 1);
    for (int i = 0; i < KSTAGES; i++) {
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.k_empty[i], 1);
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.v_empty[i], 1);
    }
    for (int t = 0; t < 2; t++)
      for (int u = 0; u < 2; u++) {
        mbar_init(&s.s_full[t][u], 1);
        mbar_init(&s.p_full[t][u], 4);
        mbar_init(&s.pv_done[t][u], 1);
      }
    mbar_init(&s.mma_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&s.tmem_base)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = s.tmem_base;
  // TMEM: tile t's two S buffers at t * 128 + u * 64 (P over each one's first 32 columns), its O at 256 + t * 64
  auto tS = [&](int t, int u) { return tmem + (uint32_t)(t * 2 * KT + u * KT); };
  auto tO = [&](int t) { return tmem + (uint32_t)(4 * KT + t * HD); };
  const int qrow = (b * H + h) * S + qt[0] * QT;  // the first tile's first row in Qh (the second follows it)
  const int krow = (b * KV + kvh) * S;            // the head's first row in Kh
  const int vrow = (b * KV + kvh) * HD;           // the head's first row in Vt

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 56;");
    if (warp == 0) {
      if (lane == 0) {
        mbar_expect_tx(&s.q_full, 2 * QT * HD * 2);
        tma_load_2d(s.q[0], &qmap, &s.q_full, 0, qrow);
        tma_load_2d(s.q[1], &qmap, &s.q_full, 0, qrow + QT);
        int issued = 0;
        for (int j = 0; j < nkv; j++) {
          const int slot = j % KSTAGES;
          const uint32_t ph = ((j / KSTAGES) & 1) ^ 1;
          if (!mbar_wait(&s.k_empty[slot], ph, error, 1)) break;
          mbar_expect_tx(&s.k_full[slot], KT * HD * 2);
          tma_load_2d(s.k[slot], &kmap, &s.k_full[slot], 0, krow + j * KT);
          if (!mbar_wait(&s.v_empty[slot], ph, error, 2)) break;
          mbar_expect_tx(&s.v_full[slot], KT * HD * 2);
          tma_load_2d(s.v[slot], &vmap, &s.v_full[slot], j * KT, vrow);
          issued = j + 1;
        }
        // no copy may still be landing when the block ends
        mbar_wait(&s.q_full, 0, error, 11);
        for (int j = issued > KSTAGES ? issued - KSTAGES : 0; j < issued; j++) {
          mbar_wait(&s.k_full[j % KSTAGES], (j / KSTAGES) & 1, error, 12);
          mbar_wait(&s.v_full[j % KSTAGES], (j / KSTAGES) & 1, error, 13);
        }
      }
    } else if (warp == 1) {
      // S_t(j) = Q_t K_j^T into tile t's buffer j % 2; O_t += P_t(j) V_j. S_t(j + 2) takes buffer j % 2 once P V_t(j)
      // has read the P there, so each softmax finds its next S ready while its last P V runs.
      const uint32_t id_s = idesc_f16(KT), id_o = idesc_f16(HD);
      auto issue_s = [&](int t, int j) {
        const int slot = j % KSTAGES;
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk++)
          mma_ss(tS(t, j & 1), smem_desc(s.q[t] + 32 * kk), smem_desc(s.k[slot] + 32 * kk), id_s, kk > 0);
        commit(&s.s_full[t][j & 1]);
      };
      auto issue_pv = [&](int t, int j) {
        const int slot = j % KSTAGES;
#pragma unroll
        for (int kk = 0; kk < KT / 16; kk++)
          mma_ts(tO(t), tS(t, j & 1) + 8 * kk, smem_desc(s.v[slot] + 32 * kk), id_o, j > 0 || kk > 0);
        commit(&s.pv_done[t][j & 1]);
      };
      bool ok = mbar_wait(&s.q_full, 0, error, 3);
      for (int j = 0; ok && j < 2; j++) {
        ok = mbar_wait(&s.k_full[j], 0, error, 4);
        if (!ok) break;
        fence_after();
        if (lane == 0) {
          issue_s(0, j);
          issue_s(1, j);
          commit(&s.k_empty[j]);
        }
        __syncwarp();
      }
      for (int j = 0; ok && j < nkv; j++) {
        const int slot = j % KSTAGES, nslot = (j + 2) % KSTAGES;
        ok = mbar_wait(&s.v_full[slot], (j / KSTAGES) & 1, error, 5);
        for (int t = 0; ok && t < 2; t++) {
          if (j >= nkv_t[t]) continue;
          ok = mbar_wait(&s.p_full[t][j & 1], (j >> 1) & 1, error, 6);
          if (!ok) break;
          fence_after();
          if (lane == 0) {
            issue_pv(t, j);
            if (t == 1) commit(&s.v_empty[slot]);
          }
          __syncwarp();
          if (j + 2 < nkv_t[t]) {
            ok = mbar_wait(&s.pv_done[t][j & 1], (j >> 1) & 1, error, 7) &&
                 mbar_wait(&s.k_full[nslot], ((j + 2) / KSTAGES) & 1, error, 8);
            if (!ok) break;
            fence_after();
            if (lane == 0) {
              issue_s(t, j + 2);
              if (t == 1) commit(&s.k_empty[nslot]);
            }
            __syncwarp();
          }
        }
      }
      // every MMA issued has completed before the block frees TMEM
      if (lane == 0) commit(&s.mma_done);
      __syncwarp();
      mbar_wait(&s.mma_done, 0, error, 14);
    }
  } else {
    // (the first warpgroup gives back 112 registers a thread, these two take 56 each: 128 x 56 + 256 x 224 = 384 x 168)
    asm volatile("setmaxnreg.inc.sync.aligned.u32 224;");
    // ---- softmax of tile t: thread r of its warpgroup owns query row qt[t] * QT + r, TMEM lane r
    const int t = (warp - 4) >> 2, r = threadIdx.x - 128 * (t + 1);
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const float c = scale * 1.4426950408889634f;  // scores to base 2
    const int q_tile = t ? qt[1] : qt[0], n = t ? nkv_t[1] : nkv_t[0];
    const uint32_t o_col = tO(t) + lane_base;
    float m = -INFINITY, l = 0.0f;
    for (int j = 0; j < n; j++) {
      mbar_wait(&s.s_full[t][j & 1], (j >> 1) & 1, error, 16);
      fence_after();
      const int off = j * KT - q_tile * QT;  // the key tile's first key less the query tile's first query
      if (off + KT - 1 > 0)
        softmax_tile<true>(tS(t, j & 1) + lane_base, o_col, r, off, c, j, m, l, &s.pv_done[t], error);
      else
        softmax_tile<false>(tS(t, j & 1) + lane_base, o_col, r, off, c, j, m, l, &s.pv_done[t], error);
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.p_full[t][j & 1]);
    }
    // O / sum into the output [b][s][h][d]
    mbar_wait(&s.pv_done[t][(n - 1) & 1], ((n - 1) >> 1) & 1, error, 17);
    fence_after();
    const float inv = 1.0f / l;
    float *dst = out + (((int64_t)b * S + q_tile * QT + r) * H + h) * HD;
#pragma unroll
    for (int ch = 0; ch < HD / 32; ch++) {
      float o[32];
      tmem_ld32(o_col + ch * 32, o);
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<float4 *>(dst + ch * 32 + i) = make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv,
                                                                     o[i + 3] * inv);
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
  }
}

int make_f16_map(CUtensorMap *map, const void *base, int64_t cols, int64_t rows, int box_cols, int box_rows) {
  return make_map(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, cols, rows, cols * 2, box_cols, box_rows,
                  CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace

size_t prefill_attention_scratch(int B, int S, int H, int KV, int D) {
  return ((size_t)B * H * S * D + 2 * (size_t)B * KV * S * D) * 2 + 4 + 256;
}

int launch_prefill_attention(float *out, const float *q, const float *k, const float *v, const float *cos_t,
                             const float *sin_t, int B, int S, int H, int KV, int D, float scale, void *scratch,
                             cudaStream_t stream) {
  if (B < 1 || S < 1 || H < 1 || KV < 1 || H % KV) return fail(B200FWD_EINVAL, "prefill attention: bad sizes");
  if (D != HD) return fail(B200FWD_EUNSUPPORTED, "prefill attention: head size 64 only");
  if (S % (2 * QT)) return fail(B200FWD_EUNSUPPORTED, "prefill attention: the sequence must be whole 256-token pairs of tiles");
  if (reinterpret_cast<uintptr_t>(scratch) % 256 || reinterpret_cast<uintptr_t>(out) % 16)
    return fail(B200FWD_EINVAL, "prefill attention: scratch on 256 bytes, out on 16");
  __half *qh = reinterpret_cast<__half *>(scratch);
  __half *kh = qh + (size_t)B * H * S * D;
  __half *vt = kh + (size_t)B * KV * S * D;
  int *error = reinterpret_cast<int *>(vt + (size_t)B * KV * S * D);
  B200_CUDA(cudaMemsetAsync(error, 0, 4, stream));
  const int threads = ((H + KV) * (D / 2) + 31) / 32 * 32;
  if (threads > 1024) return fail(B200FWD_EUNSUPPORTED, "prefill attention: more than 64 heads");
  rope_prologue<<<(unsigned)(B * S), threads, 0, stream>>>(qh, kh, q, k, cos_t, sin_t, B, S, H, KV, D);
  B200_LAUNCHED("rope_prologue");
  values_transposed<<<dim3(S / 32, B * KV, D / 32), dim3(32, 8), 0, stream>>>(vt, v, S, KV, D);
  B200_LAUNCHED("values_transposed");
  CUtensorMap qm, km, vm;
  int rc = make_f16_map(&qm, qh, D, (int64_t)B * H * S, D, QT);
  if (!rc) rc = make_f16_map(&km, kh, D, (int64_t)B * KV * S, D, KT);
  if (!rc) rc = make_f16_map(&vm, vt, S, (int64_t)B * KV * D, KT, D);
  if (rc) return rc;
  const size_t smem = sizeof(Smem) + 1024;
  B200_CUDA(cudaFuncSetAttribute(flash_attn_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  flash_attn_tc<<<(unsigned)(B * H * (S / (2 * QT))), THREADS, smem, stream>>>(qm, km, vm, out, B, S, H, KV, scale,
                                                                                 error);
  B200_LAUNCHED("flash_attn_tc");
  return 0;
}

int check_prefill_attention(const void *scratch, int B, int S, int H, int KV, int D, cudaStream_t stream) {
  const int *error = reinterpret_cast<const int *>(reinterpret_cast<const __half *>(scratch) +
                                                   (size_t)B * H * S * D + 2 * (size_t)B * KV * S * D);
  int32_t e = 0;
  B200_CUDA(cudaMemcpyAsync(&e, error, 4, cudaMemcpyDeviceToHost, stream));
  B200_CUDA(cudaStreamSynchronize(stream));
  if (e) return fail(B200FWD_ETIMEOUT, "prefill attention: a pipeline wait gave up (code " + std::to_string(e) + ")");
  return 0;
}

}  // namespace b200
