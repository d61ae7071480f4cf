// gemm_tc.cu — the int8 group-32 matmul of a prompt block or of many sequences' tokens on the 5th-generation tensor
// cores: kernel_relaxed.ts:34-67 / 164-183 (matmul_q8r, matmul_q8r_tile) for count >= 16 tokens, to the bit.
//
// The reference's number for (row r, token t) is a float chain over the row's groups of 32: each group's exact
// integer dot(w, q - 64) times (weight scale x activation scale), rounded once, added into lane g % 4 for the groups
// below the last four, the lanes added ((0 + 1) + 2) + 3, then the groups past the fours one at a time. Here:
//   - warp 0: TMA brings 128 weight rows x 128 bytes (four groups), BN tokens' activations x 128 bytes and both
//     scale tiles per stage into shared memory, 8 stages deep (128-byte swizzle; no multicast);
//   - warp 1: one thread issues one tcgen05.mma kind::i8 per group (K = 32: exactly one group) into a TMEM column
//     block of its own (128 lanes = rows, BN columns = tokens): every group's int32 sums, exact, none added to
//     another. TMEM holds several stages at once (slots), and one tcgen05.commit per stage releases a slot;
//   - warps 2..17 (epilogue): four per TMEM lane quarter, each with BN / 4 tokens, read their groups' sums
//     (tcgen05.ld) and keep the reference's four chain accumulators of each (row, token) in registers, with one
//     rounding per float operation (__fmul_rn / __fadd_rn; no contraction, built with --fmad=false).
// Every mbarrier wait has an iteration limit: past it the kernel records an error and returns (no hang).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstring>
#include <string>

#include "common.h"
#include "gemm_tc.h"

namespace b200 {
namespace {

constexpr int BM = 128;                 // rows of a tile (TMEM lanes)
constexpr int KSTAGE = 128;             // bytes of K per stage: four groups
constexpr int STAGES = 8;
constexpr int BN_MAX = 32;            // tokens of a tile at most (32 accumulators a thread)
constexpr int EPI_WARPS = 16;
constexpr int THREADS = 32 * (2 + EPI_WARPS);
constexpr uint32_t WAIT_HINT_NS = 1000000;  // 1 ms
constexpr uint32_t WAIT_TRIES = 2000;

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
// true when the phase of `parity` completed; false when the wait gave up, or another warp of the grid already did
// (the error flag is then set and every later wait returns soon: the kernel runs to its end and frees TMEM).
// try_wait with a suspend-time hint: a waiting warp sleeps until the phase completes (it takes no issue slots from
// the producer and MMA warps) or the hint's 1 ms passes; the error word (global memory) is read only then, and
// after WAIT_TRIES such expiries (about 2 s) the wait gives up.
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

// tcgen05 shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms 1024 bytes apart
__device__ __forceinline__ uint64_t smem_desc(const void *p) {
  const uint64_t addr = smem_u32(p);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3fff;            // start address
  d |= (uint64_t)1 << 16;               // leading byte offset (unused for swizzled K-major): 16 bytes
  d |= (uint64_t)(1024 >> 4) << 32;     // stride byte offset: 8 rows of 128 bytes
  d |= (uint64_t)1 << 46;               // version (Blackwell)
  d |= (uint64_t)2 << 61;               // SWIZZLE_128B
  return d;
}

// instruction descriptor: kind::i8, D int32, A and B signed int8, both K-major, M = 128, N = bn
__host__ __device__ constexpr uint32_t idesc_i8(int bn) {
  return (2u << 4)                         // D format: S32
         | (1u << 7) | (1u << 10)          // A, B: signed 8-bit
         | ((uint32_t)(bn >> 3) << 17)     // N >> 3
         | ((uint32_t)(BM >> 4) << 24);    // M >> 4
}

// D = A x B (each group's MMA writes its own column block)
__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, 0, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Two float32 lanes at once (PTX .f32x2), each lane rounded on its own. A paired multiply whose product feeds a
// paired add is fused into one fma below PTX (one rounding: not the reference's number); a product that is the addend
// of an fma cannot be fused. So the chains add as fma(one, acc, product), `one` being 1.0f from a kernel argument:
// acc * 1 is exact, and acc + product is then rounded once, as an add rounds it.
__device__ __forceinline__ uint64_t pack2(uint32_t a, uint32_t b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
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

// an int32 below 2^22 in magnitude as float32, exactly: its bits added to those of 1.5 * 2^23, less 1.5 * 2^23
constexpr uint32_t MAGIC_BITS = 0x4B400000u;
constexpr float MAGIC = 12582912.0f;

struct Smem {
  alignas(1024) uint8_t a[STAGES][BM * KSTAGE];       // 128 weight rows x four groups
  alignas(1024) uint8_t b[STAGES][BN_MAX * KSTAGE];   // the tokens x four groups
  alignas(128) float ws[STAGES][BM][4];               // the rows' four groups' scales
  alignas(128) float xs[STAGES][4 * BN_MAX];          // the tokens' scales: four rows (groups) of bn tokens
  uint64_t full[STAGES], empty[STAGES];
  uint64_t slot_full[8], slot_empty[8];  // TMEM stage slots: four groups' columns each
  uint32_t tmem_base;
};

// TPW consecutive TMEM columns (the tokens of this warp) of its 32 lanes
template <int TPW>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[TPW]);
template <>
__device__ __forceinline__ void tmem_ld<8>(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_ld<4>(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}

// Warp roles: 0 TMA producer, 1 MMA issue, 2..17 epilogue. Epilogue warp w reads TMEM lane quarter w % 4 (its 32
// rows) and token columns (w - 2) / 4 * TPW .. + TPW, and keeps the reference's four chain accumulators of each of
// its (row, token) in registers, two tokens to a 64-bit pair: the chains, their sum and the groups past the fours
// all happen in one thread. A group's sum S becomes float(S) as (the float with bits S + magic_bits) - magic.
template <int BN>
__global__ void __launch_bounds__(THREADS, 1)
    q8_gemm_tc(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
               const __grid_constant__ CUtensorMap wsmap, const __grid_constant__ CUtensorMap xsmap, GemmArgs args) {
  extern __shared__ uint8_t raw[];
  Smem &s = *reinterpret_cast<Smem *>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  constexpr int SLOTS = 512 / (4 * BN);  // TMEM holds this many stages' four groups at once
  constexpr int TPW = BN / 4;            // tokens of an epilogue warp
  constexpr int PAIRS = TPW / 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ng = args.n >> 5, ng4 = ng & ~3;
  const int kstages = (args.n + KSTAGE - 1) / KSTAGE;
  const int row0 = blockIdx.y * BM, tok0 = blockIdx.x * BN;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; i++) {
      mbar_init(&s.full[i], 1);
      // every epilogue warp done with the stage (it has seen the stage's MMAs complete, so A and B are free too)
      mbar_init(&s.empty[i], EPI_WARPS);
    }
    for (int i = 0; i < SLOTS; i++) {
      mbar_init(&s.slot_full[i], 1);
      mbar_init(&s.slot_empty[i], EPI_WARPS);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // TMEM: 512 columns, the whole of this SM's (one block per SM)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&s.tmem_base)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == 0) {
    // ---- producer: each stage's weights, activations and both scale tiles on one barrier
    if (lane == 0) {
      const int wy = args.w_row0 + row0;
      constexpr uint32_t bytes = BM * KSTAGE + BN * KSTAGE + BM * 16 + BN * 16;
      for (int k = 0; k < kstages; k++) {
        const int st = k % STAGES;
        if (!mbar_wait(&s.empty[st], ((k / STAGES) & 1) ^ 1, args.error, 1)) break;
        mbar_expect_tx(&s.full[st], bytes);
        tma_load_2d(s.a[st], &wmap, &s.full[st], k * KSTAGE, wy);
        tma_load_2d(s.b[st], &xmap, &s.full[st], k * KSTAGE, tok0);
        tma_load_2d(s.ws[st], &wsmap, &s.full[st], k * 4, wy);
        tma_load_2d(s.xs[st], &xsmap, &s.full[st], tok0, k * 4);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issue: a stage's four groups, one MMA each (K = 32, one group) into four TMEM column blocks of the
    // stage's slot, one commit per stage. A slot is free once every epilogue warp has read it.
    const uint32_t idesc = idesc_i8(BN);
    for (int k = 0; k < kstages; k++) {
      const int st = k % STAGES, slot = k % SLOTS;
      if (!mbar_wait(&s.full[st], (k / STAGES) & 1, args.error, 2)) break;
      if (!mbar_wait(&s.slot_empty[slot], ((k / SLOTS) & 1) ^ 1, args.error, 3)) break;
      tc_fence_after();
      if (lane == 0) {
        const int groups = min(4, ng - 4 * k);
        for (int j = 0; j < groups; j++)
          mma_i8(tmem + (uint32_t)((slot * 4 + j) * BN), smem_desc(s.a[st] + 32 * j), smem_desc(s.b[st] + 32 * j),
                 idesc);
        mma_commit(&s.slot_full[slot]);
      }
      __syncwarp();
    }
  } else {
    // ---- epilogue
    const int quarter = warp % 4, sub = (warp - 2) / 4;
    const uint32_t magic_bits = args.magic_bits;
    const float magic = args.magic;
    const uint64_t magic2 = pack2(__float_as_uint(magic), __float_as_uint(magic));
    const uint64_t one2 = pack2(__float_as_uint(args.one), __float_as_uint(args.one));
    const int rl = quarter * 32 + lane;  // the row within the tile
    const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(sub * TPW);
    uint64_t acc[PAIRS][4];  // chain lane j of tokens 2p (low half) and 2p + 1 (high half)
#pragma unroll
    for (int p = 0; p < PAIRS; p++)
#pragma unroll
      for (int j = 0; j < 4; j++) acc[p][j] = 0;
    for (int k = 0; k < kstages; k++) {
      const int st = k % STAGES, slot = k % SLOTS;
      mbar_wait(&s.full[st], (k / STAGES) & 1, args.error, 4);
      const int groups = min(4, ng - 4 * k);
      // the stage's groups' sums of this warp's tokens, then the slot goes back to the MMAs
      mbar_wait(&s.slot_full[slot], (k / SLOTS) & 1, args.error, 5);
      tc_fence_after();
      uint32_t v[4][TPW];
#pragma unroll
      for (int j = 0; j < 4; j++)
        if (j < groups) tmem_ld<TPW>(taddr + (uint32_t)((slot * 4 + j) * BN), v[j]);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.slot_empty[slot]);
      const float4 w4 = *reinterpret_cast<const float4 *>(s.ws[st][rl]);
      const float *xrow = s.xs[st] + sub * TPW;  // group j's scale of this warp's token t: xrow[j * BN + t]
      if (4 * k + 4 <= ng4) {
        // a whole stage below the last four: lane j of the chain takes group 4k + j, two tokens at a time
        const uint32_t wb[4] = {__float_as_uint(w4.x), __float_as_uint(w4.y), __float_as_uint(w4.z),
                                __float_as_uint(w4.w)};
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const uint64_t w2 = pack2(wb[j], wb[j]);
#pragma unroll
          for (int q = 0; q < TPW / 4; q++) {
            const uint4 x4 = *reinterpret_cast<const uint4 *>(xrow + j * BN + 4 * q);
#pragma unroll
            for (int h = 0; h < 2; h++) {
              const int p = 2 * q + h;
              const uint64_t x2 = h ? pack2(x4.z, x4.w) : pack2(x4.x, x4.y);
              // float(S) exactly, times (weight scale x activation scale), rounded once (kernel_relaxed.ts:45,55)
              const uint64_t f2 = sub2(pack2(v[j][2 * p] + magic_bits, v[j][2 * p + 1] + magic_bits), magic2);
              acc[p][j] = fma2(one2, acc[p][j], mul2(f2, mul2(w2, x2)));
            }
          }
        }
      } else {
        // the stage with the groups past the fours (kernel_relaxed.ts:57-64): the lanes added in order first
        const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
        for (int p = 0; p < PAIRS; p++) {
          float r[2];
#pragma unroll
          for (int h = 0; h < 2; h++) {
            const int t = 2 * p + h;
            float a[4];
#pragma unroll
            for (int j = 0; j < 4; j++) a[j] = h ? hi(acc[p][j]) : lo(acc[p][j]);
            float x = __fadd_rn(__fadd_rn(__fadd_rn(a[0], a[1]), a[2]), a[3]);
#pragma unroll
            for (int j = 0; j < 4; j++) {
              if (j < groups) {
                const float f = __fsub_rn(__uint_as_float(v[j][t] + magic_bits), magic);
                x = __fadd_rn(x, __fmul_rn(f, __fmul_rn(wv[j], xrow[j * BN + t])));
              }
            }
            r[h] = x;
          }
          acc[p][0] = pack2(__float_as_uint(r[0]), __float_as_uint(r[1]));
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.empty[st]);
    }
    if (ng4 == ng) {
#pragma unroll
      for (int p = 0; p < PAIRS; p++) {
        const float r0 = __fadd_rn(__fadd_rn(__fadd_rn(lo(acc[p][0]), lo(acc[p][1])), lo(acc[p][2])), lo(acc[p][3]));
        const float r1 = __fadd_rn(__fadd_rn(__fadd_rn(hi(acc[p][0]), hi(acc[p][1])), hi(acc[p][2])), hi(acc[p][3]));
        acc[p][0] = pack2(__float_as_uint(r0), __float_as_uint(r1));
      }
    }
    const int r = row0 + rl;
    if (r < args.rows) {
#pragma unroll
      for (int t = 0; t < TPW; t++) {
        const int tok = tok0 + sub * TPW + t;
        if (tok < args.count) {
          const float x = (t & 1) ? hi(acc[t >> 1][0]) : lo(acc[t >> 1][0]);
          float *o = args.out + (int64_t)tok * args.out_stride + r;
          *o = args.accumulate ? __fadd_rn(*o, x) : x;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
  }
}

#define CHECK_RC(expr)   \
  do {                   \
    int rc_ = (expr);    \
    if (rc_) return rc_; \
  } while (0)

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

}  // namespace

int make_map(CUtensorMap *map, CUtensorMapDataType type, int esize, const void *base, int64_t cols, int64_t rows,
             int64_t row_bytes, int box_cols, int box_rows, CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (!fn) return fail(B200FWD_ECUDA, "cuTensorMapEncodeTiled is not available");
  if (reinterpret_cast<uintptr_t>(base) % 16 || row_bytes % 16)
    return fail(B200FWD_EINVAL, "a TMA tensor must start on, and have rows of, multiples of 16 bytes");
  if (cols < box_cols || rows < box_rows) return fail(B200FWD_EINVAL, "a TMA box larger than its tensor");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = fn(map, type, 2, const_cast<void *>(base), dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(B200FWD_ECUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  (void)esize;
  return 0;
}

int make_i8_map(CUtensorMap *map, const void *base, int64_t cols, int64_t rows, int64_t row_bytes, int box_rows) {
  return make_map(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, base, cols, rows, row_bytes, KSTAGE, box_rows,
                  CU_TENSOR_MAP_SWIZZLE_128B);
}

int make_scale_map(CUtensorMap *map, const float *base, int64_t groups, int64_t rows, int64_t row_floats, int box_rows) {
  return make_map(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, groups, rows, row_floats * 4, 4, box_rows,
                  CU_TENSOR_MAP_SWIZZLE_NONE);
}

int make_token_scale_map(CUtensorMap *map, const float *base, int64_t tokens, int64_t groups, int64_t row_floats,
                         int box_tokens) {
  return make_map(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, tokens, groups, row_floats * 4, box_tokens, 4,
                  CU_TENSOR_MAP_SWIZZLE_NONE);
}

size_t gemm_smem_bytes() { return sizeof(Smem) + 1024; }

int launch_gemm_tc(const GemmMaps &maps, const GemmArgs &given, int bn, cudaStream_t stream) {
  GemmArgs args = given;
  args.magic_bits = MAGIC_BITS;
  args.magic = MAGIC;
  args.one = 1.0f;
  if (args.count <= 0 || args.rows <= 0) return 0;
  if (args.n % 32) return fail(B200FWD_EINVAL, "gemm: n must be whole groups of 32");
  if (bn != 16 && bn != 32) return fail(B200FWD_EINVAL, "gemm: BN must be 16 or 32");
  const size_t smem = gemm_smem_bytes();
  dim3 grid((args.count + bn - 1) / bn, (args.rows + BM - 1) / BM);
  static std::atomic<uint64_t> opted{0};
  int device = 0;
  B200_CUDA(cudaGetDevice(&device));
  const uint64_t bit = device < 64 ? (1ull << device) : 0;
  if (!bit || !(opted.load() & bit)) {
    CHECK_RC(prepare_gemm());
    if (bit) opted.fetch_or(bit);
  }
  if (bn == 16)
    q8_gemm_tc<16><<<grid, THREADS, smem, stream>>>(maps.w, maps.x, maps.ws, maps.xs, args);
  else
    q8_gemm_tc<32><<<grid, THREADS, smem, stream>>>(maps.w, maps.x, maps.ws, maps.xs, args);
  B200_LAUNCHED("q8_gemm_tc");
  return 0;
}

int prepare_gemm() {
  const size_t smem = gemm_smem_bytes();
  B200_CUDA(cudaFuncSetAttribute(q8_gemm_tc<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  B200_CUDA(cudaFuncSetAttribute(q8_gemm_tc<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  return 0;
}

}  // namespace b200
