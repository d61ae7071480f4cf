// gemm_tc.cu — the int8 group-32 matmul of a prompt block or of many sequences' tokens on the 5th-generation tensor
// cores: kernel_relaxed.ts:34-67 / 164-183 (matmul_q8r, matmul_q8r_tile) for two tokens and more, to the bit.
//
// The reference's number for (row r, token t) is a float chain over the row's groups of 32: each group's exact
// integer dot(w, q - 64), as float32, times (weight scale x activation scale), rounded once, added into lane g % 4
// for the groups below the last four, the lanes added ((0 + 1) + 2) + 3, then the groups past the fours one at a
// time. Here, in a persistent kernel (one block per SM walking tiles of 128 weight rows x BN tokens):
//   - warp 0: TMA brings 128 weight rows x 128 bytes (four groups), BN tokens' activations x 128 bytes and both
//     scale tiles per stage into shared memory, several stages deep (128-byte swizzle; no multicast);
//   - warp 1: one thread issues, per stage, into a TMEM slot of four column blocks (128 lanes = rows, BN columns =
//     tokens, one block per group): a kind::f16 MMA whose constant operands (512 x 1536, sixteen times) write
//     1.5 * 2^23 into all four blocks; one kind::i8 MMA per group (K = 32: exactly one group) that adds the
//     group's int32 sums to those words as integers, giving the bit patterns of the floats 1.5 * 2^23 + S; and a
//     second kind::f16 MMA (512 x -1536) that takes 1.5 * 2^23 off again in float32. Every step is exact (integers
//     below 2^24 throughout), so TMEM ends up holding float(S) of every (row, token, group), none added to another;
//   - warps 4..19 (epilogue): four per TMEM lane quarter, each with BN / 4 tokens, read their groups' floats
//     (tcgen05.ld) and keep the reference's four chain accumulators of each (row, token) in registers, with one
//     rounding per float operation (__fmul_rn / __fadd_rn, built with --fmad=false): per (row, token, group) a
//     scale product, a product and a chain add.
// Every mbarrier wait has an iteration limit: past it the kernel records an error and returns (no hang).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdlib>
#include <cstdint>
#include <cstring>
#include <string>

#include "common.h"
#include "gemm_tc.h"

namespace b200 {
namespace {

constexpr int BM = 128;                 // rows of a tile (TMEM lanes)
constexpr int KSTAGE = 128;             // bytes of K per stage: four groups
constexpr int EPI_WARPS = 16;
constexpr int EPI_WARP0 = 4;  // warps 0..3 (one warpgroup): the producer, the MMA issuer and two idle warps
constexpr int THREADS = 32 * (EPI_WARP0 + EPI_WARPS);
// registers per thread: THREADS x 96 at launch; the first warpgroup gives back all but 32 a thread and the four
// epilogue warpgroups take 112 (128 x 32 + 512 x 112 = 640 x 96: the launch's whole share)
constexpr int REGS_SMALL = 32, REGS_EPILOGUE = 112;
constexpr uint32_t WAIT_HINT_NS = 1000000;  // 1 ms
constexpr uint32_t WAIT_TRIES = 2000;

// f16 bit patterns of the constant operands of the offset MMAs: 16 x 512 x 1536 = 12582912 = 1.5 * 2^23
constexpr uint32_t F16_512 = 0x6000u, F16_1536 = 0x6600u, F16_MINUS_1536 = 0xE600u;

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

// descriptor of a constant operand (every element the same value): K-major, no swizzle, 8 x 16-byte core matrices
// 128 bytes apart along K and 256 bytes apart along M/N. (Whatever order the hardware walks them in, it reads
// inside the buffer and sees the one value.)
__device__ __forceinline__ uint64_t const_desc(const void *p) {
  const uint64_t addr = smem_u32(p);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3fff;
  d |= (uint64_t)(128 >> 4) << 16;
  d |= (uint64_t)(256 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}

// instruction descriptor: kind::i8, D int32, A and B signed int8, both K-major, M = 128, N = n
__host__ __device__ constexpr uint32_t idesc_i8(int n) {
  return (2u << 4)                         // D format: S32
         | (1u << 7) | (1u << 10)          // A, B: signed 8-bit
         | ((uint32_t)(n >> 3) << 17)      // N >> 3
         | ((uint32_t)(BM >> 4) << 24);    // M >> 4
}
// instruction descriptor: kind::f16, D float32, A and B float16, both K-major, M = 128, N = n
__host__ __device__ constexpr uint32_t idesc_f16(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, int acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, int acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

template <int BN>
struct Tile {
  static constexpr int STAGES = BN == 64 ? 7 : 8;
  static constexpr int SLOTS = 512 / (4 * BN);  // TMEM holds this many stages' four groups at once
  static constexpr int TPW = BN / 4;            // tokens of an epilogue warp
  static constexpr int GB = BN == 64 ? 1 : 4;   // groups whose sums an epilogue warp loads from TMEM at once
};

// a position in a ring of N buffers and the parity of its current round (advanced by one at a time: no division)
template <int N>
struct Ring {
  int i = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void next() {
    if (++i == N) {
      i = 0;
      phase ^= 1;
    }
  }
};

template <int BN>
struct Smem {
  static constexpr int STAGES = Tile<BN>::STAGES;
  alignas(1024) uint8_t a[STAGES][BM * KSTAGE];       // 128 weight rows x four groups
  alignas(1024) uint8_t b[STAGES][BN * KSTAGE];       // the tokens x four groups
  alignas(128) float ws[STAGES][BM][4];               // the rows' four groups' scales
  alignas(128) float xs[STAGES][4 * BN];              // the tokens' scales: four rows (groups) of BN tokens
  alignas(128) uint16_t ka[BM * 16];                  // the offset MMAs' constant operands (float16)
  alignas(128) uint16_t kb_plus[4 * BN * 16];
  alignas(128) uint16_t kb_minus[4 * BN * 16];
  uint64_t full[STAGES], empty[STAGES];
  uint64_t slot_full[Tile<BN>::SLOTS], slot_empty[Tile<BN>::SLOTS];
  uint64_t mma_done;
  uint32_t tmem_base;
};

// TPW consecutive TMEM columns (the tokens of this warp) of its 32 lanes (tiles of 16 tokens)
template <int TPW>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[TPW]);
template <>
__device__ __forceinline__ void tmem_ld<4>(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}

// 16 TMEM lanes x 8PP columns (PP 256-bit repetitions) from lane taddr.lane: thread t holds lane t/4 in r[4p], r[4p + 1]
// (columns 8p + 2(t%4), +1) and lane t/4 + 8 in r[4p + 2], r[4p + 3] (the same columns)
template <int PP>
__device__ __forceinline__ void tmem_ld_16x256(uint32_t taddr, uint32_t (&r)[4 * PP]);
template <>
__device__ __forceinline__ void tmem_ld_16x256<2>(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x2.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_ld_16x256<1>(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x1.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}
// the loads issued so far have landed; r (the last one's registers) is read only after this
template <int PP>
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[4 * PP]);
template <>
__device__ __forceinline__ void tmem_wait_ld<2>(uint32_t (&r)[8]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7])
               :
               : "memory");
}
template <>
__device__ __forceinline__ void tmem_wait_ld<1>(uint32_t (&r)[4]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]) : : "memory");
}

__device__ __forceinline__ uint64_t pk2(uint32_t lo, uint32_t hi) { return (uint64_t)lo | ((uint64_t)hi << 32); }
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// one * a + b rounded once, one = 1.0f handed over at run time: a + b, and no product can be folded into the add
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ float lo_f(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float hi_f(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }

// The epilogue of 64- and 32-token tiles. Epilogue warp w reads TMEM lane quarter w % 4 and token columns
// (w - 4) / 4 * TPW .. + TPW as 16x256b fragments of both 16-lane halves, so that thread t keeps four rows
// (quarter * 32 + t/4 + 8i) x PP = BN / 32 token pairs (8p + 2(t%4), +1 of the warp's TPW). Each activation-scale pair
// a thread reads from shared memory then serves four rows (against one with a thread a row), and the two tokens of a
// pair, adjacent in the fragment, go through each float operation together (.f32x2: each half rounded on its own, as
// the scalar operation rounds it): half the shared-memory reads of scales and half the float instructions. The
// arithmetic per (row, token, group) and its order are those of the general epilogue below.
template <int BN, bool TAIL>
__device__ __forceinline__ void epilogue_4x4(Smem<BN> &s, uint32_t tmem, int quarter, int sub, int lane,
                                             const GemmArgs &args, int tiles, int ntok, int kstages, int ng, int ng4,
                                             float one) {
  constexpr int STAGES = Tile<BN>::STAGES, SLOTS = Tile<BN>::SLOTS, TPW = Tile<BN>::TPW, PP = BN / 32;
  const int c = lane & 3, rq = lane >> 2;
  const uint32_t t_lo = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(sub * TPW), t_hi = t_lo + (16u << 16);
  const uint64_t one2 = pk2(__float_as_uint(one), __float_as_uint(one));
  Ring<STAGES> ring;
  Ring<SLOTS> slots;
  for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const int row0 = (tile / ntok) * BM, tok0 = (tile % ntok) * BN;
    uint64_t acc[4][PP][4];  // [row rq + 8i][token pair p][chain lane j]
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int p = 0; p < PP; p++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][p][j] = 0;
    for (int k = 0; k < kstages; k++, ring.next(), slots.next()) {
      const int st = ring.i, slot = slots.i;
      mbar_wait(&s.full[st], ring.phase, args.error, 4);
      const int groups = TAIL ? min(4, ng - 4 * k) : 4;
      mbar_wait(&s.slot_full[slot], slots.phase, args.error, 5);
      tc_fence_after();
      const float *wq = &s.ws[st][quarter * 32 + rq][0];  // row rq + 8i's group j: wq[32 * i + j]
      const float *xq = s.xs[st] + sub * TPW + 2 * c;      // group j's token pair p: xq[j * BN + 8 * p], two floats
      if (!TAIL || 4 * k + 4 <= ng4) {
        // four whole groups. Step q = 2j + h works on group j's half h (rows rq + 8i, i = 2h, 2h + 1): it waits for
        // its own TMEM load, issues the next step's, then computes, so that each load lands during a step's work.
        // Row rq + 8i, pair p: fragment registers 4p + 2(i & 1), +1.
        uint32_t v[2][4 * PP];
        uint32_t wv[4];
        uint64_t x2[PP];
        tmem_ld_16x256<PP>(t_lo + (uint32_t)(slot * 4 * BN), v[0]);
#pragma unroll
        for (int q = 0; q < 8; q++) {
          const int j = q >> 1, h = q & 1;
          tmem_wait_ld<PP>(v[q & 1]);
          if (q < 7)
            tmem_ld_16x256<PP>(((q + 1) & 1 ? t_hi : t_lo) + (uint32_t)((slot * 4 + ((q + 1) >> 1)) * BN),
                              v[(q + 1) & 1]);
          if (h == 0) {
#pragma unroll
            for (int p = 0; p < PP; p++) x2[p] = *reinterpret_cast<const uint64_t *>(xq + j * BN + 8 * p);
#pragma unroll
            for (int i = 0; i < 4; i++) wv[i] = __float_as_uint(wq[32 * i + j]);
          }
          // lane j of the chain takes group 4k + j: float(S) x (weight scale x activation scale), rounded once each
          // (kernel_relaxed.ts:45,55), added into the lane
#pragma unroll
          for (int ii = 0; ii < 2; ii++) {
            const int i = 2 * h + ii;
#pragma unroll
            for (int p = 0; p < PP; p++) {
              const int r = 4 * p + 2 * ii;
              const uint64_t sums = pk2(v[q & 1][r], v[q & 1][r + 1]);
              acc[i][p][j] = fma2(one2, acc[i][p][j], mul2(sums, mul2(pk2(wv[i], wv[i]), x2[p])));
            }
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < 4; j++) {
          uint32_t v[2][4 * PP];  // the two 16-lane halves' fragments
          uint32_t wv[4];
          uint64_t x2[PP];
          if (j < groups) {
            const uint32_t col = (uint32_t)((slot * 4 + j) * BN);
            tmem_ld_16x256<PP>(t_lo + col, v[0]);
            tmem_ld_16x256<PP>(t_hi + col, v[1]);
#pragma unroll
            for (int p = 0; p < PP; p++) x2[p] = *reinterpret_cast<const uint64_t *>(xq + j * BN + 8 * p);
#pragma unroll
            for (int i = 0; i < 4; i++) wv[i] = __float_as_uint(wq[32 * i + j]);
            tmem_wait_ld();
          }
          // the stage of the groups past the fours (kernel_relaxed.ts:57-64): the lanes added in order first (kept in
          // lane 0), then each group in turn
#pragma unroll
          for (int i = 0; i < 4; i++)
#pragma unroll
            for (int p = 0; p < PP; p++) {
              float x[2];
#pragma unroll
              for (int e = 0; e < 2; e++) {
                auto part = [&](int l) { return e ? hi_f(acc[i][p][l]) : lo_f(acc[i][p][l]); };
                x[e] = j == 0 ? __fadd_rn(__fadd_rn(__fadd_rn(part(0), part(1)), part(2)), part(3)) : part(0);
                if (j < groups) {
                  const float sum = __uint_as_float(v[i >> 1][4 * p + 2 * (i & 1) + e]);
                  const float xs = e ? hi_f(x2[p]) : lo_f(x2[p]);
                  x[e] = __fadd_rn(x[e], __fmul_rn(sum, __fmul_rn(__uint_as_float(wv[i]), xs)));
                }
              }
              acc[i][p][0] = pk2(__float_as_uint(x[0]), __float_as_uint(x[1]));
            }
        }
      }
      // the slot goes back to the MMAs, the stage's shared memory to the producer
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s.slot_empty[slot]);
        mbar_arrive(&s.empty[st]);
      }
    }
    if (!TAIL) {
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int p = 0; p < PP; p++)
          acc[i][p][0] = fma2(one2, fma2(one2, fma2(one2, acc[i][p][0], acc[i][p][1]), acc[i][p][2]), acc[i][p][3]);
    }
    // each store writes eight consecutive rows of four tokens (four 32-byte pieces)
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int r = row0 + quarter * 32 + rq + 8 * i;
      if (r >= args.rows) continue;
#pragma unroll
      for (int p = 0; p < PP; p++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
          const int tok = tok0 + sub * TPW + 8 * p + 2 * c + e;
          if (tok < args.count) {
            const float sum = e ? hi_f(acc[i][p][0]) : lo_f(acc[i][p][0]);
            float *o = args.out + (int64_t)tok * args.out_stride + r;
            *o = args.accumulate ? __fadd_rn(*o, sum) : sum;
          }
        }
    }
  }
}

// Warp roles: 0 TMA producer, 1 MMA issue, 2 and 3 idle, 4..19 epilogue. Epilogue warp w reads TMEM lane quarter
// w % 4 (its 32 rows) and token columns (w - 4) / 4 * TPW .. + TPW (64- and 32-token tiles: epilogue_4x4 above), and keeps the
// reference's four chain accumulators of each of its (row, token) in registers: the chains, their sum and the groups
// past the fours all happen in one thread. Tiles go round the blocks (tile = block, block + grid, ...): consecutive
// tiles share their weight rows, so blocks that run together read each weight row once from HBM.
// TAIL: n / 32 is not a multiple of four (groups past the fours); without it every stage is four whole groups
template <int BN, bool TAIL>
__global__ void __launch_bounds__(THREADS, 1)
    q8_gemm_tc(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
               const __grid_constant__ CUtensorMap wsmap, const __grid_constant__ CUtensorMap xsmap, GemmArgs args,
               float one) {
  using T = Tile<BN>;
  constexpr int STAGES = T::STAGES, SLOTS = T::SLOTS, TPW = T::TPW, GB = T::GB;
  pdl_launch_dependents();
  extern __shared__ uint8_t raw[];
  Smem<BN> &s = *reinterpret_cast<Smem<BN> *>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ng = args.n >> 5, ng4 = ng & ~3;
  const int kstages = (args.n + KSTAGE - 1) / KSTAGE;
  const int ntok = (args.count + BN - 1) / BN;
  const int tiles = ntok * ((args.rows + BM - 1) / BM);

  // the offset MMAs' constant operands, written through the generic proxy and made visible to the tensor cores
  for (int i = threadIdx.x; i < BM * 16 / 2; i += THREADS)
    reinterpret_cast<uint32_t *>(s.ka)[i] = F16_512 | (F16_512 << 16);
  for (int i = threadIdx.x; i < 4 * BN * 16 / 2; i += THREADS) {
    reinterpret_cast<uint32_t *>(s.kb_plus)[i] = F16_1536 | (F16_1536 << 16);
    reinterpret_cast<uint32_t *>(s.kb_minus)[i] = F16_MINUS_1536 | (F16_MINUS_1536 << 16);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
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
    mbar_init(&s.mma_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // TMEM: 512 columns, the whole of this SM's (one block per SM)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&s.tmem_base)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // the set-up above touches no global memory; the kernel before this one (the activations' producer, or the
  // residual's writer) has completed from here on
  pdl_wait();
  const uint32_t tmem = s.tmem_base;

  if (warp < EPI_WARP0) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REGS_SMALL));
  if (warp == 0) {
    // ---- producer: each stage's weights, activations and both scale tiles on one barrier
    if (lane == 0) {
      constexpr uint32_t bytes = BM * KSTAGE + BN * KSTAGE + BM * 16 + BN * 16;
      uint32_t kk = 0;
      Ring<STAGES> ring;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
        const int wy = args.w_row0 + (tile / ntok) * BM, tok0 = (tile % ntok) * BN;
        for (int k = 0; k < kstages; k++, kk++, ring.next()) {
          const int st = ring.i;
          if (!mbar_wait(&s.empty[st], ring.phase ^ 1, args.error, 1)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&s.full[st], bytes);
          tma_load_2d(s.a[st], &wmap, &s.full[st], k * KSTAGE, wy);
          tma_load_2d(s.b[st], &xmap, &s.full[st], k * KSTAGE, tok0);
          tma_load_2d(s.ws[st], &wsmap, &s.full[st], k * 4, wy);
          tma_load_2d(s.xs[st], &xsmap, &s.full[st], tok0, k * 4);
        }
      }
      // no copy may still be landing when the block ends: wait (bounded) for the last stages issued
      for (uint32_t i = kk > (uint32_t)STAGES ? kk - STAGES : 0; i < kk; i++)
        mbar_wait(&s.full[i % STAGES], (i / STAGES) & 1, args.error, 6);
    }
  } else if (warp == 1) {
    // ---- MMA issue, per stage: the offset into the stage's slot (four column blocks), one i8 MMA per group on top
    // of it, the offset taken off, one commit. A slot is free once every epilogue warp has read it.
    const uint32_t id_i8 = idesc_i8(BN), id_f16 = idesc_f16(4 * BN);
    const uint64_t ka = const_desc(s.ka), kplus = const_desc(s.kb_plus), kminus = const_desc(s.kb_minus);
    Ring<STAGES> ring;
    Ring<SLOTS> slots;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
      for (int k = 0; k < kstages; k++, ring.next(), slots.next()) {
        const int st = ring.i, slot = slots.i;
        if (!mbar_wait(&s.full[st], ring.phase, args.error, 2) ||
            !mbar_wait(&s.slot_empty[slot], slots.phase ^ 1, args.error, 3)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t d = tmem + (uint32_t)(slot * 4 * BN);
          const int groups = min(4, ng - 4 * k);
          mma_f16(d, ka, kplus, id_f16, 0);  // 1.5 * 2^23 in every word of the slot
          for (int j = 0; j < groups; j++)
            mma_i8(d + (uint32_t)(j * BN), smem_desc(s.a[st] + 32 * j), smem_desc(s.b[st] + 32 * j), id_i8, 1);
          mma_f16(d, ka, kminus, id_f16, 1);  // less 1.5 * 2^23: float(S)
          mma_commit(&s.slot_full[slot]);
        }
        __syncwarp();
      }
    }
    // every MMA issued has completed before the block frees TMEM
    if (lane == 0) mma_commit(&s.mma_done);
    __syncwarp();
    mbar_wait(&s.mma_done, 0, args.error, 7);
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REGS_EPILOGUE));
    // ---- epilogue
    const int quarter = warp % 4, sub = (warp - EPI_WARP0) / 4;
    if constexpr (BN >= 32) {
      epilogue_4x4<BN, TAIL>(s, tmem, quarter, sub, lane, args, tiles, ntok, kstages, ng, ng4, one);
    } else {
      const int rl = quarter * 32 + lane;  // the row within the tile
      const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(sub * TPW);
      Ring<STAGES> ring;
      Ring<SLOTS> slots;
      for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
        const int row0 = (tile / ntok) * BM, tok0 = (tile % ntok) * BN;
        float acc[TPW][4];  // chain lane j of token t
#pragma unroll
        for (int t = 0; t < TPW; t++)
#pragma unroll
          for (int j = 0; j < 4; j++) acc[t][j] = 0.f;
        for (int k = 0; k < kstages; k++, ring.next(), slots.next()) {
          const int st = ring.i, slot = slots.i;
          mbar_wait(&s.full[st], ring.phase, args.error, 4);
          const int groups = TAIL ? min(4, ng - 4 * k) : 4;
          mbar_wait(&s.slot_full[slot], slots.phase, args.error, 5);
          tc_fence_after();
          const float4 w4 = *reinterpret_cast<const float4 *>(s.ws[st][rl]);
          const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
          const float *xrow = s.xs[st] + sub * TPW;  // group j's scale of this warp's token t: xrow[j * BN + t]
          const bool whole = !TAIL || 4 * k + 4 <= ng4;
#pragma unroll
          for (int j0 = 0; j0 < 4; j0 += GB) {
            uint32_t v[GB][TPW];
#pragma unroll
            for (int jj = 0; jj < GB; jj++)
              if (j0 + jj < groups) tmem_ld<TPW>(taddr + (uint32_t)((slot * 4 + j0 + jj) * BN), v[jj]);
            tmem_wait_ld();
            if (whole) {
              // lane j of the chain takes group 4k + j: float(S) x (weight scale x activation scale), rounded once
              // each (kernel_relaxed.ts:45,55), added into the lane
#pragma unroll
              for (int jj = 0; jj < GB; jj++) {
                const int j = j0 + jj;
#pragma unroll
                for (int q = 0; q < TPW / 4; q++) {
                  const float4 x4 = *reinterpret_cast<const float4 *>(xrow + j * BN + 4 * q);
                  const float xv[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
                  for (int h = 0; h < 4; h++) {
                    const int t = 4 * q + h;
                    acc[t][j] = __fadd_rn(acc[t][j], __fmul_rn(__uint_as_float(v[jj][t]), __fmul_rn(wv[j], xv[h])));
                  }
                }
              }
            } else {
              // the stage of the groups past the fours (kernel_relaxed.ts:57-64): the lanes added in order first
              // (kept in acc[t][0]), then each group in turn
#pragma unroll
              for (int t = 0; t < TPW; t++) {
                float x = j0 == 0 ? __fadd_rn(__fadd_rn(__fadd_rn(acc[t][0], acc[t][1]), acc[t][2]), acc[t][3])
                                  : acc[t][0];
#pragma unroll
                for (int jj = 0; jj < GB; jj++) {
                  const int j = j0 + jj;
                  if (j < groups)
                    x = __fadd_rn(x, __fmul_rn(__uint_as_float(v[jj][t]), __fmul_rn(wv[j], xrow[j * BN + t])));
                }
                acc[t][0] = x;
              }
            }
          }
          // the slot goes back to the MMAs, the stage's shared memory to the producer
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&s.slot_empty[slot]);
            mbar_arrive(&s.empty[st]);
          }
        }
        if (!TAIL) {
#pragma unroll
          for (int t = 0; t < TPW; t++)
            acc[t][0] = __fadd_rn(__fadd_rn(__fadd_rn(acc[t][0], acc[t][1]), acc[t][2]), acc[t][3]);
        }
        const int r = row0 + rl;
        if (r < args.rows) {
#pragma unroll
          for (int t = 0; t < TPW; t++) {
            const int tok = tok0 + sub * TPW + t;
            if (tok < args.count) {
              float *o = args.out + (int64_t)tok * args.out_stride + r;
              *o = args.accumulate ? __fadd_rn(*o, acc[t][0]) : acc[t][0];
            }
          }
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

template <int BN>
size_t smem_bytes() {
  return sizeof(Smem<BN>) + 1024;
}

// per device (bit d): the kernels' shared-memory opt-in done, and the SM count
std::atomic<uint64_t> opted{0};
int sm_counts[64];

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

size_t gemm_smem_bytes() { return smem_bytes<64>(); }

int gemm_sms() {
  int device = 0;
  B200_CUDA(cudaGetDevice(&device));
  if (device < 0 || device >= 64) return 148;
  if (!(opted.load() & (1ull << device))) CHECK_RC(prepare_gemm());
  return sm_counts[device];
}

// time of a stage (128 K bytes of a tile) by tile width, in hundredths of a microsecond at 1965 MHz: measured on the
// 8B shapes with one tile per SM (16: the general epilogue; 32 and 64: epilogue_4x4)
constexpr int TC_STAGE_CUS[3] = {73, 88, 92};

int64_t gemm_tc_cost(int rows, int count, int n, int sms, int bn) {
  const int64_t tiles = (int64_t)((rows + BM - 1) / BM) * ((count + bn - 1) / bn);
  const int64_t rounds = (tiles + sms - 1) / sms;  // a block walks ceil(tiles / SMs) tiles
  return rounds * ((n + KSTAGE - 1) / KSTAGE) * TC_STAGE_CUS[bn == 16 ? 0 : bn == 32 ? 1 : 2];
}

int choose_gemm_bn(int rows, int count, int sms, int widest) {
  // B200FWD_GEMM_BN=16|32|64 fixes the width (a tuning knob for measurements; within what the token maps allow)
  static const int fixed = [] {
    const char *v = getenv("B200FWD_GEMM_BN");
    const int b = v ? atoi(v) : 0;
    return b == 16 || b == 32 || b == 64 ? b : 0;
  }();
  if (fixed && fixed <= widest && (fixed == 16 || fixed / 2 < count)) return fixed;
  // the width of the least estimated time, up to the first that holds every token in one tile (a wider tile costs
  // little more a stage than a narrower one: its rows of tokens are computed whether or not they exist)
  int best = 16;
  int64_t best_cost = INT64_MAX;
  for (int bn = 16; bn <= widest; bn *= 2) {
    if (bn > 16 && bn / 2 >= count) break;
    const int64_t cost = gemm_tc_cost(rows, count, KSTAGE, sms, bn);
    if (cost < best_cost) {
      best = bn;
      best_cost = cost;
    }
  }
  return best;
}

int launch_gemm_tc(const GemmMaps &maps, const GemmArgs &given, int bn, cudaStream_t stream) {
  const GemmArgs &args = given;
  if (args.count <= 0 || args.rows <= 0) return 0;
  if (args.n % 32) return fail(B200FWD_EINVAL, "gemm: n must be whole groups of 32");
  if (bn != 16 && bn != 32 && bn != 64) return fail(B200FWD_EINVAL, "gemm: BN must be 16, 32 or 64");
  const int sms = gemm_sms();
  if (sms <= 0) return sms < 0 ? sms : fail(B200FWD_ECUDA, "gemm: no SM count");
  const int64_t tiles = (int64_t)((args.rows + BM - 1) / BM) * ((args.count + bn - 1) / bn);
  const dim3 grid((unsigned)std::min<int64_t>(tiles, sms));
  const bool tail = (args.n / 32) % 4 != 0;
#define B200_GEMM_LAUNCH(W, T) \
  launch(q8_gemm_tc<W, T>, grid, THREADS, smem_bytes<W>(), stream, maps.w, maps.x, maps.ws, maps.xs, args, 1.0f)
  if (bn == 16)
    tail ? B200_GEMM_LAUNCH(16, true) : B200_GEMM_LAUNCH(16, false);
  else if (bn == 32)
    tail ? B200_GEMM_LAUNCH(32, true) : B200_GEMM_LAUNCH(32, false);
  else
    tail ? B200_GEMM_LAUNCH(64, true) : B200_GEMM_LAUNCH(64, false);
#undef B200_GEMM_LAUNCH
  B200_LAUNCHED("q8_gemm_tc");
  return 0;
}

int prepare_gemm() {
  int device = 0;
  B200_CUDA(cudaGetDevice(&device));
#define B200_GEMM_OPT_IN(W, T) \
  B200_CUDA(cudaFuncSetAttribute(q8_gemm_tc<W, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes<W>()))
  B200_GEMM_OPT_IN(16, false);
  B200_GEMM_OPT_IN(16, true);
  B200_GEMM_OPT_IN(32, false);
  B200_GEMM_OPT_IN(32, true);
  B200_GEMM_OPT_IN(64, false);
  B200_GEMM_OPT_IN(64, true);
#undef B200_GEMM_OPT_IN
  if (device >= 0 && device < 64) {
    int sms = 0;
    B200_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
    sm_counts[device] = sms;
    opted.fetch_or(1ull << device);
  }
  return 0;
}

}  // namespace b200
