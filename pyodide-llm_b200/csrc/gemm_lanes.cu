// gemm_lanes.cu — the int8 group-32 matmul (kernel_relaxed.ts:34-67 / 164-183, matmul_q8r and matmul_q8r_tile, to
// the bit) split four ways along K by the reference's own chain lanes, for n a multiple of 128 (no groups past the
// fours).
//
// The reference's number for (row r, token t) is four independent float chains — lane j takes the groups g with
// g % 4 == j, in order: chain_j += float(S_g) x (weight scale x activation scale), each product and sum rounded —
// then ((chain_0 + chain_1) + chain_2) + chain_3. So a tile of 128 rows x BN tokens goes to a cluster of four CTAs,
// CTA j running chain j alone over the groups j, j + 4, j + 8, ...: a quarter of the tile's K per CTA, four times
// the CTAs at work on a matrix of few row tiles, and one accumulator per (row, token) instead of four. In each CTA:
//   - warp 0: TMA brings per stage four "quads" (128-byte K blocks) of lane j's 32-byte group: 128 weight rows x 32
//     bytes and BN tokens x 32 bytes each (32-byte swizzle), the quads' weight scales and lane j's activation scales;
//   - warp 1: per stage, into a TMEM slot of four column blocks (one per quad): the offset MMA (1.5 x 2^23 in every
//     word), one kind::i8 MMA per quad (K = 32: exactly lane j's group), the offset taken off: float(S) exactly;
//   - warps 4..19 (epilogue): copy the slot's four blocks to registers, hand the slot back to the MMAs at once (the
//     next stage's MMAs run while this one is computed), then the chain: per (row, token, group) a scale product, a
//     product and the chain add, on paired float32 operations (two tokens at a time, each rounded on its own).
// At the end of a tile each epilogue warp sends its chain values to the CTA that owns its quarter of the tile's
// tokens (distributed shared memory, an mbarrier arrival with release order), and the owner adds the four lanes in
// the reference's order and writes (or adds into) the output. Tiles go round the clusters; every wait is bounded.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <string>

#include "common.h"
#include "gemm_tc.h"
#include "tcgen05.cuh"

namespace b200 {
namespace {

using namespace tc;

constexpr int BM = 128;
constexpr int LANES = 4;                 // the cluster: a CTA per chain lane
constexpr int EPI_WARPS = 16;
constexpr int EPI_WARP0 = 4;             // warps 0..3: producer, MMA issuer, two idle
constexpr int THREADS = 32 * (EPI_WARP0 + EPI_WARPS);
// registers: 640 x 96 at launch; the first warpgroup gives back all but 32 a thread, the epilogue takes 112
constexpr int REGS_SMALL = 32, REGS_EPILOGUE = 112;
constexpr uint32_t F16_512 = 0x6000u, F16_1536 = 0x6600u, F16_MINUS_1536 = 0xE600u;

template <int BN>
struct LTile {
  static constexpr int STAGES = BN == 64 ? 4 : BN == 32 ? 6 : 7;
  static constexpr int SLOTS = 512 / (4 * BN);  // TMEM holds this many stages' four blocks
  static constexpr int TPW = BN / 4;            // tokens of an epilogue warp (and of a CTA's share of a tile)
};

template <int BN>
struct LSmem {
  static constexpr int STAGES = LTile<BN>::STAGES, TPW = LTile<BN>::TPW;
  alignas(1024) uint8_t a[STAGES][4][BM * 32];  // per quad: 128 weight rows x lane j's 32 bytes (32-byte swizzle)
  alignas(1024) uint8_t b[STAGES][4][BN * 32];  // per quad: the tokens x lane j's 32 bytes
  alignas(128) float ws[STAGES][4][BM][4];      // per quad: the rows' four scales (lane j's at [j])
  alignas(128) float xs[STAGES][4][BN];         // per quad: lane j's group's scale of each token
  alignas(128) uint16_t ka[BM * 16];            // the offset MMAs' constant operands (float16)
  alignas(128) uint16_t kb_plus[4 * BN * 16];
  alignas(128) uint16_t kb_minus[4 * BN * 16];
  alignas(16) float xbuf[2][LANES - 1][BM][TPW];  // the other lanes' chain values of this CTA's tokens
  uint64_t full[STAGES], empty[STAGES];
  uint64_t slot_full[LTile<BN>::SLOTS], slot_empty[LTile<BN>::SLOTS];
  uint64_t xfull[2];
  uint64_t mma_done;
  uint32_t tmem_base;
};

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
// (w - 4) / 4 * TPW .. + TPW as 16x256b fragments of both 16-lane halves, so that thread t keeps chain `rank` of four
// rows (quarter * 32 + t/4 + 8i) x PP = BN / 32 token pairs (8p + 2(t%4), +1 of the warp's TPW): each activation-scale
// pair read from shared memory serves four rows, and a pair's two tokens (adjacent in the fragment) go through each
// float operation together. At the end of a tile the warp hands its values to the same warp of CTA `sub`, which holds
// the same (row, token) pairs of the other chains and adds the four lanes in order.
template <int BN>
__device__ __forceinline__ void lanes_epilogue_4x4(LSmem<BN> &s, uint32_t tmem, int quarter, int sub, int lane,
                                                   int rank, int cid, int ncl, const GemmArgs &args, int tiles,
                                                   int ntok, int kstages, int nquads, float one) {
  constexpr int STAGES = LTile<BN>::STAGES, SLOTS = LTile<BN>::SLOTS, TPW = LTile<BN>::TPW, PP = BN / 32;
  constexpr int NP = 4 * PP;  // the (row, token pair) pairs of a thread: n = i * PP + p
  const int c = lane & 3, rq = lane >> 2;
  const uint32_t t_lo = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(sub * TPW), t_hi = t_lo + (16u << 16);
  const uint64_t one2 = pk2(__float_as_uint(one), __float_as_uint(one));
  Ring<STAGES> ring;
  Ring<SLOTS> slots;
  int iter = 0;
  for (int tile = cid; tile < tiles; tile += ncl, iter++) {
    const int row0 = (tile / ntok) * BM, tok0 = (tile % ntok) * BN;
    uint64_t acc[NP];  // chain `rank` of row rq + 8i, tokens 8p + 2c, +1
#pragma unroll
    for (int n = 0; n < NP; n++) acc[n] = 0;
    for (int k = 0; k < kstages; k++, ring.next(), slots.next()) {
      const int st = ring.i, slot = slots.i;
      mbar_wait(&s.full[st], ring.phase, args.error, 14);
      mbar_wait(&s.slot_full[slot], slots.phase, args.error, 15);
      fence_after();
      uint32_t v[4][2][4 * PP];  // quad, 16-lane half
#pragma unroll
      for (int q = 0; q < 4; q++) {
        tmem_ld_16x256<PP>(t_lo + (uint32_t)((slot * 4 + q) * BN), v[q][0]);
        tmem_ld_16x256<PP>(t_hi + (uint32_t)((slot * 4 + q) * BN), v[q][1]);
      }
      tmem_wait_ld();
      // the slot is in registers: back to the MMAs before the arithmetic
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.slot_empty[slot]);
      const int quads = min(4, nquads - 4 * k);
#pragma unroll
      for (int q = 0; q < 4; q++) {
        if (q < quads) {
          // group 16k + 4q + rank: float(S) x (weight scale x activation scale), rounded once each
          // (kernel_relaxed.ts:45,55), added into the chain
          const float *wq = &s.ws[st][q][quarter * 32 + rq][rank];  // row rq + 8i: wq[32 * i]
          const float *xq = s.xs[st][q] + sub * TPW + 2 * c;       // token pair p: xq[8p], two floats
          uint64_t x2[PP];
#pragma unroll
          for (int p = 0; p < PP; p++) x2[p] = *reinterpret_cast<const uint64_t *>(xq + 8 * p);
#pragma unroll
          for (int i = 0; i < 4; i++) {
            const uint32_t w = __float_as_uint(wq[32 * i]);
            const uint64_t w2 = pk2(w, w);
#pragma unroll
            for (int p = 0; p < PP; p++) {
              const int r = 4 * p + 2 * (i & 1);
              acc[i * PP + p] = fma2(one2, acc[i * PP + p],
                                     mul2(pk2(v[q][i >> 1][r], v[q][i >> 1][r + 1]), mul2(w2, x2[p])));
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.empty[st]);
    }
    // ---- the four chains of this warp's (row, token) pairs meet in the same warp of CTA `sub`: a source's values at
    // [quarter][v4 k][lane] of its slot, four floats (pairs 2k, 2k + 1) each
    const int b = iter & 1;
    if (sub != rank) {
      const int from = rank < sub ? rank : rank - 1;
      const uint32_t dst =
          cluster_map(&s.xbuf[b][from][0][0], (uint32_t)sub) + (uint32_t)(quarter * (NP / 2) * 32 * 16);
#pragma unroll
      for (int k4 = 0; k4 < NP / 2; k4++)
        st_cluster_v4(dst + (uint32_t)((k4 * 32 + lane) * 16), lo_f(acc[2 * k4]), hi_f(acc[2 * k4]),
                      lo_f(acc[2 * k4 + 1]), hi_f(acc[2 * k4 + 1]));
      mbar_arrive_cluster(cluster_map(&s.xfull[b], (uint32_t)sub));
    } else {
      const bool ok = mbar_wait<true>(&s.xfull[b], (iter >> 1) & 1, args.error, 18);
      if (ok) {
#pragma unroll
        for (int k4 = 0; k4 < NP / 2; k4++) {
          float4 o[LANES - 1];
#pragma unroll
          for (int f = 0; f < LANES - 1; f++)
            o[f] = reinterpret_cast<const float4 *>(&s.xbuf[b][f][0][0])[(quarter * (NP / 2) + k4) * 32 + lane];
#pragma unroll
          for (int h = 0; h < 2; h++) {
            const int n = 2 * k4 + h, i = n / PP, p = n % PP;
            const int r = row0 + quarter * 32 + rq + 8 * i;
#pragma unroll
            for (int e = 0; e < 2; e++) {
              const int comp = 2 * h + e;
              float l[LANES];
#pragma unroll
              for (int j = 0; j < LANES; j++) {
                if (j == rank) {
                  l[j] = e ? hi_f(acc[n]) : lo_f(acc[n]);
                } else {
                  const float4 &src = o[j < rank ? j : j - 1];
                  l[j] = comp == 0 ? src.x : comp == 1 ? src.y : comp == 2 ? src.z : src.w;
                }
              }
              // kernel_relaxed.ts:57: ((lane 0 + lane 1) + lane 2) + lane 3
              const float sum = __fadd_rn(__fadd_rn(__fadd_rn(l[0], l[1]), l[2]), l[3]);
              const int tok = tok0 + sub * TPW + 8 * p + 2 * c + e;
              if (r < args.rows && tok < args.count) {
                float *out = args.out + (int64_t)tok * args.out_stride + r;
                *out = args.accumulate ? __fadd_rn(*out, sum) : sum;
              }
            }
          }
        }
      }
    }
  }
}

template <int BN>
__global__ void __cluster_dims__(LANES, 1, 1) __launch_bounds__(THREADS, 1)
    q8_gemm_lanes(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                  const __grid_constant__ CUtensorMap wsmap, const __grid_constant__ CUtensorMap xsmap, GemmArgs args,
                  float one) {
  using T = LTile<BN>;
  constexpr int STAGES = T::STAGES, SLOTS = T::SLOTS, TPW = T::TPW;
  pdl_launch_dependents();
  extern __shared__ uint8_t raw[];
  LSmem<BN> &s = *reinterpret_cast<LSmem<BN> *>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = (int)cluster_rank();  // the chain lane of this CTA
  const int cid = (int)cluster_id_x(), ncl = (int)nclusters_x();
  const int nquads = args.n >> 7;
  const int kstages = (nquads + 3) >> 2;
  const int ntok = (args.count + BN - 1) / BN;
  const int tiles = ntok * ((args.rows + BM - 1) / BM);

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
      mbar_init(&s.empty[i], EPI_WARPS);  // every epilogue warp done with the stage's scales (the MMAs are, by then)
    }
    for (int i = 0; i < SLOTS; i++) {
      mbar_init(&s.slot_full[i], 1);
      mbar_init(&s.slot_empty[i], EPI_WARPS);
    }
    // a tile's chain values from the three other CTAs: their four warps (one per row quarter) of this CTA's tokens
    for (int i = 0; i < 2; i++) mbar_init(&s.xfull[i], (LANES - 1) * 4 * 32);
    mbar_init(&s.mma_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // TMEM: 512 columns, the whole of this SM's (one block per SM)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&s.tmem_base)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  cluster_sync();  // every CTA's barriers are initialized before any arrives on them from another CTA
  // the set-up above touches no global memory; the kernel before this one has completed from here on
  pdl_wait();
  const uint32_t tmem = s.tmem_base;

  if (warp < EPI_WARP0) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REGS_SMALL));
    if (warp == 0) {
      // ---- producer: each stage's four quads of weights and activations and both scale tiles on one barrier
      if (lane == 0) {
        constexpr uint32_t bytes = 4 * BM * 32 + 4 * BN * 32 + 4 * BM * 16 + 4 * BN * 4;
        uint32_t kk = 0;
        Ring<STAGES> ring;
        bool ok = true;
        for (int tile = cid; ok && tile < tiles; tile += ncl) {
          const int wy = args.w_row0 + (tile / ntok) * BM, tok0 = (tile % ntok) * BN;
          for (int k = 0; k < kstages; k++, kk++, ring.next()) {
            const int st = ring.i;
            if (!mbar_wait(&s.empty[st], ring.phase ^ 1, args.error, 11)) {
              ok = false;
              break;
            }
            mbar_expect_tx(&s.full[st], bytes);
            tma_load_3d(s.a[st], &wmap, &s.full[st], 32 * rank, wy, 4 * k);
            tma_load_3d(s.b[st], &xmap, &s.full[st], 32 * rank, tok0, 4 * k);
            tma_load_3d(s.ws[st], &wsmap, &s.full[st], 0, wy, 4 * k);
            tma_load_3d(s.xs[st], &xsmap, &s.full[st], tok0, rank, 4 * k);
          }
        }
        // no copy may still be landing when the block ends: wait (bounded) for the last stages issued
        for (uint32_t i = kk > (uint32_t)STAGES ? kk - STAGES : 0; i < kk; i++)
          mbar_wait(&s.full[i % STAGES], (i / STAGES) & 1, args.error, 16);
      }
    } else if (warp == 1) {
      // ---- MMA issue, per stage: the offset into the slot's four blocks, one i8 MMA per quad, the offset off
      const uint32_t id_i8 = idesc_i8(BM, BN), id_f16 = idesc_f16(BM, 4 * BN);
      const uint64_t ka = desc_const(s.ka), kplus = desc_const(s.kb_plus), kminus = desc_const(s.kb_minus);
      Ring<STAGES> ring;
      Ring<SLOTS> slots;
      bool ok = true;
      for (int tile = cid; ok && tile < tiles; tile += ncl) {
        for (int k = 0; k < kstages; k++, ring.next(), slots.next()) {
          const int st = ring.i, slot = slots.i;
          if (!mbar_wait(&s.full[st], ring.phase, args.error, 12) ||
              !mbar_wait(&s.slot_empty[slot], slots.phase ^ 1, args.error, 13)) {
            ok = false;
            break;
          }
          fence_after();
          if (lane == 0) {
            const uint32_t d = tmem + (uint32_t)(slot * 4 * BN);
            const int quads = min(4, nquads - 4 * k);
            mma_f16(d, ka, kplus, id_f16, 0);  // 1.5 * 2^23 in every word of the slot
            for (int q = 0; q < quads; q++)
              mma_i8(d + (uint32_t)(q * BN), desc_sw32(s.a[st][q]), desc_sw32(s.b[st][q]), id_i8, 1);
            mma_f16(d, ka, kminus, id_f16, 1);  // less 1.5 * 2^23: float(S)
            mma_commit(&s.slot_full[slot]);
          }
          __syncwarp();
        }
      }
      if (lane == 0) mma_commit(&s.mma_done);
      __syncwarp();
      mbar_wait(&s.mma_done, 0, args.error, 17);
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REGS_EPILOGUE));
    // ---- epilogue: warp (quarter, sub) reads TMEM lanes quarter * 32.. (its rows) and tokens sub * TPW.. + TPW
    const int quarter = warp % 4, sub = (warp - EPI_WARP0) / 4;
    if constexpr (BN >= 32) {
      lanes_epilogue_4x4<BN>(s, tmem, quarter, sub, lane, rank, cid, ncl, args, tiles, ntok, kstages, nquads, one);
    } else {
      const int rl = quarter * 32 + lane;
      const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(sub * TPW);
      const uint64_t one2 = pk2(__float_as_uint(one), __float_as_uint(one));
      Ring<STAGES> ring;
      Ring<SLOTS> slots;
      int iter = 0;
      for (int tile = cid; tile < tiles; tile += ncl, iter++) {
        const int row0 = (tile / ntok) * BM, tok0 = (tile % ntok) * BN;
        uint64_t acc[TPW / 2];  // chain `rank` of tokens 2p, 2p + 1
#pragma unroll
        for (int p = 0; p < TPW / 2; p++) acc[p] = 0;
        for (int k = 0; k < kstages; k++, ring.next(), slots.next()) {
          const int st = ring.i, slot = slots.i;
          mbar_wait(&s.full[st], ring.phase, args.error, 14);
          mbar_wait(&s.slot_full[slot], slots.phase, args.error, 15);
          fence_after();
          uint32_t v[4][TPW];
#pragma unroll
          for (int q = 0; q < 4; q++) tmem_ld<TPW>(taddr + (uint32_t)((slot * 4 + q) * BN), v[q]);
          tmem_wait_ld();
          // the slot is in registers: back to the MMAs before the arithmetic
          fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s.slot_empty[slot]);
          const int quads = min(4, nquads - 4 * k);
#pragma unroll
          for (int q = 0; q < 4; q++) {
            if (q < quads) {
              // group 16k + 4q + rank: float(S) x (weight scale x activation scale), rounded once each
              // (kernel_relaxed.ts:45,55), added into the chain
              const uint32_t w = __float_as_uint(s.ws[st][q][rl][rank]);
              const uint64_t w2 = pk2(w, w);
              const float *xrow = s.xs[st][q] + sub * TPW;
#pragma unroll
              for (int p4 = 0; p4 < TPW / 4; p4++) {
                const uint4 x4 = *reinterpret_cast<const uint4 *>(xrow + 4 * p4);
                acc[2 * p4] = fma2(one2, acc[2 * p4],
                                   mul2(pk2(v[q][4 * p4], v[q][4 * p4 + 1]), mul2(w2, pk2(x4.x, x4.y))));
                acc[2 * p4 + 1] = fma2(one2, acc[2 * p4 + 1],
                                       mul2(pk2(v[q][4 * p4 + 2], v[q][4 * p4 + 3]), mul2(w2, pk2(x4.z, x4.w))));
              }
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&s.empty[st]);
        }
        // ---- the four chains of this warp's (row, token) pairs meet in CTA `sub`
        const int b = iter & 1;
        if (sub != rank) {
          const int from = rank < sub ? rank : rank - 1;
          const uint32_t dst = cluster_map(&s.xbuf[b][from][rl][0], (uint32_t)sub);
#pragma unroll
          for (int p4 = 0; p4 < TPW / 4; p4++)
            st_cluster_v4(dst + 16 * p4, lo_f(acc[2 * p4]), hi_f(acc[2 * p4]), lo_f(acc[2 * p4 + 1]),
                          hi_f(acc[2 * p4 + 1]));
          mbar_arrive_cluster(cluster_map(&s.xfull[b], (uint32_t)sub));
        } else {
          const bool ok = mbar_wait<true>(&s.xfull[b], (iter >> 1) & 1, args.error, 18);
          const int r = row0 + rl;
          if (ok && r < args.rows) {
#pragma unroll
            for (int t = 0; t < TPW; t++) {
              const int tok = tok0 + sub * TPW + t;
              const float mine = (t & 1) ? hi_f(acc[t >> 1]) : lo_f(acc[t >> 1]);
              float l[LANES];
#pragma unroll
              for (int j = 0; j < LANES; j++)
                l[j] = j == rank ? mine : s.xbuf[b][j < rank ? j : j - 1][rl][t];
              // kernel_relaxed.ts:57: ((lane 0 + lane 1) + lane 2) + lane 3
              const float sum = __fadd_rn(__fadd_rn(__fadd_rn(l[0], l[1]), l[2]), l[3]);
              if (tok < args.count) {
                float *o = args.out + (int64_t)tok * args.out_stride + r;
                *o = args.accumulate ? __fadd_rn(*o, sum) : sum;
              }
            }
          }
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while another may still write its shared memory
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
  }
}

template <int BN>
size_t lanes_smem_bytes() {
  return sizeof(LSmem<BN>) + 1024;
}

// per device (bit d): the kernels' opt-in done; the clusters of each width that fit at once
std::atomic<uint64_t> lanes_opted{0};
int lanes_clusters[64][3];

PFN_cuTensorMapEncodeTiled_v12000 encode3_fn() {
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

int make_map3(CUtensorMap *map, CUtensorMapDataType type, const void *base, const uint64_t dims[3],
              const uint64_t strides[2], const uint32_t box[3], CUtensorMapSwizzle swizzle) {
  auto fn = encode3_fn();
  if (!fn) return fail(B200FWD_ECUDA, "cuTensorMapEncodeTiled is not available");
  if (reinterpret_cast<uintptr_t>(base) % 16 || strides[0] % 16 || strides[1] % 16)
    return fail(B200FWD_EINVAL, "a TMA tensor must start on, and step by, multiples of 16 bytes");
  for (int i = 0; i < 3; i++)
    if (dims[i] < box[i]) return fail(B200FWD_EINVAL, "a TMA box larger than its tensor");
  cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  cuuint64_t st[2] = {strides[0], strides[1]};
  cuuint32_t bx[3] = {box[0], box[1], box[2]};
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult r = fn(map, type, 3, const_cast<void *>(base), d, st, bx, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(B200FWD_ECUDA, "cuTensorMapEncodeTiled (3-D) failed: " + std::to_string((int)r));
  return 0;
}

template <int BN>
int opt_in_lanes(int device) {
  B200_CUDA(cudaFuncSetAttribute(q8_gemm_lanes<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)lanes_smem_bytes<BN>()));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(LANES * 64);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = lanes_smem_bytes<BN>();
  int n = 0;
  B200_CUDA(cudaOccupancyMaxActiveClusters(&n, q8_gemm_lanes<BN>, &cfg));
  lanes_clusters[device][BN == 16 ? 0 : BN == 32 ? 1 : 2] = n;
  return 0;
}

}  // namespace

int make_lane_weight_maps(CUtensorMap *wmap, CUtensorMap *smap, const void *w, const float *s, int64_t n,
                          int64_t rows, int64_t sstride) {
  if (n % 128) return fail(B200FWD_EINVAL, "lane maps: n must be whole quads of 128");
  // weights [rows][n]: dims (byte of a quad, row, quad), boxes of 32 bytes x 128 rows x 4 quads, 32-byte swizzle
  const uint64_t wd[3] = {128, (uint64_t)rows, (uint64_t)(n / 128)};
  const uint64_t wst[2] = {(uint64_t)n, 128};
  const uint32_t wb[3] = {32, BM, 4};
  int rc = make_map3(wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, wd, wst, wb, CU_TENSOR_MAP_SWIZZLE_32B);
  if (rc) return rc;
  // scales [rows][sstride floats]: dims (scale of a quad, row, quad), boxes of 4 x 128 rows x 4 quads
  const uint64_t sd[3] = {4, (uint64_t)rows, (uint64_t)(sstride / 4)};
  const uint64_t sst[2] = {(uint64_t)sstride * 4, 16};
  const uint32_t sb[3] = {4, BM, 4};
  return make_map3(smap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, s, sd, sst, sb, CU_TENSOR_MAP_SWIZZLE_NONE);
}

int make_lane_token_maps(CUtensorMap *xmap, CUtensorMap *xsmap, const int8_t *xq, const float *xs, int64_t tokens,
                         int64_t row_bytes, int64_t k, int64_t tp, int bn) {
  if (k % 128 || row_bytes < k || tp % 4) return fail(B200FWD_EINVAL, "lane maps: activations of whole quads");
  // activations [tokens][row_bytes], k of them used: dims (byte of a quad, token, quad), boxes of 32 bytes x bn
  // tokens x 4 quads
  const uint64_t xd[3] = {128, (uint64_t)tokens, (uint64_t)(k / 128)};
  const uint64_t xst[2] = {(uint64_t)row_bytes, 128};
  const uint32_t xb[3] = {32, (uint32_t)bn, 4};
  int rc = make_map3(xmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, xq, xd, xst, xb, CU_TENSOR_MAP_SWIZZLE_32B);
  if (rc) return rc;
  // activation scales [k / 32 groups][tp tokens] (one row per group): dims (token, lane, quad), boxes of bn x 1 x 4
  const uint64_t sd[3] = {(uint64_t)tokens, 4, (uint64_t)(k / 128)};
  const uint64_t sst[2] = {(uint64_t)tp * 4, (uint64_t)tp * 16};
  const uint32_t sb[3] = {(uint32_t)bn, 1, 4};
  return make_map3(xsmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, xs, sd, sst, sb, CU_TENSOR_MAP_SWIZZLE_NONE);
}

int prepare_gemm_lanes() {
  int device = 0;
  B200_CUDA(cudaGetDevice(&device));
  if (device < 0 || device >= 64) return fail(B200FWD_EUNSUPPORTED, "gemm lanes: device index past 63");
  if (lanes_opted.load() & (1ull << device)) return 0;
  int rc = opt_in_lanes<16>(device);
  if (!rc) rc = opt_in_lanes<32>(device);
  if (!rc) rc = opt_in_lanes<64>(device);
  if (rc) return rc;
  lanes_opted.fetch_or(1ull << device);
  return 0;
}

bool gemm_lanes_fits(int n, int rows, int count) {
  // whole quads, and at least four stages a tile (the exchange buffers' reuse two tiles later is ordered by the
  // stages in between); a whole 128-row box
  return n % 128 == 0 && n / 128 >= 16 && rows >= BM && count > 0;
}

// time of a stage of one lane (four quads of K) by tile width, in hundredths of a microsecond at 1965 MHz, and the
// kernel's fixed cost: measured on the 8B shapes
constexpr int LANES_STAGE_CUS[3] = {81, 96, 140};
constexpr int LANES_FIXED_CUS = 300;

bool gemm_lanes_pays(int rows, int count, int n, int sms, int widest) {
  // B200FWD_GEMM_LANES=2 takes the lane-split kernel wherever it fits (a tuning knob for measurements)
  static const bool forced = [] {
    const char *v = getenv("B200FWD_GEMM_LANES");
    return v && v[0] == '2';
  }();
  if (forced) return true;
  // a cluster of four CTAs takes a tile at a time: rounds of tiles over the clusters, a quarter of K's stages each
  const int lbn = choose_lanes_bn(count, widest);
  const int64_t tiles = (int64_t)((rows + BM - 1) / BM) * ((count + lbn - 1) / lbn);
  const int64_t clusters = std::max(1, sms / LANES);
  const int64_t lanes = (tiles + clusters - 1) / clusters * ((n / 128 + 3) / 4) *
                            LANES_STAGE_CUS[lbn == 16 ? 0 : lbn == 32 ? 1 : 2] +
                        LANES_FIXED_CUS;
  const int bn = choose_gemm_bn(rows, count, sms, widest);
  return lanes < gemm_tc_cost(rows, count, n, sms, bn);
}

int choose_lanes_bn(int count, int widest) {
  const int bn = count <= 16 ? 16 : count <= 32 ? 32 : 64;
  return bn <= widest ? bn : widest;
}

bool gemm_lanes_enabled() {
  static const bool on = [] {
    const char *v = getenv("B200FWD_GEMM_LANES");
    return !(v && v[0] == '0');
  }();
  return on;
}

int launch_gemm_lanes(const GemmMaps &maps, const GemmArgs &args, int bn, cudaStream_t stream) {
  if (args.count <= 0 || args.rows <= 0) return 0;
  if (!gemm_lanes_fits(args.n, args.rows, args.count)) return fail(B200FWD_EINVAL, "gemm lanes: unsupported shape");
  if (bn != 16 && bn != 32 && bn != 64) return fail(B200FWD_EINVAL, "gemm lanes: BN must be 16, 32 or 64");
  int rc = prepare_gemm_lanes();
  if (rc) return rc;
  int device = 0;
  B200_CUDA(cudaGetDevice(&device));
  const int fit = lanes_clusters[device][bn == 16 ? 0 : bn == 32 ? 1 : 2];
  if (fit <= 0) return fail(B200FWD_EUNSUPPORTED, "gemm lanes: no cluster of four fits");
  const int64_t tiles = (int64_t)((args.rows + BM - 1) / BM) * ((args.count + bn - 1) / bn);
  const dim3 grid((unsigned)(LANES * std::min<int64_t>(tiles, fit)));
#define B200_LANES_LAUNCH(W) \
  launch(q8_gemm_lanes<W>, grid, THREADS, lanes_smem_bytes<W>(), stream, maps.w, maps.x, maps.ws, maps.xs, args, 1.0f)
  if (bn == 16)
    B200_LANES_LAUNCH(16);
  else if (bn == 32)
    B200_LANES_LAUNCH(32);
  else
    B200_LANES_LAUNCH(64);
#undef B200_LANES_LAUNCH
  B200_LAUNCHED("q8_gemm_lanes");
  return 0;
}

}  // namespace b200
