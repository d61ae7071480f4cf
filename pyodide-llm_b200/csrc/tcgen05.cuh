// tcgen05.cuh — the sm_100a building blocks the tensor-core matmuls share: mbarriers with bounded waits, TMA tile
// loads, shared-memory matrix descriptors, tcgen05.mma / commit / ld, and the cluster (distributed shared memory)
// operations of the lane-split matmul.
#pragma once

#include <cuda.h>
#include <cstdint>

namespace b200 {
namespace tc {

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
// (the error word is then set and every later wait returns soon: the kernel runs to its end and frees TMEM).
// try_wait with a suspend-time hint: a waiting warp sleeps until the phase completes or the hint's 1 ms passes; the
// error word (global memory) is read only then, and after WAIT_TRIES such expiries (about 2 s) the wait gives up.
// acquire.cluster: writes another CTA of the cluster made before its release-arrive are visible after the wait.
template <bool CLUSTER = false>
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *error, int code) {
  const uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0;; i++) {
    uint32_t done;
    if (CLUSTER)
      asm volatile(
          "{\n\t.reg .pred p;\n\t"
          "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
          "selp.u32 %0, 1, 0, p;\n\t}"
          : "=r"(done)
          : "r"(addr), "r"(parity), "r"(WAIT_HINT_NS)
          : "memory");
    else
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
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// tcgen05 shared-memory matrix descriptor, K-major, 128-byte swizzle: 8-row atoms of 128-byte rows, 1024 bytes apart
__device__ __forceinline__ uint64_t desc_sw128(const void *p) {
  const uint64_t addr = smem_u32(p);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3fff;         // start address
  d |= (uint64_t)1 << 16;            // leading byte offset (unused for swizzled K-major): 16 bytes
  d |= (uint64_t)(1024 >> 4) << 32;  // stride byte offset: 8 rows of 128 bytes
  d |= (uint64_t)1 << 46;            // version (Blackwell)
  d |= (uint64_t)2 << 61;            // SWIZZLE_128B
  return d;
}
// K-major, 32-byte swizzle: rows of 32 bytes (one K block of int8), 8-row atoms 256 bytes apart
__device__ __forceinline__ uint64_t desc_sw32(const void *p) {
  const uint64_t addr = smem_u32(p);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3fff;
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(256 >> 4) << 32;   // stride byte offset: 8 rows of 32 bytes
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)6 << 61;            // SWIZZLE_32B
  return d;
}
// descriptor of a constant operand (every element the same value): K-major, no swizzle, 8 x 16-byte core matrices
// 128 bytes apart along K and 256 bytes apart along M/N. (Whatever order the hardware walks them in, it reads
// inside the buffer and sees the one value.)
__device__ __forceinline__ uint64_t desc_const(const void *p) {
  const uint64_t addr = smem_u32(p);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3fff;
  d |= (uint64_t)(128 >> 4) << 16;
  d |= (uint64_t)(256 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}

// instruction descriptor: kind::i8, D int32, A and B signed int8, both K-major, M = m, N = n
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
  return (2u << 4)                         // D format: S32
         | (1u << 7) | (1u << 10)          // A, B: signed 8-bit
         | ((uint32_t)(n >> 3) << 17)      // N >> 3
         | ((uint32_t)(m >> 4) << 24);     // M >> 4
}
// instruction descriptor: kind::f16, D float32, A and B float16, both K-major, M = m, N = n
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
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
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// N consecutive TMEM columns of this warp's 32 lanes, not waited for (tmem_wait_ld before use)
template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[N]);
template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
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

// 16 TMEM lanes x 8PP columns (PP 256-bit repetitions) from lane taddr.lane, not waited for: thread t holds lane t/4
// in r[4p], r[4p + 1] (columns 8p + 2(t%4), +1) and lane t/4 + 8 in r[4p + 2], r[4p + 3] (the same columns)
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

// ---- clusters: this CTA's rank, another CTA's shared memory, arrivals on another CTA's mbarrier
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t nclusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// the shared::cluster address of this CTA's shared variable at `p` in the CTA of rank `rank`
__device__ __forceinline__ uint32_t cluster_map(const void *p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}
// one arrival on the mbarrier at `addr` (a shared::cluster address), ordered after this thread's earlier writes
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

}  // namespace tc
}  // namespace b200
