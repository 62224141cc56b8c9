// tcgen05 / TMA / mbarrier primitives shared by the tensor-core kernels (sm_100a).
#pragma once

#include <cuda.h>

#include "sb_device.cuh"

namespace sb {
namespace tc5 {

// shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms 1024 B apart
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;                 // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;       // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                 // descriptor version (sm100)
  d |= (uint64_t)2 << 61;                 // 128-byte swizzle
  return d;
}

// instruction descriptor of kind::f16 with bf16 A and B, fp32 D, K-major both, M=128, N=n
__device__ __forceinline__ uint32_t idesc_bf16(uint32_t n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((128u >> 4) << 24);
}

// the same with f16 A and B
__device__ __forceinline__ uint32_t idesc_f16(uint32_t n) {
  return (1u << 4) | ((n >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem, uint64_t ad, uint64_t bd, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
      "l"(ad), "l"(bd), "r"(id), "r"(acc));
}

__device__ __forceinline__ void commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// TMA tensor load of a 2-D box at (c0, c1), completing on an mbarrier (no multicast)
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 32 consecutive TMEM columns of this warp's 32 lanes; completion is awaited separately
__device__ __forceinline__ void ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }

__device__ __forceinline__ void arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}

// one lane of a converged warp
__device__ __forceinline__ bool elect_one() {
  uint32_t p;
  asm volatile("{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n selp.u32 %0, 1, 0, e;\n}\n" : "=r"(p));
  return p != 0;
}

// OR of `pred` over the `count` threads of named barrier `id`
__device__ __forceinline__ bool bar_any(uint32_t id, uint32_t count, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n barrier.red.or.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}

// Bounded mbarrier wait of a CTA with an abort flag in shared memory: up to 256 polls without a
// suspend hint first, then (for limits of 256 and more) `limit` polls with one; on timeout it sets
// *err and the abort flag and returns false. It returns false early once another role has set the
// abort flag. PROBE (the kernel variant of the timeout-path test) makes `limit` non-blocking probes.
template <bool PROBE = false>
__device__ __forceinline__ bool wait_bounded(volatile int* abort_flag, int* err, uint32_t bar, uint32_t parity,
                                             uint32_t limit) {
  if constexpr (PROBE) {
#pragma unroll 1
    for (uint32_t i = 0; i < limit; ++i)
      if (mbar_test_wait(bar, parity)) return true;
    atomicExch(err, 1);
    *abort_flag = 1;
    return false;
  }
  for (uint32_t i = 0; i < 256u && i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  for (uint32_t i = 0; limit >= 256u && i < limit; ++i) {
    if (mbar_try_wait_sleep(bar, parity, 1000u)) return true;
    if ((i & 63u) == 63u && *abort_flag) return false;
  }
  atomicExch(err, 1);
  *abort_flag = 1;
  return false;
}

}  // namespace tc5
}  // namespace sb
