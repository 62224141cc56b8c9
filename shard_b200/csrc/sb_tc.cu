// Grouped expert GEMV/GEMM on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// One CTA walks ITEMS = (expert or shared expert, 128-row block of a weight matrix) of the
// device-side permutation (shared expert first), round-robin or, when the launch has an item
// counter, taking the next item as it gets to it (the producer fetches and hands each item to the
// other roles through a small shared-memory queue); an item runs its expert's token PASSES (up to 16
// B rows each) over the K stages (128 K per stage). Roles (192 threads):
//   warp 4     producer: lane 0 keeps up to ST stages of asynchronous copies in flight. A stage is
//                - the weight tile, 128 rows x 128 K, by a TMA tensor load that lands it directly
//                  in the 128B-swizzled K-major operand form tcgen05.mma reads: fp4 weights use the
//                  16U4_ALIGN16B element type (each 16 packed e2m1 values land in the low 8 bytes
//                  of a 16-byte slot, the form kind::f8f6f4 reads e2m1 in), FP8 weights are bytes;
//                - the pass's B tile (16 rows x 128 B e4m3, pre-swizzled by the panel kernel) and
//                  its 16 row scales, by plain bulk copies;
//                - the weight scales of the stage (NVFP4 8 B / MXFP4 4 B per row, FP8 two fp32).
//   warp 5     MMA issuer: allocates TMEM; lane 0 issues tcgen05.mma (M=128, N=16, K=32) and
//              tcgen05.commit. fp4 weights: one fresh 16-column TMEM slot per 32-K chunk (their
//              per-16 / per-32 scales are applied at readback); FP8: the stage's 4 chunks
//              accumulate into one slot (one 128x128 block scale per stage).
//   warps 0-3  readback: thread r owns weight row r (TMEM lane r); per stage it loads the used
//              columns with tcgen05.ld, applies the weight scales and the B row scales in fp32 and
//              accumulates; then the epilogue (W13: SwiGLU pairs rows r / r+64 -> h bf16; W2 /
//              DENSE: bf16 rows of o).
// The three roles run decoupled through mbarriers across item and pass boundaries. An operand slot
// (weight tile + B tile) is released by tcgen05.commit as soon as its MMAs have read it, so the
// ring holds only copies in flight and tiles waiting for the tensor core; the small per-stage
// scales live in a deeper side ring released by the readback. The MMA issuer runs ahead of the
// readback by up to SA accumulator groups.
// The tensor core sums exact products (e2m1 x e4m3 and e4m3 x e4m3 are exact in fp32).
//
// Every wait is bounded: on timeout the CTA records an error in *err and winds down.
#include <cudaTypedefs.h>

#include "sb_device.cuh"
#include "sb_launch.h"

namespace sb {
namespace tc {

constexpr int NTHREADS = 192;
constexpr int PRODUCER_WARP = 4;
constexpr int MMA_WARP = 5;
constexpr int ST = 5;           // operand ring (weight tile + B tile), released by the MMA commit
constexpr int UNIT = 2;         // stages per unit (one accumulator group, side slot and readback)
constexpr int SA = 2;           // accumulator groups (units) in TMEM
constexpr int SS = 6;           // side ring (scales of a unit), released by the readback
constexpr int NB = 16;          // MMA N (columns per chunk slot)
constexpr int SCOLS = 4 * NB;   // TMEM columns of one stage (4 chunk slots)
constexpr int GCOLS = UNIT * SCOLS;  // TMEM columns of one accumulator group
constexpr int TMEM_COLS = SA * GCOLS;
constexpr int A_BYTES = 128 * 128;
constexpr int B_BYTES = NB * 128;
constexpr int SCL_BYTES = 1024;
constexpr uint32_t WAIT_LIMIT = 1u << 16;  // polls; each may sleep up to ~1 us

constexpr int SF_SRC = 512;      // one scale-factor copy source: 32 rows x 16 B
constexpr int SF_A_COL = 64;     // block-scaled items: TMEM columns of the group holding the weight
constexpr int SF_B_COL = 68;     // and activation scale factors (the accumulator is columns 0-15)

// One item: (expert or shared expert / dense matrix, 128-row block, pass), and its K range.
struct Item {
  int shared, expert, rb, cnt, base, pb, pass;
  int ks, kn, j0, j1;   // piece ks of kn, stages [j0, j1)
};
constexpr int IQ = 4;           // dynamic schedule: items queued from the producer to the other roles

struct Smem {
  uint8_t A[ST][A_BYTES];       // 1024-aligned (128B swizzle atoms)
  uint8_t B[ST][B_BYTES];
  uint8_t sfa[ST][SF_SRC];      // block-scaled FP8 items: the stage's weight scale factors
  uint8_t sfb[ST][SF_SRC];      // block-scaled items: the stage's activation scale factors
  uint8_t scl[SS][UNIT * SCL_BYTES];
  float asc[SS][UNIT * NB];
  uint64_t full[ST], aempty[ST], sfull[SS], sempty[SS], gfull[SA], gempty[SA];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int klast;                    // K pieces: this CTA's piece was the last of its block to finish
  Item iq[IQ];                  // dynamic schedule: the producer's items in order (pass < 0: the end)
  uint64_t iqfull[IQ], iqempty[IQ];
  __nv_bfloat16 xchg[64][18];   // W13 epilogue: the up rows' bf16 values
};
constexpr int SMEM_BYTES = (int)sizeof(Smem) + 1024;
static_assert(2 * (SMEM_BYTES + 1024) <= 233472, "two CTAs per SM (1 KB reserved per CTA)");

__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;                 // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;       // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                 // descriptor version (sm100)
  d |= (uint64_t)2 << 61;                 // 128-byte swizzle
  return d;
}

// kind::f8f6f4, D fp32, A format afmt (0 e4m3, 5 e2m1), B e4m3, K-major both, M=128, N=NB
__device__ __forceinline__ uint32_t idesc(uint32_t afmt) {
  return (1u << 4) | (afmt << 7) | (0u << 10) | ((uint32_t)(NB >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void mma(uint32_t tmem, uint64_t ad, uint64_t bd, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
      "l"(ad), "l"(bd), "r"(id), "r"(acc));
}

// Block-scaled MMA (kind::mxf8f6f4.block_scale, one ue8m0 scale per 32 K for A and for B): the
// instruction descriptor names the A format (0 e4m3, 5 e2m1), B e4m3, M=128, N=NB, E8M0 scale
// factors, and which byte (32-K block kb of the stage) of the scale-factor words both operands use.
__device__ __forceinline__ uint32_t idesc_bs(uint32_t afmt, uint32_t kb) {
  return (kb << 4) | (afmt << 7) | (0u << 10) | ((uint32_t)(NB >> 3) << 17) | (1u << 23) | ((128u >> 4) << 24) |
         (kb << 29);
}

// sfa / sfb: TMEM addresses of the scale factors, the byte within their 32-bit columns in bits 30-31
__device__ __forceinline__ void mma_bs(uint32_t tmem, uint64_t ad, uint64_t bd, uint32_t id, uint32_t sfa, uint32_t sfb,
                                       uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n}\n" ::"r"(tmem),
      "l"(ad), "l"(bd), "r"(id), "r"(acc), "r"(sfa), "r"(sfb));
}

// Scale factors of 128 rows into TMEM: a 32-row x 16-byte shared-memory source (row i = the four
// scale words of rows i, 32 + i, 64 + i, 96 + i) lands in lane i of every 32-lane sub-partition,
// columns taddr .. taddr + 3 (column c = rows 32c + i, byte b = 32-K block b).
__device__ __forceinline__ void cp_sf(uint32_t taddr, uint32_t src) {
  uint64_t d = 0;
  d |= (uint64_t)((src >> 4) & 0x3FFFu);
  d |= (uint64_t)(128 >> 4) << 16;       // leading byte offset (one core matrix along K: unused)
  d |= (uint64_t)(128 >> 4) << 32;       // stride byte offset: 8 rows x 16 B core matrices
  d |= (uint64_t)1 << 46;                // descriptor version (sm100); no swizzle
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;\n" ::"r"(taddr), "l"(d) : "memory");
}

// a power-of-two fp32 scale as its e8m0 byte (0 -> 2^-127, only for empty activation rows)
__device__ __forceinline__ uint32_t e8m0_of(float v) { return (__float_as_uint(v) >> 23) & 0xFFu; }

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

// 16 / 4 consecutive TMEM columns of this warp's 32 lanes; completion is awaited separately
__device__ __forceinline__ void ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void ld4(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}
__device__ __forceinline__ void ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }

__device__ __forceinline__ void arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool aborted(Smem& sm) { return *reinterpret_cast<volatile int*>(&sm.abort) != 0; }

__device__ __forceinline__ void set_abort(Smem& sm, int* err, bool flag_err) {
  if (flag_err) atomicExch(err, 1);
  *reinterpret_cast<volatile int*>(&sm.abort) = 1;
}

// bounded wait; on timeout flag the CTA (and the launch) and return false. `limit` polls: up to 256
// without a suspend hint first (most waits end within a few hundred cycles), then `limit` polls that
// may each sleep up to ~1 us. PROBE (the kernel variant of the timeout-path test, launched only when
// a test wait limit is set) makes `limit` non-blocking probes instead, so a phase not complete at
// that moment runs the wait out; the production variant compiles only the polling loops.
template <bool PROBE = false>
__device__ __forceinline__ bool wait(Smem& sm, int* err, uint32_t bar, uint32_t parity, uint32_t limit = WAIT_LIMIT) {
  if constexpr (PROBE) {
#pragma unroll 1
    for (uint32_t i = 0; i < limit; ++i)
      if (mbar_test_wait(bar, parity)) return true;
    set_abort(sm, err, true);
    return false;
  }
  for (uint32_t i = 0; i < 256u && i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  for (uint32_t i = 0; limit >= 256u && i < limit; ++i) {
    if (mbar_try_wait_sleep(bar, parity, 1000u)) return true;
    if ((i & 63u) == 63u && aborted(sm)) return false;
  }
  set_abort(sm, err, true);
  return false;
}

// bounded wait by a whole warp; true only if every lane saw the phase complete (reconverges the warp)
template <bool PROBE = false>
__device__ __forceinline__ bool warp_wait(Smem& sm, int* err, uint32_t bar, uint32_t parity,
                                          uint32_t limit = WAIT_LIMIT) {
  const bool ok = wait<PROBE>(sm, err, bar, parity, limit);
  return __all_sync(0xffffffffu, ok);
}

// one lane of a converged warp (the issuing lane of the producer and MMA warps)
__device__ __forceinline__ bool elect_one() {
  uint32_t p;
  asm volatile("{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n selp.u32 %0, 1, 0, e;\n}\n" : "=r"(p));
  return p != 0;
}

// OR of `pred` over the 128 worker threads, on named barrier 1 (a uniform decision for all of them)
__device__ __forceinline__ bool workers_any(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n barrier.red.or.pred q, 1, 128, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)pred)
      : "memory");
  return r != 0;
}

// An ITEM is one pass (up to 16 B rows of one expert's tokens) over one 128-row block of a weight
// matrix. Items are numbered pass-major: item = pass * nrb + rb, passes being the shared expert's
// (or the dense matrix's) first, then each active expert's in slot order, so a hot expert's passes
// run on different CTAs at about the same time and share its weight tiles through L2.
// K pieces. The dense matrix's items (the shared-expert slot of the item space) may be split along
// K into ksplit pieces of kstages stages: item = (pass, row block, piece), numbered piece-minor, any
// routed items following unsplit. Each piece writes its fp32 partial accumulator to the workspace
// and counts itself in; the last piece of a (pass, row block) to finish sums the pieces in K order
// and runs the epilogue. This occupies the GPU when a dense matrix has few row blocks.

template <int FMT_R>
__device__ __forceinline__ Item item_of(const GroupedArgs& a, const TcPlan& plan, int item, int nrb, int nst) {
  Item it;
  it.ks = 0;
  it.kn = 1;
  it.j0 = 0;
  it.j1 = nst;
  if (a.ksplit > 1) {
    const int nsh = plan.n_sh_pass * nrb;   // shared items before the split
    if (item < nsh * a.ksplit) {
      it.kn = a.ksplit;
      it.ks = item % a.ksplit;
      item /= a.ksplit;
      it.j0 = it.ks * a.kstages;
      it.j1 = min(nst, it.j0 + a.kstages);
    } else {
      item -= nsh * (a.ksplit - 1);
    }
  }
  const int p = item / nrb;
  it.rb = item - p * nrb;
  it.pass = p;
  if (p < plan.n_sh_pass) {
    it.shared = 1;
    it.expert = 0;
    it.cnt = a.m;
    it.base = 0;
    it.pb = p * tc_pass_max(a.mode == MODE_DENSE ? FMT_R : FMT_FP8);
  } else {
    const int q = p - plan.n_sh_pass;
    const int slot = plan.pass_slot[q];
    it.shared = 0;
    it.pb = plan.pass_pb[q];
    it.expert = a.active[slot];
    it.cnt = a.counts[it.expert];
    it.base = a.offsets[it.expert];
  }
  return it;
}

__host__ __device__ inline int stage_sbytes(int fmt) { return fmt == FMT_NVFP4 ? 1024 : (fmt == FMT_MXFP4 ? 512 : 16); }

// error flag of launches without a workspace
__device__ int g_tc_dense_err = 0;

struct TcArgs {
  CUtensorMap map_routed;   // weights of the routed bank (or unused)
  CUtensorMap map_shared;   // weights of the shared expert / dense matrix
  GroupedArgs g;
  TcPlan plan;
};

// DYN: the items come from the launch's item counter (a separate instantiation, so the round-robin
// kernel compiles without the queue)
template <int FMT_R, bool PROBE, bool DYN>
__global__ void __launch_bounds__(NTHREADS, 2) tc_grouped_kernel(const __grid_constant__ TcArgs ta) {
  const GroupedArgs& a = ta.g;
  extern __shared__ uint8_t dyn_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(dyn_raw) + 1023) & ~(uintptr_t)1023);
  int* err = a.err != nullptr ? a.err : &g_tc_dense_err;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;

  if (tid == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(smem_addr(&sm.full[s]), 1);
      mbar_init(smem_addr(&sm.aempty[s]), 1);
    }
    for (int s = 0; s < SS; ++s) {
      mbar_init(smem_addr(&sm.sfull[s]), 1);
      mbar_init(smem_addr(&sm.sempty[s]), 4);
    }
    for (int q = 0; q < SA; ++q) {
      mbar_init(smem_addr(&sm.gfull[q]), 1);
      mbar_init(smem_addr(&sm.gempty[q]), 4);
    }
    for (int q = 0; q < IQ; ++q) {
      mbar_init(smem_addr(&sm.iqfull[q]), 1);
      mbar_init(smem_addr(&sm.iqempty[q]), 5);   // the MMA warp and the 4 readback warps
    }
    mbar_init(smem_addr(&sm.drain), 1);
    sm.abort = 0;
    mbar_init_fence();
  }
  if (warp == MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_addr(&sm.tmem_base)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tbase = sm.tmem_base;
  // everything above touched only this CTA's shared memory and TMEM; the inputs come after
  pdl_wait();
  pdl_trigger();

  const int P = a.m * a.topk;
  const int K = a.k;
  const int nst = K / 128;
  const int nrb = a.n_rows / 128;
  const int n_pass = (a.has_shared ? ta.plan.n_sh_pass : 0) +
                     (a.mode == MODE_DENSE ? 0 : ta.plan.pass_off[*a.n_active]);
  const int n_items = n_pass * nrb + (a.ksplit > 1 && a.has_shared ? ta.plan.n_sh_pass * nrb * (a.ksplit - 1) : 0);
  const bool w13 = a.mode == MODE_W13;
  constexpr bool dyn = DYN;   // items from the launch-wide counter (zeroed by the panel kernel)
  // the limit of the consumer-side waits (the MMA issuer's and the readback's); the producer's waits
  // for free slots and the final drains keep WAIT_LIMIT
  const uint32_t clim = a.wait_limit ? a.wait_limit : WAIT_LIMIT;

  // per-item constants shared by the roles
  auto item_fmt = [&](const Item& it) { return it.shared ? (a.mode == MODE_DENSE ? FMT_R : FMT_FP8) : FMT_R; };
  // items whose weights and activations both carry power-of-two scales run block-scaled
  auto block_scaled = [&](int fmt) { return ((a.bs_mask >> fmt) & 1) != 0; };

  // Stages are grouped in UNITS of up to UNIT consecutive stages of one pass: one side-ring slot
  // (scales), one accumulator group and one readback per unit. g counts stages, u units.
  if (warp == PRODUCER_WARP) {
    // the whole warp runs the loop (uniform control flow); one elected lane issues the copies
    if (elect_one()) {
      prefetch_map(&ta.map_routed);
      prefetch_map(&ta.map_shared);
    }
    __syncwarp();
    uint32_t g = 0, u = 0, qn = 0;
    bool ok = true;
    // Items come from a launch-wide counter when the launch has one (each CTA takes the next item as
    // it gets to it, so CTAs that drew heavier items take fewer), else round-robin. The next item's
    // index and descriptor are fetched one item ahead, so their global loads overlap this item.
    auto fetch = [&]() -> int {
      int v = 0;
      if (lane == 0) v = atomicAdd(a.sched, 1);
      return __shfl_sync(0xffffffffu, v, 0);
    };
    int item = dyn ? fetch() : (int)blockIdx.x;
    Item nxt = item < n_items ? item_of<FMT_R>(a, ta.plan, item, nrb, nst) : Item{};
    while (ok) {
      if (dyn) {
        // publish the item (or the end) to the MMA issuer and the readback
        const uint32_t qs = qn % IQ;
        if (!warp_wait(sm, err, smem_addr(&sm.iqempty[qs]), ((qn / IQ) & 1u) ^ 1u)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          Item e = nxt;
          if (item >= n_items) e.pass = -1;
          sm.iq[qs] = e;
          arrive(smem_addr(&sm.iqfull[qs]));
        }
        __syncwarp();
        ++qn;
      }
      if (item >= n_items) break;
      const Item it = nxt;
      const int next = dyn ? fetch() : item + (int)gridDim.x;
      if (next < n_items) nxt = item_of<FMT_R>(a, ta.plan, next, nrb, nst);
      item = next;
      const int fmt = item_fmt(it);
      const WeightSet& ws = it.shared ? a.shared : a.routed;
      const CUtensorMap* map = it.shared ? &ta.map_shared : &ta.map_routed;
      const uint32_t abytes = fmt == FMT_FP8 ? 16384u : 8192u;
      const uint32_t sb = stage_sbytes(fmt);
      const int row0 = ((it.shared ? 0 : it.expert) * nrb + it.rb) * nst * 128;
      const uint8_t* sbase = ws.s + (it.shared ? 0 : (size_t)it.expert * ws.s_stride) + (size_t)it.rb * nst * sb;
      {
        if (__any_sync(0xffffffffu, *reinterpret_cast<volatile int*>(err) != 0)) {
          set_abort(sm, err, false);
          ok = false;
          break;
        }
        const size_t pst = (size_t)it.pass * nst;
        for (int j = it.j0; j < it.j1 && ok; j += UNIT, ++u) {
          const int ns = min(UNIT, it.j1 - j);
          const uint32_t us = u % SS;
          if (!warp_wait(sm, err, smem_addr(&sm.sempty[us]), ((u / SS) & 1u) ^ 1u)) {
            ok = false;
            break;
          }
          if (elect_one()) {
            const uint32_t sbar = smem_addr(&sm.sfull[us]);
            mbar_expect_tx(sbar, ns * (NB * 4 + sb));
            bulk_g2s(smem_addr(sm.asc[us]), ta.plan.apanel + (pst + j) * NB, ns * NB * 4, sbar);
            bulk_g2s(smem_addr(sm.scl[us]), sbase + (size_t)j * sb, ns * sb, sbar);
          }
          __syncwarp();
          for (int t = 0; t < ns; ++t, ++g) {
            const uint32_t s = g % ST;
            if (!warp_wait(sm, err, smem_addr(&sm.aempty[s]), ((g / ST) & 1u) ^ 1u)) {
              ok = false;
              break;
            }
            if (elect_one()) {
              const uint32_t bar = smem_addr(&sm.full[s]);
              mbar_expect_tx(bar, abytes + B_BYTES);
              tma_load_2d(smem_addr(sm.A[s]), map, 0, row0 + (j + t) * 128, bar);
              bulk_g2s(smem_addr(sm.B[s]), ta.plan.bpanel + (pst + j + t) * B_BYTES, B_BYTES, bar);
            }
            __syncwarp();
          }
        }
      }
    }
    // before the CTA's shared memory is released: wait for copies still in flight (only when a
    // wait gave up; otherwise every stage and unit was consumed)
    for (uint32_t h = g > (uint32_t)ST ? g - ST : 0; h < g; ++h)
      for (uint32_t i = 0; i < WAIT_LIMIT; ++i)
        if (mbar_try_wait(smem_addr(&sm.full[h % ST]), (h / ST) & 1u)) break;
    for (uint32_t h = u > (uint32_t)SS ? u - SS : 0; h < u; ++h)
      for (uint32_t i = 0; i < WAIT_LIMIT; ++i)
        if (mbar_try_wait(smem_addr(&sm.sfull[h % SS]), (h / SS) & 1u)) break;
  } else if (warp == MMA_WARP) {
    // the whole warp runs the loop (uniform control flow); one elected lane issues MMAs and commits.
    // g counts stages, u units, gq accumulator groups (one per unit, or one per block-scaled item)
    uint32_t g = 0, u = 0, gq = 0, qn = 0;
    bool ok = true;
    int item = blockIdx.x;
    Item nxt = !dyn && item < n_items ? item_of<FMT_R>(a, ta.plan, item, nrb, nst) : Item{};
    while (ok) {
      Item it;
      if (dyn) {
        const uint32_t qs = qn % IQ;
        if (!warp_wait<PROBE>(sm, err, smem_addr(&sm.iqfull[qs]), (qn / IQ) & 1u, clim)) {
          ok = false;
          break;
        }
        it = sm.iq[qs];
        __syncwarp();
        if (lane == 0) arrive(smem_addr(&sm.iqempty[qs]));
        ++qn;
        if (it.pass < 0) break;
      } else {
        if (item >= n_items) break;
        it = nxt;
        if (item + (int)gridDim.x < n_items) nxt = item_of<FMT_R>(a, ta.plan, item + gridDim.x, nrb, nst);
        item += gridDim.x;
      }
      const int fmt = item_fmt(it);
      if (block_scaled(fmt)) {
        // the whole K into one 16-column accumulator; per stage the weight and activation scale
        // factors are copied into the group's scale-factor columns ahead of the stage's 4 MMAs (the
        // copies and MMAs of this thread execute in issue order)
        const uint32_t q = gq % SA;
        if (!warp_wait<PROBE>(sm, err, smem_addr(&sm.gempty[q]), ((gq / SA) & 1u) ^ 1u, clim)) {
          ok = false;
          break;
        }
        const uint32_t cacc = tbase + q * GCOLS, csfa = cacc + SF_A_COL, csfb = cacc + SF_B_COL;
        const uint32_t afmt = fmt == FMT_FP8 ? 0u : 5u;
        for (int j = it.j0; j < it.j1 && ok; j += UNIT, ++u) {
          const int ns = min(UNIT, it.j1 - j);
          const uint32_t us = u % SS;
          if (!warp_wait<PROBE>(sm, err, smem_addr(&sm.sfull[us]), (u / SS) & 1u, clim)) {
            ok = false;
            break;
          }
          for (int t = 0; t < ns; ++t, ++g) {
            const uint32_t s = g % ST;
            if (!warp_wait<PROBE>(sm, err, smem_addr(&sm.full[s]), (g / ST) & 1u, clim)) {
              ok = false;
              break;
            }
            fence_after();
            // scale-factor sources: FP8 weights' two 128x128 block scales (rows 0-63, 64-127) spread
            // over the 128 rows; MXFP4 weights' scales are already in copy order in the side slot;
            // the pass's 16 activation scales (one per 128 K, the same for the stage's 4 blocks)
            uint32_t sfa_src;
            if (fmt == FMT_FP8) {
              const float* rec = reinterpret_cast<const float*>(sm.scl[us] + t * 16);
              const uint32_t lo = e8m0_of(rec[0]) * 0x01010101u, hi = e8m0_of(rec[1]) * 0x01010101u;
              *reinterpret_cast<uint4*>(sm.sfa[s] + lane * 16) = make_uint4(lo, lo, hi, hi);
              sfa_src = smem_addr(sm.sfa[s]);
            } else {
              sfa_src = smem_addr(sm.scl[us] + t * 512);
            }
            if (lane < NB) {
              const uint32_t e = e8m0_of(sm.asc[us][t * NB + lane]) * 0x01010101u;
              *reinterpret_cast<uint4*>(sm.sfb[s] + lane * 16) = make_uint4(e, e, e, e);
            }
            fence_proxy_async_smem();
            __syncwarp();
            const uint32_t abase = smem_addr(sm.A[s]), bbase = smem_addr(sm.B[s]);
            if (elect_one()) {
              cp_sf(csfa, sfa_src);
              cp_sf(csfb, smem_addr(sm.sfb[s]));
#pragma unroll
              for (int c = 0; c < 4; ++c)
                mma_bs(cacc, sdesc(abase + c * 32), sdesc(bbase + c * 32), idesc_bs(afmt, (uint32_t)c),
                       csfa | ((uint32_t)c << 30), csfb | ((uint32_t)c << 30), (j + t > it.j0 || c > 0) ? 1u : 0u);
              commit(smem_addr(&sm.aempty[s]));   // operand slot and its scale-factor sources
            }
            __syncwarp();
          }
          if (!ok) break;
          // the side slot is free once the copies that read it have completed (4 arrivals expected)
          if (elect_one())
#pragma unroll
            for (int i = 0; i < 4; ++i) commit(smem_addr(&sm.sempty[us]));
          __syncwarp();
        }
        if (!ok) break;
        if (elect_one()) commit(smem_addr(&sm.gfull[q]));
        __syncwarp();
        ++gq;
        continue;
      }
      const uint32_t id = idesc(fmt == FMT_FP8 ? 0u : 5u);
      {
        for (int j = it.j0; j < it.j1 && ok; j += UNIT, ++u, ++gq) {
          const int ns = min(UNIT, it.j1 - j);
          const uint32_t q = gq % SA;
          if (!warp_wait<PROBE>(sm, err, smem_addr(&sm.gempty[q]), ((gq / SA) & 1u) ^ 1u, clim)) {
            ok = false;
            break;
          }
          for (int t = 0; t < ns; ++t, ++g) {
            const uint32_t s = g % ST;
            if (!warp_wait<PROBE>(sm, err, smem_addr(&sm.full[s]), (g / ST) & 1u, clim)) {
              ok = false;
              break;
            }
            fence_after();
            const uint32_t abase = smem_addr(sm.A[s]), bbase = smem_addr(sm.B[s]);
            const uint32_t cols = tbase + q * GCOLS + t * SCOLS;
            if (elect_one()) {
              if (fmt == FMT_FP8) {
#pragma unroll
                for (int c = 0; c < 4; ++c)
                  mma(cols, sdesc(abase + c * 32), sdesc(bbase + c * 32), id, c > 0 ? 1u : 0u);
              } else {
                // one fresh slot per 32-K chunk: each chunk's partial is scaled on readback
#pragma unroll
                for (int c = 0; c < 4; ++c) mma(cols + c * NB, sdesc(abase + c * 32), sdesc(bbase + c * 32), id, 0u);
              }
              commit(smem_addr(&sm.aempty[s]));   // the operand slot is free once these MMAs have read it
            }
            __syncwarp();
          }
          if (!ok) break;
          if (elect_one()) commit(smem_addr(&sm.gfull[q]));
          __syncwarp();
        }
      }
    }
    // every MMA issued by the elected lane has completed once `drain` fires
    if (elect_one()) commit(smem_addr(&sm.drain));
    __syncwarp();
    for (uint32_t i = 0; i < WAIT_LIMIT; ++i)
      if (mbar_try_wait_sleep(smem_addr(&sm.drain), 0, 1000u)) break;
  } else {
    // ── readback + epilogue (warps 0-3) ──
    const int r = tid;  // weight row of the item = TMEM lane
    uint32_t u = 0, gq = 0, qn = 0;
    bool ok = true;
    int item = blockIdx.x;
    Item nxt = !dyn && item < n_items ? item_of<FMT_R>(a, ta.plan, item, nrb, nst) : Item{};
    for (;;) {
      Item it;
      if (dyn) {
        const uint32_t qs = qn % IQ;
        if (ok) ok = warp_wait<PROBE>(sm, err, smem_addr(&sm.iqfull[qs]), (qn / IQ) & 1u, clim);
        // one decision for all four warps (the epilogue's named barriers need all of them)
        if (workers_any(!ok)) break;
        it = sm.iq[qs];
        __syncwarp();
        if (lane == 0) arrive(smem_addr(&sm.iqempty[qs]));
        ++qn;
        if (it.pass < 0) break;
      } else {
        if (item >= n_items) break;
        it = nxt;
        if (item + (int)gridDim.x < n_items) nxt = item_of<FMT_R>(a, ta.plan, item + gridDim.x, nrb, nst);
        item += gridDim.x;
      }
      const int fmt = item_fmt(it);
      const WeightSet& ws = it.shared ? a.shared : a.routed;
      const int pm = tc_pass_max(fmt);
      const bool nv = fmt == FMT_NVFP4;
      const uint32_t sb = stage_sbytes(fmt);
      float ts = 1.f;
      if (nv && ws.ts != nullptr) {
        const float* tsp = ws.ts + (it.shared ? 0 : (size_t)it.expert * ws.ts_stride);
        ts = (w13 && r >= 64) ? tsp[1] : tsp[0];
      }
      bool stop = false;
      {
        const int pb = it.pb;
        const int pc = min(pm, it.cnt - pb);
        const int ncol = nv ? 2 * pc : pc;     // used columns of each chunk slot
        const bool narrow = ncol <= 4;
        // the pass's tokens: lane t holds token t's output row and routing weight (epilogue)
        int my_orow = 0;
        float my_wgt = 1.f;
        if (lane < pc) {
          const int i = pb + lane;
          if (it.shared) {
            my_orow = a.mode == MODE_DENSE ? i : (w13 && a.hpad ? a.hsh0 : P) + i;
          } else {
            const int qp = it.base + i;
            const int tok = a.pair_tok[qp], slot = a.pair_slot[qp];
            if (w13) {
              my_orow = a.hpad ? wide_pbase(it.base, it.expert) + i : qp;
              my_wgt = a.topk_w[(size_t)tok * a.topk + slot];
            } else {
              my_orow = tok * a.topk + slot;
            }
          }
        }
        float acc[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) acc[t] = 0.f;
        if (block_scaled(fmt)) {
          // one readback of the fully scaled accumulator per pass; the side slots went to the MMA warp
          const uint32_t q = gq % SA;
          u += (uint32_t)((it.j1 - it.j0 + UNIT - 1) / UNIT);
          if (ok) ok = warp_wait<PROBE>(sm, err, smem_addr(&sm.gfull[q]), (gq / SA) & 1u, clim);
          if (ok) {
            fence_after();
            uint32_t d[16];
            ld16(tbase + ((uint32_t)(warp * 32) << 16) + q * GCOLS, d);
            ld_wait();
            fence_before();
            __syncwarp();
            if (lane == 0) arrive(smem_addr(&sm.gempty[q]));
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[i] = __uint_as_float(d[i]);
          }
          ++gq;
        } else
        for (int j = it.j0; j < it.j1; j += UNIT, ++u, ++gq) {
          const int ns = min(UNIT, it.j1 - j);
          const uint32_t us = u % SS, q = gq % SA;
          // this unit's scales first (they landed long ago), so their loads overlap the MMA wait
          if (ok) ok = warp_wait<PROBE>(sm, err, smem_addr(&sm.sfull[us]), (u / SS) & 1u, clim);
          if (!ok) continue;
          float sc[UNIT][8];
#pragma unroll
          for (int t = 0; t < UNIT; ++t) {
            const uint8_t* sp = sm.scl[us] + t * sb;
            if (fmt == FMT_FP8) {
              const float* sw = reinterpret_cast<const float*>(sp);
              sc[t][0] = w13 ? sw[r >= 64 ? 1 : 0] : sw[0];
#pragma unroll
              for (int c = 1; c < 8; ++c) sc[t][c] = 0.f;
            } else if (nv) {
              const uint2 sv = t < ns ? *reinterpret_cast<const uint2*>(sp + r * 8) : make_uint2(0u, 0u);
              uint32_t h01, h23, h45, h67;
              e4m3x4_to_f16x2x2(sv.x, h01, h23);
              e4m3x4_to_f16x2x2(sv.y, h45, h67);
              const float2 f01 = __half22float2(*reinterpret_cast<__half2*>(&h01));
              const float2 f23 = __half22float2(*reinterpret_cast<__half2*>(&h23));
              const float2 f45 = __half22float2(*reinterpret_cast<__half2*>(&h45));
              const float2 f67 = __half22float2(*reinterpret_cast<__half2*>(&h67));
              sc[t][0] = f01.x; sc[t][1] = f01.y; sc[t][2] = f23.x; sc[t][3] = f23.y;
              sc[t][4] = f45.x; sc[t][5] = f45.y; sc[t][6] = f67.x; sc[t][7] = f67.y;
            } else {
              const uint32_t sv = t < ns ? *reinterpret_cast<const uint32_t*>(sp + mx_scale_off(r)) : 0u;
#pragma unroll
              for (int c = 0; c < 4; ++c) sc[t][c] = e8m0_to_f32(sv >> (8 * c));
#pragma unroll
              for (int c = 4; c < 8; ++c) sc[t][c] = 0.f;
            }
          }
          if (ok) ok = warp_wait<PROBE>(sm, err, smem_addr(&sm.gfull[q]), (gq / SA) & 1u, clim);
          if (!ok) continue;
          fence_after();
          const uint32_t taddr = tbase + ((uint32_t)(warp * 32) << 16) + q * GCOLS;
          // acc[i] += (stage partial of column i) * (its B row's activation scale)
          auto fold = [&](int t, const float (&blk)[16]) {
            const float4* ap = reinterpret_cast<const float4*>(sm.asc[us] + t * NB);
            const float4 a0 = ap[0], a1 = ap[1], a2 = ap[2], a3 = ap[3];
            const float av[16] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w,
                                  a2.x, a2.y, a2.z, a2.w, a3.x, a3.y, a3.z, a3.w};
            // NVFP4: token i's rows 2i / 2i+1 share one scale
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[i] = fmaf(blk[i], av[nv ? (2 * i) & (NB - 1) : i], acc[i]);
          };
          if (fmt == FMT_FP8) {
            // one accumulated 16-column slot per stage
            uint32_t d[UNIT][16];
#pragma unroll
            for (int t = 0; t < UNIT; ++t) {
              if (t < ns) {
                if (narrow) ld4(taddr + t * SCOLS, d[t]); else ld16(taddr + t * SCOLS, d[t]);
              }
            }
            ld_wait();
            fence_before();
            __syncwarp();
            if (lane == 0) arrive(smem_addr(&sm.gempty[q]));
#pragma unroll
            for (int t = 0; t < UNIT; ++t) {
              if (t >= ns) continue;
              float blk[16];
#pragma unroll
              for (int c = 0; c < 16; ++c) blk[c] = (narrow && c >= 4) ? 0.f : __uint_as_float(d[t][c]) * sc[t][0];
              fold(t, blk);
            }
          } else if (narrow) {
            // columns 0-3 of the 4 chunk slots of each stage
            uint32_t d[UNIT][16];
#pragma unroll
            for (int t = 0; t < UNIT; ++t)
              if (t < ns)
#pragma unroll
                for (int c = 0; c < 4; ++c) ld4(taddr + t * SCOLS + c * NB, &d[t][4 * c]);
            ld_wait();
            fence_before();
            __syncwarp();
            if (lane == 0) arrive(smem_addr(&sm.gempty[q]));
#pragma unroll
            for (int t = 0; t < UNIT; ++t) {
              if (t >= ns) continue;
              float blk[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) blk[i] = 0.f;
              if (nv) {
                // column 2i: first 16 K of each chunk (group 2c), column 2i+1: second (group 2c+1)
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                  float v = 0.f;
#pragma unroll
                  for (int c = 0; c < 4; ++c) {
                    v = fmaf(__uint_as_float(d[t][4 * c + 2 * i]), sc[t][2 * c], v);
                    v = fmaf(__uint_as_float(d[t][4 * c + 2 * i + 1]), sc[t][2 * c + 1], v);
                  }
                  blk[i] = v;
                }
              } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  float v = 0.f;
#pragma unroll
                  for (int c = 0; c < 4; ++c) v = fmaf(__uint_as_float(d[t][4 * c + i]), sc[t][c], v);
                  blk[i] = v;
                }
              }
              fold(t, blk);
            }
          } else {
            // all 16 columns: two chunk slots (32 columns) per TMEM load round
#pragma unroll
            for (int t = 0; t < UNIT; ++t) {
              if (t >= ns) continue;
              float blk[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) blk[i] = 0.f;
#pragma unroll
              for (int half = 0; half < 2; ++half) {
                uint32_t da[16], db[16];
                ld16(taddr + t * SCOLS + (2 * half) * NB, da);
                ld16(taddr + t * SCOLS + (2 * half + 1) * NB, db);
                ld_wait();
                const int c0 = 2 * half, c1 = 2 * half + 1;
                if (nv) {
#pragma unroll
                  for (int i = 0; i < 8; ++i) {
                    float v = fmaf(__uint_as_float(da[2 * i]), sc[t][2 * c0], blk[i]);
                    v = fmaf(__uint_as_float(da[2 * i + 1]), sc[t][2 * c0 + 1], v);
                    v = fmaf(__uint_as_float(db[2 * i]), sc[t][2 * c1], v);
                    blk[i] = fmaf(__uint_as_float(db[2 * i + 1]), sc[t][2 * c1 + 1], v);
                  }
                } else {
#pragma unroll
                  for (int i = 0; i < 16; ++i) {
                    float v = fmaf(__uint_as_float(da[i]), sc[t][c0], blk[i]);
                    blk[i] = fmaf(__uint_as_float(db[i]), sc[t][c1], v);
                  }
                }
              }
              fold(t, blk);
            }
            fence_before();
            __syncwarp();
            if (lane == 0) arrive(smem_addr(&sm.gempty[q]));
          }
          __syncwarp();
          if (lane == 0) arrive(smem_addr(&sm.sempty[us]));
        }
        // one decision for all workers: the W13 epilogue below synchronises them
        if (workers_any(!ok || aborted(sm))) stop = true;
        bool merged_away = false;
        if (!stop && it.kn > 1) {
          // a K piece: publish the partial, count in; the last piece of the block sums all of them
          // in K order (its own from registers) and goes on to the epilogue
          const int kid = it.pass * nrb + it.rb;
          float* blk = a.part + (size_t)kid * it.kn * 2048;
          float4* mine = reinterpret_cast<float4*>(blk + (size_t)it.ks * 2048 + r * 16);
#pragma unroll
          for (int v = 0; v < 4; ++v) mine[v] = make_float4(acc[4 * v], acc[4 * v + 1], acc[4 * v + 2], acc[4 * v + 3]);
          __threadfence();
          asm volatile("bar.sync 1, 128;\n" ::: "memory");
          if (r == 0) {
            const int prev = atomicAdd(a.kcnt + kid, 1);
            sm.klast = prev == it.kn - 1;
            if (sm.klast) a.kcnt[kid] = 0;   // ready for the next launch
          }
          asm volatile("bar.sync 1, 128;\n" ::: "memory");
          if (sm.klast) {
            __threadfence();
#pragma unroll
            for (int t = 0; t < 16; ++t) acc[t] = 0.f;
            // this piece's own partial included, re-read; per float4 of the pass's tokens, eight
            // pieces' loads in flight at a time, added in piece order
            const int nq = pc <= 4 ? 1 : (pc <= 8 ? 2 : 4);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              if (v >= nq) continue;
              float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
              for (int q0 = 0; q0 < it.kn; q0 += 8) {
                float4 w[8];
#pragma unroll
                for (int dq = 0; dq < 8; ++dq)
                  w[dq] = q0 + dq < it.kn
                              ? __ldcg(reinterpret_cast<const float4*>(blk + (size_t)(q0 + dq) * 2048 + r * 16) + v)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int dq = 0; dq < 8; ++dq) {
                  sum.x += w[dq].x;
                  sum.y += w[dq].y;
                  sum.z += w[dq].z;
                  sum.w += w[dq].w;
                }
              }
              acc[4 * v] = sum.x;
              acc[4 * v + 1] = sum.y;
              acc[4 * v + 2] = sum.z;
              acc[4 * v + 3] = sum.w;
            }
          } else {
            merged_away = true;
          }
          asm volatile("bar.sync 1, 128;\n" ::: "memory");   // klast is rewritten by the next piece
        }
        if (!stop && !merged_away) {
          if (w13) {
            // rows r < 64 are w1 (gate) rows, r >= 64 the matching w3 (up) rows
            const int I = a.n_rows / 2;
            if (r >= 64) {
#pragma unroll
              for (int t = 0; t < 16; ++t) sm.xchg[r - 64][t] = __float2bfloat16_rn(acc[t] * ts);
            }
            asm volatile("bar.sync 1, 128;\n" ::: "memory");
            if (r < 64) {
              const float lim = a.swiglu_limit;
#pragma unroll
              for (int t = 0; t < 16; ++t) {
                if (t < pc) {
                  const int orow = __shfl_sync(0xffffffffu, my_orow, t);
                  const float wgt = __shfl_sync(0xffffffffu, my_wgt, t);
                  float gv = bf16_round(acc[t] * ts);
                  float uv = __bfloat162float(sm.xchg[r][t]);
                  if (lim > 0.f) {
                    uv = fminf(fmaxf(uv, -lim), lim);
                    gv = fminf(gv, lim);
                  }
                  float h = silu(gv) * uv;
                  if (!it.shared) h = wgt * h;
                  a.hbf[(size_t)orow * I + it.rb * 64 + r] = __float2bfloat16_rn(h);
                }
              }
            }
            asm volatile("bar.sync 1, 128;\n" ::: "memory");   // xchg is rewritten by the next pass
          } else {
            const int n0 = it.rb * 128;
#pragma unroll
            for (int t = 0; t < 16; ++t) {
              if (t < pc) {
                const int orow = __shfl_sync(0xffffffffu, my_orow, t);
                a.o[(size_t)orow * a.n_rows + n0 + r] = __float2bfloat16_rn(acc[t] * ts);
              }
            }
          }
        }
      }
      if (stop) break;
    }
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == MMA_WARP)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tbase), "r"(TMEM_COLS));
}

// ── B panels: the activation operand of every pass, one 2 KB swizzled tile per (pass, stage) ──
// CTA (group of PANEL_STAGES stages, slot): slot 0 is the shared expert / dense matrix when present,
// then the active slots. Thread (row = tid / 8, chunk c = tid % 8) writes the 16-byte chunk c of B
// row `row` of every stage of the group, its loads for all the group's stages issued first.
// W13 / DENSE: the e4m3 row slice and its scale are copied. W2: the bf16 h row slice is quantised
// to e4m3 with one scale per 128 K (act_quant, kernel.py:40-125): amax over the 8 threads of the
// row, scale = amax/448 (or its power-of-two ceiling), q = e4m3(v / scale).
constexpr int PANEL_STAGES = 4;

__global__ void __launch_bounds__(128) panel_kernel(PanelArgs a) {
  const int j0 = blockIdx.x * PANEL_STAGES;
  const int slot = blockIdx.y;
  const int K = a.k, nst = K / 128, nkb = K / 128;
  const int P = a.m * a.topk;
  pdl_wait();
  pdl_trigger();
  if (blockIdx.x == 0 && blockIdx.y == 0) {
    if (a.kzero != nullptr)
      for (int i = threadIdx.x; i < a.nkzero; i += blockDim.x) a.kzero[i] = 0;
    if (a.zero_err != nullptr && threadIdx.x == 0) *a.zero_err = 0;
    if (a.zero_sched != nullptr && threadIdx.x == 0) *a.zero_sched = 0;
  }
  int shared, cnt, base, pass0, nv;
  int hrow0 = -1;   // W2, hybrid: first h row of the expert in the padded row space
  if (slot < a.has_shared) {
    shared = 1;
    cnt = a.m;
    base = 0;
    pass0 = 0;
    nv = a.nv_shared;
  } else {
    const int s = slot - a.has_shared;
    if (s >= *a.n_active) return;
    const int e = a.active[s];
    shared = 0;
    cnt = a.counts[e];
    if (a.hot_min > 0 && cnt >= a.hot_min) return;   // a hot expert of the hybrid dispatch
    base = a.offsets[e];
    if (a.hpad) hrow0 = wide_pbase(base, e);
    pass0 = a.n_sh_pass + a.pass_off[s];
    nv = a.nv_routed;
  }
  const int pm = nv ? 8 : 16;
  const int row = threadIdx.x >> 3, c = threadIdx.x & 7;
  const int tslot = nv ? row >> 1 : row;
  const bool keep = nv ? ((c & 1) == (row & 1)) : true;
  for (int pb = 0, pi = 0; pb < cnt; pb += pm, ++pi) {
    const int i = pb + tslot;
    const bool valid = tslot < pm && i < cnt;
    int srow = 0;
    if (valid) {
      if (a.mode != MODE_W2) srow = (shared || a.pair_tok == nullptr) ? i : a.pair_tok[base + i];
      else srow = shared ? (a.hpad ? a.hsh0 : P) + i : (hrow0 >= 0 ? hrow0 : base) + i;
    }
    uint4 v[PANEL_STAGES];
    float sc[PANEL_STAGES];
    if (a.mode != MODE_W2) {
#pragma unroll
      for (int u = 0; u < PANEL_STAGES; ++u) {
        const int j = j0 + u;
        v[u] = make_uint4(0u, 0u, 0u, 0u);
        sc[u] = 0.f;
        if (valid && j < nst) {
          v[u] = *reinterpret_cast<const uint4*>(a.xq + (size_t)srow * K + (size_t)j * 128 + c * 16);
          sc[u] = a.xs[(size_t)srow * nkb + j];
        }
      }
    } else {
      uint4 hv[PANEL_STAGES][2];
#pragma unroll
      for (int u = 0; u < PANEL_STAGES; ++u) {
        const int j = j0 + u;
        hv[u][0] = hv[u][1] = make_uint4(0u, 0u, 0u, 0u);
        if (valid && j < nst) {
          const uint4* hp = reinterpret_cast<const uint4*>(a.hbf + (size_t)srow * K + (size_t)j * 128 + c * 16);
          hv[u][0] = hp[0];
          hv[u][1] = hp[1];
        }
      }
#pragma unroll
      for (int u = 0; u < PANEL_STAGES; ++u) {
        float f[16];
        const __nv_bfloat162* p0 = reinterpret_cast<const __nv_bfloat162*>(&hv[u][0]);
        const __nv_bfloat162* p1 = reinterpret_cast<const __nv_bfloat162*>(&hv[u][1]);
        float am = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 x0 = __bfloat1622float2(p0[e]), x1 = __bfloat1622float2(p1[e]);
          f[2 * e] = x0.x;
          f[2 * e + 1] = x0.y;
          f[8 + 2 * e] = x1.x;
          f[8 + 2 * e + 1] = x1.y;
        }
#pragma unroll
        for (int e = 0; e < 16; ++e) am = fmaxf(am, fabsf(f[e]));
        // the 8 threads of a row are 8 consecutive lanes
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 4));
        v[u] = make_uint4(0u, 0u, 0u, 0u);
        sc[u] = 0.f;
        if (valid && j0 + u < nst) {
          const float s_ = act_scale(am, a.act_pow2 != 0);
          uint8_t qb[16];
          if (a.act_pow2) {
            const float inv = __frcp_rn(s_);   // exact: s_ is a power of two
#pragma unroll
            for (int e = 0; e < 16; ++e) qb[e] = act_q_pow2(f[e], inv);
          } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) qb[e] = act_q(f[e], s_);
          }
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            w[e] = (uint32_t)qb[4 * e] | ((uint32_t)qb[4 * e + 1] << 8) | ((uint32_t)qb[4 * e + 2] << 16) |
                   ((uint32_t)qb[4 * e + 3] << 24);
          v[u] = make_uint4(w[0], w[1], w[2], w[3]);
          sc[u] = s_;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < PANEL_STAGES; ++u) {
      const int j = j0 + u;
      if (j >= nst) break;
      const size_t tile = (size_t)(pass0 + pi) * nst + j;
      *reinterpret_cast<uint4*>(a.bpanel + tile * B_BYTES + row * 128 + ((c ^ (row & 7)) << 4)) =
          keep ? v[u] : make_uint4(0u, 0u, 0u, 0u);
      if (c == 0) a.apanel[tile * NB + row] = valid ? sc[u] : 0.f;
    }
  }
}

// ── host side ───────────────────────────────────────────────────────────────────────────────────

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// Weight tiles of a TC-tiled bank as a 2-D tensor [rows][128 K]: fp4 as 16U4_ALIGN16B (64 B of
// packed values per row in memory, 128 B per row in shared memory), FP8 as bytes. A box is one
// stage: 128 rows x 128 K, swizzled 128 B.
static cudaError_t make_map(CUtensorMap* map, const void* base, int fmt, uint64_t rows) {
  memset(map, 0, sizeof *map);
  if (base == nullptr || rows == 0) return cudaSuccess;
  PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
  if (enc == nullptr) return cudaErrorNotSupported;
  const bool fp8 = fmt == FMT_FP8;
  const cuuint64_t dims[2] = {128, rows};
  const cuuint64_t strides[1] = {fp8 ? 128u : 64u};
  const cuuint32_t box[2] = {128, 128};
  const cuuint32_t es[2] = {1, 1};
  const CUresult r = enc(map, fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 2,
                         const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int F, bool PROBE, bool DYN>
static cudaError_t launch_tc_variant(const TcArgs& a, int grid, cudaStream_t st) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(tc_grouped_kernel<F, PROBE, DYN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         SMEM_BYTES);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  return launch_pdl(tc_grouped_kernel<F, PROBE, DYN>, dim3(grid), dim3(NTHREADS), SMEM_BYTES, st, a);
}

// the probing variant only when a test wait limit is set; the item-counter variant only when the
// launch has a counter
template <int F>
static cudaError_t launch_tc_one(const TcArgs& a, int grid, cudaStream_t st) {
  if (a.g.sched != nullptr)
    return a.g.wait_limit ? launch_tc_variant<F, true, true>(a, grid, st) : launch_tc_variant<F, false, true>(a, grid, st);
  return a.g.wait_limit ? launch_tc_variant<F, true, false>(a, grid, st) : launch_tc_variant<F, false, false>(a, grid, st);
}

}  // namespace tc

cudaError_t launch_tc_panel(const PanelArgs& a, int max_slots, cudaStream_t st) {
  if (max_slots < 1) return cudaSuccess;
  dim3 grid((a.k / 128 + tc::PANEL_STAGES - 1) / tc::PANEL_STAGES, max_slots);
  return launch_pdl(tc::panel_kernel, grid, dim3(128), 0, st, a);
}

cudaError_t launch_tc_grouped(const GroupedArgs& g, const TcPlan& plan, int max_items, cudaStream_t st) {
  tc::TcArgs a;
  a.g = g;
  a.plan = plan;
  const uint64_t nst = (uint64_t)g.k / 128, nrb = (uint64_t)g.n_rows / 128;
  cudaError_t e = tc::make_map(&a.map_routed, g.mode == MODE_DENSE ? nullptr : g.routed.w, g.routed.fmt,
                               (uint64_t)g.n_experts * nrb * nst * 128);
  if (e != cudaSuccess) return e;
  e = tc::make_map(&a.map_shared, g.has_shared ? g.shared.w : nullptr, g.mode == MODE_DENSE ? g.shared.fmt : FMT_FP8,
                   nrb * nst * 128);
  if (e != cudaSuccess) return e;
  int grid = 2 * num_sms();  // 2 CTAs per SM: ~100 KB shared memory and 256 TMEM columns each
  if (grid > max_items) grid = max_items;
  if (grid < 1) grid = 1;
  switch (g.routed.fmt) {
    case FMT_NVFP4: return tc::launch_tc_one<FMT_NVFP4>(a, grid, st);
    case FMT_MXFP4: return tc::launch_tc_one<FMT_MXFP4>(a, grid, st);
    default: return tc::launch_tc_one<FMT_FP8>(a, grid, st);
  }
}


// ── TC layout: canonical -> [N/128 row-blocks][K/128 stages][...] ─────────────────────────────────
// fp4 values   [128 rows][64 B]                  (128 K packed, low nibble first)
// FP8 values   [128 rows][128 B]
// NVFP4 scales [128 rows][8 B]                   (the row's 8 group scales of the stage)
// MXFP4 scales [32][4 rows][4 B]: row r's four per-32 scales at 16 (r % 32) + 4 (r / 32), the order in
//              which tcgen05.cp .32x128b.warpx4 lands them as the block-scaled MMA's scale factors
//              (TMEM lane r % 32 of every sub-partition, column r / 32, byte = 32-K block)
// FP8 scales   [4] fp32: block scale of rows 0-63, of rows 64-127, 2 zero pads (16-byte copies)
// W13 row-blocks hold 64 w1 rows then the same 64 w3 rows (rb covers intermediate 64*rb..+63).
__device__ __forceinline__ int64_t tc_row(int kind, int64_t n, int64_t rb, int r) {
  if (kind == 1) return r < 64 ? 64 * rb + r : n / 2 + 64 * rb + (r - 64);
  return 128 * rb + r;
}

__global__ void tc_tile_values_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int fmt, int kind,
                                      int64_t n_mat, int64_t n, int64_t k) {
  const int64_t nrb = n / 128, nst = k / 128;
  const int rowb = fmt == FMT_FP8 ? 128 : 64;   // bytes of a row per stage
  const int64_t pieces = rowb / 16;             // 16-byte pieces per row per stage
  const int64_t units = n_mat * nrb * nst * 128 * pieces;
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < units; u += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = u % pieces;
    const int64_t rest = u / pieces;
    const int r = (int)(rest & 127);
    const int64_t j = (rest >> 7) % nst;
    const int64_t rb = ((rest >> 7) / nst) % nrb;
    const int64_t mat = ((rest >> 7) / nst) / nrb;
    const int64_t src_row = mat * n + tc_row(kind, n, rb, r);
    const uint8_t* s = src + src_row * (k * rowb / 128) + j * rowb + c * 16;
    uint8_t* d = dst + u * 16;
    *reinterpret_cast<uint4*>(d) = *reinterpret_cast<const uint4*>(s);
  }
}

__global__ void tc_tile_scales_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int fmt, int kind,
                                      int64_t n_mat, int64_t n, int64_t k) {
  const int64_t nrb = n / 128, nst = k / 128;
  if (fmt == FMT_FP8) {
    const float* s = reinterpret_cast<const float*>(src);
    float* d = reinterpret_cast<float*>(dst);
    const int64_t nsrb = (n + 127) / 128, nkb = k / 128;
    const int64_t units = n_mat * nrb * nst;
    for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < units; u += (int64_t)gridDim.x * blockDim.x) {
      const int64_t j = u % nst, rb = (u / nst) % nrb, mat = (u / nst) / nrb;
      const float* m = s + mat * nsrb * nkb;
      d[4 * u] = m[(tc_row(kind, n, rb, 0) / 128) * nkb + j];
      d[4 * u + 1] = m[(tc_row(kind, n, rb, 64) / 128) * nkb + j];
      d[4 * u + 2] = 0.f;
      d[4 * u + 3] = 0.f;
    }
  } else {
    const int per = fmt == FMT_NVFP4 ? 8 : 4;           // scale bytes per row per stage
    const int64_t rowb = fmt == FMT_NVFP4 ? k / 16 : k / 32;
    const int64_t units = n_mat * nrb * nst * 128;
    for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < units; u += (int64_t)gridDim.x * blockDim.x) {
      const int r = (int)(u & 127);
      const int64_t j = (u >> 7) % nst, rb = ((u >> 7) / nst) % nrb, mat = ((u >> 7) / nst) / nrb;
      const uint8_t* s = src + (mat * n + tc_row(kind, n, rb, r)) * rowb + j * per;
      uint8_t* d = dst + (u - r) * per + (fmt == FMT_MXFP4 ? mx_scale_off(r) : r * per);
      for (int i = 0; i < per; ++i) d[i] = s[i];
    }
  }
}

cudaError_t launch_tc_tile(int fmt, int kind, bool scales, const void* src, void* dst, int64_t n_mat, int64_t n,
                           int64_t k, cudaStream_t st) {
  const int64_t units = n_mat * (n / 128) * (k / 128) * 1024;
  int64_t b = (units + 255) / 256;
  const int grid = (int)(b < 1 ? 1 : (b > 262144 ? 262144 : b));
  if (scales)
    tc_tile_scales_kernel<<<grid, 256, 0, st>>>((const uint8_t*)src, (uint8_t*)dst, fmt, kind, n_mat, n, k);
  else
    tc_tile_values_kernel<<<grid, 256, 0, st>>>((const uint8_t*)src, (uint8_t*)dst, fmt, kind, n_mat, n, k);
  return cudaGetLastError();
}

}  // namespace sb
