// Gate logits of prefill batches on the tensor cores (Gate.forward's F.linear, model.py:570):
// part[s][t][e] = sum over the K-split s of bf16 x[t] . bf16 W[e], fp32.
//
// The same partial-logit layout as the split-K GEMV (sb_route.cu, gate_logits_kernel) with the same
// split width, so route_kernel adds the splits in the same fixed order. A CTA computes one tile of
// 128 experts x 128 tokens over one K split: tcgen05.mma kind::f16 (bf16 x bf16, fp32 in TMEM,
// K = 16 per instruction) on 64-K stages that TMA brings in 128-byte-swizzled (rows past E or M are
// filled with zeros and their results never stored). The products are exact and the sums fp32, so
// the logits match the reference's fp32 F.linear up to summation order, and a token's logits do not
// depend on the other tokens of its tile.
//
// Roles (192 threads): warp 4 producer (TMA), warp 5 MMA issuer (allocates TMEM), warps 0-3 write
// the tile (TMEM lane = expert row). Every wait is bounded.
#include <cudaTypedefs.h>

#include "sb_launch.h"
#include "sb_tcgen05.cuh"

namespace sb {
namespace gtc {

using namespace tc5;

constexpr int NTHREADS = 192;
constexpr int PRODUCER_WARP = 4;
constexpr int MMA_WARP = 5;
constexpr int TILE_E = 128, TILE_T = 128;
constexpr int ST = 4;                          // stage ring
constexpr int A_BYTES = TILE_E * 128;          // 128 expert rows x 64 bf16
constexpr int B_BYTES = TILE_T * 128;          // 128 token rows x 64 bf16
constexpr uint32_t WAIT_LIMIT = 1u << 16;

struct Smem {
  uint8_t A[ST][A_BYTES];                      // 1024-aligned (128B swizzle atoms)
  uint8_t B[ST][B_BYTES];
  uint64_t full[ST], empty[ST], done;
  uint32_t tmem_base;
  int abort;
};
constexpr int SMEM_BYTES = (int)sizeof(Smem) + 1024;

struct GateArgs {
  CUtensorMap map_w;   // W [E][H] bf16: box 64 x 128
  CUtensorMap map_x;   // x [M][H] bf16: box 64 x 128
  float* part;
  int m, e, h, kspl;
  int* err;
};

__device__ int g_gate_err = 0;

__global__ void __launch_bounds__(NTHREADS, 1) gate_tc_kernel(const __grid_constant__ GateArgs ga) {
  extern __shared__ uint8_t dyn_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(dyn_raw) + 1023) & ~(uintptr_t)1023);
  int* err = ga.err != nullptr ? ga.err : &g_gate_err;
  volatile int* abort_flag = &sm.abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int e0 = blockIdx.x * TILE_E, t0 = blockIdx.y * TILE_T, ks = blockIdx.z;
  const int nk = ga.kspl / 64;

  if (tid == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(smem_addr(&sm.full[s]), 1);
      mbar_init(smem_addr(&sm.empty[s]), 1);
    }
    mbar_init(smem_addr(&sm.done), 1);
    sm.abort = 0;
    mbar_init_fence();
  }
  if (warp == MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_addr(&sm.tmem_base)),
                 "r"(TILE_T));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tbase = sm.tmem_base;
  pdl_wait();
  pdl_trigger();
  auto wait = [&](uint32_t bar, uint32_t parity) { return wait_bounded(abort_flag, err, bar, parity, WAIT_LIMIT); };

  if (warp == PRODUCER_WARP) {
    if (lane == 0) {
      prefetch_map(&ga.map_w);
      prefetch_map(&ga.map_x);
      int k = 0;
      for (; k < nk; ++k) {
        const int s = k % ST;
        if (!wait(smem_addr(&sm.empty[s]), ((k / ST) & 1u) ^ 1u)) break;
        const uint32_t bar = smem_addr(&sm.full[s]);
        mbar_expect_tx(bar, A_BYTES + B_BYTES);
        const int kx = ks * ga.kspl + k * 64;
        tma_load_2d(smem_addr(sm.A[s]), &ga.map_w, kx, e0, bar);
        tma_load_2d(smem_addr(sm.B[s]), &ga.map_x, kx, t0, bar);
      }
      // copies still in flight (only when a wait gave up) land before the CTA exits
      for (int h = k > ST ? k - ST : 0; h < k; ++h)
        for (uint32_t i = 0; i < WAIT_LIMIT; ++i)
          if (mbar_try_wait(smem_addr(&sm.full[h % ST]), (h / ST) & 1u)) break;
    }
  } else if (warp == MMA_WARP) {
    if (lane == 0) {
      const uint32_t id = idesc_bf16(TILE_T);
      int k = 0;
      for (; k < nk; ++k) {
        const int s = k % ST;
        if (!wait(smem_addr(&sm.full[s]), (k / ST) & 1u)) break;
        fence_after();
        const uint32_t a = smem_addr(sm.A[s]), b = smem_addr(sm.B[s]);
#pragma unroll
        for (int j = 0; j < 4; ++j) mma_f16(tbase, sdesc(a + j * 32), sdesc(b + j * 32), id, (k > 0 || j > 0) ? 1u : 0u);
        commit(smem_addr(&sm.empty[s]));
      }
      // the accumulator is complete (or the CTA is winding down) once every issued MMA has run
      commit(smem_addr(&sm.done));
    }
  } else {
    // warps 0-3: TMEM lane r = expert e0 + r; columns = tokens t0 ..
    const int r = tid;
    const bool ok = wait(smem_addr(&sm.done), 0);
    if (__all_sync(0xffffffffu, ok) && !*abort_flag) {
      fence_after();
      const int e = e0 + r;
      const int nt = min(TILE_T, ga.m - t0);
      float* out = ga.part + ((size_t)ks * ga.m + t0) * ga.e + e;
      for (int c = 0; c < nt; c += 32) {
        uint32_t d[32];
        ld32(tbase + ((uint32_t)(warp * 32) << 16) + c, d);
        ld_wait();
        if (e < ga.e) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (c + j < nt) out[(size_t)(c + j) * ga.e] = __uint_as_float(d[j]);
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == MMA_WARP)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tbase), "r"(TILE_T));
}

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

// bf16 [rows][h] as a 2-D tensor with 64 x 128 boxes, 128-byte swizzle
static cudaError_t map_rows(CUtensorMap* map, const void* base, uint64_t rows, uint64_t h) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
  if (enc == nullptr) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {h, rows};
  const cuuint64_t strides[1] = {h * 2};
  const cuuint32_t box[2] = {64, 128};
  const cuuint32_t es[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace gtc

cudaError_t launch_gate_tc(const void* x, const void* w, float* part, int m, int e, int h, int kspl, int* err,
                           cudaStream_t st) {
  gtc::GateArgs a;
  memset(&a, 0, sizeof a);
  cudaError_t rc = gtc::map_rows(&a.map_w, w, (uint64_t)e, (uint64_t)h);
  if (rc != cudaSuccess) return rc;
  rc = gtc::map_rows(&a.map_x, x, (uint64_t)m, (uint64_t)h);
  if (rc != cudaSuccess) return rc;
  a.part = part;
  a.m = m;
  a.e = e;
  a.h = h;
  a.kspl = kspl;
  a.err = err;
  static bool configured = false;
  if (!configured) {
    rc = cudaFuncSetAttribute(gtc::gate_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, gtc::SMEM_BYTES);
    if (rc != cudaSuccess) return rc;
    configured = true;
  }
  const dim3 grid((e + gtc::TILE_E - 1) / gtc::TILE_E, (m + gtc::TILE_T - 1) / gtc::TILE_T, h / kspl);
  return launch_pdl(gtc::gate_tc_kernel, grid, dim3(gtc::NTHREADS), gtc::SMEM_BYTES, st, a);
}

}  // namespace sb
