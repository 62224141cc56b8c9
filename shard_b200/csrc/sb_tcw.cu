// Grouped expert GEMM at prefill widths on the tensor cores: bf16 operands and the whole K reduced
// in TMEM, so each pass is read back once (the verify-width kernel, sb_tc.cu, reads back per stage).
//
// Items are (pass, 128-row block) as in sb_tc.cu, with passes of up to WN = 128 tokens. Operands per
// 64-K sub-stage:
//   A  the weight tile dequantised to bf16 by the worker warps from a compact staging copy:
//      NVFP4 e2m1 x e4m3 (scale per 16) and MXFP4 e2m1 x e8m0 (per 32) are exact in bf16 (at most
//      6 significant bits); FP8 e4m3 x its 128x128 block scale (a power of two here). The NVFP4
//      tensor scale is applied in the epilogue.
//   B  the pass's activation rows, bf16 values of the act-quantised activations, from an
//      expert-ordered activation matrix by 2-D TMA boxes of 32 rows, 128-byte swizzled. With
//      power-of-two activation scales (ue8m0) e4m3 x scale is exact in bf16; with fp32 scales the
//      product is carried as two bf16 planes, hi = bf16(v) and lo = bf16(v - hi) (~16 significant
//      bits), and each sub-stage multiplies A by both into the same accumulator.
// tcgen05.mma kind::f16 (M=128, N = tokens rounded up to 16, K=16) accumulates the whole K into one
// of two TMEM accumulators (double-buffered across passes); the products are exact and the sum is
// fp32, the reference's dequant-then-fp32-matmul up to summation order.
//
// Roles (192 threads): warps 0-3 convert (thread r = weight row r) and, after a pass's last
// sub-stage, run its epilogue (TMEM lanes = rows); warp 4 producer (TMA / bulk copies); warp 5 MMA
// issuer (allocates TMEM). Every wait is bounded; on timeout the CTA records an error and winds down.
#include <cudaTypedefs.h>

#include "sb_launch.h"
#include "sb_tcgen05.cuh"

namespace sb {
namespace tcw {

using namespace tc5;

constexpr int NTHREADS = 192;
constexpr int PRODUCER_WARP = 4;
constexpr int MMA_WARP = 5;
constexpr int WN = TC_WIDE_PASS;        // tokens (B rows) per pass
constexpr int SC = 4;                   // staging ring (compact weight stage + scales)
constexpr int SAR = 2;                  // bf16 A tiles (64 K)
constexpr int SBR = 2;                  // bf16 B tiles (64 K)
constexpr int STG_W = 8192;             // fp4: 128 rows x 64 B (128 K); FP8: 128 rows x 64 B (64 K)
constexpr int STG_S = 1024;             // NVFP4 [128][8 B], MXFP4 [128][4 B], FP8 16 B
constexpr int A_BYTES = 128 * 128;      // 128 rows x 64 bf16
constexpr int B_BYTES = WN * 128;       // WN rows x 64 bf16
constexpr int BOX_ROWS = 32;
constexpr int TMEM_COLS = 2 * WN;
constexpr uint32_t WAIT_LIMIT = 1u << 16;

struct Smem {
  uint8_t A[SAR][A_BYTES];              // 1024-aligned (128B swizzle atoms)
  uint8_t B[SBR][B_BYTES];
  uint8_t stg[SC][STG_W + STG_S];
  uint64_t sfull[SC], sempty[SC], afull[SAR], aempty[SAR], bfull[SBR], bempty[SBR], accfull[2], accempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  float xchg[64][33];
};
constexpr int SMEM_BYTES = (int)sizeof(Smem) + 1024;

struct WideArgs {
  CUtensorMap map_b;        // activations, bf16 [rows][k]: box 64 x 32, 128-byte swizzle
  CUtensorMap map_w8;       // FP8 routed bank as bytes [rows][128]: box 64 x 128 (unused for fp4)
  CUtensorMap map_w8_sh;    // the FP8 shared expert / dense matrix, same form
  GroupedArgs g;
  TcPlan plan;
  int use_w8, use_w8_sh;    // which FP8 maps were encoded (the others stay zeroed and untouched)
  int b_split;              // B carries a residual plane (rows b_lo_row.. of map_b)
  int b_lo_row;
};

struct Item {
  int shared, expert, rb, cnt, base, pb, pass;
};

template <int FMT_R>
__device__ __forceinline__ Item item_of(const GroupedArgs& a, const TcPlan& plan, int item, int nrb) {
  Item it;
  const int p = item / nrb;
  it.rb = item - p * nrb;
  it.pass = p;
  if (p < plan.n_sh_pass) {
    it.shared = 1;
    it.expert = 0;
    it.cnt = a.m;
    it.base = 0;
    it.pb = p * WN;
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

__device__ int g_tcw_dense_err = 0;

// f16x2 holding exactly representable values -> bf16x2
__device__ __forceinline__ uint32_t f16x2_to_bf16x2(uint32_t h) {
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h));
  const __nv_bfloat162 b = __floats2bfloat162_rn(f.x, f.y);
  return *reinterpret_cast<const uint32_t*>(&b);
}

__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t s2) {
  const __nv_bfloat162 r =
      __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&a), *reinterpret_cast<const __nv_bfloat162*>(&s2));
  return *reinterpret_cast<const uint32_t*>(&r);
}

__device__ __forceinline__ uint32_t bf16_splat(float v) {
  const __nv_bfloat162 b = __floats2bfloat162_rn(v, v);
  return *reinterpret_cast<const uint32_t*>(&b);
}

// Row r's 64 values of one sub-stage -> 8 swizzled 16-byte chunks of the bf16 A tile.
//   fp4: src = the row's 32 packed bytes (4 groups of 16 values); scl = the row's scale bytes of
//        the sub-stage (NVFP4: 4 e4m3, MXFP4: 2 e8m0)
//   FP8: src = the row's 64 e4m3 bytes; wsc = its block scale
template <int FMT>
__device__ __forceinline__ void convert_row(const uint8_t* src, uint32_t scl, float wsc, uint8_t* dst, int r) {
  if (FMT == FMT_FP8) {
    const uint32_t s2 = bf16_splat(wsc);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint2 v = *reinterpret_cast<const uint2*>(src + c * 8);
      uint32_t h0, h1, h2, h3;
      e4m3x4_to_f16x2x2(v.x, h0, h1);
      e4m3x4_to_f16x2x2(v.y, h2, h3);
      uint4 o;
      o.x = bmul2(f16x2_to_bf16x2(h0), s2);
      o.y = bmul2(f16x2_to_bf16x2(h1), s2);
      o.z = bmul2(f16x2_to_bf16x2(h2), s2);
      o.w = bmul2(f16x2_to_bf16x2(h3), s2);
      *reinterpret_cast<uint4*>(dst + ((c ^ (r & 7)) << 4)) = o;
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint2 v = *reinterpret_cast<const uint2*>(src + q * 8);   // 16 values
      uint32_t h[8];
      e2m1x8_to_f16x2x4(v.x, h[0], h[1], h[2], h[3]);
      e2m1x8_to_f16x2x4(v.y, h[4], h[5], h[6], h[7]);
      uint32_t b[8];
      if (FMT == FMT_NVFP4) {
        // e2m1 x e4m3 in f16 is exact (<= 6 significant bits, |v| <= 2688, >= 2^-10)
        uint32_t sh0, sh1;
        e4m3x4_to_f16x2x2(scl, sh0, sh1);
        const uint32_t sq = (q & 1) ? splat_hi(q < 2 ? sh0 : sh1) : splat_lo(q < 2 ? sh0 : sh1);
#pragma unroll
        for (int e = 0; e < 8; ++e) b[e] = f16x2_to_bf16x2(hmul2_u32(h[e], sq));
      } else {
        // MXFP4: the power-of-two e8m0 scale of the 32 values (groups q/2), applied in bf16
        const uint32_t eb = (scl >> (8 * (q >> 1))) & 0xFFu;
        const uint32_t sbits = eb ? (eb << 7) : 0x0040u;          // 2^(eb-127) as bf16
        const uint32_t s2 = sbits | (sbits << 16);
#pragma unroll
        for (int e = 0; e < 8; ++e) b[e] = bmul2(f16x2_to_bf16x2(h[e]), s2);
      }
      const int c0 = 2 * q, c1 = 2 * q + 1;
      *reinterpret_cast<uint4*>(dst + ((c0 ^ (r & 7)) << 4)) = make_uint4(b[0], b[1], b[2], b[3]);
      *reinterpret_cast<uint4*>(dst + ((c1 ^ (r & 7)) << 4)) = make_uint4(b[4], b[5], b[6], b[7]);
    }
  }
}

template <int FMT_R>
__global__ void __launch_bounds__(NTHREADS, 2) tcw_kernel(const __grid_constant__ WideArgs wa) {
  const GroupedArgs& a = wa.g;
  extern __shared__ uint8_t dyn_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(dyn_raw) + 1023) & ~(uintptr_t)1023);
  int* err = a.err != nullptr ? a.err : &g_tcw_dense_err;
  volatile int* abort_flag = &sm.abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;

  if (tid == 0) {
    for (int s = 0; s < SC; ++s) {
      mbar_init(smem_addr(&sm.sfull[s]), 1);
      mbar_init(smem_addr(&sm.sempty[s]), 4);
    }
    for (int s = 0; s < SAR; ++s) {
      mbar_init(smem_addr(&sm.afull[s]), 4);
      mbar_init(smem_addr(&sm.aempty[s]), 1);
    }
    for (int s = 0; s < SBR; ++s) {
      mbar_init(smem_addr(&sm.bfull[s]), 1);
      mbar_init(smem_addr(&sm.bempty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_addr(&sm.accfull[s]), 1);
      mbar_init(smem_addr(&sm.accempty[s]), 4);
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
  const int nsub = K / 64;
  const int nrb = a.n_rows / 128;
  const int n_pass = (a.has_shared ? wa.plan.n_sh_pass : 0) +
                     (a.mode == MODE_DENSE ? 0 : wa.plan.pass_off[*a.n_active]);
  const int n_items = n_pass * nrb;
  const bool w13 = a.mode == MODE_W13;
  const int nb = wa.b_split ? 2 : 1;   // B tiles per sub-stage
  auto item_fmt = [&](const Item& it) { return it.shared ? (a.mode == MODE_DENSE ? FMT_R : FMT_FP8) : FMT_R; };
  auto pass_tokens = [&](const Item& it) { return min(WN, it.cnt - it.pb); };
  auto wait = [&](uint32_t bar, uint32_t parity) { return wait_bounded(abort_flag, err, bar, parity, WAIT_LIMIT); };
  auto warp_wait = [&](uint32_t bar, uint32_t parity) { return __all_sync(0xffffffffu, wait(bar, parity)); };

  if (warp == PRODUCER_WARP) {
    if (elect_one()) {
      prefetch_map(&wa.map_b);
      if (wa.use_w8) prefetch_map(&wa.map_w8);
      if (wa.use_w8_sh) prefetch_map(&wa.map_w8_sh);
    }
    __syncwarp();
    uint32_t c = 0, gb = 0;   // compact stages (staging ring), B tiles (B ring)
    bool ok = true;
    Item nxt = blockIdx.x < n_items ? item_of<FMT_R>(a, wa.plan, blockIdx.x, nrb) : Item{};
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
      const Item it = nxt;
      if (item + (int)gridDim.x < n_items) nxt = item_of<FMT_R>(a, wa.plan, item + gridDim.x, nrb);
      if (__any_sync(0xffffffffu, *reinterpret_cast<volatile int*>(err) != 0)) {
        *abort_flag = 1;
        break;
      }
      const int fmt = item_fmt(it);
      const bool fp4 = fmt != FMT_FP8;
      const WeightSet& ws = it.shared ? a.shared : a.routed;
      const int nst = K / 128;
      const uint32_t sb = fmt == FMT_NVFP4 ? 1024u : (fmt == FMT_MXFP4 ? 512u : 16u);
      const uint8_t* wbase = ws.w + (it.shared ? 0 : (size_t)it.expert * ws.w_stride) + (size_t)it.rb * nst * 8192;
      const uint8_t* sbase = ws.s + (it.shared ? 0 : (size_t)it.expert * ws.s_stride) + (size_t)it.rb * nst * sb;
      const int row8 = ((it.shared ? 0 : it.expert) * nrb + it.rb) * nst * 128;   // FP8 bank row of stage 0
      const CUtensorMap* map8 = it.shared ? &wa.map_w8_sh : &wa.map_w8;
      const int pc = pass_tokens(it);
      const int nbox = (pc + BOX_ROWS - 1) / BOX_ROWS;
      const int brow0 = it.shared ? P + it.pb : it.base + it.pb;
      for (int i = 0; i < nsub && ok; ++i) {
        if (!fp4 || (i & 1) == 0) {
          const uint32_t s = c % SC;
          if (!warp_wait(smem_addr(&sm.sempty[s]), ((c / SC) & 1u) ^ 1u)) {
            ok = false;
            break;
          }
          if (elect_one()) {
            const uint32_t bar = smem_addr(&sm.sfull[s]);
            mbar_expect_tx(bar, 8192u + sb);
            if (fp4) {
              bulk_g2s(smem_addr(sm.stg[s]), wbase + (size_t)(i >> 1) * 8192, 8192, bar);
              bulk_g2s(smem_addr(sm.stg[s] + STG_W), sbase + (size_t)(i >> 1) * sb, sb, bar);
            } else {
              tma_load_2d(smem_addr(sm.stg[s]), map8, (i & 1) * 64, row8 + (i >> 1) * 128, bar);
              bulk_g2s(smem_addr(sm.stg[s] + STG_W), sbase + (size_t)(i >> 1) * 16, 16, bar);
            }
          }
          __syncwarp();
          ++c;
        }
        for (int h = 0; h < nb; ++h, ++gb) {
          const uint32_t sbf = gb % SBR;
          if (!warp_wait(smem_addr(&sm.bempty[sbf]), ((gb / SBR) & 1u) ^ 1u)) {
            ok = false;
            break;
          }
          if (elect_one()) {
            const uint32_t bar = smem_addr(&sm.bfull[sbf]);
            const int row = brow0 + h * wa.b_lo_row;
            mbar_expect_tx(bar, (uint32_t)nbox * BOX_ROWS * 128u);
            for (int b = 0; b < nbox; ++b)
              tma_load_2d(smem_addr(sm.B[sbf] + b * BOX_ROWS * 128), &wa.map_b, i * 64, row + b * BOX_ROWS, bar);
          }
          __syncwarp();
        }
      }
    }
    // copies still in flight (only when a wait gave up) land before the CTA exits
    for (uint32_t h = c > (uint32_t)SC ? c - SC : 0; h < c; ++h)
      for (uint32_t i = 0; i < WAIT_LIMIT; ++i)
        if (mbar_try_wait(smem_addr(&sm.sfull[h % SC]), (h / SC) & 1u)) break;
    for (uint32_t h = gb > (uint32_t)SBR ? gb - SBR : 0; h < gb; ++h)
      for (uint32_t i = 0; i < WAIT_LIMIT; ++i)
        if (mbar_try_wait(smem_addr(&sm.bfull[h % SBR]), (h / SBR) & 1u)) break;
  } else if (warp == MMA_WARP) {
    uint32_t g = 0, gb = 0, np = 0;  // sub-stages (A ring), B tiles, passes (accumulator buffers)
    bool ok = true;
    Item nxt = blockIdx.x < n_items ? item_of<FMT_R>(a, wa.plan, blockIdx.x, nrb) : Item{};
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++np) {
      const Item it = nxt;
      if (item + (int)gridDim.x < n_items) nxt = item_of<FMT_R>(a, wa.plan, item + gridDim.x, nrb);
      const uint32_t n = (uint32_t)((pass_tokens(it) + 15) & ~15);
      const uint32_t id = idesc_bf16(n);
      const uint32_t buf = np & 1u;
      const uint32_t tacc = tbase + buf * WN;
      if (!warp_wait(smem_addr(&sm.accempty[buf]), ((np >> 1) & 1u) ^ 1u)) break;
      for (int i = 0; i < nsub && ok; ++i, ++g) {
        const uint32_t sa = g % SAR;
        if (!warp_wait(smem_addr(&sm.afull[sa]), (g / SAR) & 1u)) {
          ok = false;
          break;
        }
        const uint32_t abase = smem_addr(sm.A[sa]);
        for (int h = 0; h < nb; ++h, ++gb) {
          const uint32_t sbf = gb % SBR;
          if (!warp_wait(smem_addr(&sm.bfull[sbf]), (gb / SBR) & 1u)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t bbase = smem_addr(sm.B[sbf]);
          if (elect_one()) {
#pragma unroll
            for (int k = 0; k < 4; ++k)
              mma_f16(tacc, sdesc(abase + k * 32), sdesc(bbase + k * 32), id, (i > 0 || h > 0 || k > 0) ? 1u : 0u);
            commit(smem_addr(&sm.bempty[sbf]));
          }
          __syncwarp();
        }
        if (!ok) break;
        if (elect_one()) {
          commit(smem_addr(&sm.aempty[sa]));
          if (i == nsub - 1) commit(smem_addr(&sm.accfull[buf]));
        }
        __syncwarp();
      }
    }
    if (elect_one()) commit(smem_addr(&sm.drain));
    __syncwarp();
    for (uint32_t i = 0; i < WAIT_LIMIT; ++i)
      if (mbar_try_wait_sleep(smem_addr(&sm.drain), 0, 1000u)) break;
  } else {
    // ── convert + epilogue (warps 0-3): thread r = weight row r = TMEM lane r ──
    const int r = tid;
    uint32_t g = 0, c = 0, np = 0;
    bool ok = true;
    Item nxt = blockIdx.x < n_items ? item_of<FMT_R>(a, wa.plan, blockIdx.x, nrb) : Item{};
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++np) {
      const Item it = nxt;
      if (item + (int)gridDim.x < n_items) nxt = item_of<FMT_R>(a, wa.plan, item + gridDim.x, nrb);
      const int fmt = item_fmt(it);
      const bool fp4 = fmt != FMT_FP8;
      const WeightSet& ws = it.shared ? a.shared : a.routed;
      const int pc = pass_tokens(it);
      // the pass's tokens, 32 per chunk: lane t of chunk j holds token 32j + t's output row and weight
      int my_orow[WN / 32];
      float my_wgt[WN / 32];
#pragma unroll
      for (int j = 0; j < WN / 32; ++j) {
        my_orow[j] = 0;
        my_wgt[j] = 1.f;
        const int t = 32 * j + lane;
        if (t < pc) {
          const int i = it.pb + t;
          if (it.shared) {
            my_orow[j] = a.mode == MODE_DENSE ? i : P + i;
          } else {
            const int qp = it.base + i;
            const int tok = a.pair_tok[qp], slot = a.pair_slot[qp];
            if (w13) {
              my_orow[j] = qp;
              my_wgt[j] = a.topk_w[(size_t)tok * a.topk + slot];
            } else {
              my_orow[j] = tok * a.topk + slot;
            }
          }
        }
      }
      float ts = 1.f;
      if (fmt == FMT_NVFP4 && ws.ts != nullptr) {
        const float* tsp = ws.ts + (it.shared ? 0 : (size_t)it.expert * ws.ts_stride);
        ts = (w13 && r >= 64) ? tsp[1] : tsp[0];
      }
      // convert every sub-stage of the pass
      for (int i = 0; i < nsub; ++i, ++g) {
        const uint32_t s = c % SC, sa = g % SAR;
        if (!fp4 || (i & 1) == 0) {
          if (ok) ok = __all_sync(0xffffffffu, wait(smem_addr(&sm.sfull[s]), (c / SC) & 1u));
        }
        if (ok) ok = __all_sync(0xffffffffu, wait(smem_addr(&sm.aempty[sa]), ((g / SAR) & 1u) ^ 1u));
        if (ok) {
          const uint8_t* stg = sm.stg[s];
          uint8_t* dst = sm.A[sa] + r * 128;
          if (fmt == FMT_FP8) {
            const float* sw = reinterpret_cast<const float*>(stg + STG_W);
            convert_row<FMT_FP8>(stg + r * 64, 0u, w13 ? sw[r >= 64 ? 1 : 0] : sw[0], dst, r);
          } else if (fmt == FMT_NVFP4) {
            const uint32_t sc4 = *reinterpret_cast<const uint32_t*>(stg + STG_W + r * 8 + (i & 1) * 4);
            convert_row<FMT_NVFP4>(stg + r * 64 + (i & 1) * 32, sc4, 0.f, dst, r);
          } else {
            const uint32_t sc2 = *reinterpret_cast<const uint16_t*>(stg + STG_W + r * 4 + (i & 1) * 2);
            convert_row<FMT_MXFP4>(stg + r * 64 + (i & 1) * 32, sc2, 0.f, dst, r);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) arrive(smem_addr(&sm.afull[sa]));
        }
        if (!fp4 || (i & 1) == 1) {
          __syncwarp();
          if (ok && lane == 0) arrive(smem_addr(&sm.sempty[s]));
          ++c;
        }
      }
      // epilogue: this pass's accumulator -> h (W13, SwiGLU) or o (W2 / dense)
      const uint32_t buf = np & 1u;
      if (ok) ok = __all_sync(0xffffffffu, wait(smem_addr(&sm.accfull[buf]), (np >> 1) & 1u));
      if (bar1_any(!ok || *abort_flag)) break;
      fence_after();
      const uint32_t taddr = tbase + ((uint32_t)(warp * 32) << 16) + buf * WN;
      const int I = a.n_rows / 2;
#pragma unroll
      for (int j = 0; j < WN / 32; ++j) {
        if (32 * j >= pc) break;                       // uniform across the workers
        uint32_t d[32];
        ld32(taddr + 32 * j, d);
        ld_wait();
        if (w13) {
          if (r >= 64) {
#pragma unroll
            for (int t = 0; t < 32; ++t) sm.xchg[r - 64][t] = bf16_round(__uint_as_float(d[t]) * ts);
          }
          asm volatile("bar.sync 1, 128;\n" ::: "memory");
          if (r < 64) {
            const float lim = a.swiglu_limit;
#pragma unroll
            for (int t = 0; t < 32; ++t) {
              const int orow = __shfl_sync(0xffffffffu, my_orow[j], t);
              const float wgt = __shfl_sync(0xffffffffu, my_wgt[j], t);
              if (32 * j + t < pc) {
                float gv = bf16_round(__uint_as_float(d[t]) * ts);
                float uv = sm.xchg[r][t];
                if (lim > 0.f) {
                  uv = fminf(fmaxf(uv, -lim), lim);
                  gv = fminf(gv, lim);
                }
                float hv = silu(gv) * uv;
                if (!it.shared) hv = wgt * hv;
                a.hbf[(size_t)orow * I + it.rb * 64 + r] = __float2bfloat16_rn(hv);
              }
            }
          }
          asm volatile("bar.sync 1, 128;\n" ::: "memory");
        } else {
          const int n0 = it.rb * 128;
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            const int orow = __shfl_sync(0xffffffffu, my_orow[j], t);
            if (32 * j + t < pc) a.o[(size_t)orow * a.n_rows + n0 + r] = __float2bfloat16_rn(__uint_as_float(d[t]) * ts);
          }
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) arrive(smem_addr(&sm.accempty[buf]));
    }
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == MMA_WARP)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tbase), "r"(TMEM_COLS));
}

// ── activation matrices of the wide path (B operands) ──
// W13: row q < P = dequant(act_quant(x))[pair_tok[q]] (routed pairs in expert order), row P + i = the
// same of token i (the shared expert). W2: row q = dequant(act_quant(h))[q] for every row of h.
// dequant(act_quant(v)) = e4m3 code * its per-128 scale, formed in fp32. bf16 holds it exactly when
// the scale is a power of two; otherwise (split) rows `rows + q` hold the residual bf16(v - hi).
__device__ __forceinline__ void store_hi_lo(const float (&v)[8], __nv_bfloat16* hi, int64_t lo_off, int split) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __nv_bfloat162 b = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
    h[j] = *reinterpret_cast<const uint32_t*>(&b);
    const float2 bf = __bfloat1622float2(b);
    const __nv_bfloat162 r = __floats2bfloat162_rn(v[2 * j] - bf.x, v[2 * j + 1] - bf.y);
    l[j] = *reinterpret_cast<const uint32_t*>(&r);
  }
  *reinterpret_cast<uint4*>(hi) = make_uint4(h[0], h[1], h[2], h[3]);
  if (split) *reinterpret_cast<uint4*>(hi + lo_off) = make_uint4(l[0], l[1], l[2], l[3]);
}

__global__ void __launch_bounds__(256) wide_x_kernel(const uint8_t* __restrict__ xq, const float* __restrict__ xs,
                                                     const int32_t* __restrict__ pair_tok, int m, int P, int h,
                                                     int split, __nv_bfloat16* __restrict__ xw) {
  pdl_wait();
  pdl_trigger();
  const int nv = h / 8, nkb = h / 128;
  const int64_t rows = (int64_t)(P + m), units = rows * nv;
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < units; u += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(u / nv), v = (int)(u % nv);
    const int tok = row < P ? pair_tok[row] : row - P;
    const uint2 qv = *reinterpret_cast<const uint2*>(xq + (size_t)tok * h + v * 8);
    const float s = xs[(size_t)tok * nkb + (v * 8) / 128];
    uint32_t hh[4];
    e4m3x4_to_f16x2x2(qv.x, hh[0], hh[1]);
    e4m3x4_to_f16x2x2(qv.y, hh[2], hh[3]);
    float f[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&hh[j]));
      f[2 * j] = t.x * s;
      f[2 * j + 1] = t.y * s;
    }
    store_hi_lo(f, xw + (size_t)row * h + v * 8, rows * h, split);
  }
}

// one warp per (row, 128-block) of h: act_quant (kernel.py:40-125), then back to bf16 (hi, and the
// residual plane at rows + row when the scales are fp32)
__global__ void __launch_bounds__(256) wide_h_kernel(const __nv_bfloat16* __restrict__ hbf, int64_t rows, int k,
                                                     int pow2, __nv_bfloat16* __restrict__ hw) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int nkb = k / 128;
  const int64_t units = rows * nkb;
  for (int64_t u = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; u < units;
       u += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int64_t row = u / nkb;
    const int b = (int)(u % nkb);
    const uint2 raw = *reinterpret_cast<const uint2*>(hbf + row * k + b * 128 + lane * 4);
    const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&raw);
    const float2 f0 = __bfloat1622float2(p[0]), f1 = __bfloat1622float2(p[1]);
    float am = fmaxf(fmaxf(fabsf(f0.x), fabsf(f0.y)), fmaxf(fabsf(f1.x), fabsf(f1.y)));
    am = warp_max(am);
    const float sc = act_scale(am, pow2 != 0);
    float q[4];
    if (pow2) {
      const float inv = __frcp_rn(sc);   // exact: a power of two
      q[0] = e4m3_to_f32(act_q_pow2(f0.x, inv));
      q[1] = e4m3_to_f32(act_q_pow2(f0.y, inv));
      q[2] = e4m3_to_f32(act_q_pow2(f1.x, inv));
      q[3] = e4m3_to_f32(act_q_pow2(f1.y, inv));
    } else {
      q[0] = e4m3_to_f32(act_q(f0.x, sc));
      q[1] = e4m3_to_f32(act_q(f0.y, sc));
      q[2] = e4m3_to_f32(act_q(f1.x, sc));
      q[3] = e4m3_to_f32(act_q(f1.y, sc));
    }
    uint32_t hv[2], lv[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float v0 = q[2 * j] * sc, v1 = q[2 * j + 1] * sc;
      const __nv_bfloat162 hb = __floats2bfloat162_rn(v0, v1);
      const float2 hf = __bfloat1622float2(hb);
      const __nv_bfloat162 lb = __floats2bfloat162_rn(v0 - hf.x, v1 - hf.y);
      hv[j] = *reinterpret_cast<const uint32_t*>(&hb);
      lv[j] = *reinterpret_cast<const uint32_t*>(&lb);
    }
    *reinterpret_cast<uint2*>(hw + row * k + b * 128 + lane * 4) = make_uint2(hv[0], hv[1]);
    if (!pow2) *reinterpret_cast<uint2*>(hw + (rows + row) * k + b * 128 + lane * 4) = make_uint2(lv[0], lv[1]);
  }
}

// ── host side ──

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

static cudaError_t encode(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t rows,
                          uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw) {
  memset(map, 0, sizeof *map);
  if (base == nullptr || rows == 0) return cudaSuccess;
  PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
  if (enc == nullptr) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t es[2] = {1, 1};
  const CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int F>
static cudaError_t launch_one(const WideArgs& a, int grid, cudaStream_t st) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(tcw_kernel<F>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  return launch_pdl(tcw_kernel<F>, dim3(grid), dim3(NTHREADS), SMEM_BYTES, st, a);
}

}  // namespace tcw

cudaError_t launch_tc_wide(const GroupedArgs& g, const TcPlan& plan, const void* bmat, int64_t b_rows, int split,
                           int max_items, cudaStream_t st) {
  tcw::WideArgs a;
  a.g = g;
  a.plan = plan;
  a.b_split = split ? 1 : 0;
  a.b_lo_row = (int)b_rows;
  const uint64_t nst = (uint64_t)g.k / 128, nrb = (uint64_t)g.n_rows / 128;
  cudaError_t e = tcw::encode(&a.map_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, bmat, (uint64_t)g.k,
                              (uint64_t)b_rows * (split ? 2 : 1), (uint64_t)g.k * 2, 64, tcw::BOX_ROWS,
                              CU_TENSOR_MAP_SWIZZLE_128B);
  if (e != cudaSuccess) return e;
  const bool r8 = g.mode != MODE_DENSE && g.routed.fmt == FMT_FP8;
  e = tcw::encode(&a.map_w8, CU_TENSOR_MAP_DATA_TYPE_UINT8, r8 ? g.routed.w : nullptr, 128,
                  (uint64_t)g.n_experts * nrb * nst * 128, 128, 64, 128, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (e != cudaSuccess) return e;
  const bool s8 = g.has_shared && (g.mode != MODE_DENSE || g.shared.fmt == FMT_FP8);
  e = tcw::encode(&a.map_w8_sh, CU_TENSOR_MAP_DATA_TYPE_UINT8, s8 ? g.shared.w : nullptr, 128, nrb * nst * 128, 128,
                  64, 128, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (e != cudaSuccess) return e;
  a.use_w8 = r8 ? 1 : 0;
  a.use_w8_sh = s8 ? 1 : 0;
  int grid = 2 * num_sms();
  if (grid > max_items) grid = max_items;
  if (grid < 1) grid = 1;
  switch (g.routed.fmt) {
    case FMT_NVFP4: return tcw::launch_one<FMT_NVFP4>(a, grid, st);
    case FMT_MXFP4: return tcw::launch_one<FMT_MXFP4>(a, grid, st);
    default: return tcw::launch_one<FMT_FP8>(a, grid, st);
  }
}

cudaError_t launch_wide_x(const uint8_t* xq, const float* xs, const int32_t* pair_tok, int m, int P, int h, int split,
                          __nv_bfloat16* xw, cudaStream_t st) {
  const int64_t units = (int64_t)(P + m) * (h / 8);
  const int64_t b = (units + 255) / 256;
  const unsigned grid = (unsigned)(b < 1 ? 1 : (b > 65535 ? 65535 : b));
  return launch_pdl(tcw::wide_x_kernel, dim3(grid), dim3(256), 0, st, xq, xs, pair_tok, m, P, h, split, xw);
}

cudaError_t launch_wide_h(const __nv_bfloat16* hbf, int64_t rows, int k, int pow2, __nv_bfloat16* hw, cudaStream_t st) {
  const int64_t warps = rows * (k / 128);
  const int64_t b = (warps * 32 + 255) / 256;
  const unsigned grid = (unsigned)(b < 1 ? 1 : (b > 65535 ? 65535 : b));
  return launch_pdl(tcw::wide_h_kernel, dim3(grid), dim3(256), 0, st, hbf, rows, k, pow2, hw);
}

}  // namespace sb
