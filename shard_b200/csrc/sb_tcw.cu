// Grouped expert GEMM at prefill widths on the tensor cores (tcx_kernel): 16-bit operands and the
// whole K reduced in TMEM, so each pass is read back once (the verify-width kernel, sb_tc.cu, reads
// back per stage).
//
// Items are (pass, pair of 128-row blocks) over the same pass table as sb_tc.cu, with passes of up to
// WN = 128 tokens. The MMA is tcgen05.mma kind::f16 with the pass's tokens as its M side (128 TMEM
// lanes, one token per lane) and the item's 256 weight rows as its N side, K = 16 per instruction.
// Operands per 64-K sub-stage:
//   weights (B, shared memory)  a producer warp copies each stage in compact form (TMA, swizzled so
//      that thread r reading row r is free of bank conflicts) with its scales into a staging ring;
//      8 converter warps, one thread per weight row, dequantise it into a 128B-swizzled K-major
//      16-bit tile:
//        NVFP4  e2m1 x its e4m3 scale (per 16) in f16: exact (<= 6 significant bits, 2^-10..2688);
//               the fp32 tensor scale is applied in the epilogue;
//        FP8    e4m3 x its 128x128 block scale / c_A in f16, c_A = 16 x the item's first block
//               scale (a power of two for ue8m0 scales): exact while the row block's scales stay
//               within 2^+-11 of it; c_A is applied in the epilogue;
//        MXFP4  e2m1 x its e8m0 scale (per 32) in bf16: exact (e8m0 exceeds the f16 range).
//   tokens (A, shared memory)  a loader warp bulk-copies the pass's rows of the padded chunk-major
//      activation matrix (wide_x / wide_h kernels): dequant(act_quant(v)) = e4m3 x scale divided by a
//      power of two c_B per row (f16), exact for power-of-two activation scales; fp32 scales are
//      carried as two planes, hi = round(v) and lo = round(v - hi), both multiplied into the same
//      accumulator; K3-mode bf16 activations are copied as they are (bf16, c_B = 1).
// Two TMEM accumulators (128 lanes x 256 columns each) alternate across passes. The products are
// exact and the sum is fp32, the reference's dequant-then-fp32-matmul up to summation order. The
// epilogue (the converter warps; lane = token) scales by the powers of two c_A c_B and the NVFP4
// tensor scale; W13 pairs each gate column with its up column inside one thread (SwiGLU or situ),
// W2 writes o rows.
//
// One CTA per SM (352 threads), persistent over the items: warps 0-7 convert and run the epilogue,
// warp 8 weight producer, warp 9 MMA issuer (allocates TMEM), warp 10 token loader. The token ring's
// 16 KB slots hold the tiles of 4, 2 or 1 sub-stages (passes of <= 32, <= 64, <= 128 tokens). Every
// wait is bounded; on timeout the CTA records an error and winds down.
#include <cudaTypedefs.h>

#include "sb_launch.h"
#include "sb_tcgen05.cuh"

namespace sb {
namespace tcw {

using namespace tc5;

constexpr int NWORK = 8;                // converter / epilogue warps: one thread per weight row
constexpr int WN = TC_WIDE_PASS;        // tokens per pass
constexpr int STG_W = 8192;             // fp4: 128 rows x 64 B (128 K); FP8: 128 rows x 64 B (64 K)
constexpr int STG_S = 1024;             // NVFP4 [128][8 B], MXFP4 [128][4 B], FP8 16 B
constexpr int B_BYTES = WN * 128;       // a token tile slot: WN rows x 64 16-bit values
constexpr int BOX_ROWS = 32;
constexpr int BOX_BYTES = BOX_ROWS * 128;
constexpr uint32_t WAIT_LIMIT = 1u << 16;

struct WideArgs {
  CUtensorMap map_w4;       // fp4 routed bank as bytes [rows/2][128]: box 128 x 64, 128-byte swizzle
  CUtensorMap map_w8;       // FP8 routed bank as bytes [rows][128]: box 64 x 128, 64-byte swizzle
  CUtensorMap map_w8_sh;    // the FP8 shared expert, same form
  GroupedArgs g;
  TcPlan plan;
  const uint8_t* bmat;      // activations, chunk-major: [plane][k/64][r_pad][128 B], 128B-swizzled rows
  const float* cvec;        // [r_pad] the power of two c_B each B row was divided by
  int64_t r_pad;            // rows of the padded row space
  int sb_row;               // first row of the shared expert's tokens
  int use_w4, use_w8, use_w8_sh;   // which weight maps were encoded (the others stay zeroed)
  int b_split;              // B carries a residual plane (the second plane of bmat); passes <= 64
};

// Padded row space of the B matrices: expert e's rows start at pbase(offsets[e], e), a multiple of 8
// (its passes then start at multiples of 8 too); the shared expert's tokens follow at sb_row.
__host__ __device__ __forceinline__ int pbase(int off, int e) { return wide_pbase(off, e); }

struct Item {
  int shared, expert, rb, cnt, base, pb, pass;
};

__device__ __forceinline__ Item item_of(const GroupedArgs& a, const TcPlan& plan, int item, int nrb, int wn) {
  Item it;
  const int p = item / nrb;
  it.rb = item - p * nrb;
  it.pass = p;
  if (p < plan.n_sh_pass) {
    it.shared = 1;
    it.expert = 0;
    it.cnt = a.m;
    it.base = 0;
    it.pb = p * wn;
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

__device__ __forceinline__ uint32_t f16_splat(float v) {
  const __half2 h = __float2half2_rn(v);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// 16-byte chunk c (0-3) of staging row r. fp4 stages arrive as 64 rows of 128 B (weight rows 2q and
// 2q+1) with TMA's 128-byte swizzle (chunk index XOR q & 7); FP8 stages as 128 rows of 64 B with the
// 64-byte swizzle (chunk index XOR (r >> 1) & 3). Either way thread r reading row r is free of bank
// conflicts.
__device__ __forceinline__ uint4 stg_chunk(const uint8_t* stg, int r, int c) {
  return *reinterpret_cast<const uint4*>(stg + r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
}
__device__ __forceinline__ uint4 stg_chunk4(const uint8_t* stg, int r, int c) {
  const int q = r >> 1, cc = ((r & 1) << 2) | c;
  return *reinterpret_cast<const uint4*>(stg + q * 128 + ((cc ^ (q & 7)) << 4));
}

// Thread (row r, half hh) converts its row's values of one staging stage into 32-bit words (two
// 16-bit values each, K ascending). fp4 stages hold 128 K: the thread takes sub-stage hh
// (K 64hh .. 64hh+63, staging chunks 2hh, 2hh+1) -> 32 columns.
//   NVFP4: e2m1 x e4m3 group scale (scale bytes 4hh .. 4hh+3 of the row) in f16
__device__ __forceinline__ void convert_nvfp4(const uint8_t* stg, int r, int hh, uint32_t (&o)[32]) {
  const uint32_t sc4 = *reinterpret_cast<const uint32_t*>(stg + STG_W + r * 8 + hh * 4);
  uint32_t sh0, sh1;
  e4m3x4_to_f16x2x2(sc4, sh0, sh1);
  const uint32_t sq[4] = {splat_lo(sh0), splat_hi(sh0), splat_lo(sh1), splat_hi(sh1)};
#pragma unroll
  for (int cc = 0; cc < 2; ++cc) {
    const uint4 v = stg_chunk4(stg, r, 2 * hh + cc);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t* q = o + 16 * cc + 4 * j;
      e2m1x8_to_f16x2x4(w[j], q[0], q[1], q[2], q[3]);
      const uint32_t s = sq[2 * cc + (j >> 1)];
#pragma unroll
      for (int e = 0; e < 4; ++e) q[e] = hmul2_u32(q[e], s);
    }
  }
}

//   MXFP4: e2m1 x e8m0 group scale (scale bytes 2hh, 2hh+1) in bf16
__device__ __forceinline__ void convert_mxfp4(const uint8_t* stg, int r, int hh, uint32_t (&o)[32]) {
#pragma unroll
  for (int cc = 0; cc < 2; ++cc) {
    const uint32_t eb = stg[STG_W + mx_scale_off(r) + hh * 2 + cc];
    const uint32_t sbits = eb ? (eb << 7) : 0x0040u;          // 2^(eb-127) as bf16
    const uint32_t s2 = sbits | (sbits << 16);
    const uint4 v = stg_chunk4(stg, r, 2 * hh + cc);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t* q = o + 16 * cc + 4 * j;
      e2m1x8_to_f16x2x4(w[j], q[0], q[1], q[2], q[3]);
#pragma unroll
      for (int e = 0; e < 4; ++e) q[e] = bmul2(f16x2_to_bf16x2(q[e]), s2);
    }
  }
}

//   FP8 stages hold 64 K (one sub-stage): the thread takes K 32hh .. 32hh+31 (chunks 2hh, 2hh+1)
//   -> 16 columns, e4m3 x (block scale / c_A) in f16 (s2)
__device__ __forceinline__ void convert_fp8(const uint8_t* stg, int r, int hh, uint32_t s2, uint32_t (&o)[16]) {
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const uint4 v = stg_chunk(stg, r, 2 * hh + c);
    uint32_t* q = o + 8 * c;
    e4m3x4_to_f16x2x2(v.x, q[0], q[1]);
    e4m3x4_to_f16x2x2(v.y, q[2], q[3]);
    e4m3x4_to_f16x2x2(v.z, q[4], q[5]);
    e4m3x4_to_f16x2x2(v.w, q[6], q[7]);
#pragma unroll
    for (int e = 0; e < 8; ++e) q[e] = hmul2_u32(q[e], s2);
  }
}

// B slot geometry of a pass of pc tokens: boxes of 32 rows per sub-stage tile (rounded up to a power
// of two, so that tiles tile a 16 KB slot), and the sub-stages one slot holds
struct BGeom {
  int nbox, nboxp, spb;
};
__device__ __forceinline__ BGeom bgeom(int pc, int nb) {
  BGeom b;
  b.nbox = (pc + BOX_ROWS - 1) / BOX_ROWS;
  b.nboxp = b.nbox <= 1 ? 1 : (b.nbox <= 2 ? 2 : 4);
  b.spb = (B_BYTES / BOX_BYTES) / (b.nboxp * nb);
  return b;
}


// ── the prefill kernel ──
namespace x {
constexpr int NEPI = 4;                      // epilogue warps: one per TMEM lane quarter (token = lane)
constexpr int NTHREADS = 32 * (NWORK + 3 + NEPI);
constexpr int PRODUCER_WARP = NWORK, MMA_WARP = NWORK + 1, TLOAD_WARP = NWORK + 2;   // then the epilogue warps
constexpr int ROWS = 256;                    // weight rows per item (two 128-row blocks) = MMA N
constexpr int SC = 3;                        // staging ring: one stage of both row blocks per slot
constexpr int SW = 3;                        // f16 weight tiles (64 K each)
constexpr int STT = 3;                       // token tiles: 16 KB slots of 4, 2 or 1 sub-stages
constexpr int STG_RB = STG_W + STG_S;        // one row block's staging bytes (9 KB, 1024-aligned)
constexpr int W_BYTES = ROWS * 128;
constexpr int T_BYTES = WN * 128;
constexpr int TMEM_COLS = 2 * ROWS;          // two accumulators of 128 token lanes x 256 columns

struct Smem {
  uint8_t W[SW][W_BYTES];                    // 1024-aligned (128B swizzle atoms)
  uint8_t T[STT][T_BYTES];
  uint8_t stg[SC][2 * STG_RB];
  float ca[2][ROWS];                         // FP8: c_A of each weight row, per accumulator buffer
  uint64_t sfull[SC], sempty[SC], wfull[SW], wempty[SW], tfull[STT], tempty[STT], accfull[2], accempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};
constexpr int SMEM_BYTES = (int)sizeof(Smem) + 1024;
static_assert(SMEM_BYTES <= 232448, "shared memory of one CTA per SM");

template <int FMT_R, bool PROBE>
__global__ void __launch_bounds__(NTHREADS, 1) tcx_kernel(const __grid_constant__ WideArgs wa) {
  const GroupedArgs& a = wa.g;
  extern __shared__ uint8_t dyn_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(dyn_raw) + 1023) & ~(uintptr_t)1023);
  int* err = a.err != nullptr ? a.err : &g_tcw_dense_err;
  volatile int* abort_flag = &sm.abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;

  if (tid == 0) {
    for (int s = 0; s < SC; ++s) {
      mbar_init(smem_addr(&sm.sfull[s]), 1);
      mbar_init(smem_addr(&sm.sempty[s]), NWORK);
    }
    for (int s = 0; s < SW; ++s) {
      mbar_init(smem_addr(&sm.wfull[s]), NWORK);
      mbar_init(smem_addr(&sm.wempty[s]), 1);
    }
    for (int s = 0; s < STT; ++s) {
      mbar_init(smem_addr(&sm.tfull[s]), 1);
      mbar_init(smem_addr(&sm.tempty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_addr(&sm.accfull[s]), 1);
      mbar_init(smem_addr(&sm.accempty[s]), NEPI);
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
  pdl_wait();
  pdl_trigger();

  const int P = a.m * a.topk;
  const int K = a.k;
  const int nsub = K / 64;
  const int nst = K / 128;
  const int nrb = a.n_rows / 128;
  const int nrp = nrb / 2;                        // row-block pairs per matrix (nrb is even)
  const int nb = wa.b_split ? 2 : 1;
  const int wn = wa.b_split ? WN / 2 : WN;
  const int n_pass = (a.has_shared ? wa.plan.n_sh_pass : 0) + wa.plan.pass_off[*a.n_active];
  const int n_items = n_pass * nrp;
  const bool w13 = a.mode == MODE_W13;
  auto item_fmt = [&](const Item& it) { return it.shared ? FMT_FP8 : FMT_R; };
  auto pass_tokens = [&](const Item& it) { return min(wn, it.cnt - it.pb); };
  auto wait = [&](uint32_t bar, uint32_t parity) { return wait_bounded(abort_flag, err, bar, parity, WAIT_LIMIT); };
  auto warp_wait = [&](uint32_t bar, uint32_t parity) { return __all_sync(0xffffffffu, wait(bar, parity)); };
  // consumer-side waits (the MMA issuer's on its operands, the converters' on the staging copies and
  // the epilogue's on the accumulator) take the launch's limit; waits for free slots and the final
  // drains keep WAIT_LIMIT
  const uint32_t clim = a.wait_limit ? a.wait_limit : WAIT_LIMIT;
  auto cwait = [&](uint32_t bar, uint32_t parity) { return wait_bounded<PROBE>(abort_flag, err, bar, parity, clim); };

  if (warp == PRODUCER_WARP) {
    // both row blocks' weight stages (TMA) and their scales (bulk copies) into one staging slot
    if (elect_one()) {
      if (wa.use_w4) prefetch_map(&wa.map_w4);
      if (wa.use_w8) prefetch_map(&wa.map_w8);
      if (wa.use_w8_sh) prefetch_map(&wa.map_w8_sh);
    }
    __syncwarp();
    uint32_t c = 0;
    bool ok = true;
    Item nxt = blockIdx.x < n_items ? item_of(a, wa.plan, blockIdx.x, nrp, wn) : Item{};
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
      const Item it = nxt;
      if (item + (int)gridDim.x < n_items) nxt = item_of(a, wa.plan, item + gridDim.x, nrp, wn);
      if (__any_sync(0xffffffffu, *reinterpret_cast<volatile int*>(err) != 0)) {
        *abort_flag = 1;
        break;
      }
      const int fmt = item_fmt(it);
      const bool fp4 = fmt != FMT_FP8;
      const WeightSet& ws = it.shared ? a.shared : a.routed;
      const uint32_t sb = fmt == FMT_NVFP4 ? 1024u : (fmt == FMT_MXFP4 ? 512u : 16u);
      const CUtensorMap* mapw = fp4 ? &wa.map_w4 : (it.shared ? &wa.map_w8_sh : &wa.map_w8);
      const int nstg = fp4 ? nst : nsub;
      for (int st = 0; st < nstg; ++st, ++c) {
        const uint32_t s = c % SC;
        if (!warp_wait(smem_addr(&sm.sempty[s]), ((c / SC) & 1u) ^ 1u)) {
          ok = false;
          break;
        }
        if (elect_one()) {
          const uint32_t bar = smem_addr(&sm.sfull[s]);
          mbar_expect_tx(bar, 2u * (8192u + sb));
          for (int h = 0; h < 2; ++h) {
            const int rb = 2 * it.rb + h;
            const int row0 = ((it.shared ? 0 : it.expert) * nrb + rb) * nst * 128;
            const uint8_t* sbase = ws.s + (it.shared ? 0 : (size_t)it.expert * ws.s_stride) + (size_t)rb * nst * sb;
            const uint32_t dst = smem_addr(sm.stg[s] + h * STG_RB);
            if (fp4)
              tma_load_2d(dst, mapw, 0, (row0 >> 1) + st * 64, bar);
            else
              tma_load_2d(dst, mapw, (st & 1) * 64, row0 + (st >> 1) * 128, bar);
            bulk_g2s(dst + STG_W, sbase + (size_t)(fp4 ? st : st >> 1) * sb, sb, bar);
          }
        }
        __syncwarp();
      }
    }
    for (uint32_t h = c > (uint32_t)SC ? c - SC : 0; h < c; ++h)
      for (uint32_t i = 0; i < WAIT_LIMIT; ++i)
        if (mbar_try_wait(smem_addr(&sm.sfull[h % SC]), (h / SC) & 1u)) break;
  } else if (warp == TLOAD_WARP) {
    // token tiles: one bulk copy per sub-stage and plane
    uint32_t gt = 0;
    bool ok = true;
    const size_t plane = (size_t)(K / 64) * (size_t)wa.r_pad * 128;
    Item nxt = blockIdx.x < n_items ? item_of(a, wa.plan, blockIdx.x, nrp, wn) : Item{};
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
      const Item it = nxt;
      if (item + (int)gridDim.x < n_items) nxt = item_of(a, wa.plan, item + gridDim.x, nrp, wn);
      const int pc = pass_tokens(it);
      const BGeom bg = bgeom(pc, nb);
      const int brow0 = it.shared ? wa.sb_row + it.pb : pbase(it.base, it.expert) + it.pb;
      const uint32_t bytes = (uint32_t)((pc + 7) & ~7) * 128u;
      for (int i = 0; i < nsub; i += bg.spb, ++gt) {
        const uint32_t ts = gt % STT;
        if (!warp_wait(smem_addr(&sm.tempty[ts]), ((gt / STT) & 1u) ^ 1u)) {
          ok = false;
          break;
        }
        const int cnt = min(bg.spb, nsub - i);
        if (elect_one()) {
          const uint32_t bar = smem_addr(&sm.tfull[ts]);
          mbar_expect_tx(bar, (uint32_t)(cnt * nb) * bytes);
          for (int j = 0; j < cnt; ++j)
            for (int h = 0; h < nb; ++h)
              bulk_g2s(smem_addr(sm.T[ts] + (j * nb + h) * bg.nboxp * BOX_BYTES),
                       wa.bmat + h * plane + ((size_t)(i + j) * wa.r_pad + brow0) * 128, bytes, bar);
        }
        __syncwarp();
      }
    }
    for (uint32_t h = gt > (uint32_t)STT ? gt - STT : 0; h < gt; ++h)
      for (uint32_t i = 0; i < WAIT_LIMIT; ++i)
        if (mbar_try_wait(smem_addr(&sm.tfull[h % STT]), (h / STT) & 1u)) break;
  } else if (warp == MMA_WARP) {
    // one thread: per sub-stage 4 tcgen05.mma M=128 (tokens) x N=256 (weight rows) x K=16
    if (lane == 0) {
      uint32_t gw = 0, gt = 0, np = 0;
      bool ok = true;
      Item nxt = blockIdx.x < n_items ? item_of(a, wa.plan, blockIdx.x, nrp, wn) : Item{};
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++np) {
        const Item it = nxt;
        if (item + (int)gridDim.x < n_items) nxt = item_of(a, wa.plan, item + gridDim.x, nrp, wn);
        const int pc = pass_tokens(it);
        const BGeom bg = bgeom(pc, nb);
        const uint32_t id = item_fmt(it) == FMT_MXFP4 ? idesc_bf16(ROWS) : idesc_f16(ROWS);
        const uint32_t buf = np & 1u;
        const uint32_t tacc = tbase + buf * ROWS;
        const uint32_t tile = (uint32_t)(nb * bg.nboxp * BOX_BYTES);
        if (!wait(smem_addr(&sm.accempty[buf]), ((np >> 1) & 1u) ^ 1u)) break;
        for (int i = 0; i < nsub && ok; ++i, ++gw) {
          const uint32_t sws = gw % SW, ts = gt % STT;
          const int j = i & (bg.spb - 1);
          if (!cwait(smem_addr(&sm.wfull[sws]), (gw / SW) & 1u) ||
              (j == 0 && !cwait(smem_addr(&sm.tfull[ts]), (gt / STT) & 1u))) {
            ok = false;
            break;
          }
          fence_after();
          const uint64_t bd = sdesc(smem_addr(sm.W[sws]));
          for (int h = 0; h < nb; ++h) {
            const uint64_t ad = sdesc(smem_addr(sm.T[ts]) + (uint32_t)j * tile + (uint32_t)h * (tile / nb));
#pragma unroll
            for (int k = 0; k < 4; ++k)
              mma_f16(tacc, ad + 2 * k, bd + 2 * k, id, (i > 0 || h > 0 || k > 0) ? 1u : 0u);
          }
          commit(smem_addr(&sm.wempty[sws]));
          if (j == bg.spb - 1 || i == nsub - 1) {
            commit(smem_addr(&sm.tempty[ts]));
            ++gt;
          }
          if (i == nsub - 1) commit(smem_addr(&sm.accfull[buf]));
        }
      }
      commit(smem_addr(&sm.drain));
      for (uint32_t i = 0; i < WAIT_LIMIT; ++i)
        if (mbar_try_wait_sleep(smem_addr(&sm.drain), 0, 1000u)) break;
    }
    __syncwarp();
  } else if (warp < NWORK) {
    // ── convert (thread t = weight row t of the item's 256) ──
    const int t = tid, hb = t >> 7, r = t & 127;
    uint32_t c = 0, gw = 0, np = 0;
    bool ok = true;
    Item nxt = blockIdx.x < n_items ? item_of(a, wa.plan, blockIdx.x, nrp, wn) : Item{};
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++np) {
      const Item it = nxt;
      if (item + (int)gridDim.x < n_items) nxt = item_of(a, wa.plan, item + gridDim.x, nrp, wn);
      const int fmt = item_fmt(it);
      const bool fp4 = fmt != FMT_FP8;
      const int pc = pass_tokens(it);
      const int brow0 = it.shared ? wa.sb_row + it.pb : pbase(it.base, it.expert) + it.pb;
      // ca[buf] is read by the epilogue of the item two before this one: wait until it is done
      const uint32_t cbuf = np & 1u;
      if (ok) ok = __all_sync(0xffffffffu, wait(smem_addr(&sm.accempty[cbuf]), ((np >> 1) & 1u) ^ 1u));
      float ica = 1.f;
      if (fmt != FMT_FP8) sm.ca[cbuf][t] = 1.f;
      const int nstg = fp4 ? nst : nsub;
      for (int st = 0; st < nstg; ++st, ++c) {
        const uint32_t s = c % SC;
        if (ok) ok = __all_sync(0xffffffffu, cwait(smem_addr(&sm.sfull[s]), (c / SC) & 1u));
        const uint8_t* stg = sm.stg[s] + hb * STG_RB;
        uint32_t s2 = 0;
        if (ok && fmt == FMT_FP8) {
          const float sw = reinterpret_cast<const float*>(stg + STG_W)[w13 && r >= 64 ? 1 : 0];
          if (st == 0) {
            const float ca = sw > 0.f ? sw * 16.f : 1.f;
            ica = 1.f / ca;
            sm.ca[cbuf][t] = ca;
          }
          s2 = f16_splat(sw * ica);
        }
        for (int u = 0; u < (fp4 ? 2 : 1); ++u, ++gw) {
          const uint32_t sws = gw % SW;
          // convert into registers first, then claim the tile slot: a slot is held only for the
          // stores, which shortens its round trip through the MMA and back
          uint32_t o[32];
          if (!ok) continue;
          if (fmt == FMT_FP8) {
            uint32_t o0[16], o1[16];
            convert_fp8(stg, r, 0, s2, o0);
            convert_fp8(stg, r, 1, s2, o1);
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              o[e] = o0[e];
              o[16 + e] = o1[e];
            }
          } else if (fmt == FMT_NVFP4) {
            convert_nvfp4(stg, r, u, o);
          } else {
            convert_mxfp4(stg, r, u, o);
          }
          ok = __all_sync(0xffffffffu, wait(smem_addr(&sm.wempty[sws]), ((gw / SW) & 1u) ^ 1u));
          if (!ok) continue;
          uint8_t* dst = sm.W[sws] + t * 128;
#pragma unroll
          for (int k = 0; k < 8; ++k)
            *reinterpret_cast<uint4*>(dst + ((k ^ (t & 7)) << 4)) = make_uint4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) arrive(smem_addr(&sm.wfull[sws]));
        }
        __syncwarp();
        if (ok && lane == 0) arrive(smem_addr(&sm.sempty[s]));
      }
    }
  } else {
    // ── epilogue (the last NEPI warps): TMEM lane = token 32 (warp & 3) + lane, both row blocks of the
    // item in turn; it runs while the converters and the MMA work on the next item ──
    const int tok = (warp & 3) * 32 + lane;
    uint32_t np = 0;
    bool ok = true;
    Item nxt = blockIdx.x < n_items ? item_of(a, wa.plan, blockIdx.x, nrp, wn) : Item{};
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++np) {
      const Item it = nxt;
      if (item + (int)gridDim.x < n_items) nxt = item_of(a, wa.plan, item + gridDim.x, nrp, wn);
      const int fmt = item_fmt(it);
      const WeightSet& ws = it.shared ? a.shared : a.routed;
      const int pc = pass_tokens(it);
      const int brow0 = it.shared ? wa.sb_row + it.pb : pbase(it.base, it.expert) + it.pb;
      // the per-token values first: their latency overlaps the wait for the accumulator
      const bool valid = tok < pc;
      float cb = 1.f, wgt = 1.f;
      int orow = 0;
      if (valid) {
        const int i = it.pb + tok;
        cb = wa.cvec[brow0 + tok];
        if (w13) {
          orow = brow0 + tok;
          if (!it.shared) {
            const int qp = it.base + i;
            wgt = a.topk_w[(size_t)a.pair_tok[qp] * a.topk + a.pair_slot[qp]];
          }
        } else if (it.shared) {
          orow = P + i;
        } else {
          const int qp = it.base + i;
          orow = a.pair_tok[qp] * a.topk + a.pair_slot[qp];
        }
      }
      float ts0 = 1.f, ts1 = 1.f;   // NVFP4 tensor scales: w1 (or w2) rows, w3 rows
      if (fmt == FMT_NVFP4 && ws.ts != nullptr) {
        const float* tsp = ws.ts + (it.shared ? 0 : (size_t)it.expert * ws.ts_stride);
        ts0 = tsp[0];
        ts1 = w13 ? tsp[1] : tsp[0];
      }
      const uint32_t buf = np & 1u;
      if (ok) ok = __all_sync(0xffffffffu, cwait(smem_addr(&sm.accfull[buf]), (np >> 1) & 1u));
      if (bar_any(2, 32 * NEPI, !ok || *abort_flag)) break;
      fence_after();
      for (int hh = 0; hh < 2; ++hh) {
        const int rb = 2 * it.rb + hh;
        const uint32_t taddr = tbase + ((uint32_t)((warp & 3) * 32) << 16) + buf * ROWS + 128 * hh;
        const float* cav = sm.ca[buf] + 128 * hh;
        if (w13) {
          const int I = a.n_rows / 2;
          const float lim = a.swiglu_limit;
#pragma unroll
          for (int c0 = 0; c0 < 64; c0 += 32) {
            uint32_t gd[32], ud[32];
            ld32(taddr + c0, gd);
            ld32(taddr + 64 + c0, ud);
            ld_wait();
            uint32_t hv[16];
#pragma unroll
            for (int q = 0; q < 32; q += 2) {
              float h2[2];
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                float gv = bf16_round(__uint_as_float(gd[q + e]) * cb * (cav[c0 + q + e] * ts0));
                float uv = bf16_round(__uint_as_float(ud[q + e]) * cb * (cav[64 + c0 + q + e] * ts1));
                float hvv;
                if (a.activation == ACT_SITU) {
                  hvv = situ(gv, uv, a.act_beta, a.act_lbeta);
                } else {
                  if (lim > 0.f) {
                    uv = fminf(fmaxf(uv, -lim), lim);
                    gv = fminf(gv, lim);
                  }
                  hvv = silu(gv) * uv;
                }
                if (!it.shared && !a.weight_after) hvv = wgt * hvv;
                h2[e] = hvv;
              }
              const __nv_bfloat162 b = __floats2bfloat162_rn(h2[0], h2[1]);
              hv[q / 2] = *reinterpret_cast<const uint32_t*>(&b);
            }
            if (valid) {
              uint4* dst = reinterpret_cast<uint4*>(a.hbf + (size_t)orow * I + rb * 64 + c0);
#pragma unroll
              for (int v = 0; v < 4; ++v) dst[v] = make_uint4(hv[4 * v], hv[4 * v + 1], hv[4 * v + 2], hv[4 * v + 3]);
            }
          }
        } else {
#pragma unroll
          for (int c0 = 0; c0 < 128; c0 += 32) {
            uint32_t d[32];
            ld32(taddr + c0, d);
            ld_wait();
            uint32_t ov[16];
#pragma unroll
            for (int q = 0; q < 32; q += 2) {
              const __nv_bfloat162 b = __floats2bfloat162_rn(__uint_as_float(d[q]) * cb * (cav[c0 + q] * ts0),
                                                             __uint_as_float(d[q + 1]) * cb * (cav[c0 + q + 1] * ts0));
              ov[q / 2] = *reinterpret_cast<const uint32_t*>(&b);
            }
            if (valid) {
              uint4* dst = reinterpret_cast<uint4*>(a.o + (size_t)orow * a.n_rows + rb * 128 + c0);
#pragma unroll
              for (int v = 0; v < 4; ++v) dst[v] = make_uint4(ov[4 * v], ov[4 * v + 1], ov[4 * v + 2], ov[4 * v + 3]);
            }
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
}  // namespace x

// ── activation matrices of the wide path (B operands), one warp per row ──
// Row space: routed pair q of expert e at pbase(offsets[e], e) + (q - offsets[e]), the shared
// expert's token i at sb_row + i (W13: the same x row; W2: the rows of h, which the W13 epilogue
// writes in this row space). Layout chunk-major: [plane][k/64][r_pad][64 values], the 16-byte chunk
// c of a row's 64-K chunk stored at position c ^ (row & 7).
// The values: dequant(act_quant(v)) = e4m3 code x its per-128 scale, formed in fp32 and divided by
// the row's c_B (cvec[row]): f16 rows use c_B = 2^ceil(log2(max scale)) / 128, bf16 rows (routed
// rows of MXFP4 layers) c_B = 1. Exact in 16 bits for power-of-two scales; otherwise (split) the
// second plane holds the residuals v - hi.
template <bool BF>
__device__ __forceinline__ void store_hi_lo(const float (&v)[8], uint16_t* hi, int64_t lo_off, int split) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (BF) {
      const __nv_bfloat162 b = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
      const float2 back = __bfloat1622float2(b);
      const __nv_bfloat162 rr = __floats2bfloat162_rn(v[2 * j] - back.x, v[2 * j + 1] - back.y);
      h[j] = *reinterpret_cast<const uint32_t*>(&b);
      l[j] = *reinterpret_cast<const uint32_t*>(&rr);
    } else {
      const __half2 b = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
      const float2 back = __half22float2(b);
      const __half2 rr = __floats2half2_rn(v[2 * j] - back.x, v[2 * j + 1] - back.y);
      h[j] = *reinterpret_cast<const uint32_t*>(&b);
      l[j] = *reinterpret_cast<const uint32_t*>(&rr);
    }
  }
  *reinterpret_cast<uint4*>(hi) = make_uint4(h[0], h[1], h[2], h[3]);
  if (split) *reinterpret_cast<uint4*>(hi + lo_off) = make_uint4(l[0], l[1], l[2], l[3]);
}

// element offset of the 8-value chunk v (k = 8v .. 8v+7) of row `row`
__device__ __forceinline__ int64_t cm_off(int64_t row, int v, int64_t r_pad) {
  return ((int64_t)(v >> 3) * r_pad + row) * 64 + (((v & 7) ^ (int)(row & 7)) << 3);
}

__device__ __forceinline__ float row_c(float smax, bool bf) { return bf ? 1.f : pow2_ceil(smax) * (1.f / 128.f); }

__global__ void __launch_bounds__(256) wide_x_kernel(const uint8_t* __restrict__ xq, const float* __restrict__ xs,
                                                     const int32_t* __restrict__ pair_tok,
                                                     const int32_t* __restrict__ offsets, int n_experts, int m, int P,
                                                     int h, int64_t r_pad, int sb_row, int split, int routed_bf16,
                                                     int hot_min, uint16_t* __restrict__ xw,
                                                     float* __restrict__ cvec) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int nkb = h / 128;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t q = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; q < P + m; q += nw) {
    int tok, row;
    if (q < P) {
      int lo = 0, hi = n_experts;   // the expert of pair q: the last e with offsets[e] <= q
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (offsets[mid] <= q) lo = mid; else hi = mid;
      }
      // hybrid dispatch: only the hot experts' rows are read by the prefill kernel
      if (hot_min > 0 && offsets[lo + 1] - offsets[lo] < hot_min) continue;
      tok = pair_tok[q];
      row = pbase(offsets[lo], lo) + (int)(q - offsets[lo]);
    } else {
      tok = (int)(q - P);
      row = sb_row + tok;
    }
    const bool bf = routed_bf16 && q < P;
    const float* sr = xs + (size_t)tok * nkb;
    float smax = 0.f;
    for (int b = lane; b < nkb; b += 32) smax = fmaxf(smax, sr[b]);
    const float cb = row_c(warp_max(smax), bf);
    const float icb = 1.f / cb;   // a power of two
    for (int v = lane; v < h / 8; v += 32) {
      const uint2 qv = *reinterpret_cast<const uint2*>(xq + (size_t)tok * h + v * 8);
      const float s = sr[v >> 4] * icb;
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
      if (bf)
        store_hi_lo<true>(f, xw + cm_off(row, v, r_pad), r_pad * h, split);
      else
        store_hi_lo<false>(f, xw + cm_off(row, v, r_pad), r_pad * h, split);
    }
    if (lane == 0) cvec[row] = cb;
  }
}

// act_quant (kernel.py:40-125) of row `row` of h (rows of the padded row space; padding rows hold
// no data and their results are never read), block by block, then back to 16 bits: lane l holds
// values 4l..4l+3 of each 128-block; a first sweep finds the row's largest scale (for c_B)
__global__ void __launch_bounds__(256) wide_h_kernel(const __nv_bfloat16* __restrict__ hbf, int64_t rows,
                                                     int64_t r_pad, int sb_row, int k, int pow2, int routed_bf16,
                                                     const int32_t* __restrict__ offsets, int n_experts, int hot_min,
                                                     int sh_rows, uint16_t* __restrict__ hw,
                                                     float* __restrict__ cvec) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int nkb = k / 128;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; row < rows; row += nw) {
    if (hot_min > 0) {
      // hybrid dispatch: only the rows the prefill kernel reads, those of hot experts (and of the
      // shared expert when it runs there)
      if (row >= sb_row) {
        if (row >= (int64_t)sb_row + sh_rows) continue;
      } else {
        int lo = 0, hi = n_experts;   // the last e whose padded rows start at or before row
        while (hi - lo > 1) {
          const int mid = (lo + hi) >> 1;
          if (pbase(offsets[mid], mid) <= row) lo = mid; else hi = mid;
        }
        const int cnt = offsets[lo + 1] - offsets[lo];
        if (cnt < hot_min || row - pbase(offsets[lo], lo) >= cnt) continue;
      }
    }
    const bool bf = routed_bf16 && row < sb_row;
    const __nv_bfloat16* hr = hbf + row * k;
    // the block's 4 values of this lane, and the block's amax
    auto load = [&](int b, float (&f)[4]) {
      const uint2 raw = *reinterpret_cast<const uint2*>(hr + b * 128 + lane * 4);
      const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&raw);
      const float2 f0 = __bfloat1622float2(p[0]), f1 = __bfloat1622float2(p[1]);
      f[0] = f0.x;
      f[1] = f0.y;
      f[2] = f1.x;
      f[3] = f1.y;
      return warp_max(fmaxf(fmaxf(fabsf(f[0]), fabsf(f[1])), fmaxf(fabsf(f[2]), fabsf(f[3]))));
    };
    float smax = 0.f;
    for (int b = 0; b < nkb; ++b) {
      float f[4];
      smax = fmaxf(smax, act_scale(load(b, f), pow2 != 0));
    }
    const float cb = row_c(smax, bf);
    const float icb = 1.f / cb;
    for (int b = 0; b < nkb; ++b) {
      float f[4];
      const float sc = act_scale(load(b, f), pow2 != 0);
      float q[4];
      if (pow2) {
        const float inv = __frcp_rn(sc);   // exact: a power of two
#pragma unroll
        for (int e = 0; e < 4; ++e) q[e] = e4m3_to_f32(act_q_pow2(f[e], inv));
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) q[e] = e4m3_to_f32(act_q(f[e], sc));
      }
      const float s = sc * icb;
      uint32_t hv[2], lv[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float v0 = q[2 * j] * s, v1 = q[2 * j + 1] * s;
        if (bf) {
          const __nv_bfloat162 hb = __floats2bfloat162_rn(v0, v1);
          const float2 hf = __bfloat1622float2(hb);
          const __nv_bfloat162 lb = __floats2bfloat162_rn(v0 - hf.x, v1 - hf.y);
          hv[j] = *reinterpret_cast<const uint32_t*>(&hb);
          lv[j] = *reinterpret_cast<const uint32_t*>(&lb);
        } else {
          const __half2 hb = __floats2half2_rn(v0, v1);
          const float2 hf = __half22float2(hb);
          const __half2 lb = __floats2half2_rn(v0 - hf.x, v1 - hf.y);
          hv[j] = *reinterpret_cast<const uint32_t*>(&hb);
          lv[j] = *reinterpret_cast<const uint32_t*>(&lb);
        }
      }
      // values 4 lane .. 4 lane + 3 of block b: half of an 8-value chunk
      const int v = b * 16 + (lane >> 1);
      const int64_t off = cm_off(row, v, r_pad) + (lane & 1) * 4;
      *reinterpret_cast<uint2*>(hw + off) = make_uint2(hv[0], hv[1]);
      if (!pow2) *reinterpret_cast<uint2*>(hw + off + r_pad * k) = make_uint2(lv[0], lv[1]);
    }
    if (lane == 0) cvec[row] = cb;
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

template <int F, bool PROBE>
static cudaError_t launch_variant(const WideArgs& a, int grid, cudaStream_t st) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e =
        cudaFuncSetAttribute(x::tcx_kernel<F, PROBE>, cudaFuncAttributeMaxDynamicSharedMemorySize, x::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  return launch_pdl(x::tcx_kernel<F, PROBE>, dim3(grid), dim3(x::NTHREADS), x::SMEM_BYTES, st, a);
}

template <int F>
static cudaError_t launch_one(const WideArgs& a, int grid, cudaStream_t st) {
  // the probing variant only when a test wait limit is set
  return a.g.wait_limit ? launch_variant<F, true>(a, grid, st) : launch_variant<F, false>(a, grid, st);
}

// K3 mode: the bf16 activations enter the expert GEMMs as they are (W4A16). Pair q's token row of x
// (or row `row` of h) is copied into the padded chunk-major operand layout, 16 bytes per lane step,
// with the row's divisor c_B = 1.
__global__ void __launch_bounds__(256) wide_x_raw_kernel(const uint16_t* __restrict__ x,
                                                         const int32_t* __restrict__ pair_tok,
                                                         const int32_t* __restrict__ offsets, int n_experts, int P,
                                                         int h, int64_t r_pad, uint16_t* __restrict__ xw,
                                                         float* __restrict__ cvec) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t q = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; q < P; q += nw) {
    int lo = 0, hi = n_experts;   // the expert of pair q: the last e with offsets[e] <= q
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (offsets[mid] <= q) lo = mid; else hi = mid;
    }
    const int tok = pair_tok[q];
    const int64_t row = pbase(offsets[lo], lo) + (int)(q - offsets[lo]);
    for (int v = lane; v < h / 8; v += 32)
      *reinterpret_cast<uint4*>(xw + cm_off(row, v, r_pad)) = *reinterpret_cast<const uint4*>(x + (size_t)tok * h + v * 8);
    if (lane == 0) cvec[row] = 1.f;
  }
}

__global__ void __launch_bounds__(256) wide_h_raw_kernel(const uint16_t* __restrict__ hbf, int64_t rows, int64_t r_pad,
                                                         int k, uint16_t* __restrict__ hw, float* __restrict__ cvec) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; row < rows; row += nw) {
    for (int v = lane; v < k / 8; v += 32)
      *reinterpret_cast<uint4*>(hw + cm_off(row, v, r_pad)) = *reinterpret_cast<const uint4*>(hbf + row * k + v * 8);
    if (lane == 0) cvec[row] = 1.f;
  }
}

static unsigned warp_grid(int64_t rows) {
  const int64_t b = (rows + 7) / 8;   // one warp per row, 8 warps per block
  return (unsigned)(b < 1 ? 1 : (b > 65535 ? 65535 : b));
}

}  // namespace tcw

cudaError_t launch_tc_wide(const GroupedArgs& g, const TcPlan& plan, const void* bmat, const float* cvec,
                           int64_t r_pad, int sb_row, int split, int max_items, cudaStream_t st) {
  if (g.mode == MODE_DENSE) return cudaErrorInvalidValue;
  tcw::WideArgs a;
  a.g = g;
  a.plan = plan;
  a.cvec = cvec;
  a.r_pad = r_pad;
  a.sb_row = sb_row;
  a.b_split = split ? 1 : 0;
  const uint64_t nst = (uint64_t)g.k / 128, nrb = (uint64_t)g.n_rows / 128;
  const uint64_t bank_rows = (uint64_t)g.n_experts * nrb * nst * 128;
  a.bmat = reinterpret_cast<const uint8_t*>(bmat);
  cudaError_t e = cudaSuccess;
  const bool r4 = g.routed.fmt != FMT_FP8;
  e = tcw::encode(&a.map_w4, CU_TENSOR_MAP_DATA_TYPE_UINT8, r4 ? g.routed.w : nullptr, 128, bank_rows / 2, 128, 128,
                  64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (e != cudaSuccess) return e;
  e = tcw::encode(&a.map_w8, CU_TENSOR_MAP_DATA_TYPE_UINT8, r4 ? nullptr : g.routed.w, 128, bank_rows, 128, 64, 128,
                  CU_TENSOR_MAP_SWIZZLE_64B);
  if (e != cudaSuccess) return e;
  e = tcw::encode(&a.map_w8_sh, CU_TENSOR_MAP_DATA_TYPE_UINT8, g.has_shared ? g.shared.w : nullptr, 128,
                  nrb * nst * 128, 128, 64, 128, CU_TENSOR_MAP_SWIZZLE_64B);
  if (e != cudaSuccess) return e;
  a.use_w4 = r4 ? 1 : 0;
  a.use_w8 = r4 ? 0 : 1;
  a.use_w8_sh = g.has_shared ? 1 : 0;
  int grid = num_sms();   // one CTA per SM (its shared memory), persistent over the items
  if (grid > max_items) grid = max_items;
  if (grid < 1) grid = 1;
  switch (g.routed.fmt) {
    case FMT_NVFP4: return tcw::launch_one<FMT_NVFP4>(a, grid, st);
    case FMT_MXFP4: return tcw::launch_one<FMT_MXFP4>(a, grid, st);
    default: return tcw::launch_one<FMT_FP8>(a, grid, st);
  }
}

cudaError_t launch_wide_x(const uint8_t* xq, const float* xs, const int32_t* pair_tok, const int32_t* offsets,
                          int n_experts, int m, int P, int h, int64_t r_pad, int sb_row, int split, int routed_bf16,
                          int hot_min, void* xw, float* cvec, cudaStream_t st) {
  return launch_pdl(tcw::wide_x_kernel, dim3(tcw::warp_grid((int64_t)P + m)), dim3(256), 0, st, xq, xs, pair_tok,
                    offsets, n_experts, m, P, h, r_pad, sb_row, split, routed_bf16, hot_min,
                    reinterpret_cast<uint16_t*>(xw), cvec);
}

cudaError_t launch_wide_x_raw(const void* x, const int32_t* pair_tok, const int32_t* offsets, int n_experts, int P,
                              int h, int64_t r_pad, void* xw, float* cvec, cudaStream_t st) {
  return launch_pdl(tcw::wide_x_raw_kernel, dim3(tcw::warp_grid(P)), dim3(256), 0, st, (const uint16_t*)x, pair_tok,
                    offsets, n_experts, P, h, r_pad, (uint16_t*)xw, cvec);
}

cudaError_t launch_wide_h_raw(const __nv_bfloat16* hbf, int64_t rows, int64_t r_pad, int k, void* hw, float* cvec,
                              cudaStream_t st) {
  return launch_pdl(tcw::wide_h_raw_kernel, dim3(tcw::warp_grid(rows)), dim3(256), 0, st, (const uint16_t*)hbf, rows,
                    r_pad, k, (uint16_t*)hw, cvec);
}

cudaError_t launch_wide_h(const __nv_bfloat16* hbf, int64_t rows, int64_t r_pad, int sb_row, int k, int pow2,
                          int routed_bf16, const int32_t* offsets, int n_experts, int hot_min, int sh_rows, void* hw,
                          float* cvec, cudaStream_t st) {
  return launch_pdl(tcw::wide_h_kernel, dim3(tcw::warp_grid(rows)), dim3(256), 0, st, hbf, rows, r_pad, sb_row, k,
                    pow2, routed_bf16, offsets, n_experts, hot_min, sh_rows, reinterpret_cast<uint16_t*>(hw), cvec);
}

}  // namespace sb
