// Routing and token permutation of the MoE stage forward.
//
//   gate_logits_kernel   logits[M, E] = fp32(x) . fp32(W_gate)^T            (Gate.forward, model.py:570)
//   route_kernel         score, selection bias, sorted top-k, weights renormalised and scaled
//                        (model.py:571-589), hash routing through tid2eid (model.py:581-582), and
//                        the per-128 e4m3 quantisation of x for the expert GEMVs (act_quant,
//                        kernel.py:40-125)
//   permute_kernel       per-expert (token, slot) lists in ascending expert id (tokens ascending
//                        within an expert up to 2048 pairs; any order above, which no output sees);
//                        the list of active experts; all on the device, so the
//                        forward never drains to the host (the reference's bincount().tolist(),
//                        model.py:639, is the sync this replaces)
#include "sb_device.cuh"
#include "sb_launch.h"

namespace sb {

// Split-K gate GEMV. CTA (e-group of 8 experts, K-split s of 512, token group of 32): each warp takes
// one expert row's 512-wide K slice (1 KB, two 16-byte loads per lane, issued before any math) and
// dots it with the slice of every token of the group (L1/L2 resident). Partial logits go to
// part[s][t][e]; route_kernel adds the splits in ascending s, so the sum order is fixed. bf16 x bf16
// products are exact in fp32; only the summation order differs from the reference's fp32 F.linear.
constexpr int GATE_TOKENS = 32;


__global__ void __launch_bounds__(256) gate_logits_kernel(const __nv_bfloat16* __restrict__ x,
                                                          const __nv_bfloat16* __restrict__ w,
                                                          float* __restrict__ part, int m, int e_total,
                                                          int h) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * 8 + warp;
  const int ks = blockIdx.y;
  const int t0 = blockIdx.z * GATE_TOKENS;
  pdl_wait();
  pdl_trigger();
  if (e >= e_total) return;
  const int nt = min(GATE_TOKENS, m - t0);
  const int kspl = gate_ksplit(h);
  const bool two = kspl == 512;
  const int k0 = ks * kspl;
  const uint4* wr = reinterpret_cast<const uint4*>(w + (size_t)e * h + k0);
  const uint4 wv0 = __ldg(wr + lane);
  const uint4 wv1 = two ? __ldg(wr + 32 + lane) : make_uint4(0u, 0u, 0u, 0u);
  float wf[16];
  {
    const __nv_bfloat162* p0 = reinterpret_cast<const __nv_bfloat162*>(&wv0);
    const __nv_bfloat162* p1 = reinterpret_cast<const __nv_bfloat162*>(&wv1);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 a = __bfloat1622float2(p0[q]), b = __bfloat1622float2(p1[q]);
      wf[2 * q] = a.x;
      wf[2 * q + 1] = a.y;
      wf[8 + 2 * q] = b.x;
      wf[8 + 2 * q + 1] = b.y;
    }
  }
  float* out = part + ((size_t)ks * m + t0) * e_total + e;
  for (int j0 = 0; j0 < nt; j0 += 8) {
    uint4 xv0[8], xv1[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j0 + j < nt) {
        const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)(t0 + j0 + j) * h + k0);
        xv0[j] = __ldg(xr + lane);
        xv1[j] = two ? __ldg(xr + 32 + lane) : make_uint4(0u, 0u, 0u, 0u);
      }
    }
    float p[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float acc = 0.f;
      if (j0 + j < nt) {
        const __nv_bfloat162* p0 = reinterpret_cast<const __nv_bfloat162*>(&xv0[j]);
        const __nv_bfloat162* p1 = reinterpret_cast<const __nv_bfloat162*>(&xv1[j]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 a = __bfloat1622float2(p0[q]), b = __bfloat1622float2(p1[q]);
          acc = fmaf(a.x, wf[2 * q], acc);
          acc = fmaf(a.y, wf[2 * q + 1], acc);
          acc = fmaf(b.x, wf[8 + 2 * q], acc);
          acc = fmaf(b.y, wf[8 + 2 * q + 1], acc);
        }
      }
      p[j] = acc;
    }
    // reduce-scatter over the xor tree 16, 8, 4, 2, 1 (the pairings of a warp_sum, so every
    // token's sum is bitwise the one warp_sum gives): after it, lane l holds the sum of token
    // 4*b4(l) + 2*b3(l) + b2(l), where bk(l) is bit k of l
    {
      const int h = (lane >> 4) & 1;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float send = h ? p[i] : p[i + 4], keep = h ? p[i + 4] : p[i];
        p[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
      }
    }
    {
      const int h = (lane >> 3) & 1;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const float send = h ? p[i] : p[i + 2], keep = h ? p[i + 2] : p[i];
        p[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
      }
    }
    {
      const int h = (lane >> 2) & 1;
      const float send = h ? p[0] : p[1], keep = h ? p[1] : p[0];
      p[0] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    p[0] += __shfl_xor_sync(0xffffffffu, p[0], 2);
    p[0] += __shfl_xor_sync(0xffffffffu, p[0], 1);
    {
      const int j = 4 * ((lane >> 4) & 1) + 2 * ((lane >> 3) & 1) + ((lane >> 2) & 1);
      if ((lane & 3) == 0 && j0 + j < nt) out[(size_t)(j0 + j) * e_total] = p[0];
    }
  }
}

// (value, expert) ordering of the top-k: larger value first, lower expert id on ties
__device__ __forceinline__ bool before(float va, int ea, float vb, int eb) {
  return va > vb || (va == vb && ea < eb);
}

// One CTA per token: warp 0 routes while warps 1-3 quantise x[t] (act_quant, one 128-block per
// warp-iteration, loads issued up front). SPL = expert slots per lane (E <= 32 * SPL): every lane
// sorts its slots once (bitonic network, biased score descending, ties to the lower id), then k
// rounds of a warp-wide argmax over the lanes' current heads (redux.sync max of the value, then min
// of the expert id among the lanes holding it) pick the top-k in order.
__device__ __forceinline__ void quant_row(const RouteArgs& a, int t, int w, int nw, int lane) {
  const __nv_bfloat16* xr = a.x + (size_t)t * a.hidden;
  const int nb = a.hidden / 128;
  for (int b0 = w; b0 < nb; b0 += 4 * nw) {
    uint2 raw[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int b = b0 + nw * u;
      if (b < nb) raw[u] = *reinterpret_cast<const uint2*>(xr + b * 128 + lane * 4);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int b = b0 + nw * u;
      if (b < nb) {
        const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&raw[u]);
        const float2 f0 = __bfloat1622float2(p[0]), f1 = __bfloat1622float2(p[1]);
        float am = fmaxf(fmaxf(fabsf(f0.x), fabsf(f0.y)), fmaxf(fabsf(f1.x), fabsf(f1.y)));
        am = warp_max(am);
        const float s = act_scale(am, a.act_pow2);
        const uint32_t q = (uint32_t)act_q(f0.x, s) | ((uint32_t)act_q(f0.y, s) << 8) |
                           ((uint32_t)act_q(f1.x, s) << 16) | ((uint32_t)act_q(f1.y, s) << 24);
        *reinterpret_cast<uint32_t*>(a.xq + (size_t)t * a.hidden + b * 128 + lane * 4) = q;
        if (lane == 0) a.xs[(size_t)t * nb + b] = s;
      }
    }
  }
}

template <int SPL>
__global__ void __launch_bounds__(128) route_kernel(RouteArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x;
  pdl_wait();
  pdl_trigger();
  if (t >= a.m) return;
  if (warp != 0) {
    if (a.xq != nullptr) quant_row(a, t, warp - 1, 3, lane);
    return;
  }
  const int E = a.n_experts;
  const int nsplit = a.hidden / gate_ksplit(a.hidden);
  // logits: split 0 + split 1 + ... in ascending split order; the loads of 4 splits are issued
  // before their adds (one memory latency per 4 splits)
  float sc[SPL];
#pragma unroll
  for (int i = 0; i < SPL; ++i) sc[i] = 0.f;
  for (int ks0 = 0; ks0 < nsplit; ks0 += 4) {
    float pv[4][SPL];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float* pk = a.logits + ((size_t)(ks0 + u) * a.m + t) * E;
#pragma unroll
      for (int i = 0; i < SPL; ++i) {
        const int e = lane + 32 * i;
        pv[u][i] = (ks0 + u < nsplit && e < E) ? pk[e] : 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int i = 0; i < SPL; ++i)
        if (ks0 + u < nsplit) sc[i] = (ks0 + u == 0) ? pv[u][i] : sc[i] + pv[u][i];
  }
#pragma unroll
  for (int i = 0; i < SPL; ++i) {
    if (a.logits_bf16) sc[i] = bf16_round(sc[i]);   // a bf16 router GEMM's output
    if (lane + 32 * i >= E) sc[i] = -INFINITY;
  }
  if (a.score_func == SCORE_SOFTMAX) {
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < SPL; ++i) mx = fmaxf(mx, sc[i]);
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < SPL; ++i) {
      const int e = lane + 32 * i;
      sc[i] = e < E ? expf(sc[i] - mx) : 0.f;
      sum += sc[i];
    }
    sum = warp_sum(sum);
#pragma unroll
    for (int i = 0; i < SPL; ++i) sc[i] = __fdiv_rn(sc[i], sum);
  } else if (a.score_func == SCORE_SIGMOID) {
#pragma unroll
    for (int i = 0; i < SPL; ++i) sc[i] = __fdiv_rn(1.0f, 1.0f + expf(-sc[i]));
  } else {
#pragma unroll
    for (int i = 0; i < SPL; ++i) {
      const float l = sc[i];
      sc[i] = sqrtf(l > 20.f ? l : log1pf(expf(l)));
    }
  }
  const int K = a.topk;
  int sel[16];
  float wsel[16];
  if (a.tid2eid != nullptr) {
    // hash routing: the ids come from the table, weights still from the unbiased scores
    const int64_t id = a.input_ids[t];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (j < K) {
        int e = a.tid2eid[id * K + j];
        e = e < 0 ? 0 : (e >= E ? E - 1 : e);  // the host validates the table; this only keeps
        sel[j] = e;                             // a corrupt one from indexing out of bounds
        float mine = 0.f;
#pragma unroll
        for (int i = 0; i < SPL; ++i)
          if (lane + 32 * i == e) mine = sc[i];
        wsel[j] = __shfl_sync(0xffffffffu, mine, e & 31);
      }
    }
  } else {
    // lane-local (biased value, expert, unbiased score), sorted once
    float bv[SPL], uv[SPL];
    int be[SPL];
#pragma unroll
    for (int i = 0; i < SPL; ++i) {
      const int e = lane + 32 * i;
      bv[i] = e < E ? sc[i] + (a.bias ? a.bias[e] : 0.f) : -INFINITY;
      be[i] = e < E ? e : 0x7fffffff;
      uv[i] = sc[i];
    }
#pragma unroll
    for (int k2 = 2; k2 <= SPL; k2 <<= 1)
#pragma unroll
      for (int j2 = k2 >> 1; j2 > 0; j2 >>= 1)
#pragma unroll
        for (int i = 0; i < SPL; ++i) {
          const int l = i ^ j2;
          if (l > i) {
            const bool desc = (i & k2) == 0;
            const bool swap = desc ? before(bv[l], be[l], bv[i], be[i]) : before(bv[i], be[i], bv[l], be[l]);
            if (swap) {
              const float tv = bv[i], tu = uv[i];
              const int te = be[i];
              bv[i] = bv[l];
              uv[i] = uv[l];
              be[i] = be[l];
              bv[l] = tv;
              uv[l] = tu;
              be[l] = te;
            }
          }
        }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (j < K) {
        // float -> order-preserving unsigned key; the largest head value, then its lowest id
        const uint32_t b = __float_as_uint(bv[0] + 0.0f);   // -0 -> +0: equal values tie on the id
        const uint32_t key = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
        const uint32_t kmax = __reduce_max_sync(0xffffffffu, key);
        int e = (int)__reduce_min_sync(0xffffffffu, key == kmax ? (uint32_t)be[0] : 0x7fffffffu);
        if (e >= E) e = j;  // only reachable with NaN scores; keeps every id in range
        sel[j] = e;
        const float mine = be[0] == e ? uv[0] : 0.f;
        wsel[j] = __shfl_sync(0xffffffffu, mine, e & 31);
        if (be[0] == e) {  // the owner pops its head
#pragma unroll
          for (int i = 0; i + 1 < SPL; ++i) {
            bv[i] = bv[i + 1];
            be[i] = be[i + 1];
            uv[i] = uv[i + 1];
          }
          bv[SPL - 1] = -INFINITY;
          be[SPL - 1] = 0x7fffffff;
        }
      }
    }
  }
  if (a.score_func != SCORE_SOFTMAX && !a.no_renorm) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j < K) s += wsel[j];
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j < K) wsel[j] = __fdiv_rn(wsel[j], s);
  }
  if (lane < K) {
    float w = 0.f;
    int e = 0;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j == lane) {
        w = wsel[j];
        e = sel[j];
      }
    w *= a.route_scale;
    a.topk_idx[(size_t)t * K + lane] = e;
    a.topk_w[(size_t)t * K + lane] = w;
    if (a.out_idx) a.out_idx[(size_t)t * K + lane] = e;
    if (a.out_w) a.out_w[(size_t)t * K + lane] = w;
  }
}

// Single CTA. counts -> exclusive offsets -> stable placement (pair p = t*K + j, ascending p
// within each expert, i.e. ascending token) -> active expert list. Deterministic.
// pairs whose expert ids are staged in shared memory (with 2 * 1024 ints of counters: < 48 KB)
constexpr int PERMUTE_SMEM_PAIRS = 8192;

// pairs up to which the placement is stable (tokens ascending within an expert, by one warp)
constexpr int PERMUTE_STABLE_PAIRS = 2048;

__global__ void __launch_bounds__(1024) permute_kernel(PermuteArgs a) {
  extern __shared__ int smem[];
  int* cnt = smem;                       // [E]
  int* cursor = smem + a.n_experts;      // [E]
  int* tk = smem + 2 * a.n_experts;      // [P] copy of topk_idx when it fits (PERMUTE_SMEM_PAIRS)
  __shared__ int warp_tot[32];
  const int E = a.n_experts, P = a.m * a.topk;
  const bool staged = P <= PERMUTE_SMEM_PAIRS;
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == 0 && a.err) *a.err = (a.gate_err != nullptr && *a.gate_err != 0) ? 1 : 0;
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    const int e = a.topk_idx[p];
    if (staged) tk[p] = e;
    atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  // exclusive scan of cnt over E (E <= 1024 = blockDim), and of the active flags
  const int e = threadIdx.x;
  const int c = e < E ? cnt[e] : 0;
  const int flag = c > 0 ? 1 : 0;
  // passes of expert e: in the first table, or (a hot expert of the hybrid dispatch) the second
  const bool hot = a.hot_min > 0 && c >= a.hot_min;
  const int np = (a.pass_max > 0 && !hot) ? (c + a.pass_max - 1) / a.pass_max : 0;
  const int np2 = hot ? (c + a.pass_max2 - 1) / a.pass_max2 : 0;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = c, fincl = flag, pincl = np, qincl = np2;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    const int fv = __shfl_up_sync(0xffffffffu, fincl, o);
    const int pv = __shfl_up_sync(0xffffffffu, pincl, o);
    const int qv = __shfl_up_sync(0xffffffffu, qincl, o);
    if (lane >= o) {
      incl += v;
      fincl += fv;
      pincl += pv;
      qincl += qv;
    }
  }
  __shared__ int warp_ftot[32], warp_ptot[32], warp_qtot[32];
  if (lane == 31) {
    warp_tot[warp] = incl;
    warp_ftot[warp] = fincl;
    warp_ptot[warp] = pincl;
    warp_qtot[warp] = qincl;
  }
  __syncthreads();
  if (warp == 0) {
    int v = warp_tot[lane], fv = warp_ftot[lane], pv = warp_ptot[lane], qv = warp_qtot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, v, o);
      const int fu = __shfl_up_sync(0xffffffffu, fv, o);
      const int pu = __shfl_up_sync(0xffffffffu, pv, o);
      const int qu = __shfl_up_sync(0xffffffffu, qv, o);
      if (lane >= o) {
        v += u;
        fv += fu;
        pv += pu;
        qv += qu;
      }
    }
    warp_tot[lane] = v;
    warp_ftot[lane] = fv;
    warp_ptot[lane] = pv;
    warp_qtot[lane] = qv;
  }
  __syncthreads();
  const int base = warp > 0 ? warp_tot[warp - 1] : 0;
  const int fbase = warp > 0 ? warp_ftot[warp - 1] : 0;
  const int pbase = warp > 0 ? warp_ptot[warp - 1] : 0;
  const int qbase = warp > 0 ? warp_qtot[warp - 1] : 0;
  if (e < E) {
    const int off = base + incl - c;
    a.offsets[e] = off;
    a.counts[e] = c;
    cursor[e] = off;
    if (flag) a.active[fbase + fincl - 1] = e;
    if (flag && a.pass_off) {
      const int slot = fbase + fincl - 1, p0 = pbase + pincl - np;
      a.pass_off[slot] = p0;
      for (int i = 0; i < np; ++i) {   // the pass table: every routed pass's slot and first token
        a.pass_slot[p0 + i] = slot;
        a.pass_pb[p0 + i] = i * a.pass_max;
      }
    }
    if (flag && a.pass_off2) {
      const int slot = fbase + fincl - 1, q0 = qbase + qincl - np2;
      a.pass_off2[slot] = q0;
      for (int i = 0; i < np2; ++i) {
        a.pass_slot2[q0 + i] = slot;
        a.pass_pb2[q0 + i] = i * a.pass_max2;
      }
    }
    if (e == E - 1) {
      a.offsets[E] = base + incl;
      *a.n_active = fbase + fincl;
      if (a.pass_off) a.pass_off[fbase + fincl] = pbase + pincl;
      if (a.pass_off2) a.pass_off2[fbase + fincl] = qbase + qincl;
    }
  }
  __syncthreads();
  if (P > PERMUTE_STABLE_PAIRS) {
    // Large batches: every thread places pairs through the shared cursors. The order of an expert's
    // pairs then varies between runs, but no output does: every grouped kernel computes each
    // token's rows independently of the other tokens of its pass (row invariance, asserted
    // bit-for-bit by the parity tests), and outputs are indexed by (token, slot), not by position.
    for (int p = threadIdx.x; p < P; p += blockDim.x) {
      const int ex = staged ? tk[p] : a.topk_idx[p];
      const int pos = atomicAdd(&cursor[ex], 1);
      a.pair_tok[pos] = p / a.topk;
      a.pair_slot[pos] = p % a.topk;
    }
    return;
  }
  // stable placement by one warp, 32 pairs at a time in ascending p
  if (warp == 0) {
    for (int p0 = 0; p0 < P; p0 += 32) {
      const int p = p0 + lane;
      const int ex = p < P ? (staged ? tk[p] : a.topk_idx[p]) : -1 - lane;
      const unsigned same = __match_any_sync(0xffffffffu, ex);
      const int rank = __popc(same & ((1u << lane) - 1u));
      const int leader = __ffs(same) - 1;
      int pos = 0;
      if (p < P) pos = cursor[ex] + rank;
      __syncwarp();
      if (p < P && lane == leader) cursor[ex] += __popc(same);
      __syncwarp();
      if (p < P) {
        a.pair_tok[pos] = p / a.topk;
        a.pair_slot[pos] = p % a.topk;
      }
    }
  }
}

cudaError_t launch_gate_logits(const void* x, const void* w, float* logits, int m, int e, int h,
                               cudaStream_t st) {
  dim3 grid((e + 7) / 8, h / gate_ksplit(h), (m + GATE_TOKENS - 1) / GATE_TOKENS);
  return launch_pdl(gate_logits_kernel, grid, dim3(256), 0, st, (const __nv_bfloat16*)x, (const __nv_bfloat16*)w,
                    logits, m, e, h);
}

cudaError_t launch_route(const RouteArgs& a, cudaStream_t st) {
  const int spl = (a.n_experts + 31) / 32;
  const dim3 grid(a.m), block(128);
  if (spl <= 1) return launch_pdl(route_kernel<1>, grid, block, 0, st, a);
  if (spl <= 2) return launch_pdl(route_kernel<2>, grid, block, 0, st, a);
  if (spl <= 4) return launch_pdl(route_kernel<4>, grid, block, 0, st, a);
  if (spl <= 8) return launch_pdl(route_kernel<8>, grid, block, 0, st, a);
  if (spl <= 16) return launch_pdl(route_kernel<16>, grid, block, 0, st, a);
  return launch_pdl(route_kernel<32>, grid, block, 0, st, a);
}

cudaError_t launch_permute(const PermuteArgs& a, cudaStream_t st) {
  const int P = a.m * a.topk;
  const size_t smem = (size_t)(2 * a.n_experts + (P <= PERMUTE_SMEM_PAIRS ? P : 0)) * sizeof(int);
  return launch_pdl(permute_kernel, dim3(1), dim3(1024), smem, st, a);
}

}  // namespace sb
