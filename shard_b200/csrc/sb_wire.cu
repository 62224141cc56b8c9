// The FP8 activation wire of a pipeline stage boundary (engines/deepseek_v4/v4_pipe.py:335-384):
// e4m3 with ONE bf16 scale per row of the last dim, so a position's wire bytes depend on that
// position's values alone.
//   pack    scale = bf16(clamp(amax / 448, 1e-8, bf16 max)) with amax over the row in fp32;
//           q = e4m3(clamp(x / scale, +-448)), dividing by that same rounded scale
//   unpack  y = bf16(e4m3(q) * scale)   (the fp32 product is exact; one rounding)
// An inf in a row saturates to 448 there and leaves the other values of the row finite (the scale's
// upper clamp). NaN inputs are not part of the contract: the row's scale becomes NaN.
//
// combine_pack_kernel is the MoE combine (sb_grouped.cu's combine_kernel) with the pack fused in:
// one CTA per token owns the whole row, so the stage's last layer emits the wire format directly.
#include "sb_device.cuh"
#include "sb_launch.h"

namespace sb {

constexpr float WIRE_BF16_MAX = 3.3895313892515355e38f;
constexpr int WIRE_THREADS = 256;
constexpr int WIRE_VPT = 4;   // 8-element vectors per thread kept in registers: rows of up to 8192

__device__ __forceinline__ float wire_scale(float amax) {
  float s = __fdiv_rn(amax, 448.0f);
  s = fminf(fmaxf(s, 1e-8f), WIRE_BF16_MAX);
  return bf16_round(s);
}

__device__ __forceinline__ uint2 wire_q8(const uint4& v, float s) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&v);
  uint32_t w[2] = {0u, 0u};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = __bfloat1622float2(p[e]);
    const uint32_t q0 = f32_to_e4m3(fminf(fmaxf(__fdiv_rn(f.x, s), -448.0f), 448.0f));
    const uint32_t q1 = f32_to_e4m3(fminf(fmaxf(__fdiv_rn(f.y, s), -448.0f), 448.0f));
    w[e >> 1] |= (q0 | (q1 << 8)) << (16 * (e & 1));
  }
  return make_uint2(w[0], w[1]);
}

__device__ __forceinline__ float amax8(const uint4& v, float m) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = __bfloat1622float2(p[e]);
    // NaN-propagating max: the row's scale becomes NaN like torch's amax
    m = (f.x != f.x) ? f.x : fmaxf(m, fabsf(f.x));
    m = (f.y != f.y) ? f.y : fmaxf(m, fabsf(f.y));
  }
  return m;
}

// block-wide NaN-propagating max of non-negative values
__device__ __forceinline__ float block_amax(float m, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float x = __shfl_xor_sync(0xffffffffu, m, o);
    m = (x != x) ? x : fmaxf(m, x);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (warp == 0) {
    m = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float x = __shfl_xor_sync(0xffffffffu, m, o);
      m = (x != x) ? x : fmaxf(m, x);
    }
    if (lane == 0) red[0] = m;
  }
  __syncthreads();
  return red[0];
}

// one CTA per row; rows longer than WIRE_THREADS * WIRE_VPT vectors are read twice
__global__ void __launch_bounds__(WIRE_THREADS) wire_pack_kernel(const __nv_bfloat16* __restrict__ x, int64_t dim,
                                                                 uint8_t* __restrict__ q, __nv_bfloat16* __restrict__ s) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int64_t nv = dim / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * dim);
  pdl_wait();
  pdl_trigger();
  uint4 v[WIRE_VPT];
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < WIRE_VPT; ++i) {
    const int64_t k = threadIdx.x + (int64_t)i * WIRE_THREADS;
    v[i] = k < nv ? xr[k] : make_uint4(0u, 0u, 0u, 0u);
    m = amax8(v[i], m);
  }
  for (int64_t k = threadIdx.x + (int64_t)WIRE_VPT * WIRE_THREADS; k < nv; k += WIRE_THREADS) m = amax8(xr[k], m);
  const float sc = wire_scale(block_amax(m, red));
  uint2* qr = reinterpret_cast<uint2*>(q + row * dim);
#pragma unroll
  for (int i = 0; i < WIRE_VPT; ++i) {
    const int64_t k = threadIdx.x + (int64_t)i * WIRE_THREADS;
    if (k < nv) qr[k] = wire_q8(v[i], sc);
  }
  for (int64_t k = threadIdx.x + (int64_t)WIRE_VPT * WIRE_THREADS; k < nv; k += WIRE_THREADS) qr[k] = wire_q8(xr[k], sc);
  if (threadIdx.x == 0) s[row] = __float2bfloat16_rn(sc);
}

__global__ void __launch_bounds__(256) wire_unpack_kernel(const uint8_t* __restrict__ q, const __nv_bfloat16* __restrict__ s,
                                                          int64_t rows, int64_t dim, __nv_bfloat16* __restrict__ y) {
  pdl_wait();
  pdl_trigger();
  const int64_t nv = rows * (dim / 8);
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < nv; k += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = k / (dim / 8);
    const float sc = __bfloat162float(s[row]);
    const uint2 w = reinterpret_cast<const uint2*>(q)[k];
    uint4 out;
    uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t pair = ((e < 2 ? w.x : w.y) >> (16 * (e & 1))) & 0xFFFFu;
      const float a = e4m3_to_f32(pair & 0xFFu) * sc, b = e4m3_to_f32(pair >> 8) * sc;
      const __nv_bfloat162 r = __floats2bfloat162_rn(a, b);
      o[e] = *reinterpret_cast<const uint32_t*>(&r);
    }
    reinterpret_cast<uint4*>(y)[k] = out;
  }
}

// The MoE combine with the wire pack fused in. One CTA per token, each thread up to WIRE_VPT 8-column
// vectors. The token's slot order (ascending expert id, a slot dropped when a later slot names the
// same expert: v4_moe_grouped.py:98-118) is sorted once per thread; each vector is then the fp32 sum
// of its slot rows in that order plus the shared expert, rounded to bf16 (the layer's y), and the
// row's bf16 values are packed as pack() would pack y.
template <int KP>
__global__ void __launch_bounds__(WIRE_THREADS) combine_pack_kernel(const __nv_bfloat16* __restrict__ o,
                                                                    const int32_t* __restrict__ topk_idx, int m, int K,
                                                                    int h, int has_shared, __nv_bfloat16* __restrict__ y,
                                                                    uint8_t* __restrict__ q, __nv_bfloat16* __restrict__ s) {
  __shared__ float red[32];
  const int t = blockIdx.x;
  const int P = m * K;
  const int nv = h / 8;
  pdl_wait();
  pdl_trigger();
  int key[KP], slot[KP];
#pragma unroll
  for (int j = 0; j < KP; ++j) {
    key[j] = j < K ? topk_idx[(size_t)t * K + j] : 0x7fffffff;
    slot[j] = j;
  }
#pragma unroll
  for (int j = 0; j < KP; ++j) {
    bool later = false;
#pragma unroll
    for (int j2 = j + 1; j2 < KP; ++j2) later |= (j < K && j2 < K && key[j2] == key[j]);
    if (later) key[j] = 0x7fffffff;
  }
#pragma unroll
  for (int k2 = 2; k2 <= KP; k2 <<= 1)
#pragma unroll
    for (int j2 = k2 >> 1; j2 > 0; j2 >>= 1)
#pragma unroll
      for (int i = 0; i < KP; ++i) {
        const int l = i ^ j2;
        if (l > i) {
          const bool up = (i & k2) == 0;
          if (up ? key[i] > key[l] : key[i] < key[l]) {
            const int tk = key[i], ts = slot[i];
            key[i] = key[l];
            slot[i] = slot[l];
            key[l] = tk;
            slot[l] = ts;
          }
        }
      }
  uint4 yv[WIRE_VPT];
  float am = 0.f;
#pragma unroll
  for (int i = 0; i < WIRE_VPT; ++i) {
    const int v = threadIdx.x + i * WIRE_THREADS;
    yv[i] = make_uint4(0u, 0u, 0u, 0u);
    if (v < nv) {
      uint4 r[KP + 1];
#pragma unroll
      for (int j = 0; j < KP; ++j)
        if (key[j] != 0x7fffffff) r[j] = *reinterpret_cast<const uint4*>(o + ((size_t)t * K + slot[j]) * h + v * 8);
      if (has_shared) r[KP] = *reinterpret_cast<const uint4*>(o + ((size_t)P + t) * h + v * 8);
      float acc[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll
      for (int j = 0; j <= KP; ++j) {
        const bool use = j < KP ? key[j] != 0x7fffffff : has_shared != 0;
        if (use) {
          const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&r[j]);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(p[e]);
            acc[2 * e] += f.x;
            acc[2 * e + 1] += f.y;
          }
        }
      }
      __nv_bfloat162* op = reinterpret_cast<__nv_bfloat162*>(&yv[i]);
#pragma unroll
      for (int e = 0; e < 4; ++e) op[e] = __floats2bfloat162_rn(acc[2 * e], acc[2 * e + 1]);
      if (y) *reinterpret_cast<uint4*>(y + (size_t)t * h + v * 8) = yv[i];
      am = amax8(yv[i], am);
    }
  }
  const float sc = wire_scale(block_amax(am, red));
#pragma unroll
  for (int i = 0; i < WIRE_VPT; ++i) {
    const int v = threadIdx.x + i * WIRE_THREADS;
    if (v < nv) reinterpret_cast<uint2*>(q + (size_t)t * h)[v] = wire_q8(yv[i], sc);
  }
  if (threadIdx.x == 0) s[t] = __float2bfloat16_rn(sc);
}

cudaError_t launch_wire_pack(const void* x, int64_t rows, int64_t dim, uint8_t* q, void* s, cudaStream_t st) {
  return launch_pdl(wire_pack_kernel, dim3((unsigned)rows), dim3(WIRE_THREADS), 0, st, (const __nv_bfloat16*)x, dim, q,
                    (__nv_bfloat16*)s);
}

cudaError_t launch_wire_unpack(const uint8_t* q, const void* s, int64_t rows, int64_t dim, void* y, cudaStream_t st) {
  const int64_t nv = rows * (dim / 8);
  int64_t b = (nv + 255) / 256;
  const unsigned grid = (unsigned)(b < 1 ? 1 : (b > 65535 ? 65535 : b));
  return launch_pdl(wire_unpack_kernel, dim3(grid), dim3(256), 0, st, q, (const __nv_bfloat16*)s, rows, dim,
                    (__nv_bfloat16*)y);
}

cudaError_t launch_combine_pack(const __nv_bfloat16* o, const int32_t* topk_idx, int m, int topk, int h,
                                int has_shared, __nv_bfloat16* y, uint8_t* q, __nv_bfloat16* s, cudaStream_t st) {
  const dim3 grid(m), block(WIRE_THREADS);
  if (topk <= 2) return launch_pdl(combine_pack_kernel<2>, grid, block, 0, st, o, topk_idx, m, topk, h, has_shared, y, q, s);
  if (topk <= 4) return launch_pdl(combine_pack_kernel<4>, grid, block, 0, st, o, topk_idx, m, topk, h, has_shared, y, q, s);
  if (topk <= 8) return launch_pdl(combine_pack_kernel<8>, grid, block, 0, st, o, topk_idx, m, topk, h, has_shared, y, q, s);
  return launch_pdl(combine_pack_kernel<16>, grid, block, 0, st, o, topk_idx, m, topk, h, has_shared, y, q, s);
}


// ── the block around the MoE operator: residual add and RMSNorm (model.py:189-202, 701-706) ──
// One CTA per row: x <- bf16(x + y) (when y is given), then out = bf16(w * (x * rsqrt(mean(x^2) +
// eps))) in fp32 (w = 1 when not given), as RMSNorm.forward computes it on the bf16 residual stream.
__global__ void __launch_bounds__(WIRE_THREADS) residual_rmsnorm_kernel(uint16_t* __restrict__ x,
                                                                        const uint16_t* __restrict__ y, int64_t dim,
                                                                        const float* __restrict__ w, float eps,
                                                                        uint16_t* __restrict__ out) {
  __shared__ float red[WIRE_THREADS / 32];
  pdl_wait();
  pdl_trigger();
  const int64_t row = blockIdx.x;
  uint16_t* xr = x + row * dim;
  float ss = 0.f;
  for (int64_t v = threadIdx.x; v < dim / 8; v += blockDim.x) {
    uint4 a = reinterpret_cast<const uint4*>(xr)[v];
    if (y != nullptr) {
      const uint4 b = reinterpret_cast<const uint4*>(y + row * dim)[v];
      __nv_bfloat162* pa = reinterpret_cast<__nv_bfloat162*>(&a);
      const __nv_bfloat162* pb = reinterpret_cast<const __nv_bfloat162*>(&b);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 fa = __bfloat1622float2(pa[e]), fb = __bfloat1622float2(pb[e]);
        pa[e] = __floats2bfloat162_rn(fa.x + fb.x, fa.y + fb.y);
      }
      reinterpret_cast<uint4*>(xr)[v] = a;
    }
    const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&a);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(pa[e]);
      ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
    }
  }
  if (out == nullptr) return;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < WIRE_THREADS / 32; ++i) tot += red[i];
  const float r = rsqrtf(tot / (float)dim + eps);
  for (int64_t v = threadIdx.x; v < dim / 8; v += blockDim.x) {
    // this thread's own writes of x above: re-read them
    const uint4 a = reinterpret_cast<const uint4*>(xr)[v];
    const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&a);
    uint4 o4;
    __nv_bfloat162* po = reinterpret_cast<__nv_bfloat162*>(&o4);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(pa[e]);
      const float w0 = w != nullptr ? w[v * 8 + 2 * e] : 1.f, w1 = w != nullptr ? w[v * 8 + 2 * e + 1] : 1.f;
      po[e] = __floats2bfloat162_rn(w0 * (f.x * r), w1 * (f.y * r));
    }
    reinterpret_cast<uint4*>(out + row * dim)[v] = o4;
  }
}

cudaError_t launch_residual_rmsnorm(void* x, const void* y, int64_t rows, int64_t dim, const float* w, float eps,
                                    void* out, cudaStream_t st) {
  return launch_pdl(residual_rmsnorm_kernel, dim3((unsigned)rows), dim3(WIRE_THREADS), 0, st, (uint16_t*)x,
                    (const uint16_t*)y, dim, w, eps, (uint16_t*)out);
}

}  // namespace sb
