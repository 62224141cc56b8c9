// Device helpers shared by the MoE-stage kernels (sm_100a).
//
// Number formats: e2m1 (fp4, two per byte, low nibble = even K), e4m3 (fp8), e8m0 (power-of-two
// scale byte), bf16 activations, fp32 accumulation. The conversions below go through the CUDA
// fp4/fp8 intrinsics (cvt.rn.f16x2.e2m1x2 / cvt.rn.f16x2.e4m3x2 on sm_100a), which are exact:
// every e2m1 and e4m3 value is representable in fp16.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_fp4.h>
#include <stdint.h>

namespace sb {

constexpr int FMT_NVFP4 = 1;
constexpr int FMT_MXFP4 = 2;
constexpr int FMT_FP8 = 3;

constexpr int SCORE_SOFTMAX = 0;
constexpr int SCORE_SIGMOID = 1;
constexpr int SCORE_SQRTSOFTPLUS = 2;

// ── conversions ────────────────────────────────────────────────────────────────────────────────

// one byte = two e2m1 codes -> f16x2 (low nibble -> low half)
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte) {
  __half2_raw r = __nv_cvt_fp4x2_to_halfraw2((__nv_fp4x2_storage_t)(byte & 0xFFu), __NV_E2M1);
  return (uint32_t)r.x | ((uint32_t)r.y << 16);
}

// two e4m3 bytes (low byte first) -> f16x2 (low byte -> low half)
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two) {
  __half2_raw r = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(two & 0xFFFFu), __NV_E4M3);
  return (uint32_t)r.x | ((uint32_t)r.y << 16);
}

// four bytes of e2m1 pairs -> four f16x2 (byte i -> r_i), one cvt per byte, no repacking
__device__ __forceinline__ void e2m1x8_to_f16x2x4(uint32_t w, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                  uint32_t& r3) {
  asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %4;\n"
      " cvt.rn.f16x2.e2m1x2 %0, b0;\n cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      " cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n}"
      : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
      : "r"(w));
}

// four e4m3 bytes -> two f16x2 (bytes 0,1 -> d0; bytes 2,3 -> d1)
__device__ __forceinline__ void e4m3x4_to_f16x2x2(uint32_t w, uint32_t& d0, uint32_t& d1) {
  asm("{\n .reg .b16 lo, hi;\n mov.b32 {lo, hi}, %2;\n cvt.rn.f16x2.e4m3x2 %0, lo;\n"
      " cvt.rn.f16x2.e4m3x2 %1, hi;\n}"
      : "=r"(d0), "=r"(d1)
      : "r"(w));
}

__device__ __forceinline__ float e4m3_to_f32(uint32_t byte) {
  __half_raw r = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)(byte & 0xFFu), __NV_E4M3);
  return __half2float(__half(r));
}

__device__ __forceinline__ uint8_t f32_to_e4m3(float v) {
  return (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
}

// e8m0 byte -> 2^(b-127) (b in [1, 254]; 0 maps to 2^-127 via the subnormal pattern)
__device__ __forceinline__ float e8m0_to_f32(uint32_t b) {
  b &= 0xFFu;
  return b ? __uint_as_float(b << 23) : __uint_as_float(0x00400000u);
}

__device__ __forceinline__ float bf16_round(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// f16x2 with both halves = the low (or high) half of s
__device__ __forceinline__ uint32_t splat_lo(uint32_t s) { return (s & 0xFFFFu) | (s << 16); }
__device__ __forceinline__ uint32_t splat_hi(uint32_t s) { return (s >> 16) | (s & 0xFFFF0000u); }

// 2^ceil(log2(x)) for a positive normal x, read off the IEEE bits: the exponent, plus one unless
// the mantissa is zero. Exact at powers of two, which is the property the activation scale rule
// (ue8m0) needs.
__device__ __forceinline__ float pow2_ceil(float x) {
  uint32_t b = __float_as_uint(x);
  int e = (int)((b >> 23) & 0xFFu) - 127 + ((b & 0x7FFFFFu) != 0u);
  e = e < -126 ? -126 : (e > 127 ? 127 : e);
  return __uint_as_float((uint32_t)(e + 127) << 23);
}

// per-block activation scale: amax floored at 1e-4, then 2^ceil(log2(amax/448)) or amax/448
__device__ __forceinline__ float act_scale(float amax, bool pow2) {
  amax = fmaxf(amax, 1e-4f);
  float x = amax * (1.0f / 448.0f);
  return pow2 ? pow2_ceil(x) : x;
}

__device__ __forceinline__ uint8_t act_q(float v, float s) {
  float q = __fdiv_rn(v, s);
  q = fminf(fmaxf(q, -448.0f), 448.0f);
  return f32_to_e4m3(q);
}

// act_q with the reciprocal of a power-of-two scale: v * (1/s) is exactly v / s for such s
__device__ __forceinline__ uint8_t act_q_pow2(float v, float inv_s) {
  float q = v * inv_s;
  q = fminf(fmaxf(q, -448.0f), 448.0f);
  return f32_to_e4m3(q);
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

// K3's SituAndMul on one (gate, up) pair in fp32 (modeling_kimi_linear.py:64-82):
// (beta * tanh(g / beta)) * sigmoid(g) * up', up' = linear_beta * tanh(up / linear_beta) when
// linear_beta is set (lbeta > 0), else up
__device__ __forceinline__ float situ(float g, float u, float beta, float lbeta) {
  const float a = beta * tanhf(g / beta) * (1.0f / (1.0f + expf(-g)));
  const float up = lbeta > 0.f ? lbeta * tanhf(u / lbeta) : u;
  return a * up;
}

// ── tensor-core fragments (mma.sync, fp32 accumulate) ───────────────────────────────────────────
// m16n8k16 f16: A rows g / g+8, k {2t,2t+1} and {2t+8,2t+9}; B (k x n) k {2t,2t+1},{2t+8,2t+9}, n = g;
// C rows g / g+8, cols {2t, 2t+1}   (g = lane/4, t = lane%4)
__device__ __forceinline__ void mma_f16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// m16n8k32 e4m3: A rows g / g+8, k 4t..4t+3 and 16+4t..; B k 4t.. / 16+4t.., n = g
__device__ __forceinline__ void mma_e4m3(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ── bulk async copies (TMA, non-tensor) and mbarriers ───────────────────────────────────────────

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}

// global -> shared bulk copy completing on an mbarrier (16-byte aligned addresses, size % 16 == 0)
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// non-blocking probe of the phase (try_wait may suspend the thread for a while before it returns)
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint (ns): the thread sleeps in hardware until the phase completes
// or the hint expires, instead of spinning on issue slots
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after `limit` polls (each poll may suspend the thread for a while in
// hardware) and returns false, so a lost completion can never hang the GPU.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint32_t limit = (1u << 24)) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// Programmatic dependent launch: a kernel launched with programmatic stream serialisation may start
// while the previous kernel of the stream is still running; pdl_wait() returns once that kernel has
// completed and its memory is visible, so everything a kernel reads or writes comes after it.
// pdl_trigger() lets the next kernel of the stream start launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace sb
