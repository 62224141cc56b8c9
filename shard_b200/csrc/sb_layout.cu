// Load-time weight layout: canonical [N, K] matrices -> the tiled fragment layout the grouped
// GEMV kernels stream.
//
// Tiled layout (per matrix), g = lane/4, t = lane%4, rg/rg8 = canonical rows of tile rows g / g+8:
//   FP4 values   [N/16 tiles][K/64 chunk pairs][32 lanes][16 B]; each 8-byte half is one 32-wide K
//                chunk: bytes W[rg][c+2t], W[rg8][c+2t], W[rg][c+2t+1], W[rg8][c+2t+1], then the same
//                at c+8 (c = 16 * chunk, byte columns of the packed row). Byte i is the e2m1 pair of
//                A-fragment register i of an m16n8k16 step, with the step's 16 K positions taken as
//                {4t..4t+3} of each 16-wide half of the chunk; the activation is read in the same
//                order, so the dot product is unchanged.
//   NVFP4 scales [N/16][K/64][8 g][8 B]: per chunk S[rg][2ch], S[rg8][2ch], S[rg][2ch+1], S[rg8][2ch+1]
//   MXFP4 scales [N/16][K/64][8 g][4 B]: per chunk S[rg][ch], S[rg8][ch]
//   FP8 values   [N/16][K/32][32 lanes][16 B]: W[rg][c+4t..+3], W[rg8][..], W[rg][c+16+4t..], W[rg8][..]
//                (the m16n8k32 e4m3 A fragment, c = 32 * chunk)
//   FP8 scales   [N/16][K/128][2] fp32: the 128x128 block scale of tile rows 0-7 and of rows 8-15
// W13 row map: tile rows 0-7 are w1 rows 8*tile.., rows 8-15 the w3 rows with the same index.
#include "sb_device.cuh"
#include "sb_launch.h"

namespace sb {

__device__ __forceinline__ int64_t row_of(int kind, int64_t n, int64_t tile, int r) {
  if (kind == 1) {  // W13
    const int64_t half = n / 2;
    return r < 8 ? 8 * tile + r : half + 8 * tile + (r - 8);
  }
  return 16 * tile + r;
}

__global__ void tile_fp4_values_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                       int kind, int64_t n_mat, int64_t n, int64_t k) {
  const int64_t ncp = k / 64, tiles = n / 16;
  const int64_t units = n_mat * tiles * ncp * 32;
  const int64_t rowb = k / 2;
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < units;
       u += (int64_t)gridDim.x * blockDim.x) {
    const int lane = (int)(u & 31);
    const int64_t cp = (u >> 5) % ncp;
    const int64_t tile = ((u >> 5) / ncp) % tiles;
    const int64_t mat = ((u >> 5) / ncp) / tiles;
    const int g = lane >> 2, t = lane & 3;
    const uint8_t* m = src + mat * n * rowb;
    const uint8_t* r0 = m + row_of(kind, n, tile, g) * rowb;
    const uint8_t* r8 = m + row_of(kind, n, tile, g + 8) * rowb;
    uint8_t out[16];
#pragma unroll
    for (int sub = 0; sub < 2; ++sub) {
      const int64_t c = (cp * 2 + sub) * 16;
      uint8_t* o = out + sub * 8;
      o[0] = r0[c + 2 * t];
      o[1] = r8[c + 2 * t];
      o[2] = r0[c + 2 * t + 1];
      o[3] = r8[c + 2 * t + 1];
      o[4] = r0[c + 8 + 2 * t];
      o[5] = r8[c + 8 + 2 * t];
      o[6] = r0[c + 8 + 2 * t + 1];
      o[7] = r8[c + 8 + 2 * t + 1];
    }
    uint4 v;
    memcpy(&v, out, 16);
    reinterpret_cast<uint4*>(dst)[u] = v;
  }
}

__global__ void tile_fp8_values_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                       int kind, int64_t n_mat, int64_t n, int64_t k) {
  const int64_t nch = k / 32, tiles = n / 16;
  const int64_t units = n_mat * tiles * nch * 32;
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < units;
       u += (int64_t)gridDim.x * blockDim.x) {
    const int lane = (int)(u & 31);
    const int64_t ch = (u >> 5) % nch;
    const int64_t tile = ((u >> 5) / nch) % tiles;
    const int64_t mat = ((u >> 5) / nch) / tiles;
    const int g = lane >> 2, t = lane & 3;
    const uint8_t* m = src + mat * n * k;
    const uint8_t* r0 = m + row_of(kind, n, tile, g) * k + ch * 32;
    const uint8_t* r8 = m + row_of(kind, n, tile, g + 8) * k + ch * 32;
    uint8_t out[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      out[j] = r0[4 * t + j];
      out[4 + j] = r8[4 * t + j];
      out[8 + j] = r0[16 + 4 * t + j];
      out[12 + j] = r8[16 + 4 * t + j];
    }
    uint4 v;
    memcpy(&v, out, 16);
    reinterpret_cast<uint4*>(dst)[u] = v;
  }
}

// NVFP4 (per16 = 1) / MXFP4 (per16 = 0) scale bytes
__global__ void tile_fp4_scales_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                       int kind, int per16, int64_t n_mat, int64_t n, int64_t k) {
  const int64_t ncp = k / 64, tiles = n / 16;
  const int64_t units = n_mat * tiles * ncp * 8;
  const int64_t rowb = per16 ? k / 16 : k / 32;
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < units;
       u += (int64_t)gridDim.x * blockDim.x) {
    const int g = (int)(u & 7);
    const int64_t cp = (u >> 3) % ncp;
    const int64_t tile = ((u >> 3) / ncp) % tiles;
    const int64_t mat = ((u >> 3) / ncp) / tiles;
    const uint8_t* m = src + mat * n * rowb;
    const uint8_t* r0 = m + row_of(kind, n, tile, g) * rowb;
    const uint8_t* r8 = m + row_of(kind, n, tile, g + 8) * rowb;
    if (per16) {
      uint8_t out[8];
#pragma unroll
      for (int sub = 0; sub < 2; ++sub) {
        const int64_t ch = cp * 2 + sub;
        out[sub * 4 + 0] = r0[2 * ch];
        out[sub * 4 + 1] = r8[2 * ch];
        out[sub * 4 + 2] = r0[2 * ch + 1];
        out[sub * 4 + 3] = r8[2 * ch + 1];
      }
      uint2 v;
      memcpy(&v, out, 8);
      reinterpret_cast<uint2*>(dst)[u] = v;
    } else {
      uint8_t out[4];
      out[0] = r0[2 * cp];
      out[1] = r8[2 * cp];
      out[2] = r0[2 * cp + 1];
      out[3] = r8[2 * cp + 1];
      uint32_t v;
      memcpy(&v, out, 4);
      reinterpret_cast<uint32_t*>(dst)[u] = v;
    }
  }
}

__global__ void tile_fp8_scales_kernel(const float* __restrict__ src, float* __restrict__ dst, int kind,
                                       int64_t n_mat, int64_t n, int64_t k) {
  const int64_t nkb = k / 128, tiles = n / 16, nrb = (n + 127) / 128;
  const int64_t units = n_mat * tiles * nkb;
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < units;
       u += (int64_t)gridDim.x * blockDim.x) {
    const int64_t kb = u % nkb;
    const int64_t tile = (u / nkb) % tiles;
    const int64_t mat = (u / nkb) / tiles;
    const float* m = src + mat * nrb * nkb;
    dst[2 * u] = m[(row_of(kind, n, tile, 0) / 128) * nkb + kb];
    dst[2 * u + 1] = m[(row_of(kind, n, tile, 8) / 128) * nkb + kb];
  }
}

static int grid_for(int64_t units) {
  int64_t b = (units + 255) / 256;
  return (int)(b < 1 ? 1 : (b > 65535 * 4 ? 65535 * 4 : b));
}

cudaError_t launch_tile_weights(int fmt, int kind, const void* src, void* dst, int64_t n_mat, int64_t n,
                                int64_t k, cudaStream_t st) {
  if (fmt == FMT_FP8) {
    const int64_t units = n_mat * (n / 16) * (k / 32) * 32;
    tile_fp8_values_kernel<<<grid_for(units), 256, 0, st>>>((const uint8_t*)src, (uint8_t*)dst, kind, n_mat,
                                                            n, k);
  } else {
    const int64_t units = n_mat * (n / 16) * (k / 64) * 32;
    tile_fp4_values_kernel<<<grid_for(units), 256, 0, st>>>((const uint8_t*)src, (uint8_t*)dst, kind, n_mat,
                                                            n, k);
  }
  return cudaGetLastError();
}

cudaError_t launch_tile_scales(int fmt, int kind, const void* src, void* dst, int64_t n_mat, int64_t n,
                               int64_t k, cudaStream_t st) {
  if (fmt == FMT_FP8) {
    const int64_t units = n_mat * (n / 16) * (k / 128);
    tile_fp8_scales_kernel<<<grid_for(units), 256, 0, st>>>((const float*)src, (float*)dst, kind, n_mat, n, k);
  } else {
    const int64_t units = n_mat * (n / 16) * (k / 64) * 8;
    tile_fp4_scales_kernel<<<grid_for(units), 256, 0, st>>>((const uint8_t*)src, (uint8_t*)dst, kind,
                                                            fmt == FMT_NVFP4 ? 1 : 0, n_mat, n, k);
  }
  return cudaGetLastError();
}

}  // namespace sb
