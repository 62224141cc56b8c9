// Host-side launch interface between the C-ABI layer (sb_abi.cu) and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stddef.h>
#include <stdint.h>

namespace sb {

struct RouteArgs {
  const float* logits;       // [M, E]
  const float* bias;         // [E] or null
  const int32_t* tid2eid;    // [vocab, K] or null
  const int64_t* input_ids;  // [M] (hash routing)
  int m, n_experts, topk, score_func, act_pow2, hidden;
  float route_scale;
  int32_t* topk_idx;         // [M, K]
  float* topk_w;             // [M, K]
  int64_t* out_idx;          // optional [M, K]
  float* out_w;              // optional [M, K]
  const __nv_bfloat16* x;    // [M, H]
  uint8_t* xq;               // [M, H] e4m3 (null: skip the quantisation)
  float* xs;                 // [M, H/128]
};

struct PermuteArgs {
  const int32_t* topk_idx;
  int m, topk, n_experts;
  int32_t* counts;   // [E]
  int32_t* offsets;  // [E+1]
  int32_t* active;   // [E]
  int32_t* n_active; // [1]
  int32_t* pair_tok; // [M*K]
  int32_t* pair_slot;// [M*K]
  int32_t* err;      // cleared here, before the grouped kernels run
};

// One family of tiled weight matrices (one per expert, or a single matrix).
struct WeightSet {
  const uint8_t* w;
  const uint8_t* s;
  const float* ts;     // NVFP4 tensor scales, ts_stride floats per expert, or null
  size_t w_stride;     // bytes per expert
  size_t s_stride;
  int ts_stride;
  int fmt;
};

enum GroupedMode { MODE_W13 = 0, MODE_W2 = 1, MODE_DENSE = 2 };

struct GroupedArgs {
  int mode;
  int m, topk;
  int n_rows;          // rows N of each weight matrix (w13: 2I, w2: H, dense: N)
  int k;               // contraction K (w13: H, w2: I)
  int has_shared;
  int act_pow2;
  float swiglu_limit;
  WeightSet routed, shared;
  const int32_t* counts;
  const int32_t* offsets;
  const int32_t* active;
  const int32_t* n_active;
  const int32_t* pair_tok;
  const int32_t* pair_slot;
  const float* topk_w;
  const uint8_t* bq;   // B operand rows (e4m3), row stride k
  const float* bs;     // B scales, row stride k/128
  uint8_t* hq;         // W13 out: e4m3 h rows (stride I)
  float* hs;           // W13 out: h scales (stride I/128)
  __nv_bfloat16* o;    // W2 / DENSE out (bf16), row stride n_rows
  int items_per_expert;
  int* err;            // device flag: set to 1 if a bounded wait gave up (must start at 0)
};

cudaError_t launch_gate_logits(const void* x, const void* w, float* logits, int m, int e, int h, cudaStream_t st);
cudaError_t launch_route(const RouteArgs& a, cudaStream_t st);
cudaError_t launch_permute(const PermuteArgs& a, cudaStream_t st);
cudaError_t launch_grouped(const GroupedArgs& a, int max_items, int grid_cap, cudaStream_t st);
cudaError_t launch_combine(const __nv_bfloat16* o, const int32_t* topk_idx, int m, int topk, int h,
                           int has_shared, __nv_bfloat16* y, cudaStream_t st);
cudaError_t launch_act_quant(const void* x, int64_t m, int64_t k, int pow2, uint8_t* q, float* s, cudaStream_t st);
cudaError_t launch_tile_weights(int fmt, int kind, const void* src, void* dst, int64_t n_mat, int64_t n,
                                int64_t k, cudaStream_t st);
cudaError_t launch_tile_scales(int fmt, int kind, const void* src, void* dst, int64_t n_mat, int64_t n,
                               int64_t k, cudaStream_t st);
cudaError_t launch_selftest(float* out, cudaStream_t st);

int num_sms();

}  // namespace sb
