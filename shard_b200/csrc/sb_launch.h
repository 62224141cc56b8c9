// Host-side launch interface between the C-ABI layer (sb_abi.cu) and the kernels.
#pragma once

#include <cuda.h>
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
  int logits_bf16, no_renorm;  // router variants: bf16-rounded logits, no renormalisation
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
  int32_t* err;      // set here, before the grouped kernels: 0, or 1 if *gate_err is set
  const int32_t* gate_err;   // the tensor-core gate's flag when that gate ran, else null
  int pass_max;      // tensor-core path: tokens per pass of a routed expert (0: no pass table)
  int32_t* pass_off; // [E+1] by active slot: first pass of the slot, total passes at [n_active]
  int32_t* pass_slot;// [routed passes] active slot of each pass
  int32_t* pass_pb;  // [routed passes] first token (within its expert) of each pass
  // hybrid dispatch: experts routing >= hot_min tokens get their passes (of pass_max2 tokens) in a
  // second table, for the prefill kernel, and none in the first (hot_min 0: one table)
  int hot_min;
  int pass_max2;
  int32_t* pass_off2;
  int32_t* pass_slot2;
  int32_t* pass_pb2;
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
  int items_per_expert;  // row blocks per weight matrix (items per pass, tensor-core path)
  int* err;            // device flag: set to 1 if a bounded wait gave up (must start at 0)
  __nv_bfloat16* hbf;  // tensor-core path: h in bf16 (W13 writes it, the W2 panel quantises it)
  int n_experts;       // tensor-core path: matrices in the routed bank
  uint32_t wait_limit; // tensor-core path: polls of the consumer-side waits (0: the kernel's default)
  int bs_mask;         // verify kernel: bit f set = items of weight format f run block-scaled
                       // (FMT_MXFP4, FMT_FP8; only with power-of-two activation and weight scales)
  int activation;      // ACT_SWIGLU (Expert.forward) or ACT_SITU (K3's SituAndMul)
  float act_beta, act_lbeta;  // situ: beta, and linear_beta (0: up is not transformed)
  int weight_after;    // 1: the routing weight is not applied to h (the combine applies it to o)
  int ksplit;          // verify kernel, DENSE: K pieces of each item (<= 1: none)
  int kstages;         // stages (128 K) per piece, a multiple of the kernel's unit of 2
  float* part;         // ksplit > 1: fp32 partials [n_sh_pass * nrb][ksplit][128 rows][16]
  int* kcnt;           // ksplit > 1: [n_sh_pass * nrb] pieces finished (zeroed by the panel kernel)
  int* sched;          // verify kernel: launch-wide item counter (zeroed beforehand), or NULL for a
                       // round-robin schedule
  int hpad;            // verify kernel, W13: h rows in the prefill kernel's padded row space (hybrid),
  int hsh0;            // the shared expert's first h row there
};

enum Activation { ACT_SWIGLU = 0, ACT_SITU = 1 };

// Tensor-core path: the activation operand of every pass, prepared before the grouped launch.
// Pass order: the shared expert's (or the dense matrix's) passes first, then each active expert's
// in active-slot order. A pass holds up to 16 B rows: 16 tokens, or for NVFP4 weights 8 tokens
// twice (rows 2t / 2t+1 keep the first / second 16 K of every 32 K, so each output column pair
// carries the two per-16 partial sums).
struct TcPlan {
  const uint8_t* bpanel;    // [pass][stage][16 rows][128 B] e4m3, 128-byte swizzled
  const float* apanel;      // [pass][stage][16] activation scale of each B row (0 for empty rows)
  const int32_t* pass_off;  // [E+1] by active slot (routed passes follow the n_sh_pass shared ones)
  const int32_t* pass_slot; // [routed passes] active slot of each routed pass
  const int32_t* pass_pb;   // [routed passes] first token of each routed pass within its expert
  int n_sh_pass;
};

struct PanelArgs {
  int mode;                 // MODE_W13 / MODE_DENSE: e4m3 rows; MODE_W2: bf16 rows quantised here
  int m, topk, k, act_pow2;
  int has_shared, n_sh_pass;
  int nv_routed, nv_shared; // 1: NVFP4 weights (8 tokens per pass, split rows)
  const uint8_t* xq;        // [rows][k] e4m3 (W13: tokens; DENSE: the caller's activations)
  const float* xs;          // [rows][k/128]
  const __nv_bfloat16* hbf; // W2: [P + m][k] bf16
  const int32_t* counts;
  const int32_t* offsets;
  const int32_t* active;
  const int32_t* n_active;
  const int32_t* pass_off;
  const int32_t* pair_tok;
  uint8_t* bpanel;
  float* apanel;
  int* kzero;               // counters of the next grouped launch's K pieces, zeroed here (or NULL)
  int nkzero;
  int* zero_err;            // the next grouped launch's error flag, cleared here (or NULL)
  int* zero_sched;          // the next grouped launch's item counter, cleared here (or NULL)
  int hot_min;              // hybrid dispatch: routed experts with >= hot_min tokens are skipped
  int hpad;                 // W2: h rows in the prefill kernel's padded row space (hybrid),
  int hsh0;                 // the shared expert's first h row there
};

__host__ __device__ inline int tc_pass_max(int fmt) { return fmt == 1 ? 8 : 16; }

// Hybrid dispatch: a routed expert is "hot", and runs on the prefill kernel, when it routes at least
// three of the verify kernel's passes' worth of tokens, four for FP8 experts (the measured
// break-even of a 128-token prefill pass against narrow verify passes that each stream the expert's
// weights; the verify kernel streams FP8 closer to the HBM rate).
__host__ __device__ inline int hybrid_hot_min(int fmt) { return fmt == 3 ? 4 * tc_pass_max(fmt) : 3 * tc_pass_max(fmt); }

// Padded row space of the prefill kernel's operands: expert e's rows start at a multiple of 8.
__host__ __device__ inline int wide_pbase(int off, int e) { return (off + 8 * e + 7) & ~7; }

// Byte offset of weight row r's four e8m0 scales within a tensor-core-layout MXFP4 scale stage
// (128 rows x 4 per-32 scales): 16 (r % 32) + 4 (r / 32), the source order of the scale-factor copy
// into tensor memory (sb_tc.cu).
__host__ __device__ inline int mx_scale_off(int r) { return 16 * (r & 31) + 4 * (r >> 5); }

// K-split width of the gate logits (both kernels): 512 when H allows it, else 256 (H % 256 == 0).
__host__ __device__ inline int gate_ksplit(int h) { return h % 512 == 0 ? 512 : 256; }
cudaError_t launch_gate_logits(const void* x, const void* w, float* logits, int m, int e, int h, cudaStream_t st);
// the same partial logits on the tensor cores (sb_gate.cu), for prefill batches
cudaError_t launch_gate_tc(const void* x, const void* w, float* part, int m, int e, int h, int kspl, int* err,
                           cudaStream_t st);
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
cudaError_t launch_tc_panel(const PanelArgs& a, int max_slots, cudaStream_t st);
cudaError_t launch_tc_grouped(const GroupedArgs& a, const TcPlan& plan, int max_items, cudaStream_t st);
// K3 mode (KimiSparseMoeBlock.moe_infer): the caller's routing into the workspace (ids checked against
// the expert count: an id out of range sets *err to 1 and is replaced by 0), the bf16 activations
// copied as they are into the prefill kernel's operand layouts, and the slot-order weighted combine.
cudaError_t launch_routing_in(const int64_t* idx_in, const float* w_in, int m, int topk, int n_experts,
                              int32_t* topk_idx, float* topk_w, int* err, cudaStream_t st);
cudaError_t launch_wide_x_raw(const void* x, const int32_t* pair_tok, const int32_t* offsets, int n_experts, int P,
                              int h, int64_t r_pad, void* xw, float* cvec, cudaStream_t st);
cudaError_t launch_wide_h_raw(const __nv_bfloat16* hbf, int64_t rows, int64_t r_pad, int k, void* hw, float* cvec,
                              cudaStream_t st);
cudaError_t launch_combine_weighted(const __nv_bfloat16* o, const float* topk_w, int m, int topk, int h,
                                    __nv_bfloat16* y, cudaStream_t st);
cudaError_t launch_wire_pack(const void* x, int64_t rows, int64_t dim, uint8_t* q, void* s, cudaStream_t st);
cudaError_t launch_residual_rmsnorm(void* x, const void* y, int64_t rows, int64_t dim, const float* w, float eps,
                                    void* out, cudaStream_t st);
cudaError_t launch_wire_unpack(const uint8_t* q, const void* s, int64_t rows, int64_t dim, void* y, cudaStream_t st);
cudaError_t launch_combine_pack(const __nv_bfloat16* o, const int32_t* topk_idx, int m, int topk, int h,
                                int has_shared, __nv_bfloat16* y, uint8_t* q, __nv_bfloat16* s, cudaStream_t st);
constexpr int TC_WIDE_PASS = 128;   // tokens per pass of the prefill kernel (sb_tcw.cu)
// Prefill kernel (sb_tcw.cu). B operand matrices live in a padded row space of r_pad rows (expert e's
// rows from a multiple of 8, the shared expert's tokens from sb_row), chunk-major and 128B-swizzled;
// 16-bit rows (f16, or bf16 for the routed rows of MXFP4 layers), each divided by the power of two
// cvec[row]; with `split` a second plane of residuals follows, so that hi + lo carries a
// non-power-of-two activation scale's product.
constexpr int wide_sb_row(int64_t P, int64_t n_experts) { return (int)((P + 8 * n_experts + 7) & ~(int64_t)7); }
cudaError_t launch_tc_wide(const GroupedArgs& g, const TcPlan& plan, const void* bmat, const float* cvec,
                           int64_t r_pad, int sb_row, int split, int max_items, cudaStream_t st);
// (hot_min > 0: the hybrid dispatch, rows of experts routing fewer tokens are skipped; m: the shared
// expert's rows, 0 when it does not run in the prefill kernel)
cudaError_t launch_wide_x(const uint8_t* xq, const float* xs, const int32_t* pair_tok, const int32_t* offsets,
                          int n_experts, int m, int P, int h, int64_t r_pad, int sb_row, int split, int routed_bf16,
                          int hot_min, void* xw, float* cvec, cudaStream_t st);
// (hot_min > 0: the hybrid dispatch, only hot experts' rows and the first sh_rows shared rows)
cudaError_t launch_wide_h(const __nv_bfloat16* hbf, int64_t rows, int64_t r_pad, int sb_row, int k, int pow2,
                          int routed_bf16, const int32_t* offsets, int n_experts, int hot_min, int sh_rows, void* hw,
                          float* cvec, cudaStream_t st);
cudaError_t launch_tc_tile(int fmt, int kind, bool scales, const void* src, void* dst, int64_t n_mat, int64_t n,
                           int64_t k, cudaStream_t st);

int num_sms();

// Launch with programmatic stream serialisation (the kernel must call pdl_wait() before it touches
// memory another kernel of the stream reads or writes).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace sb
