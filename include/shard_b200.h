/* shard_b200 — C ABI of the B200 (sm_100a) MoE stage forward.
 *
 * One shared library, libshard_b200.so, exports every entry point below. Signatures carry plain
 * device pointers, sizes and a cudaStream_t (passed as void*), never framework types, so any host
 * (Python ctypes, cgo, JNI, C++) can bind them. All work is enqueued on the caller's stream; no
 * entry point synchronises the device, allocates device memory or branches on device data on the
 * host, so the forward is capturable into a CUDA graph and needs no host sync.
 *
 * Reference interfaces each entry point replaces are cited as leyten/shard file:line.
 *
 * Return value: SB_OK (0) or a negative SB_ERR_* code; sb_last_error() describes the last failure
 * on the calling thread.
 */
#ifndef SHARD_B200_H
#define SHARD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SB_ABI_VERSION 7

enum sb_status {
  SB_OK = 0,
  SB_ERR_ARG = -1,        /* null pointer / bad enum */
  SB_ERR_SHAPE = -2,      /* a dimension the kernels cannot hold (see each entry) */
  SB_ERR_FORMAT = -3,     /* unsupported weight format */
  SB_ERR_WORKSPACE = -4,  /* workspace too small */
  SB_ERR_CUDA = -5,       /* a CUDA launch failed */
  SB_ERR_UNSUPPORTED = -6 /* a configuration the forward declines (caller falls back) */
};

/* Weight formats of routed experts (shared experts are always SB_FMT_FP8). */
enum sb_format {
  SB_FMT_NVFP4 = 1, /* e2m1 x2 per byte (low nibble first), e4m3 scale per 16 K, fp32 tensor scale */
  SB_FMT_MXFP4 = 2, /* e2m1 x2 per byte, e8m0 scale per 32 K (the reference's fp4 expert format) */
  SB_FMT_FP8 = 3    /* e4m3, fp32 scale per 128x128 block */
};

/* Gate score functions, model.py:571-576 (Gate.forward). */
enum sb_score { SB_SCORE_SOFTMAX = 0, SB_SCORE_SIGMOID = 1, SB_SCORE_SQRTSOFTPLUS = 2 };

/* Which matrix a tiling call lays out. W13 fuses w1 and w3 ([2I, H], w1 rows then w3 rows, the
 * reference's bank form, engines/deepseek_v4/v4_moe_grouped.py:382-540); a tile interleaves 8 w1
 * rows with the same 8 w3 rows so one tensor-core tile yields gate and up values for the same
 * intermediate index. PLAIN is any other [N, K] matrix (w2, dense projections). */
enum sb_matrix_kind { SB_MAT_PLAIN = 0, SB_MAT_W13 = 1 };

/* Weight layouts (the forward's two kernel families).
 *  SB_LAYOUT_FRAGMENT  16-row tiles of mma.sync register fragments (grouped_kernel).
 *  SB_LAYOUT_TC        128-row blocks x 128-K stages for tcgen05 (one TMA box per stage): fp4 values
 *                      [128 rows][64 B], FP8 values [128 rows][128 B], NVFP4 scales [128 rows][8 B], MXFP4
 *                      scales [128 rows][4 B], FP8 scales [4] fp32 (block scale of rows 0-63, of rows
 *                      64-127, two zero pads). A W13 block holds 64 w1 rows then the same 64 w3 rows.
 *                      Pass the layout OR'ed into `kind` of the tiling calls (e.g. SB_MAT_W13 | SB_KIND_TC). */
enum sb_layout { SB_LAYOUT_FRAGMENT = 0, SB_LAYOUT_TC = 1 };
#define SB_KIND_TC 4

/* One MoE layer as the forward reads it. All pointers are device pointers; weights are in the
 * layout `layout` names, produced by sb_tile_weights / sb_tile_scales: SB_LAYOUT_TC (the default of
 * the Python host, the tcgen05 kernels) stores 128-row blocks x 128-K stages, one TMA box per stage;
 * SB_LAYOUT_FRAGMENT stores 16-row tiles of mma.sync register fragments for the mma.sync kernel
 * family. See enum sb_layout.
 * Mirrors the state MoE.forward reads, model.py:614-649: self.gate.{weight,bias,tid2eid,
 * score_func,route_scale,topk}, the expert bank, self.shared_experts, Expert.swiglu_limit. */
typedef struct sb_moe_layer {
  int32_t hidden;        /* H (dim): multiple of 256 */
  int32_t inter;         /* I (moe_inter_dim): multiple of 128 */
  int32_t n_experts;     /* E routed experts: 1..1024 */
  int32_t topk;          /* k: 1..16 */
  int32_t expert_fmt;    /* sb_format */
  int32_t has_shared;    /* 1: one FP8 shared expert (n_shared_experts == 1) */
  int32_t score_func;    /* sb_score */
  int32_t act_pow2;      /* 1: activation scales 2^ceil(log2(amax/448)) (scale_fmt "ue8m0"); 0: amax/448 */
  float route_scale;
  float swiglu_limit;    /* 0 disables the clamp */
  const void* gate_w;    /* bf16 [E, H] */
  const float* gate_bias;/* fp32 [E] (selection only) or NULL */
  const int32_t* tid2eid;/* hash routing: int32 [vocab, k], or NULL for score routing */
  int64_t vocab;
  /* routed experts, tiled: expert e's w13 at w13 + e * sb_tiled_bytes(fmt, 2I, H), etc. */
  const void* w13;
  const void* w13_s;
  const float* w13_ts;   /* NVFP4: fp32 [E, 2] tensor scales (w1, w3); else NULL */
  const void* w2;
  const void* w2_s;
  const float* w2_ts;    /* NVFP4: fp32 [E] tensor scales; else NULL */
  /* shared expert (FP8, tiled) */
  const void* sh_w13;
  const void* sh_w13_s;
  const void* sh_w2;
  const void* sh_w2_s;
  int32_t layout;        /* sb_layout of every weight above */
  /* Router variants of other engines' MoE call sites (0 = the V4 Gate.forward):
   * logits_bf16  round the fp32 router logits to bf16 before scoring (a bf16 F.linear router,
   *              engines/minimax_m25/m25_stage.py:412-416)
   * no_renorm    keep the selected sigmoid/sqrtsoftplus weights un-normalised (FusedMoE
   *              renormalize=False, m25_stage.py:301) */
  int32_t logits_bf16;
  int32_t no_renorm;
  /* Which tensor-core grouped kernels run the experts (SB_LAYOUT_TC only): the verify kernel
   * (per-stage readback, passes of 8-16 tokens), the prefill kernel (16-bit operands, the whole K in
   * TMEM, passes of 128 tokens), or the hybrid dispatch (SB_PREFILL_HYBRID: each routed expert that
   * routes at least 24 tokens (NVFP4), 48 (MXFP4) or 64 (FP8), three or four verify passes, on the
   * prefill kernel, the others on the verify kernel; the shared expert on the prefill kernel from
   * 256 tokens on, 128 with fp32 activation scales). SB_PREFILL_AUTO picks the hybrid dispatch when
   * the batch routes at least 4 tokens per expert on average, else the verify kernel, and always the
   * verify kernel for FP8 experts (it streams FP8 weights faster than the prefill kernel). A forced
   * VERIFY or WIDE choice is row-invariant (a token's output does not depend on its batch); the
   * hybrid dispatch is not, since an expert's kernel depends on the batch. The kernels differ only in
   * summation order. The prefill kernel's dequantised weights are exact for NVFP4, MXFP4 and for
   * FP8 whose 128x128 block scales are powers of two; pick SB_PREFILL_VERIFY for FP8 banks with
   * other scales. */
  int32_t prefill;
  /* 1: every FP8 128x128 block scale of the layer (the shared expert's and, for FP8 experts, the
   * routed bank's) is a power of two, as in ue8m0-scaled checkpoints (the reference stores them as
   * float8_e8m0fnu, model.py:143-147). With power-of-two activation scales (act_pow2) the verify
   * kernel then runs FP8 items on the block-scaled tensor-core MMA (ue8m0 scale factors, the whole K
   * accumulated in tensor memory); MXFP4 items run it whenever act_pow2. 0: FP8 items keep the
   * per-stage readback, which applies any fp32 scale. */
  int32_t fp8_pow2;
  /* Which MoE call site the layer serves (enum sb_moe_mode):
   * SB_MODE_V4  MoE.forward of DeepSeek-V4 (model.py:634-649): the gate routes, activations are
   *             act_quant'ed to e4m3 per 128, SwiGLU, the routing weight scales h before w2, the
   *             combine sums in ascending expert id with the shared expert last.
   * SB_MODE_K3  KimiSparseMoeBlock.moe_infer of Kimi-K3 (vendor/kimi_k3_ref/modeling_kimi_linear.py:
   *             850-876, the seam engines/kimi_k3/k3_moe_mxfp4.py:405-412 replaces): the caller routes
   *             (sb_moe_forward_routed), activations stay bf16 (4-bit weights, 16-bit activations),
   *             the activation is situ (below), each expert's bf16 output is scaled by its routing
   *             weight in fp32 and the slots are summed in slot order. MXFP4 experts, no shared
   *             expert, tensor-core layout; the prefill kernel runs every batch size. */
  int32_t mode;
  /* SB_MODE_K3's SituAndMul (modeling_kimi_linear.py:64-82): (beta tanh(g / beta)) sigmoid(g) times
   * up, up replaced by linear_beta tanh(up / linear_beta) when linear_beta > 0. */
  float situ_beta;
  float situ_linear_beta;
} sb_moe_layer;

enum sb_moe_mode { SB_MODE_V4 = 0, SB_MODE_K3 = 1 };

enum sb_prefill { SB_PREFILL_AUTO = 0, SB_PREFILL_VERIFY = 1, SB_PREFILL_WIDE = 2, SB_PREFILL_HYBRID = 3 };

/* ── introspection ───────────────────────────────────────────────────────────────────────────── */
int sb_abi_version(void);
const char* sb_last_error(void);

/* Bytes of one tiled [N, K] weight matrix, values and scales (identical to the canonical sizes). */
size_t sb_tiled_bytes(int fmt, int64_t n, int64_t k);
size_t sb_tiled_scale_bytes(int fmt, int kind, int64_t n, int64_t k);

/* ── load-time layout (replaces _relayout_moe / bank_layout, v4_moe_grouped.py:382-540) ───────── */
/* Canonical -> tiled, for n_mat matrices of [N, K] stored back to back.
 * src: fp4 packed [n_mat, N, K/2] (low nibble first) or fp8 [n_mat, N, K].  dst: same bytes. */
int sb_tile_weights(int fmt, int kind, const void* src, void* dst, int64_t n_mat, int64_t n, int64_t k,
                    void* stream);
/* src scales: NVFP4 e4m3 [n_mat, N, K/16]; MXFP4 e8m0 [n_mat, N, K/32]; FP8 fp32 [n_mat, N/128, K/128]. */
int sb_tile_scales(int fmt, int kind, const void* src, void* dst, int64_t n_mat, int64_t n, int64_t k,
                   void* stream);

/* ── the kernel-level seam (the reference's `kernel` module, kernel.py:105-125, 257-273, 518-536) ── */
/* act_quant: bf16 x [M, K] -> e4m3 q [M, K] + fp32 s [M, K/128]; pow2 selects scale_fmt "ue8m0". */
int sb_act_quant(const void* x, int64_t m, int64_t k, int pow2, void* q, float* s, void* stream);
/* fp8_gemm / fp4_gemm: y bf16 [M, N] = dequant(q, s) @ dequant(W)^T with W tiled (PLAIN kind, `layout`).
 * ts: NVFP4 tensor scale (device fp32 [1]) or NULL. The tensor-core layout needs a workspace of
 * sb_qgemm_workspace_bytes() (the activation panel, and for narrow batches (m <= 64) of matrices
 * with few 128-row blocks the fp32 partials of K pieces, summed in K order by the last piece of each
 * block; the split depends on the shape alone); the size for m serves every m' <= m. The fragment
 * layout needs none (0, NULL ok). */
size_t sb_qgemm_workspace_bytes(int fmt, int layout, int64_t n, int64_t k, int64_t m);
int sb_qgemm(int fmt, int layout, const void* w, const void* w_s, const float* ts, int64_t n, int64_t k,
             const void* q, const float* s, int64_t m, void* y, void* workspace, size_t workspace_bytes,
             void* stream);

/* sb_qgemm over the tensor-core layout (SB_LAYOUT_TC weights, n % 128 == 0) for callers that cannot
 * allocate device memory: it allocates nothing and takes no workspace. No counterpart in the
 * reference (its fp8_gemm / fp4_gemm allocate through torch).
 * Its scratch is a file-scope device region of SB_QGEMM_STATIC_SCRATCH_BYTES per device: the
 * error flag (cleared by every call before its kernels run) and the activation panel of
 * ceil(m / p) passes x k/128 stages, 2112 bytes each (p = 8 for NVFP4, 16 otherwise). Shapes that
 * need more return SB_ERR_SHAPE with the byte count (at k = 7168: m <= 272, or m <= 136 for NVFP4).
 * Every call looks up the region's address on the current device (cudaGetSymbolAddress); the first
 * call on a device also loads the library's module there, so make that first call before any stream
 * capture. Every call on a device uses the same region: calls that overlap in time (other streams,
 * other threads) race on it and must be serialised by the caller. */
#define SB_QGEMM_STATIC_SCRATCH_BYTES (2u << 20)
int sb_qgemm_static(int fmt, const void* w, const void* w_s, const float* ts, int64_t n, int64_t k,
                    const void* q, const float* s, int64_t m, void* y, void* stream);
/* The error flag of the last sb_qgemm_static call on the current device: *host_out = 0, or 1 if one of
 * its kernels gave up a bounded wait (its y is then incomplete). Enqueues the read on `stream`
 * after that call and synchronises the stream. The next sb_qgemm_static call clears the flag. */
int sb_qgemm_static_error(int* host_out, void* stream);

/* ── the MoE stage forward (MoE.forward, model.py:634-649; Gate.forward :569-589;
 *    Expert.forward :601-611; grouped decode v4_moe_grouped.py:634-709) ──────────────────────── */
/* Bytes of workspace for a forward of up to m tokens (the size serves every m' <= m). Forwards that
 * share a workspace must not overlap on the GPU. */
size_t sb_moe_workspace_bytes(const sb_moe_layer* layer, int64_t m);
/* x bf16 [M, H] -> y bf16 [M, H]. input_ids int64 [M] (read only for hash routing; may be NULL
 * otherwise). Optional outputs (NULL to skip): routing weights fp32 [M, k] and top-k indices
 * int64 [M, k] exactly as Gate.forward returns them. */
int sb_moe_forward(const sb_moe_layer* layer, const void* x, int64_t m, const int64_t* input_ids,
                   void* y, float* out_weights, int64_t* out_indices, void* workspace,
                   size_t workspace_bytes, void* stream);

/* The forward with the caller's routing, for SB_MODE_K3 layers (KimiSparseMoeBlock.moe_infer(x,
 * topk_ids, topk_weight), modeling_kimi_linear.py:850-876): x bf16 [M, H], topk_idx int64 [M, k]
 * (distinct ids per token, as topk returns them), topk_w fp32 [M, k] -> y bf16 [M, H]. An id outside
 * [0, E) is replaced by 0 and sets the workspace error flag. gate_w may be NULL for such layers. */
int sb_moe_forward_routed(const sb_moe_layer* layer, const void* x, int64_t m, const int64_t* topk_idx,
                          const float* topk_w, void* y, void* workspace, size_t workspace_bytes, void* stream);

/* sb_moe_forward that also records up to six CUDA events (cudaEvent_t, NULL entries skipped) on
 * the stream: before routing, after routing, after the permutation, after the grouped w13 pass,
 * after the grouped w2 pass, after the combine. For per-phase timing; same results. */
int sb_moe_forward_profiled(const sb_moe_layer* layer, const void* x, int64_t m, const int64_t* input_ids,
                            void* y, float* out_weights, int64_t* out_indices, void* workspace,
                            size_t workspace_bytes, void* stream, void* const* events);

/* sb_moe_forward whose last step also emits the stage-boundary FP8 wire form of y (the combine with
 * the pack fused in; the pack is sb_wire_pack's): q e4m3 [M, H], scale bf16 [M]. y may be NULL when
 * only the wire form is needed. hidden <= 8192. */
int sb_moe_forward_wire(const sb_moe_layer* layer, const void* x, int64_t m, const int64_t* input_ids, void* y,
                        void* q, void* scale, float* out_weights, int64_t* out_indices, void* workspace,
                        size_t workspace_bytes, void* stream);

/* ── the stage-boundary FP8 wire (engines/deepseek_v4/v4_pipe.py:335-384, _pack_t / _unpack_t) ─── */
/* pack: x bf16 [rows, dim] -> q e4m3 [rows, dim], scale bf16 [rows]; one scale per row:
 * bf16(clamp(amax / 448, 1e-8, bf16 max)), q = e4m3(clamp(x / scale, +-448)). dim % 8 == 0. */
int sb_wire_pack(const void* x, int64_t rows, int64_t dim, void* q, void* scale, void* stream);
/* unpack: y bf16 [rows, dim] = bf16(e4m3(q) * scale). */
int sb_wire_unpack(const void* q, const void* scale, int64_t rows, int64_t dim, void* y, void* stream);

/* The block around the MoE operator (Block.forward's ffn half, model.py:701-706, without its
 * hyper-connections; RMSNorm.forward, model.py:197-202): x bf16 [rows, dim] (in/out) <- bf16(x + y)
 * when y is given (the residual stream), then out bf16 = bf16(weight * (x * rsqrt(mean(x^2) + eps))) in
 * fp32; weight NULL means ones; out NULL does the residual add alone. dim % 8 == 0. */
int sb_residual_rmsnorm(void* x, const void* y, int64_t rows, int64_t dim, const float* weight, float eps, void* out,
                        void* stream);

/* Routing alone (Gate.forward, model.py:569-589): weights fp32 [M, k], indices int64 [M, k]. */
int sb_moe_route(const sb_moe_layer* layer, const void* x, int64_t m, const int64_t* input_ids,
                 float* out_weights, int64_t* out_indices, void* workspace, size_t workspace_bytes,
                 void* stream);

/* Test hook of the timeout path. Sets, for every later launch in this process, the number of polls
 * the tensor-core kernels' consumer-side waits (on operands and accumulators) make before they give
 * up: the kernel then sets the workspace error flag, drains its copies and MMAs in flight, frees its
 * tensor memory and returns, and the forward's output is incomplete. Waits for free slots and the
 * final drains keep their normal limits. polls = 0 restores each kernel's default. */
int sb_debug_set_wait_limit(int64_t polls);

/* Format self-test: decodes a fixed set of e2m1 / e4m3 / e8m0 codes on the device into out
 * (fp32 [64]) so a test can compare them with the host tables. */
int sb_selftest_formats(float* out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SHARD_B200_H */
