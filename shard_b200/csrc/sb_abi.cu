// extern "C" entry points of libshard_b200.so (declared in include/shard_b200.h).
//
// Every entry point validates its shapes and pointers on the host, then enqueues kernels on the
// caller's stream. None allocates, synchronises or reads device memory on the host.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <string>

#include "../../include/shard_b200.h"
#include "sb_launch.h"

namespace {

thread_local std::string g_err;

// Consumer-side wait limit of the tensor-core kernels (polls; 0 = each kernel's default), set by
// sb_debug_set_wait_limit for tests of the timeout path.
std::atomic<uint32_t> g_wait_limit{0};

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return SB_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

// The forward's scratch regions, carved from one caller-provided workspace.
struct Workspace {
  int32_t* err;      // offset 0: device error flag (set afresh by every forward; 1 = a bounded wait gave up);
                     // offset 4: the tensor-core gate's flag (cleared before it runs), folded into it
  float* logits;
  int32_t* topk_idx;
  float* topk_w;
  uint8_t* xq;
  float* xs;
  int32_t* counts;
  int32_t* offsets;
  int32_t* active;
  int32_t* n_active;
  int32_t* pair_tok;
  int32_t* pair_slot;
  uint8_t* hq;
  float* hs;
  __nv_bfloat16* o;
  __nv_bfloat16* hbf;  // tensor-core layout: h in bf16 (quantised per 128 K into the w2 panel)
  int32_t* pass_off;   // tensor-core layout: first pass of each active slot
  int32_t* pass_slot;  //                     slot and first token of every routed pass
  int32_t* pass_pb;
  uint8_t* bpanel;     // tensor-core layout: B tiles of every (pass, stage)
  float* apanel;       //                     and their row scales
  __nv_bfloat16* xw;   // prefill kernel: act-quantised x as bf16, routed pairs in expert order + shared rows
  __nv_bfloat16* hw;   //                 act-quantised h as bf16, rows of h
  float* cx;           //                 the power of two each row of xw / hw was divided by
  float* ch;
  bool wide;           // the forward runs the prefill kernel alone
  bool hybrid;         // the forward runs the hybrid dispatch (both kernels)
  int64_t sb_row;      //   the padded row space: the shared expert's first row, and all rows
  int64_t wide_rows;
  int n_sh_pass;       // shared passes of the first pass table's kernel
  int n_sh_pass2;      // hybrid: shared passes of the prefill kernel
  int32_t* pass_off2;  // hybrid: the prefill kernel's pass table (hot experts)
  int32_t* pass_slot2;
  int32_t* pass_pb2;
  size_t bytes;
};

// The expert kernels of a forward on the tensor-core layout: the verify kernel alone, the prefill
// kernel alone, or the hybrid dispatch (each routed expert on the kernel its token count suits: the
// hot ones, routing >= sb::hybrid_hot_min tokens, on the prefill kernel, the others on the verify
// kernel; the shared expert on the prefill kernel from 2 full passes on). By default the hybrid
// dispatch runs once a batch routes >= 4 tokens per expert on average, below that the verify kernel;
// FP8 expert banks stay on the verify kernel, which streams FP8 weights faster than the prefill
// kernel converts them (measured at c3's shapes).
enum Kernels { K_VERIFY = 0, K_WIDE = 1, K_HYBRID = 2 };
constexpr int64_t HYBRID_TOKENS_PER_EXPERT = 4;
// the tensor-core gate takes the hybrid dispatch's batches of >= 128 tokens (one full tile; at c4's
// M=256 the CUDA-core gate GEMV took 8% of the forward) and every batch of a forced prefill kernel
constexpr int64_t TC_GATE_MIN_TOKENS = 128;
int kernels(const sb_moe_layer* L, int64_t m) {
  if (L->mode == SB_MODE_K3) return K_WIDE;   // 16-bit activations: the prefill kernel at every size
  if (L->layout != SB_LAYOUT_TC || L->prefill == SB_PREFILL_VERIFY) return K_VERIFY;
  if (L->prefill == SB_PREFILL_WIDE) return K_WIDE;
  if (L->prefill == SB_PREFILL_HYBRID) return K_HYBRID;
  if (L->expert_fmt == SB_FMT_FP8) return K_VERIFY;
  return m * L->topk >= HYBRID_TOKENS_PER_EXPERT * (int64_t)L->n_experts ? K_HYBRID : K_VERIFY;
}
bool use_wide(const sb_moe_layer* L, int64_t m) { return kernels(L, m) == K_WIDE; }
bool use_hybrid(const sb_moe_layer* L, int64_t m) { return kernels(L, m) == K_HYBRID; }
bool tc_gate(const sb_moe_layer* L, int64_t m) {
  return use_wide(L, m) || (use_hybrid(L, m) && m >= TC_GATE_MIN_TOKENS);
}

// Tokens per pass of a routed expert and of the shared expert. The prefill kernel takes passes of
// 128 tokens, or 64 when fp32 activation scales double its B operand (hi and lo planes).
int64_t wide_pass(const sb_moe_layer* L) {
  return (L->act_pow2 || L->mode == SB_MODE_K3) ? sb::TC_WIDE_PASS : sb::TC_WIDE_PASS / 2;
}

// hi and lo planes of the prefill kernel's B operands (fp32 activation scales), else one
int64_t wide_planes(const sb_moe_layer* L) { return (L->act_pow2 || L->mode == SB_MODE_K3) ? 1 : 2; }

// hybrid dispatch: the shared expert runs on the prefill kernel once it fills HYBRID_SHARED_PASSES of
// its passes (below that its many narrow verify passes spread over the verify kernel's CTAs beat a
// few long prefill items)
constexpr int64_t HYBRID_SHARED_PASSES = 2;
bool hybrid_shared_wide(const sb_moe_layer* L, int64_t m) {
  return L->has_shared && use_hybrid(L, m) && m >= HYBRID_SHARED_PASSES * wide_pass(L);
}

// Tokens per pass of the first pass table (the only one, or the hybrid dispatch's verify table).
int64_t routed_pass_max(const sb_moe_layer* L, int64_t m) {
  return use_wide(L, m) ? wide_pass(L) : sb::tc_pass_max(L->expert_fmt);
}

// Tensor-core layout: passes of the shared expert in the first table's kernel (FP8: 16 tokens each,
// more in the prefill kernel), and in the hybrid dispatch's prefill kernel.
int64_t shared_passes(const sb_moe_layer* L, int64_t m) {
  if (!L->has_shared || hybrid_shared_wide(L, m)) return 0;
  const int64_t pm = use_wide(L, m) ? wide_pass(L) : 16;
  return (m + pm - 1) / pm;
}
int64_t shared_passes_wide(const sb_moe_layer* L, int64_t m) {
  return hybrid_shared_wide(L, m) ? (m + wide_pass(L) - 1) / wide_pass(L) : 0;
}

// Upper bound of the routed passes of one grouped launch: sum over experts of
// ceil(count / pass_max) <= P / pass_max + (active experts).
int64_t max_routed_passes(const sb_moe_layer* L, int64_t m) {
  const int64_t P = m * L->topk, E = L->n_experts;
  return P / routed_pass_max(L, m) + (P < E ? P : E);
}
int64_t max_routed_passes_wide(const sb_moe_layer* L, int64_t m) {
  const int64_t P = m * L->topk, E = L->n_experts;
  return use_hybrid(L, m) ? P / wide_pass(L) + (P < E ? P : E) : 0;
}

int64_t max_passes(const sb_moe_layer* L, int64_t m) { return shared_passes(L, m) + max_routed_passes(L, m); }

Workspace carve(const sb_moe_layer* L, int64_t m, uint8_t* base) {
  Workspace w;
  const int64_t E = L->n_experts, K = L->topk, H = L->hidden, I = L->inter;
  const int64_t P = m * K, R = P + m;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t* p = base ? base + off : nullptr;
    off += align256(bytes);
    return p;
  };
  w.err = (int32_t*)take(4 * sizeof(int32_t));   // [0] error flag, [1] gate / routing flag, [2] item counter
  // partial gate logits, one [M, E] slab per 512- (or 256-) wide K split
  w.logits = (float*)take(sizeof(float) * m * E * (H / (H % 512 == 0 ? 512 : 256)));
  w.topk_idx = (int32_t*)take(sizeof(int32_t) * P);
  w.topk_w = (float*)take(sizeof(float) * P);
  w.xq = take((size_t)m * H);
  w.xs = (float*)take(sizeof(float) * m * (H / 128));
  w.counts = (int32_t*)take(sizeof(int32_t) * E);
  w.offsets = (int32_t*)take(sizeof(int32_t) * (E + 1));
  w.active = (int32_t*)take(sizeof(int32_t) * E);
  w.n_active = (int32_t*)take(sizeof(int32_t));
  w.pair_tok = (int32_t*)take(sizeof(int32_t) * P);
  w.pair_slot = (int32_t*)take(sizeof(int32_t) * P);
  const bool tc = L->layout == SB_LAYOUT_TC;
  w.hq = take(tc ? 0 : (size_t)R * I);
  w.hs = (float*)take(tc ? 0 : sizeof(float) * R * (I / 128));
  w.o = (__nv_bfloat16*)take(sizeof(__nv_bfloat16) * R * H);
  // the prefill kernel keeps h in the padded row space of its B operands (wide_rows >= R)
  w.wide = use_wide(L, m);
  w.hybrid = use_hybrid(L, m);
  const bool wide_ops = w.wide || w.hybrid;   // the prefill kernel's operand matrices
  w.sb_row = sb::wide_sb_row(P, E);
  w.wide_rows = w.sb_row + ((m + 7) & ~(int64_t)7);
  w.hbf = (__nv_bfloat16*)take(tc ? sizeof(__nv_bfloat16) * (wide_ops ? w.wide_rows : R) * I : 0);
  w.pass_off = (int32_t*)take(tc ? sizeof(int32_t) * (E + 1) : 0);
  w.pass_slot = (int32_t*)take(tc ? sizeof(int32_t) * max_routed_passes(L, m) : 0);
  w.pass_pb = (int32_t*)take(tc ? sizeof(int32_t) * max_routed_passes(L, m) : 0);
  const int64_t panel_tiles = tc && !w.wide ? max_passes(L, m) * ((H > I ? H : I) / 128) : 0;
  w.bpanel = take((size_t)panel_tiles * 2048);
  w.apanel = (float*)take((size_t)panel_tiles * 16 * sizeof(float));
  // fp32 activation scales: a residual plane below each matrix (hi + lo)
  const int64_t planes = wide_planes(L);
  w.xw = (__nv_bfloat16*)take(wide_ops ? sizeof(__nv_bfloat16) * planes * w.wide_rows * H : 0);
  w.hw = (__nv_bfloat16*)take(wide_ops ? sizeof(__nv_bfloat16) * planes * w.wide_rows * I : 0);
  w.cx = (float*)take(wide_ops ? sizeof(float) * w.wide_rows : 0);
  w.ch = (float*)take(wide_ops ? sizeof(float) * w.wide_rows : 0);
  w.n_sh_pass = (int)shared_passes(L, m);
  w.n_sh_pass2 = (int)shared_passes_wide(L, m);
  w.pass_off2 = (int32_t*)take(w.hybrid ? sizeof(int32_t) * (E + 1) : 0);
  w.pass_slot2 = (int32_t*)take(w.hybrid ? sizeof(int32_t) * max_routed_passes_wide(L, m) : 0);
  w.pass_pb2 = (int32_t*)take(w.hybrid ? sizeof(int32_t) * max_routed_passes_wide(L, m) : 0);
  w.bytes = off;
  return w;
}

int check_layer(const sb_moe_layer* L) {
  if (!L) return fail(SB_ERR_ARG, "layer is NULL");
  if (L->hidden <= 0 || L->hidden % 256) return fail(SB_ERR_SHAPE, "hidden=%d must be a positive multiple of 256", L->hidden);
  if (L->inter <= 0 || L->inter % 128) return fail(SB_ERR_SHAPE, "inter=%d must be a positive multiple of 128", L->inter);
  if (L->n_experts < 1 || L->n_experts > 1024) return fail(SB_ERR_SHAPE, "n_experts=%d outside 1..1024", L->n_experts);
  if (L->topk < 1 || L->topk > 16 || L->topk > L->n_experts)
    return fail(SB_ERR_SHAPE, "topk=%d outside 1..min(16, n_experts)", L->topk);
  if (L->expert_fmt != SB_FMT_NVFP4 && L->expert_fmt != SB_FMT_MXFP4 && L->expert_fmt != SB_FMT_FP8)
    return fail(SB_ERR_FORMAT, "expert_fmt=%d unknown", L->expert_fmt);
  if (L->score_func < 0 || L->score_func > 2) return fail(SB_ERR_ARG, "score_func=%d unknown", L->score_func);
  if (L->mode != SB_MODE_V4 && L->mode != SB_MODE_K3) return fail(SB_ERR_ARG, "mode=%d unknown", L->mode);
  if (L->mode == SB_MODE_K3 &&
      (L->expert_fmt != SB_FMT_MXFP4 || L->has_shared || L->layout != SB_LAYOUT_TC || L->tid2eid ||
       !(L->situ_beta > 0.f) || L->situ_linear_beta < 0.f))
    return fail(SB_ERR_UNSUPPORTED,
                "K3 mode needs MXFP4 experts in the tensor-core layout, no shared expert, no hash routing, "
                "situ_beta > 0 and situ_linear_beta >= 0");
  if (L->mode == SB_MODE_V4 && !L->gate_w) return fail(SB_ERR_ARG, "gate_w is NULL");
  if (!L->w13 || !L->w13_s || !L->w2 || !L->w2_s) return fail(SB_ERR_ARG, "routed expert bank pointer is NULL");
  if (L->expert_fmt == SB_FMT_NVFP4 && (!L->w13_ts || !L->w2_ts))
    return fail(SB_ERR_ARG, "NVFP4 experts need w13_ts and w2_ts");
  if (L->has_shared && (!L->sh_w13 || !L->sh_w13_s || !L->sh_w2 || !L->sh_w2_s))
    return fail(SB_ERR_ARG, "shared expert pointer is NULL");
  if (!aligned16(L->w13) || !aligned16(L->w2) || (L->gate_w && !aligned16(L->gate_w)) ||
      (L->has_shared && (!aligned16(L->sh_w13) || !aligned16(L->sh_w2))))
    return fail(SB_ERR_ARG, "weight pointers must be 16-byte aligned");
  if (L->tid2eid && L->vocab <= 0) return fail(SB_ERR_ARG, "tid2eid given with vocab=%lld", (long long)L->vocab);
  if (L->layout != SB_LAYOUT_FRAGMENT && L->layout != SB_LAYOUT_TC) return fail(SB_ERR_ARG, "layout=%d unknown", L->layout);
  if (L->prefill < SB_PREFILL_AUTO || L->prefill > SB_PREFILL_HYBRID) return fail(SB_ERR_ARG, "prefill=%d unknown", L->prefill);
  return SB_OK;
}

sb::WeightSet routed_set(const sb_moe_layer* L, bool w13) {
  sb::WeightSet s;
  const int64_t H = L->hidden, I = L->inter;
  const int64_t n = w13 ? 2 * I : H, k = w13 ? H : I;
  s.w = (const uint8_t*)(w13 ? L->w13 : L->w2);
  s.s = (const uint8_t*)(w13 ? L->w13_s : L->w2_s);
  s.ts = L->expert_fmt == SB_FMT_NVFP4 ? (w13 ? L->w13_ts : L->w2_ts) : nullptr;
  s.ts_stride = w13 ? 2 : 1;
  s.w_stride = sb_tiled_bytes(L->expert_fmt, n, k);
  s.s_stride = sb_tiled_scale_bytes(L->expert_fmt, L->layout == SB_LAYOUT_TC ? SB_KIND_TC : 0, n, k);
  s.fmt = L->expert_fmt;
  return s;
}

sb::WeightSet shared_set(const sb_moe_layer* L, bool w13) {
  sb::WeightSet s;
  memset(&s, 0, sizeof s);
  s.w = (const uint8_t*)(w13 ? L->sh_w13 : L->sh_w2);
  s.s = (const uint8_t*)(w13 ? L->sh_w13_s : L->sh_w2_s);
  s.fmt = SB_FMT_FP8;
  return s;
}

}  // namespace

extern "C" {

int sb_abi_version(void) { return SB_ABI_VERSION; }

const char* sb_last_error(void) { return g_err.c_str(); }

size_t sb_tiled_bytes(int fmt, int64_t n, int64_t k) {
  if (fmt == SB_FMT_FP8) return (size_t)(n * k);
  if (fmt == SB_FMT_NVFP4 || fmt == SB_FMT_MXFP4) return (size_t)(n * k / 2);
  return 0;
}

size_t sb_tiled_scale_bytes(int fmt, int kind, int64_t n, int64_t k) {
  if (fmt == SB_FMT_NVFP4) return (size_t)(n * (k / 16));
  if (fmt == SB_FMT_MXFP4) return (size_t)(n * (k / 32));
  if (fmt == SB_FMT_FP8) return (kind & SB_KIND_TC) ? (size_t)((n / 128) * (k / 128) * 16) : (size_t)((n / 16) * (k / 128) * 8);
  return 0;
}

static int check_tile_args(int fmt, int kind, const void* src, const void* dst, int64_t n_mat, int64_t n, int64_t k) {
  if (!src || !dst) return fail(SB_ERR_ARG, "tile: NULL pointer");
  if (fmt != SB_FMT_NVFP4 && fmt != SB_FMT_MXFP4 && fmt != SB_FMT_FP8) return fail(SB_ERR_FORMAT, "tile: format %d", fmt);
  if ((kind & 3) != SB_MAT_PLAIN && (kind & 3) != SB_MAT_W13) return fail(SB_ERR_ARG, "tile: kind %d", kind);
  if ((kind & SB_KIND_TC) && (n < 128 || n % 128))
    return fail(SB_ERR_SHAPE, "tile: the tensor-core layout needs n %% 128 == 0 (n=%lld)", (long long)n);
  if (n_mat < 1 || n < 32 || n % 32 || k < 128 || k % 128)
    return fail(SB_ERR_SHAPE, "tile: need n %% 32 == 0 and k %% 128 == 0 (n=%lld k=%lld)", (long long)n, (long long)k);
  if ((kind & 3) == SB_MAT_W13 && (n / 2) % 128)
    return fail(SB_ERR_SHAPE, "tile: W13 needs the intermediate size n/2 %% 128 == 0 (n=%lld)", (long long)n);
  return SB_OK;
}

int sb_tile_weights(int fmt, int kind, const void* src, void* dst, int64_t n_mat, int64_t n, int64_t k, void* stream) {
  int rc = check_tile_args(fmt, kind, src, dst, n_mat, n, k);
  if (rc) return rc;
  if (!aligned16(dst)) return fail(SB_ERR_ARG, "tile: dst must be 16-byte aligned");
  if (kind & SB_KIND_TC)
    return cuda_check(sb::launch_tc_tile(fmt, kind & 3, false, src, dst, n_mat, n, k, (cudaStream_t)stream), "tile_weights");
  return cuda_check(sb::launch_tile_weights(fmt, kind, src, dst, n_mat, n, k, (cudaStream_t)stream), "tile_weights");
}

int sb_tile_scales(int fmt, int kind, const void* src, void* dst, int64_t n_mat, int64_t n, int64_t k, void* stream) {
  int rc = check_tile_args(fmt, kind, src, dst, n_mat, n, k);
  if (rc) return rc;
  if ((reinterpret_cast<uintptr_t>(dst) & 7u) != 0) return fail(SB_ERR_ARG, "tile: scale dst must be 8-byte aligned");
  if (kind & SB_KIND_TC)
    return cuda_check(sb::launch_tc_tile(fmt, kind & 3, true, src, dst, n_mat, n, k, (cudaStream_t)stream), "tile_scales");
  return cuda_check(sb::launch_tile_scales(fmt, kind, src, dst, n_mat, n, k, (cudaStream_t)stream), "tile_scales");
}

int sb_act_quant(const void* x, int64_t m, int64_t k, int pow2, void* q, float* s, void* stream) {
  if (!x || !q || !s) return fail(SB_ERR_ARG, "act_quant: NULL pointer");
  if (m < 0 || k <= 0 || k % 128) return fail(SB_ERR_SHAPE, "act_quant: k=%lld must be a multiple of 128", (long long)k);
  if (m == 0) return SB_OK;
  return cuda_check(sb::launch_act_quant(x, m, k, pow2, (uint8_t*)q, s, (cudaStream_t)stream), "act_quant");
}

// Dense tensor-core GEMM scratch: error flag, then the B panel of ceil(m / pass_max) passes.
static size_t qgemm_ws(int fmt, int layout, int64_t k, int64_t m, uint8_t* base, int** err, uint8_t** bpanel,
                       float** apanel) {
  if (layout != SB_LAYOUT_TC) return 0;
  const int64_t pm = sb::tc_pass_max(fmt);
  const int64_t tiles = ((m + pm - 1) / pm) * (k / 128);
  size_t off = 0;
  if (err) *err = base ? (int*)(base + off) : nullptr;
  off += 256;
  if (bpanel) *bpanel = base ? base + off : nullptr;
  off += align256((size_t)tiles * 2048);
  if (apanel) *apanel = base ? (float*)(base + off) : nullptr;
  off += align256((size_t)tiles * 16 * sizeof(float));
  return off;
}

// K pieces of a dense GEMM on the tensor-core layout. A narrow batch (m <= 64) of a matrix with few
// 128-row blocks gives the verify kernel fewer items than its 2 CTAs per SM, each streaming its
// rows' whole K through one ring, so most of HBM's bandwidth stays unused; splitting K into pieces
// of >= 2 stages raises the items to about 2 per SM (the reference re-tiles the same GEMV shapes
// for the same reason, v4_fp8_gemv.py:156-270). Returns the piece count (1: no split) and the
// stages per piece.
static int qgemm_ksplit(int fmt, int64_t n, int64_t k, int64_t m, int* kstages) {
  const int nst = (int)(k / 128);
  *kstages = nst;
  if (m < 1 || m > 64 || n % 128) return 1;
  const int64_t pm = sb::tc_pass_max(fmt);
  const int64_t items = ((m + pm - 1) / pm) * (n / 128);
  const int64_t target = 2 * 148;   // B200's SMs: a fixed figure, so the split (and the summation
                                    // order) is a function of the shape alone
  if (items >= target) return 1;
  int want = (int)((target + items - 1) / items);
  if (want > nst / 2) want = nst / 2;
  if (want < 2) return 1;
  const int per = (((nst + want - 1) / want) + 1) & ~1;   // a multiple of the kernel's 2-stage unit
  *kstages = per;
  return (nst + per - 1) / per;
}

// The pieces' fp32 partials ([pass x row block][piece][128 rows][16 tokens]) and their per-block
// counters, placed after the activation panel.
static size_t qgemm_part_bytes(int fmt, int64_t n, int64_t k, int64_t m) {
  int per = 0;
  const int ks = qgemm_ksplit(fmt, n, k, m, &per);
  if (ks <= 1) return 0;
  const int64_t pm = sb::tc_pass_max(fmt);
  const int64_t blocks = ((m + pm - 1) / pm) * (n / 128);
  return align256((size_t)blocks * ks * 2048 * sizeof(float)) + align256((size_t)blocks * sizeof(int32_t));
}

size_t sb_qgemm_workspace_bytes(int fmt, int layout, int64_t n, int64_t k, int64_t m) {
  if (k < 128 || k % 128 || m < 0) return 0;
  const int64_t mm = m < 1 ? 1 : m;
  size_t need = qgemm_ws(fmt, layout, k, mm, nullptr, nullptr, nullptr, nullptr);
  if (layout == SB_LAYOUT_TC)   // every m' <= m: the split ones add their partials
    for (int64_t q = 1; q <= mm && q <= 64; ++q) {
      const size_t e = qgemm_ws(fmt, layout, k, q, nullptr, nullptr, nullptr, nullptr) + qgemm_part_bytes(fmt, n, k, q);
      if (e > need) need = e;
    }
  return need;
}

int sb_qgemm(int fmt, int layout, const void* w, const void* w_s, const float* ts, int64_t n, int64_t k,
             const void* q, const float* s, int64_t m, void* y, void* workspace, size_t workspace_bytes,
             void* stream) {
  if (!w || !w_s || !q || !s || !y) return fail(SB_ERR_ARG, "qgemm: NULL pointer");
  if (fmt != SB_FMT_NVFP4 && fmt != SB_FMT_MXFP4 && fmt != SB_FMT_FP8) return fail(SB_ERR_FORMAT, "qgemm: format %d", fmt);
  if (fmt == SB_FMT_NVFP4 && !ts) return fail(SB_ERR_ARG, "qgemm: NVFP4 needs a tensor scale");
  if (n < 32 || n % 32 || k < 128 || k % 128 || m < 0 || m > (1 << 24))
    return fail(SB_ERR_SHAPE, "qgemm: need n %% 32 == 0, k %% 128 == 0 (n=%lld k=%lld m=%lld)", (long long)n,
                (long long)k, (long long)m);
  if (!aligned16(w)) return fail(SB_ERR_ARG, "qgemm: weights must be 16-byte aligned");
  if (m == 0) return SB_OK;
  sb::GroupedArgs a;
  memset(&a, 0, sizeof a);
  a.mode = sb::MODE_DENSE;
  a.m = (int)m;
  a.topk = 1;
  a.n_rows = (int)n;
  a.k = (int)k;
  a.has_shared = 1;
  a.shared.w = (const uint8_t*)w;
  a.shared.s = (const uint8_t*)w_s;
  a.shared.ts = ts;
  a.shared.ts_stride = 1;
  a.shared.fmt = fmt;
  a.routed = a.shared;
  a.bq = (const uint8_t*)q;
  a.bs = s;
  a.o = (__nv_bfloat16*)y;
  if (layout == SB_LAYOUT_TC) {
    if (n % 128) return fail(SB_ERR_SHAPE, "qgemm: the tensor-core layout needs n %% 128 == 0");
    int* err = nullptr;
    uint8_t* bpanel = nullptr;
    float* apanel = nullptr;
    const size_t panel = qgemm_ws(fmt, layout, k, m, (uint8_t*)workspace, &err, &bpanel, &apanel);
    int kstages = 0;
    const int ksplit = qgemm_ksplit(fmt, n, k, m, &kstages);
    const size_t need = panel + qgemm_part_bytes(fmt, n, k, m);
    if (!workspace || workspace_bytes < need)
      return fail(SB_ERR_WORKSPACE, "qgemm: workspace %zu bytes < %zu needed", workspace_bytes, need);
    if (!aligned16(q)) return fail(SB_ERR_ARG, "qgemm: activations must be 16-byte aligned");
    cudaStream_t st = (cudaStream_t)stream;
    int rc = SB_OK;
    const int pm = sb::tc_pass_max(fmt);
    sb::PanelArgs pa;
    memset(&pa, 0, sizeof pa);
    pa.mode = sb::MODE_DENSE;
    pa.m = (int)m;
    pa.topk = 1;
    pa.k = (int)k;
    pa.has_shared = 1;
    pa.n_sh_pass = (int)((m + pm - 1) / pm);
    pa.nv_shared = fmt == SB_FMT_NVFP4;
    pa.xq = (const uint8_t*)q;
    pa.xs = s;
    pa.bpanel = bpanel;
    pa.apanel = apanel;
    pa.zero_err = err;   // cleared by the panel kernel, which the grouped kernel waits for
    if (ksplit > 1) {
      // K pieces: partials after the panel, then the counters, zeroed by the panel kernel
      const int64_t blocks = (int64_t)pa.n_sh_pass * (n / 128);
      a.ksplit = ksplit;
      a.kstages = kstages;
      a.part = (float*)((uint8_t*)workspace + panel);
      a.kcnt = (int*)((uint8_t*)workspace + panel + align256((size_t)blocks * ksplit * 2048 * sizeof(float)));
      pa.kzero = a.kcnt;
      pa.nkzero = (int)blocks;
    }
    rc = cuda_check(sb::launch_tc_panel(pa, 1, st), "qgemm panel");
    if (rc) return rc;
    sb::TcPlan plan;
    plan.bpanel = bpanel;
    plan.apanel = apanel;
    plan.pass_off = nullptr;
    plan.pass_slot = nullptr;
    plan.pass_pb = nullptr;
    plan.n_sh_pass = pa.n_sh_pass;
    a.shared.s_stride = 0;
    a.routed = a.shared;
    a.err = err;
    a.wait_limit = g_wait_limit.load(std::memory_order_relaxed);
    a.items_per_expert = (int)(n / 128);
    return cuda_check(sb::launch_tc_grouped(a, plan, plan.n_sh_pass * a.items_per_expert * ksplit, st), "qgemm");
  }
  a.items_per_expert = (int)((n + 255) / 256);
  return cuda_check(sb::launch_grouped(a, a.items_per_expert, 0, (cudaStream_t)stream), "qgemm");
}

}  // extern "C"

// Scratch of sb_qgemm_static: one file-scope region per device, shared by every call on that device.
// Bytes [0, 4) are the error flag (must be 0 when the kernels start: each call clears it first);
// then the activation panel (B tiles, then their row scales), rewritten in full by every call.
static __device__ __align__(256) uint8_t g_qgemm_static_scratch[SB_QGEMM_STATIC_SCRATCH_BYTES];

namespace {

// Device address of the current device's static scratch. It is looked up on every call (a host-side
// table lookup once the module is loaded on the device), so a device reset or a new primary context
// never leaves a stale address behind. The first call on a device loads the module there: that
// first call comes before any stream capture.
int static_scratch(void** out) {
  void* p = nullptr;
  const int rc = cuda_check(cudaGetSymbolAddress(&p, g_qgemm_static_scratch), "qgemm_static: cudaGetSymbolAddress");
  if (rc) return rc;
  *out = p;
  return SB_OK;
}

}  // namespace

extern "C" {

int sb_qgemm_static(int fmt, const void* w, const void* w_s, const float* ts, int64_t n, int64_t k, const void* q,
                    const float* s, int64_t m, void* y, void* stream) {
  if (!w || !w_s || !q || !s || !y) return fail(SB_ERR_ARG, "qgemm_static: NULL pointer");
  if (fmt != SB_FMT_NVFP4 && fmt != SB_FMT_MXFP4 && fmt != SB_FMT_FP8)
    return fail(SB_ERR_FORMAT, "qgemm_static: format %d", fmt);
  if (fmt == SB_FMT_NVFP4 && !ts) return fail(SB_ERR_ARG, "qgemm_static: NVFP4 needs a tensor scale");
  if (n < 128 || n % 128 || k < 128 || k % 128 || m < 0 || m > (1 << 24))
    return fail(SB_ERR_SHAPE, "qgemm_static: need n %% 128 == 0, k %% 128 == 0 (n=%lld k=%lld m=%lld)",
                (long long)n, (long long)k, (long long)m);
  if (!aligned16(w) || !aligned16(q)) return fail(SB_ERR_ARG, "qgemm_static: weights and activations must be 16-byte aligned");
  const size_t need = qgemm_ws(fmt, SB_LAYOUT_TC, k, m, nullptr, nullptr, nullptr, nullptr);
  if (need > (size_t)SB_QGEMM_STATIC_SCRATCH_BYTES)
    return fail(SB_ERR_SHAPE,
                "qgemm_static: m=%lld k=%lld needs %zu bytes of scratch, more than the %zu-byte static region "
                "(use sb_qgemm with a workspace, or split m)",
                (long long)m, (long long)k, need, (size_t)SB_QGEMM_STATIC_SCRATCH_BYTES);
  if (m == 0) return SB_OK;
  void* base = nullptr;
  int rc = static_scratch(&base);
  if (rc) return rc;
  int* err = nullptr;
  uint8_t* bpanel = nullptr;
  float* apanel = nullptr;
  qgemm_ws(fmt, SB_LAYOUT_TC, k, m, (uint8_t*)base, &err, &bpanel, &apanel);
  cudaStream_t st = (cudaStream_t)stream;
  rc = cuda_check(cudaMemsetAsync(err, 0, sizeof(int), st), "qgemm_static");
  if (rc) return rc;
  const int pm = sb::tc_pass_max(fmt);
  sb::PanelArgs pa;
  memset(&pa, 0, sizeof pa);
  pa.mode = sb::MODE_DENSE;
  pa.m = (int)m;
  pa.topk = 1;
  pa.k = (int)k;
  pa.has_shared = 1;
  pa.n_sh_pass = (int)((m + pm - 1) / pm);
  pa.nv_shared = fmt == SB_FMT_NVFP4;
  pa.xq = (const uint8_t*)q;
  pa.xs = s;
  pa.bpanel = bpanel;
  pa.apanel = apanel;
  rc = cuda_check(sb::launch_tc_panel(pa, 1, st), "qgemm_static panel");
  if (rc) return rc;
  sb::TcPlan plan;
  plan.bpanel = bpanel;
  plan.apanel = apanel;
  plan.pass_off = nullptr;
  plan.pass_slot = nullptr;
  plan.pass_pb = nullptr;
  plan.n_sh_pass = pa.n_sh_pass;
  sb::GroupedArgs a;
  memset(&a, 0, sizeof a);
  a.mode = sb::MODE_DENSE;
  a.m = (int)m;
  a.topk = 1;
  a.n_rows = (int)n;
  a.k = (int)k;
  a.has_shared = 1;
  a.shared.w = (const uint8_t*)w;
  a.shared.s = (const uint8_t*)w_s;
  a.shared.ts = ts;
  a.shared.ts_stride = 1;
  a.shared.fmt = fmt;
  a.routed = a.shared;
  a.o = (__nv_bfloat16*)y;
  a.err = err;
  a.items_per_expert = (int)(n / 128);
  return cuda_check(sb::launch_tc_grouped(a, plan, plan.n_sh_pass * a.items_per_expert, st), "qgemm_static");
}

int sb_qgemm_static_error(int* host_out, void* stream) {
  if (!host_out) return fail(SB_ERR_ARG, "qgemm_static_error: NULL pointer");
  void* base = nullptr;
  int rc = static_scratch(&base);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  rc = cuda_check(cudaMemcpyAsync(host_out, base, sizeof(int), cudaMemcpyDeviceToHost, st), "qgemm_static_error");
  if (rc) return rc;
  return cuda_check(cudaStreamSynchronize(st), "qgemm_static_error");
}

size_t sb_moe_workspace_bytes(const sb_moe_layer* layer, int64_t m) {
  if (check_layer(layer) != SB_OK || m < 0) return 0;
  if (m < 1) m = 1;
  size_t need = carve(layer, m, nullptr).bytes;
  // A workspace sized for m serves every m' <= m. Between the batch sizes where the kernel choice
  // changes (the default's switch to the hybrid dispatch; the hybrid dispatch moving the shared
  // expert to the prefill kernel) every buffer grows with m, so the largest batch below each switch
  // covers the rest.
  if (layer->layout == SB_LAYOUT_TC) {
    const int64_t sw[2] = {(HYBRID_TOKENS_PER_EXPERT * layer->n_experts + layer->topk - 1) / layer->topk,
                           HYBRID_SHARED_PASSES * wide_pass(layer)};
    for (int64_t q : sw) {
      if (q - 1 >= 1 && q - 1 < m) {
        const size_t v = carve(layer, q - 1, nullptr).bytes;
        if (v > need) need = v;
      }
    }
  }
  return need;
}

static int route_impl(const sb_moe_layer* L, const void* x, int64_t m, const int64_t* ids, float* out_w,
                      int64_t* out_idx, const Workspace& w, bool quant, cudaStream_t st) {
  // prefill batches take the tensor-core gate (under a forced prefill kernel every batch does, so a
  // token's logits come from the same kernel whether it runs alone or in its batch)
  const bool tcg = tc_gate(L, m);
  if (tcg) {
    const int rc0 = cuda_check(cudaMemsetAsync(w.err + 1, 0, sizeof(int32_t), st), "gate flag");
    if (rc0) return rc0;
  }
  int rc = tcg
               ? cuda_check(sb::launch_gate_tc(x, L->gate_w, w.logits, (int)m, L->n_experts, L->hidden,
                                               sb::gate_ksplit(L->hidden), w.err + 1, st),
                            "gate_tc")
               : cuda_check(sb::launch_gate_logits(x, L->gate_w, w.logits, (int)m, L->n_experts, L->hidden, st),
                            "gate_logits");
  if (rc) return rc;
  sb::RouteArgs r;
  r.logits = w.logits;
  r.bias = L->gate_bias;
  r.tid2eid = L->tid2eid;
  r.input_ids = ids;
  r.m = (int)m;
  r.n_experts = L->n_experts;
  r.topk = L->topk;
  r.score_func = L->score_func;
  r.act_pow2 = L->act_pow2;
  r.hidden = L->hidden;
  r.route_scale = L->route_scale;
  r.logits_bf16 = L->logits_bf16;
  r.no_renorm = L->no_renorm;
  r.topk_idx = w.topk_idx;
  r.topk_w = w.topk_w;
  r.out_idx = out_idx;
  r.out_w = out_w;
  r.x = (const __nv_bfloat16*)x;
  r.xq = quant ? w.xq : nullptr;
  r.xs = w.xs;
  return cuda_check(sb::launch_route(r, st), "route");
}

int sb_moe_route(const sb_moe_layer* layer, const void* x, int64_t m, const int64_t* input_ids, float* out_weights,
                 int64_t* out_indices, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_layer(layer);
  if (rc) return rc;
  if (layer->mode == SB_MODE_K3) return fail(SB_ERR_UNSUPPORTED, "K3-mode layers have no router");
  if (!x) return fail(SB_ERR_ARG, "x is NULL");
  if (m < 0 || m > (1 << 20)) return fail(SB_ERR_SHAPE, "m=%lld outside 0..2^20", (long long)m);
  if (m == 0) return SB_OK;
  if (layer->tid2eid && !input_ids) return fail(SB_ERR_ARG, "hash routing needs input_ids");
  Workspace w = carve(layer, m, (uint8_t*)workspace);
  if (!workspace || workspace_bytes < w.bytes)
    return fail(SB_ERR_WORKSPACE, "workspace %zu bytes < %zu needed", workspace_bytes, w.bytes);
  return route_impl(layer, x, m, input_ids, out_weights, out_indices, w, false, (cudaStream_t)stream);
}

static int forward_impl(const sb_moe_layer* layer, const void* x, int64_t m, const int64_t* input_ids, void* y,
                        float* out_weights, int64_t* out_indices, void* workspace, size_t workspace_bytes,
                        void* stream, void* const* events, void* wire_q = nullptr, void* wire_s = nullptr,
                        const int64_t* ext_idx = nullptr, const float* ext_w = nullptr) {
  cudaStream_t st = (cudaStream_t)stream;
  auto mark = [&](int i) {
    if (events && events[i]) cudaEventRecord((cudaEvent_t)events[i], st);
  };
  int rc = check_layer(layer);
  if (rc) return rc;
  const sb_moe_layer* L = layer;
  if (!x || (!y && !wire_q)) return fail(SB_ERR_ARG, "x or y is NULL");
  if (!aligned16(x) || !aligned16(y) || !aligned16(wire_q)) return fail(SB_ERR_ARG, "x, y and q must be 16-byte aligned");
  if (wire_q && (!wire_s || layer->hidden > 8192))
    return fail(SB_ERR_SHAPE, "wire output needs a scale buffer and hidden <= 8192 (hidden=%d)", layer->hidden);
  if (m < 0 || m > (1 << 20)) return fail(SB_ERR_SHAPE, "m=%lld outside 0..2^20", (long long)m);
  if (m == 0) return SB_OK;
  if (L->tid2eid && !input_ids) return fail(SB_ERR_ARG, "hash routing needs input_ids");
  if ((int64_t)m * L->topk > (1 << 22)) return fail(SB_ERR_SHAPE, "m * topk too large");
  const bool k3 = L->mode == SB_MODE_K3;
  if (k3 != (ext_idx != nullptr))
    return fail(SB_ERR_UNSUPPORTED, k3 ? "K3-mode layers take the caller's routing (sb_moe_forward_routed)"
                                       : "the caller's routing is taken by K3-mode layers only");
  if (k3 && (!ext_w || wire_q)) return fail(SB_ERR_ARG, "K3 mode: routing weights needed, no wire output");
  Workspace w = carve(L, m, (uint8_t*)workspace);
  if (!workspace || workspace_bytes < w.bytes)
    return fail(SB_ERR_WORKSPACE, "workspace %zu bytes < %zu needed", workspace_bytes, w.bytes);
  mark(0);
  if (k3) {
    // the caller's routing; an id out of range raises the second flag word, folded in by the permutation
    rc = cuda_check(cudaMemsetAsync(w.err + 1, 0, sizeof(int32_t), st), "routing flag");
    if (rc) return rc;
    rc = cuda_check(sb::launch_routing_in(ext_idx, ext_w, (int)m, L->topk, L->n_experts, w.topk_idx, w.topk_w,
                                          w.err + 1, st),
                    "routing in");
  } else {
    rc = route_impl(L, x, m, input_ids, out_weights, out_indices, w, true, st);
  }
  if (rc) return rc;
  mark(1);
  sb::PermuteArgs p;
  memset(&p, 0, sizeof p);
  p.topk_idx = w.topk_idx;
  p.m = (int)m;
  p.topk = L->topk;
  p.n_experts = L->n_experts;
  p.counts = w.counts;
  p.offsets = w.offsets;
  p.active = w.active;
  p.n_active = w.n_active;
  p.pair_tok = w.pair_tok;
  p.pair_slot = w.pair_slot;
  p.err = w.err;
  p.gate_err = tc_gate(L, m) ? w.err + 1 : nullptr;   // the tensor-core gate's (or the routing input's) flag
  if (w.hybrid) {
    p.hot_min = sb::hybrid_hot_min(L->expert_fmt);
    p.pass_max2 = (int)wide_pass(L);
    p.pass_off2 = w.pass_off2;
    p.pass_slot2 = w.pass_slot2;
    p.pass_pb2 = w.pass_pb2;
  }
  p.pass_max = L->layout == SB_LAYOUT_TC ? (int)routed_pass_max(L, m) : 0;
  p.pass_off = L->layout == SB_LAYOUT_TC ? w.pass_off : nullptr;
  p.pass_slot = w.pass_slot;
  p.pass_pb = w.pass_pb;
  rc = cuda_check(sb::launch_permute(p, st), "permute");
  if (rc) return rc;
  mark(2);

  const int64_t H = L->hidden, I = L->inter, P = m * L->topk;
  const int64_t max_active = P < L->n_experts ? P : L->n_experts;
  sb::GroupedArgs g;
  memset(&g, 0, sizeof g);
  g.m = (int)m;
  g.topk = L->topk;
  g.has_shared = L->has_shared;
  g.act_pow2 = L->act_pow2;
  g.swiglu_limit = L->swiglu_limit;
  g.counts = w.counts;
  g.offsets = w.offsets;
  g.active = w.active;
  g.n_active = w.n_active;
  g.pair_tok = w.pair_tok;
  g.pair_slot = w.pair_slot;
  g.topk_w = w.topk_w;
  g.err = w.err;
  g.wait_limit = g_wait_limit.load(std::memory_order_relaxed);
  // the verify kernel's block-scaled items: MXFP4 with power-of-two activation scales, FP8 when its
  // block scales are powers of two as well
  g.bs_mask = L->act_pow2 ? ((1 << SB_FMT_MXFP4) | (L->fp8_pow2 ? (1 << SB_FMT_FP8) : 0)) : 0;
  g.activation = L->mode == SB_MODE_K3 ? sb::ACT_SITU : sb::ACT_SWIGLU;
  g.act_beta = L->situ_beta;
  g.act_lbeta = L->situ_linear_beta;
  g.weight_after = L->mode == SB_MODE_K3;
  const int n_units = (int)(max_active + (L->has_shared ? 1 : 0));
  if (L->layout == SB_LAYOUT_TC && w.wide) {
    // prefill kernel: x (act-quantised, bf16) in expert order, w13 (+ SwiGLU -> h), h act-quantised
    // as bf16, w2
    sb::TcPlan plan;
    memset(&plan, 0, sizeof plan);
    plan.pass_off = w.pass_off;
    plan.pass_slot = w.pass_slot;
    plan.pass_pb = w.pass_pb;
    plan.n_sh_pass = w.n_sh_pass;
    const int split = (int)wide_planes(L) - 1;
    const int rbf = L->expert_fmt == SB_FMT_MXFP4 ? 1 : 0;   // MXFP4 experts take bf16 operands
    rc = k3 ? cuda_check(sb::launch_wide_x_raw(x, w.pair_tok, w.offsets, L->n_experts, (int)P, (int)H, w.wide_rows,
                                                w.xw, w.cx, st),
                         "wide x (bf16)")
            : cuda_check(sb::launch_wide_x(w.xq, w.xs, w.pair_tok, w.offsets, L->n_experts, (int)m, (int)P, (int)H,
                                           w.wide_rows, (int)w.sb_row, split, rbf, 0, w.xw, w.cx, st),
                         "wide x");
    if (rc) return rc;
    g.mode = sb::MODE_W13;
    g.n_rows = (int)(2 * I);
    g.k = (int)H;
    g.routed = routed_set(L, true);
    g.shared = shared_set(L, true);
    g.hbf = w.hbf;
    g.n_experts = L->n_experts;
    g.items_per_expert = (int)(I / 64);
    const int64_t n_pass_max = max_passes(L, m);
    rc = cuda_check(sb::launch_tc_wide(g, plan, w.xw, w.cx, w.wide_rows, (int)w.sb_row, split,
                                       (int)(n_pass_max * g.items_per_expert), st),
                    "wide w13");
    if (rc) return rc;
    mark(3);
    rc = k3 ? cuda_check(sb::launch_wide_h_raw(w.hbf, w.wide_rows, w.wide_rows, (int)I, w.hw, w.ch, st), "wide h (bf16)")
            : cuda_check(sb::launch_wide_h(w.hbf, w.wide_rows, w.wide_rows, (int)w.sb_row, (int)I, L->act_pow2, rbf,
                                           w.offsets, L->n_experts, 0, 0, w.hw, w.ch, st),
                         "wide h");
    if (rc) return rc;
    g.mode = sb::MODE_W2;
    g.n_rows = (int)H;
    g.k = (int)I;
    g.routed = routed_set(L, false);
    g.shared = shared_set(L, false);
    g.o = w.o;
    g.items_per_expert = (int)(H / 128);
    rc = cuda_check(sb::launch_tc_wide(g, plan, w.hw, w.ch, w.wide_rows, (int)w.sb_row, split,
                                       (int)(n_pass_max * g.items_per_expert), st),
                    "wide w2");
    if (rc) return rc;
  } else if (L->layout == SB_LAYOUT_TC && w.hybrid) {
    // hybrid dispatch: cold experts (and a narrow shared expert) on the verify kernel, hot experts
    // (and a wide shared expert) on the prefill kernel; h of both in the prefill kernel's padded row
    // space, o of both in the combine's (token, slot) rows
    const bool shw = hybrid_shared_wide(L, m);
    const int hot = sb::hybrid_hot_min(L->expert_fmt);
    const int split = (int)wide_planes(L) - 1;
    const int rbf = L->expert_fmt == SB_FMT_MXFP4 ? 1 : 0;
    sb::TcPlan vplan;   // verify kernel: the first pass table (cold experts)
    vplan.bpanel = w.bpanel;
    vplan.apanel = w.apanel;
    vplan.pass_off = w.pass_off;
    vplan.pass_slot = w.pass_slot;
    vplan.pass_pb = w.pass_pb;
    vplan.n_sh_pass = w.n_sh_pass;
    sb::TcPlan wplan;   // prefill kernel: the second (hot experts)
    memset(&wplan, 0, sizeof wplan);
    wplan.pass_off = w.pass_off2;
    wplan.pass_slot = w.pass_slot2;
    wplan.pass_pb = w.pass_pb2;
    wplan.n_sh_pass = w.n_sh_pass2;
    rc = cuda_check(sb::launch_wide_x(w.xq, w.xs, w.pair_tok, w.offsets, L->n_experts, shw ? (int)m : 0, (int)P,
                                      (int)H, w.wide_rows, (int)w.sb_row, split, rbf, hot, w.xw, w.cx, st),
                    "hybrid wide x");
    if (rc) return rc;
    sb::PanelArgs pa;
    memset(&pa, 0, sizeof pa);
    pa.mode = sb::MODE_W13;
    pa.m = (int)m;
    pa.topk = L->topk;
    pa.k = (int)H;
    pa.act_pow2 = L->act_pow2;
    pa.has_shared = shw ? 0 : L->has_shared;
    pa.n_sh_pass = w.n_sh_pass;
    pa.nv_routed = L->expert_fmt == SB_FMT_NVFP4;
    pa.nv_shared = 0;
    pa.xq = w.xq;
    pa.xs = w.xs;
    pa.hbf = w.hbf;
    pa.counts = w.counts;
    pa.offsets = w.offsets;
    pa.active = w.active;
    pa.n_active = w.n_active;
    pa.pass_off = w.pass_off;
    pa.pair_tok = w.pair_tok;
    pa.bpanel = w.bpanel;
    pa.apanel = w.apanel;
    pa.hot_min = hot;
    pa.hpad = 1;
    pa.hsh0 = (int)w.sb_row;
    rc = cuda_check(sb::launch_tc_panel(pa, n_units, st), "hybrid w13 panel");
    if (rc) return rc;
    sb::GroupedArgs gv = g;   // the verify kernel's launches
    gv.has_shared = shw ? 0 : L->has_shared;
    gv.hpad = 1;
    gv.hsh0 = (int)w.sb_row;
    gv.mode = sb::MODE_W13;
    gv.n_rows = (int)(2 * I);
    gv.k = (int)H;
    gv.routed = routed_set(L, true);
    gv.shared = shared_set(L, true);
    gv.hbf = w.hbf;
    gv.n_experts = L->n_experts;
    gv.items_per_expert = (int)(I / 64);
    const int64_t v_pass_max = max_passes(L, m);
    rc = cuda_check(sb::launch_tc_grouped(gv, vplan, (int)(v_pass_max * gv.items_per_expert), st), "hybrid w13 verify");
    if (rc) return rc;
    sb::GroupedArgs gw = g;   // the prefill kernel's launches
    gw.has_shared = shw ? L->has_shared : 0;
    gw.mode = sb::MODE_W13;
    gw.n_rows = (int)(2 * I);
    gw.k = (int)H;
    gw.routed = routed_set(L, true);
    gw.shared = shared_set(L, true);
    gw.hbf = w.hbf;
    gw.n_experts = L->n_experts;
    gw.items_per_expert = (int)(I / 64);
    const int64_t w_pass_max = shared_passes_wide(L, m) + max_routed_passes_wide(L, m);
    rc = cuda_check(sb::launch_tc_wide(gw, wplan, w.xw, w.cx, w.wide_rows, (int)w.sb_row, split,
                                       (int)(w_pass_max * gw.items_per_expert), st),
                    "hybrid w13 prefill");
    if (rc) return rc;
    mark(3);
    pa.mode = sb::MODE_W2;
    pa.k = (int)I;
    rc = cuda_check(sb::launch_tc_panel(pa, n_units, st), "hybrid w2 panel");
    if (rc) return rc;
    rc = cuda_check(sb::launch_wide_h(w.hbf, w.wide_rows, w.wide_rows, (int)w.sb_row, (int)I, L->act_pow2, rbf,
                                      w.offsets, L->n_experts, hot, shw ? (int)m : 0, w.hw, w.ch, st),
                    "hybrid wide h");
    if (rc) return rc;
    gv.mode = sb::MODE_W2;
    gv.n_rows = (int)H;
    gv.k = (int)I;
    gv.routed = routed_set(L, false);
    gv.shared = shared_set(L, false);
    gv.o = w.o;
    gv.items_per_expert = (int)(H / 128);
    rc = cuda_check(sb::launch_tc_grouped(gv, vplan, (int)(v_pass_max * gv.items_per_expert), st), "hybrid w2 verify");
    if (rc) return rc;
    gw.mode = sb::MODE_W2;
    gw.n_rows = (int)H;
    gw.k = (int)I;
    gw.routed = routed_set(L, false);
    gw.shared = shared_set(L, false);
    gw.o = w.o;
    gw.items_per_expert = (int)(H / 128);
    rc = cuda_check(sb::launch_tc_wide(gw, wplan, w.hw, w.ch, w.wide_rows, (int)w.sb_row, split,
                                       (int)(w_pass_max * gw.items_per_expert), st),
                    "hybrid w2 prefill");
    if (rc) return rc;
  } else if (L->layout == SB_LAYOUT_TC) {
    // tensor-core path: w13 panel, w13 (+ SwiGLU -> h bf16), w2 panel (act_quant of h), w2
    sb::TcPlan plan;
    plan.bpanel = w.bpanel;
    plan.apanel = w.apanel;
    plan.pass_off = w.pass_off;
    plan.pass_slot = w.pass_slot;
    plan.pass_pb = w.pass_pb;
    plan.n_sh_pass = w.n_sh_pass;
    sb::PanelArgs pa;
    memset(&pa, 0, sizeof pa);
    pa.mode = sb::MODE_W13;
    pa.m = (int)m;
    pa.topk = L->topk;
    pa.k = (int)H;
    pa.act_pow2 = L->act_pow2;
    pa.has_shared = L->has_shared;
    pa.n_sh_pass = w.n_sh_pass;
    pa.nv_routed = L->expert_fmt == SB_FMT_NVFP4;
    pa.nv_shared = 0;
    pa.xq = w.xq;
    pa.xs = w.xs;
    pa.hbf = w.hbf;
    pa.counts = w.counts;
    pa.offsets = w.offsets;
    pa.active = w.active;
    pa.n_active = w.n_active;
    pa.pass_off = w.pass_off;
    pa.pair_tok = w.pair_tok;
    pa.bpanel = w.bpanel;
    pa.apanel = w.apanel;
    // FP8 expert banks take their items from a launch-wide counter (measured at c3: 3-5% faster
    // forwards); fp4 banks keep the round-robin schedule, which measured ~1% faster for them
    if (L->expert_fmt == SB_FMT_FP8) {
      pa.zero_sched = w.err + 2;
      g.sched = w.err + 2;
    }
    rc = cuda_check(sb::launch_tc_panel(pa, n_units, st), "tc w13 panel");
    if (rc) return rc;
    g.mode = sb::MODE_W13;
    g.n_rows = (int)(2 * I);
    g.k = (int)H;
    g.routed = routed_set(L, true);
    g.shared = shared_set(L, true);
    g.hbf = w.hbf;
    g.n_experts = L->n_experts;
    g.items_per_expert = (int)(I / 64);
    const int64_t n_pass_max = max_passes(L, m);
    rc = cuda_check(sb::launch_tc_grouped(g, plan, (int)(n_pass_max * g.items_per_expert), st), "tc w13");
    if (rc) return rc;
    mark(3);
    pa.mode = sb::MODE_W2;
    pa.k = (int)I;
    rc = cuda_check(sb::launch_tc_panel(pa, n_units, st), "tc w2 panel");
    if (rc) return rc;
    g.mode = sb::MODE_W2;
    g.n_rows = (int)H;
    g.k = (int)I;
    g.routed = routed_set(L, false);
    g.shared = shared_set(L, false);
    g.o = w.o;
    g.items_per_expert = (int)(H / 128);
    rc = cuda_check(sb::launch_tc_grouped(g, plan, (int)(n_pass_max * g.items_per_expert), st), "tc w2");
    if (rc) return rc;
  } else {
  // w13 (+ SwiGLU, + act_quant of h)
  g.mode = sb::MODE_W13;
  g.n_rows = (int)(2 * I);
  g.k = (int)H;
  g.routed = routed_set(L, true);
  g.shared = shared_set(L, true);
  g.bq = w.xq;
  g.bs = w.xs;
  g.hq = w.hq;
  g.hs = w.hs;
  g.items_per_expert = (int)(I / 128);
  rc = cuda_check(sb::launch_grouped(g, n_units * g.items_per_expert, 0, st), "grouped w13");
  if (rc) return rc;
  mark(3);
  // w2
  g.mode = sb::MODE_W2;
  g.n_rows = (int)H;
  g.k = (int)I;
  g.routed = routed_set(L, false);
  g.shared = shared_set(L, false);
  g.bq = w.hq;
  g.bs = w.hs;
  g.o = w.o;
  g.items_per_expert = (int)((H + 255) / 256);
  rc = cuda_check(sb::launch_grouped(g, n_units * g.items_per_expert, 0, st), "grouped w2");
  if (rc) return rc;
  }
  mark(4);
  if (k3)
    rc = cuda_check(sb::launch_combine_weighted(w.o, w.topk_w, (int)m, L->topk, (int)H, (__nv_bfloat16*)y, st),
                    "combine (weighted)");
  else if (wire_q)
    rc = cuda_check(sb::launch_combine_pack(w.o, w.topk_idx, (int)m, L->topk, (int)H, L->has_shared,
                                            (__nv_bfloat16*)y, (uint8_t*)wire_q, (__nv_bfloat16*)wire_s, st),
                    "combine+pack");
  else
    rc = cuda_check(sb::launch_combine(w.o, w.topk_idx, (int)m, L->topk, (int)H, L->has_shared,
                                       (__nv_bfloat16*)y, st),
                    "combine");
  if (rc) return rc;
  mark(5);
  return SB_OK;
}

int sb_moe_forward(const sb_moe_layer* layer, const void* x, int64_t m, const int64_t* input_ids, void* y,
                   float* out_weights, int64_t* out_indices, void* workspace, size_t workspace_bytes, void* stream) {
  return forward_impl(layer, x, m, input_ids, y, out_weights, out_indices, workspace, workspace_bytes, stream,
                      nullptr);
}

int sb_moe_forward_profiled(const sb_moe_layer* layer, const void* x, int64_t m, const int64_t* input_ids, void* y,
                            float* out_weights, int64_t* out_indices, void* workspace, size_t workspace_bytes,
                            void* stream, void* const* events) {
  return forward_impl(layer, x, m, input_ids, y, out_weights, out_indices, workspace, workspace_bytes, stream,
                      events);
}

int sb_moe_forward_routed(const sb_moe_layer* layer, const void* x, int64_t m, const int64_t* topk_idx,
                          const float* topk_w, void* y, void* workspace, size_t workspace_bytes, void* stream) {
  if (m > 0 && (!topk_idx || !topk_w)) return fail(SB_ERR_ARG, "topk_idx or topk_w is NULL");
  if (m == 0) {
    const int rc = check_layer(layer);
    return rc ? rc : SB_OK;
  }
  return forward_impl(layer, x, m, nullptr, y, nullptr, nullptr, workspace, workspace_bytes, stream, nullptr, nullptr,
                      nullptr, topk_idx, topk_w);
}

int sb_moe_forward_wire(const sb_moe_layer* layer, const void* x, int64_t m, const int64_t* input_ids, void* y,
                        void* q, void* scale, float* out_weights, int64_t* out_indices, void* workspace,
                        size_t workspace_bytes, void* stream) {
  if (!q) return fail(SB_ERR_ARG, "q is NULL");
  return forward_impl(layer, x, m, input_ids, y, out_weights, out_indices, workspace, workspace_bytes, stream, nullptr,
                      q, scale);
}

int sb_wire_pack(const void* x, int64_t rows, int64_t dim, void* q, void* scale, void* stream) {
  if (!x || !q || !scale) return fail(SB_ERR_ARG, "wire_pack: NULL pointer");
  if (rows < 0 || rows > (1 << 30) || dim <= 0 || dim % 8)
    return fail(SB_ERR_SHAPE, "wire_pack: need rows >= 0 and dim a positive multiple of 8 (rows=%lld dim=%lld)",
                (long long)rows, (long long)dim);
  if (!aligned16(x) || (reinterpret_cast<uintptr_t>(q) & 7u)) return fail(SB_ERR_ARG, "wire_pack: x 16-byte, q 8-byte aligned");
  if (rows == 0) return SB_OK;
  return cuda_check(sb::launch_wire_pack(x, rows, dim, (uint8_t*)q, scale, (cudaStream_t)stream), "wire_pack");
}

int sb_wire_unpack(const void* q, const void* scale, int64_t rows, int64_t dim, void* y, void* stream) {
  if (!q || !scale || !y) return fail(SB_ERR_ARG, "wire_unpack: NULL pointer");
  if (rows < 0 || rows > (1 << 30) || dim <= 0 || dim % 8)
    return fail(SB_ERR_SHAPE, "wire_unpack: need rows >= 0 and dim a positive multiple of 8 (rows=%lld dim=%lld)",
                (long long)rows, (long long)dim);
  if (!aligned16(y) || (reinterpret_cast<uintptr_t>(q) & 7u)) return fail(SB_ERR_ARG, "wire_unpack: y 16-byte, q 8-byte aligned");
  if (rows == 0) return SB_OK;
  return cuda_check(sb::launch_wire_unpack((const uint8_t*)q, scale, rows, dim, y, (cudaStream_t)stream), "wire_unpack");
}

int sb_residual_rmsnorm(void* x, const void* y, int64_t rows, int64_t dim, const float* weight, float eps, void* out,
                        void* stream) {
  if (!x) return fail(SB_ERR_ARG, "residual_rmsnorm: x is NULL");
  if (rows < 0 || rows > (1 << 30) || dim <= 0 || dim % 8)
    return fail(SB_ERR_SHAPE, "residual_rmsnorm: need rows >= 0 and dim a positive multiple of 8 (rows=%lld dim=%lld)",
                (long long)rows, (long long)dim);
  if (!aligned16(x) || !aligned16(y) || !aligned16(out)) return fail(SB_ERR_ARG, "residual_rmsnorm: 16-byte alignment");
  if (!(eps >= 0.f)) return fail(SB_ERR_ARG, "residual_rmsnorm: eps must be >= 0");
  if (rows == 0) return SB_OK;
  return cuda_check(sb::launch_residual_rmsnorm(x, y, rows, dim, weight, eps, out, (cudaStream_t)stream),
                    "residual_rmsnorm");
}

int sb_debug_set_wait_limit(int64_t polls) {
  if (polls < 0 || polls > (int64_t)UINT32_MAX) return fail(SB_ERR_ARG, "debug_set_wait_limit: %lld", (long long)polls);
  g_wait_limit.store((uint32_t)polls, std::memory_order_relaxed);
  return SB_OK;
}

int sb_selftest_formats(float* out, void* stream) {
  if (!out) return fail(SB_ERR_ARG, "selftest: NULL pointer");
  return cuda_check(sb::launch_selftest(out, (cudaStream_t)stream), "selftest");
}

}  // extern "C"
