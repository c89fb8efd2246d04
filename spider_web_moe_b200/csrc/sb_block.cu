// Whole-block driver and the small exported entry points.
//
// sb_block_forward runs SpiderMoELayer.forward (spider_moe/model.py:240-317)
// for a range of loops as a fixed sequence of kernels on one stream, with all
// scratch carved from the caller's workspace.  No step needs the host to read
// device data, so the whole sequence can be captured in a CUDA graph.
//
// Per loop:
//   1  sb_router            top-k over experts                       (model.py:254-258)
//   2  sb_group (sources)   rows grouped by selected source expert
//   3  sb_gather_rows       h rows in source order
//   4  grouped GEMM         edge logits of the selected sources      (model.py:261-263)
//   5  sb_edge_topm         top-M destinations + softmax             (model.py:264-266)
//   6  sb_group (dest.)     (token, destination) pairs, coefficients summed
//   7  sb_gather_rows       h rows in destination order
//   8  grouped GEMM         c * W_edge[d] h                          (model.py:271-288)
//   9  sb_group (experts)   dispatch plan                            (dispatch.py:56-115)
//  10  sb_combine_rows      messages, scattered into expert order
//  11  grouped GEMM         up projection + GELU / SwiGLU            (sparse_experts.py:60-61)
//  12  grouped GEMM         down projection * routing weight         (sparse_experts.py:62-63)
//  13  sb_combine_ln        delta + LayerNorm epilogue               (model.py:317)
#include <atomic>
#include <cstring>
#include <mutex>
#include <vector>

#include "sb_common.cuh"
#include "sb_internal.h"

namespace sb {

int current_sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = v > 0 ? v : 148;
  }
  return cached[dev];
}

int current_cc_major() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (!cached[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrComputeCapabilityMajor, dev);
    cached[dev] = v;
  }
  return cached[dev];
}

static std::atomic<unsigned long long> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

bool pdl_enabled() {
  static int cached = -1;
  if (cached < 0) {
    const char* v = getenv("SPIDER_B200_PDL");
    cached = (v && v[0] == '0') ? 0 : 1;
  }
  return cached == 1;
}

static int act_size(int dt) { return dt == SB_F32 ? 4 : 2; }

__global__ void remap_local_kernel(const int32_t* __restrict__ idx, int n, int E, int rank, int world,
                                   int32_t* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int e = idx[i];
    out[i] = (e >= 0 && e < E && e % world == rank) ? e / world : -1;
  }
}

// ------------------------------------------------------------------ stage timing
// Optional per-stage CUDA-event timing of sb_block_forward (a profiling aid;
// off by default, never used during graph capture).
constexpr int kNumStages = 14;
static const char* kStageNames[kNumStages] = {
    "router", "group_sources", "gather_sources", "gemm_edge_logits", "edge_topm", "group_destinations",
    "gather_destinations", "gemm_edge_values", "group_experts", "combine_messages", "gemm_expert_up",
    "gemm_expert_down", "combine_layernorm", "dequant_experts"};
struct StageTiming {
  bool on = false;
  std::vector<std::pair<int, std::pair<cudaEvent_t, cudaEvent_t>>> marks;
  std::mutex mu;
};
static StageTiming g_timing;

struct StageScope {
  int stage;
  cudaStream_t st;
  cudaEvent_t a = nullptr, b = nullptr;
  StageScope(int s, cudaStream_t stream) : stage(s), st(stream) {
    if (!g_timing.on) return;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    cudaEventRecord(a, st);
  }
  ~StageScope() {
    if (!a) return;
    cudaEventRecord(b, st);
    std::lock_guard<std::mutex> lk(g_timing.mu);
    g_timing.marks.push_back({stage, {a, b}});
  }
};

// Packed expert-parallel rows -> contiguous local ids (out of range -> -1) and weights.
__global__ void unpack_meta_kernel(const uint8_t* __restrict__ rows, int64_t pitch, int64_t meta_off, int n, int K,
                                   int G, int32_t* __restrict__ ids, float* __restrict__ w) {
  pdl_wait();
  pdl_trigger();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n * K; i += gridDim.x * blockDim.x) {
    const int r = i / K, k = i - r * K;
    const uint8_t* m = rows + static_cast<int64_t>(r) * pitch + meta_off;
    const int e = reinterpret_cast<const int32_t*>(m)[k];
    ids[i] = (e >= 0 && e < G) ? e : -1;
    w[i] = reinterpret_cast<const float*>(m + static_cast<int64_t>(K) * 4)[k];
  }
}

// ------------------------------------------------------------------ workspace layout

struct BlockBuffers {
  int* status;
  int32_t *top_idx; float* top_w;
  int32_t *src_off, *src_row, *src_slot, *src_inv; float* src_w;
  void* x_src; float* elog;
  int32_t* edge_idx; float* edge_w;
  int32_t *dst_off, *dst_row, *dst_slot, *dst_inv; float* dst_w;
  void* x_dst; float* y_msg;
  float* msg_f32;
  void* msg_act;
  int32_t *ffn_off, *ffn_row, *ffn_slot, *ffn_inv; float* ffn_w;
  int32_t *dst_rank, *ffn_rank; float *dst_wsc, *ffn_wsc;  // scratch of the two-plan grouping launch
  int32_t *cc_dst, *cc_ffn;                                  // its chunk counts (multi-CTA schedule)
  void* x_ffn; void* act; float* y_ffn;
  void *w_up_bf, *w_down_bf;  // bf16 copies of fp8 / int4 expert weights (prefill batches), or NULL
  void* hbuf[2];
  void* group_ws; size_t group_ws_bytes;
  int64_t cap_dst, y_msg_stride, y_ffn_stride;
};

static int max_splits_for(int n_tokens) { return n_tokens <= 512 ? 4 : 1; }

// Prefill-size batches of fp8 / int4 experts convert the expert weights to
// bf16 once per sb_block_forward call, into the workspace, and run the
// expert GEMMs on the bf16 tensor-core schedules (the CTA-pair kernel)
// instead of dequantising every weight tile in shared memory inside each
// loop's GEMM -- with many rows per expert the GEMMs are tensor-bound and the
// in-GEMM conversion is what limits them.  The conversion is the one the
// GEMM does in shared memory (fp8 e4m3 -> bf16 exactly, the per-row scale
// still applied to the accumulator; int4 -> bf16(q * group scale)), so the
// results are the same.  From this many expected rows per expert:
constexpr int kDequantOnceMinRows = 128;
// SPIDER_B200_DEQUANT_ONCE=0 keeps fp8 / int4 prefill on the in-GEMM dequant (for comparisons).
static bool dequant_once_enabled() {
  static const bool v = [] {
    const char* e = std::getenv("SPIDER_B200_DEQUANT_ONCE");
    return !(e && e[0] == '0');
  }();
  return v;
}

static bool dequant_once_possible(const sb_block_dims& d, int n_tokens) {
  return (d.wfmt == SB_W_FP8 || d.wfmt == SB_W_INT4) && d.engine != SB_ENGINE_SIMT && d.act_dtype == SB_BF16 &&
         static_cast<int64_t>(n_tokens) * d.top_k >= static_cast<int64_t>(kDequantOnceMinRows) * d.num_experts &&
         dequant_once_enabled();
}

// Columns of the dense routing logits (router + every source's edge logits),
// or 0 for expert counts whose E*E logits are too wide to compute densely.
constexpr int kDenseRouteMaxE = 32;
static int64_t dense_route_cols(const sb_block_dims& d) {
  const int64_t E = d.num_experts;
  return E <= kDenseRouteMaxE ? E + E * E : 0;
}

static size_t carve_block(const sb_block_dims& d, int n_cap, void* base, size_t size, BlockBuffers* b) {
  Carver c(base, size);
  const int64_t N = n_cap, H = d.hidden, E = d.num_experts, K = d.top_k, M = d.edges_per_expert, U = d.ffn;
  const int as = act_size(d.act_dtype);
  const int64_t cap_dst = N * (E < K * M ? E : K * M);
  const int64_t small = N < 512 ? N : 512;
  const int64_t small_dst = small * (E < K * M ? E : K * M);
  const int64_t msg_rows = cap_dst > 4 * small_dst ? cap_dst : 4 * small_dst;
  const int64_t ffn_rows = N * K > 4 * small * K ? N * K : 4 * small * K;
  b->status = c.take<int>(kStatusBytes / sizeof(int));
  b->top_idx = c.take<int32_t>(N * K);
  b->top_w = c.take<float>(N * K);
  b->src_off = c.take<int32_t>(E + 1);
  b->src_row = c.take<int32_t>(N * K);
  b->src_slot = c.take<int32_t>(N * K);
  b->src_w = c.take<float>(N * K);
  b->src_inv = c.take<int32_t>(N * K);
  b->x_src = c.take<char>(N * K * H * as);
  b->elog = c.take<float>(N * (dense_route_cols(d) > K * E ? dense_route_cols(d) : K * E));
  b->edge_idx = c.take<int32_t>(N * K * M);
  b->edge_w = c.take<float>(N * K * M);
  b->dst_off = c.take<int32_t>(E + 1);
  b->dst_row = c.take<int32_t>(cap_dst);
  b->dst_slot = c.take<int32_t>(cap_dst);
  b->dst_w = c.take<float>(cap_dst);
  b->dst_inv = c.take<int32_t>(N * K * M);
  b->x_dst = c.take<char>(cap_dst * H * as);
  b->y_msg = c.take<float>(msg_rows * H);
  b->msg_f32 = c.take<float>(N * H);
  b->msg_act = c.take<char>(N * H * as);
  b->ffn_off = c.take<int32_t>(E + 1);
  b->ffn_row = c.take<int32_t>(N * K);
  b->ffn_slot = c.take<int32_t>(N * K);
  b->ffn_w = c.take<float>(N * K);
  b->ffn_inv = c.take<int32_t>(N * K);
  b->x_ffn = c.take<char>(N * K * H * as);
  b->act = c.take<char>(N * K * U * as);
  b->y_ffn = c.take<float>(ffn_rows * H);
  b->w_up_bf = b->w_down_bf = nullptr;
  if (dequant_once_possible(d, static_cast<int>(N))) {
    const int64_t up_rows = (d.activation == SB_ACT_SWIGLU ? 2 : 1) * U;
    b->w_up_bf = c.take<__nv_bfloat16>(E * up_rows * H);
    b->w_down_bf = c.take<__nv_bfloat16>(E * H * U);
  }
  b->hbuf[0] = c.take<char>(N * H * as);
  b->hbuf[1] = c.take<char>(N * H * as);
  b->dst_rank = c.take<int32_t>(N * K * M);
  b->dst_wsc = c.take<float>(N * K * M);
  b->ffn_rank = c.take<int32_t>(N * K);
  b->ffn_wsc = c.take<float>(N * K);
  b->cc_dst = c.take<int32_t>((N * K * M + kGroupChunk - 1) / kGroupChunk * E);
  b->cc_ffn = c.take<int32_t>((N * K + kGroupChunk - 1) / kGroupChunk * E);
  b->group_ws_bytes = sb_group_workspace_bytes(static_cast<int>(N), static_cast<int>(K * M), static_cast<int>(E));
  b->group_ws = c.take<char>(b->group_ws_bytes);
  b->cap_dst = cap_dst;
  return c.overflow ? static_cast<size_t>(-1) : align_up(c.used, 256);
}

static int check_dims(const sb_block_dims* d) {
  if (!d || d->hidden <= 0 || d->hidden % 8 || d->num_experts <= 0 || d->num_experts > 256 || d->top_k <= 0 ||
      d->edges_per_expert <= 0 || d->top_k * d->edges_per_expert > 64 || d->ffn <= 0 || d->ffn % 8 || d->num_loops <= 0 ||
      d->max_tokens < 0 || (d->act_dtype != SB_F32 && d->act_dtype != SB_BF16) ||
      d->wfmt < SB_W_F32 || d->wfmt > SB_W_INT4 || (d->activation != SB_ACT_GELU && d->activation != SB_ACT_SWIGLU))
    return SB_ERR_ARG;
  if (d->top_k > 32 || d->edges_per_expert > 32) return SB_ERR_UNSUPPORTED;
  if (d->wfmt == SB_W_INT4 && (d->group_size <= 0 || d->hidden % d->group_size || d->ffn % d->group_size))
    return SB_ERR_ARG;
  if (d->wfmt == SB_W_F32 && d->act_dtype != SB_F32) return SB_ERR_ARG;
  return SB_OK;
}

static int run_gemm(sb_grouped_gemm_args& a, int engine_pref, cudaStream_t st) {
  if (engine_pref == SB_ENGINE_SIMT) return gemm_simt(a, st);
  const bool tc_ok = tcgen05_supported(a);
  if (engine_pref == SB_ENGINE_TCGEN05) return tc_ok ? gemm_tcgen05(a, st) : SB_ERR_UNSUPPORTED;
  return tc_ok ? gemm_tcgen05(a, st) : gemm_simt(a, st);
}

// Whether a GEMM reads its token rows straight from the unpermuted matrix
// (gather inside the GEMM) instead of from a permuted copy.  The CUDA-core
// engine always can; the tcgen05 engine for column tiles up to 64.
static bool gemm_gathers(const sb_grouped_gemm_args& a, int engine) {
  if (engine == SB_ENGINE_SIMT) return true;
  const bool tc = tcgen05_supported(a);
  if (!tc) return engine == SB_ENGINE_AUTO;  // AUTO falls back to the CUDA-core engine
  // The quantised decode kernel loads up to 128 rows per item: one tiled box
  // from a permuted copy beats 32 four-row gathers per K step.
  if (tc_qdec(a)) return false;
  return tc_tile_n(a) <= 64;
}

// K-split factor for a LINEAR GEMM: spread small grids over the SMs.
static int pick_splits(int m_rows, int k, int rows_hint, int groups, int max_splits, bool tc, int bound) {
  const int m_tiles = (m_rows + 127) / 128;
  const int per_group = (rows_hint + groups - 1) / (groups > 0 ? groups : 1);
  const bool fixed = bound > 0 && bound <= 64;
  const int bn = fixed ? 64 : per_group <= 16 ? 16 : per_group <= 32 ? 32 : per_group <= 64 ? 64 : per_group <= 128 ? 128 : 256;
  int tiles = fixed ? m_tiles * (groups < rows_hint ? groups : rows_hint)
                    : m_tiles * (rows_hint / bn + (groups < rows_hint ? groups : rows_hint));
  if (tiles < 1) tiles = 1;
  // Small column tiles run two CTAs per SM: aim for about two CTAs per SM.
  const int target = (bn <= 64 ? 2 : 1) * current_sm_count();
  int s = 1;
  while (s * 2 <= max_splits && tiles * s * 2 <= target && (k % ((tc ? 64 : 32) * s * 2)) == 0) s *= 2;
  return s;
}

// The up projection of a SwiGLU block reads the gate and up rows interleaved
// in one tensor (SB_EPI_SWIGLU_IL: 2 * ffn rows per expert); the w_gate
// fields of the block weights are not used.
static void fill_expert_gemm(sb_grouped_gemm_args& a, const sb_block_dims& d, bool up, const void* w,
                             const void* sc, const float* bias, const void*, const void*, const float*) {
  std::memset(&a, 0, sizeof(a));
  a.engine = d.engine;
  a.wfmt = d.wfmt;
  a.act_dtype = d.act_dtype;
  a.m_rows = up ? (d.activation == SB_ACT_SWIGLU ? 2 * d.ffn : d.ffn) : d.hidden;
  a.k = up ? d.hidden : d.ffn;
  a.group_size = d.group_size;
  a.lda = a.k;
  a.a_group_rows = a.m_rows;
  a.a_rows_total = static_cast<int64_t>(d.num_experts) * a.m_rows;
  a.a = w;
  a.a_scale = sc;
  a.bias = bias;
  a.bias_group_stride = a.m_rows;
}

// Restrict an expert GEMM to the experts e = rank + world * g of one rank.
static void shard_expert_gemm(sb_grouped_gemm_args& a, const sb_block_dims& d, int rank, int world) {
  if (world <= 1) return;
  const int64_t shift_rows = static_cast<int64_t>(rank) * a.m_rows;
  auto shift = [&](const void* p, int64_t elems_per_row_bytes) -> const void* {
    return p ? static_cast<const char*>(p) + shift_rows * elems_per_row_bytes : nullptr;
  };
  int64_t row_bytes = d.wfmt == SB_W_F32 ? a.lda * 4 : d.wfmt == SB_W_BF16 ? a.lda * 2 : d.wfmt == SB_W_FP8 ? a.lda : a.lda / 2;
  a.a = shift(a.a, row_bytes);
  a.a_gate = shift(a.a_gate, row_bytes);
  if (d.wfmt == SB_W_FP8) {
    a.a_scale = shift(a.a_scale, 4);
    a.a_gate_scale = shift(a.a_gate_scale, 4);
  } else if (d.wfmt == SB_W_INT4) {
    a.a_scale = shift(a.a_scale, (a.lda / d.group_size) * 2);
    a.a_gate_scale = shift(a.a_gate_scale, (a.lda / d.group_size) * 2);
  }
  a.bias = a.bias ? a.bias + shift_rows : nullptr;
  a.bias_gate = a.bias_gate ? a.bias_gate + shift_rows : nullptr;
  a.a_group_rows = static_cast<int64_t>(world) * a.m_rows;
  a.bias_group_stride = a.a_group_rows;
  a.a_rows_total -= shift_rows;
}

}  // namespace sb

using namespace sb;

extern "C" SB_API int sb_capabilities(void) {
  int caps = 1;  // compiled for sm_100a
  if (current_cc_major() == 10) caps |= 2;
  return caps;
}

extern "C" SB_API const char* sb_version(void) { return "spider_b200 0.1 (sm_100a)"; }

extern "C" SB_API const char* sb_error_string(int code) {
  switch (code) {
    case SB_OK: return "ok";
    case SB_ERR_ARG: return "bad argument";
    case SB_ERR_INDEX: return "index out of range";
    case SB_ERR_UNSUPPORTED: return "unsupported shape or format";
    case SB_ERR_NO_DEVICE: return "no sm_100 device";
    case SB_ERR_WORKSPACE: return "workspace missing or too small";
    case SB_ERR_DEVICE_STATUS: return "a kernel recorded a device-side status";
    default:
      if (code >= SB_ERR_CUDA_BASE) return cudaGetErrorString(static_cast<cudaError_t>(code - SB_ERR_CUDA_BASE));
      return "unknown error";
  }
}

extern "C" SB_API size_t sb_status_offset(void) { return 0; }

extern "C" SB_API int sb_grouped_gemm(const sb_grouped_gemm_args* args, void* stream) {
  if (!args) return SB_ERR_ARG;
  const sb_grouped_gemm_args& a = *args;
  if (!a.a || !a.x || !a.out || (!a.offsets && a.num_groups != 1) || a.num_groups <= 0 || a.m_rows <= 0 ||
      a.k <= 0 || a.lda < a.k ||
      a.ldx < a.k || a.max_rows < 0 || a.splits <= 0 || a.a_rows_total <= 0 ||
      (a.epilogue != SB_EPI_LINEAR && a.splits != 1) || (a.epilogue == SB_EPI_SWIGLU && !a.a_gate) ||
      (a.wfmt != SB_W_BF16 && a.wfmt != SB_W_F32 && !a.a_scale) || a.epilogue < 0 || a.epilogue > 3)
    return SB_ERR_ARG;
  if (a.max_rows == 0) return SB_OK;
  sb_grouped_gemm_args c = a;
  return run_gemm(c, a.engine, static_cast<cudaStream_t>(stream));
}

extern "C" SB_API size_t sb_block_workspace_bytes(const sb_block_dims* dims) {
  if (check_dims(dims) != SB_OK) return 0;
  BlockBuffers b;
  return carve_block(*dims, dims->max_tokens > 0 ? dims->max_tokens : 1, nullptr, ~size_t(0) >> 1, &b);
}

// Batches from this many tokens compute the router logits with the grouped
// GEMM (tensor cores) instead of the CUDA-core router kernel.
constexpr int kRouterGemmMinTokens = 128;

// The fused router + edge-generator kernel re-reads a selected source's E
// generator rows for every token: it is used while those reads (N*K*E*H
// elements) stay within this many bytes, a few microseconds of L2 traffic
// (SPIDER_B200_FUSED_ROUTE_BYTES overrides; 0 disables the fused kernel).
static double fused_route_max_bytes() {
  static const double v = [] {
    const char* e = std::getenv("SPIDER_B200_FUSED_ROUTE_BYTES");
    return e ? std::atof(e) : 32.0 * 1024 * 1024;
  }();
  return v;
}

// Steps 1-8 of one loop: routing, edge graph and the edge-value GEMM.  Leaves
// the routing in b.top_idx / b.top_w and the message partials in b.y_msg.
// With `ffn_planned` non-null the expert dispatch plan (step 9) is built in
// the same launch as the destination plan when both fit one CTA each, and
// *ffn_planned says whether that happened.
static bool fuse_ln_route_enabled() {
  static const bool v = [] {
    const char* e = std::getenv("SPIDER_B200_FUSE_LN_ROUTE");
    return !(e && e[0] == '0');
  }();
  return v;
}

// Whether a batch of N tokens takes the fused per-token route kernel.
static bool use_fused_route(const sb_block_dims& d, int N) {
  const double gen_bytes = static_cast<double>(N) * d.top_k * d.num_experts * d.hidden * act_size(d.act_dtype);
  return gen_bytes <= fused_route_max_bytes() &&
         route_edges_smem(d.act_dtype, d.hidden, d.num_experts, d.top_k) <= kRouteEdgesMaxSmem;
}

// Whether a batch of N tokens computes all router and edge logits with one
// dense GEMM over the packed routing rows (then one selection kernel) instead
// of the router, the source grouping and gather, the edge-logit GEMM over the
// selected sources and the top-M kernel.  The dense product computes E / K
// times the edge-logit FLOPs the selected sources need, so it is taken while
// those FLOPs stay small next to the loop (here: at most 8 GFLOP, a few
// microseconds of tensor time) and the batch is large enough for a GEMM.
constexpr double kDenseRouteMaxFlops = 8e9;
static bool use_dense_route(const sb_block_dims& d, const sb_block_weights* w, int N) {
  const int64_t cols = dense_route_cols(d);
  if (!w->route_w || !cols || d.engine == SB_ENGINE_SIMT || N < kRouterGemmMinTokens) return false;
  if (w->router_w != w->route_w ||
      static_cast<const char*>(w->gen_w) !=
          static_cast<const char*>(w->route_w) + static_cast<int64_t>(d.num_experts) * d.hidden * act_size(d.act_dtype))
    return false;
  return 2.0 * N * cols * d.hidden <= kDenseRouteMaxFlops;
}

// SPIDER_B200_MULTI_PLAN=0 keeps large batches on separate sb_group launches
// for the two plans and a separate row gather (for comparisons).
static bool multi_plan_enabled() {
  static const bool v = [] {
    const char* e = std::getenv("SPIDER_B200_MULTI_PLAN");
    return !(e && e[0] == '0');
  }();
  return v;
}

// `routed`: the fused route of this loop already ran (inside the previous
// loop's LayerNorm kernel); steps 1-5 are skipped.
static int route_loop(const sb_block_dims& d, const sb_block_weights* w, BlockBuffers& b, const void* cur, int N,
                      int l, int* msg_splits_out, bool* ffn_planned, bool routed, cudaStream_t st) {
  int rc = SB_OK;
  const int H = d.hidden, E = d.num_experts, K = d.top_k, M = d.edges_per_expert;
  const int KM = K * M;
  const int dense_fmt = d.act_dtype == SB_F32 ? SB_W_F32 : SB_W_BF16;
  const int64_t cap_dst = static_cast<int64_t>(N) * (E < KM ? E : KM);
  const bool tc_pref = d.engine != SB_ENGINE_SIMT;
#define SB_TRY(x) do { rc = (x); if (rc) return rc; } while (0)
  const bool fused = use_fused_route(d, N);
  if (fused && routed) {
    // router, edge logits and top-M already in b.top_* / b.edge_*
  } else if (fused) {
    // 1-5 in one kernel: router, edge logits of the selected sources, top-M
    StageScope sc_(0, st);
    SB_TRY(route_edges(cur, d.act_dtype, N, H, w->router_w, w->loop_bias + static_cast<int64_t>(l) * E, E, K, w->gen_w,
                       w->gen_bias + static_cast<int64_t>(l) * E * E, M, b.top_idx, b.top_w, b.edge_idx, b.edge_w,
                       st));
  } else if (use_dense_route(d, w, N)) {
    // 1-5 as one GEMM of every router and edge logit ([N, E + E*E], biases
    // added by the selection) and one selection kernel
    StageScope sc_(0, st);
    const int64_t cols = dense_route_cols(d);
    sb_grouped_gemm_args a;
    std::memset(&a, 0, sizeof(a));
    a.engine = d.engine; a.wfmt = dense_fmt; a.act_dtype = d.act_dtype; a.epilogue = SB_EPI_LINEAR;
    a.num_groups = 1; a.m_rows = static_cast<int>(cols); a.k = H; a.a_group_rows = cols; a.lda = H;
    a.a_rows_total = cols; a.a = w->route_w; a.bias = nullptr; a.bias_group_stride = cols;
    a.x = cur; a.ldx = H; a.max_rows = N; a.rows_hint = N; a.offsets = nullptr;
    a.out = b.elog; a.ldo = cols; a.splits = 1; a.split_stride = 0; a.status = b.status;
    SB_TRY(run_gemm(a, d.engine, st));
    SB_TRY(select_dense(b.elog, cols, N, E, K, M, w->loop_bias + static_cast<int64_t>(l) * E,
                        w->gen_bias + static_cast<int64_t>(l) * E * E, b.top_idx, b.top_w, b.edge_idx, b.edge_w, st));
  } else {
    // 1. router: large batches as a one-group GEMM (logits into the edge-logit
    // buffer, free until step 4) and a top-K kernel; small ones in one kernel
    if (N >= kRouterGemmMinTokens && d.engine != SB_ENGINE_SIMT) {
      StageScope sc_(0, st);
      sb_grouped_gemm_args a;
      std::memset(&a, 0, sizeof(a));
      a.engine = d.engine; a.wfmt = dense_fmt; a.act_dtype = d.act_dtype; a.epilogue = SB_EPI_LINEAR;
      a.num_groups = 1; a.m_rows = E; a.k = H; a.a_group_rows = E; a.lda = H; a.a_rows_total = E;
      a.a = w->router_w; a.bias = w->loop_bias + static_cast<int64_t>(l) * E; a.bias_group_stride = E;
      a.x = cur; a.ldx = H; a.max_rows = N; a.rows_hint = N; a.offsets = nullptr;
      // K-split to spread small batches over the SMs; the partials must fit
      // the edge-logit buffer (N*K*E floats)
      int rs = pick_splits(E, H, N, 1, max_splits_for(N), tc_pref, 0);
      while (rs > 1 && rs > K) rs >>= 1;
      a.out = b.elog; a.ldo = E; a.splits = rs; a.split_stride = static_cast<int64_t>(N) * E; a.status = b.status;
      SB_TRY(run_gemm(a, d.engine, st));
      SB_TRY(router_from_logits(b.elog, E, rs, static_cast<int64_t>(N) * E, N, E, K, b.top_idx, b.top_w, st));
    } else {
      StageScope sc_(0, st);
      SB_TRY(sb_router(cur, d.act_dtype, N, H, w->router_w, w->loop_bias + static_cast<int64_t>(l) * E, E, K, b.top_idx,
                       b.top_w, nullptr, st));
    }
    // 2-3. rows grouped by selected source; gather h (inside the GEMM when it can)
    { StageScope sc_(1, st); SB_TRY(sb_group(b.top_idx, nullptr, N, K, E, 0, b.src_off, b.src_row, b.src_slot, b.src_w,
                                           b.src_inv, b.group_ws, b.group_ws_bytes, st)); }
    // 4. edge logits of the selected sources: rows [s*E, s*E+E) of the generator
    {
      sb_grouped_gemm_args a;
      std::memset(&a, 0, sizeof(a));
      a.engine = d.engine; a.wfmt = dense_fmt; a.act_dtype = d.act_dtype; a.epilogue = SB_EPI_LINEAR;
      a.num_groups = E; a.m_rows = E; a.k = H; a.a_group_rows = E; a.lda = H;
      a.a_rows_total = static_cast<int64_t>(E) * E; a.a = w->gen_w;
      a.bias = w->gen_bias + static_cast<int64_t>(l) * E * E; a.bias_group_stride = E;
      a.x = b.x_src; a.ldx = H; a.max_rows = N * K; a.rows_hint = N * K; a.group_rows_bound = N; a.offsets = b.src_off;
      a.out = b.elog; a.ldo = E; a.splits = 1; a.status = b.status;
      if (gemm_gathers(a, d.engine)) {
        a.x = cur; a.x_row_index = b.src_row; a.x_rows = N;
      } else {
        StageScope sc_(2, st);
        SB_TRY(sb_gather_rows(cur, d.act_dtype, H, b.src_row, b.src_off, E, N * K, b.x_src, st));
      }
      { StageScope sc_(3, st); SB_TRY(run_gemm(a, d.engine, st)); }
    }
    // 5. top-M destinations per (token, source)
    { StageScope sc_(4, st); SB_TRY(sb_edge_topm(b.elog, E, E, M, b.src_slot, b.src_off, E, N * K, b.edge_idx, b.edge_w, st)); }
  }
  // 8's operands (sizes only): whether the edge-value GEMM gathers its token
  // rows itself or reads them from x_dst
  sb_grouped_gemm_args a;
  std::memset(&a, 0, sizeof(a));
  a.engine = d.engine; a.wfmt = dense_fmt; a.act_dtype = d.act_dtype; a.epilogue = SB_EPI_LINEAR;
  a.num_groups = E; a.m_rows = H; a.k = H; a.a_group_rows = H; a.lda = H;
  a.a_rows_total = static_cast<int64_t>(E) * H; a.a = w->edge_w;
  a.x = b.x_dst; a.ldx = H; a.max_rows = static_cast<int>(cap_dst);
  a.rows_hint = static_cast<int>(cap_dst * 7 / 8); a.group_rows_bound = N; a.offsets = b.dst_off; a.row_scale = b.dst_w;
  const int msg_splits = pick_splits(H, H, a.rows_hint, E, max_splits_for(N), tc_pref, N);
  a.splits = msg_splits; a.split_stride = cap_dst * H;
  a.out = b.y_msg; a.ldo = H; a.status = b.status;
  const bool edge_gathers = gemm_gathers(a, d.engine);
  // 6-7. (token, destination) pairs with summed coefficients (and, when asked,
  // the expert dispatch plan of step 9 in the same launches): one CTA per plan
  // for small batches, else both plans' two passes in two launches
  bool both = false;
  if (ffn_planned) {
    const GroupJob jd{b.edge_idx, b.edge_w, N, KM, E, 0, b.dst_off, b.dst_row, b.dst_slot, b.dst_w, b.dst_inv,
                      b.dst_rank, b.dst_wsc};
    const GroupJob jf{b.top_idx, b.top_w, N, K, E, SB_GROUP_POSITIVE_ONLY, b.ffn_off, b.ffn_row, b.ffn_slot, b.ffn_w,
                      b.ffn_inv, b.ffn_rank, b.ffn_wsc};
    StageScope sc_(5, st);
    rc = group_pair_launch(jd, jf, st);
    if (rc == SB_ERR_UNSUPPORTED && multi_plan_enabled()) {
      rc = group_pair_multi_launch(jd, jf, b.cc_dst, b.cc_ffn, st);
    }
    if (rc != SB_OK && rc != SB_ERR_UNSUPPORTED) return rc;
    both = rc == SB_OK;
    *ffn_planned = both;
  }
  if (!both) {
    StageScope sc_(5, st);
    SB_TRY(sb_group(b.edge_idx, b.edge_w, N, KM, E, 0, b.dst_off, b.dst_row, b.dst_slot, b.dst_w, b.dst_inv,
                    b.group_ws, b.group_ws_bytes, st));
  }
  // 8. c[t,d] * W_edge[d] h[t]
  {
    if (edge_gathers) {
      a.x = cur; a.x_row_index = b.dst_row; a.x_rows = N;
    } else {
      StageScope sc_(6, st);
      SB_TRY(sb_gather_rows(cur, d.act_dtype, H, b.dst_row, b.dst_off, E, static_cast<int>(cap_dst), b.x_dst, st));
    }
    { StageScope sc_(7, st); SB_TRY(run_gemm(a, d.engine, st)); }
    *msg_splits_out = msg_splits;
  }
#undef SB_TRY
  return SB_OK;
}

static int check_block_args(const sb_block_dims& d, const sb_block_weights* w, bool need_experts, bool need_dense) {
  if (!w) return SB_ERR_ARG;
  // routing picks top_k distinct experts and edges_per_expert distinct destinations
  if (need_dense && (d.top_k > d.num_experts || d.edges_per_expert > d.num_experts)) return SB_ERR_ARG;
  if (need_dense && (!w->router_w || !w->loop_bias || !w->gen_w || !w->gen_bias || !w->edge_w || !w->ln_w || !w->ln_b))
    return SB_ERR_ARG;
  if (need_experts && (!w->w_up || !w->b_up || !w->w_down || !w->b_down ||
                       (d.activation == SB_ACT_SWIGLU && d.ffn % 64) ||
                       ((d.wfmt == SB_W_FP8 || d.wfmt == SB_W_INT4) && (!w->s_up || !w->s_down))))
    return SB_ERR_ARG;
  return SB_OK;
}

extern "C" SB_API int sb_block_forward(const sb_block_dims* dims, const sb_block_weights* w, const void* h_in,
                                       const void* x0, void* h_out, int n_tokens, int loop_begin, int loop_end,
                                       void* workspace, size_t workspace_bytes, const sb_block_taps* taps,
                                       void* stream) {
  int rc = check_dims(dims);
  if (rc) return rc;
  const sb_block_dims& d = *dims;
  if (check_block_args(d, w, true, true) || n_tokens < 0 || n_tokens > d.max_tokens || loop_begin < 0 ||
      loop_end > d.num_loops || loop_begin > loop_end)
    return SB_ERR_ARG;
  if (n_tokens == 0 || loop_begin == loop_end) return SB_OK;
  if (!h_in || !x0 || !h_out) return SB_ERR_ARG;
  BlockBuffers b;
  const size_t need = carve_block(d, d.max_tokens, workspace, workspace_bytes, &b);
  if (!workspace || need == static_cast<size_t>(-1) || workspace_bytes < need) return SB_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int N = n_tokens, H = d.hidden, E = d.num_experts, K = d.top_k, M = d.edges_per_expert, U = d.ffn;
  const int KM = K * M;
  const int64_t cap_dst = static_cast<int64_t>(N) * (E < KM ? E : KM);
  const bool tc_pref = d.engine != SB_ENGINE_SIMT;
  const void* cur = h_in;
#define SB_TRY(x) do { rc = (x); if (rc) return rc; } while (0)
  // decode: loop l's LayerNorm kernel also routes loop l+1 (SPIDER_B200_FUSE_LN_ROUTE=0 disables)
  const bool fuse_next = use_fused_route(d, N) && fuse_ln_route_enabled();
  bool routed = false;
  // prefill with fp8 / int4 experts: the expert weights in bf16 once for all loops of this call
  const bool deq = b.w_up_bf && dequant_once_possible(d, N);
  if (deq) {
    StageScope sc_(13, st);
    const int64_t up_rows = static_cast<int64_t>(d.activation == SB_ACT_SWIGLU ? 2 : 1) * U;
    SB_TRY(dequant_to_bf16(d.wfmt, w->w_up, w->s_up, d.group_size, static_cast<int64_t>(E) * up_rows, H, b.w_up_bf,
                           st));
    SB_TRY(dequant_to_bf16(d.wfmt, w->w_down, w->s_down, d.group_size, static_cast<int64_t>(E) * H, U, b.w_down_bf,
                           st));
  }
  // the expert GEMMs on the bf16 copies: fp8 keeps its per-row scale in the epilogue
  auto use_copy = [&](sb_grouped_gemm_args& a, void* copy) {
    if (!deq) return;
    a.wfmt = SB_W_BF16;
    a.a = copy;
    if (d.wfmt != SB_W_FP8) a.a_scale = nullptr;
  };
  for (int l = loop_begin; l < loop_end; ++l) {
    void* next = (l == loop_end - 1) ? h_out : b.hbuf[(l - loop_begin) & 1];
    int msg_splits = 1;
    bool ffn_planned = false;
    SB_TRY(route_loop(d, w, b, cur, N, l, &msg_splits, &ffn_planned, routed, st));
    // 9. dispatch plan of the expert FFN (unless built with the destination plan)
    if (!ffn_planned) {
      StageScope sc_(8, st);
      SB_TRY(sb_group(b.top_idx, b.top_w, N, K, E, SB_GROUP_POSITIVE_ONLY, b.ffn_off, b.ffn_row, b.ffn_slot, b.ffn_w,
                      b.ffn_inv, b.group_ws, b.group_ws_bytes, st));
    }
    // 10-11. messages (sum over the token's destinations), then up projection +
    // activation with the message rows gathered in expert order.
    {
      sb_grouped_gemm_args a;
      fill_expert_gemm(a, d, true, w->w_up, w->s_up, w->b_up, w->w_gate, w->s_gate, w->b_gate);
      use_copy(a, b.w_up_bf);
      a.epilogue = d.activation == SB_ACT_SWIGLU ? SB_EPI_SWIGLU_IL : SB_EPI_GELU;
      a.num_groups = E; a.x = b.x_ffn; a.ldx = H; a.max_rows = N * K; a.rows_hint = N * K; a.group_rows_bound = N;
      a.offsets = b.ffn_off; a.out = b.act; a.ldo = U; a.splits = 1; a.status = b.status;
      const bool gather = gemm_gathers(a, d.engine);
      float* msg_out = (taps && taps->messages) ? b.msg_f32 : nullptr;
      { StageScope sc_(9, st); SB_TRY(sb_combine_rows(b.y_msg, H, msg_splits, cap_dst * H, b.dst_inv, KM, N, H, msg_out,
                                                  gather ? nullptr : b.ffn_inv, K, gather ? b.msg_act : b.x_ffn,
                                                  d.act_dtype, st)); }
      if (gather) {
        a.x = b.msg_act; a.x_row_index = b.ffn_row; a.x_rows = N;
      }
      { StageScope sc_(10, st); SB_TRY(run_gemm(a, d.engine, st)); }
    }
    // 12. down projection, scaled by the routing weight
    int ffn_splits = 1;
    {
      sb_grouped_gemm_args a;
      fill_expert_gemm(a, d, false, w->w_down, w->s_down, w->b_down, nullptr, nullptr, nullptr);
      use_copy(a, b.w_down_bf);
      a.epilogue = SB_EPI_LINEAR;
      a.num_groups = E; a.x = b.act; a.ldx = U; a.max_rows = N * K; a.rows_hint = N * K; a.group_rows_bound = N;
      a.offsets = b.ffn_off; a.row_scale = b.ffn_w;
      ffn_splits = pick_splits(H, U, N * K, E, max_splits_for(N), tc_pref, N);
      a.splits = ffn_splits; a.split_stride = static_cast<int64_t>(N) * K * H;
      a.out = b.y_ffn; a.ldo = H; a.status = b.status;
      { StageScope sc_(11, st); SB_TRY(run_gemm(a, d.engine, st)); }
    }
    // 13. delta + LayerNorm epilogue; in decode also the next loop's routing
    // (steps 1-5 of loop l+1) in the same kernel
    routed = false;
    if (l + 1 < loop_end && fuse_next) {
      StageScope sc_(12, st);
      const RouteArgs ra{w->router_w, w->loop_bias + static_cast<int64_t>(l + 1) * E, w->gen_w,
                         w->gen_bias + static_cast<int64_t>(l + 1) * E * E, E, K, M, b.top_idx, b.top_w, b.edge_idx,
                         b.edge_w};
      rc = combine_ln_route(b.y_ffn, H, ffn_splits, static_cast<int64_t>(N) * K * H, b.ffn_inv, K, cur, x0,
                            d.act_dtype, N, H, w->ln_w, w->ln_b, d.residual_scale, d.reinject, d.ln_eps, next, ra, st);
      if (rc != SB_OK && rc != SB_ERR_UNSUPPORTED) return rc;
      routed = rc == SB_OK;
    }
    if (!routed) {
      StageScope sc_(12, st);
      SB_TRY(sb_combine_ln(b.y_ffn, H, ffn_splits, static_cast<int64_t>(N) * K * H, b.ffn_inv, K, nullptr, cur, x0,
                           d.act_dtype, N, H, w->ln_w, w->ln_b, d.residual_scale, d.reinject, d.ln_eps, next,
                           (taps && taps->delta && l == loop_end - 1) ? taps->delta : nullptr, st));
    }
    if (taps && l == loop_end - 1) {
      auto cp = [&](void* dst, const void* src, size_t bytes) -> int {
        return dst ? cuda_status(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, st)) : SB_OK;
      };
      SB_TRY(cp(taps->top_idx, b.top_idx, sizeof(int32_t) * N * K));
      SB_TRY(cp(taps->top_w, b.top_w, sizeof(float) * N * K));
      SB_TRY(cp(taps->edge_idx, b.edge_idx, sizeof(int32_t) * N * KM));
      SB_TRY(cp(taps->edge_w, b.edge_w, sizeof(float) * N * KM));
      SB_TRY(cp(taps->messages, b.msg_f32, sizeof(float) * static_cast<size_t>(N) * H));
      SB_TRY(cp(taps->ffn_offsets, b.ffn_off, sizeof(int32_t) * (E + 1)));
      SB_TRY(cp(taps->ffn_rows, b.ffn_row, sizeof(int32_t) * N * K));
      SB_TRY(cp(taps->ffn_weights, b.ffn_w, sizeof(float) * N * K));
    }
    cur = next;
  }
#undef SB_TRY
  return SB_OK;
}

extern "C" SB_API int sb_block_route(const sb_block_dims* dims, const sb_block_weights* w, const void* h, int n_tokens,
                                     int loop_idx, void* messages, float* messages_f32, int32_t* top_idx, float* top_w,
                                     void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_dims(dims);
  if (rc) return rc;
  const sb_block_dims& d = *dims;
  if (check_block_args(d, w, false, true) || n_tokens < 0 || n_tokens > d.max_tokens || loop_idx < 0 ||
      loop_idx >= d.num_loops)
    return SB_ERR_ARG;
  if (n_tokens == 0) return SB_OK;
  if (!h || !messages || !top_idx || !top_w) return SB_ERR_ARG;
  BlockBuffers b;
  const size_t need = carve_block(d, d.max_tokens, workspace, workspace_bytes, &b);
  if (!workspace || need == static_cast<size_t>(-1) || workspace_bytes < need) return SB_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int N = n_tokens, H = d.hidden, E = d.num_experts, K = d.top_k, KM = K * d.edges_per_expert;
  const int64_t cap_dst = static_cast<int64_t>(N) * (E < KM ? E : KM);
  int msg_splits = 1;
  if ((rc = route_loop(d, w, b, h, N, loop_idx, &msg_splits, nullptr, false, st))) return rc;
  if ((rc = sb_combine_rows(b.y_msg, H, msg_splits, cap_dst * H, b.dst_inv, KM, N, H, messages_f32, nullptr, K,
                            messages, d.act_dtype, st)))
    return rc;
  if ((rc = cuda_status(cudaMemcpyAsync(top_idx, b.top_idx, sizeof(int32_t) * N * K, cudaMemcpyDeviceToDevice, st))))
    return rc;
  return cuda_status(cudaMemcpyAsync(top_w, b.top_w, sizeof(float) * N * K, cudaMemcpyDeviceToDevice, st));
}

// ------------------------------------------------------------------ sparse expert delta

static size_t carve_delta(const sb_block_dims& d, int n, void* base, size_t size, BlockBuffers* b) {
  Carver c(base, size);
  const int64_t N = n, H = d.hidden, E = d.num_experts, K = d.top_k, U = d.ffn;
  const int as = act_size(d.act_dtype);
  b->status = c.take<int>(kStatusBytes / sizeof(int));
  b->top_idx = c.take<int32_t>(N * K);  // local expert ids
  b->ffn_off = c.take<int32_t>(E + 1);
  b->ffn_row = c.take<int32_t>(N * K);
  b->ffn_slot = c.take<int32_t>(N * K);
  b->ffn_w = c.take<float>(N * K);
  b->ffn_inv = c.take<int32_t>(N * K);
  b->x_ffn = c.take<char>(N * K * H * as);
  b->msg_act = c.take<char>(N * H * as);
  b->act = c.take<char>(N * K * U * as);
  b->y_ffn = c.take<float>(4 * N * K * H);
  b->group_ws_bytes = sb_group_workspace_bytes(static_cast<int>(N), static_cast<int>(K), static_cast<int>(E));
  b->group_ws = c.take<char>(b->group_ws_bytes);
  return c.overflow ? static_cast<size_t>(-1) : align_up(c.used, 256);
}

extern "C" SB_API size_t sb_expert_rows_workspace_bytes(const sb_block_dims* dims, int n_rows) {
  if (check_dims(dims) != SB_OK || n_rows < 0) return 0;
  BlockBuffers b;
  return carve_delta(*dims, n_rows > 0 ? n_rows : 1, nullptr, ~size_t(0) >> 1, &b) +
         align_up(static_cast<size_t>(n_rows > 0 ? n_rows : 1) * dims->top_k * 4, 256);
}

// The owner's experts on received rows.  With `peer` (peer transport) the rows
// are this rank's region's receive rows, the first kernel waits for every
// rank's dispatch flag and the last writes the results into the sources'
// regions and raises the return flags (instead of writing `out`).
static int expert_rows_impl(const sb_block_dims* dims, const sb_block_weights* w, const void* rows, int64_t row_pitch,
                            int n_rows, int expected_pairs, float* out, void* workspace, size_t workspace_bytes,
                            cudaStream_t st, const EpPeerArgs* peer) {
  int rc = check_dims(dims);
  if (rc) return rc;
  const sb_block_dims& d = *dims;
  const int es = d.act_dtype == SB_F32 ? 4 : 2;
  const int64_t meta_off = static_cast<int64_t>(d.hidden) * es;
  if (check_block_args(d, w, true, false) || n_rows < 0 || row_pitch % 16 ||
      row_pitch < meta_off + 8LL * d.top_k)
    return SB_ERR_ARG;
  if (n_rows == 0) return SB_OK;
  if (!rows || (!out && !peer)) return SB_ERR_ARG;
  BlockBuffers b;
  const size_t need = carve_delta(d, n_rows, workspace, workspace_bytes, &b);
  const size_t wbytes = align_up(static_cast<size_t>(n_rows) * d.top_k * 4, 256);
  if (!workspace || need == static_cast<size_t>(-1) || workspace_bytes < need + wbytes) return SB_ERR_WORKSPACE;
  float* top_w = reinterpret_cast<float*>(static_cast<char*>(workspace) + need);
  const int N = n_rows, H = d.hidden, K = d.top_k, U = d.ffn, G = d.num_experts;
  const int ldx = static_cast<int>(row_pitch / es);
  // Most received rows are padding: tile choices follow the expected real pairs.
  // When those average at most 32 per expert, a 64-row tile per expert is
  // planned (an expert with more rows is covered by its CTA looping).
  const int hint = expected_pairs > 0 ? expected_pairs : N * K;
  const int row_plan = hint <= 32 * G ? (N < 64 ? N : 64) : N;
#define SB_TRY(x) do { rc = (x); if (rc) return rc; } while (0)
  // dispatch plan over the rows' local expert ids: one kernel reading the row
  // metadata, or (many rows) unpack, then sb_group
  rc = derived_group_launch(0, rows, row_pitch, meta_off, nullptr, G, N, K, G, SB_GROUP_POSITIVE_ONLY, b.ffn_off,
                            b.ffn_row, b.ffn_slot, b.ffn_w, b.ffn_inv, b.group_ws, b.group_ws_bytes, st,
                            peer ? peer->own : nullptr, peer ? peer->ctrl_off : 0, peer ? peer->world : 0,
                            peer ? peer->status : nullptr);
  if (rc == SB_ERR_UNSUPPORTED) {
    if (peer) SB_TRY(sb_ep_wait(peer->own, peer->world, peer->cap, row_pitch, H, 0, peer->status, st));
    SB_TRY(launch(unpack_meta_kernel, dim3((N * K + 255) / 256), dim3(256), 0, st, static_cast<const uint8_t*>(rows),
                  row_pitch, meta_off, N, K, G, b.top_idx, top_w));
    SB_TRY(sb_group(b.top_idx, top_w, N, K, G, SB_GROUP_POSITIVE_ONLY, b.ffn_off, b.ffn_row, b.ffn_slot, b.ffn_w,
                    b.ffn_inv, b.group_ws, b.group_ws_bytes, st));
  } else if (rc) {
    return rc;
  }
  {
    sb_grouped_gemm_args a;
    fill_expert_gemm(a, d, true, w->w_up, w->s_up, w->b_up, w->w_gate, w->s_gate, w->b_gate);
    a.epilogue = d.activation == SB_ACT_SWIGLU ? SB_EPI_SWIGLU_IL : SB_EPI_GELU;
    a.num_groups = G; a.x = b.x_ffn; a.ldx = H; a.max_rows = N * K; a.rows_hint = hint; a.group_rows_bound = row_plan;
    a.offsets = b.ffn_off; a.out = b.act; a.ldo = U; a.splits = 1; a.status = b.status;
    sb_grouped_gemm_args g = a;
    g.x = rows; g.ldx = ldx; g.x_row_index = b.ffn_row; g.x_rows = N;
    // decided on the plain operand: large tiles read materialised rows on the
    // tensor cores rather than gathering on the CUDA-core engine
    if (gemm_gathers(a, d.engine)) {
      a = g;
    } else {
      // materialise the message rows (first hidden columns of each packed row), then in expert order
      SB_TRY(cuda_status(cudaMemcpy2DAsync(b.msg_act, static_cast<size_t>(H) * es, rows, row_pitch,
                                           static_cast<size_t>(H) * es, N, cudaMemcpyDeviceToDevice, st)));
      SB_TRY(sb_gather_rows(b.msg_act, d.act_dtype, H, b.ffn_row, b.ffn_off, G, N * K, b.x_ffn, st));
    }
    SB_TRY(run_gemm(a, d.engine, st));
  }
  int splits = 1;
  {
    sb_grouped_gemm_args a;
    fill_expert_gemm(a, d, false, w->w_down, w->s_down, w->b_down, nullptr, nullptr, nullptr);
    a.epilogue = SB_EPI_LINEAR;
    a.num_groups = G; a.x = b.act; a.ldx = U; a.max_rows = N * K; a.rows_hint = hint; a.group_rows_bound = row_plan;
    a.offsets = b.ffn_off; a.row_scale = b.ffn_w;
    splits = pick_splits(H, U, hint, G, 4, d.engine != SB_ENGINE_SIMT, row_plan);
    a.splits = splits; a.split_stride = static_cast<int64_t>(N) * K * H;
    a.out = b.y_ffn; a.ldo = H; a.status = b.status;
    SB_TRY(run_gemm(a, d.engine, st));
  }
  if (peer)
    SB_TRY(combine_rows_peer(b.y_ffn, H, splits, static_cast<int64_t>(N) * K * H, b.ffn_inv, K, N, H, *peer, st));
  else
    SB_TRY(sb_combine_rows(b.y_ffn, H, splits, static_cast<int64_t>(N) * K * H, b.ffn_inv, K, N, H, out, nullptr, 0,
                           nullptr, d.act_dtype, st));
#undef SB_TRY
  return SB_OK;
}

extern "C" SB_API int sb_expert_rows(const sb_block_dims* dims, const sb_block_weights* w, const void* rows,
                                     int64_t row_pitch, int n_rows, int expected_pairs, float* out, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  return expert_rows_impl(dims, w, rows, row_pitch, n_rows, expected_pairs, out, workspace, workspace_bytes,
                          static_cast<cudaStream_t>(stream), nullptr);
}

extern "C" SB_API int sb_expert_rows_peer(const sb_block_dims* dims, const sb_block_weights* w, void* region,
                                          void* const* regions, int world, int rank, int cap, int64_t row_pitch,
                                          int expected_pairs, int* status, void* workspace, size_t workspace_bytes,
                                          void* stream) {
  if (!dims || !region || !regions || world <= 0 || rank < 0 || rank >= world || cap <= 0 ||
      !sb_ep_peer_region_bytes(world, cap, row_pitch, dims->hidden))
    return SB_ERR_ARG;
  EpPeerArgs pa;
  pa.regions = regions;
  pa.own = region;
  pa.world = world;
  pa.rank = rank;
  pa.cap = cap;
  pa.status = status;
  ep_region_offsets(world, cap, row_pitch, dims->hidden, &pa.ret_off, &pa.ctrl_off);
  return expert_rows_impl(dims, w, region, row_pitch, world * cap, expected_pairs, nullptr, workspace,
                          workspace_bytes, static_cast<cudaStream_t>(stream), &pa);
}

extern "C" SB_API size_t sb_expert_delta_workspace_bytes(const sb_block_dims* dims, int n_tokens) {
  if (check_dims(dims) != SB_OK || n_tokens < 0) return 0;
  BlockBuffers b;
  return carve_delta(*dims, n_tokens > 0 ? n_tokens : 1, nullptr, ~size_t(0) >> 1, &b);
}

extern "C" SB_API int sb_expert_delta(const sb_block_dims* dims, const sb_block_weights* w, const void* messages,
                                      const int32_t* top_idx, const float* top_w, int n_tokens, int rank,
                                      int world, float* delta, void* workspace, size_t workspace_bytes,
                                      void* stream) {
  int rc = check_dims(dims);
  if (rc) return rc;
  const sb_block_dims& d = *dims;
  if (!w || !w->w_up || !w->b_up || !w->w_down || !w->b_down || n_tokens < 0 || world <= 0 || rank < 0 ||
      rank >= world || (d.activation == SB_ACT_SWIGLU && (!w->w_gate || !w->b_gate)) ||
      ((d.wfmt == SB_W_FP8 || d.wfmt == SB_W_INT4) && (!w->s_up || !w->s_down)))
    return SB_ERR_ARG;
  if (n_tokens == 0) return SB_OK;
  if (!messages || !top_idx || !top_w || !delta) return SB_ERR_ARG;
  BlockBuffers b;
  const size_t need = carve_delta(d, n_tokens, workspace, workspace_bytes, &b);
  if (!workspace || need == static_cast<size_t>(-1) || workspace_bytes < need) return SB_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int N = n_tokens, H = d.hidden, E = d.num_experts, K = d.top_k, U = d.ffn;
  const int G = (E - rank + world - 1) / world;
  if (G <= 0) return cuda_status(cudaMemsetAsync(delta, 0, sizeof(float) * static_cast<size_t>(N) * H, st));
  rc = launch(remap_local_kernel, dim3((N * K + 255) / 256), dim3(256), 0, st, top_idx, N * K, E, rank, world,
              b.top_idx);
  if (rc) return rc;
#define SB_TRY(x) do { rc = (x); if (rc) return rc; } while (0)
  SB_TRY(sb_group(b.top_idx, top_w, N, K, G, SB_GROUP_POSITIVE_ONLY, b.ffn_off, b.ffn_row, b.ffn_slot, b.ffn_w,
                  b.ffn_inv, b.group_ws, b.group_ws_bytes, st));
  {
    sb_grouped_gemm_args a;
    fill_expert_gemm(a, d, true, w->w_up, w->s_up, w->b_up, w->w_gate, w->s_gate, w->b_gate);
    shard_expert_gemm(a, d, rank, world);
    a.epilogue = d.activation == SB_ACT_SWIGLU ? SB_EPI_SWIGLU_IL : SB_EPI_GELU;
    a.num_groups = G; a.x = b.x_ffn; a.ldx = H; a.max_rows = N * K; a.rows_hint = N * K; a.group_rows_bound = N;
    a.offsets = b.ffn_off; a.out = b.act; a.ldo = U; a.splits = 1; a.status = b.status;
    if (gemm_gathers(a, d.engine)) {
      a.x = messages; a.x_row_index = b.ffn_row; a.x_rows = N;
    } else {
      SB_TRY(sb_gather_rows(messages, d.act_dtype, H, b.ffn_row, b.ffn_off, G, N * K, b.x_ffn, st));
    }
    SB_TRY(run_gemm(a, d.engine, st));
  }
  int splits = 1;
  {
    sb_grouped_gemm_args a;
    fill_expert_gemm(a, d, false, w->w_down, w->s_down, w->b_down, nullptr, nullptr, nullptr);
    shard_expert_gemm(a, d, rank, world);
    a.epilogue = SB_EPI_LINEAR;
    a.num_groups = G; a.x = b.act; a.ldx = U; a.max_rows = N * K; a.rows_hint = N * K; a.group_rows_bound = N;
    a.offsets = b.ffn_off; a.row_scale = b.ffn_w;
    splits = pick_splits(H, U, N * K, G, 4, d.engine != SB_ENGINE_SIMT, N);
    a.splits = splits; a.split_stride = static_cast<int64_t>(N) * K * H;
    a.out = b.y_ffn; a.ldo = H; a.status = b.status;
    SB_TRY(run_gemm(a, d.engine, st));
  }
  SB_TRY(sb_combine_rows(b.y_ffn, H, splits, static_cast<int64_t>(N) * K * H, b.ffn_inv, K, N, H, delta, nullptr, 0,
                         nullptr, d.act_dtype, st));
#undef SB_TRY
  return SB_OK;
}

extern "C" SB_API int sb_stage_timing(int enable) {
  std::lock_guard<std::mutex> lk(g_timing.mu);
  g_timing.on = enable != 0;
  if (enable) {
    for (auto& m : g_timing.marks) {
      cudaEventDestroy(m.second.first);
      cudaEventDestroy(m.second.second);
    }
    g_timing.marks.clear();
  }
  return SB_OK;
}

extern "C" SB_API int sb_stage_timing_read(double* ms, int* launches, int n_stages) {
  if (!ms || !launches || n_stages < kNumStages) return SB_ERR_ARG;
  std::lock_guard<std::mutex> lk(g_timing.mu);
  for (int i = 0; i < kNumStages; ++i) { ms[i] = 0.0; launches[i] = 0; }
  int rc = SB_OK;
  for (auto& m : g_timing.marks) {
    float t = 0.f;
    cudaError_t e = cudaEventSynchronize(m.second.second);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&t, m.second.first, m.second.second);
    if (e != cudaSuccess) rc = cuda_status(e);
    ms[m.first] += t;
    launches[m.first] += 1;
    cudaEventDestroy(m.second.first);
    cudaEventDestroy(m.second.second);
  }
  g_timing.marks.clear();
  return rc;
}

extern "C" SB_API const char* sb_stage_name(int stage) {
  return (stage >= 0 && stage < kNumStages) ? kStageNames[stage] : "";
}

extern "C" SB_API unsigned long long sb_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

extern "C" SB_API int sb_num_stages(void) { return kNumStages; }

// ---------------------------------------------------------------------------
// Loop statistics (model.py:327-343): router probabilities, the routed and
// edge load histograms over all E sources, both losses, exit confidence.
// ---------------------------------------------------------------------------
struct StatsBuffers {
  int* status;
  LoopStatsAcc acc;
  int32_t* top_idx;
  float* top_w;
  float* elog;
};

static size_t carve_stats(const sb_block_dims& d, int n, void* base, size_t size, StatsBuffers* b) {
  Carver c(base, size);
  const int64_t N = n, E = d.num_experts, K = d.top_k;
  b->status = c.take<int>(kStatusBytes / sizeof(int));
  b->acc.expert_count = c.take<uint32_t>(E);
  b->acc.edge_count = c.take<uint32_t>(E);
  b->acc.prob_sum = c.take<float>(kLoopStatsMaxParts * E);
  b->acc.importance = c.take<float>(kLoopStatsMaxParts * E);
  b->top_idx = c.take<int32_t>(N * K);
  b->top_w = c.take<float>(N * K);
  b->elog = c.take<float>(N * E * E);
  return c.overflow ? static_cast<size_t>(-1) : align_up(c.used, 256);
}

extern "C" SB_API size_t sb_loop_stats_workspace_bytes(const sb_block_dims* dims, int n_tokens) {
  if (check_dims(dims) != SB_OK || n_tokens < 0) return 0;
  StatsBuffers b;
  return carve_stats(*dims, n_tokens > 0 ? n_tokens : 1, nullptr, ~size_t(0) >> 1, &b);
}

extern "C" SB_API int sb_loop_stats(const sb_block_dims* dims, const sb_block_weights* w, int loop_idx,
                                    const void* h_in, const void* h_out, const int32_t* top_idx, int n_tokens,
                                    const float* exit_w, const float* exit_b, float* router_probs, float* confidence,
                                    float* stats, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_dims(dims);
  if (rc) return rc;
  const sb_block_dims& d = *dims;
  if (!w || !w->router_w || !w->loop_bias || !w->gen_w || !w->gen_bias || loop_idx < 0 || loop_idx >= d.num_loops ||
      n_tokens < 0 || !stats || !workspace || (n_tokens > 0 && (!h_in || !router_probs)) ||
      ((confidence != nullptr) != (h_out != nullptr)) || (confidence && (!exit_w || !exit_b)))
    return SB_ERR_ARG;
  StatsBuffers b;
  const size_t need = carve_stats(d, n_tokens > 0 ? n_tokens : 1, workspace, workspace_bytes, &b);
  if (need > workspace_bytes) return SB_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int H = d.hidden, E = d.num_experts, K = d.top_k, M = d.edges_per_expert;
  // status word and the two [E] counters are contiguous at the front
  rc = cuda_status(cudaMemsetAsync(b.status, 0,
                                   reinterpret_cast<char*>(b.acc.prob_sum) - reinterpret_cast<char*>(b.status), st));
  if (rc) return rc;
  if (n_tokens > 0) {
    rc = sb_router(h_in, d.act_dtype, n_tokens, H, w->router_w, w->loop_bias + static_cast<int64_t>(loop_idx) * E, E,
                   K, b.top_idx, b.top_w, router_probs, st);
    if (rc) return rc;
    // edge logits of every (token, source): one dense group of E*E generator rows
    sb_grouped_gemm_args a;
    std::memset(&a, 0, sizeof(a));
    a.engine = d.engine; a.wfmt = d.act_dtype == SB_F32 ? SB_W_F32 : SB_W_BF16; a.act_dtype = d.act_dtype;
    a.epilogue = SB_EPI_LINEAR;
    a.num_groups = 1; a.m_rows = E * E; a.k = H; a.a_group_rows = E * E; a.lda = H;
    a.a_rows_total = static_cast<int64_t>(E) * E; a.a = w->gen_w;
    a.bias = w->gen_bias + static_cast<int64_t>(loop_idx) * E * E; a.bias_group_stride = E * E;
    a.x = h_in; a.ldx = H; a.max_rows = n_tokens; a.rows_hint = n_tokens; a.offsets = nullptr;
    a.out = b.elog; a.ldo = E * E; a.splits = 1; a.status = b.status;
    rc = run_gemm(a, d.engine, st);
    if (rc) return rc;
  }
  return loop_stats_launch(b.elog, router_probs, top_idx ? top_idx : b.top_idx, h_out, d.act_dtype, exit_w, exit_b,
                           n_tokens, H, E, K, M, confidence, b.acc, stats, st);
}

// ---------------------------------------------------------------------------
// Lumen workspace (lumen.py:81-123): two one-group GEMMs and two warp-per-token
// kernels (sb_lumen.cu).
// ---------------------------------------------------------------------------
struct LumenBuffers {
  int* status;
  float* qv;
  void* values;
  float* c;
  float* raw;
};

static size_t carve_lumen(int n, int H, int S, int D, void* base, size_t size, LumenBuffers* b) {
  Carver c(base, size);
  b->status = c.take<int>(kStatusBytes / sizeof(int));
  b->qv = c.take<float>(static_cast<int64_t>(n) * (S + D));
  b->values = c.take<char>(static_cast<int64_t>(n) * D * 4);
  b->c = c.take<float>(n);
  b->raw = c.take<float>(static_cast<int64_t>(n) * H);
  return c.overflow ? static_cast<size_t>(-1) : align_up(c.used, 256);
}

extern "C" SB_API size_t sb_lumen_workspace_bytes(int n_tokens, int hidden, int slots, int slot_dim) {
  if (n_tokens < 0 || hidden <= 0 || slots <= 0 || slot_dim <= 0) return 0;
  LumenBuffers b;
  return carve_lumen(n_tokens > 0 ? n_tokens : 1, hidden, slots, slot_dim, nullptr, ~size_t(0) >> 1, &b);
}

extern "C" SB_API int sb_lumen_forward(int act_dtype, int engine, int n_tokens, int hidden, int slots, int slot_dim,
                                       const sb_lumen_weights* w, const void* h, void* out, float* slot_weights,
                                       float* values, float* broadcast, float* broadcast_norm, void* workspace,
                                       size_t workspace_bytes, void* stream) {
  if ((act_dtype != SB_F32 && act_dtype != SB_BF16) || n_tokens < 0 || hidden <= 0 || hidden % 8 || slots <= 0 ||
      slots > 32 || slot_dim <= 0 || !w || !w->wqv || !w->qv_bias || !w->w_o || !w->gate_w || !w->gate_b ||
      !w->ln_w || !w->ln_b || !workspace || engine < SB_ENGINE_AUTO || engine > SB_ENGINE_TCGEN05)
    return SB_ERR_ARG;
  if (n_tokens == 0) return SB_OK;
  if (!h || !out) return SB_ERR_ARG;
  LumenBuffers b;
  const size_t need = carve_lumen(n_tokens, hidden, slots, slot_dim, workspace, workspace_bytes, &b);
  if (need == static_cast<size_t>(-1) || workspace_bytes < need) return SB_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int H = hidden, S = slots, D = slot_dim;
  const int wfmt = act_dtype == SB_F32 ? SB_W_F32 : SB_W_BF16;
  int rc = cuda_status(cudaMemsetAsync(b.status, 0, kStatusBytes, st));
  if (rc) return rc;
  {  // scores and values
    sb_grouped_gemm_args a;
    std::memset(&a, 0, sizeof(a));
    a.engine = engine; a.wfmt = wfmt; a.act_dtype = act_dtype; a.epilogue = SB_EPI_LINEAR;
    a.num_groups = 1; a.m_rows = S + D; a.k = H; a.a_group_rows = S + D; a.lda = H; a.a_rows_total = S + D;
    a.a = w->wqv; a.bias = w->qv_bias; a.bias_group_stride = S + D;
    a.x = h; a.ldx = H; a.max_rows = n_tokens; a.rows_hint = n_tokens; a.offsets = nullptr;
    a.out = b.qv; a.ldo = S + D; a.splits = 1; a.status = b.status;
    rc = run_gemm(a, engine, st);
    if (rc) return rc;
  }
  rc = lumen_mix_launch(b.qv, n_tokens, S, D, act_dtype, b.values, b.c, slot_weights, values, st);
  if (rc) return rc;
  {  // raw = c * (W_o values)
    sb_grouped_gemm_args a;
    std::memset(&a, 0, sizeof(a));
    a.engine = engine; a.wfmt = wfmt; a.act_dtype = act_dtype; a.epilogue = SB_EPI_LINEAR;
    a.num_groups = 1; a.m_rows = H; a.k = D; a.a_group_rows = H; a.lda = D; a.a_rows_total = H;
    a.a = w->w_o; a.x = b.values; a.ldx = D; a.max_rows = n_tokens; a.rows_hint = n_tokens; a.offsets = nullptr;
    a.row_scale = b.c; a.out = b.raw; a.ldo = H; a.splits = 1; a.status = b.status;
    rc = run_gemm(a, engine, st);
    if (rc) return rc;
  }
  return lumen_gate_ln_launch(h, b.raw, n_tokens, H, act_dtype, w->gate_w, w->gate_b, w->ln_w, w->ln_b, w->ln_eps, out,
                              broadcast, broadcast_norm, st);
}
