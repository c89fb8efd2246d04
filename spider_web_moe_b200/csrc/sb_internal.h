// Internal host-side helpers shared by the translation units of libspider_b200.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "spider_b200.h"

namespace sb {

inline int cuda_status(cudaError_t e) { return e == cudaSuccess ? SB_OK : SB_ERR_CUDA_BASE + static_cast<int>(e); }

inline int sb_last_launch_status() { return cuda_status(cudaGetLastError()); }

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Bump allocator over a caller-owned workspace; every carve is 256-byte aligned.
struct Carver {
  char* base;
  size_t size;
  size_t used = 0;
  bool overflow = false;
  Carver(void* b, size_t s) : base(static_cast<char*>(b)), size(s) {}
  template <typename T>
  T* take(size_t count) {
    used = align_up(used, 256);
    T* p = base ? reinterpret_cast<T*>(base + used) : nullptr;
    used += count * sizeof(T);
    if (used > size) overflow = true;
    return p;
  }
};

// Bytes reserved at the start of every workspace for the device status word.
constexpr size_t kStatusBytes = 256;

// Grouped GEMM engines (sb_gemm_simt.cu, sb_gemm_tc.cu).
int gemm_simt(const sb_grouped_gemm_args& a, cudaStream_t st);
int gemm_tcgen05(const sb_grouped_gemm_args& a, cudaStream_t st);
bool tcgen05_supported(const sb_grouped_gemm_args& a);
int tc_tile_n(const sb_grouped_gemm_args& a);  // column tile the tcgen05 engine picks
bool tc_fixed_groups(const sb_grouped_gemm_args& a);
// fp8 / int4 decode problems go to the persistent quantised decode kernel
bool tc_qdec(const sb_grouped_gemm_args& a);

// Kernel launch with programmatic stream serialization (PDL), unless disabled
// by SPIDER_B200_PDL=0.  Kernels launched this way call pdl_wait() first.
bool pdl_enabled();

// Kernel launches enqueued by this library (also those recorded into a CUDA
// graph while capturing); read by sb_kernel_launches().
void note_launch();

template <typename... KArgs, typename... Args>
inline int launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                  Args&&... args) {
  note_launch();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cuda_status(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...));
}

// Grouping kernel launch on caller-chosen scratch (sb_group.cu).
int group_launch_with_scratch(const int32_t* idx, const float* w, int n_rows, int slots, int num_groups, int flags,
                              int32_t* offsets, int32_t* perm_row, int32_t* perm_slot, float* perm_w, int32_t* inv,
                              int32_t* rank_scratch, float* w_scratch, cudaStream_t st);

// One grouping (sb_group's arguments with explicit scratch of n_rows*slots
// entries each); two of them run as one launch of two CTAs (sb_group.cu).
struct GroupJob {
  const int32_t* idx;
  const float* w;
  int n_rows, slots, num_groups, flags;
  int32_t* offsets;
  int32_t* perm_row;
  int32_t* perm_slot;
  float* perm_w;
  int32_t* inv;
  int32_t* rank_scratch;
  float* w_scratch;
};
// SB_ERR_UNSUPPORTED when either grouping is too large for one CTA.
int group_pair_launch(const GroupJob& j0, const GroupJob& j1, cudaStream_t st);
// The same two groupings with the multi-CTA two-pass schedule of sb_group
// (identical positions), both in one count launch and one place launch;
// cc0 / cc1 hold ceil(entries / 256) * num_groups counts per job.
constexpr int kGroupChunk = 256;
int group_pair_multi_launch(const GroupJob& j0, const GroupJob& j1, int32_t* cc0, int32_t* cc1, cudaStream_t st);

// Router + edge generator + edge top-M of small batches in one kernel
// (sb_router.cu); SB_ERR_UNSUPPORTED when its shared memory would exceed
// kRouteEdgesMaxSmem.
constexpr size_t kRouteEdgesMaxSmem = 160 * 1024;
size_t route_edges_smem(int act_dtype, int hidden, int E, int K);
int route_edges(const void* h, int act_dtype, int n_tokens, int hidden, const void* router_w, const float* rbias,
                int E, int K, const void* gen_w, const float* gen_bias, int M, int32_t* top_idx, float* top_w,
                int32_t* edge_idx, float* edge_w, cudaStream_t st);

// Peer-transport operands (region layout in sb_ep_dev.cuh): where the owner's
// combined rows go and which flags the kernels raise or wait for.
struct EpPeerArgs {
  void* const* regions;  // device array of the world regions as mapped here (null: not peer mode)
  void* own;             // this rank's region
  int world, rank, cap;
  int64_t ret_off, ctrl_off;
  int* status;
};
// EP region layout (sb_ep.cu): returns ret_off / ctrl_off for the region.
void ep_region_offsets(int world, int cap, int64_t row_pitch, int hidden, int64_t* ret_off, int64_t* ctrl_off);
// Row combine whose results go to the sources' regions (row t = q * cap + j
// to rank q's returned row [rank][j]) and then raise the return flags (sb_combine.cu).
int combine_rows_peer(const float* y, int64_t ldy, int splits, int64_t split_stride, const int32_t* inv, int slots,
                      int n_tokens, int cols, const EpPeerArgs& peer, cudaStream_t st);

// Routing operands of one loop (fused route kernels).
struct RouteArgs {
  const void* router_w;
  const float* router_bias;  // loop_bias of the loop routed
  const void* gen_w;
  const float* gen_bias;     // per-loop generator bias of the loop routed
  int E, K, M;
  int32_t* top_idx;
  float* top_w;
  int32_t* edge_idx;
  float* edge_w;
};
// LayerNorm epilogue of one loop and routing of the next in one kernel (one
// CTA per token, decode sizes; sb_combine.cu); SB_ERR_UNSUPPORTED when the
// routing's shared memory exceeds kRouteEdgesMaxSmem.
int combine_ln_route(const float* y, int64_t ldy, int splits, int64_t split_stride, const int32_t* inv, int slots,
                     const void* h, const void* x0, int act_dtype, int n_tokens, int cols, const float* ln_w,
                     const float* ln_b, float alpha, float beta, float eps, void* out, const RouteArgs& r,
                     cudaStream_t st);

// sb_group over ids derived in the grouping kernel itself (sb_group.cu): mode 0
// ids / weights from packed expert-parallel rows, mode 1 owner = top_idx % G.
// SB_ERR_UNSUPPORTED above 1024 entries; `workspace` as sb_group's.
// With wait_region (peer transport, mode 0) the kernel first waits for every
// rank's dispatch flag in that region.
int derived_group_launch(int mode, const void* rows, int64_t pitch, int64_t meta_off, const int32_t* top_idx,
                         int num_experts, int n, int K, int G, int flags, int32_t* offsets, int32_t* perm_row,
                         int32_t* perm_slot, float* perm_w, int32_t* inv, void* workspace, size_t workspace_bytes,
                         cudaStream_t st, void* wait_region = nullptr, int64_t ctrl_off = 0, int wait_world = 0,
                         int* status = nullptr);

// Top-K routing of router logits that a grouped GEMM computed (sb_router.cu).
int router_from_logits(const float* logits, int ld, int splits, int64_t split_stride, int n_tokens, int E, int K,
                       int32_t* top_idx, float* top_w, cudaStream_t st);

// Router + edge top-M of one token per warp from one row of dense logits
// [n_tokens, ld] (sb_router.cu): columns [0, E) the router logits, then the
// E x E edge logits of every source (s*E + d), all before their biases
// (rbias [E], gbias [E*E], added here in fp32).
int select_dense(const float* logits, int64_t ld, int n_tokens, int E, int K, int M, const float* rbias,
                 const float* gbias, int32_t* top_idx, float* top_w, int32_t* edge_idx, float* edge_w,
                 cudaStream_t st);

// fp8 e4m3 (exact) / int4 (bf16(q * group scale)) weights [rows, k] -> bf16 [rows, k]
// (sb_gemm_tc.cu): the values the tcgen05 GEMM's shared-memory conversion makes.
int dequant_to_bf16(int wfmt, const void* q, const void* scales, int group_size, int64_t rows, int64_t k, void* out,
                    cudaStream_t st);

// Device properties cached per device.
int current_sm_count();
int current_cc_major();

// Accumulators of the loop statistics (sb_stats.cu): integer counts [E],
// zeroed by the caller, and per-CTA float partials [kLoopStatsMaxParts, E].
constexpr int kLoopStatsMaxParts = 1024;
struct LoopStatsAcc {
  float* prob_sum;
  uint32_t* expert_count;
  uint32_t* edge_count;
  float* importance;
};
// Histograms of the full edge logits elog [N, E*E], the router probabilities
// probs [N, E] and the routing top_idx [N, K]; exit-head confidence of h_out
// into `confidence` (may be null); then the normalised statistics into stats [3E + 2].
int loop_stats_launch(const float* elog, const float* probs, const int32_t* top_idx, const void* h_out,
                      int act_dtype, const float* exit_w, const float* exit_b, int N, int H, int E, int K, int M,
                      float* confidence, LoopStatsAcc acc, float* stats, cudaStream_t st);

// Lumen kernels (sb_lumen.cu): softmax / slot mix after GEMM 1, gate +
// LayerNorm after GEMM 2.
int lumen_mix_launch(const float* qv, int n, int S, int D, int act_dtype, void* values, float* c, float* slot_w,
                     float* values_f32, cudaStream_t st);
int lumen_gate_ln_launch(const void* h, const float* raw, int n, int H, int act_dtype, const float* gate_w,
                         const float* gate_b, const float* ln_w, const float* ln_b, float eps, void* out,
                         float* broadcast, float* bnorm, cudaStream_t st);

}  // namespace sb
