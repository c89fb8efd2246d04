/*
 * spider_b200.h -- C ABI of the B200-native recurrent Spider-MoE block.
 *
 * The library (libspider_b200.so, built for sm_100a) exports plain extern "C"
 * functions: raw device pointers, sizes and a cudaStream_t passed as void*.
 * No torch types cross this boundary.  Every function returns an int status
 * (0 = ok), the convention of the reference C ABI
 * (kernels/include/spider_kernels.h:26-150: 0 ok, 1 bad argument, 2 index out
 * of range) extended with the codes below.  Work is only enqueued on the given
 * stream; nothing synchronises.  The library never allocates device memory on
 * a hot path: scratch space is a caller-owned workspace whose size the
 * *_workspace_bytes queries return (the pattern of the reference's
 * spider_cuda_expert_workspace_bytes, kernels/cuda/spider_expert_v2.cu:61-64).
 *
 * The arithmetic follows the reference PyTorch block (spider_moe/model.py:
 * 240-317), not the reference's own native kernels (which use tanh-GELU and a
 * static CSR graph, kernels/scalar/scalar.cpp:55-73).
 */
#ifndef SPIDER_B200_H
#define SPIDER_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(_WIN32)
#define SB_API __declspec(dllexport)
#else
#define SB_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ codes */
enum {
  SB_OK = 0,
  SB_ERR_ARG = 1,           /* bad argument (reference code 1) */
  SB_ERR_INDEX = 2,         /* index out of range (reference code 2) */
  SB_ERR_UNSUPPORTED = 3,   /* shape / format this build does not handle */
  SB_ERR_NO_DEVICE = 4,     /* no sm_100 device current */
  SB_ERR_WORKSPACE = 5,     /* workspace missing or too small */
  SB_ERR_DEVICE_STATUS = 6, /* a kernel recorded a device-side status word */
  SB_ERR_CUDA_BASE = 1000   /* 1000 + cudaError_t of a failed runtime call */
};

/* activation storage / compute types of the token rows */
enum { SB_F32 = 0, SB_BF16 = 1 };
/* expert weight formats (spider_moe/quant.py) */
enum {
  SB_W_F32 = 0,  /* fp32 weights (CUDA-core engine only) */
  SB_W_BF16 = 1,
  SB_W_FP8 = 2,  /* e4m3 bytes + fp32 scale per output row (quant.py:146-169) */
  SB_W_INT4 = 3  /* packed nibbles, even index low, + bf16 scale per row group (quant.py:89-143) */
};
/* expert activation */
enum { SB_ACT_GELU = 0, SB_ACT_SWIGLU = 1 };
/* grouped-GEMM epilogues */
enum {
  SB_EPI_LINEAR = 0, /* out_f32[row, m] = (acc + bias[m]) * row_scale[row]  (bias, scale optional) */
  SB_EPI_GELU = 1,   /* out_act[row, m] = gelu_erf(acc + bias[m])                             */
  SB_EPI_SWIGLU = 2, /* out_act[row, m] = silu(acc_gate + bias_gate[m]) * (acc + bias[m])      */
  /* SwiGLU with the gate and up rows of one weight tensor a, interleaved in
   * blocks of 64: rows [128 b, 128 b + 64) are the gate rows of output
   * features [64 b, 64 b + 64) and rows [128 b + 64, 128 b + 128) their up
   * rows (scales and biases interleaved the same way).  m_rows counts the
   * interleaved rows (a multiple of 128); the output has m_rows / 2 features:
   * out_act[row, f] = silu(acc[gate row of f] + bias) * (acc[up row of f] + bias).
   * One MMA operand covers both halves, so the tensor core runs its widest
   * tiles on SwiGLU as on the other epilogues.  a_gate is not used. */
  SB_EPI_SWIGLU_IL = 3
};
/* GEMM engines */
enum { SB_ENGINE_AUTO = 0, SB_ENGINE_SIMT = 1, SB_ENGINE_TCGEN05 = 2 };
/* grouping flags */
enum { SB_GROUP_POSITIVE_ONLY = 1 };

/* ------------------------------------------------------------------ info */
/* Bit 0: library built for sm_100a; bit 1: current device is compute capability 10.x. */
SB_API int sb_capabilities(void);
SB_API const char* sb_version(void);
SB_API const char* sb_error_string(int code);

/* ------------------------------------------------------------------ router
 * Replaces spider_router_f32 (kernels/include/spider_kernels.h:26-28) and the
 * router lines of SpiderMoELayer.forward (spider_moe/model.py:254-258):
 * logits = h . router_w^T + loop_bias_l; fp32 softmax over E; top-k of the
 * probabilities (descending; equal values -> smaller expert id first);
 * weights renormalised by max(sum, 1e-9).  probs may be NULL.
 * h: [n_tokens, hidden] (act_dtype); router_w: [E, hidden] (act_dtype). */
SB_API int sb_router(const void* h, int act_dtype, int n_tokens, int hidden, const void* router_w,
                     const float* loop_bias_l, int num_experts, int top_k, int32_t* top_idx,
                     float* top_w, float* probs, void* stream);

/* ------------------------------------------------------------------ grouping
 * Replaces build_dispatch_plan (spider_infer/forge/ep/dispatch.py:56-115) as a
 * device permutation.  Entries are idx[row, slot] (row-major, `slots` per row).
 * Within a row, repeats of a group id are merged into the first occurrence and
 * their weights summed (sparse_experts.py:52-55).  With SB_GROUP_POSITIVE_ONLY
 * an entry whose summed weight is <= 0 is dropped (dispatch.py:94).  Groups
 * are laid out in ascending id, each with its rows in ascending order, so the
 * permutation is identical to the reference plan.
 * Outputs: offsets[G+1]; for permuted position p < offsets[G]: perm_row[p]
 * (token row), perm_slot[p] (row*slots+slot of the first occurrence),
 * perm_w[p] (summed weight; w may be NULL -> 1); inv[row*slots+slot] = p or -1.
 * Group ids outside [0, G) are skipped (expert-parallel ranks pass ids already
 * mapped to local experts, -1 for remote ones). */
SB_API size_t sb_group_workspace_bytes(int n_rows, int slots, int num_groups);
SB_API int sb_group(const int32_t* idx, const float* w, int n_rows, int slots, int num_groups,
                    int flags, int32_t* offsets, int32_t* perm_row, int32_t* perm_slot,
                    float* perm_w, int32_t* inv, void* workspace, size_t workspace_bytes,
                    void* stream);

/* No reference counterpart: the grouping of sb_group for callers that cannot
 * allocate device memory -- a thin C / ctypes / cgo binding that only forwards
 * pointers it was given and owns no GPU allocator, or a host process whose
 * device memory is all reserved up front by another allocator's pool.
 * Same arguments and results as sb_group, without the workspace: its scratch
 * is a fixed device array of SB_GROUP_NOALLOC_MAX_ENTRIES entries (n_rows *
 * slots) inside the library, held on every device that loads the library until
 * the process exits.  Larger inputs return SB_ERR_WORKSPACE.  All calls on a
 * device share the array (it keeps the last call's contents; nothing in it has
 * to start at zero), so calls whose kernels can overlap on the GPU race.  The
 * first call on a device looks up the array's address (cudaGetSymbolAddress,
 * with that device current) and should come before any stream capture.  The
 * address is cached per device ordinal for the life of the process: it assumes
 * the CUDA runtime's primary context and no cudaDeviceReset afterwards.
 * Nothing is allocated. */
#define SB_GROUP_NOALLOC_MAX_ENTRIES 65536
SB_API int sb_group_noalloc(const int32_t* idx, const float* w, int n_rows, int slots, int num_groups,
                            int flags, int32_t* offsets, int32_t* perm_row, int32_t* perm_slot,
                            float* perm_w, int32_t* inv, void* stream);

/* dst[p, :] = src[perm_row[p], :] for p < offsets[num_groups] (rows of `cols` elements). */
SB_API int sb_gather_rows(const void* src, int act_dtype, int cols, const int32_t* perm_row,
                          const int32_t* offsets, int num_groups, int max_rows, void* dst,
                          void* stream);

/* ------------------------------------------------------------------ grouped GEMM
 * Replaces spider_expert_grouped_gemm_f32/_f16 (spider_kernels.h:89-97) and
 * spider_cuda_expert_grouped_gemm_v2_f32 (spider_cuda.h:22-26).  For every
 * group g and permuted row r in [offsets[g], offsets[g+1]):
 *   acc[r, m] = sum_k A_g[m, k] * x[r, k],  A_g = rows g*a_group_rows + [0, m_rows) of a
 * followed by the epilogue.  Weights (a) are K-major [rows, lda] in wfmt; x is
 * [x_rows, ldx] in act_dtype.  With splits > 1 (SB_EPI_LINEAR only) split s
 * covers k in [s*k/splits, (s+1)*k/splits) and writes out + s*split_stride;
 * only split 0 adds the bias. */
typedef struct sb_grouped_gemm_args {
  int engine;             /* SB_ENGINE_* */
  int wfmt;               /* SB_W_* */
  int act_dtype;          /* SB_F32 / SB_BF16 (x and GELU/SwiGLU outputs) */
  int epilogue;           /* SB_EPI_* */
  int num_groups;
  int m_rows;             /* output features per group */
  int k;                  /* reduction length */
  int group_size;         /* int4 group size along k */
  int64_t a_group_rows;   /* row offset between groups in a */
  int64_t lda;            /* elements per row of a (bytes per row = lda/2 for int4) */
  int64_t a_rows_total;   /* rows of a (bounds of the weight tensor) */
  const void* a;
  const void* a_scale;    /* fp8: float[a_rows_total]; int4: bf16[a_rows_total, lda/group_size];
                             bf16: NULL, or float[a_rows_total] row scales applied to the accumulator
                             (fp8 weights converted to bf16 exactly keep their per-channel scale) */
  const void* a_gate;     /* SwiGLU gate weights, same layout as a */
  const void* a_gate_scale;
  const float* bias;      /* bias[g*bias_group_stride + m], may be NULL */
  const float* bias_gate;
  int64_t bias_group_stride;
  const void* x;
  int64_t ldx;
  /* Optional gather: when x_row_index is not NULL, permuted row r of the B
   * operand is row x_row_index[r] of x (x then has x_rows rows); otherwise x
   * holds the permuted rows themselves. */
  const int32_t* x_row_index;
  int x_rows;
  int max_rows;           /* rows allocated in x / out (upper bound of offsets[G]) */
  int rows_hint;          /* host estimate of offsets[G] (tile shape choice only) */
  int group_rows_bound;   /* rows per group the tile is planned for: an upper bound, or 0 if unknown
                             (tile choice only; larger groups are still computed correctly) */
  const int32_t* offsets; /* [G+1] device; NULL with num_groups == 1: one group of all max_rows rows */
  const float* row_scale; /* [max_rows] per permuted row, SB_EPI_LINEAR only, may be NULL */
  void* out;
  int64_t ldo;
  int splits;
  int64_t split_stride;
  int* status;            /* device status word (may be NULL) */
} sb_grouped_gemm_args;

SB_API int sb_grouped_gemm(const sb_grouped_gemm_args* args, void* stream);

/* ------------------------------------------------------------------ edge top-M
 * Replaces spider_edge_topk_f32 (spider_kernels.h:58-60; scalar_phase1_2.cpp:
 * 11-47) and model.py:264-266 for the rows the router selected: for permuted
 * row p (a (token, source) pair) take logits[p, 0:E], top-M (descending,
 * equal values -> smaller destination first), softmax over the M values;
 * write edge_idx[perm_slot[p]*M + m], edge_w[...]. */
SB_API int sb_edge_topm(const float* logits, int64_t ld, int num_experts, int edges,
                        const int32_t* perm_slot, const int32_t* offsets, int num_groups,
                        int max_rows, int32_t* edge_idx, float* edge_w, void* stream);

/* ------------------------------------------------------------------ combines
 * Row combine: out[t, :] = sum_{j<slots, inv[t*slots+j]>=0} sum_s y[s][inv[t*slots+j], :]
 * (fixed ascending order, no atomics; slots <= 64, splits <= 8).  out_f32 may be NULL.  If scatter_out is
 * not NULL the combined row is also written there in act_dtype: to rows
 * scatter_inv[t*scatter_slots+k] >= 0, or to row t when scatter_inv is NULL. */
SB_API int sb_combine_rows(const float* y, int64_t ldy, int splits, int64_t split_stride,
                           const int32_t* inv, int slots, int n_tokens, int cols, float* out_f32,
                           const int32_t* scatter_inv, int scatter_slots, void* scatter_out,
                           int act_dtype, void* stream);

/* Loop epilogue, replaces spider_loop_epilogue_f32 (spider_kernels.h:99-101)
 * with the block's LayerNorm (model.py:317):
 *   u = (h + alpha * delta) + beta * x0,  out = LayerNorm(u) * ln_w + ln_b,
 * where delta[t] = sum over the token's expert rows of y (inv / splits as in
 * sb_combine_rows) or, if y is NULL, the dense delta_in [n_tokens, cols].
 * delta_out (may be NULL) receives the fp32 delta. */
SB_API int sb_combine_ln(const float* y, int64_t ldy, int splits, int64_t split_stride,
                         const int32_t* inv, int slots, const float* delta_in, const void* h,
                         const void* x0, int act_dtype, int n_tokens, int cols, const float* ln_w,
                         const float* ln_b, float alpha, float beta, float eps, void* out,
                         float* delta_out, void* stream);

/* ------------------------------------------------------------------ whole block
 * Replaces spider_moe_loop_step_f32 / spider_cuda_moe_loop_step_f32
 * (spider_kernels.h:113-121, spider_cuda.h:36-45) with the semantics of
 * SpiderMoELayer.forward (model.py:240-317) applied for loops
 * [loop_begin, loop_end) (SpiderWebLM._run_recurrent_full, model.py:445-448). */
typedef struct sb_block_dims {
  int hidden, num_experts, top_k, edges_per_expert, ffn, num_loops;
  int act_dtype;   /* SB_F32 or SB_BF16 (token rows and dense weights) */
  int wfmt;        /* expert weight format */
  int activation;  /* SB_ACT_* */
  int group_size;  /* int4 */
  int engine;      /* SB_ENGINE_* for the grouped GEMMs */
  int max_tokens;
  float residual_scale, reinject, ln_eps;
} sb_block_dims;

typedef struct sb_block_weights {
  const void* router_w;   /* [E, H] act dtype              router.weight           */
  const float* loop_bias; /* [L, E]                         loop_bias               */
  const void* gen_w;      /* [E*E, H] act dtype             edge_generator.weight[:, :H] */
  const float* gen_bias;  /* [L, E*E] edge_generator.bias + weight[:, H:] . loop_embedding[l] */
  const void* edge_w;     /* [E, H, H] act dtype            edge_value.{d}.weight   */
  const void* w_up;   const void* s_up;   const float* b_up;   /* [E, U, H] */
  /* SB_ACT_SWIGLU: w_up / s_up / b_up hold the gate and up projections
   * interleaved as SB_EPI_SWIGLU_IL describes ([E, 2U, H]); the w_gate fields
   * are not used and may be NULL. */
  const void* w_gate; const void* s_gate; const float* b_gate;
  const void* w_down; const void* s_down; const float* b_down; /* [E, H, U] */
  const float* ln_w;  const float* ln_b;                       /* norm.{weight,bias} */
  /* Optional [E + E*E, H] act dtype: the router rows followed by gen_w's rows
   * in one buffer (router_w == route_w and gen_w == route_w + E*H then).  Given
   * it, large batches compute every router and edge logit in one GEMM (the
   * dense edge-generator product model.py:261-263 forms) instead of grouping
   * tokens by selected source; NULL keeps the grouped route. */
  const void* route_w;
} sb_block_weights;

/* Optional copies of the last executed loop's intermediates (any may be NULL). */
typedef struct sb_block_taps {
  int32_t* top_idx;     /* [n, K]     */
  float* top_w;         /* [n, K]     */
  int32_t* edge_idx;    /* [n, K, M]  (for each selected source, in router slot order) */
  float* edge_w;        /* [n, K, M]  */
  float* messages;      /* [n, H] fp32 */
  float* delta;         /* [n, H] fp32 */
  int32_t* ffn_offsets; /* [E+1]      */
  int32_t* ffn_rows;    /* [n*K]      */
  float* ffn_weights;   /* [n*K]      */
} sb_block_taps;

SB_API size_t sb_block_workspace_bytes(const sb_block_dims* dims);
SB_API int sb_block_forward(const sb_block_dims* dims, const sb_block_weights* w, const void* h_in,
                            const void* x0, void* h_out, int n_tokens, int loop_begin,
                            int loop_end, void* workspace, size_t workspace_bytes,
                            const sb_block_taps* taps, void* stream);

/* ------------------------------------------------------------------ loop statistics
 * Replaces the return_stats=True tail of SpiderMoELayer.forward
 * (spider_moe/model.py:327-343) for loop loop_idx: h_in [n, H] is the loop's
 * input, h_out [n, H] its output (both dims->act_dtype), top_idx [n, K] the
 * loop's routing (NULL: recomputed here).  Writes router_probs [n, E] fp32,
 * confidence [n] = sigmoid(h_out . exit_w + exit_b[0]) (exit_w fp32 [H], exit_b
 * fp32 [1], both device memory; pass
 * h_out and confidence both NULL to skip it) and
 * stats [3E + 2] fp32 = expert_load[E] | edge_load[E] | edge_importance[E] |
 * aux_loss | edge_loss, the edge histograms taken over the top-M destinations
 * of ALL E sources as the reference does.  Workspace status word at offset 0. */
SB_API size_t sb_loop_stats_workspace_bytes(const sb_block_dims* dims, int n_tokens);
SB_API int sb_loop_stats(const sb_block_dims* dims, const sb_block_weights* w, int loop_idx,
                         const void* h_in, const void* h_out, const int32_t* top_idx, int n_tokens,
                         const float* exit_w, const float* exit_b, float* router_probs, float* confidence,
                         float* stats, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------ early-exit active set
 * One step of the early-exit decode loop SpiderWebLM._run_recurrent_decode
 * (spider_moe/model.py:462-472) with the ActiveSet primitives
 * (spider_moe/active_set.py: drop, compact_active, scatter_active).  h_new
 * [n_active, positions, hidden] is loop l's output for the active batch rows
 * act_idx [n_active] (ascending), x0c [n_active, positions, hidden] their block
 * inputs.  confidence[r] = sigmoid(h_new[r, 0, :] . exit_w + exit_b[0])
 * (exit_w fp32 [hidden], exit_b fp32 [1]); row r leaves when confidence >
 * threshold.  Writes h_full[act_idx[r]] = h_new[r] for every r, and for the
 * rows that stay, in order: act_next, h_next and x0_next (the next loop's
 * compact inputs) and *n_next (device int32).  flags: scratch of n_active
 * int32; confidence [n_active] optional.  h_next / x0_next / h_full must not
 * overlap h_new / x0c.  Row pointers 16-byte aligned. */
SB_API int sb_active_set_step(int act_dtype, int n_active, int positions, int hidden, const void* h_new,
                              const void* x0c, const int32_t* act_idx, const float* exit_w,
                              const float* exit_b, float threshold, void* h_full, int32_t* act_next,
                              void* h_next, void* x0_next, int32_t* n_next, int32_t* flags,
                              float* confidence, void* stream);

/* ------------------------------------------------------------------ Lumen workspace
 * Replaces LumenWorkspace.forward (spider_moe/lumen.py:81-123), applied by
 * SpiderMoELayer.forward after its LayerNorm (model.py:318-323) when
 * cfg.use_lumen: scores = W_q h + slot_bias, w = softmax(scores), values =
 * W_v h, raw = W_o ((sum_s w_s^2) values), gate = sigmoid(gate . [h ; raw] +
 * gate_bias), out = LayerNorm(h + gate raw).  wqv stacks write_q.weight [S, H]
 * over write_v.weight [D, H] (act dtype), qv_bias = slot_bias then D zeros
 * (fp32), w_o = slot_to_h.weight [H, D] (act dtype), gate_w = gate.weight
 * [2H] fp32, gate_b [1] fp32, ln_w / ln_b = norm [H] fp32.  Optional outputs
 * (NULL to skip): slot_weights [n, S], values [n, D], broadcast = gate raw
 * [n, H] and its L2 norm [n], all fp32.  1 <= S <= 32. */
typedef struct sb_lumen_weights {
  const void* wqv;
  const float* qv_bias;
  const void* w_o;
  const float* gate_w;
  const float* gate_b;
  const float* ln_w;
  const float* ln_b;
  float ln_eps;
} sb_lumen_weights;

SB_API size_t sb_lumen_workspace_bytes(int n_tokens, int hidden, int slots, int slot_dim);
SB_API int sb_lumen_forward(int act_dtype, int engine, int n_tokens, int hidden, int slots, int slot_dim,
                            const sb_lumen_weights* w, const void* h, void* out, float* slot_weights,
                            float* values, float* broadcast, float* broadcast_norm, void* workspace,
                            size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------ Dobu expert offload
 * Helpers of the offload store (spider_moe/expert_store.py:120-166), whose
 * experts live in host memory with a few resident in device slots.
 * sb_active_experts: active[e] = 1 when some token's summed routing weight for
 * e is positive (the experts the reference materialises), else 0.
 * sb_remap_routes: routing rewritten onto device slots: idx_out = slot_of[e],
 * w_out = w where slot_of[e] >= 0, else slot 0 with weight 0 (dropped by the
 * positive-only grouping), so sb_expert_delta over the slots computes the
 * experts of one wave. */
SB_API int sb_active_experts(const int32_t* top_idx, const float* top_w, int n_tokens, int top_k,
                             int num_experts, int32_t* active, void* stream);
SB_API int sb_remap_routes(const int32_t* top_idx, const float* top_w, int n_tokens, int top_k,
                           const int32_t* slot_of, int num_experts, int32_t* idx_out, float* w_out,
                           void* stream);

/* ------------------------------------------------------------------ sparse expert delta
 * Replaces sparse_expert_delta (spider_moe/sparse_experts.py:11-68) for one
 * rank: delta[t] = sum over the token's experts e in [0, E) with e % world ==
 * rank of tw * ffn_e(messages[t]) (no cross-rank reduction; the caller
 * all-reduces as expert_parallel.all_reduce_sum_ does). */
SB_API size_t sb_expert_delta_workspace_bytes(const sb_block_dims* dims, int n_tokens);
SB_API int sb_expert_delta(const sb_block_dims* dims, const sb_block_weights* w,
                           const void* messages, const int32_t* top_idx, const float* top_w,
                           int n_tokens, int rank, int world, float* delta, void* workspace,
                           size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------ expert parallel
 * Token-sharded expert parallelism.  Each rank routes its own tokens
 * (sb_block_route), sends each token's message row once to every rank owning
 * one of its experts (owner = e % world, spider_moe/expert_parallel.py:29-30)
 * with a fixed-capacity all-to-all, the owners run their experts
 * (sb_expert_delta on the received rows, local expert ids), the results come
 * back with a second all-to-all and sb_combine_ln sums them (inv = ret_pos).
 *
 * sb_block_route replaces the router + graph part of SpiderMoELayer.forward
 * (model.py:254-288) for loop loop_idx: messages [n, H] in act dtype (and
 * optionally fp32), top_idx / top_w [n, K].  Uses the sb_block_forward
 * workspace; needs no expert weights. */
SB_API int sb_block_route(const sb_block_dims* dims, const sb_block_weights* w, const void* h, int n_tokens,
                          int loop_idx, void* messages, float* messages_f32, int32_t* top_idx, float* top_w,
                          void* workspace, size_t workspace_bytes, void* stream);

/* Dispatch packing (no reference counterpart; the reference all-reduces the
 * full delta instead, expert_parallel.py:33-37).  send [world, cap] rows of
 * sb_ep_row_pitch() bytes: [message row (hidden x act dtype) | K int32 | K fp32].
 * Row (q, j) is the j-th token (ascending) that owner q must see, with q's
 * local expert id per slot (-1: not q's expert, or an unused row) and the
 * routing weight.  ret_pos [n, K]: position q*cap + j of the returned combined
 * row for the first slot of each owner, else -1.  cap >= n_tokens. */
SB_API size_t sb_ep_row_pitch(int hidden, int act_dtype, int top_k);
SB_API size_t sb_ep_pack_workspace_bytes(int n_tokens, int top_k, int world);
SB_API int sb_ep_pack(const int32_t* top_idx, const float* top_w, const void* messages, int act_dtype,
                      int n_tokens, int hidden, int top_k, int num_experts, int world, int cap, void* send,
                      int32_t* ret_pos, void* workspace, size_t workspace_bytes, void* stream);

/* Peer-memory exchange of the same rows (no reference counterpart: it replaces
 * the all-to-all pair of the token-sharded step with stores into the peers'
 * memory over NVLink).  Each rank owns one region of sb_ep_peer_region_bytes():
 * recv rows [world][cap][row_pitch] | returned rows [world][cap][hidden] fp32 at
 * the next 256-byte boundary | flags.  sb_ep_peer_create allocates and zeroes it
 * (cudaMalloc: set-up only, never on the per-step path) and writes its 64-byte
 * CUDA IPC handle; every rank maps the others' handles with sb_ep_peer_map.
 * `regions` is a DEVICE array of world region pointers as mapped in this process
 * (its own region at index rank).
 *   sb_ep_dispatch: sb_ep_pack, but row (q, j) goes straight to rank q's recv
 *     row [rank][j], then rank's dispatch flag is raised in every region.
 *   sb_ep_wait(kind 0 dispatch / 1 return): waits (on the device, bounded: about
 *     2 s, then SB_DEVERR_PEER_WAIT in *status) until every rank has raised this
 *     rank's flag once more than this rank has waited before.
 *   sb_ep_return: rows [q][cap][hidden] of this owner's results to rank q's
 *     returned rows [rank][cap], then the return flag is raised in every region.
 * One step per loop: dispatch -> wait(0) -> sb_expert_rows on the recv rows ->
 * return -> wait(1) -> sb_combine_ln on the returned rows with ret_pos.  All
 * ranks must take the same steps; regions must not be shared between blocks. */
SB_API size_t sb_ep_peer_region_bytes(int world, int cap, int64_t row_pitch, int hidden);
SB_API int sb_ep_peer_create(int world, int cap, int64_t row_pitch, int hidden, void** region, void* ipc_handle);
SB_API int sb_ep_peer_map(const void* ipc_handle, void** region);
SB_API int sb_ep_peer_unmap(void* region);
SB_API int sb_ep_peer_destroy(void* region);
SB_API int sb_ep_dispatch(const int32_t* top_idx, const float* top_w, const void* messages, int act_dtype,
                          int n_tokens, int hidden, int top_k, int num_experts, int world, int rank, int cap,
                          void* const* regions, int32_t* ret_pos, void* workspace, size_t workspace_bytes,
                          void* stream);
SB_API int sb_ep_wait(void* region, int world, int cap, int64_t row_pitch, int hidden, int kind, int* status,
                      void* stream);
SB_API int sb_ep_return(const float* rows_out, int world, int rank, int cap, int64_t row_pitch, int hidden,
                        void* const* regions, void* stream);
/* The same step with the waits and the return inside the neighbouring kernels:
 *   sb_expert_rows_peer = sb_ep_wait(kind 0) + sb_expert_rows on the region's
 *     receive rows (world * cap rows) + sb_ep_return of the results;
 *   sb_ep_epilogue_peer = sb_ep_wait(kind 1) + sb_combine_ln of the region's
 *     returned rows with ret_pos (slots = top_k). */
SB_API int sb_expert_rows_peer(const sb_block_dims* dims, const sb_block_weights* w, void* region,
                               void* const* regions, int world, int rank, int cap, int64_t row_pitch,
                               int expected_pairs, int* status, void* workspace, size_t workspace_bytes,
                               void* stream);
SB_API int sb_ep_epilogue_peer(void* region, int world, int cap, int64_t row_pitch, const int32_t* ret_pos,
                               int top_k, const void* h, const void* x0, int act_dtype, int n_tokens, int hidden,
                               const float* ln_w, const float* ln_b, float alpha, float beta, float eps, void* out,
                               int* status, void* stream);

/* Owner side: rows in the packed layout above (n_rows of row_pitch bytes, ids
 * are local expert ids in [0, dims->num_experts)); out[r] = sum over the row's
 * slots of w * ffn_id(row message), fp32 [n_rows, hidden].  The expert part of
 * sparse_expert_delta (sparse_experts.py:51-63) for received rows.
 * expected_pairs (0: n_rows * K) is the number of (row, expert) pairs the caller
 * expects -- most received rows are padding -- and only steers tile shapes. */
SB_API size_t sb_expert_rows_workspace_bytes(const sb_block_dims* dims, int n_rows);
SB_API int sb_expert_rows(const sb_block_dims* dims, const sb_block_weights* w, const void* rows,
                          int64_t row_pitch, int n_rows, int expected_pairs, float* out, void* workspace,
                          size_t workspace_bytes, void* stream);

/* Byte offset of the device status word inside every workspace above. */
SB_API size_t sb_status_offset(void);

/* Bits kernels OR into a device status word.  Every wait on the device (an
 * mbarrier of the TMA / MMA pipeline, a peer rank's exchange flag) gives up
 * after about 2 s of %globaltimer time, records its bit, lets its own copies
 * in flight land and returns, so a lost arrival or a dead peer leaves an error
 * the host reads (SB_ERR_DEVICE_STATUS) instead of a hung GPU. */
enum {
  SB_DEVERR_TMA_WAIT = 1 << 0,  /* producer / consumer gave up on a TMA barrier */
  SB_DEVERR_MMA_WAIT = 1 << 1,  /* gave up on an MMA-completion barrier */
  SB_DEVERR_CONV_WAIT = 1 << 2, /* gave up on the weight-dequant barrier */
  SB_DEVERR_EPI_WAIT = 1 << 3,  /* epilogue gave up on the accumulator barrier */
  SB_DEVERR_BAD_INDEX = 1 << 4, /* an index outside its range was met and skipped */
  SB_DEVERR_DRAIN = 1 << 5,     /* in-flight copies not drained before exit */
  SB_DEVERR_PEER_WAIT = 1 << 6  /* gave up waiting for a peer rank's exchange flag */
};

/* ------------------------------------------------------------------ profiling aid
 * Per-stage CUDA-event timing of sb_block_forward (no reference counterpart;
 * off by default and not for use during stream capture).  sb_stage_timing(1)
 * clears and starts collecting; sb_stage_timing_read synchronises the
 * recorded events and returns, per stage, the summed milliseconds and the
 * number of launches (arrays of at least sb_num_stages() entries). */
SB_API int sb_num_stages(void);
SB_API const char* sb_stage_name(int stage);
SB_API int sb_stage_timing(int enable);
SB_API int sb_stage_timing_read(double* ms, int* launches, int n_stages);

/* Kernel launches this library has enqueued since it was loaded, counting
 * those recorded into a CUDA graph during stream capture (no reference
 * counterpart): the difference around one captured forward is the number of
 * kernels each replay runs. */
SB_API unsigned long long sb_kernel_launches(void);

#ifdef __cplusplus
}
#endif
#endif /* SPIDER_B200_H */
