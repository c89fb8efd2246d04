// Router and edge top-M kernels (memory-bound, one warp per token / pair).
//
// sb_router follows SpiderMoELayer.forward lines 254-258 (spider_moe/model.py):
//   logits = h . W_r^T + loop_bias[l];  probs = softmax_fp32(logits);
//   top_w, top_idx = topk(probs, K);    top_w /= max(sum(top_w), 1e-9)
// sb_edge_topm follows lines 264-266: top-M of a source's E destination logits,
// then an fp32 softmax over the M selected values.
#include "sb_common.cuh"
#include "sb_route_dev.cuh"
#include "sb_internal.h"

namespace sb {

// One CTA per kRouterTok tokens.  Their hidden rows are staged in shared
// memory; warp w computes the logits of experts w, w+8, ... for all of them,
// four experts (and their weight loads) at a time, so the weight rows are read
// once per CTA and many loads are in flight.  Warps 0..kRouterTok-1 then do the
// softmax and top-k of one token each.
constexpr int kRouterTok = 4;
constexpr int kRouterEPI = 4;  // experts per iteration of a warp

template <typename T>
__global__ void __launch_bounds__(kRouterWarps * 32)
router_kernel(const T* __restrict__ h, int n_tokens, int hidden, const T* __restrict__ wr,
              const float* __restrict__ bias, int E, int K, int32_t* __restrict__ top_idx,
              float* __restrict__ top_w, float* __restrict__ probs_out) {
  extern __shared__ __align__(16) uint8_t router_smem[];
  T* sh = reinterpret_cast<T*>(router_smem);                                       // [kRouterTok][hidden]
  float* slog = reinterpret_cast<float*>(router_smem + kRouterTok * hidden * sizeof(T));  // [kRouterTok][E]
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t0 = blockIdx.x * kRouterTok;
  const int ntok = min(kRouterTok, n_tokens - t0);
  const int nchunks = hidden >> 3;  // 8 elements per 16-byte (bf16) / 32-byte (fp32) chunk
  // stage the token rows (16-byte vectors)
  {
    const int vec_per_row = hidden * static_cast<int>(sizeof(T)) / 16;
    const uint4* src = reinterpret_cast<const uint4*>(h + static_cast<size_t>(t0) * hidden);
    uint4* dst = reinterpret_cast<uint4*>(sh);
    for (int i = threadIdx.x; i < ntok * vec_per_row; i += blockDim.x) dst[i] = src[i];
  }
  __syncthreads();
  for (int e0 = warp * kRouterEPI; e0 < E; e0 += kRouterWarps * kRouterEPI) {
    float acc[kRouterEPI][kRouterTok];
#pragma unroll
    for (int j = 0; j < kRouterEPI; ++j)
#pragma unroll
      for (int t = 0; t < kRouterTok; ++t) acc[j][t] = 0.f;
    for (int c = lane; c < nchunks; c += 32) {
      float wv[kRouterEPI][8];
#pragma unroll
      for (int j = 0; j < kRouterEPI; ++j)
        if (e0 + j < E) Vec8<T>::load(wr + static_cast<size_t>(e0 + j) * hidden + c * 8, wv[j]);
#pragma unroll
      for (int t = 0; t < kRouterTok; ++t) {
        if (t < ntok) {
          float hv[8];
          Vec8<T>::load(sh + t * hidden + c * 8, hv);
#pragma unroll
          for (int j = 0; j < kRouterEPI; ++j)
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[j][t] = fmaf(hv[i], wv[j][i], acc[j][t]);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int j = 0; j < kRouterEPI; ++j)
#pragma unroll
        for (int t = 0; t < kRouterTok; ++t) acc[j][t] += __shfl_xor_sync(0xffffffffu, acc[j][t], o);
    if (lane == 0) {
#pragma unroll
      for (int j = 0; j < kRouterEPI; ++j)
        if (e0 + j < E)
#pragma unroll
          for (int t = 0; t < kRouterTok; ++t) slog[t * E + e0 + j] = acc[j][t] + bias[e0 + j];
    }
  }
  __syncthreads();
  if (warp >= ntok) return;
  int sel_i;
  float sel_w;
  router_select(slog + warp * E, E, K, lane, probs_out ? probs_out + static_cast<size_t>(t0 + warp) * E : nullptr,
                sel_i, sel_w);
  if (lane < K) {
    top_idx[static_cast<size_t>(t0 + warp) * K + lane] = sel_i;
    top_w[static_cast<size_t>(t0 + warp) * K + lane] = sel_w;
  }
}

// Sum over the 32 lanes of 32 values per lane, returned transposed: lane L
// gets the total of v[L].  Five butterfly steps, each halving the values a
// lane keeps (31 shuffles instead of 32 x 5).
SB_DEVINL float warp_transpose_sum32(float (&v)[32], int lane) {
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) {
    const bool upper = lane & d;
#pragma unroll
    for (int i = 0; i < d; ++i) {
      const float send = upper ? v[i] : v[i + d];
      const float keep = upper ? v[i + d] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, d);
    }
  }
  return v[0];
}

// Router for large batches: a CTA stages `tok` (multiple of 8) hidden rows in
// shared memory and reuses every router weight chunk it loads across 8 of
// them; a warp task is 4 experts x 8 tokens (32 fp32 dot products, lanes
// strided over the hidden dimension), reduced with one transpose-sum.  The
// softmax / top-K / renormalisation is router_select, as in router_kernel.
constexpr int kRouterTileMaxTok = 32;

template <typename T>
__global__ void __launch_bounds__(kRouterWarps * 32)
router_tile_kernel(const T* __restrict__ h, int n_tokens, int hidden, int tok, const T* __restrict__ wr,
                   const float* __restrict__ bias, int E, int K, int32_t* __restrict__ top_idx,
                   float* __restrict__ top_w, float* __restrict__ probs_out) {
  extern __shared__ __align__(16) uint8_t tile_smem[];
  T* sh = reinterpret_cast<T*>(tile_smem);                                               // [tok][hidden]
  float* slog = reinterpret_cast<float*>(tile_smem + static_cast<size_t>(tok) * hidden * sizeof(T));  // [tok][E]
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t0 = blockIdx.x * tok;
  const int ntok = min(tok, n_tokens - t0);
  const int nchunks = hidden >> 3;
  {
    const int vec_per_row = hidden * static_cast<int>(sizeof(T)) / 16;
    const uint4* src = reinterpret_cast<const uint4*>(h + static_cast<size_t>(t0) * hidden);
    uint4* dst = reinterpret_cast<uint4*>(sh);
    for (int i = threadIdx.x; i < ntok * vec_per_row; i += blockDim.x) dst[i] = src[i];
  }
  __syncthreads();
  const int e_steps = (E + 3) / 4, t_steps = (ntok + 7) / 8;
  for (int task = warp; task < e_steps * t_steps; task += kRouterWarps) {
    const int e0 = (task % e_steps) * 4, tt0 = (task / e_steps) * 8;
    float acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0.f;
    for (int c = lane; c < nchunks; c += 32) {
      float wv[4][8];
#pragma unroll
      for (int j = 0; j < 4; ++j) Vec8<T>::load(wr + static_cast<size_t>(min(e0 + j, E - 1)) * hidden + c * 8, wv[j]);
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        float hv[8];
        Vec8<T>::load(sh + static_cast<size_t>(min(tt0 + t, ntok - 1)) * hidden + c * 8, hv);
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[j * 8 + t] = fmaf(hv[i], wv[j][i], acc[j * 8 + t]);
      }
    }
    const float sum = warp_transpose_sum32(acc, lane);  // lane = expert j * 8 + token t
    const int e = e0 + (lane >> 3), t = tt0 + (lane & 7);
    if (e < E && t < ntok) slog[t * E + e] = sum + bias[e];
  }
  __syncthreads();
  for (int t = warp; t < ntok; t += kRouterWarps) {
    int sel_i;
    float sel_w;
    router_select(slog + t * E, E, K, lane, probs_out ? probs_out + static_cast<size_t>(t0 + t) * E : nullptr,
                  sel_i, sel_w);
    if (lane < K) {
      top_idx[static_cast<size_t>(t0 + t) * K + lane] = sel_i;
      top_w[static_cast<size_t>(t0 + t) * K + lane] = sel_w;
    }
  }
}

// Softmax / top-K / renormalisation (router_select) of router logits computed
// by the grouped GEMM: one warp per token, the logits the sum of `splits`
// partial rows `split_stride` apart.
__global__ void __launch_bounds__(kRouterWarps * 32)
router_select_kernel(const float* __restrict__ logits, int ld, int splits, int64_t split_stride, int n_tokens, int E,
                     int K, int32_t* __restrict__ top_idx, float* __restrict__ top_w) {
  __shared__ float srow[kRouterWarps][kRouterMaxE];
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kRouterWarps + warp;
  if (t >= n_tokens) return;
  for (int e = lane; e < E; e += 32) {
    float v = 0.f;
    for (int s = 0; s < splits; ++s) v += logits[s * split_stride + t * ld + e];
    srow[warp][e] = v;
  }
  __syncwarp();
  int sel_i;
  float sel_w;
  router_select(srow[warp], E, K, lane, nullptr, sel_i, sel_w);
  if (lane < K) {
    top_idx[t * K + lane] = sel_i;
    top_w[t * K + lane] = sel_w;
  }
}

int router_from_logits(const float* logits, int ld, int splits, int64_t split_stride, int n_tokens, int E, int K,
                       int32_t* top_idx, float* top_w, cudaStream_t st) {
  if (n_tokens <= 0) return SB_OK;
  if (E > kRouterMaxE || K > 32 || K > E) return SB_ERR_ARG;
  return launch(router_select_kernel, dim3((n_tokens + kRouterWarps - 1) / kRouterWarps), dim3(kRouterWarps * 32), 0,
                st, logits, ld, splits, split_stride, n_tokens, E, K, top_idx, top_w);
}

// Router and edge graph of one token per warp from its dense logits row: the
// E router logits (+ loop_bias[l]: softmax, top-K, renormalisation,
// spider_moe/model.py:254-258), then for each selected source s in router
// slot order its E edge logits (columns E + s*E .., + the folded generator
// bias: top-M and softmax, model.py:260-266).  The biases are added in fp32
// after the GEMM's product sum, as F.linear adds them.
// The whole row (E + E*E logits) is loaded into shared memory in one round of
// independent loads, with the biases staged once per CTA, so a token's
// selection waits on one memory latency rather than three dependent ones.
constexpr int kSelectMaxCols = 32 + 32 * 32;  // E <= 32 (the dense route's limit)
__global__ void __launch_bounds__(kRouterWarps * 32)
select_dense_kernel(const float* __restrict__ logits, int64_t ld, int n_tokens, int E, int K, int M,
                    const float* __restrict__ rbias, const float* __restrict__ gbias, int32_t* __restrict__ top_idx,
                    float* __restrict__ top_w, int32_t* __restrict__ edge_idx, float* __restrict__ edge_w) {
  __shared__ float s_bias[kSelectMaxCols];
  __shared__ float s_row[kRouterWarps][kSelectMaxCols];
  const int cols = E + E * E;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) s_bias[c] = c < E ? rbias[c] : gbias[c - E];
  pdl_wait();
  pdl_trigger();
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* srow = s_row[warp];
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * kRouterWarps + warp; t < n_tokens;
       t += static_cast<int64_t>(gridDim.x) * kRouterWarps) {
    const float* row = logits + t * ld;
    for (int c = lane; c < cols; c += 32) srow[c] = row[c] + s_bias[c];
    __syncwarp();
    int sel_i;
    float sel_w;
    router_select(srow, E, K, lane, nullptr, sel_i, sel_w);
    if (lane < K) {
      top_idx[t * K + lane] = sel_i;
      top_w[t * K + lane] = sel_w;
    }
    for (int k = 0; k < K; ++k) {
      const int s = __shfl_sync(0xffffffffu, sel_i, k);
      int m_i;
      float m_w;
      topm_select(srow + E + s * E, E, M, lane, m_i, m_w);
      if (lane < M) {
        edge_idx[(t * K + k) * M + lane] = m_i;
        edge_w[(t * K + k) * M + lane] = m_w;
      }
    }
    __syncwarp();  // every lane done with srow before the next token overwrites it
  }
}

int select_dense(const float* logits, int64_t ld, int n_tokens, int E, int K, int M, const float* rbias,
                 const float* gbias, int32_t* top_idx, float* top_w, int32_t* edge_idx, float* edge_w,
                 cudaStream_t st) {
  if (n_tokens <= 0) return SB_OK;
  if (E > 32 || K > 32 || K > E || M > 32 || M > E || ld < E + static_cast<int64_t>(E) * E) return SB_ERR_ARG;
  int blocks = (n_tokens + kRouterWarps - 1) / kRouterWarps;
  const int cap = 8 * current_sm_count();
  blocks = blocks > cap ? cap : blocks;
  return launch(select_dense_kernel, dim3(blocks), dim3(kRouterWarps * 32), 0, st, logits, ld, n_tokens, E, K, M,
                rbias, gbias, top_idx, top_w, edge_idx, edge_w);
}

// One warp per permuted (token, source) row: top-M over E destination logits.
__global__ void __launch_bounds__(256)
edge_topm_kernel(const float* __restrict__ logits, int64_t ld, int E, int M,
                 const int32_t* __restrict__ perm_slot, const int32_t* __restrict__ offsets,
                 int G, int max_rows, int32_t* __restrict__ edge_idx, float* __restrict__ edge_w) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int rows = min(offsets[G], max_rows);
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
    const int slot = perm_slot[r];
    int sel_i;
    float sel_w;
    topm_select(logits + static_cast<int64_t>(r) * ld, E, M, lane, sel_i, sel_w);
    if (lane < M) {
      edge_idx[static_cast<int64_t>(slot) * M + lane] = sel_i;
      edge_w[static_cast<int64_t>(slot) * M + lane] = sel_w;
    }
  }
}

// Router, edge generator and edge top-M of one token per CTA (route_token).
template <typename T>
__global__ void __launch_bounds__(kRouterWarps * 32)
route_edges_kernel(const T* __restrict__ h, int hidden, const T* __restrict__ wr, const float* __restrict__ rbias,
                   int E, int K, const T* __restrict__ gen_w, const float* __restrict__ gen_bias, int M,
                   int32_t* __restrict__ top_idx, float* __restrict__ top_w, int32_t* __restrict__ edge_idx,
                   float* __restrict__ edge_w) {
  extern __shared__ __align__(16) uint8_t route_smem[];
  T* sh = reinterpret_cast<T*>(route_smem);
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  {
    const int vec_per_row = hidden * static_cast<int>(sizeof(T)) / 16;
    const uint4* src = reinterpret_cast<const uint4*>(h + static_cast<size_t>(t) * hidden);
    uint4* dst = reinterpret_cast<uint4*>(sh);
    for (int i = threadIdx.x; i < vec_per_row; i += blockDim.x) dst[i] = src[i];
  }
  __syncthreads();
  route_token(sh, t, hidden, wr, rbias, E, K, gen_w, gen_bias, M, top_idx, top_w, edge_idx, edge_w, route_smem);
}

size_t route_edges_smem(int act_dtype, int hidden, int E, int K) { return route_smem_bytes(act_dtype, hidden, E, K); }

int route_edges(const void* h, int act_dtype, int n_tokens, int hidden, const void* router_w, const float* rbias,
                int E, int K, const void* gen_w, const float* gen_bias, int M, int32_t* top_idx, float* top_w,
                int32_t* edge_idx, float* edge_w, cudaStream_t st) {
  if (n_tokens <= 0) return SB_OK;
  if (E > kRouterMaxE || K > 32 || M > 32 || K > E || M > E || hidden % 8) return SB_ERR_ARG;
  const size_t smem = route_edges_smem(act_dtype, hidden, E, K);
  if (smem > kRouteEdgesMaxSmem) return SB_ERR_UNSUPPORTED;
  const dim3 grid(n_tokens), block(kRouterWarps * 32);
  if (act_dtype == SB_F32) {
    static bool attr_set = false;
    if (!attr_set) {
      cudaFuncSetAttribute(route_edges_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, kRouteEdgesMaxSmem);
      attr_set = true;
    }
    return launch(route_edges_kernel<float>, grid, block, smem, st, static_cast<const float*>(h), hidden,
                  static_cast<const float*>(router_w), rbias, E, K, static_cast<const float*>(gen_w), gen_bias, M,
                  top_idx, top_w, edge_idx, edge_w);
  }
  if (act_dtype != SB_BF16) return SB_ERR_ARG;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(route_edges_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kRouteEdgesMaxSmem);
    attr_set = true;
  }
  return launch(route_edges_kernel<__nv_bfloat16>, grid, block, smem, st, static_cast<const __nv_bfloat16*>(h),
                hidden, static_cast<const __nv_bfloat16*>(router_w), rbias, E, K,
                static_cast<const __nv_bfloat16*>(gen_w), gen_bias, M, top_idx, top_w, edge_idx, edge_w);
}

}  // namespace sb

using namespace sb;

extern "C" SB_API int sb_router(const void* h, int act_dtype, int n_tokens, int hidden,
                                const void* router_w, const float* loop_bias_l, int num_experts,
                                int top_k, int32_t* top_idx, float* top_w, float* probs,
                                void* stream) {
  if (n_tokens < 0 || hidden <= 0 || hidden % 8 || num_experts <= 0 || num_experts > kRouterMaxE ||
      top_k <= 0 || top_k > num_experts || top_k > 32 || !router_w || !loop_bias_l || !top_idx ||
      !top_w || (n_tokens > 0 && !h))
    return SB_ERR_ARG;
  if (n_tokens == 0) return SB_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int esize = act_dtype == SB_F32 ? 4 : 2;
  if (act_dtype != SB_F32 && act_dtype != SB_BF16) return SB_ERR_ARG;
  const dim3 block(kRouterWarps * 32);
  // Large batches: the tiled kernel (weights reused across 8 staged tokens),
  // as many tokens per CTA (a multiple of 8, <= 32) as 128 KB of rows allow.
  int tile_tok = static_cast<int>((128 * 1024) / (static_cast<size_t>(hidden) * esize)) / 8 * 8;
  tile_tok = tile_tok > kRouterTileMaxTok ? kRouterTileMaxTok : tile_tok;
  if (n_tokens >= 4 * current_sm_count() && tile_tok >= 8) {
    const size_t smem = static_cast<size_t>(tile_tok) * hidden * esize + static_cast<size_t>(tile_tok) * num_experts * 4;
    const dim3 grid((n_tokens + tile_tok - 1) / tile_tok);
    if (act_dtype == SB_F32) {
      static bool attr_set = false;
      if (!attr_set) {
        cudaFuncSetAttribute(router_tile_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        attr_set = true;
      }
      return launch(router_tile_kernel<float>, grid, block, smem, st, static_cast<const float*>(h), n_tokens, hidden,
                    tile_tok, static_cast<const float*>(router_w), loop_bias_l, num_experts, top_k, top_idx, top_w,
                    probs);
    }
    static bool attr_set = false;
    if (!attr_set) {
      cudaFuncSetAttribute(router_tile_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      attr_set = true;
    }
    return launch(router_tile_kernel<__nv_bfloat16>, grid, block, smem, st, static_cast<const __nv_bfloat16*>(h),
                  n_tokens, hidden, tile_tok, static_cast<const __nv_bfloat16*>(router_w), loop_bias_l, num_experts,
                  top_k, top_idx, top_w, probs);
  }
  const dim3 grid((n_tokens + kRouterTok - 1) / kRouterTok);
  const size_t smem = static_cast<size_t>(kRouterTok) * hidden * esize + static_cast<size_t>(kRouterTok) * num_experts * 4;
  if (smem > 200 * 1024) return SB_ERR_UNSUPPORTED;
  int rc = SB_OK;
  if (act_dtype == SB_F32) {
    static bool attr_set = false;
    if (!attr_set && smem > 48 * 1024) {
      cudaFuncSetAttribute(router_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      attr_set = true;
    }
    rc = launch(router_kernel<float>, grid, block, smem, st, static_cast<const float*>(h), n_tokens, hidden,
                static_cast<const float*>(router_w), loop_bias_l, num_experts, top_k, top_idx, top_w, probs);
  } else {
    static bool attr_set = false;
    if (!attr_set && smem > 48 * 1024) {
      cudaFuncSetAttribute(router_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      attr_set = true;
    }
    rc = launch(router_kernel<__nv_bfloat16>, grid, block, smem, st, static_cast<const __nv_bfloat16*>(h), n_tokens,
                hidden, static_cast<const __nv_bfloat16*>(router_w), loop_bias_l, num_experts, top_k, top_idx, top_w,
                probs);
  }
  return rc;
}

extern "C" SB_API int sb_edge_topm(const float* logits, int64_t ld, int num_experts, int edges,
                                   const int32_t* perm_slot, const int32_t* offsets, int num_groups,
                                   int max_rows, int32_t* edge_idx, float* edge_w, void* stream) {
  if (!logits || !perm_slot || !offsets || !edge_idx || !edge_w || num_experts <= 0 ||
      num_experts > kRouterMaxE || edges <= 0 || edges > num_experts || edges > 32 ||
      ld < num_experts || num_groups <= 0 || max_rows < 0)
    return SB_ERR_ARG;
  if (max_rows == 0) return SB_OK;
  // one (token, source) row per warp: rows are independent and short, so
  // more warps in flight rather than a loop per warp
  const int warps = 8;
  const int blocks = (max_rows + warps - 1) / warps;
  return launch(edge_topm_kernel, dim3(blocks), dim3(warps * 32), 0, static_cast<cudaStream_t>(stream), logits, ld,
                num_experts, edges, perm_slot, offsets, num_groups, max_rows, edge_idx, edge_w);
}
