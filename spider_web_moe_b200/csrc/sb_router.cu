// Router and edge top-M kernels (memory-bound, one warp per token / pair).
//
// sb_router follows SpiderMoELayer.forward lines 254-258 (spider_moe/model.py):
//   logits = h . W_r^T + loop_bias[l];  probs = softmax_fp32(logits);
//   top_w, top_idx = topk(probs, K);    top_w /= max(sum(top_w), 1e-9)
// sb_edge_topm follows lines 264-266: top-M of a source's E destination logits,
// then an fp32 softmax over the M selected values.
#include "sb_common.cuh"
#include "sb_internal.h"

namespace sb {

constexpr int kRouterMaxE = 256;          // experts per lane-strided register file (8 per lane)
constexpr int kRouterWarps = 8;

// 16-byte vector of activations converted to 8 fp32 values.
template <typename T> struct Vec8;
template <> struct Vec8<float> {
  static SB_DEVINL void load(const float* p, float* v) {
    float4 a = *reinterpret_cast<const float4*>(p);
    float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
};
template <> struct Vec8<__nv_bfloat16> {
  static SB_DEVINL void load(const __nv_bfloat16* p, float* v) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(h2[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
};

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
  const int token = t0 + warp;
  float logit[kRouterMaxE / 32];
#pragma unroll
  for (int i = 0; i < kRouterMaxE / 32; ++i) logit[i] = (lane + 32 * i < E) ? slog[warp * E + lane + 32 * i] : -INFINITY;
  // fp32 softmax over E (spider_moe/model.py:256).
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < kRouterMaxE / 32; ++i) mx = fmaxf(mx, logit[i]);
  mx = warp_max(mx);
  float p[kRouterMaxE / 32];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kRouterMaxE / 32; ++i) {
    p[i] = (lane + 32 * i < E) ? expf(logit[i] - mx) : 0.f;
    s += p[i];
  }
  s = warp_sum(s);
#pragma unroll
  for (int i = 0; i < kRouterMaxE / 32; ++i) {
    p[i] = p[i] / s;
    if (probs_out && lane + 32 * i < E) probs_out[static_cast<size_t>(token) * E + lane + 32 * i] = p[i];
  }
  // top-K by repeated arg-max (model.py:257); a taken expert is masked with -1
  // (probabilities are >= 0), equal values go to the smaller expert id.
  float sel_w = 0.f, sum_w = 0.f;
  int sel_i = -1;
  for (int k = 0; k < K; ++k) {
    float bv = -1.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kRouterMaxE / 32; ++i) {
      const int e = lane + 32 * i;
      if (e < E && (p[i] > bv || (p[i] == bv && e < bi))) { bv = p[i]; bi = e; }
    }
    warp_argmax(bv, bi);
#pragma unroll
    for (int i = 0; i < kRouterMaxE / 32; ++i)
      if (lane + 32 * i == bi) p[i] = -1.f;
    sum_w += bv;
    if (lane == k) { sel_w = bv; sel_i = bi; }
  }
  // renormalise (model.py:258)
  if (lane < K) {
    top_idx[static_cast<size_t>(token) * K + lane] = sel_i;
    top_w[static_cast<size_t>(token) * K + lane] = sel_w / fmaxf(sum_w, 1e-9f);
  }
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
    float v[kRouterMaxE / 32];
#pragma unroll
    for (int i = 0; i < kRouterMaxE / 32; ++i) {
      const int e = lane + 32 * i;
      v[i] = e < E ? logits[static_cast<int64_t>(r) * ld + e] : -INFINITY;
    }
    const int slot = perm_slot[r];
    uint32_t taken = 0;  // bit i: destination lane + 32*i already selected
    float sel_v = -INFINITY, first = -INFINITY;
    int sel_i = -1;
    for (int m = 0; m < M; ++m) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < kRouterMaxE / 32; ++i) {
        const int e = lane + 32 * i;
        if (e < E && !(taken & (1u << i)) && (bi == 0x7fffffff || v[i] > bv || (v[i] == bv && e < bi))) {
          bv = v[i];
          bi = e;
        }
      }
      warp_argmax(bv, bi);
      if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
      if (m == 0) first = bv;  // the largest selected value
      if (lane == m) { sel_v = bv; sel_i = bi; }
    }
    // softmax over the M selected values (fp32): exp(v - max) / sum.
    float ex = (lane < M) ? expf(sel_v - first) : 0.f;
    const float s = warp_sum(ex);
    if (lane < M) {
      edge_idx[static_cast<int64_t>(slot) * M + lane] = sel_i;
      edge_w[static_cast<int64_t>(slot) * M + lane] = ex / s;
    }
  }
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
  const dim3 grid((n_tokens + kRouterTok - 1) / kRouterTok), block(kRouterWarps * 32);
  const int esize = act_dtype == SB_F32 ? 4 : 2;
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
  } else if (act_dtype == SB_BF16) {
    static bool attr_set = false;
    if (!attr_set && smem > 48 * 1024) {
      cudaFuncSetAttribute(router_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      attr_set = true;
    }
    rc = launch(router_kernel<__nv_bfloat16>, grid, block, smem, st, static_cast<const __nv_bfloat16*>(h), n_tokens,
                hidden, static_cast<const __nv_bfloat16*>(router_w), loop_bias_l, num_experts, top_k, top_idx, top_w,
                probs);
  } else {
    return SB_ERR_ARG;
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
  const int warps = 8;
  int blocks = (max_rows + warps - 1) / warps;
  blocks = blocks > 4 * 148 ? 4 * 148 : blocks;
  return launch(edge_topm_kernel, dim3(blocks), dim3(warps * 32), 0, static_cast<cudaStream_t>(stream), logits, ld,
                num_experts, edges, perm_slot, offsets, num_groups, max_rows, edge_idx, edge_w);
}
