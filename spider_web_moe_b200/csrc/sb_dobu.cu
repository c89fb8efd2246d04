// Dobu expert offload helpers (spider_moe/expert_store.py:120-166).
//
// The offload store keeps expert weights in host memory and a few of them in
// device slots.  Per call it needs (1) which experts some token actually uses
// -- the reference materialises expert e only when a token's summed routing
// weight for e is positive (expert_store.py:146-152) -- and (2) the routing
// rewritten onto device slots for the experts resident in this wave, so the
// grouped expert FFN runs over slots instead of expert ids.
#include "sb_common.cuh"
#include "sb_internal.h"

namespace sb {

// One thread per token: active[e] = 1 when sum_k w_k [idx_k == e] > 0.
__global__ void active_experts_kernel(const int32_t* __restrict__ idx, const float* __restrict__ w, int n, int K,
                                      int E, int32_t* __restrict__ active) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n) return;
  const int32_t* ti = idx + static_cast<int64_t>(t) * K;
  const float* tw = w + static_cast<int64_t>(t) * K;
  for (int k = 0; k < K; ++k) {
    const int e = ti[k];
    if (e < 0 || e >= E) continue;
    bool first = true;  // visit each expert of the token once, at its first slot
    for (int j = 0; j < k; ++j) first = first && ti[j] != e;
    if (!first) continue;
    float s = 0.f;
    for (int j = k; j < K; ++j) s += ti[j] == e ? tw[j] : 0.f;
    if (s > 0.f) active[e] = 1;
  }
}

// idx_out = slot_of[idx] and w_out = w where the expert has a slot in this
// wave; elsewhere slot 0 with weight 0, which the positive-only grouping drops.
__global__ void remap_routes_kernel(const int32_t* __restrict__ idx, const float* __restrict__ w, int64_t entries,
                                    const int32_t* __restrict__ slot_of, int E, int32_t* __restrict__ idx_out,
                                    float* __restrict__ w_out) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < entries;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int e = idx[i];
    const int s = (e >= 0 && e < E) ? slot_of[e] : -1;
    idx_out[i] = s >= 0 ? s : 0;
    w_out[i] = s >= 0 ? w[i] : 0.f;
  }
}

}  // namespace sb

using namespace sb;

extern "C" SB_API int sb_active_experts(const int32_t* top_idx, const float* top_w, int n_tokens, int top_k,
                                        int num_experts, int32_t* active, void* stream) {
  if (n_tokens < 0 || top_k <= 0 || num_experts <= 0 || !active || (n_tokens > 0 && (!top_idx || !top_w)))
    return SB_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = cuda_status(cudaMemsetAsync(active, 0, sizeof(int32_t) * num_experts, st));
  if (rc || n_tokens == 0) return rc;
  return launch(active_experts_kernel, dim3((n_tokens + 255) / 256), dim3(256), 0, st, top_idx, top_w, n_tokens, top_k,
                num_experts, active);
}

extern "C" SB_API int sb_remap_routes(const int32_t* top_idx, const float* top_w, int n_tokens, int top_k,
                                      const int32_t* slot_of, int num_experts, int32_t* idx_out, float* w_out,
                                      void* stream) {
  if (n_tokens < 0 || top_k <= 0 || num_experts <= 0 || !slot_of ||
      (n_tokens > 0 && (!top_idx || !top_w || !idx_out || !w_out)))
    return SB_ERR_ARG;
  if (n_tokens == 0) return SB_OK;
  const int64_t entries = static_cast<int64_t>(n_tokens) * top_k;
  const int blocks = static_cast<int>((entries + 255) / 256 < 4 * current_sm_count() ? (entries + 255) / 256
                                                                                      : 4 * current_sm_count());
  return launch(remap_routes_kernel, dim3(blocks), dim3(256), 0, static_cast<cudaStream_t>(stream), top_idx, top_w,
                entries, slot_of, num_experts, idx_out, w_out);
}
