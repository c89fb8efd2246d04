// Loop statistics of SpiderMoELayer.forward(..., return_stats=True)
// (spider_moe/model.py:327-343).
//
// The reference histograms the top-M destinations of ALL E source experts
// (edge_indices [B,T,E,M], model.py:265, 329-333), not only the K routed
// sources the block itself needs, so the statistics pass recomputes the full
// edge logits [N, E*E] (a one-group GEMM, issued by sb_loop_stats) and then:
//
//   loop_stats_kernel      one CTA per token stride: warps take (token, source)
//                          rows, select the top-M destinations with the block's
//                          own selection code and histogram them (count and
//                          summed softmax weight) in shared memory; warp 0 adds
//                          the token's router probabilities and its K routed
//                          experts; the last warp computes the exit-head
//                          confidence sigmoid(h_out . w + b).  Per-CTA
//                          counts are flushed with one integer atomic per
//                          bin, per-CTA float sums stored as partials.
//   loop_stats_finish_kernel  one CTA: the partials summed in CTA order, the
//                          normalisations and both losses.
//
// Counts are exact and the float sums have a fixed order, so the statistics
// are bitwise repeatable.
#include "sb_common.cuh"
#include "sb_route_dev.cuh"
#include "sb_internal.h"

namespace sb {

constexpr int kStatsWarps = 8;

template <typename T>
__global__ void __launch_bounds__(kStatsWarps * 32)
loop_stats_kernel(const float* __restrict__ elog, const float* __restrict__ probs,
                  const int32_t* __restrict__ top_idx, const T* __restrict__ h_out,
                  const float* __restrict__ exit_w, const float* __restrict__ exit_b, int N, int H, int E, int K, int M,
                  float* __restrict__ confidence, LoopStatsAcc acc) {
  // per-warp histograms: a warp's M selected destinations are distinct, so its
  // lanes never update one bin at once and each bin sees a fixed order
  __shared__ float s_imp[kStatsWarps][kRouterMaxE];
  __shared__ uint32_t s_ecnt[kStatsWarps][kRouterMaxE];
  __shared__ float s_psum[kRouterMaxE];
  __shared__ uint32_t s_cnt[kRouterMaxE];
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int e = lane; e < E; e += 32) {
    s_imp[warp][e] = 0.f;
    s_ecnt[warp][e] = 0u;
  }
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    s_psum[e] = 0.f;
    s_cnt[e] = 0u;
  }
  __syncthreads();
  for (int t = blockIdx.x; t < N; t += gridDim.x) {
    const float* row0 = elog + static_cast<int64_t>(t) * E * E;
    for (int s = warp; s < E; s += kStatsWarps) {
      int sel_i;
      float sel_w;
      topm_select(row0 + static_cast<int64_t>(s) * E, E, M, lane, sel_i, sel_w);
      if (lane < M) {
        s_ecnt[warp][sel_i] += 1u;
        s_imp[warp][sel_i] += sel_w;
      }
      __syncwarp();
    }
    if (warp == 0) {
      for (int e = lane; e < E; e += 32) s_psum[e] += probs[static_cast<int64_t>(t) * E + e];
      if (lane < K) atomicAdd(&s_cnt[top_idx[static_cast<int64_t>(t) * K + lane]], 1u);
    } else if (warp == kStatsWarps - 1 && confidence) {
      const T* hr = h_out + static_cast<int64_t>(t) * H;
      float z = 0.f;
      for (int i = lane; i < H; i += 32) z = fmaf(to_f32(hr[i]), exit_w[i], z);
      z = warp_sum(z) + exit_b[0];
      if (lane == 0) confidence[t] = 1.0f / (1.0f + expf(-z));
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    float imp = 0.f;
    uint32_t ecnt = 0u;
#pragma unroll
    for (int w = 0; w < kStatsWarps; ++w) {
      imp += s_imp[w][e];
      ecnt += s_ecnt[w][e];
    }
    acc.prob_sum[static_cast<int64_t>(blockIdx.x) * E + e] = s_psum[e];
    acc.importance[static_cast<int64_t>(blockIdx.x) * E + e] = imp;
    if (s_cnt[e]) atomicAdd(&acc.expert_count[e], s_cnt[e]);
    if (ecnt) atomicAdd(&acc.edge_count[e], ecnt);
  }
}

SB_DEVINL float block_sum_256(float v, float* red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = 0.f;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) r += red[w];
  return r;
}

// stats = expert_load[E] | edge_load[E] | edge_importance[E] | aux_loss | edge_loss
// (model.py:328-338).  One CTA of kRouterMaxE threads.
__global__ void __launch_bounds__(kRouterMaxE)
loop_stats_finish_kernel(LoopStatsAcc acc, int parts, int N, int E, float* __restrict__ stats) {
  __shared__ float red[kRouterMaxE / 32];
  pdl_wait();
  pdl_trigger();
  const int e = threadIdx.x;
  const bool in = e < E;
  const float cnt = in ? static_cast<float>(acc.expert_count[e]) : 0.f;
  const float ecnt = in ? static_cast<float>(acc.edge_count[e]) : 0.f;
  float imp = 0.f, psum = 0.f;
  if (in) {
    for (int b = 0; b < parts; ++b) {
      imp += acc.importance[static_cast<int64_t>(b) * E + e];
      psum += acc.prob_sum[static_cast<int64_t>(b) * E + e];
    }
  }
  const float cnt_sum = block_sum_256(cnt, red);
  const float ecnt_sum = block_sum_256(ecnt, red);
  const float imp_sum = block_sum_256(imp, red);
  const float load = cnt / fmaxf(cnt_sum, 1.0f);
  const float eload = ecnt / fmaxf(ecnt_sum, 1.0f);
  const float eimp = imp / fmaxf(imp_sum, 1e-9f);
  // probs.mean(dim=(0, 1)): the sum over tokens / N (NaN for no tokens, as torch)
  const float pmean = in ? psum / static_cast<float>(N) : 0.f;
  const float aux = block_sum_256(in ? load * pmean : 0.f, red);
  const float edge_aux = block_sum_256(in ? eload * eimp : 0.f, red);
  if (in) {
    stats[e] = load;
    stats[E + e] = eload;
    stats[2 * E + e] = eimp;
  }
  if (e == 0) {
    stats[3 * E] = static_cast<float>(E) * aux;
    stats[3 * E + 1] = static_cast<float>(E) * edge_aux;
  }
}

int loop_stats_launch(const float* elog, const float* probs, const int32_t* top_idx, const void* h_out,
                      int act_dtype, const float* exit_w, const float* exit_b, int N, int H, int E, int K, int M,
                      float* confidence, LoopStatsAcc acc, float* stats, cudaStream_t st) {
  int blocks = 0;
  if (N > 0) {
    blocks = N < 4 * current_sm_count() ? N : 4 * current_sm_count();
    if (blocks > kLoopStatsMaxParts) blocks = kLoopStatsMaxParts;
    const dim3 block(kStatsWarps * 32);
    int rc = act_dtype == SB_F32
                 ? launch(loop_stats_kernel<float>, dim3(blocks), block, 0, st, elog, probs, top_idx,
                          static_cast<const float*>(h_out), exit_w, exit_b, N, H, E, K, M, confidence, acc)
                 : launch(loop_stats_kernel<__nv_bfloat16>, dim3(blocks), block, 0, st, elog, probs, top_idx,
                          static_cast<const __nv_bfloat16*>(h_out), exit_w, exit_b, N, H, E, K, M, confidence,
                          acc);
    if (rc) return rc;
  }
  return launch(loop_stats_finish_kernel, dim3(1), dim3(kRouterMaxE), 0, st, acc, blocks, N, E, stats);
}

}  // namespace sb
