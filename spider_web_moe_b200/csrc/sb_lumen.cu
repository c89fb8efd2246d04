// Lumen global workspace after the block's LayerNorm (spider_moe/lumen.py:81-123).
//
// Per token h [H]: scores = W_q h + slot_bias [S], w = softmax(scores),
// values = W_v h [D], slots = w (x) values, mixed = sum_s w_s slots_s =
// (sum_s w_s^2) values, raw = W_o mixed, gate = sigmoid(g . [h ; raw] + b),
// out = LayerNorm(h + gate raw).  Because mixed is values scaled by
// c = sum_s w_s^2, the [S, D] slot tensor is never formed: sb_lumen_forward
// (sb_block.cu) runs
//
//   GEMM 1   [W_q ; W_v] h + [slot_bias ; 0]        one group, S + D rows
//   lumen_mix_kernel       warp per token: softmax over the S scores, c, the
//                          values cast to the activation dtype for GEMM 2
//   GEMM 2   c * (W_o values)                       row_scale = c
//   lumen_gate_ln_kernel   warp per token: gate dot over [h ; raw], the gated
//                          residual and the LayerNorm, and the broadcast norm
#include "sb_common.cuh"
#include "sb_internal.h"

namespace sb {

constexpr int kLumenWarps = 8;

template <typename T>
__global__ void __launch_bounds__(kLumenWarps * 32)
lumen_mix_kernel(const float* __restrict__ qv, int n, int S, int D, T* __restrict__ values,
                 float* __restrict__ c_out, float* __restrict__ slot_w, float* __restrict__ values_f32) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * kLumenWarps + (threadIdx.x >> 5);
  if (t >= n) return;
  const float* row = qv + static_cast<int64_t>(t) * (S + D);
  const float s = lane < S ? row[lane] : -INFINITY;
  const float mx = warp_max(s);
  const float e = lane < S ? expf(s - mx) : 0.f;
  const float w = e / warp_sum(e);
  const float c = warp_sum(w * w);
  if (lane < S && slot_w) slot_w[static_cast<int64_t>(t) * S + lane] = w;
  if (lane == 0) c_out[t] = c;
  for (int d = lane; d < D; d += 32) {
    const float v = row[S + d];
    values[static_cast<int64_t>(t) * D + d] = from_f32<T>(v);
    if (values_f32) values_f32[static_cast<int64_t>(t) * D + d] = v;
  }
}

template <typename T>
__global__ void __launch_bounds__(kLumenWarps * 32)
lumen_gate_ln_kernel(const T* __restrict__ h, const float* __restrict__ raw, int n, int H,
                     const float* __restrict__ gate_w, const float* __restrict__ gate_b,
                     const float* __restrict__ ln_w, const float* __restrict__ ln_b, float eps, T* __restrict__ out,
                     float* __restrict__ broadcast, float* __restrict__ bnorm) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * kLumenWarps + (threadIdx.x >> 5);
  if (t >= n) return;
  const T* hr = h + static_cast<int64_t>(t) * H;
  const float* rr = raw + static_cast<int64_t>(t) * H;
  float z = 0.f;
  for (int i = lane; i < H; i += 32) z = fmaf(to_f32(hr[i]), gate_w[i], fmaf(rr[i], gate_w[H + i], z));
  z = warp_sum(z) + gate_b[0];
  const float gate = 1.0f / (1.0f + expf(-z));
  // b = gate * raw and u = h + b are rounded separately, as the reference's
  // two tensor ops, in every pass and whichever outputs are written (no fma
  // contraction that would change u's rounding); mean, then the variance
  // about it (passes over the row, which stays L1/L2-resident)
  float sum = 0.f, sq = 0.f;
  for (int i = lane; i < H; i += 32) {
    const float b = __fmul_rn(gate, rr[i]);
    sum += __fadd_rn(to_f32(hr[i]), b);
    sq = fmaf(b, b, sq);
  }
  const float mean = warp_sum(sum) / static_cast<float>(H);
  if (bnorm) {
    const float nb = sqrtf(warp_sum(sq));
    if (lane == 0) bnorm[t] = nb;
  }
  float var = 0.f;
  for (int i = lane; i < H; i += 32) {
    const float u = __fadd_rn(to_f32(hr[i]), __fmul_rn(gate, rr[i])) - mean;
    var = fmaf(u, u, var);
  }
  const float rstd = rsqrtf(warp_sum(var) / static_cast<float>(H) + eps);
  for (int i = lane; i < H; i += 32) {
    const float b = __fmul_rn(gate, rr[i]);
    const float u = __fadd_rn(to_f32(hr[i]), b);
    out[static_cast<int64_t>(t) * H + i] = from_f32<T>((u - mean) * rstd * ln_w[i] + ln_b[i]);
    if (broadcast) broadcast[static_cast<int64_t>(t) * H + i] = b;
  }
}

int lumen_mix_launch(const float* qv, int n, int S, int D, int act_dtype, void* values, float* c, float* slot_w,
                     float* values_f32, cudaStream_t st) {
  const dim3 grid((n + kLumenWarps - 1) / kLumenWarps), block(kLumenWarps * 32);
  if (act_dtype == SB_F32)
    return launch(lumen_mix_kernel<float>, grid, block, 0, st, qv, n, S, D, static_cast<float*>(values), c, slot_w,
                  values_f32);
  return launch(lumen_mix_kernel<__nv_bfloat16>, grid, block, 0, st, qv, n, S, D,
                static_cast<__nv_bfloat16*>(values), c, slot_w, values_f32);
}

int lumen_gate_ln_launch(const void* h, const float* raw, int n, int H, int act_dtype, const float* gate_w,
                         const float* gate_b, const float* ln_w, const float* ln_b, float eps, void* out,
                         float* broadcast, float* bnorm, cudaStream_t st) {
  const dim3 grid((n + kLumenWarps - 1) / kLumenWarps), block(kLumenWarps * 32);
  if (act_dtype == SB_F32)
    return launch(lumen_gate_ln_kernel<float>, grid, block, 0, st, static_cast<const float*>(h), raw, n, H, gate_w,
                  gate_b, ln_w, ln_b, eps, static_cast<float*>(out), broadcast, bnorm);
  return launch(lumen_gate_ln_kernel<__nv_bfloat16>, grid, block, 0, st, static_cast<const __nv_bfloat16*>(h), raw, n,
                H, gate_w, gate_b, ln_w, ln_b, eps, static_cast<__nv_bfloat16*>(out), broadcast, bnorm);
}

}  // namespace sb
