// Deterministic combines (no float atomics) and the fused loop epilogue.
//
// sb_combine_rows sums, per token, the permuted rows its slots point at: the
// message sum over edges (spider_moe/model.py:287-288) and the expert-output
// scatter-add (combine_tokens, spider_infer/forge/ep/dispatch.py:127-134).
// sb_combine_ln adds the expert delta and applies the block's LayerNorm
// epilogue (model.py:317).
#include "sb_common.cuh"
#include "sb_internal.h"

namespace sb {

constexpr int kCombineThreads = 128;
constexpr int kMaxSlots = 64;

template <typename T>
__global__ void __launch_bounds__(kCombineThreads)
combine_rows_kernel(const float* __restrict__ y, int64_t ldy, int splits, int64_t split_stride,
                    const int32_t* __restrict__ inv, int slots, int cols,
                    float* __restrict__ out_f32, const int32_t* __restrict__ scatter_inv,
                    int scatter_slots, T* __restrict__ scatter_out) {
  __shared__ int s_rows[kMaxSlots];
  __shared__ int s_dst[kMaxSlots];
  const int t = blockIdx.x;
  if (threadIdx.x < slots) s_rows[threadIdx.x] = inv[static_cast<int64_t>(t) * slots + threadIdx.x];
  if (scatter_inv && threadIdx.x < scatter_slots)
    s_dst[threadIdx.x] = scatter_inv[static_cast<int64_t>(t) * scatter_slots + threadIdx.x];
  __syncthreads();
  for (int c = threadIdx.x * 4; c < cols; c += kCombineThreads * 4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < slots; ++j) {
      const int r = s_rows[j];
      if (r < 0) continue;
      for (int s = 0; s < splits; ++s) {
        const float4 v =
            *reinterpret_cast<const float4*>(y + s * split_stride + static_cast<int64_t>(r) * ldy + c);
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      }
    }
    if (out_f32) *reinterpret_cast<float4*>(out_f32 + static_cast<int64_t>(t) * cols + c) = acc;
    if (scatter_inv) {
      for (int k = 0; k < scatter_slots; ++k) {
        const int q = s_dst[k];
        if (q < 0) continue;
        T* o = scatter_out + static_cast<int64_t>(q) * cols + c;
        o[0] = from_f32<T>(acc.x); o[1] = from_f32<T>(acc.y);
        o[2] = from_f32<T>(acc.z); o[3] = from_f32<T>(acc.w);
      }
    }
  }
}

constexpr int kLnThreads = 256;
constexpr int kLnMaxPerThread = 16;  // hidden <= 4096

SB_DEVINL float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = 0.f;
  if (warp == 0) {
    r = lane < (kLnThreads / 32) ? red[lane] : 0.f;
    r = warp_sum(r);
    if (lane == 0) red[0] = r;
  }
  __syncthreads();
  return red[0];
}

template <typename T>
__global__ void __launch_bounds__(kLnThreads)
combine_ln_kernel(const float* __restrict__ y, int64_t ldy, int splits, int64_t split_stride,
                  const int32_t* __restrict__ inv, int slots, const float* __restrict__ delta_in,
                  const T* __restrict__ h, const T* __restrict__ x0, int cols,
                  const float* __restrict__ ln_w, const float* __restrict__ ln_b, float alpha,
                  float beta, float eps, T* __restrict__ out, float* __restrict__ delta_out) {
  __shared__ int s_rows[kMaxSlots];
  __shared__ float red[32];
  const int t = blockIdx.x;
  if (y && threadIdx.x < slots) s_rows[threadIdx.x] = inv[static_cast<int64_t>(t) * slots + threadIdx.x];
  __syncthreads();
  float u[kLnMaxPerThread];
  float local = 0.f;
#pragma unroll
  for (int i = 0; i < kLnMaxPerThread; ++i) {
    const int c = threadIdx.x + i * kLnThreads;
    u[i] = 0.f;
    if (c < cols) {
      float d = 0.f;
      if (y) {
        for (int j = 0; j < slots; ++j) {
          const int r = s_rows[j];
          if (r < 0) continue;
          for (int s = 0; s < splits; ++s) d += y[s * split_stride + static_cast<int64_t>(r) * ldy + c];
        }
      } else {
        d = delta_in[static_cast<int64_t>(t) * cols + c];
      }
      if (delta_out) delta_out[static_cast<int64_t>(t) * cols + c] = d;
      const float hv = to_f32(h[static_cast<int64_t>(t) * cols + c]);
      const float xv = to_f32(x0[static_cast<int64_t>(t) * cols + c]);
      const float a = hv + alpha * d;
      u[i] = a + beta * xv;
      local += u[i];
    }
  }
  const float mean = block_sum(local, red) / static_cast<float>(cols);
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < kLnMaxPerThread; ++i) {
    const int c = threadIdx.x + i * kLnThreads;
    if (c < cols) {
      const float dv = u[i] - mean;
      sq += dv * dv;
    }
  }
  const float var = block_sum(sq, red) / static_cast<float>(cols);
  const float rstd = rsqrtf(var + eps);
#pragma unroll
  for (int i = 0; i < kLnMaxPerThread; ++i) {
    const int c = threadIdx.x + i * kLnThreads;
    if (c < cols)
      out[static_cast<int64_t>(t) * cols + c] = from_f32<T>((u[i] - mean) * rstd * ln_w[c] + ln_b[c]);
  }
}

}  // namespace sb

using namespace sb;

extern "C" SB_API int sb_combine_rows(const float* y, int64_t ldy, int splits, int64_t split_stride,
                                      const int32_t* inv, int slots, int n_tokens, int cols,
                                      float* out_f32, const int32_t* scatter_inv, int scatter_slots,
                                      void* scatter_out, int act_dtype, void* stream) {
  if (n_tokens < 0 || cols <= 0 || cols % 4 || slots <= 0 || slots > kMaxSlots || splits <= 0 ||
      ldy < cols || (ldy % 4) || (split_stride % 4) || (scatter_inv && (scatter_slots <= 0 ||
      scatter_slots > kMaxSlots || !scatter_out)) || (n_tokens > 0 && (!y || !inv)))
    return SB_ERR_ARG;
  if (n_tokens == 0) return SB_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (act_dtype == SB_F32)
    combine_rows_kernel<float><<<n_tokens, kCombineThreads, 0, st>>>(
        y, ldy, splits, split_stride, inv, slots, cols, out_f32, scatter_inv, scatter_slots,
        static_cast<float*>(scatter_out));
  else if (act_dtype == SB_BF16)
    combine_rows_kernel<__nv_bfloat16><<<n_tokens, kCombineThreads, 0, st>>>(
        y, ldy, splits, split_stride, inv, slots, cols, out_f32, scatter_inv, scatter_slots,
        static_cast<__nv_bfloat16*>(scatter_out));
  else
    return SB_ERR_ARG;
  return sb_last_launch_status();
}

extern "C" SB_API int sb_combine_ln(const float* y, int64_t ldy, int splits, int64_t split_stride,
                                    const int32_t* inv, int slots, const float* delta_in,
                                    const void* h, const void* x0, int act_dtype, int n_tokens,
                                    int cols, const float* ln_w, const float* ln_b, float alpha,
                                    float beta, float eps, void* out, float* delta_out,
                                    void* stream) {
  if (n_tokens < 0 || cols <= 0 || cols > kLnThreads * kLnMaxPerThread || !ln_w || !ln_b ||
      (y && (!inv || slots <= 0 || slots > kMaxSlots || splits <= 0 || ldy < cols)) ||
      (!y && !delta_in) || (n_tokens > 0 && (!h || !x0 || !out)))
    return SB_ERR_ARG;
  if (n_tokens == 0) return SB_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (act_dtype == SB_F32)
    combine_ln_kernel<float><<<n_tokens, kLnThreads, 0, st>>>(
        y, ldy, splits, split_stride, inv, slots, delta_in, static_cast<const float*>(h),
        static_cast<const float*>(x0), cols, ln_w, ln_b, alpha, beta, eps, static_cast<float*>(out),
        delta_out);
  else if (act_dtype == SB_BF16)
    combine_ln_kernel<__nv_bfloat16><<<n_tokens, kLnThreads, 0, st>>>(
        y, ldy, splits, split_stride, inv, slots, delta_in, static_cast<const __nv_bfloat16*>(h),
        static_cast<const __nv_bfloat16*>(x0), cols, ln_w, ln_b, alpha, beta, eps,
        static_cast<__nv_bfloat16*>(out), delta_out);
  else
    return SB_ERR_ARG;
  return sb_last_launch_status();
}
