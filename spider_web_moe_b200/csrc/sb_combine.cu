// Deterministic combines (no float atomics) and the fused loop epilogue.
//
// sb_combine_rows sums, per token, the permuted rows its slots point at: the
// message sum over edges (spider_moe/model.py:287-288) and the expert-output
// scatter-add (combine_tokens, spider_infer/forge/ep/dispatch.py:127-134).
// sb_combine_ln adds the expert delta and applies the block's LayerNorm
// epilogue (model.py:317).
#include "sb_common.cuh"
#include "sb_internal.h"
#include "sb_ep_dev.cuh"
#include "sb_route_dev.cuh"

namespace sb {

constexpr int kCombineThreads = 256;

template <typename T> struct Vec4;
template <> struct Vec4<float> {
  static SB_DEVINL float4 load(const float* p) { return *reinterpret_cast<const float4*>(p); }
  static SB_DEVINL void store(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
};
template <> struct Vec4<__nv_bfloat16> {
  static SB_DEVINL float4 load(const __nv_bfloat16* p) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
  }
  static SB_DEVINL void store(__nv_bfloat16* p, float4 v) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t*>(&a);
    u.y = *reinterpret_cast<const uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = u;
  }
};

constexpr int kMaxSlots = 64;
constexpr int kMaxSplits = 8;
constexpr int kMaxTerms = kMaxSlots * kMaxSplits;  // (slot, split) rows summed per token
constexpr int kTermUnroll = 8;                       // row loads in flight per thread

// Offsets (elements from y) of the rows summed for token t, in the fixed
// order (slot ascending, split ascending) every sum of this file uses;
// filled by one warp, returns the count.
SB_DEVINL int build_terms(const int32_t* __restrict__ inv, int64_t t, int slots, int splits, int64_t ldy,
                          int64_t split_stride, int64_t* terms) {
  const int lane = threadIdx.x & 31;
  int n = 0;
  for (int j0 = 0; j0 < slots; j0 += 32) {
    const int j = j0 + lane;
    const int r = j < slots ? inv[t * slots + j] : -1;
    const unsigned valid = __ballot_sync(0xffffffffu, r >= 0);
    const int before = __popc(valid & ((1u << lane) - 1u));
    if (r >= 0)
      for (int s = 0; s < splits; ++s) terms[(n + before) * splits + s] = s * split_stride + static_cast<int64_t>(r) * ldy;
    n += __popc(valid);
  }
  return n * splits;
}

// acc += y[terms[e] + c] for e in order, kTermUnroll loads issued before their adds.
SB_DEVINL void sum_terms(const float* __restrict__ y, const int64_t* terms, int n, int c, float4& acc) {
  int e = 0;
  for (; e + kTermUnroll <= n; e += kTermUnroll) {
    float4 v[kTermUnroll];
#pragma unroll
    for (int q = 0; q < kTermUnroll; ++q) v[q] = *reinterpret_cast<const float4*>(y + terms[e + q] + c);
#pragma unroll
    for (int q = 0; q < kTermUnroll; ++q) {
      acc.x += v[q].x; acc.y += v[q].y; acc.z += v[q].z; acc.w += v[q].w;
    }
  }
  for (; e < n; ++e) {
    const float4 v = *reinterpret_cast<const float4*>(y + terms[e] + c);
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
}

// With peer.regions (expert-parallel owner, peer transport) the fp32 row t goes
// to rank q = t / cap's returned row [peer.me][t % cap] instead of out_f32, and
// the last CTA raises the return flags.
template <typename T>
__global__ void __launch_bounds__(kCombineThreads)
combine_rows_kernel(const float* __restrict__ y, int64_t ldy, int splits, int64_t split_stride,
                    const int32_t* __restrict__ inv, int slots, int cols,
                    float* __restrict__ out_f32, const int32_t* __restrict__ scatter_inv,
                    int scatter_slots, T* __restrict__ scatter_out, const EpPeer peer) {
  __shared__ int64_t s_terms[kMaxTerms];
  __shared__ int s_dst[kMaxSlots];
  __shared__ int s_n;
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  if (threadIdx.x < 32) {
    const int n = build_terms(inv, t, slots, splits, ldy, split_stride, s_terms);
    if (threadIdx.x == 0) s_n = n;
  }
  if (scatter_inv && threadIdx.x < scatter_slots)
    s_dst[threadIdx.x] = scatter_inv[static_cast<int64_t>(t) * scatter_slots + threadIdx.x];
  __syncthreads();
  const int n = s_n;
  float* orow = out_f32 ? out_f32 + static_cast<int64_t>(t) * cols : nullptr;
  if (peer.regions) {
    // only rows that summed a term go back: padding rows carry nothing the source reads
    const int q = t / peer.cap, j = t - q * peer.cap;
    orow = n == 0 ? nullptr
                  : reinterpret_cast<float*>(peer.regions[q] + peer.ret_off) +
                        (static_cast<int64_t>(peer.me) * peer.cap + j) * cols;
  }
  for (int c = threadIdx.x * 4; c < cols; c += kCombineThreads * 4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    sum_terms(y, s_terms, n, c, acc);
    if (orow) *reinterpret_cast<float4*>(orow + c) = acc;
    if (scatter_inv) {
      for (int k = 0; k < scatter_slots; ++k) {
        const int q = s_dst[k];
        if (q < 0) continue;
        Vec4<T>::store(scatter_out + static_cast<int64_t>(q) * cols + c, acc);
      }
    } else if (scatter_out) {
      Vec4<T>::store(scatter_out + static_cast<int64_t>(t) * cols + c, acc);
    }
  }
  if (peer.regions) ep_signal_peers(peer.regions, peer.regions[peer.me], peer.ctrl_off, peer.world, peer.me, 1);
}

constexpr int kLnThreads = 256;
constexpr int kLnMaxVec = 4;  // float4 chunks per thread: hidden <= 256*4*4 = 4096

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

// One CTA per token; thread t owns float4 chunks t, t+256, ... of the row.
// With row_copy the output row (rounded to T, as written) is also left in
// shared memory.
template <typename T>
SB_DEVINL void ln_token(const float* __restrict__ y, int64_t ldy, int splits, int64_t split_stride,
                        const int32_t* __restrict__ inv, int slots, const float* __restrict__ delta_in,
                        const T* __restrict__ h, const T* __restrict__ x0, int cols,
                        const float* __restrict__ ln_w, const float* __restrict__ ln_b, float alpha,
                        float beta, float eps, T* __restrict__ out, float* __restrict__ delta_out, T* row_copy) {
  __shared__ float red[32];
  const int64_t t = blockIdx.x;
  const int nvec = cols >> 2;
  float4 u[kLnMaxVec], hv[kLnMaxVec], xv[kLnMaxVec];
#pragma unroll
  for (int i = 0; i < kLnMaxVec; ++i) {
    const int v = threadIdx.x + i * kLnThreads;
    if (v < nvec) {
      hv[i] = Vec4<T>::load(h + t * cols + 4 * v);
      xv[i] = Vec4<T>::load(x0 + t * cols + 4 * v);
    }
  }
  __shared__ int64_t s_terms[kMaxTerms];
  __shared__ int s_n;
  if (y && threadIdx.x < 32) {
    const int n = build_terms(inv, t, slots, splits, ldy, split_stride, s_terms);
    if (threadIdx.x == 0) s_n = n;
  }
  __syncthreads();
  const int nterms = y ? s_n : 0;
  float local = 0.f;
#pragma unroll
  for (int i = 0; i < kLnMaxVec; ++i) {
    const int v = threadIdx.x + i * kLnThreads;
    u[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (v < nvec) {
      float4 d = make_float4(0.f, 0.f, 0.f, 0.f);
      if (y) {
        sum_terms(y, s_terms, nterms, 4 * v, d);
      } else {
        d = *reinterpret_cast<const float4*>(delta_in + t * cols + 4 * v);
      }
      if (delta_out) *reinterpret_cast<float4*>(delta_out + t * cols + 4 * v) = d;
      u[i].x = (hv[i].x + alpha * d.x) + beta * xv[i].x;
      u[i].y = (hv[i].y + alpha * d.y) + beta * xv[i].y;
      u[i].z = (hv[i].z + alpha * d.z) + beta * xv[i].z;
      u[i].w = (hv[i].w + alpha * d.w) + beta * xv[i].w;
      local += (u[i].x + u[i].y) + (u[i].z + u[i].w);
    }
  }
  const float mean = block_sum(local, red) / static_cast<float>(cols);
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < kLnMaxVec; ++i) {
    const int v = threadIdx.x + i * kLnThreads;
    if (v < nvec) {
      const float a = u[i].x - mean, b = u[i].y - mean, c = u[i].z - mean, e = u[i].w - mean;
      sq += (a * a + b * b) + (c * c + e * e);
    }
  }
  const float rstd = rsqrtf(block_sum(sq, red) / static_cast<float>(cols) + eps);
#pragma unroll
  for (int i = 0; i < kLnMaxVec; ++i) {
    const int v = threadIdx.x + i * kLnThreads;
    if (v < nvec) {
      const float4 g = *reinterpret_cast<const float4*>(ln_w + 4 * v);
      const float4 b = *reinterpret_cast<const float4*>(ln_b + 4 * v);
      float4 o;
      o.x = (u[i].x - mean) * rstd * g.x + b.x;
      o.y = (u[i].y - mean) * rstd * g.y + b.y;
      o.z = (u[i].z - mean) * rstd * g.z + b.z;
      o.w = (u[i].w - mean) * rstd * g.w + b.w;
      Vec4<T>::store(out + t * cols + 4 * v, o);
      if (row_copy) Vec4<T>::store(row_copy + 4 * v, o);
    }
  }
}

// With wait_region (expert-parallel source, peer transport) every CTA first
// waits for all ranks' return flags (the rows y points at are being written by
// them), and the last CTA counts the wait.
template <typename T>
__global__ void __launch_bounds__(kLnThreads)
combine_ln_kernel(const float* __restrict__ y, int64_t ldy, int splits, int64_t split_stride,
                  const int32_t* __restrict__ inv, int slots, const float* __restrict__ delta_in,
                  const T* __restrict__ h, const T* __restrict__ x0, int cols,
                  const float* __restrict__ ln_w, const float* __restrict__ ln_b, float alpha,
                  float beta, float eps, T* __restrict__ out, float* __restrict__ delta_out, uint8_t* wait_region,
                  int64_t ctrl_off, int wait_world, int* wait_status) {
  pdl_wait();
  pdl_trigger();
  uint32_t target = 0;
  if (wait_region) {
    target = ep_wait_target(wait_region, ctrl_off, wait_world, 1);
    ep_wait_cta(wait_region, ctrl_off, wait_world, 1, target, wait_status);
  }
  ln_token<T>(y, ldy, splits, split_stride, inv, slots, delta_in, h, x0, cols, ln_w, ln_b, alpha, beta, eps, out,
              delta_out, nullptr);
  if (wait_region) ep_count_wait_multi(wait_region, ctrl_off, wait_world, 1, target);
}

// Decode: the loop's LayerNorm epilogue and the next loop's routing of the
// same token in one CTA -- the new hidden row goes from the LayerNorm straight
// into shared memory for route_token (the values written to `out`).
template <typename T>
__global__ void __launch_bounds__(kLnThreads)
combine_ln_route_kernel(const float* __restrict__ y, int64_t ldy, int splits, int64_t split_stride,
                        const int32_t* __restrict__ inv, int slots, const T* __restrict__ h,
                        const T* __restrict__ x0, int cols, const float* __restrict__ ln_w,
                        const float* __restrict__ ln_b, float alpha, float beta, float eps, T* __restrict__ out,
                        const RouteArgs r) {
  extern __shared__ __align__(16) uint8_t route_smem[];
  T* sh = reinterpret_cast<T*>(route_smem);
  pdl_wait();
  pdl_trigger();
  ln_token<T>(y, ldy, splits, split_stride, inv, slots, nullptr, h, x0, cols, ln_w, ln_b, alpha, beta, eps, out,
              nullptr, sh);
  __syncthreads();
  route_token(sh, static_cast<int>(blockIdx.x), cols, static_cast<const T*>(r.router_w), r.router_bias, r.E, r.K,
              static_cast<const T*>(r.gen_w), r.gen_bias, r.M, r.top_idx, r.top_w, r.edge_idx, r.edge_w, route_smem);
}

// ------------------------------------------------------------------ warp-per-token variants
//
// Large batches: one warp per token (8 per CTA), lane L owning float4 chunks
// L, L+32, ... of the row (NV chunks, cols = 128 NV), every reduction inside
// the warp: no shared memory and no block barriers, and all of a lane's
// loads in flight at once.  The slot indices of a token are loaded by lanes
// 0..slots-1 and broadcast.
constexpr int kWarpRowsPerCta = 8;

// One token's row sum (one warp): lane L owns float4 chunks L, L+32, ...
// With peer.regions (expert-parallel owner, peer transport) row t goes to
// rank q = t / cap's returned row [peer.me][t % cap] instead of out_f32 --
// only rows that summed at least one term: the padding rows of the
// fixed-capacity exchange carry nothing the source reads.
template <typename T, int NV, bool kPeer>
SB_DEVINL void combine_row_warp(const float* __restrict__ y, int64_t ldy, int splits, int64_t split_stride,
                                const int32_t* __restrict__ inv, int slots, int64_t t, int lane,
                                float* __restrict__ out_f32, const int32_t* __restrict__ scatter_inv,
                                int scatter_slots, T* __restrict__ scatter_out, const EpPeer& peer) {
  constexpr int cols = NV * 128;
  const int my_inv0 = lane < slots ? inv[t * slots + lane] : -1;
  const int my_inv1 = lane + 32 < slots ? inv[t * slots + lane + 32] : -1;
  float4 acc[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  int terms = 0;
  for (int j = 0; j < slots; ++j) {
    const int r = __shfl_sync(0xffffffffu, j < 32 ? my_inv0 : my_inv1, j & 31);
    if (r < 0) continue;  // warp-uniform
    if (kPeer) ++terms;
    for (int s = 0; s < splits; ++s) {
      const float* row = y + s * split_stride + static_cast<int64_t>(r) * ldy;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const float4 v = *reinterpret_cast<const float4*>(row + 4 * (lane + 32 * i));
        acc[i].x += v.x; acc[i].y += v.y; acc[i].z += v.z; acc[i].w += v.w;
      }
    }
  }
  if constexpr (kPeer) {
    if (terms == 0) return;  // warp-uniform
    const int q = static_cast<int>(t / peer.cap), jj = static_cast<int>(t - static_cast<int64_t>(q) * peer.cap);
    float* orow = reinterpret_cast<float*>(peer.regions[q] + peer.ret_off) +
                  (static_cast<int64_t>(peer.me) * peer.cap + jj) * cols;
#pragma unroll
    for (int i = 0; i < NV; ++i) *reinterpret_cast<float4*>(orow + 4 * (lane + 32 * i)) = acc[i];
    return;
  }
  if (out_f32)
#pragma unroll
    for (int i = 0; i < NV; ++i) *reinterpret_cast<float4*>(out_f32 + t * cols + 4 * (lane + 32 * i)) = acc[i];
  if (scatter_inv) {
    const int my_q0 = lane < scatter_slots ? scatter_inv[t * scatter_slots + lane] : -1;
    const int my_q1 = lane + 32 < scatter_slots ? scatter_inv[t * scatter_slots + lane + 32] : -1;
    for (int k = 0; k < scatter_slots; ++k) {
      const int q = __shfl_sync(0xffffffffu, k < 32 ? my_q0 : my_q1, k & 31);
      if (q < 0) continue;
#pragma unroll
      for (int i = 0; i < NV; ++i) Vec4<T>::store(scatter_out + static_cast<int64_t>(q) * cols + 4 * (lane + 32 * i), acc[i]);
    }
  } else if (scatter_out) {
#pragma unroll
    for (int i = 0; i < NV; ++i) Vec4<T>::store(scatter_out + t * cols + 4 * (lane + 32 * i), acc[i]);
  }
}

template <typename T, int NV>
__global__ void __launch_bounds__(kWarpRowsPerCta * 32)
combine_rows_warp_kernel(const float* __restrict__ y, int64_t ldy, int splits, int64_t split_stride,
                         const int32_t* __restrict__ inv, int slots, int n_tokens, float* __restrict__ out_f32,
                         const int32_t* __restrict__ scatter_inv, int scatter_slots, T* __restrict__ scatter_out) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kWarpRowsPerCta + (threadIdx.x >> 5);
  if (t >= n_tokens) return;
  combine_row_warp<T, NV, false>(y, ldy, splits, split_stride, inv, slots, t, lane, out_f32, scatter_inv,
                                 scatter_slots, scatter_out, EpPeer{});
}

// Expert-parallel owner, peer transport: the rows go to their sources'
// regions, and the last CTA raises the return flags once every row is stored.
template <int NV>
__global__ void __launch_bounds__(kWarpRowsPerCta * 32)
combine_rows_peer_warp_kernel(const float* __restrict__ y, int64_t ldy, int splits, int64_t split_stride,
                              const int32_t* __restrict__ inv, int slots, int n_tokens, const EpPeer peer) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kWarpRowsPerCta + (threadIdx.x >> 5);
  if (t < n_tokens)
    combine_row_warp<float, NV, true>(y, ldy, splits, split_stride, inv, slots, t, lane, nullptr, nullptr, 0, nullptr,
                                      peer);
  ep_signal_peers(peer.regions, peer.regions[peer.me], peer.ctrl_off, peer.world, peer.me, 1);
}

// One token's delta sum and LayerNorm epilogue (one warp).
template <typename T, int NV>
SB_DEVINL void ln_token_warp(const float* __restrict__ y, int64_t ldy, int splits, int64_t split_stride,
                             const int32_t* __restrict__ inv, int slots, const float* __restrict__ delta_in,
                             const T* __restrict__ h, const T* __restrict__ x0, int64_t t,
                             const float* __restrict__ ln_w, const float* __restrict__ ln_b, float alpha, float beta,
                             float eps, T* __restrict__ out, float* __restrict__ delta_out) {
  const int lane = threadIdx.x & 31;
  constexpr int cols = NV * 128;
  float4 u[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) u[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (y) {
    const int my_inv0 = lane < slots ? inv[t * slots + lane] : -1;
    const int my_inv1 = lane + 32 < slots ? inv[t * slots + lane + 32] : -1;
    for (int j = 0; j < slots; ++j) {
      const int r = __shfl_sync(0xffffffffu, j < 32 ? my_inv0 : my_inv1, j & 31);
      if (r < 0) continue;  // warp-uniform
      for (int s = 0; s < splits; ++s) {
        const float* row = y + s * split_stride + static_cast<int64_t>(r) * ldy;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          const float4 v = *reinterpret_cast<const float4*>(row + 4 * (lane + 32 * i));
          u[i].x += v.x; u[i].y += v.y; u[i].z += v.z; u[i].w += v.w;
        }
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < NV; ++i) u[i] = *reinterpret_cast<const float4*>(delta_in + t * cols + 4 * (lane + 32 * i));
  }
  float local = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = 4 * (lane + 32 * i);
    if (delta_out) *reinterpret_cast<float4*>(delta_out + t * cols + c) = u[i];
    const float4 hv = Vec4<T>::load(h + t * cols + c), xv = Vec4<T>::load(x0 + t * cols + c);
    u[i].x = (hv.x + alpha * u[i].x) + beta * xv.x;
    u[i].y = (hv.y + alpha * u[i].y) + beta * xv.y;
    u[i].z = (hv.z + alpha * u[i].z) + beta * xv.z;
    u[i].w = (hv.w + alpha * u[i].w) + beta * xv.w;
    local += (u[i].x + u[i].y) + (u[i].z + u[i].w);
  }
  const float mean = warp_sum(local) / static_cast<float>(cols);
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const float a = u[i].x - mean, b = u[i].y - mean, c = u[i].z - mean, e = u[i].w - mean;
    sq += (a * a + b * b) + (c * c + e * e);
  }
  const float rstd = rsqrtf(warp_sum(sq) / static_cast<float>(cols) + eps);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = 4 * (lane + 32 * i);
    const float4 g = *reinterpret_cast<const float4*>(ln_w + c);
    const float4 b = *reinterpret_cast<const float4*>(ln_b + c);
    float4 o;
    o.x = (u[i].x - mean) * rstd * g.x + b.x;
    o.y = (u[i].y - mean) * rstd * g.y + b.y;
    o.z = (u[i].z - mean) * rstd * g.z + b.z;
    o.w = (u[i].w - mean) * rstd * g.w + b.w;
    Vec4<T>::store(out + t * cols + c, o);
  }
}


template <typename T, int NV>
__global__ void __launch_bounds__(kWarpRowsPerCta * 32)
combine_ln_warp_kernel(const float* __restrict__ y, int64_t ldy, int splits, int64_t split_stride,
                       const int32_t* __restrict__ inv, int slots, const float* __restrict__ delta_in,
                       const T* __restrict__ h, const T* __restrict__ x0, int n_tokens,
                       const float* __restrict__ ln_w, const float* __restrict__ ln_b, float alpha, float beta,
                       float eps, T* __restrict__ out, float* __restrict__ delta_out) {
  pdl_wait();
  pdl_trigger();
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kWarpRowsPerCta + (threadIdx.x >> 5);
  if (t >= n_tokens) return;
  ln_token_warp<T, NV>(y, ldy, splits, split_stride, inv, slots, delta_in, h, x0, t, ln_w, ln_b, alpha, beta, eps, out,
                       delta_out);
}

// Expert-parallel source, peer transport: every CTA first waits for all
// ranks' return flags, and the last CTA counts the wait.
template <typename T, int NV>
__global__ void __launch_bounds__(kWarpRowsPerCta * 32)
combine_ln_wait_warp_kernel(const float* __restrict__ y, int64_t ldy, const int32_t* __restrict__ inv, int slots,
                            const T* __restrict__ h, const T* __restrict__ x0, int n_tokens,
                            const float* __restrict__ ln_w, const float* __restrict__ ln_b, float alpha, float beta,
                            float eps, T* __restrict__ out, uint8_t* wait_region, int64_t ctrl_off, int wait_world,
                            int* wait_status) {
  pdl_wait();
  pdl_trigger();
  const uint32_t target = ep_wait_target(wait_region, ctrl_off, wait_world, 1);
  ep_wait_cta(wait_region, ctrl_off, wait_world, 1, target, wait_status);
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kWarpRowsPerCta + (threadIdx.x >> 5);
  if (t < n_tokens)
    ln_token_warp<T, NV>(y, ldy, 1, 0, inv, slots, nullptr, h, x0, t, ln_w, ln_b, alpha, beta, eps, out, nullptr);
  ep_count_wait_multi(wait_region, ctrl_off, wait_world, 1, target);
}

}  // namespace sb

using namespace sb;

namespace {
// Warp-per-token variants for large batches (from 512 tokens): cols a
// multiple of 128 up to 2048 (NV float4 chunks per lane).
bool use_warp_rows(int n_tokens, int cols) { return n_tokens >= 512 && cols % 128 == 0 && cols <= 2048; }

template <typename T>
int launch_combine_rows_warp(const float* y, int64_t ldy, int splits, int64_t split_stride, const int32_t* inv,
                             int slots, int n_tokens, int cols, float* out_f32, const int32_t* scatter_inv,
                             int scatter_slots, T* scatter_out, cudaStream_t st) {
  const dim3 grid((n_tokens + kWarpRowsPerCta - 1) / kWarpRowsPerCta), block(kWarpRowsPerCta * 32);
#define SB_ROWS_CASE(NV) \
  case NV: return launch(combine_rows_warp_kernel<T, NV>, grid, block, 0, st, y, ldy, splits, split_stride, inv, \
                         slots, n_tokens, out_f32, scatter_inv, scatter_slots, scatter_out);
  switch (cols / 128) {
    SB_ROWS_CASE(1) SB_ROWS_CASE(2) SB_ROWS_CASE(4) SB_ROWS_CASE(8) SB_ROWS_CASE(16)
    default: return SB_ERR_UNSUPPORTED;
  }
#undef SB_ROWS_CASE
}

int launch_combine_rows_peer_warp(const float* y, int64_t ldy, int splits, int64_t split_stride, const int32_t* inv,
                                  int slots, int n_tokens, int cols, const EpPeer& peer, cudaStream_t st) {
  const dim3 grid((n_tokens + kWarpRowsPerCta - 1) / kWarpRowsPerCta), block(kWarpRowsPerCta * 32);
#define SB_PEER_CASE(NV) \
  case NV: return launch(combine_rows_peer_warp_kernel<NV>, grid, block, 0, st, y, ldy, splits, split_stride, inv, \
                         slots, n_tokens, peer);
  switch (cols / 128) {
    SB_PEER_CASE(1) SB_PEER_CASE(2) SB_PEER_CASE(4) SB_PEER_CASE(8) SB_PEER_CASE(16)
    default: return SB_ERR_UNSUPPORTED;
  }
#undef SB_PEER_CASE
}

template <typename T>
int launch_combine_ln_warp(const float* y, int64_t ldy, int splits, int64_t split_stride, const int32_t* inv,
                           int slots, const float* delta_in, const T* h, const T* x0, int n_tokens, int cols,
                           const float* ln_w, const float* ln_b, float alpha, float beta, float eps, T* out,
                           float* delta_out, cudaStream_t st) {
  const dim3 grid((n_tokens + kWarpRowsPerCta - 1) / kWarpRowsPerCta), block(kWarpRowsPerCta * 32);
#define SB_LN_CASE(NV) \
  case NV: return launch(combine_ln_warp_kernel<T, NV>, grid, block, 0, st, y, ldy, splits, split_stride, inv, slots, \
                         delta_in, h, x0, n_tokens, ln_w, ln_b, alpha, beta, eps, out, delta_out);
  switch (cols / 128) {
    SB_LN_CASE(1) SB_LN_CASE(2) SB_LN_CASE(4) SB_LN_CASE(8) SB_LN_CASE(16)
    default: return SB_ERR_UNSUPPORTED;
  }
#undef SB_LN_CASE
}

template <typename T>
int launch_combine_ln_wait_warp(const float* y, const int32_t* inv, int slots, const T* h, const T* x0, int n_tokens,
                                int cols, const float* ln_w, const float* ln_b, float alpha, float beta, float eps,
                                T* out, uint8_t* wait_region, int64_t ctrl_off, int wait_world, int* wait_status,
                                cudaStream_t st) {
  const dim3 grid((n_tokens + kWarpRowsPerCta - 1) / kWarpRowsPerCta), block(kWarpRowsPerCta * 32);
#define SB_LNW_CASE(NV) \
  case NV: return launch(combine_ln_wait_warp_kernel<T, NV>, grid, block, 0, st, y, int64_t(cols), inv, slots, h, x0, \
                         n_tokens, ln_w, ln_b, alpha, beta, eps, out, wait_region, ctrl_off, wait_world, wait_status);
  switch (cols / 128) {
    SB_LNW_CASE(1) SB_LNW_CASE(2) SB_LNW_CASE(4) SB_LNW_CASE(8) SB_LNW_CASE(16)
    default: return SB_ERR_UNSUPPORTED;
  }
#undef SB_LNW_CASE
}
}  // namespace

extern "C" SB_API int sb_combine_rows(const float* y, int64_t ldy, int splits, int64_t split_stride,
                                      const int32_t* inv, int slots, int n_tokens, int cols,
                                      float* out_f32, const int32_t* scatter_inv, int scatter_slots,
                                      void* scatter_out, int act_dtype, void* stream) {
  if (n_tokens < 0 || cols <= 0 || cols % 4 || slots <= 0 || slots > kMaxSlots || splits <= 0 || splits > kMaxSplits ||
      ldy < cols || (ldy % 4) || (split_stride % 4) || (scatter_inv && (scatter_slots <= 0 ||
      scatter_slots > kMaxSlots || !scatter_out)) || (n_tokens > 0 && (!y || !inv)) ||
      (scatter_out && act_dtype != SB_F32 && act_dtype != SB_BF16))
    return SB_ERR_ARG;
  if (n_tokens == 0) return SB_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (use_warp_rows(n_tokens, cols)) {
    if (act_dtype == SB_BF16 || !scatter_out)
      return launch_combine_rows_warp<__nv_bfloat16>(y, ldy, splits, split_stride, inv, slots, n_tokens, cols, out_f32,
                                                     scatter_inv, scatter_slots,
                                                     static_cast<__nv_bfloat16*>(scatter_out), st);
    return launch_combine_rows_warp<float>(y, ldy, splits, split_stride, inv, slots, n_tokens, cols, out_f32,
                                           scatter_inv, scatter_slots, static_cast<float*>(scatter_out), st);
  }
  if (act_dtype == SB_F32)
    return launch(combine_rows_kernel<float>, dim3(n_tokens), dim3(kCombineThreads), 0, st, y, ldy, splits,
                  split_stride, inv, slots, cols, out_f32, scatter_inv, scatter_slots, static_cast<float*>(scatter_out),
                  EpPeer{});
  if (act_dtype == SB_BF16)
    return launch(combine_rows_kernel<__nv_bfloat16>, dim3(n_tokens), dim3(kCombineThreads), 0, st, y, ldy, splits,
                  split_stride, inv, slots, cols, out_f32, scatter_inv, scatter_slots,
                  static_cast<__nv_bfloat16*>(scatter_out), EpPeer{});
  return SB_ERR_ARG;
}

extern "C" SB_API int sb_combine_ln(const float* y, int64_t ldy, int splits, int64_t split_stride,
                                    const int32_t* inv, int slots, const float* delta_in,
                                    const void* h, const void* x0, int act_dtype, int n_tokens,
                                    int cols, const float* ln_w, const float* ln_b, float alpha,
                                    float beta, float eps, void* out, float* delta_out,
                                    void* stream) {
  if (n_tokens < 0 || cols <= 0 || cols > kLnThreads * kLnMaxVec * 4 || cols % 4 || !ln_w || !ln_b ||
      (y && (!inv || slots <= 0 || slots > kMaxSlots || splits <= 0 || splits > kMaxSplits || ldy < cols)) ||
      (!y && !delta_in) || (n_tokens > 0 && (!h || !x0 || !out)))
    return SB_ERR_ARG;
  if (n_tokens == 0) return SB_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (use_warp_rows(n_tokens, cols) && (!y || ldy % 4 == 0) && (act_dtype == SB_F32 || act_dtype == SB_BF16)) {
    if (act_dtype == SB_F32)
      return launch_combine_ln_warp<float>(y, ldy, splits, split_stride, inv, slots, delta_in,
                                           static_cast<const float*>(h), static_cast<const float*>(x0), n_tokens, cols,
                                           ln_w, ln_b, alpha, beta, eps, static_cast<float*>(out), delta_out, st);
    return launch_combine_ln_warp<__nv_bfloat16>(y, ldy, splits, split_stride, inv, slots, delta_in,
                                                 static_cast<const __nv_bfloat16*>(h),
                                                 static_cast<const __nv_bfloat16*>(x0), n_tokens, cols, ln_w, ln_b,
                                                 alpha, beta, eps, static_cast<__nv_bfloat16*>(out), delta_out, st);
  }
  if (act_dtype == SB_F32)
    return launch(combine_ln_kernel<float>, dim3(n_tokens), dim3(kLnThreads), 0, st, y, ldy, splits, split_stride,
                  inv, slots, delta_in, static_cast<const float*>(h), static_cast<const float*>(x0), cols, ln_w,
                  ln_b, alpha, beta, eps, static_cast<float*>(out), delta_out, static_cast<uint8_t*>(nullptr),
                  int64_t(0), 0, static_cast<int*>(nullptr));
  if (act_dtype == SB_BF16)
    return launch(combine_ln_kernel<__nv_bfloat16>, dim3(n_tokens), dim3(kLnThreads), 0, st, y, ldy, splits,
                  split_stride, inv, slots, delta_in, static_cast<const __nv_bfloat16*>(h),
                  static_cast<const __nv_bfloat16*>(x0), cols, ln_w, ln_b, alpha, beta, eps,
                  static_cast<__nv_bfloat16*>(out), delta_out, static_cast<uint8_t*>(nullptr), int64_t(0), 0,
                  static_cast<int*>(nullptr));
  return SB_ERR_ARG;
}

namespace sb {
int combine_ln_route(const float* y, int64_t ldy, int splits, int64_t split_stride, const int32_t* inv, int slots,
                     const void* h, const void* x0, int act_dtype, int n_tokens, int cols, const float* ln_w,
                     const float* ln_b, float alpha, float beta, float eps, void* out, const RouteArgs& r,
                     cudaStream_t st) {
  if (n_tokens <= 0) return SB_OK;
  if (!y || !inv || slots <= 0 || slots > kMaxSlots || splits <= 0 || splits > kMaxSplits || ldy < cols ||
      cols % 4 || cols > kLnThreads * kLnMaxVec * 4 || cols % 8 || r.E > kRouterMaxE || r.K > 32 || r.M > 32 ||
      r.K > r.E || r.M > r.E)
    return SB_ERR_ARG;
  const size_t smem = route_smem_bytes(act_dtype, cols, r.E, r.K);
  if (smem > kRouteEdgesMaxSmem) return SB_ERR_UNSUPPORTED;
  if (act_dtype == SB_F32) {
    static bool attr_set = false;
    if (!attr_set) {
      cudaFuncSetAttribute(combine_ln_route_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kRouteEdgesMaxSmem);
      attr_set = true;
    }
    return launch(combine_ln_route_kernel<float>, dim3(n_tokens), dim3(kLnThreads), smem, st, y, ldy, splits,
                  split_stride, inv, slots, static_cast<const float*>(h), static_cast<const float*>(x0), cols, ln_w,
                  ln_b, alpha, beta, eps, static_cast<float*>(out), r);
  }
  if (act_dtype != SB_BF16) return SB_ERR_ARG;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(combine_ln_route_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kRouteEdgesMaxSmem);
    attr_set = true;
  }
  return launch(combine_ln_route_kernel<__nv_bfloat16>, dim3(n_tokens), dim3(kLnThreads), smem, st, y, ldy, splits,
                split_stride, inv, slots, static_cast<const __nv_bfloat16*>(h),
                static_cast<const __nv_bfloat16*>(x0), cols, ln_w, ln_b, alpha, beta, eps,
                static_cast<__nv_bfloat16*>(out), r);
}
}  // namespace sb

namespace sb {
int combine_rows_peer(const float* y, int64_t ldy, int splits, int64_t split_stride, const int32_t* inv, int slots,
                      int n_tokens, int cols, const EpPeerArgs& pa, cudaStream_t st) {
  if (n_tokens <= 0 || cols % 4 || slots <= 0 || slots > kMaxSlots || splits <= 0 || splits > kMaxSplits ||
      !pa.regions || n_tokens != pa.world * pa.cap)
    return SB_ERR_ARG;
  EpPeer peer;
  peer.regions = reinterpret_cast<uint8_t* const*>(pa.regions);
  peer.world = pa.world;
  peer.me = pa.rank;
  peer.cap = pa.cap;
  peer.ret_off = pa.ret_off;
  peer.ctrl_off = pa.ctrl_off;
  if (use_warp_rows(n_tokens, cols) && ldy % 4 == 0)
    return launch_combine_rows_peer_warp(y, ldy, splits, split_stride, inv, slots, n_tokens, cols, peer, st);
  return launch(combine_rows_kernel<float>, dim3(n_tokens), dim3(kCombineThreads), 0, st, y, ldy, splits, split_stride,
                inv, slots, cols, static_cast<float*>(nullptr), static_cast<const int32_t*>(nullptr), 0,
                static_cast<float*>(nullptr), peer);
}
}  // namespace sb

extern "C" SB_API int sb_ep_epilogue_peer(void* region, int world, int cap, int64_t row_pitch,
                                          const int32_t* ret_pos, int top_k, const void* h, const void* x0,
                                          int act_dtype, int n_tokens, int hidden, const float* ln_w,
                                          const float* ln_b, float alpha, float beta, float eps, void* out,
                                          int* status, void* stream) {
  if (!region || !ret_pos || top_k <= 0 || top_k > kMaxSlots || n_tokens < 0 || hidden <= 0 || hidden % 4 ||
      hidden > kLnThreads * kLnMaxVec * 4 || !ln_w || !ln_b || (n_tokens > 0 && (!h || !x0 || !out)) ||
      !sb_ep_peer_region_bytes(world, cap, row_pitch, hidden) || n_tokens > cap)
    return SB_ERR_ARG;
  int64_t ret_off, ctrl_off;
  ep_region_offsets(world, cap, row_pitch, hidden, &ret_off, &ctrl_off);
  const float* y = reinterpret_cast<const float*>(static_cast<uint8_t*>(region) + ret_off);
  uint8_t* reg = static_cast<uint8_t*>(region);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n_tokens == 0) return sb_ep_wait(region, world, cap, row_pitch, hidden, 1, status, stream);
  if (use_warp_rows(n_tokens, hidden) && (act_dtype == SB_F32 || act_dtype == SB_BF16)) {
    if (act_dtype == SB_F32)
      return launch_combine_ln_wait_warp<float>(y, ret_pos, top_k, static_cast<const float*>(h),
                                                static_cast<const float*>(x0), n_tokens, hidden, ln_w, ln_b, alpha,
                                                beta, eps, static_cast<float*>(out), reg, ctrl_off, world, status, st);
    return launch_combine_ln_wait_warp<__nv_bfloat16>(y, ret_pos, top_k, static_cast<const __nv_bfloat16*>(h),
                                                      static_cast<const __nv_bfloat16*>(x0), n_tokens, hidden, ln_w,
                                                      ln_b, alpha, beta, eps, static_cast<__nv_bfloat16*>(out), reg,
                                                      ctrl_off, world, status, st);
  }
  if (act_dtype == SB_F32)
    return launch(combine_ln_kernel<float>, dim3(n_tokens), dim3(kLnThreads), 0, st, y, int64_t(hidden), 1,
                  int64_t(0), ret_pos, top_k, static_cast<const float*>(nullptr), static_cast<const float*>(h),
                  static_cast<const float*>(x0), hidden, ln_w, ln_b, alpha, beta, eps, static_cast<float*>(out),
                  static_cast<float*>(nullptr), reg, ctrl_off, world, status);
  if (act_dtype != SB_BF16) return SB_ERR_ARG;
  return launch(combine_ln_kernel<__nv_bfloat16>, dim3(n_tokens), dim3(kLnThreads), 0, st, y, int64_t(hidden), 1,
                int64_t(0), ret_pos, top_k, static_cast<const float*>(nullptr),
                static_cast<const __nv_bfloat16*>(h), static_cast<const __nv_bfloat16*>(x0), hidden, ln_w, ln_b,
                alpha, beta, eps, static_cast<__nv_bfloat16*>(out), static_cast<float*>(nullptr), reg, ctrl_off,
                world, status);
}
