// Device side of the token routing shared by the router kernels
// (sb_router.cu) and the fused LayerNorm + next-loop routing kernel
// (sb_combine.cu).
//
// Router (spider_moe/model.py:254-258): logits = h . W_r^T + loop_bias[l];
// fp32 softmax; top-K by repeated arg-max; renormalise by max(sum, 1e-9).
// Edge generator (model.py:260-266): a selected source s's E destination
// logits, top-M, fp32 softmax over the M selected values.
#pragma once

#include "sb_common.cuh"

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

// Softmax over one token's E router logits (fp32, spider_moe/model.py:256),
// top-K by repeated arg-max (model.py:257; a taken expert is masked with -1
// since probabilities are >= 0, equal values go to the smaller id) and the
// renormalisation of model.py:258.  One warp; lane k < K returns slot k.
template <int R>  // registers per lane: E <= 32 R
SB_DEVINL void router_select_r(const float* logits, int E, int K, int lane, float* probs_out, int& sel_i,
                               float& sel_w) {
  float logit[R];
#pragma unroll
  for (int i = 0; i < R; ++i) logit[i] = (lane + 32 * i < E) ? logits[lane + 32 * i] : -INFINITY;
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < R; ++i) mx = fmaxf(mx, logit[i]);
  mx = warp_max(mx);
  float p[R];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < R; ++i) {
    p[i] = (lane + 32 * i < E) ? expf(logit[i] - mx) : 0.f;
    s += p[i];
  }
  s = warp_sum(s);
#pragma unroll
  for (int i = 0; i < R; ++i) {
    p[i] = p[i] / s;
    if (probs_out && lane + 32 * i < E) probs_out[lane + 32 * i] = p[i];
  }
  float w = 0.f, sum_w = 0.f;
  int idx = -1;
  for (int k = 0; k < K; ++k) {
    float bv = -1.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const int e = lane + 32 * i;
      if (e < E && (p[i] > bv || (p[i] == bv && e < bi))) { bv = p[i]; bi = e; }
    }
    warp_argmax(bv, bi);
#pragma unroll
    for (int i = 0; i < R; ++i)
      if (lane + 32 * i == bi) p[i] = -1.f;
    sum_w += bv;
    if (lane == k) { w = bv; idx = bi; }
  }
  sel_i = idx;
  sel_w = w / fmaxf(sum_w, 1e-9f);
}

// Top-M of one source's E destination logits (spider_moe/model.py:264-266):
// repeated arg-max with a taken mask (equal values to the smaller id), then an
// fp32 softmax over the M selected values.  One warp; lane m < M returns slot m.
template <int R>
SB_DEVINL void topm_select_r(const float* logits, int E, int M, int lane, int& sel_i, float& sel_w) {
  float v[R];
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? logits[e] : -INFINITY;
  }
  uint32_t taken = 0;  // bit i: destination lane + 32*i already selected
  float sel_v = -INFINITY, first = -INFINITY;
  int idx = -1;
  for (int m = 0; m < M; ++m) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const int e = lane + 32 * i;
      if (e < E && !(taken & (1u << i)) && (bi == 0x7fffffff || v[i] > bv || (v[i] == bv && e < bi))) {
        bv = v[i];
        bi = e;
      }
    }
    warp_argmax(bv, bi);
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    if (m == 0) first = bv;  // the largest selected value
    if (lane == m) { sel_v = bv; idx = bi; }
  }
  const float ex = (lane < M) ? expf(sel_v - first) : 0.f;
  const float s = warp_sum(ex);
  sel_i = idx;
  sel_w = ex / s;
}

// Warp-uniform dispatch on E: only ceil(E/32) (rounded to a power of two)
// values per lane are carried through the selection loops.
SB_DEVINL void router_select(const float* logits, int E, int K, int lane, float* probs_out, int& sel_i,
                             float& sel_w) {
  if (E <= 32) router_select_r<1>(logits, E, K, lane, probs_out, sel_i, sel_w);
  else if (E <= 64) router_select_r<2>(logits, E, K, lane, probs_out, sel_i, sel_w);
  else if (E <= 128) router_select_r<4>(logits, E, K, lane, probs_out, sel_i, sel_w);
  else router_select_r<8>(logits, E, K, lane, probs_out, sel_i, sel_w);
}
SB_DEVINL void topm_select(const float* logits, int E, int M, int lane, int& sel_i, float& sel_w) {
  if (E <= 32) topm_select_r<1>(logits, E, M, lane, sel_i, sel_w);
  else if (E <= 64) topm_select_r<2>(logits, E, M, lane, sel_i, sel_w);
  else if (E <= 128) topm_select_r<4>(logits, E, M, lane, sel_i, sel_w);
  else topm_select_r<8>(logits, E, M, lane, sel_i, sel_w);
}

// Router, edge generator and edge top-M of one token per CTA, for small
// batches (decode), where recomputing a selected source's E generator rows
// per token costs less than grouping tokens by source for a GEMM.  The
// hidden row is staged in shared memory; every warp keeps the loads of four
// weight rows (two chunk steps each) in flight.  The router logits use the
// same per-lane accumulation order and tree reduction as router_kernel; the
// edge logits of a selected source s are its generator rows s*E .. s*E+E-1
// (spider_moe/model.py:260-263) dotted with the hidden row in fp32.
constexpr int kRouteRows = 4;

// acc[j] = x . rows[j] for nrows (<= 4) consecutive rows starting at `rows`.
template <typename T>
SB_DEVINL void dot_rows4(const T* __restrict__ sh, const T* __restrict__ rows, int hidden, int nrows, int nchunks,
                         int lane, float* acc) {
#pragma unroll
  for (int j = 0; j < kRouteRows; ++j) acc[j] = 0.f;
#pragma unroll 2  // measured at hidden 1024: unrolling by 1 or 4 makes the kernel ~1.5x slower
  for (int c = lane; c < nchunks; c += 32) {
    float hv[8];
    Vec8<T>::load(sh + c * 8, hv);
#pragma unroll
    for (int j = 0; j < kRouteRows; ++j) {
      if (j < nrows) {
        float wv[8];
        Vec8<T>::load(rows + static_cast<size_t>(j) * hidden + c * 8, wv);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[j] = fmaf(hv[i], wv[i], acc[j]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < kRouteRows; ++j) acc[j] = warp_sum(acc[j]);
}

// Route one token whose hidden row `sh` is staged (and synchronised) in shared
// memory; `smem` is the dynamic shared memory laid out by route_smem_bytes()
// (the row first).  All 256 threads of the CTA take part.
template <typename T>
SB_DEVINL void route_token(const T* sh, int t, int hidden, const T* __restrict__ wr, const float* __restrict__ rbias,
                           int E, int K, const T* __restrict__ gen_w, const float* __restrict__ gen_bias, int M,
                           int32_t* __restrict__ top_idx, float* __restrict__ top_w, int32_t* __restrict__ edge_idx,
                           float* __restrict__ edge_w, uint8_t* smem) {
  float* slog = reinterpret_cast<float*>(smem + ((hidden * sizeof(T) + 15) & ~size_t(15)));  // [E]
  float* selog = slog + E;                                                                 // [K][E]
  int* ssel = reinterpret_cast<int*>(selog + K * E);                                       // [K]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nchunks = hidden >> 3;
  // router logits: warp w takes rows w*4 .. w*4+3, then + 32 ...
  for (int r0 = warp * kRouteRows; r0 < E; r0 += kRouterWarps * kRouteRows) {
    const int nr = min(kRouteRows, E - r0);
    float acc[kRouteRows];
    dot_rows4<T>(sh, wr + static_cast<size_t>(r0) * hidden, hidden, nr, nchunks, lane, acc);
    if (lane == 0)
#pragma unroll
      for (int j = 0; j < kRouteRows; ++j)
        if (j < nr) slog[r0 + j] = acc[j] + rbias[r0 + j];
  }
  __syncthreads();
  if (warp == 0) {
    int sel_i;
    float sel_w;
    router_select(slog, E, K, lane, nullptr, sel_i, sel_w);
    if (lane < K) {
      top_idx[static_cast<size_t>(t) * K + lane] = sel_i;
      top_w[static_cast<size_t>(t) * K + lane] = sel_w;
      ssel[lane] = sel_i;
    }
  }
  __syncthreads();
  // edge logits: item (k, j0) = generator rows ssel[k]*E + j0 .. j0+3
  const int jsteps = (E + kRouteRows - 1) / kRouteRows;
  for (int item = warp; item < K * jsteps; item += kRouterWarps) {
    const int k = item / jsteps;
    const int j0 = (item - k * jsteps) * kRouteRows;
    const int nr = min(kRouteRows, E - j0);
    const size_t row0 = static_cast<size_t>(ssel[k]) * E + j0;
    float acc[kRouteRows];
    dot_rows4<T>(sh, gen_w + row0 * hidden, hidden, nr, nchunks, lane, acc);
    if (lane == 0)
#pragma unroll
      for (int j = 0; j < kRouteRows; ++j)
        if (j < nr) selog[k * E + j0 + j] = acc[j] + gen_bias[row0 + j];
  }
  __syncthreads();
  for (int k = warp; k < K; k += kRouterWarps) {
    int sel_i;
    float sel_w;
    topm_select(selog + k * E, E, M, lane, sel_i, sel_w);
    if (lane < M) {
      const int64_t slot = static_cast<int64_t>(t) * K + k;
      edge_idx[slot * M + lane] = sel_i;
      edge_w[slot * M + lane] = sel_w;
    }
  }
}

// Dynamic shared memory of route_token: the hidden row, E router logits, K x E
// edge logits, K selected sources.
inline size_t route_smem_bytes(int act_dtype, int hidden, int E, int K) {
  const size_t esize = act_dtype == SB_F32 ? 4 : 2;
  return ((hidden * esize + 15) & ~size_t(15)) + static_cast<size_t>(E) * 4 + static_cast<size_t>(K) * E * 4 +
         static_cast<size_t>(K) * 4;
}

}  // namespace sb
