// Device side of the dispatch-plan grouping (sb_group.cu), shared with the
// kernels that build plans in their last CTA (sb_router.cu).
//
// This is build_dispatch_plan (spider_infer/forge/ep/dispatch.py:56-115) as
// one stable permutation: groups ascending, rows ascending inside a group,
// repeated ids of one row merged into their first slot with the weights
// summed in slot order, and (optionally) entries with summed weight <= 0
// dropped.  Ranks come from warp match masks and a fixed-order scan.
#pragma once

#include "sb_common.cuh"

namespace sb {

constexpr int kGroupMaxG = 256;

// Evaluate entry e = row*slots + s: returns its group (or -1) and summed weight.
SB_DEVINL int entry_group(const int32_t* __restrict__ idx, const float* __restrict__ w, int slots,
                          int G, int flags, int64_t e, float& wsum) {
  const int64_t row0 = (e / slots) * slots;
  const int s = static_cast<int>(e - row0);
  const int g = idx[e];
  wsum = 0.f;
  if (g < 0 || g >= G) return -1;
  for (int j = 0; j < s; ++j)
    if (idx[row0 + j] == g) return -1;  // merged into an earlier slot of the same row
  float acc = 0.f;
  for (int j = 0; j < slots; ++j)
    if (idx[row0 + j] == g) acc += w ? w[row0 + j] : 1.f;
  wsum = acc;
  if ((flags & SB_GROUP_POSITIVE_ONLY) && !(acc > 0.f)) return -1;
  return g;
}

// entry_group over a copy of the rows in shared memory: s_idx / s_w hold
// entries lo .. lo + n of the grouping, lo a multiple of `slots`; `le` = e - lo.
SB_DEVINL int entry_group_staged(const int32_t* s_idx, const float* s_w, int slots, int G, int flags, int le,
                                 float& wsum) {
  const int row0 = (le / slots) * slots;
  const int s = le - row0;
  const int g = s_idx[le];
  wsum = 0.f;
  if (g < 0 || g >= G) return -1;
  for (int j = 0; j < s; ++j)
    if (s_idx[row0 + j] == g) return -1;  // merged into an earlier slot of the same row
  float acc = 0.f;
  for (int j = 0; j < slots; ++j)
    if (s_idx[row0 + j] == g) acc += s_w[row0 + j];
  wsum = acc;
  if ((flags & SB_GROUP_POSITIVE_ONLY) && !(acc > 0.f)) return -1;
  return g;
}

// The whole grouping in one CTA (any block size that is a multiple of 32).
SB_DEVINL void group_one_cta(const int32_t* __restrict__ idx, const float* __restrict__ w, int n_rows, int slots,
                             int G, int flags, int32_t* __restrict__ offsets, int32_t* __restrict__ perm_row,
                             int32_t* __restrict__ perm_slot, float* __restrict__ perm_w, int32_t* __restrict__ inv,
                             int32_t* __restrict__ rank_scratch, float* __restrict__ w_scratch) {
  __shared__ int wcnt[32][kGroupMaxG];
  __shared__ int run_total[kGroupMaxG];
  __shared__ int s_off[kGroupMaxG + 1];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nthreads = blockDim.x, nwarps = nthreads >> 5;
  const int64_t total = static_cast<int64_t>(n_rows) * slots;
  const unsigned lt_mask = (1u << lane) - 1u;
  if (total <= nthreads) {
    // one entry per thread (decode sizes): group, rank and weight stay in
    // registers instead of a round trip through the scratch arrays
    for (int i = tid; i < nwarps * kGroupMaxG; i += nthreads) (&wcnt[0][0])[i] = 0;
    __syncthreads();
    const int64_t e = tid;
    float wsum = 0.f;
    const int g = e < total ? entry_group(idx, w, slots, G, flags, e, wsum) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, g);
    const int rank_w = __popc(peers & lt_mask);
    if (g >= 0 && rank_w == 0) wcnt[warp][g] = __popc(peers);
    __syncthreads();
    for (int gg = tid; gg < G; gg += nthreads) {  // warp-order scan per group, then the group totals
      int acc = 0;
      for (int ww = 0; ww < nwarps; ++ww) {
        const int c = wcnt[ww][gg];
        wcnt[ww][gg] = acc;
        acc += c;
      }
      run_total[gg] = acc;
    }
    __syncthreads();
    if (tid == 0) {
      int acc = 0;
      for (int gg = 0; gg < G; ++gg) {
        s_off[gg] = acc;
        acc += run_total[gg];
      }
      s_off[G] = acc;
    }
    __syncthreads();
    for (int gg = tid; gg <= G; gg += nthreads) offsets[gg] = s_off[gg];
    if (e < total) {
      if (g < 0) {
        inv[e] = -1;
      } else {
        const int pos = s_off[g] + wcnt[warp][g] + rank_w;
        perm_row[pos] = static_cast<int32_t>(e / slots);
        perm_slot[pos] = static_cast<int32_t>(e);
        perm_w[pos] = wsum;
        inv[e] = pos;
      }
    }
    return;
  }
  for (int g = tid; g < G; g += nthreads) run_total[g] = 0;

  for (int64_t base = 0; base < total; base += nthreads) {
    for (int i = tid; i < nwarps * kGroupMaxG; i += nthreads) (&wcnt[0][0])[i] = 0;
    __syncthreads();
    const int64_t e = base + tid;
    float wsum = 0.f;
    const int g = e < total ? entry_group(idx, w, slots, G, flags, e, wsum) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, g);
    const int rank_w = __popc(peers & lt_mask);
    if (g >= 0 && rank_w == 0) wcnt[warp][g] = __popc(peers);
    __syncthreads();
    for (int gg = tid; gg < G; gg += nthreads) {
      int acc = run_total[gg];
      for (int ww = 0; ww < nwarps; ++ww) {
        const int c = wcnt[ww][gg];
        wcnt[ww][gg] = acc;
        acc += c;
      }
      run_total[gg] = acc;
    }
    __syncthreads();
    if (e < total) {
      rank_scratch[e] = g >= 0 ? wcnt[warp][g] + rank_w : -1;
      w_scratch[e] = wsum;
    }
    __syncthreads();
  }
  if (tid == 0) {
    int acc = 0;
    for (int g = 0; g < G; ++g) {
      s_off[g] = acc;
      acc += run_total[g];
    }
    s_off[G] = acc;
  }
  __syncthreads();
  for (int g = tid; g <= G; g += nthreads) offsets[g] = s_off[g];
  for (int64_t e = tid; e < total; e += nthreads) {
    const int r = rank_scratch[e];
    if (r < 0) {
      inv[e] = -1;
      continue;
    }
    const int g = idx[e];
    const int pos = s_off[g] + r;
    perm_row[pos] = static_cast<int32_t>(e / slots);
    perm_slot[pos] = static_cast<int32_t>(e);
    perm_w[pos] = w_scratch[e];
    inv[e] = pos;
  }
}

}  // namespace sb
