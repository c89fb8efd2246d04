// Early-exit active set of the recurrent decode
// (SpiderWebLM._run_recurrent_decode, spider_moe/model.py:450-473, with
// spider_moe/active_set.py: ActiveSet.drop, compact_active, scatter_active).
//
// After loop l ran on the compact rows of the active batch entries, one step
// (sb_active_set_step) does on the device what the reference does with
// index_copy_, an exit-head Linear, a sigmoid, a comparison and boolean
// indexing:
//
//   exit_flags_kernel      warp per active row: confidence of the row's first
//                          position, sigmoid(h . w + b); stays = !(conf > thr)
//   active_set_kernel      CTA per chunk of rows: exclusive count of the rows
//                          that stay before the chunk (every CTA re-reads the
//                          flags, n ints) plus a scan inside it; then for every
//                          row  h_full[act_idx[r]] = h_new[r]  (scatter_active)
//                          and for the rows that stay, at their rank j:
//                          act_next[j] = act_idx[r], h_next[j] = h_new[r],
//                          x0_next[j] = x0c[r] -- the next loop's compact inputs,
//                          so no separate gather runs before the next loop;
//                          the last CTA writes the new count.
//
// Rank order is the order of the current list, so the active indices stay in
// ascending batch order as ActiveSet.drop keeps them.
#include "sb_common.cuh"
#include "sb_internal.h"

namespace sb {

constexpr int kExitWarps = 8;
constexpr int kActiveChunk = 256;  // rows per CTA of active_set_kernel (= its threads)

template <typename T>
__global__ void __launch_bounds__(kExitWarps * 32)
exit_flags_kernel(const T* __restrict__ h_new, int n, int64_t row_elems, int H, const float* __restrict__ w,
                  const float* __restrict__ b, float threshold, int32_t* __restrict__ stays,
                  float* __restrict__ confidence) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int r = blockIdx.x * kExitWarps + (threadIdx.x >> 5);
  if (r >= n) return;
  const T* row = h_new + static_cast<int64_t>(r) * row_elems;  // position 0 of the row
  float z = 0.f;
  for (int i = lane; i < H; i += 32) z = fmaf(to_f32(row[i]), w[i], z);
  z = warp_sum(z) + b[0];
  if (lane == 0) {
    const float conf = 1.0f / (1.0f + expf(-z));
    stays[r] = conf > threshold ? 0 : 1;
    if (confidence) confidence[r] = conf;
  }
}

__global__ void __launch_bounds__(kActiveChunk)
active_set_kernel(const uint4* __restrict__ h_new, const uint4* __restrict__ x0c, const int32_t* __restrict__ act_idx,
                  const int32_t* __restrict__ stays, int n, int64_t row_vecs, uint4* __restrict__ h_full,
                  int32_t* __restrict__ act_next, uint4* __restrict__ h_next, uint4* __restrict__ x0_next,
                  int32_t* __restrict__ n_next) {
  __shared__ int s_scan[kActiveChunk];
  __shared__ int s_warp[kActiveChunk / 32];
  __shared__ int s_base;
  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r0 = blockIdx.x * kActiveChunk;
  // rows that stay before this chunk
  int before = 0;
  for (int i = tid; i < r0; i += blockDim.x) before += stays[i];
  before = __reduce_add_sync(0xffffffffu, before);
  if (lane == 0) s_warp[warp] = before;
  __syncthreads();
  if (tid == 0) {
    int s = 0;
    for (int w = 0; w < kActiveChunk / 32; ++w) s += s_warp[w];
    s_base = s;
  }
  __syncthreads();
  // inclusive scan of this chunk's flags (Hillis-Steele in shared memory)
  const int r = r0 + tid;
  const int mine = r < n ? stays[r] : 0;
  s_scan[tid] = mine;
  __syncthreads();
  for (int off = 1; off < kActiveChunk; off <<= 1) {
    const int v = tid >= off ? s_scan[tid - off] : 0;
    __syncthreads();
    s_scan[tid] += v;
    __syncthreads();
  }
  const int base = s_base;
  const int chunk_rows = n - r0 < kActiveChunk ? n - r0 : kActiveChunk;
  if (r < n && mine) act_next[base + s_scan[tid] - 1] = act_idx[r];
  if (blockIdx.x == gridDim.x - 1 && tid == 0) *n_next = base + s_scan[chunk_rows - 1];
  // row moves: the CTA's threads stride over (row, 16-byte vector) pairs
  const int64_t total = static_cast<int64_t>(chunk_rows) * row_vecs;
  for (int64_t i = tid; i < total; i += blockDim.x) {
    const int lr = static_cast<int>(i / row_vecs);
    const int64_t v = i - static_cast<int64_t>(lr) * row_vecs;
    const int rr = r0 + lr;
    const uint4 hv = h_new[static_cast<int64_t>(rr) * row_vecs + v];
    h_full[static_cast<int64_t>(act_idx[rr]) * row_vecs + v] = hv;
    if (stays[rr]) {
      const int j = base + s_scan[lr] - 1;
      h_next[static_cast<int64_t>(j) * row_vecs + v] = hv;
      x0_next[static_cast<int64_t>(j) * row_vecs + v] = x0c[static_cast<int64_t>(rr) * row_vecs + v];
    }
  }
}

}  // namespace sb

using namespace sb;

extern "C" SB_API int sb_active_set_step(int act_dtype, int n_active, int positions, int hidden, const void* h_new,
                                         const void* x0c, const int32_t* act_idx, const float* exit_w,
                                         const float* exit_b, float threshold, void* h_full, int32_t* act_next,
                                         void* h_next, void* x0_next, int32_t* n_next, int32_t* flags,
                                         float* confidence, void* stream) {
  if ((act_dtype != SB_F32 && act_dtype != SB_BF16) || n_active < 0 || positions <= 0 || hidden <= 0 ||
      hidden % 8 || !n_next)
    return SB_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n_active == 0) return cuda_status(cudaMemsetAsync(n_next, 0, sizeof(int32_t), st));
  if (!h_new || !x0c || !act_idx || !exit_w || !exit_b || !h_full || !act_next || !h_next || !x0_next || !flags)
    return SB_ERR_ARG;
  const int es = act_dtype == SB_F32 ? 4 : 2;
  const int64_t row_elems = static_cast<int64_t>(positions) * hidden;
  const int64_t row_vecs = row_elems * es / 16;  // hidden % 8 == 0: whole 16-byte vectors
  for (const void* p : {h_new, x0c, static_cast<const void*>(h_full), static_cast<const void*>(h_next),
                        static_cast<const void*>(x0_next)})
    if (reinterpret_cast<uintptr_t>(p) % 16) return SB_ERR_ARG;
  const dim3 g1((n_active + kExitWarps - 1) / kExitWarps);
  int rc = act_dtype == SB_F32
               ? launch(exit_flags_kernel<float>, g1, dim3(kExitWarps * 32), 0, st, static_cast<const float*>(h_new),
                        n_active, row_elems, hidden, exit_w, exit_b, threshold, flags, confidence)
               : launch(exit_flags_kernel<__nv_bfloat16>, g1, dim3(kExitWarps * 32), 0, st,
                        static_cast<const __nv_bfloat16*>(h_new), n_active, row_elems, hidden, exit_w, exit_b,
                        threshold, flags, confidence);
  if (rc) return rc;
  const dim3 g2((n_active + kActiveChunk - 1) / kActiveChunk);
  return launch(active_set_kernel, g2, dim3(kActiveChunk), 0, st, static_cast<const uint4*>(h_new),
                static_cast<const uint4*>(x0c), act_idx, static_cast<const int32_t*>(flags), n_active, row_vecs,
                static_cast<uint4*>(h_full), act_next, static_cast<uint4*>(h_next), static_cast<uint4*>(x0_next),
                n_next);
}
