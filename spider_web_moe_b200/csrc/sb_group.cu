// Device dispatch plan: stable grouping of (row, slot) entries by group id.
//
// This is build_dispatch_plan (spider_infer/forge/ep/dispatch.py:56-115) and
// the per-expert token selection of sparse_expert_delta (spider_moe/
// sparse_experts.py:51-57) as one permutation: groups in ascending id, rows
// ascending inside a group, repeated ids of one row merged into their first
// slot with the weights summed, and (optionally) entries with summed weight
// <= 0 dropped.  The result is deterministic: ranks come from warp match masks
// and a fixed-order scan, never from atomics.
#include "sb_common.cuh"
#include "sb_ep_dev.cuh"
#include "sb_group_dev.cuh"
#include "sb_internal.h"

namespace sb {

constexpr int kGroupThreads = 1024;
// Entries up to which one CTA groups everything; above it the two-pass
// kernels (measured faster from a few hundred entries: one CTA's scans over
// G groups and 32 warps serialise).
constexpr size_t kGroupSingleCtaMax = 512;
// The two-plan launch (decode) keeps one CTA per plan up to this many
// entries: one launch instead of four.
constexpr size_t kGroupPairMax = 2048;

__global__ void __launch_bounds__(kGroupThreads, 1)
group_kernel(const int32_t* __restrict__ idx, const float* __restrict__ w, int n_rows, int slots,
             int G, int flags, int32_t* __restrict__ offsets, int32_t* __restrict__ perm_row,
             int32_t* __restrict__ perm_slot, float* __restrict__ perm_w, int32_t* __restrict__ inv,
             int32_t* __restrict__ rank_scratch, float* __restrict__ w_scratch) {
  pdl_wait();
  pdl_trigger();
  group_one_cta(idx, w, n_rows, slots, G, flags, offsets, perm_row, perm_slot, perm_w, inv, rank_scratch, w_scratch);
}

// Two independent groupings in one launch, one CTA each.
__global__ void __launch_bounds__(kGroupThreads, 1) group_pair_kernel(const GroupJob j0, const GroupJob j1) {
  pdl_wait();
  pdl_trigger();
  const GroupJob& j = blockIdx.x == 0 ? j0 : j1;
  group_one_cta(j.idx, j.w, j.n_rows, j.slots, j.num_groups, j.flags, j.offsets, j.perm_row, j.perm_slot, j.perm_w,
                j.inv, j.rank_scratch, j.w_scratch);
}

// ---------------------------------------------------------------------------
// Two-pass multi-CTA grouping (large entry counts), 256-entry chunks, no
// serial step: pass 1 ranks each entry inside its chunk (warp match masks,
// then the 8 warps' counts scanned in warp order) and stores the chunk's
// per-group counts; pass 2 gives every chunk its base per group -- the counts
// of all earlier chunks plus all smaller groups -- straight from the count
// matrix, and scatters.  Positions equal the single-CTA kernel's.
constexpr int kChunk = 256;
// Entries of whole rows a chunk stages in shared memory (the chunk's 256 plus
// the parts of its first and last rows outside it); wider rows read global memory.
constexpr int kChunkStageMax = 1024;

// Pass 1 for chunk `chunk` of one grouping (a whole CTA of kChunk threads).
SB_DEVINL void group_count_chunk(const int32_t* __restrict__ idx, const float* __restrict__ w, int n_rows, int slots,
                                 int G, int flags, int chunk, int32_t* __restrict__ rank_scratch,
                                 float* __restrict__ w_scratch, int32_t* __restrict__ chunk_count) {
  __shared__ int wcnt[kChunk / 32][kGroupMaxG];
  // the whole rows the chunk's entries belong to, copied once with coalesced
  // loads: an entry's merge test reads every slot of its row
  __shared__ int32_t s_idx[kChunkStageMax];
  __shared__ float s_w[kChunkStageMax];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t total = static_cast<int64_t>(n_rows) * slots;
  for (int i = tid; i < (kChunk / 32) * G; i += kChunk) (&wcnt[0][0])[(i / G) * kGroupMaxG + i % G] = 0;
  const int64_t c0 = static_cast<int64_t>(chunk) * kChunk;
  const int64_t c1 = c0 + kChunk < total ? c0 + kChunk : total;
  const int64_t lo = (c0 / slots) * slots;
  const int64_t hi = c1 > c0 ? ((c1 - 1) / slots + 1) * slots : lo;
  const bool staged = hi - lo <= kChunkStageMax;
  if (staged)
    for (int64_t i = tid; i < hi - lo; i += kChunk) {
      s_idx[i] = idx[lo + i];
      s_w[i] = w ? w[lo + i] : 1.f;
    }
  __syncthreads();
  const int64_t e = c0 + tid;
  float wsum = 0.f;
  const int g = e >= total ? -1
                : staged  ? entry_group_staged(s_idx, s_w, slots, G, flags, static_cast<int>(e - lo), wsum)
                          : entry_group(idx, w, slots, G, flags, e, wsum);
  const unsigned peers = __match_any_sync(0xffffffffu, g);
  const int rank_w = __popc(peers & ((1u << lane) - 1u));
  if (g >= 0 && rank_w == 0) wcnt[warp][g] = __popc(peers);
  __syncthreads();
  for (int gg = tid; gg < G; gg += kChunk) {
    int acc = 0;
#pragma unroll
    for (int ww = 0; ww < kChunk / 32; ++ww) {
      const int c = wcnt[ww][gg];
      wcnt[ww][gg] = acc;
      acc += c;
    }
    chunk_count[static_cast<int64_t>(chunk) * G + gg] = acc;
  }
  __syncthreads();
  if (e < total) {
    rank_scratch[e] = g >= 0 ? wcnt[warp][g] + rank_w : -1;
    w_scratch[e] = wsum;
  }
}

// Pass 2 for chunk `chunk`: the chunk's per-group base from the count matrix,
// then the scatter.  Returns (in *pos_out, per thread) the entry's position, or -1.
SB_DEVINL void group_place_chunk(const int32_t* __restrict__ idx, int n_rows, int slots, int G, int nchunks, int chunk,
                                 const int32_t* __restrict__ rank_scratch, const float* __restrict__ w_scratch,
                                 const int32_t* __restrict__ chunk_count, int32_t* __restrict__ offsets,
                                 int32_t* __restrict__ perm_row, int32_t* __restrict__ perm_slot,
                                 float* __restrict__ perm_w, int32_t* __restrict__ inv, int& pos_out) {
  __shared__ int s_before[kChunk];      // per (group, thread-slice) partial sums, then per group
  __shared__ int s_total[kChunk];
  __shared__ int s_base[kGroupMaxG + 1];
  const int tid = threadIdx.x;
  const int me = chunk;
  pos_out = -1;
  // thread t sums chunks c = t / G, t / G + step, ... of group t % G
  const int per_g = kChunk / G > 0 ? kChunk / G : 1;
  const int gq = tid % G, sl = tid / G;
  int before = 0, all = 0;
  if (tid < per_g * G) {
    for (int c = sl; c < nchunks; c += per_g) {
      const int v = chunk_count[static_cast<int64_t>(c) * G + gq];
      all += v;
      if (c < me) before += v;
    }
  }
  s_before[tid] = before;
  s_total[tid] = all;
  __syncthreads();
  if (tid < G) {
    int b = 0, a = 0;
    for (int j = 0; j < per_g; ++j) {
      b += s_before[j * G + tid];
      a += s_total[j * G + tid];
    }
    s_before[tid] = b;  // earlier chunks' entries of group tid
    s_total[tid] = a;   // all entries of group tid
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int gg = 0; gg < G; ++gg) {
      s_base[gg] = acc;
      acc += s_total[gg];
    }
    s_base[G] = acc;
  }
  __syncthreads();
  if (me == 0)
    for (int gg = tid; gg <= G; gg += kChunk) offsets[gg] = s_base[gg];
  const int64_t total = static_cast<int64_t>(n_rows) * slots;
  const int64_t e = static_cast<int64_t>(me) * kChunk + tid;
  if (e >= total) return;
  const int r = rank_scratch[e];
  if (r < 0) {
    inv[e] = -1;
    return;
  }
  const int g = idx[e];
  const int pos = s_base[g] + s_before[g] + r;
  perm_row[pos] = static_cast<int32_t>(e / slots);
  perm_slot[pos] = static_cast<int32_t>(e);
  perm_w[pos] = w_scratch[e];
  inv[e] = pos;
  pos_out = pos;
}

__global__ void __launch_bounds__(kChunk)
group_count_kernel(const int32_t* __restrict__ idx, const float* __restrict__ w, int n_rows, int slots, int G,
                   int flags, int32_t* __restrict__ rank_scratch, float* __restrict__ w_scratch,
                   int32_t* __restrict__ chunk_count) {
  pdl_wait();
  pdl_trigger();
  group_count_chunk(idx, w, n_rows, slots, G, flags, blockIdx.x, rank_scratch, w_scratch, chunk_count);
}

__global__ void __launch_bounds__(kChunk)
group_place_kernel(const int32_t* __restrict__ idx, int n_rows, int slots, int G, int nchunks,
                   const int32_t* __restrict__ rank_scratch, const float* __restrict__ w_scratch,
                   const int32_t* __restrict__ chunk_count, int32_t* __restrict__ offsets,
                   int32_t* __restrict__ perm_row, int32_t* __restrict__ perm_slot, float* __restrict__ perm_w,
                   int32_t* __restrict__ inv) {
  pdl_wait();
  pdl_trigger();
  int pos;
  group_place_chunk(idx, n_rows, slots, G, nchunks, blockIdx.x, rank_scratch, w_scratch, chunk_count, offsets,
                    perm_row, perm_slot, perm_w, inv, pos);
}

// Two groupings' passes in one launch each: CTAs [0, nch0) take job 0's
// chunks, the rest job 1's.
__global__ void __launch_bounds__(kChunk)
group_count2_kernel(const GroupJob j0, const GroupJob j1, int nch0, int32_t* __restrict__ cc0,
                    int32_t* __restrict__ cc1) {
  pdl_wait();
  pdl_trigger();
  const bool first = static_cast<int>(blockIdx.x) < nch0;
  const GroupJob& j = first ? j0 : j1;
  group_count_chunk(j.idx, j.w, j.n_rows, j.slots, j.num_groups, j.flags, first ? blockIdx.x : blockIdx.x - nch0,
                    j.rank_scratch, j.w_scratch, first ? cc0 : cc1);
}

__global__ void __launch_bounds__(kChunk)
group_place2_kernel(const GroupJob j0, const GroupJob j1, int nch0, int nch1, const int32_t* __restrict__ cc0,
                    const int32_t* __restrict__ cc1) {
  pdl_wait();
  pdl_trigger();
  const bool first = static_cast<int>(blockIdx.x) < nch0;
  const GroupJob& j = first ? j0 : j1;
  int pos;
  group_place_chunk(j.idx, j.n_rows, j.slots, j.num_groups, first ? nch0 : nch1, first ? blockIdx.x : blockIdx.x - nch0,
                    j.rank_scratch, j.w_scratch, first ? cc0 : cc1, j.offsets, j.perm_row, j.perm_slot, j.perm_w,
                    j.inv, pos);
}

// One warp per permuted row: the source row index is read once, then every
// lane moves 16-byte vectors c, c+32, ... with four loads in flight before
// their stores.
template <typename V>
__global__ void gather_rows_kernel(const V* __restrict__ src, int vec_per_row,
                                   const int32_t* __restrict__ perm_row,
                                   const int32_t* __restrict__ offsets, int G, int max_rows,
                                   V* __restrict__ dst) {
  pdl_wait();
  pdl_trigger();
  const int rows = min(offsets[G], max_rows);
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  for (int r = blockIdx.x * wpb + (threadIdx.x >> 5); r < rows; r += gridDim.x * wpb) {
    const V* s = src + static_cast<int64_t>(perm_row[r]) * vec_per_row;
    V* d = dst + static_cast<int64_t>(r) * vec_per_row;
    int c = lane;
    for (; c + 96 < vec_per_row; c += 128) {
      const V v0 = s[c], v1 = s[c + 32], v2 = s[c + 64], v3 = s[c + 96];
      d[c] = v0;
      d[c + 32] = v1;
      d[c + 64] = v2;
      d[c + 96] = v3;
    }
    for (; c < vec_per_row; c += 32) d[c] = s[c];
  }
}

}  // namespace sb

using namespace sb;

extern "C" SB_API size_t sb_group_workspace_bytes(int n_rows, int slots, int num_groups) {
  const size_t total = static_cast<size_t>(n_rows > 0 ? n_rows : 0) * (slots > 0 ? slots : 0);
  const size_t ctas = (total + kChunk - 1) / kChunk;  // chunks of the two-pass path (>= the rank path's CTAs)
  const size_t groups = num_groups > 0 ? static_cast<size_t>(num_groups) : 1;
  return kStatusBytes + align_up(total * sizeof(int32_t), 256) + align_up(total * sizeof(float), 256) +
         align_up(ctas * groups * sizeof(int32_t), 256) + 256;
}

extern "C" SB_API int sb_group(const int32_t* idx, const float* w, int n_rows, int slots,
                               int num_groups, int flags, int32_t* offsets, int32_t* perm_row,
                               int32_t* perm_slot, float* perm_w, int32_t* inv, void* workspace,
                               size_t workspace_bytes, void* stream) {
  if (n_rows < 0 || slots <= 0 || num_groups <= 0 || num_groups > kGroupMaxG || !offsets ||
      (n_rows > 0 && (!idx || !perm_row || !perm_slot || !perm_w || !inv)))
    return SB_ERR_ARG;
  const size_t need = sb_group_workspace_bytes(n_rows, slots, num_groups);
  if (!workspace || workspace_bytes < need) return SB_ERR_WORKSPACE;
  Carver c(workspace, workspace_bytes);
  c.take<char>(kStatusBytes);
  const size_t total = static_cast<size_t>(n_rows) * slots;
  int32_t* rank_scratch = c.take<int32_t>(total);
  float* w_scratch = c.take<float>(total);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (total <= kGroupSingleCtaMax) {
    // One CTA; as many threads as entries (rounded to warps, 64..1024): fewer warps
    // to synchronise and scan when a decode batch has only a few hundred entries.
    int threads = static_cast<int>(((total + 31) / 32) * 32);
    threads = threads < 64 ? 64 : (threads > kGroupThreads ? kGroupThreads : threads);
    return launch(group_kernel, dim3(1), dim3(threads), 0, st, idx, w, n_rows, slots, num_groups, flags, offsets,
                  perm_row, perm_slot, perm_w, inv, rank_scratch, w_scratch);
  }
  const int nchunks = static_cast<int>((total + kChunk - 1) / kChunk);
  int32_t* chunk_count = c.take<int32_t>(static_cast<size_t>(nchunks) * num_groups);
  int rc = launch(group_count_kernel, dim3(nchunks), dim3(kChunk), 0, st, idx, w, n_rows, slots, num_groups, flags,
                  rank_scratch, w_scratch, chunk_count);
  if (rc) return rc;
  return launch(group_place_kernel, dim3(nchunks), dim3(kChunk), 0, st, idx, n_rows, slots, num_groups, nchunks,
                static_cast<const int32_t*>(rank_scratch), static_cast<const float*>(w_scratch),
                static_cast<const int32_t*>(chunk_count), offsets, perm_row, perm_slot, perm_w, inv);
}

namespace sb {
// ---------------------------------------------------------------------------
// Groupings whose ids are derived in the same kernel (one CTA, <= kDerivedMax
// entries): the ids and weights are staged in shared memory, then grouped as
// sb_group groups them.
//   mode 0 (expert-parallel owner side): ids / weights from the metadata of
//     packed rows (K int32 local ids, then K fp32 weights, at meta_off of each
//     row of `pitch` bytes); ids outside [0, G) are skipped.
//   mode 1 (expert-parallel sender side): id = top_idx % G (the owning rank of
//     the expert, G = world), no weights; negative experts are skipped.
constexpr int kDerivedMax = 1024;  // staging + group_one_cta fit the 48 KB of static shared memory

__global__ void __launch_bounds__(kGroupThreads, 1)
derived_group_kernel(int mode, const uint8_t* __restrict__ rows, int64_t pitch, int64_t meta_off,
                     const int32_t* __restrict__ top_idx, int num_experts, int n, int K, int G, int flags,
                     int32_t* __restrict__ offsets, int32_t* __restrict__ perm_row, int32_t* __restrict__ perm_slot,
                     float* __restrict__ perm_w, int32_t* __restrict__ inv, int32_t* __restrict__ rank_scratch,
                     float* __restrict__ w_scratch, uint8_t* wait_region, int64_t ctrl_off, int wait_world,
                     int* status) {
  __shared__ int32_t s_ids[kDerivedMax];
  __shared__ float s_w[kDerivedMax];
  pdl_wait();
  pdl_trigger();
  if (wait_region) {
    // peer transport: the rows are there once every rank raised its dispatch flag
    const uint32_t target = ep_wait_target(wait_region, ctrl_off, wait_world, 0);
    ep_wait_cta(wait_region, ctrl_off, wait_world, 0, target, status);
    if (threadIdx.x == 0) ep_seen(wait_region, ctrl_off, wait_world)[0] = target;
  }
  const int total = n * K;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    if (mode == 0) {
      const int r = i / K, k = i - r * K;
      const uint8_t* m = rows + static_cast<int64_t>(r) * pitch + meta_off;
      const int e = reinterpret_cast<const int32_t*>(m)[k];
      s_ids[i] = (e >= 0 && e < G) ? e : -1;
      s_w[i] = reinterpret_cast<const float*>(m + static_cast<int64_t>(K) * 4)[k];
    } else {
      const int e = top_idx[i];
      s_ids[i] = (e >= 0 && e < num_experts) ? e % G : -1;
      s_w[i] = 1.f;
    }
  }
  __syncthreads();
  group_one_cta(s_ids, mode == 0 ? s_w : nullptr, n, K, G, flags, offsets, perm_row, perm_slot, perm_w, inv,
                rank_scratch, w_scratch);
}

int derived_group_launch(int mode, const void* rows, int64_t pitch, int64_t meta_off, const int32_t* top_idx,
                         int num_experts, int n, int K, int G, int flags, int32_t* offsets, int32_t* perm_row,
                         int32_t* perm_slot, float* perm_w, int32_t* inv, void* workspace, size_t workspace_bytes,
                         cudaStream_t st, void* wait_region, int64_t ctrl_off, int wait_world, int* status) {
  const int64_t total = static_cast<int64_t>(n) * K;
  if (total > kDerivedMax || G > kGroupMaxG || n <= 0) return SB_ERR_UNSUPPORTED;
  if (workspace_bytes < sb_group_workspace_bytes(n, K, G)) return SB_ERR_WORKSPACE;
  Carver c(workspace, workspace_bytes);  // the scratch layout of sb_group
  c.take<char>(kStatusBytes);
  int32_t* rank_scratch = c.take<int32_t>(total);
  float* w_scratch = c.take<float>(total);
  int threads = static_cast<int>(((total + 31) / 32) * 32);
  threads = threads < 64 ? 64 : (threads > kGroupThreads ? kGroupThreads : threads);
  return launch(derived_group_kernel, dim3(1), dim3(threads), 0, st, mode, static_cast<const uint8_t*>(rows), pitch,
                meta_off, top_idx, num_experts, n, K, G, flags, offsets, perm_row, perm_slot, perm_w, inv, rank_scratch,
                w_scratch, static_cast<uint8_t*>(wait_region), ctrl_off, wait_world, status);
}

int group_pair_launch(const GroupJob& j0, const GroupJob& j1, cudaStream_t st) {
  const int64_t t0 = static_cast<int64_t>(j0.n_rows) * j0.slots, t1 = static_cast<int64_t>(j1.n_rows) * j1.slots;
  const int64_t tmax = t0 > t1 ? t0 : t1;
  if (tmax > static_cast<int64_t>(kGroupPairMax) || j0.num_groups > kGroupMaxG || j1.num_groups > kGroupMaxG)
    return SB_ERR_UNSUPPORTED;
  int threads = static_cast<int>(((tmax + 31) / 32) * 32);
  threads = threads < 64 ? 64 : (threads > kGroupThreads ? kGroupThreads : threads);
  return launch(group_pair_kernel, dim3(2), dim3(threads), 0, st, j0, j1);
}

int group_pair_multi_launch(const GroupJob& j0, const GroupJob& j1, int32_t* cc0, int32_t* cc1, cudaStream_t st) {
  if (j0.num_groups > kGroupMaxG || j1.num_groups > kGroupMaxG || j0.n_rows <= 0 || j1.n_rows <= 0 || !cc0 || !cc1)
    return SB_ERR_ARG;
  const int64_t t0 = static_cast<int64_t>(j0.n_rows) * j0.slots, t1 = static_cast<int64_t>(j1.n_rows) * j1.slots;
  const int nch0 = static_cast<int>((t0 + kChunk - 1) / kChunk), nch1 = static_cast<int>((t1 + kChunk - 1) / kChunk);
  int rc = launch(group_count2_kernel, dim3(nch0 + nch1), dim3(kChunk), 0, st, j0, j1, nch0, cc0, cc1);
  if (rc) return rc;
  return launch(group_place2_kernel, dim3(nch0 + nch1), dim3(kChunk), 0, st, j0, j1, nch0, nch1,
                static_cast<const int32_t*>(cc0), static_cast<const int32_t*>(cc1));
}

// Launch of the grouping kernel with caller-chosen scratch arrays (used by the
// no-allocation entry point, whose scratch is a fixed device array).
int group_launch_with_scratch(const int32_t* idx, const float* w, int n_rows, int slots, int num_groups, int flags,
                              int32_t* offsets, int32_t* perm_row, int32_t* perm_slot, float* perm_w, int32_t* inv,
                              int32_t* rank_scratch, float* w_scratch, cudaStream_t st) {
  const int64_t total = static_cast<int64_t>(n_rows) * slots;
  int threads = static_cast<int>(((total + 31) / 32) * 32);
  threads = threads < 64 ? 64 : (threads > kGroupThreads ? kGroupThreads : threads);
  return launch(group_kernel, dim3(1), dim3(threads), 0, st, idx, w, n_rows, slots, num_groups, flags, offsets,
                perm_row, perm_slot, perm_w, inv, rank_scratch, w_scratch);
}
}  // namespace sb

extern "C" SB_API int sb_gather_rows(const void* src, int act_dtype, int cols,
                                     const int32_t* perm_row, const int32_t* offsets, int num_groups,
                                     int max_rows, void* dst, void* stream) {
  if (!src || !perm_row || !offsets || !dst || cols <= 0 || num_groups <= 0 || max_rows < 0)
    return SB_ERR_ARG;
  const int esize = act_dtype == SB_F32 ? 4 : (act_dtype == SB_BF16 ? 2 : 0);
  if (!esize || (static_cast<int64_t>(cols) * esize) % 16) return SB_ERR_ARG;
  if (max_rows == 0) return SB_OK;
  const int vpr = cols * esize / 16;
  int blocks = (max_rows + 7) / 8;  // 8 rows (warps) per CTA
  const int cap = 8 * current_sm_count();
  blocks = blocks > cap ? cap : blocks;
  return launch(gather_rows_kernel<uint4>, dim3(blocks), dim3(256), 0, static_cast<cudaStream_t>(stream),
                static_cast<const uint4*>(src), vpr, perm_row, offsets, num_groups, max_rows, static_cast<uint4*>(dst));
}
