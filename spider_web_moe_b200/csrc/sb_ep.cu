// Expert-parallel dispatch packing for the token-sharded block.
//
// Rank r owns the experts e with e % world == r (spider_moe/expert_parallel.py:
// 29-30).  Each token is sent once to every rank that owns at least one of its
// routed experts: send row (q, j) of the fixed-capacity buffer [world, cap, H]
// carries the token's message row and, for each of its K slots, the owner's
// local expert id (e / world, or -1 when q does not own e) and the routing
// weight.  Rows are ordered by token inside each destination (a stable
// grouping by owner), unused rows carry id -1.  ret_pos[t, k] is where the
// owner's combined result for (token t, owner of slot k) comes back in the
// return buffer [world, cap, H] (first slot per owner; -1 for the others), so
// the epilogue sums exactly one returned row per (token, owner).
#include <cstring>

#include "sb_common.cuh"
#include "sb_ep_dev.cuh"
#include "sb_internal.h"

namespace sb {

__global__ void __launch_bounds__(256)
ep_owner_kernel(const int32_t* __restrict__ top_idx, int n, int E, int world, int32_t* __restrict__ owner) {
  pdl_wait();
  pdl_trigger();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int e = top_idx[i];
    owner[i] = (e >= 0 && e < E) ? e % world : -1;
  }
}

// Packed send row: [message row: H x act dtype | K int32 local ids | K fp32 weights | pad],
// row_pitch bytes (a multiple of 16).
template <typename T>
__global__ void __launch_bounds__(256)
ep_pack_kernel(const T* __restrict__ msgs, const int32_t* __restrict__ top_idx, const float* __restrict__ top_w,
               int n_tokens, int K, int E, int world, int cap, int H, int64_t row_pitch,
               const int32_t* __restrict__ off, const int32_t* __restrict__ prow, const int32_t* __restrict__ owner,
               const int32_t* __restrict__ inv, uint8_t* __restrict__ send, int32_t* __restrict__ ret_pos,
               uint8_t* const* __restrict__ regions, int me, int64_t ctrl_off) {
  pdl_wait();
  pdl_trigger();
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int vec = H * static_cast<int>(sizeof(T)) / 16;
  const int64_t meta = static_cast<int64_t>(H) * sizeof(T);
  // send rows, one warp per row
  for (int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < world * cap; row += warps) {
    const int q = row / cap, j = row - q * cap;
    const int cnt = off[q + 1] - off[q];
    int t = -1;
    if (j < cnt) t = prow[off[q] + j];
    // peer mode: straight into owner q's receive rows [me][j] over NVLink
    uint8_t* dst_row = regions ? regions[q] + (static_cast<int64_t>(me) * cap + j) * row_pitch
                               : send + static_cast<int64_t>(row) * row_pitch;
    if (lane < K) {
      int lid = -1;
      float wk = 0.f;
      if (t >= 0) {
        const int e = top_idx[static_cast<int64_t>(t) * K + lane];
        if (e >= 0 && e < E && e % world == q) lid = e / world;
        wk = top_w[static_cast<int64_t>(t) * K + lane];
      }
      reinterpret_cast<int32_t*>(dst_row + meta)[lane] = lid;
      reinterpret_cast<float*>(dst_row + meta + K * 4)[lane] = wk;
    }
    if (t >= 0) {
      const uint4* src = reinterpret_cast<const uint4*>(msgs + static_cast<int64_t>(t) * H);
      uint4* dst = reinterpret_cast<uint4*>(dst_row);
      for (int v = lane; v < vec; v += 32) dst[v] = src[v];
    }
  }
  // return positions, one thread per (token, slot): the owner's row of the
  // token's first slot it owns -- unless none of the token's slots it owns has
  // a positive weight (the owner's plan drops those, and returns no row)
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_tokens * K; i += gridDim.x * blockDim.x) {
    const int p = inv[i];
    const int e = top_idx[i];
    const int q = (e >= 0 && e < E) ? e % world : -1;
    bool any_pos = false;
    if (p >= 0 && q >= 0) {
      const int64_t t0 = static_cast<int64_t>(i / K) * K;
      for (int k2 = 0; k2 < K; ++k2) {
        const int e2 = top_idx[t0 + k2];
        if (e2 >= 0 && e2 < E && e2 % world == q && top_w[t0 + k2] > 0.f) any_pos = true;
      }
    }
    ret_pos[i] = any_pos ? q * cap + (p - off[q]) : -1;
  }
  if (regions) ep_signal_peers(regions, regions[me], ctrl_off, world, me, 0);
}

// Owner -> sources: rows [q][cap][H] of this rank's expert results go to rank
// q's return rows [me][cap][H], then the return flag is raised in every peer.
__global__ void __launch_bounds__(256)
ep_return_kernel(const float4* __restrict__ out, int world, int me, int cap, int hidden, int64_t ret_off,
                 int64_t ctrl_off, uint8_t* const* __restrict__ regions) {
  pdl_wait();
  pdl_trigger();
  const int vec = hidden / 4;
  const int64_t n = static_cast<int64_t>(world) * cap * vec;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / vec;
    const int q = static_cast<int>(row / cap), j = static_cast<int>(row - static_cast<int64_t>(q) * cap);
    const int c = static_cast<int>(i - row * vec);
    float4* dst = reinterpret_cast<float4*>(regions[q] + ret_off) + (static_cast<int64_t>(me) * cap + j) * vec + c;
    *dst = out[i];
  }
  ep_signal_peers(regions, regions[me], ctrl_off, world, me, 1);
}

// Wait until every rank raised this rank's `kind` flag once more than this
// rank has waited for before (bounded: after ~2 s the status records
// SB_DEVERR_PEER_WAIT and the kernel returns), then count the wait.
__global__ void __launch_bounds__(256)
ep_wait_kernel(uint8_t* __restrict__ region, int64_t ctrl_off, int world, int kind, int* status) {
  pdl_wait();
  pdl_trigger();
  const uint32_t target = ep_wait_target(region, ctrl_off, world, kind);
  ep_wait_cta(region, ctrl_off, world, kind, target, status);
  if (threadIdx.x == 0) ep_seen(region, ctrl_off, world)[kind] = target;
  __threadfence_system();
}

struct EpBuffers {
  int32_t *owner, *off, *prow, *pslot, *inv;
  float* pw;
  void* group_ws;
  size_t group_ws_bytes;
};

static size_t carve_ep(int n, int K, int world, void* base, size_t size, EpBuffers* b) {
  Carver c(base, size);
  c.take<char>(kStatusBytes);
  const size_t e = static_cast<size_t>(n) * K;
  b->owner = c.take<int32_t>(e);
  b->off = c.take<int32_t>(world + 1);
  b->prow = c.take<int32_t>(e);
  b->pslot = c.take<int32_t>(e);
  b->pw = c.take<float>(e);
  b->inv = c.take<int32_t>(e);
  b->group_ws_bytes = sb_group_workspace_bytes(n, K, world);
  b->group_ws = c.take<char>(b->group_ws_bytes);
  return c.overflow ? static_cast<size_t>(-1) : align_up(c.used, 256);
}

}  // namespace sb

using namespace sb;

extern "C" SB_API size_t sb_ep_pack_workspace_bytes(int n_tokens, int top_k, int world) {
  if (n_tokens < 0 || top_k <= 0 || world <= 0) return 0;
  EpBuffers b;
  return carve_ep(n_tokens > 0 ? n_tokens : 1, top_k, world, nullptr, ~size_t(0) >> 1, &b);
}

extern "C" SB_API size_t sb_ep_row_pitch(int hidden, int act_dtype, int top_k) {
  const size_t es = act_dtype == SB_F32 ? 4 : 2;
  return align_up(static_cast<size_t>(hidden) * es + static_cast<size_t>(top_k) * 8, 16);
}

extern "C" SB_API int sb_ep_pack(const int32_t* top_idx, const float* top_w, const void* messages, int act_dtype,
                                 int n_tokens, int hidden, int top_k, int num_experts, int world, int cap,
                                 void* send, int32_t* ret_pos, void* workspace, size_t workspace_bytes,
                                 void* stream) {
  const int esize = act_dtype == SB_F32 ? 4 : (act_dtype == SB_BF16 ? 2 : 0);
  if (n_tokens < 0 || hidden <= 0 || !esize || (hidden * esize) % 16 || top_k <= 0 || top_k > 32 ||
      num_experts <= 0 || world <= 0 || world > 256 || cap < n_tokens || cap <= 0)
    return SB_ERR_ARG;
  if (world * static_cast<int64_t>(cap) > 0x7fffffff) return SB_ERR_UNSUPPORTED;
  if (!send || (n_tokens > 0 && (!top_idx || !top_w || !messages || !ret_pos))) return SB_ERR_ARG;
  EpBuffers b;
  const size_t need = carve_ep(n_tokens, top_k, world, workspace, workspace_bytes, &b);
  if (!workspace || need == static_cast<size_t>(-1) || workspace_bytes < need) return SB_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int entries = n_tokens * top_k;
  int rc = SB_OK;
  if (n_tokens > 0) {
    // owners of the tokens' experts grouped in one kernel; larger batches:
    // owner ids, then sb_group
    rc = derived_group_launch(1, nullptr, 0, 0, top_idx, num_experts, n_tokens, top_k, world, 0, b.off, b.prow,
                              b.pslot, b.pw, b.inv, b.group_ws, b.group_ws_bytes, st);
    if (rc == SB_ERR_UNSUPPORTED) {
      rc = launch(ep_owner_kernel, dim3((entries + 255) / 256), dim3(256), 0, st, top_idx, entries, num_experts,
                  world, b.owner);
      if (rc) return rc;
      rc = sb_group(b.owner, nullptr, n_tokens, top_k, world, 0, b.off, b.prow, b.pslot, b.pw, b.inv, b.group_ws,
                    b.group_ws_bytes, st);
    }
  } else {
    rc = cuda_status(cudaMemsetAsync(b.off, 0, sizeof(int32_t) * (world + 1), st));
  }
  if (rc) return rc;
  const int64_t pitch = static_cast<int64_t>(sb_ep_row_pitch(hidden, act_dtype, top_k));
  const int rows = world * cap;
  int blocks = (rows * 32 + 255) / 256;
  const int lim = 4 * current_sm_count();
  blocks = blocks > lim ? lim : (blocks < 1 ? 1 : blocks);
  if (act_dtype == SB_BF16)
    return launch(ep_pack_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, st,
                  static_cast<const __nv_bfloat16*>(messages), top_idx, top_w, n_tokens, top_k, num_experts, world,
                  cap, hidden, pitch, static_cast<const int32_t*>(b.off), static_cast<const int32_t*>(b.prow),
                  static_cast<const int32_t*>(b.owner), static_cast<const int32_t*>(b.inv),
                  static_cast<uint8_t*>(send), ret_pos, static_cast<uint8_t* const*>(nullptr), 0, int64_t(0));
  return launch(ep_pack_kernel<float>, dim3(blocks), dim3(256), 0, st, static_cast<const float*>(messages), top_idx,
                top_w, n_tokens, top_k, num_experts, world, cap, hidden, pitch, static_cast<const int32_t*>(b.off),
                static_cast<const int32_t*>(b.prow), static_cast<const int32_t*>(b.owner),
                static_cast<const int32_t*>(b.inv), static_cast<uint8_t*>(send), ret_pos,
                static_cast<uint8_t* const*>(nullptr), 0, int64_t(0));
}

// ------------------------------------------------------------------ peer exchange entry points

extern "C" SB_API size_t sb_ep_peer_region_bytes(int world, int cap, int64_t row_pitch, int hidden) {
  if (world <= 0 || world > 256 || cap <= 0 || row_pitch <= 0 || row_pitch % 16 || hidden <= 0 || hidden % 4)
    return 0;
  return static_cast<size_t>(ep_region(world, cap, row_pitch, hidden).bytes);
}

extern "C" SB_API int sb_ep_peer_create(int world, int cap, int64_t row_pitch, int hidden, void** region,
                                        void* ipc_handle) {
  const size_t bytes = sb_ep_peer_region_bytes(world, cap, row_pitch, hidden);
  if (!bytes || !region || !ipc_handle) return SB_ERR_ARG;
  *region = nullptr;
  void* p = nullptr;
  int rc = cuda_status(cudaMalloc(&p, bytes));
  if (rc) return rc;
  rc = cuda_status(cudaMemset(p, 0, bytes));  // flags, counters and tickets start at zero
  if (!rc) rc = cuda_status(cudaDeviceSynchronize());
  if (!rc) {
    cudaIpcMemHandle_t h;
    rc = cuda_status(cudaIpcGetMemHandle(&h, p));
    if (!rc) std::memcpy(ipc_handle, &h, sizeof(h));
  }
  if (rc) {
    cudaFree(p);
    return rc;
  }
  *region = p;
  return SB_OK;
}

extern "C" SB_API int sb_ep_peer_map(const void* ipc_handle, void** region) {
  if (!ipc_handle || !region) return SB_ERR_ARG;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(region, h, cudaIpcMemLazyEnablePeerAccess));
}

extern "C" SB_API int sb_ep_peer_unmap(void* region) {
  return region ? cuda_status(cudaIpcCloseMemHandle(region)) : SB_ERR_ARG;
}

extern "C" SB_API int sb_ep_peer_destroy(void* region) { return region ? cuda_status(cudaFree(region)) : SB_ERR_ARG; }

extern "C" SB_API int sb_ep_dispatch(const int32_t* top_idx, const float* top_w, const void* messages, int act_dtype,
                                     int n_tokens, int hidden, int top_k, int num_experts, int world, int rank, int cap,
                                     void* const* regions, int32_t* ret_pos, void* workspace, size_t workspace_bytes,
                                     void* stream) {
  const int esize = act_dtype == SB_F32 ? 4 : (act_dtype == SB_BF16 ? 2 : 0);
  if (n_tokens < 0 || hidden <= 0 || !esize || (hidden * esize) % 16 || top_k <= 0 || top_k > 32 ||
      num_experts <= 0 || world <= 0 || world > 256 || rank < 0 || rank >= world || cap < n_tokens || cap <= 0 ||
      !regions)
    return SB_ERR_ARG;
  if (world * static_cast<int64_t>(cap) > 0x7fffffff) return SB_ERR_UNSUPPORTED;
  if (n_tokens > 0 && (!top_idx || !top_w || !messages || !ret_pos)) return SB_ERR_ARG;
  EpBuffers b;
  const size_t need = carve_ep(n_tokens, top_k, world, workspace, workspace_bytes, &b);
  if (!workspace || need == static_cast<size_t>(-1) || workspace_bytes < need) return SB_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int entries = n_tokens * top_k;
  int rc = SB_OK;
  if (n_tokens > 0) {
    // owners of the tokens' experts grouped in one kernel; larger batches:
    // owner ids, then sb_group
    rc = derived_group_launch(1, nullptr, 0, 0, top_idx, num_experts, n_tokens, top_k, world, 0, b.off, b.prow,
                              b.pslot, b.pw, b.inv, b.group_ws, b.group_ws_bytes, st);
    if (rc == SB_ERR_UNSUPPORTED) {
      rc = launch(ep_owner_kernel, dim3((entries + 255) / 256), dim3(256), 0, st, top_idx, entries, num_experts,
                  world, b.owner);
      if (rc) return rc;
      rc = sb_group(b.owner, nullptr, n_tokens, top_k, world, 0, b.off, b.prow, b.pslot, b.pw, b.inv, b.group_ws,
                    b.group_ws_bytes, st);
    }
  } else {
    rc = cuda_status(cudaMemsetAsync(b.off, 0, sizeof(int32_t) * (world + 1), st));
  }
  if (rc) return rc;
  const int64_t pitch = static_cast<int64_t>(sb_ep_row_pitch(hidden, act_dtype, top_k));
  const int64_t ctrl_off = ep_region(world, cap, pitch, hidden).ctrl_off;
  const int rows = world * cap;
  int blocks = (rows * 32 + 255) / 256;
  const int lim = 4 * current_sm_count();
  blocks = blocks > lim ? lim : (blocks < 1 ? 1 : blocks);
  uint8_t* const* regs = reinterpret_cast<uint8_t* const*>(regions);
  if (act_dtype == SB_BF16)
    return launch(ep_pack_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, st,
                  static_cast<const __nv_bfloat16*>(messages), top_idx, top_w, n_tokens, top_k, num_experts, world,
                  cap, hidden, pitch, static_cast<const int32_t*>(b.off), static_cast<const int32_t*>(b.prow),
                  static_cast<const int32_t*>(b.owner), static_cast<const int32_t*>(b.inv),
                  static_cast<uint8_t*>(nullptr), ret_pos, regs, rank, ctrl_off);
  return launch(ep_pack_kernel<float>, dim3(blocks), dim3(256), 0, st, static_cast<const float*>(messages), top_idx,
                top_w, n_tokens, top_k, num_experts, world, cap, hidden, pitch, static_cast<const int32_t*>(b.off),
                static_cast<const int32_t*>(b.prow), static_cast<const int32_t*>(b.owner),
                static_cast<const int32_t*>(b.inv), static_cast<uint8_t*>(nullptr), ret_pos, regs, rank, ctrl_off);
}

extern "C" SB_API int sb_ep_wait(void* region, int world, int cap, int64_t row_pitch, int hidden, int kind,
                                 int* status, void* stream) {
  if (!region || kind < 0 || kind > 1 || !sb_ep_peer_region_bytes(world, cap, row_pitch, hidden)) return SB_ERR_ARG;
  const int64_t ctrl_off = ep_region(world, cap, row_pitch, hidden).ctrl_off;
  return launch(ep_wait_kernel, dim3(1), dim3(world < 32 ? 32 : (world + 31) / 32 * 32), 0,
                static_cast<cudaStream_t>(stream), static_cast<uint8_t*>(region), ctrl_off, world, kind, status);
}

extern "C" SB_API int sb_ep_return(const float* rows_out, int world, int rank, int cap, int64_t row_pitch, int hidden,
                                   void* const* regions, void* stream) {
  if (!rows_out || !regions || rank < 0 || rank >= world || !sb_ep_peer_region_bytes(world, cap, row_pitch, hidden))
    return SB_ERR_ARG;
  const EpRegion r = ep_region(world, cap, row_pitch, hidden);
  const int64_t n = static_cast<int64_t>(world) * cap * (hidden / 4);
  int blocks = static_cast<int>((n + 255) / 256);
  const int lim = 4 * current_sm_count();
  blocks = blocks > lim ? lim : (blocks < 1 ? 1 : blocks);
  return launch(ep_return_kernel, dim3(blocks), dim3(256), 0, static_cast<cudaStream_t>(stream),
                reinterpret_cast<const float4*>(rows_out), world, rank, cap, hidden, r.ret_off, r.ctrl_off,
                reinterpret_cast<uint8_t* const*>(regions));
}

namespace sb {
void ep_region_offsets(int world, int cap, int64_t row_pitch, int hidden, int64_t* ret_off, int64_t* ctrl_off) {
  const EpRegion r = ep_region(world, cap, row_pitch, hidden);
  *ret_off = r.ret_off;
  *ctrl_off = r.ctrl_off;
}
}  // namespace sb
