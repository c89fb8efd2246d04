// Device side of the expert-parallel peer-memory exchange, shared by the
// packing / return kernels (sb_ep.cu), the owner's grouping (sb_group.cu) and
// the combines (sb_combine.cu).
#pragma once

#include "sb_common.cuh"

namespace sb {

// ------------------------------------------------------------------ peer exchange region
// One region per rank (cudaMalloc at set-up, mapped by the peers with CUDA
// IPC):  recv [world][cap][pitch] packed rows the peers send to this rank |
// ret [world][cap][hidden] fp32 rows the owners return to it | control:
// uint32 flag[2][world] (kind 0 dispatch, 1 return; raised by the peer q),
// uint32 seen[2] (this rank's completed waits per kind), uint32 ticket[4]
// (last-CTA counters: 0 / 1 the kernels that raise the dispatch / return
// flags, 2 / 3 multi-CTA kernels that wait for them).
struct EpRegion {
  int64_t ret_off, ctrl_off, bytes;
};
__host__ __device__ inline EpRegion ep_region(int world, int cap, int64_t pitch, int hidden) {
  EpRegion r;
  const int64_t recv = static_cast<int64_t>(world) * cap * pitch;
  r.ret_off = (recv + 255) / 256 * 256;
  const int64_t ret = static_cast<int64_t>(world) * cap * hidden * 4;
  r.ctrl_off = (r.ret_off + ret + 255) / 256 * 256;
  r.bytes = r.ctrl_off + (static_cast<int64_t>(2 * world + 6) * 4 + 255) / 256 * 256;
  return r;
}
SB_DEVINL uint32_t* ep_flags(uint8_t* region, int64_t ctrl_off, int world, int kind) {
  return reinterpret_cast<uint32_t*>(region + ctrl_off) + kind * world;
}
SB_DEVINL uint32_t* ep_seen(uint8_t* region, int64_t ctrl_off, int world) {
  return reinterpret_cast<uint32_t*>(region + ctrl_off) + 2 * world;
}
SB_DEVINL uint32_t* ep_ticket(uint8_t* region, int64_t ctrl_off, int world) {
  return reinterpret_cast<uint32_t*>(region + ctrl_off) + 2 * world + 2;
}
// Raise the `kind` flag of rank `me` in every peer's region, once all CTAs of
// the calling kernel finished their stores (last-CTA ticket in the own region).
SB_DEVINL void ep_signal_peers(uint8_t* const* regions, uint8_t* own, int64_t ctrl_off, int world, int me, int kind) {
  __shared__ bool s_last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(ep_ticket(own, ctrl_off, world) + kind, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence_system();
  for (int q = threadIdx.x; q < world; q += blockDim.x) {
    uint32_t* f = ep_flags(regions[q], ctrl_off, world, kind) + me;
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(f), "r"(1u) : "memory");
  }
  if (threadIdx.x == 0) ep_ticket(own, ctrl_off, world)[kind] = 0u;  // ready for the next launch
}


// Single-CTA wait (the whole CTA calls it): until every rank has raised this
// rank's `kind` flag once more than this rank waited for before; then counts
// the wait.  Bounded: after ~2 s SB_DEVERR_PEER_WAIT is recorded and the CTA
// goes on.  A thread spinning on one flag with acquire loads, then the CTA
// barrier, orders the peers' stores before every thread's later reads.
SB_DEVINL void ep_wait_cta(uint8_t* region, int64_t ctrl_off, int world, int kind, uint32_t target, int* status) {
  for (int q = threadIdx.x; q < world; q += blockDim.x) {
    const uint32_t* f = ep_flags(region, ctrl_off, world, kind) + q;
    const uint64_t t0 = global_ns();
    uint32_t spins = 0;
    while (true) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
      if (static_cast<int32_t>(v - target) >= 0) break;
      if (++spins > 16) __nanosleep(128);
      if ((spins & 255u) == 0 && global_ns() - t0 > kWaitLimitNs) {
        record_error(status, SB_DEVERR_PEER_WAIT);
        break;
      }
    }
  }
  __syncthreads();
}

// Target of this rank's next wait of `kind` (read before the wait; a kernel
// of several CTAs counts the wait in its last CTA, after every CTA read it).
SB_DEVINL uint32_t ep_wait_target(uint8_t* region, int64_t ctrl_off, int world, int kind) {
  return *reinterpret_cast<volatile uint32_t*>(ep_seen(region, ctrl_off, world) + kind) + 1u;
}

// End of a multi-CTA kernel that waited for `kind`: the last CTA counts the wait.
SB_DEVINL void ep_count_wait_multi(uint8_t* region, int64_t ctrl_off, int world, int kind, uint32_t target) {
  __shared__ bool s_last_w;
  __syncthreads();
  if (threadIdx.x == 0) s_last_w = atomicAdd(ep_ticket(region, ctrl_off, world) + 2 + kind, 1u) == gridDim.x - 1;
  __syncthreads();
  if (s_last_w && threadIdx.x == 0) {
    ep_seen(region, ctrl_off, world)[kind] = target;
    ep_ticket(region, ctrl_off, world)[2 + kind] = 0u;
    __threadfence();
  }
}

// Where peer-mode kernels send rows and raise flags.
struct EpPeer {
  uint8_t* const* regions;  // device array: every rank's region as mapped here
  int world, me, cap;
  int64_t ret_off, ctrl_off;
};

}  // namespace sb
