// sb_group_noalloc: the dispatch-plan grouping of sb_group for callers that
// cannot hand the library a device workspace.
//
// Some callers have no way to allocate device memory: a thin C / ctypes / cgo
// binding that only forwards pointers it was given and owns no GPU allocator,
// or a host process whose device memory is all reserved up front by another
// allocator's pool.  For them this entry point keeps its scratch (one int32
// rank and one float weight per entry) in a fixed array that lives in the
// library's device image, so nothing is allocated per call.
//
// Limits and sharing:
// * at most SB_GROUP_NOALLOC_MAX_ENTRIES (n_rows * slots) entries; larger
//   inputs are rejected with SB_ERR_WORKSPACE before anything is launched;
// * the array exists once per device that loads the library and stays
//   allocated until the process exits;
// * every call on a device uses the same array, which keeps whatever the last
//   call left there.  Nothing in it needs to start at zero: the kernel writes
//   each entry it later reads within the same launch.  Two calls whose
//   kernels can overlap on the GPU (for example on two streams with no
//   ordering between them) race on the array, so order such calls;
// * the first call on each device looks up the array's device address (with
//   that device current) and caches it; make that first call before capturing
//   a stream.  The cache is keyed by device ordinal for the life of the
//   process, so it assumes the CUDA runtime's primary context (the one the
//   runtime API uses) and no cudaDeviceReset afterwards: either would leave a
//   stale address behind.
#include <mutex>

#include "sb_common.cuh"
#include "sb_internal.h"

namespace {

constexpr size_t kMaxEntries = SB_GROUP_NOALLOC_MAX_ENTRIES;
constexpr size_t kRankBytes = kMaxEntries * sizeof(int32_t);

// Scratch: ranks [kMaxEntries] int32 followed by summed weights [kMaxEntries] float.
static __device__ __align__(256) unsigned char g_group_scratch[kMaxEntries * (sizeof(int32_t) + sizeof(float))];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {nullptr};

// Device address of g_group_scratch on the current device (looked up once).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return sb::cuda_status(e);
  if (dev < 0 || dev >= kMaxDevices) return SB_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_group_scratch);
    if (e != cudaSuccess) return sb::cuda_status(e);
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return SB_OK;
}

}  // namespace

extern "C" SB_API int sb_group_noalloc(const int32_t* idx, const float* w, int n_rows, int slots, int num_groups,
                                       int flags, int32_t* offsets, int32_t* perm_row, int32_t* perm_slot,
                                       float* perm_w, int32_t* inv, void* stream) {
  if (n_rows < 0 || slots <= 0 || num_groups <= 0 || num_groups > 256 || !offsets ||
      (n_rows > 0 && (!idx || !perm_row || !perm_slot || !perm_w || !inv)))
    return SB_ERR_ARG;
  const size_t total = static_cast<size_t>(n_rows) * static_cast<size_t>(slots);
  if (total > kMaxEntries) return SB_ERR_WORKSPACE;
  void* base = nullptr;
  const int rc = scratch_address(&base);
  if (rc != SB_OK) return rc;
  int32_t* rank_scratch = static_cast<int32_t*>(base);
  float* w_scratch = reinterpret_cast<float*>(static_cast<unsigned char*>(base) + kRankBytes);
  return sb::group_launch_with_scratch(idx, w, n_rows, slots, num_groups, flags, offsets, perm_row, perm_slot,
                                       perm_w, inv, rank_scratch, w_scratch, static_cast<cudaStream_t>(stream));
}
