// moe_sort_align_static_scratch: the expert sort of moe_sort_align, with its
// scratch (the per-CTA expert histograms) held in a fixed device array that
// the library owns, so that the call needs no workspace and allocates nothing.
//
// Who needs it: callers that cannot allocate device memory themselves, such as
// a host framework that owns every device allocation and hands its plugins no
// workspace, or a serving process that forbids allocation once it is running
// (cudaMalloc can also synchronise the device, which such callers must avoid).
//
// What it costs: kStaticScratchInts int32 (256 KiB) of device memory on every
// GPU that loads this library, held until the process exits.
#include <mutex>

#include "../../include/moe_b200.h"
#include "internal.h"

namespace {

constexpr int kStaticScratchInts = MOE_SORT_STATIC_SCRATCH_INTS;

// One histogram region shared by every call on a device.  Each call writes
// every entry it later reads (all [CTA][expert] counts of its own launch)
// before reading it, so nothing has to be cleared between calls.
static __device__ __align__(256) int g_sort_scratch[kStaticScratchInts];

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// The device address of g_sort_scratch on the current device.  In host code
// the symbol name is only a host-side handle, so the address is looked up once
// per device (cudaGetSymbolAddress, with that device current) and cached.
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return MOE_RC_CUDA_ERROR;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_sort_scratch) != cudaSuccess || p == nullptr)
      return MOE_RC_CUDA_ERROR;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return MOE_RC_OK;
}

}  // namespace

extern "C" int moe_sort_align_static_scratch(const int32_t* topk_ids, int R, int E, int e_begin,
                                             int E_local, int32_t* counts, int32_t* offsets,
                                             int64_t* offsets64, int32_t* perm, int32_t* inv,
                                             int32_t* tiles, int max_tiles, int32_t* num_tiles,
                                             int32_t* status, cudaStream_t stream) {
  if ((R > 0 && (topk_ids == nullptr || perm == nullptr)) || counts == nullptr ||
      offsets == nullptr || tiles == nullptr || num_tiles == nullptr)
    return MOE_RC_BAD_ARGUMENT;
  if (R < 0 || E_local <= 0 || max_tiles < moe_max_tiles(R, E_local)) return MOE_RC_BAD_ARGUMENT;
  // The histograms need one int per (CTA, expert); refuse what does not fit.
  const long long need = static_cast<long long>(moe::sort_num_blocks(R)) * E_local;
  if (need > kStaticScratchInts) return MOE_RC_WORKSPACE;
  void* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc != MOE_RC_OK) return rc;
  return moe::launch_sort_align(topk_ids, R, E, e_begin, E_local, MOE_BLOCK_M, scratch, counts,
                                offsets, reinterpret_cast<long long*>(offsets64), perm, inv,
                                reinterpret_cast<int4*>(tiles), max_tiles, num_tiles, status,
                                stream);
}
