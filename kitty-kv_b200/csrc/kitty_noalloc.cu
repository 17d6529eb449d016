// kitty_paged_decode_noalloc: the paged decode entry point for callers that
// cannot allocate device memory.
//
// Some callers cannot call cudaMalloc or hand out a workspace.  Examples: a
// serving engine that owns all device memory through its own arena and forbids
// allocation on the decode path, or host code driving the library through a
// thin FFI without a device allocator.  This entry point runs exactly the same
// kernels as kitty_paged_decode, but its split-K partial results (per split:
// running max, running sum and the unnormalised accumulator) live in a
// file-scope static device array of kNoAllocScratchBytes (8 MiB) instead of a
// caller-provided workspace.
//
// Properties of the static scratch:
//   * every GPU that loads the library holds the 8 MiB until the process exits;
//   * its device address is looked up once per device, on the first call made
//     with that device current (cudaGetSymbolAddress); make that first call
//     before any stream capture.  The address is cached for the life of the
//     process: after cudaDeviceReset (or any teardown of the device's primary
//     context) the module is loaded again and the cached address is stale, so
//     do not call this entry point after resetting a device;
//   * all calls share it, and it keeps the previous call's contents.  Nothing in
//     it needs to start at zero: every split writes all of its partial results
//     before the merge kernel reads them.  Calls whose kernels overlap on the GPU
//     (different streams, or other threads) race on it; order them.
//   * when the library picks the split count (num_splits == 0) it is lowered to
//     the largest count whose partials fit; an explicit num_splits whose
//     partials do not fit is rejected with KITTY_ERR_WORKSPACE.
// No cudaMalloc, cudaFree or allocating library call is made.

#include <mutex>

#include "kitty_common.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return kitty::fail(KITTY_ERR_CUDA, std::string("paged_decode_noalloc: cudaGetDevice: ") +
                                                              cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return kitty::fail(KITTY_ERR_UNSUPPORTED, "paged_decode_noalloc: device ordinal above 63");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return kitty::fail(KITTY_ERR_CUDA, std::string("paged_decode_noalloc: cudaGetSymbolAddress: ") +
                                             cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return KITTY_OK;
}

}  // namespace

extern "C" int kitty_paged_decode_noalloc(const KittyDecodeArgs* args, void* stream) {
  if (!args) return kitty::fail(KITTY_ERR_INVALID_ARGUMENT, "paged_decode_noalloc: args is NULL");
  KittyDecodeArgs a = *args;
  size_t need = 0;
  int32_t splits = 0;
  int rc = kitty_paged_decode_workspace_size(&a, &need, &splits);
  if (rc != KITTY_OK) return rc;
  if (need > kNoAllocScratchBytes) {
    if (args->num_splits > 0) {
      return kitty::fail(KITTY_ERR_WORKSPACE,
                         "paged_decode_noalloc: num_splits=" + std::to_string(args->num_splits) + " needs " +
                             std::to_string(need) + " bytes of scratch; the static scratch holds " +
                             std::to_string(kNoAllocScratchBytes) + " (pass num_splits=0 to let it fit)");
    }
    // the largest requested split count whose partials fit: the plan's slot count, and
    // so the bytes, never shrink as the request grows, so a binary search over
    // [1, splits - 1] checks about log2(splits) plans instead of stepping down by one
    int32_t lo = 1, hi = splits - 1, best = 0;
    size_t best_need = 0, tried_need = need;
    int32_t tried_splits = splits;
    while (lo <= hi) {
      const int32_t mid = lo + (hi - lo) / 2;
      a.num_splits = mid;
      size_t n = 0;
      int32_t s = 0;
      rc = kitty_paged_decode_workspace_size(&a, &n, &s);
      if (rc != KITTY_OK) return rc;
      if (n <= kNoAllocScratchBytes) {
        best = mid, best_need = n;
        lo = mid + 1;
      } else {
        tried_need = n, tried_splits = s;
        hi = mid - 1;
      }
    }
    if (best == 0)
      return kitty::fail(KITTY_ERR_WORKSPACE,
                         "paged_decode_noalloc: the smallest split plan (" + std::to_string(tried_splits) +
                             " partial slots per sequence and KV head) needs " + std::to_string(tried_need) +
                             " bytes of scratch; the static scratch holds " + std::to_string(kNoAllocScratchBytes));
    a.num_splits = best;
    need = best_need;
  }
  void* scratch = nullptr;
  if (need > 0) {
    rc = scratch_for_current_device(&scratch);
    if (rc != KITTY_OK) return rc;
  }
  a.workspace = scratch;
  a.workspace_bytes = need > 0 ? kNoAllocScratchBytes : 0;
  return kitty_paged_decode(&a, stream);
}
