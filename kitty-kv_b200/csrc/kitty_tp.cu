// Tensor-parallel output exchange over peer memory (kitty_tp_* in the C ABI).
//
// Under KV-head sharding every rank decodes its own query heads and all ranks need
// all heads.  Each rank owns an exchange region (one cudaMalloc, shared with the
// other processes through CUDA IPC):
//
//   [buffer 0][buffer 1][arrival counters: one u32 per source rank][epoch][done]
//
// A call with epoch e = epoch + 1 runs two kernels:
//   tp_put_kernel   - CTA (peer p, part): 16-byte NVLink stores of this rank's slice
//                     into buffer (e & 1) of rank p, then every thread fences at
//                     system scope, and thread 0 adds 1 to rank p's arrival counter
//                     for this rank (so rank p sees e * parts when all parts landed);
//   tp_wait_kernel  - polls this rank's own counters (acquire, bounded) until every
//                     source rank reached e * parts, copies buffer (e & 1) into the
//                     caller's output and, in the last CTA to finish, advances the
//                     epoch.
// The counters only grow, so no reset is needed between calls, and the epoch lives
// in device memory, so the same launches can be captured in a CUDA graph and
// replayed.  Alternating buffers make running ahead safe: rank r can store epoch
// e + 1 only after rank p's epoch-e stores arrived, which p's stream issues after
// it has finished with the buffer that e + 1 overwrites (epoch e - 1's).
#include <cuda_runtime.h>

#include <cstring>

#include "kitty_common.cuh"

namespace kitty {

__device__ unsigned int g_tp_error = 0;   // bit 6: a rank's arrival did not come in time

namespace {

constexpr int kTpThreads = 256;
constexpr uint32_t kErrTpTimeout = 1u << 6;
constexpr int kTpPollLimit = 1 << 24;   // x ~64 ns sleeps: about a second

__host__ __device__ inline uint64_t tp_buffer_bytes(uint64_t data_bytes) { return (data_bytes + 255) & ~uint64_t(255); }
__host__ __device__ inline uint64_t tp_counters_offset(uint64_t data_bytes) { return 2 * tp_buffer_bytes(data_bytes); }

// parts (CTAs) per destination rank of the stores: ~16 KB each, 1..16
inline int tp_parts(uint64_t src_bytes) {
  const uint64_t p = (src_bytes + 16383) / 16384;
  return int(p < 1 ? 1 : p > 16 ? 16 : p);
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kTpThreads) tp_put_kernel(KittyTpGatherArgs a, int parts) {
  const int p = blockIdx.x / parts, part = blockIdx.x - p * parts;
  const uint64_t off_c = tp_counters_offset(a.data_bytes);
  const uint8_t* own = static_cast<const uint8_t*>(a.region[a.rank]);
  const uint32_t e = *reinterpret_cast<const volatile uint32_t*>(own + off_c + 4 * KITTY_TP_MAX_RANKS) + 1u;
  uint8_t* peer = static_cast<uint8_t*>(a.region[p]);
  uint4* dst = reinterpret_cast<uint4*>(peer + (e & 1u) * tp_buffer_bytes(a.data_bytes) + a.dst_offset);
  const uint4* src = static_cast<const uint4*>(a.src);
  const uint64_t n16 = a.src_bytes / 16;
  for (uint64_t i = uint64_t(part) * kTpThreads + threadIdx.x; i < n16; i += uint64_t(parts) * kTpThreads)
    dst[i] = src[i];
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) atomicAdd_system(reinterpret_cast<unsigned int*>(peer + off_c) + a.rank, 1u);
}

__global__ void __launch_bounds__(kTpThreads) tp_wait_kernel(KittyTpGatherArgs a, int parts) {
  const uint64_t off_c = tp_counters_offset(a.data_bytes);
  uint8_t* own = static_cast<uint8_t*>(a.region[a.rank]);
  uint32_t* counters = reinterpret_cast<uint32_t*>(own + off_c);
  uint32_t* epoch = counters + KITTY_TP_MAX_RANKS;
  uint32_t* done = epoch + 1;
  const uint32_t e = *reinterpret_cast<const volatile uint32_t*>(epoch) + 1u;
  const uint32_t target = e * uint32_t(parts);
  if (threadIdx.x < a.world) {
    int it = 0;
    while (int32_t(ld_acquire_sys(counters + threadIdx.x) - target) < 0) {
      if (++it >= kTpPollLimit) {
        atomicOr(&g_tp_error, kErrTpTimeout);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  const uint4* src = reinterpret_cast<const uint4*>(own + (e & 1u) * tp_buffer_bytes(a.data_bytes));
  uint4* dst = static_cast<uint4*>(a.dst);
  const uint64_t n16 = a.data_bytes / 16;
  for (uint64_t i = uint64_t(blockIdx.x) * kTpThreads + threadIdx.x; i < n16; i += uint64_t(gridDim.x) * kTpThreads)
    dst[i] = __ldcg(src + i);   // L2: the peers' stores land there
  __syncthreads();
  if (threadIdx.x == 0) {
    // every CTA read the epoch before arriving here: the last one advances it
    __threadfence();
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      *done = 0u;
      *reinterpret_cast<volatile uint32_t*>(epoch) = e;
      __threadfence();
    }
  }
}

}  // namespace

int read_tp_error(uint32_t* flags, int clear) {
  unsigned int v = 0;
  cudaError_t err = cudaMemcpyFromSymbol(&v, g_tp_error, sizeof(v));
  if (err != cudaSuccess) return fail(KITTY_ERR_CUDA, std::string("read tp error flags: ") + cudaGetErrorString(err));
  if (clear && v) {
    const unsigned int zero = 0;
    err = cudaMemcpyToSymbol(g_tp_error, &zero, sizeof(zero));
    if (err != cudaSuccess) return fail(KITTY_ERR_CUDA, std::string("clear tp error flags: ") + cudaGetErrorString(err));
  }
  *flags = v;
  return KITTY_OK;
}

}  // namespace kitty

using kitty::fail;

extern "C" {

size_t kitty_tp_region_bytes(uint64_t data_bytes) {
  return size_t(kitty::tp_counters_offset(data_bytes) + 256);
}

int kitty_tp_region_alloc(uint64_t data_bytes, void** region) {
  kitty::clear_error();
  if (!region) return fail(KITTY_ERR_INVALID_ARGUMENT, "tp_region_alloc: region is NULL");
  *region = nullptr;
  if (data_bytes == 0 || data_bytes % 16 != 0)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "tp_region_alloc: data_bytes must be a positive multiple of 16");
  const size_t n = kitty_tp_region_bytes(data_bytes);
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, n);
  if (e != cudaSuccess) return fail(KITTY_ERR_CUDA, std::string("tp_region_alloc: ") + cudaGetErrorString(e));
  e = cudaMemset(p, 0, n);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(KITTY_ERR_CUDA, std::string("tp_region_alloc: ") + cudaGetErrorString(e));
  }
  *region = p;
  return KITTY_OK;
}

int kitty_tp_region_free(void* region) {
  kitty::clear_error();
  if (!region) return KITTY_OK;
  const cudaError_t e = cudaFree(region);
  return e == cudaSuccess ? KITTY_OK : fail(KITTY_ERR_CUDA, std::string("tp_region_free: ") + cudaGetErrorString(e));
}

int kitty_tp_ipc_handle(void* region, void* handle) {
  kitty::clear_error();
  if (!region || !handle) return fail(KITTY_ERR_INVALID_ARGUMENT, "tp_ipc_handle: NULL argument");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, region);
  if (e != cudaSuccess) return fail(KITTY_ERR_CUDA, std::string("tp_ipc_handle: ") + cudaGetErrorString(e));
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  std::memcpy(handle, &h, sizeof(h));
  return KITTY_OK;
}

int kitty_tp_ipc_open(const void* handle, void** region) {
  kitty::clear_error();
  if (!handle || !region) return fail(KITTY_ERR_INVALID_ARGUMENT, "tp_ipc_open: NULL argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(KITTY_ERR_CUDA, std::string("tp_ipc_open: ") + cudaGetErrorString(e));
  *region = p;
  return KITTY_OK;
}

int kitty_tp_ipc_close(void* region) {
  kitty::clear_error();
  if (!region) return KITTY_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(region);
  return e == cudaSuccess ? KITTY_OK : fail(KITTY_ERR_CUDA, std::string("tp_ipc_close: ") + cudaGetErrorString(e));
}

int kitty_tp_allgather(const KittyTpGatherArgs* a, void* stream) {
  kitty::clear_error();
  if (!a) return fail(KITTY_ERR_INVALID_ARGUMENT, "tp_allgather: args is NULL");
  if (a->world < 1 || a->world > KITTY_TP_MAX_RANKS || a->rank < 0 || a->rank >= a->world)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "tp_allgather: world must be 1..8 and 0 <= rank < world");
  for (int r = 0; r < a->world; ++r)
    if (!a->region[r] || !kitty::aligned(a->region[r], 256))
      return fail(KITTY_ERR_INVALID_ARGUMENT, "tp_allgather: missing or unaligned region");
  if (!a->src || !a->dst || !kitty::aligned(a->src, 16) || !kitty::aligned(a->dst, 16))
    return fail(KITTY_ERR_INVALID_ARGUMENT, "tp_allgather: src and dst must be 16-byte aligned device pointers");
  if (a->data_bytes == 0 || a->data_bytes % 16 || a->src_bytes == 0 || a->src_bytes % 16 || a->dst_offset % 16 ||
      a->dst_offset + a->src_bytes > a->data_bytes)
    return fail(KITTY_ERR_INVALID_ARGUMENT,
                "tp_allgather: sizes must be multiples of 16 and the slice must lie inside the output");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int parts = kitty::tp_parts(a->src_bytes);
  kitty::tp_put_kernel<<<a->world * parts, kitty::kTpThreads, 0, s>>>(*a, parts);
  int rc = kitty::check_launch("tp_put_kernel");
  if (rc != KITTY_OK) return rc;
  const uint64_t per_cta = uint64_t(kitty::kTpThreads) * 16 * 4;
  const int grid = int(std::min<uint64_t>(64, std::max<uint64_t>(1, (a->data_bytes + per_cta - 1) / per_cta)));
  kitty::tp_wait_kernel<<<grid, kitty::kTpThreads, 0, s>>>(*a, parts);
  return kitty::check_launch("tp_wait_kernel");
}

}  // extern "C"
