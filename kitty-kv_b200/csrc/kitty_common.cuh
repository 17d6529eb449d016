// Shared helpers for the Kitty B200 kernels: error reporting for the C ABI,
// fp16 bit helpers and the torch-compatible float32 clamps used by the
// quantisers.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/kitty_b200.h"

namespace kitty {

// Thread-local last error message behind kitty_last_error().
void set_error(const std::string& msg);
void clear_error();
const char* last_error();

inline int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

inline int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return fail(KITTY_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  }
  return KITTY_OK;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// torch.maximum / torch.minimum semantics: NaN in either operand propagates.
__device__ __forceinline__ float tmax(float a, float b) {
  return (a != a) ? a : ((b != b) ? b : fmaxf(a, b));
}
__device__ __forceinline__ float tmin(float a, float b) {
  return (a != a) ? a : ((b != b) ? b : fminf(a, b));
}
// x.clamp(min=lo): values below lo become lo, NaN stays NaN.
__device__ __forceinline__ float clamp_min(float x, float lo) { return (x < lo) ? lo : x; }

// float -> uint8 code for a value already clamped to [0, maxq] (NaN -> 0).
__device__ __forceinline__ uint32_t to_code(float x) {
  return (x == x) ? static_cast<uint32_t>(x) : 0u;
}

__device__ __forceinline__ float h2f(uint16_t bits) {
  return __half2float(__ushort_as_half(bits));
}
__device__ __forceinline__ uint16_t f2h(float x) {
  return __half_as_ushort(__float2half_rn(x));
}

}  // namespace kitty
