// Shared helpers for the Kitty B200 kernels: error reporting for the C ABI,
// fp16 bit helpers and the torch-compatible float32 clamps used by the
// quantisers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstring>
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

// 16-bit float type of a call (KITTY_DTYPE_F16 / KITTY_DTYPE_BF16): conversions of
// single values and packed pairs (low half first), NaN-propagating packed min / max,
// and the metadata store.  Widening to float32 is exact for both types.
template <bool kBf16>
struct Half16;

template <>
struct Half16<false> {
  static __device__ __forceinline__ float to_f(uint16_t x) { return __half2float(__ushort_as_half(x)); }
  static __device__ __forceinline__ float2 to_f2(uint32_t x) {
    __half2 h;
    memcpy(&h, &x, 4);
    return __half22float2(h);
  }
  // low / high 16-bit half of a word as float (one conversion each, no repacking)
  static __device__ __forceinline__ float lo_f(uint32_t x) { return __half2float(__ushort_as_half(uint16_t(x))); }
  static __device__ __forceinline__ float hi_f(uint32_t x) { return __half2float(__ushort_as_half(uint16_t(x >> 16))); }
  static __device__ __forceinline__ uint32_t min2(uint32_t a, uint32_t b) {
    __half2 x, y;
    memcpy(&x, &a, 4); memcpy(&y, &b, 4);
    const __half2 r = __hmin2_nan(x, y);
    uint32_t u; memcpy(&u, &r, 4); return u;
  }
  static __device__ __forceinline__ uint32_t max2(uint32_t a, uint32_t b) {
    __half2 x, y;
    memcpy(&x, &a, 4); memcpy(&y, &b, 4);
    const __half2 r = __hmax2_nan(x, y);
    uint32_t u; memcpy(&u, &r, 4); return u;
  }
  // scale / zero-point as stored by the reference: fp16 (RN)
  static __device__ __forceinline__ uint16_t meta(float x) { return __half_as_ushort(__float2half_rn(x)); }
  static __device__ __forceinline__ uint16_t from_f(float x) { return __half_as_ushort(__float2half_rn(x)); }
};

template <>
struct Half16<true> {
  static __device__ __forceinline__ float to_f(uint16_t x) { return __uint_as_float(uint32_t(x) << 16); }
  static __device__ __forceinline__ float2 to_f2(uint32_t x) {
    return make_float2(__uint_as_float(x << 16), __uint_as_float(x & 0xffff0000u));
  }
  static __device__ __forceinline__ float lo_f(uint32_t x) { return __uint_as_float(x << 16); }
  static __device__ __forceinline__ float hi_f(uint32_t x) { return __uint_as_float(x & 0xffff0000u); }
  static __device__ __forceinline__ uint32_t min2(uint32_t a, uint32_t b) {
    __nv_bfloat162 x, y;
    memcpy(&x, &a, 4); memcpy(&y, &b, 4);
    const __nv_bfloat162 r = __hmin2_nan(x, y);
    uint32_t u; memcpy(&u, &r, 4); return u;
  }
  static __device__ __forceinline__ uint32_t max2(uint32_t a, uint32_t b) {
    __nv_bfloat162 x, y;
    memcpy(&x, &a, 4); memcpy(&y, &b, 4);
    const __nv_bfloat162 r = __hmax2_nan(x, y);
    uint32_t u; memcpy(&u, &r, 4); return u;
  }
  // the reference returns fp16 scale / zero-point and copies them into the bf16
  // pool: fp16 (RN), then bf16 (RN)
  static __device__ __forceinline__ uint16_t meta(float x) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(__half2float(__float2half_rn(x))));
  }
  static __device__ __forceinline__ uint16_t from_f(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }
};

}  // namespace kitty
