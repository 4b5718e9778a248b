// common.cuh — shared helpers of libdop: errors, element types, reductions.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

namespace dop {

// Every host-side failure is thrown as dop::Error and turned into a status
// code at the C ABI (dop_api.cu).
struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

#define DOP_CHECK_CUDA(expr)                                                         \
  do {                                                                               \
    cudaError_t _e = (expr);                                                         \
    if (_e != cudaSuccess)                                                           \
      throw ::dop::Error(-2, std::string(#expr) + ": " + cudaGetErrorString(_e) +   \
                                 " (" __FILE__ ":" + std::to_string(__LINE__) + ")"); \
  } while (0)

#define DOP_REQUIRE(cond, msg)                                              \
  do {                                                                      \
    if (!(cond)) throw ::dop::Error(-1, std::string("invalid argument: ") + (msg)); \
  } while (0)

// Launch-error check after every kernel launch; counts launches for the
// handle that issued them.
#define DOP_LAUNCHED(counter)                                               \
  do {                                                                      \
    DOP_CHECK_CUDA(cudaGetLastError());                                     \
    ++(counter);                                                            \
  } while (0)

typedef __nv_bfloat16 bf16;

// Load/store of the activation type (float or bf16) as float.
__device__ __forceinline__ float ld(const float* p) { return *p; }
__device__ __forceinline__ float ld(const bf16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ void st(float* p, float v) { *p = v; }
__device__ __forceinline__ void st(bf16* p, float v) { *p = __float2bfloat16_rn(v); }

// Four consecutive elements of the activation type as a float4: one 16-byte
// (fp32) or 8-byte (bf16) access.  p must be aligned to that size.
__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 ld4(const bf16* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void st4(bf16* p, float4 v) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<const uint32_t*>(&a);
  u.y = *reinterpret_cast<const uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}
// The router's E weights of model row i (wr is [D, E] row-major), E == 8.
__device__ __forceinline__ void ld_row8(const float* p, float* v) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void ld_row8(const bf16* p, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[q]));
    v[2 * q] = f.x;
    v[2 * q + 1] = f.y;
  }
}
// True when p is aligned for ld4/st4 of the element type T.
template <typename T>
inline bool aligned4(const T* p) {
  return ((uintptr_t)p % (4 * sizeof(T))) == 0;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int64_t round_up(int64_t a, int64_t b) { return ceil_div(a, b) * b; }

// Number of SMs of the current device (cached per process for device 0..15).
int sm_count();

}  // namespace dop
