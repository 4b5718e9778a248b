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
