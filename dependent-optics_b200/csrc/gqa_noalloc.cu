// gqa_noalloc.cu — fp32 attention backward that allocates no device memory.
//
// dop_gqa_backward() needs a caller-provided scratch buffer (delta, one float
// per batch x head x query).  Some callers cannot provide one: their device
// memory is owned by another allocator (a framework's caching pool, a fixed
// arena handed out by the host application) and they may not call cudaMalloc
// themselves.  dop_gqa_backward_f32_noalloc() computes exactly what
// dop_gqa_backward(..., DOP_F32, ...) computes, with the same CUDA-core
// kernels, but takes delta from a fixed-size array in this library's own
// device memory.
//
// The array is a file-scope __device__ object, so every GPU that loads the
// library holds it (4 MiB) until the process exits.  Host code cannot use its
// name as a device address: every call made while its stream is not being
// captured asks the runtime for the address with cudaGetSymbolAddress (with
// the call's device current) and keeps it per device; a call made during a
// stream capture uses the kept address.  So the first call on a device
// should come before any capture, and after a cudaDeviceReset the first call
// should again be made outside a capture.  The array is shared by every
// call: each call overwrites all the delta entries it reads before reading
// them (nothing needs clearing), and calls that overlap on the GPU race on
// it.
#include <mutex>
#include <string>

#include "../../include/dop.h"
#include "kernels.cuh"

namespace dop {
int set_last_error(int code, const char* msg);
}

namespace {

constexpr int64_t kMaxDelta = int64_t(1) << 20;  // floats: batch * heads * seq <= 1,048,576

__device__ __align__(256) float g_delta_scratch[kMaxDelta];

// Device address of g_delta_scratch on the current device: looked up
// whenever `stream` is not capturing (so a context re-created after a
// cudaDeviceReset is seen), the last lookup reused during a capture.
float* delta_scratch(cudaStream_t stream) {
  static float* addr[16] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  DOP_CHECK_CUDA(cudaGetDevice(&dev));
  DOP_REQUIRE(dev >= 0 && dev < 16, "device index out of range");
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  DOP_CHECK_CUDA(cudaStreamIsCapturing(stream, &cap));
  std::lock_guard<std::mutex> lock(mu);
  if (cap == cudaStreamCaptureStatusNone) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_delta_scratch);
    if (e != cudaSuccess)
      throw dop::Error(DOP_E_CUDA, std::string("cudaGetSymbolAddress(delta scratch): ") +
                                       cudaGetErrorString(e));
    addr[dev] = static_cast<float*>(p);
  } else if (!addr[dev]) {
    throw dop::Error(DOP_E_STATE,
                     "the first dop_gqa_backward_f32_noalloc call on a device must come "
                     "before any stream capture");
  }
  return addr[dev];
}

}  // namespace

extern "C" int dop_gqa_backward_f32_noalloc(int64_t batch, int64_t seq, int64_t heads,
                                            int64_t kv_heads, int64_t head_dim, int64_t window,
                                            const float* q, const float* k, const float* v,
                                            const float* o, const float* dout, const float* lse,
                                            float* dq, float* dk, float* dv, void* stream) {
  try {
    DOP_REQUIRE(q && k && v && o && dout && lse && dq && dk && dv, "null pointer");
    DOP_REQUIRE(batch >= 1 && seq >= 1 && heads >= 1 && kv_heads >= 1 && heads % kv_heads == 0,
                "bad attention shape");
    DOP_REQUIRE(head_dim >= 2 && head_dim % 2 == 0 && window >= 1, "bad head_dim or window");
    DOP_REQUIRE(heads <= INT32_MAX && head_dim <= INT32_MAX, "heads or head_dim out of range");
    // each factor is checked first, so the product below cannot overflow
    if (batch > kMaxDelta || heads > kMaxDelta || seq > kMaxDelta ||
        batch * heads * seq > kMaxDelta)
      throw dop::Error(DOP_E_INVALID,
                       "invalid argument: batch * heads * seq (" + std::to_string(batch) +
                           " x " + std::to_string(heads) + " x " + std::to_string(seq) +
                           ") exceeds the built-in scratch of " + std::to_string(kMaxDelta) +
                           " floats; use dop_gqa_backward with a caller-provided delta_ws");
    dop::Attn a;
    a.B = batch; a.S = seq; a.H = (int)heads; a.KV = (int)kv_heads; a.hd = (int)head_dim;
    a.window = window; a.causal = true; a.scale = 1.0f / sqrtf((float)head_dim);
    int64_t launches = 0;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    dop::attn_bwd_simt<float>(a, q, k, v, o, dout, lse, delta_scratch(st), dq, dk, dv, st,
                              launches);
    return DOP_OK;
  } catch (const dop::Error& e) {
    return dop::set_last_error(e.code, e.what());
  } catch (const std::exception& e) {
    return dop::set_last_error(DOP_E_INVALID, e.what());
  }
}
