// failure.cu — the device side of failure detection: wait limits, the
// sticky error word, and self-tests that make a bounded wait run out.
//
// Every wait a libdop kernel makes on another agent (an mbarrier that a TMA
// copy or an MMA completes, a flag another rank writes) is bounded.  A wait
// that runs out records a code in the device's error word (dop_device_status),
// raises its CTA's abort flag, drains what it has in flight with bounded
// waits, frees its TMEM and returns; every later libdop kernel on that device
// sees the word set and skips its work, so the host finds the failure at its
// next status check with the context still usable.  The crate's counterpart
// is the control plane's timeout (DistError, src/dist.rs:36-56), which belongs
// to its TCP runtime.
//
// The self-tests below make a wait run out without breaking any real kernel:
// an mbarrier that nothing arrives at (the same bounded-wait routine the
// tensor-core kernels use, with TMEM held across it) and the expert
// exchange's flag barrier with a peer slot that nothing writes.
#include "../../include/dop.h"
#include "ep.cuh"
#include "tc_ptx.cuh"

namespace dop {
int set_last_error(int code, const char* msg);

namespace {

using namespace tc;

// One CTA of 64 threads: warp 1 allocates 32 TMEM columns, thread 0 waits
// on an mbarrier that nothing arrives at (bounded by the tensor-core wait
// limit; records `code`), then warp 1 frees the columns.
__global__ void k_selftest_mbarrier_expiry(int code) {
  if (tc_failed()) return;
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(smem_u32(&tmem_slot), 32);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0) mbar_wait(smem_u32(&bar), 0, &abort_flag, code);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_slot, 32);
}

}  // namespace
}  // namespace dop

namespace {
template <class F>
int guarded_call(F&& f) {
  try {
    f();
    return DOP_OK;
  } catch (const dop::Error& e) {
    return dop::set_last_error(e.code, e.what());
  } catch (const std::exception& e) {
    return dop::set_last_error(DOP_E_INVALID, e.what());
  }
}
}  // namespace

extern "C" int dop_set_wait_limits(int64_t tensor_core_ns, int64_t exchange_ns) {
  return guarded_call([&] {
    DOP_REQUIRE(tensor_core_ns >= 0 && exchange_ns >= 0, "negative wait limit");
    const uint64_t v[2] = {(uint64_t)tensor_core_ns, (uint64_t)exchange_ns};
    int* w = dop::tc_error_word();
    DOP_CHECK_CUDA(cudaMemcpy(w + 2, &v[0], 8, cudaMemcpyHostToDevice));
    DOP_CHECK_CUDA(cudaMemcpy(w + 4, &v[1], 8, cudaMemcpyHostToDevice));
  });
}

extern "C" int dop_clear_device_status(void) {
  return guarded_call([&] {
    int* w = dop::tc_error_word();
    DOP_CHECK_CUDA(cudaDeviceSynchronize());
    DOP_CHECK_CUDA(cudaMemset(w, 0, sizeof(int)));
  });
}

extern "C" int dop_selftest_wait_expiry(int which, void* stream) {
  return guarded_call([&] {
    DOP_REQUIRE(which == 0 || which == 1, "which is 0 (mbarrier) or 1 (exchange barrier)");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int64_t launches = 0;
    if (which == 0) {
      dop::tc::bind_error_word();
      dop::k_selftest_mbarrier_expiry<<<1, 64, 0, s>>>(DOP_SELFTEST_MBARRIER_CODE);
      DOP_LAUNCHED(launches);
      return;
    }
    // A two-rank view whose both "ranks" are this device's own buffer: the
    // barrier's thread for rank 1 waits on flags[k][1], which nothing writes.
    const int k = 0;
    const size_t flag_bytes = sizeof(unsigned) * dop::kEpBarriers * dop::kEpMaxWorld;
    char* buf = nullptr;
    DOP_CHECK_CUDA(cudaMalloc(&buf, flag_bytes + 2 * sizeof(char*)));
    DOP_CHECK_CUDA(cudaMemsetAsync(buf, 0, flag_bytes, s));
    char* peers_host[2] = {buf, buf};
    char** peers_dev = reinterpret_cast<char**>(buf + flag_bytes);
    DOP_CHECK_CUDA(cudaMemcpyAsync(peers_dev, peers_host, sizeof(peers_host),
                                   cudaMemcpyHostToDevice, s));
    dop::EpView v;
    v.rank = 0;
    v.world = 2;
    v.peers = peers_dev;
    v.flags = reinterpret_cast<unsigned*>(buf);
    cudaError_t e = cudaSuccess;
    try {
      dop::ep_barrier(v, k, 1u, s, launches);
    } catch (...) {
      e = cudaStreamSynchronize(s);
      cudaFree(buf);
      throw;
    }
    e = cudaStreamSynchronize(s);
    cudaFree(buf);
    DOP_CHECK_CUDA(e);
  });
}
