// wait_probe.cu -- runs the library's bounded device waits on their own, so a
// failure test can make one run out without faulting or hanging the GPU.
//
// Every wait in the kernels (mbarrier waits of the tcgen05 GEMMs, the fused
// decode kernel's grid barrier and per-segment completion counters) gives up
// after a wall-clock limit, records ASTRO_MOE_DEVICE_WAIT_TIMEOUT in a status
// word and returns; these kernels wait on a condition the test controls (a word
// it sets or not, an mbarrier that never completes its phase) with a short limit.
#include <cstdio>

#include "astro_moe.h"
#include "common.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace astro {
namespace {

// kind 0: the completion-counter wait (wait_count_geq) on *flag >= target
__global__ void wait_counter_probe_kernel(const uint32_t* flag, uint32_t target,
                                          uint64_t limit_ns, uint32_t* status, uint32_t* result) {
  if (threadIdx.x != 0) return;
  result[0] = (uint32_t)wait_count_geq(flag, target, status, limit_ns);
}

// kind 1: an mbarrier wait (tc::mbar_wait) on a barrier expecting two arrivals
// that gets `target` of them (target >= 2 completes the phase)
__global__ void wait_mbarrier_probe_kernel(uint32_t target, uint64_t limit_ns, uint32_t* status,
                                           uint32_t* result) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 2);
    abort_flag = 0;
    tc::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < target && i < 2; ++i) tc::mbar_arrive(&bar);
    result[0] = tc::mbar_wait(&bar, 0, (volatile int*)&abort_flag, status, limit_ns) ? 1u : 0u;
  }
}

}  // namespace
}  // namespace astro

using namespace astro;

extern "C" int astro_moe_wait_probe(int32_t kind, const uint32_t* flag, uint32_t target,
                                    int64_t limit_ns, uint32_t* device_status, uint32_t* result,
                                    void* stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (!device_status || !result || limit_ns <= 0 || limit_ns > 2000000000LL)
    return set_last_error(ASTRO_MOE_ERR_INVALID_ARGUMENT,
                          "wait probe: a status word, a result word and 0 < limit <= 2 s are required");
  if (kind == 0) {
    if (!flag) return set_last_error(ASTRO_MOE_ERR_INVALID_ARGUMENT, "wait probe: null flag");
    wait_counter_probe_kernel<<<1, 32, 0, st>>>(flag, target, (uint64_t)limit_ns, device_status,
                                                 result);
  } else if (kind == 1) {
    wait_mbarrier_probe_kernel<<<1, 32, 0, st>>>(target, (uint64_t)limit_ns, device_status, result);
  } else {
    return set_last_error(ASTRO_MOE_ERR_INVALID_ARGUMENT, "wait probe: unknown kind");
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    char buf[256];
    snprintf(buf, sizeof(buf), "wait probe: %s", cudaGetErrorString(e));
    return set_last_error(ASTRO_MOE_ERR_CUDA, buf);
  }
  return ASTRO_MOE_OK;
}
