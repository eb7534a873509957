// misc.cu -- small index kernels used by the C ABI's standalone gather path.
#include "common.cuh"
#include "kernels.h"

namespace astro {

// offsets[e] = first position p with ids[p] >= e, for ascending ids (the
// sorted_indices=true contract of gathered_projection.rs:24-38).  An id >= E
// or a descending pair records kDevBadExpertId.
__global__ void offsets_from_sorted_kernel(const uint32_t* __restrict__ ids, int64_t n, int E,
                                           uint32_t* __restrict__ offsets,
                                           uint32_t* __restrict__ status) {
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e <= E; e += gridDim.x * blockDim.x) {
    int64_t lo = 0, hi = n;
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if (ids[mid] < (uint32_t)e) lo = mid + 1; else hi = mid;
    }
    offsets[e] = (uint32_t)lo;
  }
  for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < n;
       p += (int64_t)gridDim.x * blockDim.x) {
    if (ids[p] >= (uint32_t)E || (p > 0 && ids[p - 1] > ids[p])) record_status(status, kDevBadExpertId);
  }
}

cudaError_t launch_offsets_from_sorted(const uint32_t* ids, int64_t n, int E, uint32_t* offsets,
                                       uint32_t* status, cudaStream_t st) {
  offsets_from_sorted_kernel<<<8, 256, 0, st>>>(ids, n, E, offsets, status);
  return cudaGetLastError();
}

// rows_out[p] = lhs ? lhs[order[p]] : order[p]
__global__ void compose_rows_kernel(const uint32_t* __restrict__ lhs,
                                    const uint32_t* __restrict__ order, int64_t n,
                                    uint32_t* __restrict__ rows_out) {
  for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < n;
       p += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t o = order[p];
    rows_out[p] = lhs ? lhs[o] : o;
  }
}

cudaError_t launch_compose_rows(const uint32_t* lhs, const uint32_t* order, int64_t n,
                                uint32_t* rows_out, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  int64_t b = (n + 255) / 256;
  if (b > 1024) b = 1024;
  compose_rows_kernel<<<(unsigned)b, 256, 0, st>>>(lhs, order, n, rows_out);
  return cudaGetLastError();
}

}  // namespace astro
