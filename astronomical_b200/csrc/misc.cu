// misc.cu -- small index kernels used by the C ABI's standalone gather path, and
// the affine dequantisation of a whole tensor (MLX dequantize).
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

// out[r, j] = bf16(fma(scale, q, bias)) of MLX's affine layout: element j of a
// row sits at bit j*bits of the row's little-endian bit stream (bits in
// {2,3,4,5,6,8}), scale and bias per `group` elements.  One thread per output
// element (a once-per-registration conversion, not a hot path).
__global__ void dequantize_affine_kernel(const uint32_t* __restrict__ packed,
                                         const uint16_t* __restrict__ scales,
                                         const uint16_t* __restrict__ biases, int64_t rows,
                                         int in_features, int group, int bits,
                                         __nv_bfloat16* __restrict__ out) {
  const int64_t words = (int64_t)in_features * bits / 32;
  const int groups = in_features / group;
  const int64_t total = rows * in_features;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / in_features;
    const int j = (int)(i - r * in_features);
    const uint32_t* row = packed + r * words;
    const int64_t bit = (int64_t)j * bits;
    const int64_t w = bit >> 5;
    const int b = (int)(bit & 31);
    uint64_t v = row[w];
    if (b + bits > 32) v |= (uint64_t)row[w + 1] << 32;
    const uint32_t q = (uint32_t)(v >> b) & ((1u << bits) - 1u);
    const float sc = bf16_to_f32(scales[r * groups + j / group]);
    const float bi = bf16_to_f32(biases[r * groups + j / group]);
    out[i] = __float2bfloat16_rn(__fmaf_rn(sc, (float)q, bi));
  }
}

cudaError_t launch_dequantize_affine(const uint32_t* packed, const void* scales,
                                     const void* biases, int64_t rows, int in_features, int group,
                                     int bits, void* out, cudaStream_t st) {
  const int64_t total = rows * in_features;
  if (total == 0) return cudaSuccess;
  int64_t b = (total + 255) / 256;
  if (b > 4096) b = 4096;
  dequantize_affine_kernel<<<(unsigned)b, 256, 0, st>>>(
      packed, (const uint16_t*)scales, (const uint16_t*)biases, rows, in_features, group, bits,
      (__nv_bfloat16*)out);
  return cudaGetLastError();
}

}  // namespace astro
