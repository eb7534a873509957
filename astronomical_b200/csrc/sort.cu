// sort.cu -- stable counting sort of (token, slot) assignments by expert id.
//
// Replaces sort_expert_assignments (sparse_experts/assignment_sort.rs:36-97):
// sorted_order = stable argsort(flat ids), inverse_order = argsort(sorted_order),
// sorted token = sorted_order / K, sorted ids = ids[sorted_order].  The expert
// offsets that MLX derives inside gather_qmm are materialised as the exclusive
// scan of the histogram; the grouped GEMMs consume them directly.
//
// One CTA of 32 warps: warp w owns a contiguous slice of the assignments, so
// stability only needs per-warp histograms (phase 1), an (expert, warp) scan
// (phase 2) and an in-order scatter where equal ids inside one 32-wide step get
// their rank from __match_any_sync (phase 3).  Ids >= E set a status bit and
// are skipped, so no write ever leaves the output arrays.
//
// With shared_rows > 0 the shared expert is appended as segment E: rows
// [n, n + shared_rows) with token t and id E, offsets[E+1] = n + shared_rows.
#include "common.cuh"
#include "kernels.h"

namespace astro {

constexpr int kSortWarps = 32;

__global__ void __launch_bounds__(kSortWarps * 32, 1) sort_assignments_kernel(
    const uint32_t* __restrict__ ids, int64_t n, int K, int E, int64_t shared_rows,
    uint32_t* __restrict__ sorted_order, uint32_t* __restrict__ inverse_order,
    uint32_t* __restrict__ sorted_ids, uint32_t* __restrict__ sorted_tokens,
    uint32_t* __restrict__ offsets, uint32_t* __restrict__ status) {
  extern __shared__ int smem_i[];
  int* cnt = smem_i;                      // [kSortWarps][E]
  int* tot = smem_i + kSortWarps * E;     // [E]
  __shared__ int warp_sums[32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t chunk = (n + kSortWarps - 1) / kSortWarps;
  const int64_t beg = (int64_t)w * chunk;
  const int64_t end = (beg + chunk < n) ? beg + chunk : n;

  for (int i = threadIdx.x; i < kSortWarps * E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();

  // phase 1: per-warp histogram
  for (int64_t base = beg; base < end; base += 32) {
    const int64_t i = base + lane;
    const bool act = i < end;
    uint32_t id = act ? ids[i] : 0xffffffffu;
    const bool ok = act && id < (uint32_t)E;
    if (act && !ok) record_status(status, kDevBadExpertId);
    const uint32_t key = ok ? id : 0xffffffffu;
    const uint32_t peers = __match_any_sync(0xffffffffu, key);
    if (ok && (__ffs(peers) - 1) == lane) cnt[w * E + id] += __popc(peers);
  }
  __syncthreads();

  // phase 2: per expert, exclusive scan over warps; then scan of totals over experts
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int ww = 0; ww < kSortWarps; ++ww) {
      const int c = cnt[ww * E + e];
      cnt[ww * E + e] = run;
      run += c;
    }
    tot[e] = run;
  }
  __syncthreads();
  // block-wide exclusive scan of tot[0..E), E <= 32 * blockDim.x
  {
    const int per = (E + blockDim.x - 1) / blockDim.x;
    const int e0 = threadIdx.x * per;
    int local = 0;
    for (int j = 0; j < per && e0 + j < E; ++j) local += tot[e0 + j];
    int incl = local;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, m);
      if (lane >= m) incl += o;
    }
    if (lane == 31) warp_sums[w] = incl;
    __syncthreads();
    if (w == 0) {
      int s = warp_sums[lane];
#pragma unroll
      for (int m = 1; m < 32; m <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, s, m);
        if (lane >= m) s += o;
      }
      warp_sums[lane] = s;  // inclusive
    }
    __syncthreads();
    int run = incl - local + (w > 0 ? warp_sums[w - 1] : 0);
    for (int j = 0; j < per && e0 + j < E; ++j) {
      const int c = tot[e0 + j];
      tot[e0 + j] = run;  // now the exclusive offset
      run += c;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    offsets[e] = (uint32_t)tot[e];
    for (int ww = 0; ww < kSortWarps; ++ww) cnt[ww * E + e] += tot[e];
  }
  if (threadIdx.x == 0) {
    const int total = warp_sums[31];
    offsets[E] = (uint32_t)total;
    if (shared_rows > 0) offsets[E + 1] = (uint32_t)(total + shared_rows);
  }
  __syncthreads();

  // phase 3: stable scatter in original order
  for (int64_t base = beg; base < end; base += 32) {
    const int64_t i = base + lane;
    const bool act = i < end;
    const uint32_t id = act ? ids[i] : 0xffffffffu;
    const bool ok = act && id < (uint32_t)E;
    const uint32_t key = ok ? id : 0xffffffffu;
    const uint32_t peers = __match_any_sync(0xffffffffu, key);
    int pos = 0;
    if (ok) pos = cnt[w * E + id] + __popc(peers & lanemask_lt());
    __syncwarp();
    if (ok && (__ffs(peers) - 1) == lane) cnt[w * E + id] += __popc(peers);
    __syncwarp();
    if (ok) {
      if (sorted_order) sorted_order[pos] = (uint32_t)i;
      if (inverse_order) inverse_order[i] = (uint32_t)pos;
      if (sorted_ids) sorted_ids[pos] = id;
      if (sorted_tokens) sorted_tokens[pos] = (uint32_t)(i / K);
    }
  }
  // shared-expert segment (token order)
  if (shared_rows > 0) {
    for (int64_t t = threadIdx.x; t < shared_rows; t += blockDim.x) {
      if (sorted_tokens) sorted_tokens[n + t] = (uint32_t)t;
      if (sorted_ids) sorted_ids[n + t] = (uint32_t)E;
    }
  }
}

cudaError_t launch_sort_assignments(const uint32_t* ids, int64_t tokens, int K, int E,
                                    int64_t shared_rows, uint32_t* sorted_order,
                                    uint32_t* inverse_order, uint32_t* sorted_ids,
                                    uint32_t* sorted_tokens, uint32_t* offsets, uint32_t* status,
                                    cudaStream_t st) {
  const int64_t n = tokens * (int64_t)K;
  const size_t smem = sizeof(int) * (size_t)(kSortWarps + 1) * E;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(sort_assignments_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
  sort_assignments_kernel<<<1, kSortWarps * 32, smem, st>>>(
      ids, n, K > 0 ? K : 1, E, shared_rows, sorted_order, inverse_order, sorted_ids,
      sorted_tokens, offsets, status);
  return cudaGetLastError();
}

// out[p, :] = src[rows[p], :] for bf16 rows of `hidden` elements (16-byte moves).
__global__ void take_rows_kernel(const uint4* __restrict__ src, const uint32_t* __restrict__ rows,
                                 int64_t n, int chunks_per_row, int64_t src_rows,
                                 uint4* __restrict__ out, uint32_t* __restrict__ status) {
  const int64_t total = n * chunks_per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = i / chunks_per_row;
    const int c = (int)(i - p * chunks_per_row);
    const uint32_t r = rows[p];
    if ((int64_t)r >= src_rows) {
      record_status(status, kDevBadShape);
      continue;
    }
    out[i] = src[(int64_t)r * chunks_per_row + c];
  }
}

cudaError_t launch_take_rows(const void* src, int64_t src_rows, const uint32_t* rows, int64_t n,
                             int hidden, void* out, uint32_t* status, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  const int chunks = hidden / 8;
  const int64_t total = n * chunks;
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 16) blocks = 148 * 16;
  take_rows_kernel<<<(unsigned)blocks, threads, 0, st>>>((const uint4*)src, rows, n, chunks,
                                                         src_rows, (uint4*)out, status);
  return cudaGetLastError();
}

}  // namespace astro
