// sort.cu -- stable counting sort of (token, slot) assignments by expert id.
//
// Replaces sort_expert_assignments (sparse_experts/assignment_sort.rs:36-97):
// sorted_order = stable argsort(flat ids), inverse_order = argsort(sorted_order),
// sorted token = sorted_order / K, sorted ids = ids[sorted_order].  The expert
// offsets that MLX derives inside gather_qmm are materialised as the exclusive
// scan of the histogram; the grouped GEMMs consume them directly.
//
// Two passes over tiles of 2048 assignments: per-tile histograms, then each
// tile computes its bases (global exclusive scan over experts, plus earlier
// tiles, plus earlier warps of the tile) and scatters its assignments in order;
// equal ids inside one 32-wide step get their rank from __match_any_sync.  Ids
// >= E set a status bit and are skipped, so no write leaves the output arrays.
// When all assignments fit one tile (decode batches, n <= 2048) the histogram
// pass is skipped: the single scatter block counts for itself.
//
// With shared_rows > 0 the shared expert is appended as segment E: rows
// [n, n + shared_rows) with token t and id E, offsets[E+1] = n + shared_rows.
#include "common.cuh"
#include "kernels.h"

namespace astro {

// Tiles of kSortTile assignments; inside a tile warp w owns a contiguous run of
// kSortTile / kSortWarps assignments, so stability needs only per-warp counts.
constexpr int kSortWarps = 16;
constexpr int kSortTile = 2048;
constexpr int kPerWarp = kSortTile / kSortWarps;  // 128

int64_t sort_tiles(int64_t n) { return (n + kSortTile - 1) / kSortTile; }

int sort_launch_count(int64_t n) { return sort_tiles(n) > 1 ? 2 : 1; }

size_t sort_scratch_bytes(int64_t n, int E) {
  return sizeof(int) * (size_t)(sort_tiles(n) > 0 ? sort_tiles(n) : 1) * (size_t)E;
}

// pass 1: histogram of each tile -> tile_hist[g][e]
__global__ void __launch_bounds__(kSortWarps * 32) sort_hist_kernel(
    const uint32_t* __restrict__ ids, int64_t n, int E, int* __restrict__ tile_hist,
    uint32_t* __restrict__ status) {
  extern __shared__ int hist[];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int64_t beg = (int64_t)blockIdx.x * kSortTile + (int64_t)w * kPerWarp;
  for (int it = 0; it < kPerWarp; it += 32) {
    const int64_t i = beg + it + lane;
    const bool act = i < n;
    const uint32_t id = act ? ids[i] : 0xffffffffu;
    const bool ok = act && id < (uint32_t)E;
    if (act && !ok) record_status(status, kDevBadExpertId);
    const uint32_t peers = __match_any_sync(0xffffffffu, ok ? id : 0xffffffffu);
    if (ok && (__ffs(peers) - 1) == lane) atomicAdd(&hist[id], __popc(peers));
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    tile_hist[(int64_t)blockIdx.x * E + e] = hist[e];
}

// pass 2: every tile derives its bases (global exclusive scan over experts of
// all tiles' counts + counts of earlier tiles + counts of earlier warps of the
// tile) and scatters its assignments in order.
__global__ void __launch_bounds__(kSortWarps * 32) sort_scatter_kernel(
    const uint32_t* __restrict__ ids, int64_t n, int K, int E, int tiles,
    const int* __restrict__ tile_hist, int64_t shared_rows, uint32_t* __restrict__ sorted_order,
    uint32_t* __restrict__ inverse_order, uint32_t* __restrict__ sorted_ids,
    uint32_t* __restrict__ sorted_tokens, uint32_t* __restrict__ offsets,
    uint32_t* __restrict__ status) {
  extern __shared__ int sm[];
  int* cnt = sm;                             // [kSortWarps][E]
  int* base = sm + kSortWarps * E;           // [E] counts of earlier tiles
  int* totals = sm + (kSortWarps + 1) * E;   // [E] counts of all tiles
  __shared__ int warp_sums[32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int g = blockIdx.x;
  for (int i = threadIdx.x; i < kSortWarps * E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  const int64_t beg = (int64_t)g * kSortTile + (int64_t)w * kPerWarp;
  for (int it = 0; it < kPerWarp; it += 32) {
    const int64_t i = beg + it + lane;
    const uint32_t id = (i < n) ? ids[i] : 0xffffffffu;
    const bool ok = id < (uint32_t)E;
    if (!tile_hist && i < n && !ok) record_status(status, kDevBadExpertId);
    const uint32_t peers = __match_any_sync(0xffffffffu, ok ? id : 0xffffffffu);
    if (ok && (__ffs(peers) - 1) == lane) cnt[w * E + id] += __popc(peers);
  }
  // totals over all tiles and the count of earlier tiles, per expert; a single
  // tile (tile_hist == nullptr) takes its totals from its own warp counts
  if (!tile_hist) __syncthreads();
  const int per = (E + blockDim.x - 1) / blockDim.x;
  const int e0 = threadIdx.x * per;
  int local = 0;
  for (int q = 0; q < per && e0 + q < E; ++q) {
    const int e = e0 + q;
    int total = 0, before = 0;
    if (tile_hist) {
      for (int t = 0; t < tiles; ++t) {
        const int c = tile_hist[(int64_t)t * E + e];
        total += c;
        if (t < g) before += c;
      }
    } else {
      for (int ww = 0; ww < kSortWarps; ++ww) total += cnt[ww * E + e];
    }
    base[e] = before;
    local += total;
    totals[e] = total;
  }
  __syncthreads();
  // block-wide exclusive scan of the totals
  int incl = local;
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, incl, m);
    if (lane >= m) incl += o;
  }
  if (lane == 31) warp_sums[w] = incl;
  __syncthreads();
  if (w == 0) {
    int s = lane < kSortWarps ? warp_sums[lane] : 0;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, s, m);
      if (lane >= m) s += o;
    }
    if (lane < kSortWarps) warp_sums[lane] = s;
  }
  __syncthreads();
  {
    int run = incl - local + (w > 0 ? warp_sums[w - 1] : 0);
    for (int q = 0; q < per && e0 + q < E; ++q) {
      const int e = e0 + q;
      const int total = totals[e];
      if (g == 0) offsets[e] = (uint32_t)run;
      int b = run + base[e];
      for (int ww = 0; ww < kSortWarps; ++ww) {
        const int c = cnt[ww * E + e];
        cnt[ww * E + e] = b;
        b += c;
      }
      run += total;
    }
  }
  if (g == 0 && threadIdx.x == blockDim.x - 1) {
    const int total = warp_sums[kSortWarps - 1];
    offsets[E] = (uint32_t)total;
    if (shared_rows > 0) offsets[E + 1] = (uint32_t)(total + shared_rows);
  }
  __syncthreads();
  for (int it = 0; it < kPerWarp; it += 32) {
    const int64_t i = beg + it + lane;
    const uint32_t id = (i < n) ? ids[i] : 0xffffffffu;
    const bool ok = id < (uint32_t)E;
    const uint32_t peers = __match_any_sync(0xffffffffu, ok ? id : 0xffffffffu);
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
  // shared-expert segment (token order), split over the tiles
  if (shared_rows > 0) {
    for (int64_t t = (int64_t)g * blockDim.x + threadIdx.x; t < shared_rows;
         t += (int64_t)tiles * blockDim.x) {
      if (sorted_tokens) sorted_tokens[n + t] = (uint32_t)t;
      if (sorted_ids) sorted_ids[n + t] = (uint32_t)E;
    }
  }
}

cudaError_t launch_sort_assignments(const uint32_t* ids, int64_t tokens, int K, int E,
                                    int64_t shared_rows, uint32_t* sorted_order,
                                    uint32_t* inverse_order, uint32_t* sorted_ids,
                                    uint32_t* sorted_tokens, uint32_t* offsets, uint32_t* status,
                                    void* scratch, cudaStream_t st) {
  const int64_t n = tokens * (int64_t)K;
  const int tiles = (int)(n > 0 ? sort_tiles(n) : 1);
  int* tile_hist = reinterpret_cast<int*>(scratch);
  const size_t smem1 = sizeof(int) * (size_t)E;
  const size_t smem2 = sizeof(int) * (size_t)(kSortWarps + 2) * E;
  if (smem2 > 48 * 1024)
    cudaFuncSetAttribute(sort_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem2);
  if (tiles > 1) {
    sort_hist_kernel<<<tiles, kSortWarps * 32, smem1, st>>>(ids, n, E, tile_hist, status);
  } else {
    tile_hist = nullptr;  // one tile: the scatter pass counts (and checks ids) itself
  }
  sort_scatter_kernel<<<tiles, kSortWarps * 32, smem2, st>>>(
      ids, n, K > 0 ? K : 1, E, tiles, tile_hist, shared_rows, sorted_order, inverse_order,
      sorted_ids, sorted_tokens, offsets, status);
  return cudaGetLastError();
}

// out[p, :] = src[rows[p], :] for bf16 rows of `hidden` elements (16-byte moves);
// rows == nullptr takes row p.  PERM8: each 8-element chunk in the grouped GEMMs'
// K order (perm8_bf16).  One warp per output row: the row index is read once and
// each lane keeps kTakeBatch loads in flight before it stores them.
constexpr int kTakeBatch = 8;
constexpr int kTakeWarps = 8;  // warps per block

template <bool PERM8>
__global__ void __launch_bounds__(kTakeWarps * 32) take_rows_kernel(
    const uint4* __restrict__ src, const uint32_t* __restrict__ rows, int64_t n,
    int chunks_per_row, int64_t src_rows, uint4* __restrict__ out, uint32_t* __restrict__ status) {
  const int lane = threadIdx.x & 31;
  const int64_t stride = (int64_t)gridDim.x * kTakeWarps;
  for (int64_t p = (int64_t)blockIdx.x * kTakeWarps + (threadIdx.x >> 5); p < n; p += stride) {
    const uint32_t r = rows ? __ldg(rows + p) : (uint32_t)p;
    if ((int64_t)r >= src_rows) {
      if (lane == 0) record_status(status, kDevBadShape);
      continue;
    }
    const uint4* s = src + (int64_t)r * chunks_per_row;
    uint4* o = out + p * chunks_per_row;
    for (int c0 = 0; c0 < chunks_per_row; c0 += 32 * kTakeBatch) {
      uint4 v[kTakeBatch];
#pragma unroll
      for (int j = 0; j < kTakeBatch; ++j) {
        const int c = c0 + j * 32 + lane;
        if (c < chunks_per_row) v[j] = s[c];
      }
#pragma unroll
      for (int j = 0; j < kTakeBatch; ++j) {
        const int c = c0 + j * 32 + lane;
        if (c < chunks_per_row) o[c] = PERM8 ? perm8_bf16(v[j]) : v[j];
      }
    }
  }
}

cudaError_t launch_take_rows(const void* src, int64_t src_rows, const uint32_t* rows, int64_t n,
                             int hidden, void* out, uint32_t* status, cudaStream_t st,
                             bool perm8) {
  if (n == 0) return cudaSuccess;
  const int chunks = hidden / 8;
  int64_t blocks = (n + kTakeWarps - 1) / kTakeWarps;
  if (blocks > 148 * 8) blocks = 148 * 8;  // one resident wave, rows strided over it
  if (perm8)
    take_rows_kernel<true><<<(unsigned)blocks, kTakeWarps * 32, 0, st>>>(
        (const uint4*)src, rows, n, chunks, src_rows, (uint4*)out, status);
  else
    take_rows_kernel<false><<<(unsigned)blocks, kTakeWarps * 32, 0, st>>>(
        (const uint4*)src, rows, n, chunks, src_rows, (uint4*)out, status);
  return cudaGetLastError();
}

}  // namespace astro
