// ep.cu -- row bookkeeping of the expert-parallel block (config 3).
//
// Expert parallelism has no counterpart in the reference (MLX runs one device);
// it partitions experts in blocks over the ranks of one node: rank r owns experts
// [r*El, (r+1)*El).  After the all-to-all dispatch a rank holds, from every
// source s, the rows that s sorted for its experts: source-major, and within a
// source ordered by expert.  The grouped GEMMs want expert-major rows, so:
//   ep_segments_kernel: from the received counts C[s][e] (world x El) it derives
//     the start of every (s, e) run in the received order (source-major scan) and
//     in expert-major order (expert-major scan), and the expert offsets
//     [El + 2] of the expert-major rows (segment El = this rank's shared-expert
//     rows appended after the routed ones);
//   ep_perm_kernel: one block per (s, e) run writes dest[q] (expert-major
//     position of received row q) and src_of[dest[q]] = q.
// The caller gathers rows with take_rows: states = recv[src_of], and after the
// GEMMs out = yrows[dest], which restores the received order for the return
// all-to-all.  Sizes: world <= 8, El * world <= 2048.
#include "common.cuh"
#include "kernels.h"

namespace astro {
namespace {

constexpr int kSegThreads = 1024;
constexpr int kMaxRuns = 2048;  // world * experts-per-rank

// exclusive block scan of v over all threads (kSegThreads), returns the total
ASTRO_DEVINL uint32_t block_exclusive_scan(uint32_t& v, uint32_t* warp_tot) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  uint32_t incl = v;
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    const uint32_t o = __shfl_up_sync(0xffffffffu, incl, m);
    if (lane >= m) incl += o;
  }
  if (lane == 31) warp_tot[w] = incl;
  __syncthreads();
  if (w == 0) {
    uint32_t t = warp_tot[lane];
    uint32_t ti = t;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
      const uint32_t o = __shfl_up_sync(0xffffffffu, ti, m);
      if (lane >= m) ti += o;
    }
    warp_tot[lane] = ti - t;  // exclusive warp bases
    if (lane == 31) warp_tot[32] = ti;
  }
  __syncthreads();
  const uint32_t total = warp_tot[32];
  v = incl - v + warp_tot[w];
  __syncthreads();
  return total;
}

__global__ void __launch_bounds__(kSegThreads) ep_segments_kernel(
    const uint32_t* __restrict__ counts, int world, int El, int shared_rows,
    uint32_t* __restrict__ src_start, uint32_t* __restrict__ exp_start,
    uint32_t* __restrict__ offsets) {
  __shared__ uint32_t warp_tot[33];
  __shared__ uint32_t s_exp[kMaxRuns];
  const int runs = world * El;
  // two runs per thread (runs <= 2048): i = 2t, 2t + 1
  // source-major order: run index i = s * El + e
  {
    const int i0 = 2 * threadIdx.x, i1 = i0 + 1;
    const uint32_t c0 = i0 < runs ? counts[i0] : 0u, c1 = i1 < runs ? counts[i1] : 0u;
    uint32_t v = c0 + c1;
    block_exclusive_scan(v, warp_tot);
    if (i0 < runs) src_start[i0] = v;
    if (i1 < runs) src_start[i1] = v + c0;
  }
  // expert-major order: position j = e * world + s holds run (s, e)
  {
    const int j0 = 2 * threadIdx.x, j1 = j0 + 1;
    auto run_of = [&](int j) { return (j % world) * El + j / world; };
    const uint32_t c0 = j0 < runs ? counts[run_of(j0)] : 0u;
    const uint32_t c1 = j1 < runs ? counts[run_of(j1)] : 0u;
    uint32_t v = c0 + c1;
    const uint32_t total = block_exclusive_scan(v, warp_tot);
    if (j0 < runs) {
      exp_start[run_of(j0)] = v;
      s_exp[j0] = v;
    }
    if (j1 < runs) {
      exp_start[run_of(j1)] = v + c0;
      s_exp[j1] = v + c0;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < El; e += kSegThreads) offsets[e] = s_exp[e * world];
    if (threadIdx.x == 0) {
      offsets[El] = total;
      offsets[El + 1] = total + (uint32_t)shared_rows;
    }
  }
}

__global__ void ep_perm_kernel(const uint32_t* __restrict__ counts,
                               const uint32_t* __restrict__ src_start,
                               const uint32_t* __restrict__ exp_start, uint32_t* __restrict__ dest,
                               uint32_t* __restrict__ src_of) {
  const int run = blockIdx.x;
  const uint32_t n = counts[run], q0 = src_start[run], d0 = exp_start[run];
  for (uint32_t r = threadIdx.x; r < n; r += blockDim.x) {
    dest[q0 + r] = d0 + r;
    src_of[d0 + r] = q0 + r;
  }
}

}  // namespace

cudaError_t launch_ep_permutation(const uint32_t* counts, int world, int El, int shared_rows,
                                  uint32_t* src_start, uint32_t* exp_start, uint32_t* offsets,
                                  uint32_t* dest, uint32_t* src_of, cudaStream_t st) {
  if (world < 1 || El < 1 || world * El > kMaxRuns) return cudaErrorInvalidValue;
  ep_segments_kernel<<<1, kSegThreads, 0, st>>>(counts, world, El, shared_rows, src_start,
                                                exp_start, offsets);
  ep_perm_kernel<<<world * El, 128, 0, st>>>(counts, src_start, exp_start, dest, src_of);
  return cudaGetLastError();
}

}  // namespace astro

// ===========================================================================
// Peer-memory exchange.  Each rank's receive and return buffers are mapped into
// every peer (CUDA IPC), so the dispatch gather stores a token row straight into
// the destination rank's receive buffer over NVLink, and the expert side stores
// each output row straight into its source rank's return buffer: the all-to-all
// is fused into the kernels that produce the rows.  No kernel waits on another
// GPU; the host orders the phases with stream-ordered collectives.  Every remote
// store is checked against the destination buffer's capacity (a bad row is
// recorded in the status word and skipped).
namespace astro {
namespace {

struct PeerTable {
  uint4* base[kMaxPeers];
  int64_t cap_rows[kMaxPeers];
  int64_t off[kMaxPeers];    // first row written in that peer's buffer
  int64_t start[kMaxPeers];  // first local row (sorted position or received row) for that peer
};

// row p (sorted position) of this rank's assignments: destination rank d =
// sorted_ids[p] / El, copied from x[sorted_tokens[p]] to peer d's receive row
// off[d] + p - start[d]
__global__ void ep_push_rows_kernel(const uint4* __restrict__ x, const uint32_t* __restrict__ stok,
                                   const uint32_t* __restrict__ sids, int64_t n, int El, int world,
                                   int chunks, int64_t x_rows, const __grid_constant__ PeerTable t,
                                   uint32_t* __restrict__ status) {
  const int64_t total = n * chunks;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = i / chunks;
    const int c = (int)(i - p * chunks);
    const uint32_t d = sids[p] / (uint32_t)El;
    const uint32_t tok = stok[p];
    if (d >= (uint32_t)world || tok >= (uint64_t)x_rows) {
      record_status(status, kDevBadShape);
      continue;
    }
    const int64_t row = t.off[d] + (p - t.start[d]);
    if (row < 0 || row >= t.cap_rows[d]) {
      record_status(status, kDevBadShape);
      continue;
    }
    t.base[d][row * chunks + c] = x[(int64_t)tok * chunks + c];
  }
}

// received row q (source-major) of source s (start[s] <= q < start[s+1]) holds
// expert-major row dest[q] of yrows; stored to source s's return row
// off[s] + q - start[s]
__global__ void ep_return_rows_kernel(const uint4* __restrict__ yrows,
                                     const uint32_t* __restrict__ dest, int64_t n, int world,
                                     int chunks, int64_t y_rows,
                                     const __grid_constant__ PeerTable t,
                                     uint32_t* __restrict__ status) {
  const int64_t total = n * chunks;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t q = i / chunks;
    const int c = (int)(i - q * chunks);
    int s = 0;
    while (s + 1 < world && q >= t.start[s + 1]) ++s;
    const uint32_t src = dest[q];
    const int64_t row = t.off[s] + (q - t.start[s]);
    if (src >= (uint64_t)y_rows || row < 0 || row >= t.cap_rows[s]) {
      record_status(status, kDevBadShape);
      continue;
    }
    t.base[s][row * chunks + c] = yrows[(int64_t)src * chunks + c];
  }
}

PeerTable make_table(void* const* bases, const int64_t* caps, const int64_t* offs,
                     const int64_t* starts, int world) {
  PeerTable t{};
  for (int i = 0; i < world && i < kMaxPeers; ++i) {
    t.base[i] = reinterpret_cast<uint4*>(bases[i]);
    t.cap_rows[i] = caps[i];
    t.off[i] = offs[i];
    t.start[i] = starts[i];
  }
  return t;
}

int grid_rows(int64_t n, int chunks) {
  const int64_t threads = 256, total = n * chunks;
  int64_t b = (total + threads - 1) / threads;
  return (int)(b < 1 ? 1 : (b > 148 * 16 ? 148 * 16 : b));
}

}  // namespace

cudaError_t launch_ep_push_rows(const void* x, int64_t x_rows, const uint32_t* stok,
                                const uint32_t* sids, int64_t n, int El, int world, int H,
                                void* const* peer_bases, const int64_t* peer_cap_rows,
                                const int64_t* peer_offs, const int64_t* starts, uint32_t* status,
                                cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  if (world < 1 || world > kMaxPeers || H % 8) return cudaErrorInvalidValue;
  const PeerTable t = make_table(peer_bases, peer_cap_rows, peer_offs, starts, world);
  ep_push_rows_kernel<<<grid_rows(n, H / 8), 256, 0, st>>>(
      reinterpret_cast<const uint4*>(x), stok, sids, n, El, world, H / 8, x_rows, t, status);
  return cudaGetLastError();
}

cudaError_t launch_ep_return_rows(const void* yrows, int64_t y_rows, const uint32_t* dest,
                                  int64_t n, int world, int H, void* const* peer_bases,
                                  const int64_t* peer_cap_rows, const int64_t* peer_offs,
                                  const int64_t* starts, uint32_t* status, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  if (world < 1 || world > kMaxPeers || H % 8) return cudaErrorInvalidValue;
  const PeerTable t = make_table(peer_bases, peer_cap_rows, peer_offs, starts, world);
  ep_return_rows_kernel<<<grid_rows(n, H / 8), 256, 0, st>>>(
      reinterpret_cast<const uint4*>(yrows), dest, n, world, H / 8, y_rows, t, status);
  return cudaGetLastError();
}

}  // namespace astro
