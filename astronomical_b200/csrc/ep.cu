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
    const uint32_t* __restrict__ counts, int cstride, int world, int El, int shared_rows,
    uint32_t* __restrict__ src_start, uint32_t* __restrict__ exp_start,
    uint32_t* __restrict__ offsets) {
  __shared__ uint32_t warp_tot[33];
  __shared__ uint32_t s_exp[kMaxRuns];
  const int runs = world * El;
  // two runs per thread (runs <= 2048): i = 2t, 2t + 1
  // source-major order: run index i = s * El + e
  {
    const int i0 = 2 * threadIdx.x, i1 = i0 + 1;
    auto cnt = [&](int i) { return counts[(i / El) * cstride + i % El]; };  // run i = s*El + e
    const uint32_t c0 = i0 < runs ? cnt(i0) : 0u, c1 = i1 < runs ? cnt(i1) : 0u;
    uint32_t v = c0 + c1;
    block_exclusive_scan(v, warp_tot);
    if (i0 < runs) src_start[i0] = v;
    if (i1 < runs) src_start[i1] = v + c0;
  }
  // expert-major order: position j = e * world + s holds run (s, e)
  {
    const int j0 = 2 * threadIdx.x, j1 = j0 + 1;
    auto run_of = [&](int j) { return (j % world) * El + j / world; };
    auto cnt = [&](int i) { return counts[(i / El) * cstride + i % El]; };
    const uint32_t c0 = j0 < runs ? cnt(run_of(j0)) : 0u;
    const uint32_t c1 = j1 < runs ? cnt(run_of(j1)) : 0u;
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

__global__ void ep_perm_kernel(const uint32_t* __restrict__ counts, int cstride, int El,
                               const uint32_t* __restrict__ src_start,
                               const uint32_t* __restrict__ exp_start, int64_t cap,
                               uint32_t* __restrict__ dest, uint32_t* __restrict__ src_of) {
  const int run = blockIdx.x;
  const uint32_t n = counts[(run / El) * cstride + run % El], q0 = src_start[run],
                 d0 = exp_start[run];
  if ((int64_t)q0 + n > cap || (int64_t)d0 + n > cap) return;  // inconsistent counts
  for (uint32_t r = threadIdx.x; r < n; r += blockDim.x) {
    dest[q0 + r] = d0 + r;
    src_of[d0 + r] = q0 + r;
  }
}

}  // namespace

cudaError_t launch_ep_permutation_strided(const uint32_t* counts, int cstride, int world, int El,
                                          int shared_rows, int64_t cap, uint32_t* src_start,
                                          uint32_t* exp_start, uint32_t* offsets, uint32_t* dest,
                                          uint32_t* src_of, cudaStream_t st) {
  if (world < 1 || El < 1 || world * El > kMaxRuns || cstride < El) return cudaErrorInvalidValue;
  ep_segments_kernel<<<1, kSegThreads, 0, st>>>(counts, cstride, world, El, shared_rows, src_start,
                                                exp_start, offsets);
  ep_perm_kernel<<<world * El, 128, 0, st>>>(counts, cstride, El, src_start, exp_start, cap, dest,
                                             src_of);
  return cudaGetLastError();
}

cudaError_t launch_ep_permutation(const uint32_t* counts, int world, int El, int shared_rows,
                                  uint32_t* src_start, uint32_t* exp_start, uint32_t* offsets,
                                  uint32_t* dest, uint32_t* src_of, cudaStream_t st) {
  // counts from this process's own all-to-all: the receive buffers were sized from them
  return launch_ep_permutation_strided(counts, El, world, El, shared_rows, INT64_MAX, src_start,
                                       exp_start, offsets, dest, src_of, st);
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

// ===========================================================================
// Device-planned peer exchange: counts travel through per-rank mailboxes
// (uint32 [world][El] per-expert counts received, then [world][world] rows each
// rank sends each rank), so every placement below is computed on the device and
// a layer needs no host synchronisation.
namespace astro {
namespace {

struct PeerPtrs {
  void* p[kMaxPeers];
};

// this rank's counts into every rank's mailbox: per-expert counts of rank d's
// experts into d's slot [me][*]; per-destination totals into row me of every
// rank's matrix
__global__ void ep_post_counts_kernel(const uint32_t* __restrict__ offsets, int El, int world,
                                      int me, int stride, const __grid_constant__ PeerPtrs mbox) {
  for (int i = threadIdx.x; i < world * El; i += blockDim.x) {
    const int d = i / El, e = i - d * El;
    const uint32_t c = offsets[d * El + e + 1] - offsets[d * El + e];
    reinterpret_cast<uint32_t*>(mbox.p[d])[me * stride + e] = c;
  }
  for (int i = threadIdx.x; i < world * world; i += blockDim.x) {
    const int r = i / world, d = i - r * world;  // to rank r: my total for d
    const uint32_t c = offsets[(d + 1) * El] - offsets[d * El];
    reinterpret_cast<uint32_t*>(mbox.p[r])[world * stride + me * world + d] = c;
  }
}

// prefix sums of the send matrix M[s][d] (this rank's mailbox) needed by a block
struct Placement {
  int64_t send_start[kMaxPeers];   // my rows for d start at this sorted position
  int64_t dest_off[kMaxPeers];     // ... and land from this row of d's receive buffer
  int64_t recv_start[kMaxPeers];   // rows from s start at this received row
  int64_t ret_off[kMaxPeers];      // ... and return to this row of s's return buffer
  int64_t recv_total;
};

ASTRO_DEVINL void load_placement(const uint32_t* __restrict__ M, int world, int me, Placement* P) {
  __shared__ uint32_t m[kMaxPeers * kMaxPeers];
  if (threadIdx.x < world * world) m[threadIdx.x] = __ldcg(M + threadIdx.x);  // one round trip
  __syncthreads();
  if (threadIdx.x == 0) {
    int64_t a = 0, t = 0;
    for (int d = 0; d < world; ++d) {
      P->send_start[d] = a;
      a += m[me * world + d];
      int64_t o = 0;
      for (int s = 0; s < me; ++s) o += m[s * world + d];
      P->dest_off[d] = o;
    }
    for (int s = 0; s < world; ++s) {
      P->recv_start[s] = t;
      t += m[s * world + me];
      int64_t o = 0;
      for (int d = 0; d < me; ++d) o += m[s * world + d];
      P->ret_off[s] = o;
    }
    P->recv_total = t;
  }
  __syncthreads();
}

__global__ void ep_push_rows_dev_kernel(const uint4* __restrict__ x, const uint32_t* __restrict__ stok,
                                       const uint32_t* __restrict__ sids, int64_t n, int El,
                                       int world, int me, int chunks, int64_t x_rows,
                                       const uint32_t* __restrict__ M,
                                       const __grid_constant__ PeerPtrs recv, int64_t cap_rows,
                                       uint32_t* __restrict__ status) {
  __shared__ Placement P;
  load_placement(M, world, me, &P);
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
    const int64_t row = P.dest_off[d] + (p - P.send_start[d]);
    if (row < 0 || row >= cap_rows) {
      record_status(status, kDevBadShape);
      continue;
    }
    reinterpret_cast<uint4*>(recv.p[d])[row * chunks + c] = x[(int64_t)tok * chunks + c];
  }
}

// received rows -> expert-major states (src_of), then this rank's own tokens
// appended as the shared expert's rows after the routed ones
template <bool PERM8>
__global__ void ep_gather_states_kernel(const uint4* __restrict__ recv,
                                        const uint32_t* __restrict__ src_of,
                                        const uint4* __restrict__ x, int64_t T, int world, int me,
                                        int chunks, const uint32_t* __restrict__ M,
                                        int64_t cap_rows, uint4* __restrict__ states,
                                        uint32_t* __restrict__ status) {
  __shared__ Placement P;
  load_placement(M, world, me, &P);
  const int64_t n = P.recv_total;
  if (n > cap_rows) {  // counts inconsistent with the receive buffer: touch nothing
    if (threadIdx.x == 0) record_status(status, kDevBadShape);
    return;
  }
  const int64_t total = (n + T) * chunks;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t q = i / chunks;
    const int c = (int)(i - q * chunks);
    if (q < n) {
      const uint32_t s = src_of[q];
      if (s >= (uint64_t)n) {
        record_status(status, kDevBadShape);
        continue;
      }
      const uint4 v = recv[(int64_t)s * chunks + c];
      states[q * chunks + c] = PERM8 ? perm8_bf16(v) : v;
    } else {
      const uint4 v = x[(q - n) * chunks + c];
      states[q * chunks + c] = PERM8 ? perm8_bf16(v) : v;
    }
  }
}

__global__ void ep_return_rows_dev_kernel(const uint4* __restrict__ yrows,
                                          const uint32_t* __restrict__ dest, int world, int me,
                                          int chunks, int64_t y_rows,
                                          const uint32_t* __restrict__ M,
                                          const __grid_constant__ PeerPtrs ret, int64_t cap_rows,
                                          uint32_t* __restrict__ status) {
  __shared__ Placement P;
  load_placement(M, world, me, &P);
  if (P.recv_total > y_rows) {
    if (threadIdx.x == 0) record_status(status, kDevBadShape);
    return;
  }
  const int64_t total = P.recv_total * chunks;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t q = i / chunks;
    const int c = (int)(i - q * chunks);
    int s = 0;
    while (s + 1 < world && q >= P.recv_start[s + 1]) ++s;
    const uint32_t src = dest[q];
    const int64_t row = P.ret_off[s] + (q - P.recv_start[s]);
    if (src >= (uint64_t)y_rows || row < 0 || row >= cap_rows) {
      record_status(status, kDevBadShape);
      continue;
    }
    reinterpret_cast<uint4*>(ret.p[s])[row * chunks + c] = yrows[(int64_t)src * chunks + c];
  }
}

PeerPtrs make_ptrs(void* const* p, int world) {
  PeerPtrs t{};
  for (int i = 0; i < world && i < kMaxPeers; ++i) t.p[i] = p[i];
  return t;
}

}  // namespace

cudaError_t launch_ep_post_counts(const uint32_t* offsets, int El, int world, int me,
                                  void* const* mailboxes, int stride, cudaStream_t st) {
  if (world < 1 || world > kMaxPeers || stride < El) return cudaErrorInvalidValue;
  ep_post_counts_kernel<<<1, 256, 0, st>>>(offsets, El, world, me, stride,
                                           make_ptrs(mailboxes, world));
  return cudaGetLastError();
}

cudaError_t launch_ep_push_rows_dev(const void* x, int64_t x_rows, const uint32_t* stok,
                                    const uint32_t* sids, int64_t n, int El, int world, int me,
                                    int H, const uint32_t* M, void* const* peer_recv,
                                    int64_t cap_rows, uint32_t* status, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  if (world < 1 || world > kMaxPeers || H % 8) return cudaErrorInvalidValue;
  ep_push_rows_dev_kernel<<<grid_rows(n, H / 8), 256, 0, st>>>(
      reinterpret_cast<const uint4*>(x), stok, sids, n, El, world, me, H / 8, x_rows, M,
      make_ptrs(peer_recv, world), cap_rows, status);
  return cudaGetLastError();
}

cudaError_t launch_ep_gather_states(const void* recv, const uint32_t* src_of, const void* x,
                                    int64_t T, int world, int me, int H, const uint32_t* M,
                                    int64_t cap_rows, void* states, uint32_t* status,
                                    cudaStream_t st, bool perm8) {
  if (world < 1 || world > kMaxPeers || H % 8) return cudaErrorInvalidValue;
  if (perm8)
    ep_gather_states_kernel<true><<<148 * 8, 256, 0, st>>>(
        reinterpret_cast<const uint4*>(recv), src_of, reinterpret_cast<const uint4*>(x), T, world,
        me, H / 8, M, cap_rows, reinterpret_cast<uint4*>(states), status);
  else
    ep_gather_states_kernel<false><<<148 * 8, 256, 0, st>>>(
        reinterpret_cast<const uint4*>(recv), src_of, reinterpret_cast<const uint4*>(x), T, world,
        me, H / 8, M, cap_rows, reinterpret_cast<uint4*>(states), status);
  return cudaGetLastError();
}

cudaError_t launch_ep_return_rows_dev(const void* yrows, int64_t y_rows, const uint32_t* dest,
                                      int world, int me, int H, const uint32_t* M,
                                      void* const* peer_ret, int64_t cap_rows, uint32_t* status,
                                      cudaStream_t st) {
  if (world < 1 || world > kMaxPeers || H % 8) return cudaErrorInvalidValue;
  ep_return_rows_dev_kernel<<<148 * 8, 256, 0, st>>>(
      reinterpret_cast<const uint4*>(yrows), dest, world, me, H / 8, y_rows, M,
      make_ptrs(peer_ret, world), cap_rows, status);
  return cudaGetLastError();
}

}  // namespace astro

namespace astro {
namespace {
__global__ void ep_copy_shared_rows_kernel(const uint4* __restrict__ yrows, int world, int me,
                                           int64_t T, int chunks, const uint32_t* __restrict__ M,
                                           int64_t y_rows, uint4* __restrict__ out) {
  __shared__ Placement P;
  load_placement(M, world, me, &P);
  const int64_t base = P.recv_total;
  if (base + T > y_rows) return;  // inconsistent counts (the gather recorded it)
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < T * chunks;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = yrows[base * chunks + i];
}
}  // namespace

cudaError_t launch_ep_copy_shared_rows(const void* yrows, int64_t y_rows, int world, int me,
                                       int64_t T, int H, const uint32_t* M, void* out,
                                       cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  ep_copy_shared_rows_kernel<<<148 * 2, 256, 0, st>>>(reinterpret_cast<const uint4*>(yrows), world,
                                                      me, T, H / 8, M, y_rows,
                                                      reinterpret_cast<uint4*>(out));
  return cudaGetLastError();
}
}  // namespace astro
