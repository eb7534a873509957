// moe_gemm.cu -- grouped expert GEMM on the 5th-generation tensor cores (sm_100a).
//
// Computes the gathered projections of the sorted MoE block
// (runtime-integration/src/mlx_quantized_operations.rs:100-157, gather_qmm with
// transpose=true and sorted indices) for MLX affine 4-bit, group-64 weights:
//
//   gate/up : act[row, f] = swiglu(bf16(x_row . Wg[e,f]), bf16(x_row . Wu[e,f]))
//             (qwen3_5_moe/model/resident_execution.rs:210-258 + mlx_compiled_swiglu.rs)
//   down    : y[row, f]   = bf16(act_row . Wd[e,f])
//   router  : logits[t,e] = bf16(x_t . Wr[e])        (forward.rs:52-93, dense bf16)
//
// Rows of one expert are contiguous after the sort, so a work unit is (expert
// segment, tile of <= kMaxN rows, block of weight rows).  The GEMM is "swap-AB":
// the weight tile is the MMA's A operand (M = 128 weight rows) and the token rows
// are B (N = the tile's row count rounded up to 16), so an expert with 130 rows
// costs N = 144, not two 128-row tiles, and every weight tile is dequantised once
// per unit.  A work item is one 64-wide K block (one quantisation group).
//
// Rings (per CTA, persistent, one CTA per SM):
//   raw  smem (kRawStages x 4 KB)  int4 weight rows, MLX layout, by TMA  <- warp 0
//   B    smem (kOpStages x 20 KB)  token rows, bf16, 128-byte swizzle, TMA <- warp 2
//   A    TMEM (kOpStages x 32 col) dequantised weights, written with one
//                                  tcgen05.st per row per item <- warps 12-27
//   scale table smem (2 units)     the unit's scales/biases, [group][A row] <- warp 3
// The MMA reads A from tensor memory, so shared memory only carries the raw
// codes, the token rows and the scale table; operand slots complete in pairs
// (one full barrier per two slots: their token bytes and dequant warps) and each
// slot has one empty barrier (one MMA commit).
// A tile of token rows is covered by the fewest 128/64/32/16-row boxes (each TMA
// issue has a fixed cost) and only rows the MMA reads are fetched; the rows are
// stored in the dequantisers' K order (perm8_bf16), so the conversion needs no
// byte permutes.  Four groups of 4 dequant warps take items round robin (nibbles
// -> bf16 with bf16x2 FMAs, w = s*q + b); each thread converts one 64-element
// weight row per item.  Warp 1 runs the MMA loop as a whole warp and one elected
// lane issues tcgen05.mma (M=128, N<=160, K=16), two K blocks per wait, into one
// of two TMEM accumulators and commits; eight epilogue warps (two per TMEM
// sub-partition) drain the others: tcgen05.ld -> SwiGLU (bf16 pairs) / bf16 ->
// global.  For gate/up the 128 A rows hold 64 gate and 64 up rows, interleaved
// in 16-row groups so each gate row and its up row land in lanes l and l+16 of
// the same epilogue warp (one shuffle pairs them).
// With full token tiles (prefill), a gate/up unit of the scale-table mode covers
// two weight-row blocks (FB = 2): one token-row slot per K block feeds the MMAs
// of both blocks, which accumulate into the two TMEM accumulators.
// The routed experts may be stacked tensors or the pages of a page pool
// (slot_of maps a segment to its slot; codes and scales get their own strides).
//
// Every mbarrier wait is bounded (2 s); on timeout the kernel records
// kDevWaitTimeout, waits (bounded) for its own copies and MMAs, frees TMEM and
// returns.  No cluster multicast is used anywhere.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <initializer_list>

#include "moe_gemm.h"
#include "tc_ptx.cuh"

namespace astro {

enum GemmMode : int { kGateUp = 0, kDown = 1, kRouter = 2 };

constexpr int kBM = 128;                  // weight rows per tile (MMA M)
constexpr int kBK = 64;                   // K per item = one quantisation group
constexpr int kMaxN = 160;                // token rows per tile (MMA N)
constexpr int kBoxRows = 16;              // granularity of token rows per TMA box
constexpr int kBoxKinds = 4;              // token-row boxes of 128, 64, 32 and 16 rows
constexpr int kABytes = kBM * kBK * 2;    // 16 KB bf16 A tile
constexpr int kBBytes = kMaxN * kBK * 2;  // 20 KB bf16 B tile
constexpr int kRawBytes = kBM * 32;       // 4 KB int4 A tile
constexpr int kRawStages = 8;   // multiple of kDqGroups
constexpr int kOpStages = 6;              // operand slots: B tile in smem (+ A tile, see below)
// Dequantised weights go to TMEM (A from tensor memory), so an operand slot of the
// quantised modes is just the B tile; the router's bf16 A comes by TMA into smem.
template <int MODE> constexpr int op_bytes() { return MODE == 2 ? kABytes + kBBytes : kBBytes; }
// Gate/up units of the scale-table mode cover FB = 2 weight-row blocks that
// share every token-row tile: one B slot per 64-wide K block feeds the MMAs of
// both blocks (their A tiles are two TMEM slots, their accumulators the two TMEM
// accumulators), so the token rows cross L2 -> SM once per two blocks.  The
// accumulators then hold one unit, so its epilogue does not overlap the next
// unit's MMAs; the operand rings keep filling meanwhile.
template <int FB> constexpr int b_slots() { return kOpStages / FB; }
template <int MODE, int FB = 1> constexpr int smem_bytes() {
  return b_slots<FB>() * op_bytes<MODE>() + (MODE == 2 ? 0 : kRawStages * kRawBytes) + 1024;
}
constexpr int kMaxSeg = 1025;
// Warp roles.  A warp can only reach the TMEM lanes of its own SM sub-partition
// (warp % 4), so the dequantisers, which write A rows 32*(warp%4).. into TMEM,
// and the epilogue warps, which read accumulator rows the same way, each cover
// all four sub-partitions.
constexpr int kRawWarp = 0, kMmaWarp = 1, kBWarp = 2;
// Warp 3 (scale-table mode, VEC == 0): copies a unit's scales and biases from
// global memory into shared memory, transposed to [group][A row], one unit ahead
// of the dequantisers (two buffers).  The mode needs K / 64 groups to be a
// multiple of 8 between 8 and kMaxScaleGroups (K = 512 ... 4096).
constexpr int kScaleWarp = 3;
constexpr int kScaleBufs = 2;
constexpr int kMaxScaleGroups = 64;
constexpr int kMaxScaleGroupsFB2 = 48;  // two blocks' tables, double-buffered, fit shared memory
__host__ __device__ constexpr int scale_buf_bytes(int groups) { return 2 * groups * 128 * 2; }  // scales + biases
constexpr int kEpiFirst = 4;       // warps 4..11: epilogue, two per TMEM sub-partition
constexpr int kEpiWarps = 8;
constexpr int kDqFirst = kEpiFirst + kEpiWarps;  // warps 12..27: dequantisers
constexpr int kDqGroups = 4;       // groups taking items round robin
constexpr int kDqGroupWarps = 4;   // one warp per sub-partition = 32 A rows each
constexpr int kDequantWarps = kDqGroups * kDqGroupWarps;
constexpr int kThreadsQ = (kDqFirst + kDequantWarps) * 32;
constexpr int kThreadsR = kDqFirst * 32;  // router: no dequantisers (A comes by TMA)

// epilogue: which half of the chunks (0/1) this warp drains, or -1
ASTRO_DEVINL int epi_half(int w) {
  return (w >= kEpiFirst && w < kEpiFirst + kEpiWarps) ? (w - kEpiFirst) / 4 : -1;
}
// dequant: group * 4 + warp-in-group, or -1 (warp-in-group == warp % 4)
ASTRO_DEVINL int dq_slot(int w) { return w >= kDqFirst ? w - kDqFirst : -1; }
static_assert(kOpStages % 2 == 0, "operand slots complete in pairs");
constexpr int kAccs = 2;                                    // TMEM accumulators in flight
constexpr int kAColsPerStage = kBK / 2;                     // 64 bf16 per row = 32 columns
constexpr int kACol0 = kAccs * kMaxN;                       // first TMEM column of the A ring
constexpr uint32_t kTmemCols = 512;
static_assert(kACol0 + kOpStages * kAColsPerStage <= (int)kTmemCols,
              "accumulators and the A ring must fit in TMEM");
static_assert(kRawStages % kDqGroups == 0, "raw ring must split evenly over dequant groups");
static_assert(kBBytes % 1024 == 0 && kABytes % 1024 == 0, "SW128 tiles need 1024-byte alignment");

struct GemmParams {
  CUtensorMap tm_a[2][2];  // [routed, shared][gate|down, up] raw int4 maps; router: bf16 map
  CUtensorMap tm_b[kBoxKinds];  // token rows, bf16, boxes {64, 128|64|32|16}, 128-byte swizzle
  const uint16_t* scales[2][2];
  const uint16_t* biases[2][2];
  int64_t a_row_base[2][2];   // first tensor row of expert 0 (the up half of a fused tensor: I)
  int64_t a_expert_rows[2];   // tensor rows per expert (I, 2I when fused, H for down)
  int64_t a_sb_expert_rows[2];  // scale/bias rows per expert (differs for pages)
  const uint32_t* slot_of;    // routed segment -> expert index in the stacks (pages); null: itself
  int groups_per_row;         // scales per weight row = K / 64
  int scale_vec;              // 0: shared-memory scale table; else groups per vector load (8, 4, 1)
  const uint32_t* seg_offsets;  // [nseg + 1]; nullptr: one segment [0, total_rows)
  int nseg;
  int shared_seg;
  int total_rows;
  int kblocks;     // K / 64
  int fb_count;    // weight-row blocks per segment
  int tile_rows;   // token rows per tile (<= kMaxN)
  uint16_t* out;   // bf16 output matrix
  int64_t ldo;
  int out_cols;    // valid output columns (router: E)
  int out_rows;    // rows available in `out`
  uint32_t* status;
};

struct Unit {
  int seg, row0, nrows, fb;
};

struct SmemCtl {
  uint64_t raw_full[kRawStages], raw_empty[kRawStages];
  // operand slots fill in pairs: op_full[s / 2] completes when both items of the
  // pair (slots 2i, 2i+1 of one ring round) are in; op_empty is per slot
  uint64_t op_full[kOpStages / 2], op_empty[kOpStages];
  uint64_t tfull[kAccs], tempty[kAccs];
  uint64_t mma_done;
  uint64_t sc_full[kScaleBufs], sc_empty[kScaleBufs];
  uint32_t tmem_base;
  int abort;
  int total_units;
  int prefix[kMaxSeg + 1];
  int offs[kMaxSeg + 1];
};

// expert index of a routed segment in the stacked tensors (a slot for pages)
ASTRO_DEVINL int64_t expert_of(const GemmParams& p, int seg) {
  return p.slot_of ? (int64_t)p.slot_of[seg] : (int64_t)seg;
}

// unit u -> (segment, rows, first weight-row block); a tile has fb_count / FB units
template <int FB>
ASTRO_DEVINL bool decode_unit(const SmemCtl& c, const GemmParams& p, int u, Unit& out) {
  const int per_tile = p.fb_count / FB;
  const int tile = u / per_tile;
  out.fb = (u - tile * per_tile) * FB;
  int lo = 0, hi = p.nseg - 1;
  while (lo < hi) {  // last segment whose first tile <= tile
    const int mid = (lo + hi + 1) >> 1;
    if (c.prefix[mid] <= tile) lo = mid; else hi = mid - 1;
  }
  out.seg = lo;
  out.row0 = c.offs[lo] + (tile - c.prefix[lo]) * p.tile_rows;
  const int end = c.offs[lo + 1];
  out.nrows = min(p.tile_rows, end - out.row0);
  return out.nrows > 0;
}

// 8 int4 codes (MLX order: code j at bits 4j) -> 8 bf16 = scale*q + bias, as
// four 32-bit words (q0,q4) (q1,q5) (q2,q6) (q3,q7): the GEMMs' K order
// (perm8_bf16), so no byte permutes are needed.  128+q is formed exactly by
// OR-ing the code into the mantissa of bf16 128.0; subtracting 128 is exact; one
// bf16x2 FMA per pair.
ASTRO_DEVINL uint4 dequant8(uint32_t w, __nv_bfloat162 s2, __nv_bfloat162 b2) {
  const __nv_bfloat162 k128 = __floats2bfloat162_rn(128.0f, 128.0f);
  uint32_t t[4];
  t[0] = (w & 0x000f000fu) | 0x43004300u;          // (q0, q4)
  t[1] = ((w >> 4) & 0x000f000fu) | 0x43004300u;   // (q1, q5)
  t[2] = ((w >> 8) & 0x000f000fu) | 0x43004300u;   // (q2, q6)
  t[3] = ((w >> 12) & 0x000f000fu) | 0x43004300u;  // (q3, q7)
  uint32_t v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 q = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&t[i]), k128);
    __nv_bfloat162 r = __hfma2(q, s2, b2);
    v[i] = *reinterpret_cast<uint32_t*>(&r);
  }
  return make_uint4(v[0], v[1], v[2], v[3]);
}

// ring bookkeeping for item k in a ring of S slots
ASTRO_DEVINL int slot_of(int k, int S) { return k % S; }
ASTRO_DEVINL uint32_t full_parity(int k, int S) { return (uint32_t)(k / S) & 1u; }
ASTRO_DEVINL uint32_t empty_parity(int k, int S) { return ((uint32_t)(k / S) & 1u) ^ 1u; }

template <int MODE, int VEC, int FB>
__global__ void __launch_bounds__(MODE == kRouter ? kThreadsR : kThreadsQ, 1)
    moe_gemm_kernel(const __grid_constant__ GemmParams p) {
  static_assert(FB == 1 || (FB == 2 && MODE == kGateUp && VEC == 0),
                "two weight-row blocks per unit: gate/up with the scale table only");
  constexpr int kBS = b_slots<FB>();  // token-row (B) slots
  extern __shared__ uint8_t smem_raw[];
  __shared__ SmemCtl ctl;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  constexpr int kOpBytes = op_bytes<MODE>();
  uint8_t* ring_op = smem;                                 // kBS x ([A tile,] B tile)
  uint8_t* ring_raw = ring_op + kBS * kOpBytes;            // kRawStages x kRawBytes
  auto a_at = [&](int s) { return ring_op + s * kOpBytes; };           // router only
  auto b_at = [&](int s) { return ring_op + s * kOpBytes + (kOpBytes - kBBytes); };
  auto raw_at = [&](int s) { return ring_raw + s * kRawBytes; };
  // scale-table mode: kScaleBufs x FB x ([groups][128] scales, then [groups][128] biases)
  uint8_t* ring_sc = ring_raw + kRawStages * kRawBytes;
  auto sc_at = [&](int b) {
    return reinterpret_cast<uint16_t*>(ring_sc + b * FB * scale_buf_bytes(p.groups_per_row));
  };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort = &ctl.abort;
  const int KB = p.kblocks;
  constexpr int kFeat = (MODE == kGateUp) ? 64 : 128;  // output features per unit

  // ---- setup: segment table, barriers (warp kRawWarp), TMEM (warp kMmaWarp) ----
  if (warp == kRawWarp) {
    int carry = 0;
    for (int base = 0; base < p.nseg; base += 32) {
      const int s = base + lane;
      int c = 0;
      if (s < p.nseg) {
        const int o0 = p.seg_offsets ? (int)p.seg_offsets[s] : 0;
        const int o1 = p.seg_offsets ? (int)p.seg_offsets[s + 1] : p.total_rows;
        c = (o1 - o0 + p.tile_rows - 1) / p.tile_rows;
        ctl.offs[s] = o0;
        if (s == p.nseg - 1) ctl.offs[s + 1] = o1;
      }
      int incl = c;
#pragma unroll
      for (int m = 1; m < 32; m <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, incl, m);
        if (lane >= m) incl += o;
      }
      if (s < p.nseg) ctl.prefix[s] = carry + incl - c;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      ctl.prefix[p.nseg] = carry;
      ctl.total_units = carry * (p.fb_count / FB);
      ctl.abort = 0;
      for (int s = 0; s < kRawStages; ++s) {
        tc::mbar_init(&ctl.raw_full[s], 1);
        tc::mbar_init(&ctl.raw_empty[s], kDqGroupWarps);
      }
      // an operand slot is full after the token producer's expect-tx arrival
      // (+ its bytes) and the A tile: 4 dequant warps, or the weight producer's
      // expect-tx arrival for the router's TMA-loaded bf16 A
      for (int s = 0; s < kOpStages; ++s) {
        if constexpr (FB == 2) {
          // one slot per K block: the token producer's arrival and both A tiles
          if (s < kBS) {
            tc::mbar_init(&ctl.op_full[s], 1 + FB * kDqGroupWarps);
            tc::mbar_init(&ctl.op_empty[s], 1);
          }
        } else {
          if ((s & 1) == 0)
            tc::mbar_init(&ctl.op_full[s >> 1], 2 * (1 + (MODE == kRouter ? 1 : kDqGroupWarps)));
          tc::mbar_init(&ctl.op_empty[s], 1);
        }
      }
      for (int a = 0; a < kAccs; ++a) {
        tc::mbar_init(&ctl.tfull[a], 1);
        tc::mbar_init(&ctl.tempty[a], kEpiWarps);
      }
      tc::mbar_init(&ctl.mma_done, 1);
      for (int b = 0; b < kScaleBufs; ++b) {
        tc::mbar_init(&ctl.sc_full[b], 1);
        tc::mbar_init(&ctl.sc_empty[b], kDequantWarps);
      }
      tc::fence_mbar_init();
      for (int b = 0; b < kBoxKinds; ++b) tc::prefetch_tmap(&p.tm_b[b]);
      tc::prefetch_tmap(&p.tm_a[0][0]);
    }
  } else if (warp == kMmaWarp) {
    tc::tmem_alloc(&ctl.tmem_base, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = ctl.tmem_base;
  const int total_units = ctl.total_units;

  if (warp == kRawWarp) {
    // ================= weight producer (raw int4 rows; router: bf16 A) =================
    if (lane == 0) {
      int k = 0;
      int last_k = -1;
      for (int u = blockIdx.x; u < total_units && !*abort; u += gridDim.x) {
        Unit U;
        if (!decode_unit<FB>(ctl, p, u, U)) continue;
        const bool shared = (U.seg == p.shared_seg);
        const int wi = shared ? 1 : 0;
        const int64_t e = shared ? 0 : expert_of(p, U.seg);
        for (int kb = 0; kb < KB; ++kb) {
          for (int h = 0; h < FB; ++h, ++k) {  // weight-row block U.fb + h of the unit
          if constexpr (MODE == kRouter) {
            const int s = slot_of(k, kOpStages);
            if (!tc::mbar_wait(&ctl.op_empty[s], empty_parity(k, kOpStages), abort, p.status))
              goto raw_done;
            tc::mbar_arrive_expect_tx(&ctl.op_full[s >> 1], (uint32_t)kABytes);
            tc::tma_load_2d(a_at(s), &p.tm_a[0][0], kb * kBK, U.fb * kBM, &ctl.op_full[s >> 1]);
          } else {
            const int s = slot_of(k, kRawStages);
            if (!tc::mbar_wait(&ctl.raw_empty[s], empty_parity(k, kRawStages), abort, p.status))
              goto raw_done;
            tc::mbar_arrive_expect_tx(&ctl.raw_full[s], (uint32_t)kRawBytes);
            if constexpr (MODE == kGateUp) {
              const int64_t r0 = e * p.a_expert_rows[wi] + (int64_t)(U.fb + h) * 64;
              tc::tma_load_2d(raw_at(s), &p.tm_a[wi][0], kb * 8,
                              (int32_t)(p.a_row_base[wi][0] + r0), &ctl.raw_full[s]);
              tc::tma_load_2d(raw_at(s) + 2048, &p.tm_a[wi][1], kb * 8,
                              (int32_t)(p.a_row_base[wi][1] + r0), &ctl.raw_full[s]);
            } else {
              const int64_t r0 = e * p.a_expert_rows[wi] + (int64_t)(U.fb + h) * kBM;
              tc::tma_load_2d(raw_at(s), &p.tm_a[wi][0], kb * 8,
                              (int32_t)(p.a_row_base[wi][0] + r0), &ctl.raw_full[s]);
            }
          }
          last_k = k;
          }
        }
      }
    raw_done:
      if (*abort) {
        // let this thread's own copies land before the CTA exits (bounded)
        int dummy = 0;
        // only the last issue of each slot can still be in flight
        const int ring = (MODE == kRouter) ? kOpStages : kRawStages;
        for (int k2 = (last_k - ring + 1 > 0 ? last_k - ring + 1 : 0); k2 <= last_k; ++k2) {
          if (MODE == kRouter)
            tc::mbar_wait(&ctl.op_full[slot_of(k2, kOpStages) >> 1], full_parity(k2, kOpStages),
                          (volatile int*)&dummy, nullptr, 50000000ull);
          else
            tc::mbar_wait(&ctl.raw_full[slot_of(k2, kRawStages)], full_parity(k2, kRawStages),
                          (volatile int*)&dummy, nullptr, 50000000ull);
        }
      }
    }
  } else if (warp == kBWarp) {
    // ================= token-row producer =================
    if (lane == 0) {
      int k = 0;
      int last_k = -1;
      for (int u = blockIdx.x; u < total_units && !*abort; u += gridDim.x) {
        Unit U;
        if (!decode_unit<FB>(ctl, p, u, U)) continue;
        // cover the rows the MMA reads with the fewest boxes (each TMA issue has a
        // fixed cost): 144 rows -> one 128-row box and one 16-row box
        const int rows16 = (U.nrows + kBoxRows - 1) / kBoxRows * kBoxRows;
        const uint32_t bytes = (uint32_t)rows16 * 128;
        for (int kb = 0; kb < KB; ++kb, ++k) {
          const int s = slot_of(k, kBS);
          if (!tc::mbar_wait(&ctl.op_empty[s], empty_parity(k, kBS), abort, p.status))
            goto b_done;
          uint64_t* full = &ctl.op_full[FB == 2 ? s : s >> 1];
          tc::mbar_arrive_expect_tx(full, bytes);
          int off = 0;
#pragma unroll
          for (int b = 0; b < kBoxKinds; ++b) {
            const int box = 128 >> b;
            while (rows16 - off >= box) {
              tc::tma_load_2d(b_at(s) + off * 128, &p.tm_b[b], kb * kBK, U.row0 + off, full);
              off += box;
            }
          }
          last_k = k;
        }
      }
    b_done:
      if (*abort) {
        int dummy = 0;
        for (int k2 = (last_k - kBS + 1 > 0 ? last_k - kBS + 1 : 0); k2 <= last_k; ++k2)
          tc::mbar_wait(&ctl.op_full[FB == 2 ? slot_of(k2, kBS) : slot_of(k2, kBS) >> 1],
                        full_parity(k2, kBS), (volatile int*)&dummy, nullptr, 50000000ull);
      }
    }
  } else if (warp == kScaleWarp) {
    // ================= scale-table loader (VEC == 0) =================
    if constexpr (VEC == 0 && MODE != kRouter) {
      const int G = p.groups_per_row;
      int ui = 0;
      for (int u = blockIdx.x; u < total_units && !*abort; u += gridDim.x, ++ui) {
        Unit U;
        if (!decode_unit<FB>(ctl, p, u, U)) break;
        const int buf = ui & 1;
        if (!tc::mbar_wait(&ctl.sc_empty[buf], ((uint32_t)(ui >> 1) & 1u) ^ 1u, abort, p.status))
          break;
        const bool shared = (U.seg == p.shared_seg);
        const int wsel = shared ? 1 : 0;
        const int64_t e = shared ? 0 : expert_of(p, U.seg);
        for (int h = 0; h < FB; ++h) {  // table of weight-row block U.fb + h
        uint16_t* ssm = sc_at(buf) + h * 2 * G * kBM;
        uint16_t* bsm = ssm + G * kBM;
        // this lane copies A rows r = lane + 32 q (the rows the dequantisers'
        // thread r converts), eight groups per 16-byte load
        const uint4* sp[4];
        const uint4* bp[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          int j = 0, f_local = lane + 32 * q;
          if constexpr (MODE == kGateUp) {
            j = lane < 16 ? 0 : 1;
            f_local = q * 16 + (lane & 15);
          }
          const int64_t grow = p.a_row_base[wsel][j] + e * p.a_sb_expert_rows[wsel] +
                               (int64_t)(U.fb + h) * kFeat + f_local;
          sp[q] = reinterpret_cast<const uint4*>(p.scales[wsel][j] + grow * G);
          bp[q] = reinterpret_cast<const uint4*>(p.biases[wsel][j] + grow * G);
        }
        for (int v = 0; v < G / 8; ++v) {
          uint4 sv[4], bv[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            sv[q] = __ldg(sp[q] + v);
            bv[q] = __ldg(bp[q] + v);
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t ws[4] = {sv[q].x, sv[q].y, sv[q].z, sv[q].w};
            const uint32_t wb[4] = {bv[q].x, bv[q].y, bv[q].z, bv[q].w};
            const int r = lane + 32 * q;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              ssm[(8 * v + i) * kBM + r] = (uint16_t)(ws[i >> 1] >> (16 * (i & 1)));
              bsm[(8 * v + i) * kBM + r] = (uint16_t)(wb[i >> 1] >> (16 * (i & 1)));
            }
          }
        }
        }
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&ctl.sc_full[buf]);
      }
    }
  } else if (warp == kMmaWarp) {
    // ================= MMA issuer =================
    // The whole warp runs the loop, so its bookkeeping is warp-uniform; one
    // elected lane (always lane 0 with all lanes active) issues the MMAs and
    // commits.  A loop run by lane 0 alone measured 1.6x slower per K block on
    // B200 when the warps sharing its scheduler keep the ALU pipe busy, as the
    // dequantisers do.
    {
      int os = 0;          // operand slot of the next item
      uint32_t oph = 0;    // its round parity
      int acc = 0;
      uint32_t acc_phase = 0;
      // descriptors of operand slot 0; slot s adds s * (slot bytes >> 4) to the
      // low word (the 14-bit start-address field cannot carry: smem < 256 KB)
      const uint64_t bd0 = tc::sdesc_sw128(tc::smem_u32(b_at(0)));
      const uint32_t b_lo0 = (uint32_t)bd0, b_hi = (uint32_t)(bd0 >> 32);
      const uint64_t ad0 = tc::sdesc_sw128(tc::smem_u32(a_at(0)));
      const uint32_t a_lo0 = (uint32_t)ad0, a_hi = (uint32_t)(ad0 >> 32);
      constexpr uint32_t kSlotStep = (uint32_t)(kOpBytes >> 4);
      const uint32_t a_tmem0 = tmem_base + (uint32_t)kACol0;
      if constexpr (FB == 2) {
        // K block kb of a unit: slot ks holds its token rows (B) and the A tiles
        // of both weight-row blocks (TMEM slots 2 ks, 2 ks + 1); block h
        // accumulates into TMEM columns h * kMaxN.  One wait covers 8 MMAs.
        int ks = 0;
        uint32_t kph = 0;
        for (int u = blockIdx.x; u < total_units && !*abort; u += gridDim.x) {
          Unit U;
          if (!decode_unit<FB>(ctl, p, u, U)) continue;
          const int n = (U.nrows + 15) & ~15;
          const uint32_t idesc = tc::idesc_bf16(kBM, n);
          if (!tc::mbar_wait(&ctl.tempty[0], acc_phase ^ 1u, abort, p.status)) break;
          tc::tc_fence_after();
          for (int kb = 0; kb < KB; ++kb) {
            if (!tc::mbar_wait(&ctl.op_full[ks], kph, abort, p.status)) goto mma_done;
            tc::tc_fence_after();
            if (tc::elect_one()) {
              const uint32_t b_lo = b_lo0 + (uint32_t)ks * kSlotStep;
#pragma unroll
              for (int h = 0; h < FB; ++h)
                tc::mma4_bf16_ts(tmem_base + (uint32_t)(h * kMaxN),
                                 a_tmem0 + (uint32_t)((FB * ks + h) * kAColsPerStage), b_lo, b_hi,
                                 idesc, (uint32_t)kb);
              tc::mma_commit(&ctl.op_empty[ks]);
            }
            __syncwarp();
            if (++ks == kBS) { ks = 0; kph ^= 1u; }
          }
          if (tc::elect_one()) tc::mma_commit(&ctl.tfull[0]);
          __syncwarp();
          acc_phase ^= 1u;
        }
      } else {
      for (int u = blockIdx.x; u < total_units && !*abort; u += gridDim.x) {
        Unit U;
        if (!decode_unit<FB>(ctl, p, u, U)) continue;
        const int n = (U.nrows + 15) & ~15;
        const uint32_t idesc = tc::idesc_bf16(kBM, n);
        if (!tc::mbar_wait(&ctl.tempty[acc], acc_phase ^ 1u, abort, p.status)) break;
        tc::tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * kMaxN);
        // Items are issued in pairs: every barrier wait between MMA issues stalls
        // the issue until the tensor pipe has worked off the MMAs already issued
        // (about 450 cycles a round on B200), so one wait covers two 64-wide K
        // blocks (576 cycles of MMA at N = 144).  A unit with an odd number of
        // K blocks leaves a pair split across units: its first item waits, the
        // second one is covered.
        auto issue = [&](int k, int s) {
          const uint32_t b_lo = b_lo0 + (uint32_t)s * kSlotStep;
          if constexpr (MODE == kRouter) {
            tc::mma4_bf16_ss(d_tmem, a_lo0 + (uint32_t)s * kSlotStep, a_hi, b_lo, b_hi, idesc,
                             (uint32_t)k);
          } else {
            // K = 16 bf16 = 8 TMEM columns of A per MMA, 32 bytes of B
            tc::mma4_bf16_ts(d_tmem, a_tmem0 + (uint32_t)(s * kAColsPerStage), b_lo, b_hi, idesc,
                             (uint32_t)k);
          }
          tc::mma_commit(&ctl.op_empty[s]);
        };
        for (int kb = 0; kb < KB;) {
          const bool pair = (os & 1) == 0 && kb + 1 < KB;
          if ((os & 1) == 0) {
            if (!tc::mbar_wait(&ctl.op_full[os >> 1], oph, abort, p.status)) goto mma_done;
            tc::tc_fence_after();
          }
          if (tc::elect_one()) {
            issue(kb, os);
            if (pair) issue(kb + 1, os + 1);
          }
          __syncwarp();
          const int step = pair ? 2 : 1;
          kb += step;
          os += step;
          if (os == kOpStages) { os = 0; oph ^= 1u; }
        }
        if (tc::elect_one()) tc::mma_commit(&ctl.tfull[acc]);
        __syncwarp();
        if (++acc == kAccs) { acc = 0; acc_phase ^= 1u; }
      }
      }  // FB == 1
    mma_done:
      // every MMA issued by this warp's lane 0 completes before TMEM is released
      if (tc::elect_one()) {
        tc::mma_commit(&ctl.mma_done);
        int dummy = 0;
        tc::mbar_wait(&ctl.mma_done, 0, (volatile int*)&dummy, p.status, 200000000ull);
      }
      __syncwarp();
    }
  } else if (epi_half(warp) >= 0) {
    // ================= epilogue (TMEM -> registers -> global) =================
    // Two warps per TMEM sub-partition take alternate 16-column chunks; the
    // load of the next chunk is in flight while the current one is converted.
    const int sub = warp & 3;                    // TMEM sub-partition this warp may access
    const int half = epi_half(warp);             // which alternate chunks
    int acc = 0;
    uint32_t acc_phase = 0;
    auto process = [&](const uint32_t (&v)[16], const Unit& U, int fb, int cb) {
      const int rbase = U.row0 + cb * 16;
      if constexpr (MODE == kGateUp) {
        // Lane l < 16 holds gate feature f = 16*sub + l for the chunk's 16 token
        // rows, lane l + 16 the up feature f.  Each lane packs its values in
        // bf16 pairs of rows (2i, 2i+1); lanes l and l+16 trade pairs so that
        // lane l finishes rows 0..7 and lane l + 16 rows 8..15 of feature f.
        const bool lo_half = lane < 16;
        // feature f goes to its position in the K order of the down GEMM's B
        const int f = fb * 64 + sub * 16 + (lane & 15);
        const int col = (f & ~7) | perm8_pos(f & 7);
        const int r0 = lo_half ? 0 : 8;  // first chunk row of this lane
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const __nv_bfloat162 b = __floats2bfloat162_rn(__uint_as_float(v[2 * i]),
                                                         __uint_as_float(v[2 * i + 1]));
          pk[i] = *reinterpret_cast<const uint32_t*>(&b);
        }
        const bool full = cb * 16 + 16 <= U.nrows && rbase + 16 <= p.out_rows;
        uint16_t* dst = p.out + (int64_t)(rbase + r0) * p.ldo + col;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t recv = __shfl_xor_sync(0xffffffffu, lo_half ? pk[4 + i] : pk[i], 16);
          const uint32_t g2 = lo_half ? pk[i] : recv, u2 = lo_half ? recv : pk[4 + i];
          const __nv_bfloat162 o = swiglu_bf16x2(*reinterpret_cast<const __nv_bfloat162*>(&g2),
                                                 *reinterpret_cast<const __nv_bfloat162*>(&u2));
          const uint32_t ob = *reinterpret_cast<const uint32_t*>(&o);
          const int j = r0 + 2 * i;  // chunk row of the low half
          if (full) {
            dst[(int64_t)(2 * i) * p.ldo] = (uint16_t)ob;
            dst[(int64_t)(2 * i + 1) * p.ldo] = (uint16_t)(ob >> 16);
          } else if (col < p.out_cols) {
            if (cb * 16 + j < U.nrows && rbase + j < p.out_rows)
              dst[(int64_t)(2 * i) * p.ldo] = (uint16_t)ob;
            if (cb * 16 + j + 1 < U.nrows && rbase + j + 1 < p.out_rows)
              dst[(int64_t)(2 * i + 1) * p.ldo] = (uint16_t)(ob >> 16);
          }
        }
      } else {
        // lanes l and l^1 trade one value so each stores a bf16 pair of
        // adjacent features: even lanes token 2m, odd lanes token 2m+1
        const int colbase = fb * kFeat + 32 * sub + (lane & ~1);
        const bool odd = lane & 1;
        const bool full = cb * 16 + 16 <= U.nrows && rbase + 16 <= p.out_rows &&
                          colbase + 1 < p.out_cols;
        __nv_bfloat162* dst2 =
            reinterpret_cast<__nv_bfloat162*>(p.out + (int64_t)(rbase + (odd ? 1 : 0)) * p.ldo + colbase);
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const uint32_t send = odd ? v[2 * m] : v[2 * m + 1];
          const uint32_t recv = __shfl_xor_sync(0xffffffffu, send, 1);
          const float lo = __uint_as_float(odd ? recv : v[2 * m]);
          const float hi = __uint_as_float(odd ? v[2 * m + 1] : recv);
          const int j = 2 * m + (odd ? 1 : 0);
          const int row = rbase + j;
          if (full) {
            // row rbase + j = the first row of this lane + 2m
            *reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<uint16_t*>(dst2) +
                                               (int64_t)(2 * m) * p.ldo) =
                __floats2bfloat162_rn(lo, hi);
          } else if (j + cb * 16 < U.nrows && row < p.out_rows && colbase < p.out_cols) {
            uint16_t* dst = p.out + (int64_t)row * p.ldo + colbase;
            if (colbase + 1 < p.out_cols) {
              const __nv_bfloat162 pr = __floats2bfloat162_rn(lo, hi);
              *reinterpret_cast<__nv_bfloat162*>(dst) = pr;
            } else {
              dst[0] = f32_to_bf16(lo);
            }
          }
        }
      }
    };
    for (int u = blockIdx.x; u < total_units && !*abort; u += gridDim.x) {
      Unit U;
      if (!decode_unit<FB>(ctl, p, u, U)) continue;
      if (!tc::mbar_wait(&ctl.tfull[acc], acc_phase, abort, p.status)) break;
      tc::tc_fence_after();
      const int nch = ((U.nrows + 15) & ~15) / 16;
      // chunks q of the unit: FB == 2 runs over both accumulators (weight-row
      // blocks U.fb, U.fb + 1: chunks nch of each), else over accumulator acc
      const uint32_t tb = tmem_base + ((uint32_t)(32 * sub) << 16) +
                          (uint32_t)((FB == 2 ? 0 : acc) * kMaxN);
      const int nq = FB * nch;
      auto blk = [&](int q) { return (FB == 2 && q >= nch) ? 1 : 0; };
      auto tcol = [&](int q) { return (uint32_t)(blk(q) * (kMaxN - 16 * nch) + q * 16); };
      uint32_t va[16], vb[16];
      int q = half;
      if (q < nq) tc::tmem_ld16(tb + tcol(q), va);
      while (q < nq) {
        tc::tmem_ld_wait16(va);
        if (q + 2 < nq) tc::tmem_ld16(tb + tcol(q + 2), vb);
        process(va, U, U.fb + blk(q), q - blk(q) * nch);
        q += 2;
        if (q >= nq) break;
        tc::tmem_ld_wait16(vb);
        if (q + 2 < nq) tc::tmem_ld16(tb + tcol(q + 2), va);
        process(vb, U, U.fb + blk(q), q - blk(q) * nch);
        q += 2;
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&ctl.tempty[acc]);
      if (FB == 2) {
        acc_phase ^= 1u;
      } else if (++acc == kAccs) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  } else if constexpr (MODE != kRouter) {
    if (dq_slot(warp) >= 0) {
    // ================= dequantisers =================
    // Group g takes items k = g, g + kDqGroups, ...  Thread r converts weight row r
    // of the A tile (64 elements = 8 packed words) per item.  The row's scales and
    // biases come from the shared-memory table (VEC == 0) or VEC groups per
    // vector load, one vector ahead of use.
    const int grp = dq_slot(warp) / kDqGroupWarps;
    const int r = (warp & 3) * 32 + lane;  // A tile row = TMEM lane this thread may write
    const uint32_t lane_addr = (uint32_t)((warp & 3) * 32) << 16;
    int raw_row, j, f_local;
    if constexpr (MODE == kGateUp) {
      const int within = r & 31, g4 = r >> 5;
      j = within < 16 ? 0 : 1;
      f_local = g4 * 16 + (within & 15);
      raw_row = j * 64 + f_local;
    } else {
      j = 0;
      f_local = r;
      raw_row = r;
    }
    auto row_of = [&](int ui, int64_t& grow, int& wsel) -> bool {
      const int u = blockIdx.x + ui * gridDim.x;
      if (u >= total_units) return false;
      Unit U;
      if (!decode_unit<FB>(ctl, p, u, U)) return false;
      const bool shared = (U.seg == p.shared_seg);
      wsel = shared ? 1 : 0;
      const int64_t e = shared ? 0 : expert_of(p, U.seg);
      grow = p.a_row_base[wsel][j] + e * p.a_sb_expert_rows[wsel] + (int64_t)U.fb * kFeat + f_local;
      return true;
    };
    auto load_vec = [&](int wsel, int64_t grow, int vid, uint4& vs, uint4& vb) {
      const int64_t off = grow * p.groups_per_row + (int64_t)vid * VEC;
      const uint16_t* sp = p.scales[wsel][j] + off;
      const uint16_t* bp = p.biases[wsel][j] + off;
      if constexpr (VEC == 8) {
        vs = __ldg(reinterpret_cast<const uint4*>(sp));
        vb = __ldg(reinterpret_cast<const uint4*>(bp));
      } else if constexpr (VEC == 4) {
        const uint2 a = __ldg(reinterpret_cast<const uint2*>(sp));
        const uint2 c = __ldg(reinterpret_cast<const uint2*>(bp));
        vs = make_uint4(a.x, a.y, 0u, 0u);
        vb = make_uint4(c.x, c.y, 0u, 0u);
      } else {
        vs = make_uint4(__ldg(sp), 0u, 0u, 0u);
        vb = make_uint4(__ldg(bp), 0u, 0u, 0u);
      }
    };
    auto pick = [](const uint4& v, int q) -> uint16_t {
      const uint32_t w = (q < 4) ? ((q < 2) ? v.x : v.y) : ((q < 6) ? v.z : v.w);
      return (uint16_t)((q & 1) ? (w >> 16) : (w & 0xffffu));
    };
    if constexpr (VEC == 0) {
      // scale-table mode: the unit's scales and biases are in shared memory,
      // [block][group][A row]; KB >= 8, so every group has items in every unit and
      // a unit ends at most once per item.  Item it of a unit is K block it / FB of
      // weight-row block it % FB (with FB == 2 a group keeps one block).
      int ui = 0, it = grp;
      int rs = grp, os = grp;
      uint32_t rph = 0, oph = 0;
      int waited = -1;
      while (!*abort) {
        if (blockIdx.x + ui * gridDim.x >= total_units) break;
        if (ui != waited) {
          if (!tc::mbar_wait(&ctl.sc_full[ui & 1], (uint32_t)(ui >> 1) & 1u, abort, p.status))
            break;
          waited = ui;
        }
        const int kb = it / FB;
        const uint16_t* ssm = sc_at(ui & 1) + (it - kb * FB) * 2 * p.groups_per_row * kBM;
        const uint16_t s16 = ssm[kb * kBM + r];
        const uint16_t b16 = ssm[(p.groups_per_row + kb) * kBM + r];
        if (!tc::mbar_wait(&ctl.raw_full[rs], rph, abort, p.status)) break;
        const uint4 w0 = *reinterpret_cast<const uint4*>(raw_at(rs) + raw_row * 32);
        const uint4 w1 = *reinterpret_cast<const uint4*>(raw_at(rs) + raw_row * 32 + 16);
        const __nv_bfloat162 s2 = __bfloat162bfloat162(__ushort_as_bfloat16(s16));
        const __nv_bfloat162 b2 = __bfloat162bfloat162(__ushort_as_bfloat16(b16));
        uint32_t o[32];
        const uint32_t ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint4 d = dequant8(ws[i], s2, b2);
          o[4 * i] = d.x; o[4 * i + 1] = d.y; o[4 * i + 2] = d.z; o[4 * i + 3] = d.w;
        }
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&ctl.raw_empty[rs]);
        // the slot's previous MMAs are done (FB == 2: one barrier per K-block slot)
        if (!tc::mbar_wait(&ctl.op_empty[FB == 2 ? os >> 1 : os], oph ^ 1u, abort, p.status))
          break;
        tc::tc_fence_after();
        tc::tmem_st32(tmem_base + lane_addr + (uint32_t)(kACol0 + os * kAColsPerStage), o);
        tc::tmem_st_wait();
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&ctl.op_full[os >> 1]);
        it += kDqGroups;
        if (it >= FB * KB) {  // this warp is done with the unit's scale table
          it -= FB * KB;
          if (lane == 0) tc::mbar_arrive(&ctl.sc_empty[ui & 1]);
          ++ui;
        }
        rs += kDqGroups;
        if (rs >= kRawStages) { rs -= kRawStages; rph ^= 1u; }
        os += kDqGroups;
        if (os >= kOpStages) { os -= kOpStages; oph ^= 1u; }
      }
    } else {
    int ui = 0, kb = grp;
    while (kb >= KB) { kb -= KB; ++ui; }
    int rs = grp, os = grp;       // ring slots of item k = grp, grp + kDqGroups, ...
    uint32_t rph = 0, oph = 0;    // their round parities
    int cu = -1, cw = 0;          // decoded unit of the current item
    int64_t cg = 0;
    int c_ui = -1, c_vid = -1;    // vector in use
    uint4 cs = make_uint4(0, 0, 0, 0), cb = cs;
    int n_ui = -1, n_vid = -1;    // prefetched vector
    uint4 ns = cs, nb = cs;
    while (!*abort) {
      if (ui != cu) {
        if (!row_of(ui, cg, cw)) break;
        cu = ui;
      }
      const int vid = kb / VEC;
      if (ui != c_ui || vid != c_vid) {
        if (ui == n_ui && vid == n_vid) { cs = ns; cb = nb; }
        else load_vec(cw, cg, vid, cs, cb);
        c_ui = ui;
        c_vid = vid;
        int pui = ui, pvid = vid + 1;
        if (pvid * VEC >= KB) { pui = ui + 1; pvid = 0; }
        int64_t pg = cg;
        int pw = cw;
        if (pui == ui || row_of(pui, pg, pw)) {
          load_vec(pw, pg, pvid, ns, nb);
          n_ui = pui;
          n_vid = pvid;
        } else {
          n_ui = -1;
        }
      }
      const int q = kb - vid * VEC;
      const uint16_t s16 = pick(cs, q), b16 = pick(cb, q);
      if (!tc::mbar_wait(&ctl.raw_full[rs], rph, abort, p.status)) break;
      const uint4 w0 = *reinterpret_cast<const uint4*>(raw_at(rs) + raw_row * 32);
      const uint4 w1 = *reinterpret_cast<const uint4*>(raw_at(rs) + raw_row * 32 + 16);
      const __nv_bfloat162 s2 = __bfloat162bfloat162(__ushort_as_bfloat16(s16));
      const __nv_bfloat162 b2 = __bfloat162bfloat162(__ushort_as_bfloat16(b16));
      uint32_t o[32];  // 64 bf16 of row r in K order, two per TMEM column
      const uint32_t ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint4 d = dequant8(ws[i], s2, b2);
        o[4 * i] = d.x; o[4 * i + 1] = d.y; o[4 * i + 2] = d.z; o[4 * i + 3] = d.w;
      }
      // the raw slot is free once its words are consumed
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&ctl.raw_empty[rs]);
      if (!tc::mbar_wait(&ctl.op_empty[os], oph ^ 1u, abort, p.status)) break;
      tc::tc_fence_after();
      tc::tmem_st32(tmem_base + lane_addr + (uint32_t)(kACol0 + os * kAColsPerStage), o);
      tc::tmem_st_wait();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&ctl.op_full[os >> 1]);
      kb += kDqGroups;
      while (kb >= KB) { kb -= KB; ++ui; }
      rs += kDqGroups;
      if (rs >= kRawStages) { rs -= kRawStages; rph ^= 1u; }
      os += kDqGroups;
      if (os >= kOpStages) { os -= kOpStages; oph ^= 1u; }
    }
    }  // VEC != 0
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ===========================================================================
// host side
// ===========================================================================
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2D map over a row-major matrix: `cols` elements of `elem_bytes` per row.
bool make_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int elem_bytes,
              uint64_t cols, uint64_t rows, uint32_t box_cols, uint32_t box_rows,
              CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (!fn || !base || rows == 0) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct PlanData {
  GemmParams gate_up{};
  GemmParams down{};
  GemmParams router{};
  int sms = 148;
};

// How the dequantisers get scales: 0 = the shared-memory table loaded by warp 3
// (groups a multiple of 8 in [8, kMaxScaleGroups], 16-byte aligned tensors), else
// the widest per-thread vector (8 or 4 groups) every scale/bias row allows, or 1.
int vec_for(int groups, std::initializer_list<const void*> ptrs) {
  bool table = groups % 8 == 0 && groups >= 8 && groups <= kMaxScaleGroups;
  for (const void* ptr : ptrs)
    if (ptr && (reinterpret_cast<uintptr_t>(ptr) & 15)) table = false;
  if (table) return 0;
  for (int v : {8, 4}) {
    if (groups % v) continue;
    bool ok = true;
    for (const void* ptr : ptrs)
      if (ptr && (reinterpret_cast<uintptr_t>(ptr) & (uintptr_t)(2 * v - 1))) ok = false;
    if (ok) return v;
  }
  return 1;
}

int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

template <int MODE, int VEC, int FB = 1>
cudaError_t launch_vec(const GemmParams& p, int max_units, cudaStream_t st) {
  const int threads = MODE == kRouter ? kThreadsR : kThreadsQ;
  // the scale-table mode adds its buffers (sized for the largest table)
  constexpr int kSmem =
      smem_bytes<MODE, FB>() +
      (VEC == 0 ? kScaleBufs * FB * scale_buf_bytes(FB == 2 ? kMaxScaleGroupsFB2 : kMaxScaleGroups)
                : 0);
  static_assert(kSmem + sizeof(SmemCtl) <= 227 * 1024, "shared memory budget");
  const int smem = VEC == 0 ? smem_bytes<MODE, FB>() +
                                  kScaleBufs * FB * scale_buf_bytes(p.groups_per_row)
                            : kSmem;
  max_units = (max_units + FB - 1) / FB;
  static uint64_t configured = 0;  // per-device bit
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured & bit)) {
    cudaError_t e = cudaFuncSetAttribute(moe_gemm_kernel<MODE, VEC, FB>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return e;
    configured |= bit;
  }
  int grid = sm_count();
  if (max_units < grid) grid = max_units;
  if (grid <= 0) return cudaSuccess;
  moe_gemm_kernel<MODE, VEC, FB><<<grid, threads, smem, st>>>(p);
  return cudaGetLastError();
}

// pair: gate/up units may cover two weight-row blocks (FB = 2)
template <int MODE>
cudaError_t launch(const GemmParams& p, int max_units, cudaStream_t st, bool pair = false) {
  if constexpr (MODE == kRouter) {
    return launch_vec<MODE, 1>(p, max_units, st);
  } else {
    if (p.scale_vec == 0) {
      if constexpr (MODE == kGateUp)
        if (pair && p.groups_per_row <= kMaxScaleGroupsFB2 && p.fb_count % 2 == 0)
          return launch_vec<MODE, 0, 2>(p, max_units, st);
      return launch_vec<MODE, 0>(p, max_units, st);
    }
    if (p.scale_vec == 8) return launch_vec<MODE, 8>(p, max_units, st);
    if (p.scale_vec == 4) return launch_vec<MODE, 4>(p, max_units, st);
    return launch_vec<MODE, 1>(p, max_units, st);
  }
}

}  // namespace

int moe_gemm_plan(const astro_moe_layer_weights& w, MoeGemmPlan* plan, int router_rows,
                  const PagedStacks* paged) {
  plan->ok = false;
  plan->w = w;
  if (plan->dev) {
    delete reinterpret_cast<PlanData*>(plan->dev);
    plan->dev = nullptr;
  }
  const int H = w.hidden, E = w.experts, I = w.intermediate, Is = w.shared_intermediate;
  // eligible profile: 4-bit, group 64, shapes that tile exactly
  if (w.bits != 4 || w.group_size != 64) return 0;
  // (an even number of 64-wide K blocks on both projections: operand slots
  // complete in pairs)
  if (H % 128 != 0 || I % 128 != 0 || (Is != 0 && Is != I)) return 0;
  if (E > 1024 || !encode_fn()) return 0;
  auto* d = new PlanData();
  d->sms = sm_count();
  const CUtensorMapDataType U32 = CU_TENSOR_MAP_DATA_TYPE_UINT32;
  const uint64_t wh = (uint64_t)H / 8, wi = (uint64_t)I / 8;
  bool ok = true;
  // paged experts: per projection, a map over the pool from the tensor's offset
  // in the first page to the pool's end, rows of `pitch` bytes; a slot is
  // page_bytes / pitch rows further on
  const int64_t rq_h = (int64_t)H / 2, rq_i = (int64_t)I / 2;            // code row bytes
  const int64_t rs_h = (int64_t)(H / 64) * 2, rs_i = (int64_t)(I / 64) * 2;  // scale row bytes
  auto pool_map = [&](CUtensorMap* m, int proj, int64_t pitch, uint32_t box_rows) {
    const int64_t total = paged->slots * paged->page_bytes;
    return make_map(m, paged->pool + paged->off_q[proj], U32, 4, (uint64_t)(pitch / 4),
                    (uint64_t)((total - paged->off_q[proj]) / pitch), 8, box_rows,
                    CU_TENSOR_MAP_SWIZZLE_NONE);
  };
  auto pool_ptr = [&](const int64_t* off, int proj) {
    return reinterpret_cast<const uint16_t*>(paged->pool + off[proj]);
  };
  // gate/up
  GemmParams& g = d->gate_up;
  const int64_t gate_rows = w.gate_up_fused ? 2LL * I : (int64_t)I;
  if (paged) {
    ok &= pool_map(&g.tm_a[0][0], 0, rq_h, 64);
    ok &= pool_map(&g.tm_a[0][1], 1, rq_h, 64);
    g.a_row_base[0][0] = g.a_row_base[0][1] = 0;
    g.scales[0][0] = pool_ptr(paged->off_s, 0);
    g.biases[0][0] = pool_ptr(paged->off_b, 0);
    g.scales[0][1] = pool_ptr(paged->off_s, 1);
    g.biases[0][1] = pool_ptr(paged->off_b, 1);
    g.a_expert_rows[0] = paged->page_bytes / rq_h;
    g.a_sb_expert_rows[0] = paged->page_bytes / rs_h;
  } else {
  ok &= make_map(&g.tm_a[0][0], w.gate.packed, U32, 4, wh, (uint64_t)E * gate_rows, 8, 64,
                 CU_TENSOR_MAP_SWIZZLE_NONE);
  if (w.gate_up_fused) {
    g.tm_a[0][1] = g.tm_a[0][0];
    g.a_row_base[0][0] = 0;
    g.a_row_base[0][1] = I;
    g.scales[0][1] = (const uint16_t*)w.gate.scales;
    g.biases[0][1] = (const uint16_t*)w.gate.biases;
  } else {
    ok &= make_map(&g.tm_a[0][1], w.up.packed, U32, 4, wh, (uint64_t)E * I, 8, 64,
                   CU_TENSOR_MAP_SWIZZLE_NONE);
    g.a_row_base[0][0] = g.a_row_base[0][1] = 0;
    g.scales[0][1] = (const uint16_t*)w.up.scales;
    g.biases[0][1] = (const uint16_t*)w.up.biases;
  }
  g.scales[0][0] = (const uint16_t*)w.gate.scales;
  g.biases[0][0] = (const uint16_t*)w.gate.biases;
  g.a_expert_rows[0] = gate_rows;
  g.a_sb_expert_rows[0] = gate_rows;
  }  // stacked experts
  if (Is > 0) {
    ok &= make_map(&g.tm_a[1][0], w.shared_gate.packed, U32, 4, wh, (uint64_t)Is, 8, 64,
                   CU_TENSOR_MAP_SWIZZLE_NONE);
    ok &= make_map(&g.tm_a[1][1], w.shared_up.packed, U32, 4, wh, (uint64_t)Is, 8, 64,
                   CU_TENSOR_MAP_SWIZZLE_NONE);
    g.scales[1][0] = (const uint16_t*)w.shared_gate.scales;
    g.biases[1][0] = (const uint16_t*)w.shared_gate.biases;
    g.scales[1][1] = (const uint16_t*)w.shared_up.scales;
    g.biases[1][1] = (const uint16_t*)w.shared_up.biases;
    g.a_expert_rows[1] = g.a_sb_expert_rows[1] = Is;
  }
  g.groups_per_row = H / 64;
  g.scale_vec = vec_for(H / 64, {g.scales[0][0], g.biases[0][0], g.scales[0][1], g.biases[0][1],
                                 w.shared_gate.scales, w.shared_gate.biases, w.shared_up.scales,
                                 w.shared_up.biases});
  g.kblocks = H / 64;
  g.fb_count = I / 64;
  g.tile_rows = kMaxN;
  g.out_cols = I;
  g.ldo = I;
  // down
  GemmParams& dn = d->down;
  if (paged) {
    ok &= pool_map(&dn.tm_a[0][0], 2, rq_i, 128);
    dn.scales[0][0] = pool_ptr(paged->off_s, 2);
    dn.biases[0][0] = pool_ptr(paged->off_b, 2);
    dn.a_expert_rows[0] = paged->page_bytes / rq_i;
    dn.a_sb_expert_rows[0] = paged->page_bytes / rs_i;
  } else {
    ok &= make_map(&dn.tm_a[0][0], w.down.packed, U32, 4, wi, (uint64_t)E * H, 8, 128,
                   CU_TENSOR_MAP_SWIZZLE_NONE);
    dn.scales[0][0] = (const uint16_t*)w.down.scales;
    dn.biases[0][0] = (const uint16_t*)w.down.biases;
    dn.a_expert_rows[0] = dn.a_sb_expert_rows[0] = H;
  }
  if (Is > 0) {
    ok &= make_map(&dn.tm_a[1][0], w.shared_down.packed, U32, 4, wi, (uint64_t)H, 8, 128,
                   CU_TENSOR_MAP_SWIZZLE_NONE);
    dn.scales[1][0] = (const uint16_t*)w.shared_down.scales;
    dn.biases[1][0] = (const uint16_t*)w.shared_down.biases;
    dn.a_expert_rows[1] = dn.a_sb_expert_rows[1] = H;
  }
  dn.groups_per_row = I / 64;
  dn.scale_vec = vec_for(I / 64, {dn.scales[0][0], dn.biases[0][0], w.shared_down.scales,
                                  w.shared_down.biases});
  dn.kblocks = I / 64;
  dn.fb_count = H / 128;
  dn.tile_rows = kMaxN;
  dn.out_cols = H;
  dn.ldo = H;
  // router (dense bf16 A by TMA); its row count may exceed the stacked experts'
  // (expert parallelism: all experts are routed, only the local ones are stacked)
  GemmParams& rt = d->router;
  const int R = router_rows > 0 ? router_rows : E;
  ok &= make_map(&rt.tm_a[0][0], w.router_weight, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                 (uint64_t)H, (uint64_t)R, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  rt.kblocks = H / 64;
  rt.fb_count = (R + 127) / 128;
  rt.tile_rows = 64;
  rt.out_cols = R;
  rt.ldo = R;
  rt.shared_seg = -1;
  rt.nseg = 1;
  rt.seg_offsets = nullptr;
  if (!ok) {
    delete d;
    return 0;  // not eligible: the CUDA-core path serves this layer
  }
  plan->dev = d;
  plan->ok = true;
  return 0;
}

void moe_gemm_release(MoeGemmPlan& plan) {
  if (plan.dev) delete reinterpret_cast<PlanData*>(plan.dev);
  plan.dev = nullptr;
  plan.ok = false;
}

// use_tensor_cores option: >= 0 (auto/on) selects the tcgen05 path for eligible
// layers; < 0 forces the CUDA-core kernels.
bool moe_gemm_enabled(const MoeGemmPlan& plan, int opt) { return plan.ok && opt >= 0; }

size_t moe_gemm_scratch_bytes() { return 256; }

static bool bind_b(GemmParams& p, const void* rows_ptr, int64_t rows, int K) {
  bool ok = true;
  for (int b = 0; b < kBoxKinds; ++b)
    ok &= make_map(&p.tm_b[b], rows_ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)K,
                   (uint64_t)rows, 64, (uint32_t)(128 >> b), CU_TENSOR_MAP_SWIZZLE_128B);
  return ok;
}

cudaError_t moe_gemm_router(const MoeGemmPlan& plan, const void* x, int64_t tokens, void* logits,
                            void* scratch, uint32_t* status, cudaStream_t st) {
  (void)scratch;
  auto* d = reinterpret_cast<PlanData*>(plan.dev);
  if (!d) return cudaErrorNotSupported;
  GemmParams p = d->router;
  if (!bind_b(p, x, tokens, plan.w.hidden)) return cudaErrorInvalidValue;
  p.total_rows = (int)tokens;
  p.out = (uint16_t*)logits;
  p.out_rows = (int)tokens;
  p.status = status;
  const int units = (int)((tokens + 63) / 64) * p.fb_count;
  return launch<kRouter>(p, units, st);
}

cudaError_t moe_gemm_gate_up(const MoeGemmPlan& plan, const void* states, int64_t rows,
                             const uint32_t* offsets, void* act, void* scratch, uint32_t* status,
                             cudaStream_t st, const uint32_t* slot_of) {
  (void)scratch;
  auto* d = reinterpret_cast<PlanData*>(plan.dev);
  if (!d) return cudaErrorNotSupported;
  GemmParams p = d->gate_up;
  if (!bind_b(p, states, rows, plan.w.hidden)) return cudaErrorInvalidValue;
  const bool shared = plan.w.shared_intermediate > 0;
  p.seg_offsets = offsets;
  p.nseg = plan.w.experts + (shared ? 1 : 0);
  p.shared_seg = shared ? plan.w.experts : -1;
  p.total_rows = (int)rows;
  p.out = (uint16_t*)act;
  p.out_rows = (int)rows;
  p.status = status;
  p.slot_of = slot_of;
  const int max_units = (int)((rows + kMaxN - 1) / kMaxN + p.nseg) * p.fb_count;
  // Two weight-row blocks per unit pay off for full token tiles (prefill: gate/up
  // 229 us against 235 us at T = 4096 on B200); with a few rows per segment
  // (decode) the epilogue no longer overlaps the next unit and the grid has half
  // the units (115 us against 107 us per layer at T = 64), so the pairing starts
  // at 64 rows per segment on average.
  const bool pair = rows >= 64 * (int64_t)p.nseg;
  return launch<kGateUp>(p, max_units, st, pair);
}

cudaError_t moe_gemm_down(const MoeGemmPlan& plan, const void* act, int64_t rows,
                          const uint32_t* offsets, void* yrows, void* scratch, uint32_t* status,
                          cudaStream_t st, const uint32_t* slot_of) {
  (void)scratch;
  auto* d = reinterpret_cast<PlanData*>(plan.dev);
  if (!d) return cudaErrorNotSupported;
  GemmParams p = d->down;
  if (!bind_b(p, act, rows, plan.w.intermediate)) return cudaErrorInvalidValue;
  const bool shared = plan.w.shared_intermediate > 0;
  p.seg_offsets = offsets;
  p.nseg = plan.w.experts + (shared ? 1 : 0);
  p.shared_seg = shared ? plan.w.experts : -1;
  p.total_rows = (int)rows;
  p.out = (uint16_t*)yrows;
  p.out_rows = (int)rows;
  p.status = status;
  p.slot_of = slot_of;
  const int max_units = (int)((rows + kMaxN - 1) / kMaxN + p.nseg) * p.fb_count;
  return launch<kDown>(p, max_units, st);
}

}  // namespace astro
