// decode.cu -- the small-batch (decode) kernels of the MoE block: a router GEMV
// and the gathered int4 gate/up (+SwiGLU) and down GEMVs over the active experts.
//
// At decode batch sizes (config 2: T in {1, 4, 16, 64}) each routed expert sees a
// handful of token rows, so the block is bound by streaming the selected experts'
// weights from HBM (1,769,472 B per expert) and by fixed per-launch latency, not
// by MMA throughput.  These kernels therefore:
//   * stream each weight row exactly once with 128-bit coalesced loads that skip
//     L1 (a warp reads 512 contiguous bytes per instruction);
//   * dequantise in registers (MLX affine int4, group 64: w = bf16(s*q + b), the
//     same rounded weight the oracle and the tensor-core path use) and
//     accumulate in fp32, reducing across lanes with warp shuffles;
//   * visit only non-empty expert segments: every block compacts the expert
//     offsets into a list of active segments in shared memory, so the grid can be
//     sized for the worst case without launching a block per idle expert;
//   * read token rows through the sorted-token indirection (no row gather).
// Semantics are gather_qmm's (mlx_quantized_operations.rs:100-157) and the
// router projection's (qwen3_5_moe/model/forward.rs:52-93); the accumulation
// order is defined here (lane-strided partial sums, butterfly reduction), so
// outputs match the oracle to the block tolerance, not bit for bit.
#include "combine_dev.cuh"
#include "common.cuh"
#include "kernels.h"
#include "route_dev.cuh"

namespace astro {
namespace {

constexpr int kThreads = 256;      // router blocks
constexpr int kWarps = kThreads / 32;
constexpr int kGemvThreads = 512;  // GEMV blocks: one per SM, 16 warps
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kMaxSegs = 1025;  // 1024 routed experts + the shared expert
constexpr int kRouterTokens = 8;  // tokens per router block

// Weights are read once: bypass L1.
ASTRO_DEVINL uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
ASTRO_DEVINL uint4 ld_cached(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

ASTRO_DEVINL float lo_f(uint32_t v) { return __uint_as_float(v << 16); }
ASTRO_DEVINL float hi_f(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// 8 bf16 in a uint4 -> fp32
ASTRO_DEVINL void bf16x8_to_f32(const uint4& v, float (&f)[8]) {
  f[0] = lo_f(v.x); f[1] = hi_f(v.x); f[2] = lo_f(v.y); f[3] = hi_f(v.y);
  f[4] = lo_f(v.z); f[5] = hi_f(v.z); f[6] = lo_f(v.w); f[7] = hi_f(v.w);
}

// One packed word (8 nibbles, element i at bits 4i) -> 4 bf16x2 pairs
// (element i, element i + 4) of w = bf16(s * q + b).
ASTRO_DEVINL void dequant_word(uint32_t v, __nv_bfloat162 s2, __nv_bfloat162 b2,
                               uint32_t (&out)[4]) {
  const __nv_bfloat162 k128 = __floats2bfloat162_rn(128.0f, 128.0f);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t t = ((v >> (4 * i)) & 0x000f000fu) | 0x43004300u;  // bf16 (128 + q)
    __nv_bfloat162 q = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&t), k128);
    __nv_bfloat162 w = __hfma2(q, s2, b2);
    out[i] = *reinterpret_cast<uint32_t*>(&w);
  }
}

// 32 consecutive elements (a uint4 of packed words) -> 16 bf16x2 pairs; pair
// 4c + i holds elements (8c + i, 8c + i + 4).
ASTRO_DEVINL void dequant32(const uint4& q, uint16_t s, uint16_t b, uint32_t (&w)[16]) {
  const __nv_bfloat162 s2 = __halves2bfloat162(__ushort_as_bfloat16(s), __ushort_as_bfloat16(s));
  const __nv_bfloat162 b2 = __halves2bfloat162(__ushort_as_bfloat16(b), __ushort_as_bfloat16(b));
  uint32_t t[4];
  dequant_word(q.x, s2, b2, t);
  w[0] = t[0]; w[1] = t[1]; w[2] = t[2]; w[3] = t[3];
  dequant_word(q.y, s2, b2, t);
  w[4] = t[0]; w[5] = t[1]; w[6] = t[2]; w[7] = t[3];
  dequant_word(q.z, s2, b2, t);
  w[8] = t[0]; w[9] = t[1]; w[10] = t[2]; w[11] = t[3];
  dequant_word(q.w, s2, b2, t);
  w[12] = t[0]; w[13] = t[1]; w[14] = t[2]; w[15] = t[3];
}

// acc += sum over the 8 elements of chunk c of w * x
ASTRO_DEVINL float dot8(const uint32_t (&w)[16], int c, const float (&x)[8], float acc) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t p = w[4 * c + i];
    acc = __fmaf_rn(lo_f(p), x[i], acc);
    acc = __fmaf_rn(hi_f(p), x[i + 4], acc);
  }
  return acc;
}

ASTRO_DEVINL float warp_sum(float v) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}
ASTRO_DEVINL float half_warp_sum(float v) {
#pragma unroll
  for (int m = 8; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}

// Compacts the non-empty segments of offsets[0..nseg] (ascending) into `list`,
// leaving out routed segments whose slot is kSlotElsewhere and, with
// skip_shared, the shared segment; returns their count.  Called by every thread
// of the block.
template <int NT>
ASTRO_DEVINL int active_segments(const uint32_t* __restrict__ offsets, int nseg, uint16_t* list,
                                 int* warp_cnt, const uint32_t* slot_of, int shared_seg,
                                 bool skip_shared) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int base = 0;
  for (int s0 = 0; s0 < nseg; s0 += NT) {
    const int s = s0 + threadIdx.x;
    bool ne = s < nseg && offsets[s + 1] > offsets[s];
    if (ne) ne = s == shared_seg ? !skip_shared : !(slot_of && slot_of[s] == kSlotElsewhere);
    const uint32_t bal = __ballot_sync(0xffffffffu, ne);
    if (lane == 0) warp_cnt[w] = __popc(bal);
    __syncthreads();
    int before = 0, total = 0;
#pragma unroll
    for (int i = 0; i < NT / 32; ++i) {
      const int c = warp_cnt[i];
      before += i < w ? c : 0;
      total += c;
    }
    if (ne) list[base + before + __popc(bal & lanemask_lt())] = (uint16_t)s;
    base += total;
    __syncthreads();
  }
  return base;
}

// ---------------------------------------------------------------------------
// router: logits[t, e] = bf16(x_t . Wr[e]); block = 8 experts x 8 tokens, the
// tokens' rows staged in shared memory, one warp per expert row.
template <int J>  // H = 256 * J
__global__ void __launch_bounds__(kThreads) router_gemv_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t T, const __nv_bfloat16* __restrict__ wr, int E,
    __nv_bfloat16* __restrict__ logits) {
  constexpr int H = 256 * J;
  constexpr int kRowVec = H / 8;  // uint4 per row
  extern __shared__ uint4 xs[];   // [kRouterTokens][kRowVec]
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t t0 = (int64_t)blockIdx.y * kRouterTokens;
  const int nt = (int)(T - t0 < kRouterTokens ? T - t0 : kRouterTokens);
  const uint4* xsrc = reinterpret_cast<const uint4*>(x + t0 * H);
  for (int i = threadIdx.x; i < nt * kRowVec; i += kThreads) xs[i] = ld_cached(xsrc + i);
  __syncthreads();
  const int e = blockIdx.x * kWarps + w;
  if (e >= E) return;
  // eight K slices of H / 8: a slice's lane products are summed per lane, then
  // across the warp, and the slice sums are added in order -- the fused decode
  // kernel's order, so both paths give the same logits
  constexpr int kSliceVecs = kRowVec / 8, kPerLane = (kSliceVecs + 31) / 32;
  uint4 wv[8][kPerLane];
  const uint4* wrow = reinterpret_cast<const uint4*>(wr + (int64_t)e * H);
#pragma unroll
  for (int s = 0; s < 8; ++s)
#pragma unroll
    for (int k = 0; k < kPerLane; ++k)
      wv[s][k] = (k * 32 + lane < kSliceVecs) ? ld_stream(wrow + s * kSliceVecs + k * 32 + lane)
                                              : make_uint4(0u, 0u, 0u, 0u);
  float acc[kRouterTokens];
#pragma unroll
  for (int t = 0; t < kRouterTokens; ++t) acc[t] = 0.0f;
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    float part[kRouterTokens];
#pragma unroll
    for (int t = 0; t < kRouterTokens; ++t) part[t] = 0.0f;
#pragma unroll
    for (int k = 0; k < kPerLane; ++k) {
      if (k * 32 + lane < kSliceVecs) {
        float wf[8];
        bf16x8_to_f32(wv[s][k], wf);
#pragma unroll
        for (int t = 0; t < kRouterTokens; ++t) {
          if (t < nt) {
            float xf[8];
            bf16x8_to_f32(xs[t * kRowVec + s * kSliceVecs + k * 32 + lane], xf);
#pragma unroll
            for (int i = 0; i < 8; ++i) part[t] = __fmaf_rn(wf[i], xf[i], part[t]);
          }
        }
      }
    }
#pragma unroll
    for (int t = 0; t < kRouterTokens; ++t)
      if (t < nt) acc[t] = __fadd_rn(acc[t], warp_sum(part[t]));
  }
#pragma unroll
  for (int t = 0; t < kRouterTokens; ++t)
    if (t < nt && lane == 0) logits[(t0 + t) * E + e] = __float2bfloat16_rn(acc[t]);
}

// ---------------------------------------------------------------------------
// Token rows of the current segment are staged in shared memory, kRowChunk rows
// per pass.  Lane l reads 16-byte chunks 4l..4l+3 of a 1024-element (or
// 512-element) step, so 8 lanes of one access phase would hit two bank groups;
// storing chunk q at q ^ ((q >> 3) & 7) spreads them over all eight.
constexpr int kRowChunk = 8;
constexpr int kRowChunkGU = 4;  // gate/up: fewer accumulators, no register spills

ASTRO_DEVINL int swz(int q) { return q ^ ((q >> 3) & 7); }

// Cooperative copy of rows p .. p+n-1 (row index through `rows` when given) of
// a bf16 matrix with `vecs` uint4 per row into xs[n][vecs] (swizzled).  Rows
// outside [0, limit) record kDevBadShape and are read as row 0.
ASTRO_DEVINL void stage_rows(uint4* xs, const uint4* __restrict__ src, const uint32_t* rows,
                             uint32_t p, int n, int vecs, int64_t limit, uint32_t* status) {
  for (int i = threadIdx.x; i < n * vecs; i += kGemvThreads) {
    const int j = i / vecs, q = i - j * vecs;
    int64_t r = rows ? (int64_t)rows[p + j] : (int64_t)(p + j);
    if (r >= limit) {
      record_status(status, kDevBadShape);
      r = 0;
    }
    xs[j * vecs + swz(q)] = ld_cached(src + r * vecs + q);
  }
}

// Packed codes and scales of one lane's share of a weight row: STEPS 16-byte
// code vectors and, per step, (scale | bias << 16).
template <int STEPS> struct RowRegs {
  uint4 q[STEPS];
  uint32_t sb[STEPS];
};

// rows of expert e, row f of a stacked tensor: packed codes and scales/biases
ASTRO_DEVINL int64_t q_row(const AffineRef& W, int64_t e, int64_t f) {
  return e * W.expert_rows + W.row_offset + f;
}
ASTRO_DEVINL int64_t sb_row(const AffineRef& W, int64_t e, int64_t f) {
  return e * (W.sb_expert_rows ? W.sb_expert_rows : W.expert_rows) + W.row_offset + f;
}

// Issues the loads of row f of expert e (one lane's share; nothing waits on
// them until use).
template <int STEPS>
ASTRO_DEVINL void load_row(RowRegs<STEPS>& r, const AffineRef& W, int64_t e, int64_t f, int words,
                           int groups, int qoff, int goff, int qstride, int gstride) {
  const uint32_t* q = reinterpret_cast<const uint32_t*>(W.q) + q_row(W, e, f) * words + qoff;
  const uint16_t* ps = reinterpret_cast<const uint16_t*>(W.s) + sb_row(W, e, f) * groups + goff;
  const uint16_t* pb = reinterpret_cast<const uint16_t*>(W.b) + sb_row(W, e, f) * groups + goff;
#pragma unroll
  for (int s = 0; s < STEPS; ++s) r.q[s] = ld_stream(q + s * qstride);
#pragma unroll
  for (int s = 0; s < STEPS; ++s)
    r.sb[s] = (uint32_t)__ldg(ps + s * gstride) | ((uint32_t)__ldg(pb + s * gstride) << 16);
}

// gate/up + SwiGLU.  Item = (active segment, 16 consecutive features); warp w
// owns feature f = base + w: its gate row and up row.  Lane l holds elements
// [1024 s + 32 l, +32) of a row, inside quantisation group 16 s + l / 2.  The
// next item's codes are loaded while the current one is computed.
template <int STEPS>  // in_features = 1024 * STEPS
__global__ void __launch_bounds__(kGemvThreads, 1) decode_gate_up_kernel(GroupedGemvDesc d) {
  extern __shared__ uint4 xs[];  // [kRowChunkGU][H / 8]
  __shared__ uint16_t list[kMaxSegs];
  __shared__ int warp_cnt[kGemvWarps];
  const int n_act = active_segments<kGemvThreads>(d.seg_offsets, d.nseg, list, warp_cnt, d.slot_of,
                                                  d.shared_seg, d.skip_shared);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  constexpr int H = 1024 * STEPS;
  constexpr int kVecs = H / 8, kWords = H / 8, kGroups = H / 64;
  const int per_seg = d.out_features / kGemvWarps;
  const int64_t items = (int64_t)n_act * per_seg;
  const uint4* xsrc = reinterpret_cast<const uint4*>(d.x);
  __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(d.y);
  auto load_item = [&](int64_t it, RowRegs<STEPS>& ga, RowRegs<STEPS>& ua) {
    const int seg = list[it / per_seg];
    const int f = (int)(it % per_seg) * kGemvWarps + w;
    const int sh = seg == d.shared_seg ? 1 : 0;
    // select by value (a dynamic index into the parameter block would copy it to local memory)
    const AffineRef A = sh ? d.wa[1] : d.wa[0];
    const AffineRef B = sh ? d.wb[1] : d.wb[0];
    const int64_t e = sh ? 0 : (d.slot_of ? (int64_t)d.slot_of[seg] : seg);
    load_row<STEPS>(ga, A, e, f, kWords, kGroups, lane * 4, lane / 2, 128, 16);
    load_row<STEPS>(ua, B, e, f, kWords, kGroups, lane * 4, lane / 2, 128, 16);
  };
  RowRegs<STEPS> ga, ua, gn, un;
  int64_t it = blockIdx.x;
  if (it < items) load_item(it, ga, ua);
  for (; it < items; it += gridDim.x) {
    if (it + gridDim.x < items) load_item(it + gridDim.x, gn, un);
    const int seg = list[it / per_seg];
    const int f = (int)(it % per_seg) * kGemvWarps + w;
    uint32_t p0 = d.seg_offsets[seg], p1 = d.seg_offsets[seg + 1];
    if (p1 > (uint64_t)d.rows_total) p1 = (uint32_t)d.rows_total;
    for (uint32_t p = p0; p < p1; p += kRowChunkGU) {
      const int n = (int)(p1 - p < (uint32_t)kRowChunkGU ? p1 - p : (uint32_t)kRowChunkGU);
      __syncthreads();  // the previous pass is done with xs
      stage_rows(xs, xsrc, d.x_rows, p, n, kVecs, d.x_limit, d.status);
      __syncthreads();
      float g[kRowChunkGU], u[kRowChunkGU];
#pragma unroll
      for (int j = 0; j < kRowChunkGU; ++j) g[j] = u[j] = 0.f;
#pragma unroll
      for (int s = 0; s < STEPS; ++s) {
        uint32_t wg[16], wu[16];
        dequant32(ga.q[s], (uint16_t)ga.sb[s], (uint16_t)(ga.sb[s] >> 16), wg);
        dequant32(ua.q[s], (uint16_t)ua.sb[s], (uint16_t)(ua.sb[s] >> 16), wu);
#pragma unroll
        for (int j = 0; j < kRowChunkGU; ++j) {
          if (j < n) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              float xf[8];
              bf16x8_to_f32(xs[j * kVecs + swz(s * 128 + lane * 4 + c)], xf);
              g[j] = dot8(wg, c, xf, g[j]);
              u[j] = dot8(wu, c, xf, u[j]);
            }
          }
        }
      }
#pragma unroll
      for (int j = 0; j < kRowChunkGU; ++j) {
        if (j < n) {
          const float gs = warp_sum(g[j]), us = warp_sum(u[j]);
          if (lane == 0 && p + j < (uint64_t)d.y_limit)
            y[(int64_t)(p + j) * d.ldy + f] =
                __float2bfloat16_rn(swiglu_bf16(round_bf16(gs), round_bf16(us)));
        }
      }
    }
    ga = gn;
    ua = un;
  }
}

// ---------------------------------------------------------------------------
// down projection.  Item = (active segment, 64 output rows); warp w owns rows
// base + 4w .. base + 4w + 3, half-warp h rows 4w + 2h and 4w + 2h + 1.  Lane l
// of a half holds elements [512 s + 32 l, +32) of a row (group 8 s + l / 2).
// Activation rows are read by sorted position; the next item's codes are
// loaded while the current one is computed.
template <int STEPS>  // in_features = 512 * STEPS
__global__ void __launch_bounds__(kGemvThreads, 1) decode_down_kernel(GroupedGemvDesc d) {
  extern __shared__ uint4 xs[];  // [kRowChunk][K / 8]
  __shared__ uint16_t list[kMaxSegs];
  __shared__ int warp_cnt[kGemvWarps];
  const int n_act = active_segments<kGemvThreads>(d.seg_offsets, d.nseg, list, warp_cnt, d.slot_of,
                                                  d.shared_seg, d.skip_shared);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int half = lane >> 4, li = lane & 15;
  constexpr int K = 512 * STEPS;
  constexpr int kVecs = K / 8, kWords = K / 8, kGroups = K / 64;
  constexpr int kRowsPerHalf = 2;
  constexpr int kRowsPerItem = 2 * kRowsPerHalf * kGemvWarps;  // 64
  const int per_seg = d.out_features / kRowsPerItem;
  const int64_t items = (int64_t)n_act * per_seg;
  const uint4* xsrc = reinterpret_cast<const uint4*>(d.x);
  __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(d.y);
  auto first_row = [&](int64_t it) {
    return (int)(it % per_seg) * kRowsPerItem + w * 2 * kRowsPerHalf + half * kRowsPerHalf;
  };
  auto load_item = [&](int64_t it, RowRegs<STEPS> (&rr)[kRowsPerHalf]) {
    const int seg = list[it / per_seg];
    const int sh = seg == d.shared_seg ? 1 : 0;
    const AffineRef A = sh ? d.wa[1] : d.wa[0];
    const int64_t e = sh ? 0 : (d.slot_of ? (int64_t)d.slot_of[seg] : seg);
#pragma unroll
    for (int r = 0; r < kRowsPerHalf; ++r)
      load_row<STEPS>(rr[r], A, e, first_row(it) + r, kWords, kGroups, li * 4, li / 2, 64, 8);
  };
  RowRegs<STEPS> cur[kRowsPerHalf], nxt[kRowsPerHalf];
  int64_t it = blockIdx.x;
  if (it < items) load_item(it, cur);
  for (; it < items; it += gridDim.x) {
    if (it + gridDim.x < items) load_item(it + gridDim.x, nxt);
    const int seg = list[it / per_seg];
    const int r0 = first_row(it);
    uint32_t p0 = d.seg_offsets[seg], p1 = d.seg_offsets[seg + 1];
    if (p1 > (uint64_t)d.rows_total) p1 = (uint32_t)d.rows_total;
    for (uint32_t p = p0; p < p1; p += kRowChunk) {
      const int n = (int)(p1 - p < (uint32_t)kRowChunk ? p1 - p : (uint32_t)kRowChunk);
      __syncthreads();
      stage_rows(xs, xsrc, nullptr, p, n, kVecs, d.x_limit, d.status);
      __syncthreads();
#pragma unroll
      for (int r = 0; r < kRowsPerHalf; ++r) {
        float a[kRowChunk];
#pragma unroll
        for (int j = 0; j < kRowChunk; ++j) a[j] = 0.f;
#pragma unroll
        for (int s = 0; s < STEPS; ++s) {
          uint32_t wd[16];
          dequant32(cur[r].q[s], (uint16_t)cur[r].sb[s], (uint16_t)(cur[r].sb[s] >> 16), wd);
#pragma unroll
          for (int j = 0; j < kRowChunk; ++j) {
            if (j < n) {
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                float xf[8];
                bf16x8_to_f32(xs[j * kVecs + swz(s * 64 + li * 4 + c)], xf);
                a[j] = dot8(wd, c, xf, a[j]);
              }
            }
          }
        }
#pragma unroll
        for (int j = 0; j < kRowChunk; ++j) {
          if (j < n) {
            const float v = half_warp_sum(a[j]);
            if (li == 0 && p + j < (uint64_t)d.y_limit)
              y[(int64_t)(p + j) * d.ldy + r0 + r] = __float2bfloat16_rn(v);
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kRowsPerHalf; ++r) cur[r] = nxt[r];
  }
}

int grid_for(int64_t items_upper) {
  const int64_t cap = 148;  // one 16-warp block per SM
  return (int)(items_upper < 1 ? 1 : (items_upper < cap ? items_upper : cap));
}

// ===========================================================================
// Fused decode block: the whole MoE block for T <= kFusedMaxTokens tokens in one
// cooperative launch (one 16-warp block per SM).  Phases:
//   1. router logits and the shared-expert gate logit (x staged in shared
//      memory up to 16 tokens); one thread per block issues bulk L2 prefetches
//      of the shared expert's weights;
//   -- grid barrier --
//   2. every block routes all T tokens and sorts the T*K assignments in its own
//      shared memory (identical inputs give identical results in every block, so
//      no barrier follows); block 0 publishes ids, scores and offsets;
//   3. gate/up + SwiGLU over (active segment, 32 features) items -> act rows;
//      each finished item adds one to its segment's completion counter;
//   4. down over (active segment, 64 output rows) items -> expert rows; a
//      block starts a segment's down items once all of that segment's gate/up
//      items are counted (no grid barrier: early blocks go on while late ones
//      finish gate/up);
//      phases 3 and 4 run on warp tensor-core tiles (mma.sync m16n8k16, bf16
//      operands, fp32 accumulation): a pass covers at most 16 token rows, so
//      each warp keeps one 16-row weight tile in registers, with no shared-memory
//      or tensor-memory hand-off of the A operand, and the CUDA cores only
//      dequantise; each block takes a contiguous share of the items;
//   -- grid barrier --
//   5. weighted combine with the gated shared expert -> out.
// Launch gaps and the per-kernel dependency chains of the multi-kernel path
// disappear.  Routing, sort order, dequantised weights and the combine are the
// multi-kernel path's; the projections add the same fp32 products in another
// order (tensor-core tiles, four K quarters summed in a fixed order), so the two
// paths agree to the block tolerance and routing is bit-identical.
constexpr int kFusedMaxTokens = 64;
constexpr int kStageTokens = 16;  // token rows staged (pair-interleaved) at a time
constexpr int kFusedMaxExperts = 256;
constexpr int kFusedMaxAssign = 512;
static_assert(kFusedMaxExperts <= kGemvThreads, "one thread per expert in the count scan");

// Items of the active segments, m per segment, each costing its segment's
// 16-row passes P (cum[i] = passes of the segments before list entry i,
// cum[na] = all): the first item whose cost starts at or after `target`.
ASTRO_DEVINL int item_at_cost(const int* cum, const uint16_t* list, const uint32_t* offs, int na,
                              int m, int64_t target) {
  int lo = 0, hi = na - 1;  // largest i with m * cum[i] <= target
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if ((int64_t)m * cum[mid] <= target) lo = mid;
    else hi = mid - 1;
  }
  const int seg = list[lo];
  const int64_t P = (offs[seg + 1] - offs[seg] + 15) / 16;
  const int64_t k = (target - (int64_t)m * cum[lo] + P - 1) / P;
  return lo * m + (int)(k < m ? k : m);
}

// Block b's share [lo, hi) of those items: contiguous (a block's consecutive
// items mostly share a segment and neighbouring rows) and of near-equal cost,
// so the shared expert's many-row items do not pile up on a few blocks.
ASTRO_DEVINL void block_range(const int* cum, const uint16_t* list, const uint32_t* offs, int na,
                              int m, bool single_pass, int& lo, int& hi) {
  if (single_pass || na == 0) {  // every item costs one pass
    lo = (int)((int64_t)na * m * blockIdx.x / gridDim.x);
    hi = (int)((int64_t)na * m * (blockIdx.x + 1) / gridDim.x);
    return;
  }
  const int64_t C = (int64_t)m * cum[na];
  lo = item_at_cost(cum, list, offs, na, m, C * blockIdx.x / gridDim.x);
  hi = blockIdx.x + 1 == gridDim.x ? na * m
                                   : item_at_cost(cum, list, offs, na, m, C * (blockIdx.x + 1) / gridDim.x);
}

// ---- warp tensor-core tiles for the fused decode projections ----
// mma.sync m16n8k16: A (16 x 16, bf16) = 16 weight rows, B (16 x 8, bf16) = 8
// token rows, D (16 x 8) fp32 += A B.  Lane l holds A rows l/4 and l/4 + 8 and
// B column l/4, at K positions 2(l%4) + {0, 1} and + 8.  A packed int4 word
// dequantises most cheaply into the pairs (element i, element i + 4), so every
// 8-element chunk of K is taken in the order (0,4,1,5,2,6,3,7): lane l%4 = c
// reads words 2c and 2c + 1 of each 64-wide group (elements 16c .. 16c + 15),
// and the token rows are staged with each 16-byte chunk pair-interleaved the
// same way.  Both operands see one permutation of K, so the products and the
// fp32 sum are those of the natural order up to the order of addition.
ASTRO_DEVINL void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                 uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// (element i, element i + 4) of a packed word as bf16 s * q + b (i = 0 .. 3)
ASTRO_DEVINL uint32_t dq_pair(uint32_t v, int i, __nv_bfloat162 s2, __nv_bfloat162 b2) {
  const __nv_bfloat162 k128 = __floats2bfloat162_rn(128.0f, 128.0f);
  const uint32_t tq = ((v >> (4 * i)) & 0x000f000fu) | 0x43004300u;  // bf16 (128 + q)
  const __nv_bfloat162 q = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&tq), k128);
  const __nv_bfloat162 w = __hfma2(q, s2, b2);
  return *reinterpret_cast<const uint32_t*>(&w);
}

// 8 natural-order bf16 -> the pairs (0,4) (1,5) (2,6) (3,7)
ASTRO_DEVINL uint4 pair_interleave(const uint4& v) {
  return make_uint4(__byte_perm(v.x, v.z, 0x5410), __byte_perm(v.x, v.z, 0x7632),
                    __byte_perm(v.y, v.w, 0x5410), __byte_perm(v.y, v.w, 0x7632));
}

ASTRO_DEVINL uint2 ld_stream2(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}

// KG consecutive bf16 (a row's scales or biases over the tile's groups) in
// (KG + 1) / 2 words, loaded as one vector; nothing waits on it until use.
template <int KG> struct Bf16Vec {
  uint32_t w[(KG + 1) / 2];
  ASTRO_DEVINL void load(const uint16_t* p) {
    if constexpr (KG == 8) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
      w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    } else if constexpr (KG == 4) {
      const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
      w[0] = v.x; w[1] = v.y;
    } else {
      static_assert(KG == 2, "2, 4 or 8 groups per K quarter");
      w[0] = __ldg(reinterpret_cast<const unsigned int*>(p));
    }
  }
  ASTRO_DEVINL __nv_bfloat162 pair(int G) const {  // value G in both halves
    const uint16_t h = (uint16_t)(w[G >> 1] >> (16 * (G & 1)));
    return __halves2bfloat162(__ushort_as_bfloat16(h), __ushort_as_bfloat16(h));
  }
};

// One lane's share of a 16-row tile over KG groups of K: rows r and r + 8
// (codes: words 2c, 2c + 1 of each group; the groups' scales and biases).
template <int KG> struct TileRegs {
  uint2 qa[KG], qb[KG];
  Bf16Vec<KG> sa, ba, sb, bb;
};
// Issues the tile's loads (the scale and bias rows must be 2*KG-byte aligned).
template <int KG>
ASTRO_DEVINL void load_tile(TileRegs<KG>& R, const AffineRef& W, int64_t e, int64_t r, int K,
                            int g0, int c) {
  const int words = K / 8, groups = K / 64;
  const uint32_t* qa = reinterpret_cast<const uint32_t*>(W.q) + q_row(W, e, r) * words + g0 * 8 + 2 * c;
  const uint32_t* qb = qa + (int64_t)8 * words;
  const uint16_t* s = reinterpret_cast<const uint16_t*>(W.s);
  const uint16_t* b = reinterpret_cast<const uint16_t*>(W.b);
  const int64_t ra = sb_row(W, e, r) * groups + g0, rb = ra + (int64_t)8 * groups;
#pragma unroll
  for (int G = 0; G < KG; ++G) {
    R.qa[G] = ld_stream2(qa + G * 8);
    R.qb[G] = ld_stream2(qb + G * 8);
  }
  R.sa.load(s + ra);
  R.ba.load(b + ra);
  R.sb.load(s + rb);
  R.bb.load(b + rb);
}

// D0 (+ D1) += tile x token rows over the tile's KG groups.  x0 / x1: this
// lane's B rows (pair-interleaved, at the tile's first group + 32 c bytes).
template <int KG>
ASTRO_DEVINL void tile_mma(const TileRegs<KG>& R, const uint8_t* x0, const uint8_t* x1, bool two,
                           float (&d0)[4], float (&d1)[4]) {
#pragma unroll
  for (int G = 0; G < KG; ++G) {
    const __nv_bfloat162 sa = R.sa.pair(G), ba = R.ba.pair(G);
    const __nv_bfloat162 sb = R.sb.pair(G), bb = R.bb.pair(G);
    const uint4 u0 = *reinterpret_cast<const uint4*>(x0 + G * 128);
    const uint4 u1 = *reinterpret_cast<const uint4*>(x0 + G * 128 + 16);
    uint4 v0 = u0, v1 = u1;
    if (two) {
      v0 = *reinterpret_cast<const uint4*>(x1 + G * 128);
      v1 = *reinterpret_cast<const uint4*>(x1 + G * 128 + 16);
    }
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const uint32_t wa = s < 2 ? R.qa[G].x : R.qa[G].y;
      const uint32_t wb = s < 2 ? R.qb[G].x : R.qb[G].y;
      const int i0 = 2 * (s & 1);
      const uint32_t a0 = dq_pair(wa, i0, sa, ba), a2 = dq_pair(wa, i0 + 1, sa, ba);
      const uint32_t a1 = dq_pair(wb, i0, sb, bb), a3 = dq_pair(wb, i0 + 1, sb, bb);
      const uint4& xu = s < 2 ? u0 : u1;
      mma_bf16_16816(d0, a0, a1, a2, a3, (s & 1) ? xu.z : xu.x, (s & 1) ? xu.w : xu.y);
      if (two) {
        const uint4& xv = s < 2 ? v0 : v1;
        mma_bf16_16816(d1, a0, a1, a2, a3, (s & 1) ? xv.z : xv.x, (s & 1) ? xv.w : xv.y);
      }
    }
  }
}

constexpr int kStageRows = 16;  // activation rows staged per down pass
constexpr int kRedFloats = 4 * 4 * 2 * 4 * 32;
// bytes of the phase-1 / phase-2 / phase-4 union at the start of shared memory
template <int H, int I> constexpr int kUnionBytes() {
  constexpr int a = kStageTokens * H * 2, b = kFusedMaxTokens * kFusedMaxExperts * 2,
                c = kStageRows * (I * 2 + 16);
  return a > b ? (a > c ? a : c) : (b > c ? b : c);
}
template <int H, int I> constexpr int fused_smem_bytes() {
  return kUnionBytes<H, I>() + kStageTokens * (H * 2 + 16) + kRedFloats * 4;
}

// fp32 partial sums of the four K quarters: [quarter][tile][chunk][reg][lane]
ASTRO_DEVINL int red_at(int quarter, int tile, int chunk, int reg, int lane) {
  return (((quarter * 4 + tile) * 2 + chunk) * 4 + reg) * 32 + lane;
}
// the quarters' sum, in a fixed order, of output (row r of tile, token column j)
ASTRO_DEVINL float red_sum(const float* red, int tile, int r, int j) {
  const int ch = j >> 3, c = j & 7;
  const int ln = (r & 7) * 4 + (c >> 1), rg = (r >> 3) * 2 + (c & 1);
  float v = 0.f;
#pragma unroll
  for (int q = 0; q < 4; ++q) v = __fadd_rn(v, red[red_at(q, tile, ch, rg, ln)]);
  return v;
}

struct FusedDecodeParams {
  const __nv_bfloat16* x;  // [T, H]
  static FusedDecodeParams from(const DecodeFusedArgs& a) {
    FusedDecodeParams p;
    p.x = reinterpret_cast<const __nv_bfloat16*>(a.x);
    p.T = a.T;
    p.E = a.E;
    p.K = a.K;
    p.normalize = a.normalize;
    p.sorted = a.sorted;
    p.has_shared = a.has_shared;
    p.wr = reinterpret_cast<const __nv_bfloat16*>(a.wr);
    p.wg = reinterpret_cast<const __nv_bfloat16*>(a.wg);
    for (int i = 0; i < 2; ++i) {
      p.gate[i] = a.gate[i];
      p.up[i] = a.up[i];
      p.down[i] = a.down[i];
    }
    p.logits = reinterpret_cast<__nv_bfloat16*>(a.logits);
    p.gate_logit = reinterpret_cast<__nv_bfloat16*>(a.gate_logit);
    p.ids = a.ids;
    p.scores = reinterpret_cast<__nv_bfloat16*>(a.scores);
    p.offsets = a.offsets;
    p.act = reinterpret_cast<__nv_bfloat16*>(a.act);
    p.yrows = reinterpret_cast<__nv_bfloat16*>(a.yrows);
    p.out = reinterpret_cast<__nv_bfloat16*>(a.out);
    p.barrier = a.barrier;
    p.seg_done = a.seg_done;
    p.status = a.status;
    return p;
  }
  int T, E, K, normalize, sorted, has_shared;
  const __nv_bfloat16* wr;  // [E, H]
  const __nv_bfloat16* wg;  // [H] shared-expert gate (has_shared)
  AffineRef gate[2], up[2], down[2];  // [routed, shared]
  __nv_bfloat16* logits;      // [T, E]
  __nv_bfloat16* gate_logit;  // [T]
  uint32_t* ids;              // [T * K]
  __nv_bfloat16* scores;      // [T * K]
  uint32_t* offsets;          // [E + 2]
  __nv_bfloat16* act;         // [T * K + T, I]
  __nv_bfloat16* yrows;       // [T * K + T, H]
  __nv_bfloat16* out;         // [T, H]
  uint32_t* barrier;          // {arrivals, exits}; both zero between launches
  uint32_t* seg_done;         // [E + 1] gate/up items finished per segment; zero between launches
  uint32_t* status;
};

// Grid-wide barrier number `nth` (1, 2, 3) of a cooperative launch: every block
// adds one to the arrival word with a release reduction (no round trip) and
// polls it with acquire loads until nth * gridDim arrivals are in, so the last
// arrival releases everyone after one trip through L2.  The wait is bounded
// (2 s): on timeout it records kDevWaitTimeout and returns false, and the
// caller skips the rest of the kernel.  grid_exit() zeroes the words again once
// every block has passed the last barrier.
ASTRO_DEVINL bool grid_barrier(uint32_t* bar, uint32_t nth, uint32_t* status, int* flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t target = nth * gridDim.x;
    uint32_t v;
    int ok = 1;
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
    uint64_t t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    uint32_t spins = 0;
    while (true) {
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(bar) : "memory");
      if (v >= target) break;
      if ((++spins & 255u) == 0) {
        uint64_t t1;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
        if (t1 - t0 > 2000000000ull) {
          record_status(status, kDevWaitTimeout);
          ok = 0;
          break;
        }
      }
    }
    *flag = ok;
  }
  __syncthreads();
  return *flag != 0;
}

// After the last barrier: the last block to get here zeroes both words for the
// next launch (no block polls the arrival word any more).
ASTRO_DEVINL void grid_exit(uint32_t* bar) {
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(bar + 1) : "memory");
    if (old == gridDim.x - 1) {
      asm volatile("st.relaxed.gpu.global.u32 [%0], 0;" ::"l"(bar) : "memory");
      asm volatile("st.relaxed.gpu.global.u32 [%0], 0;" ::"l"(bar + 1) : "memory");
    }
  }
}

// one bulk prefetch of [p, p + bytes) into L2 (p 16-byte aligned, bytes a
// multiple of 16; callers keep pieces at or below 32 KB)
ASTRO_DEVINL void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// the grid's share of [p, p + bytes): 16 KB pieces, block b taking pieces b,
// b + grid, ... (issued by the calling thread)
ASTRO_DEVINL void prefetch_l2_grid(const void* p, int64_t bytes) {
  constexpr int64_t kPiece = 16384;
  const char* c = reinterpret_cast<const char*>(p);
  for (int64_t off = (int64_t)blockIdx.x * kPiece; off < bytes; off += (int64_t)gridDim.x * kPiece)
    prefetch_l2_bulk(c + off, (uint32_t)(bytes - off < kPiece ? bytes - off : kPiece));
}

template <int H, int I>
__global__ void __launch_bounds__(kGemvThreads, 1) decode_fused_kernel(FusedDecodeParams P) {
  constexpr int kVecs = H / 8;            // uint4 per x row
  constexpr int kXpStride = H * 2 + 16, kApStride = I * 2 + 16;  // padded: no bank conflicts
  // dynamic shared memory: [union: x rows (phase 1) | logits (phase 2) | act rows
  // (phase 4)] [token rows, pair-interleaved] [partial sums]
  extern __shared__ uint4 smem[];
  uint4* xs = smem;  // phase 1, T <= kStageTokens: [T][kVecs], swizzled
  __nv_bfloat16* s_logits = reinterpret_cast<__nv_bfloat16*>(smem);  // phase 2: [T][E]
  uint8_t* ap = reinterpret_cast<uint8_t*>(smem);                      // phase 4: [kStageRows]
  uint8_t* xp = reinterpret_cast<uint8_t*>(smem) + kUnionBytes<H, I>();  // [kStageTokens] rows
  float* red = reinterpret_cast<float*>(xp + kStageTokens * kXpStride);  // partial sums
  __shared__ uint32_t s_ids[kFusedMaxAssign];
  __shared__ __nv_bfloat16 s_sc16[kFusedMaxAssign];
  __shared__ float s_score[kFusedMaxAssign];
  __shared__ uint32_t s_inv[kFusedMaxAssign];
  __shared__ uint32_t s_stok[kFusedMaxAssign + kFusedMaxTokens];
  __shared__ uint8_t s_wcnt[kFusedMaxAssign / 32][kFusedMaxExperts];  // ids per warp of assignments
  __shared__ uint32_t s_offs[kFusedMaxExperts + 2];
  __shared__ uint16_t s_list[kFusedMaxExperts + 1];
  __shared__ int s_cum[kFusedMaxExperts + 2];  // 16-row passes before each active segment
  __shared__ float s_sg[kFusedMaxTokens];
  __shared__ int s_wsum[kGemvWarps], s_wnz[kGemvWarps];  // per-warp scan totals
  __shared__ int s_flag;
  __shared__ int s_ready;
  __shared__ int s_nact;

  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int T = P.T, E = P.E, K = P.K, N = T * K;
  const int gtid = blockIdx.x * kGemvThreads + threadIdx.x, nthreads = gridDim.x * kGemvThreads;

  // ---- phase 1: router logits (+ shared gate logit) ----
  // Block b computes router rows b, b + grid, ...: two rows per pass, each split
  // into eight K slices of H / 8 (warp w: row w >> 3 of the pass, slice w & 7);
  // a warp's slice sums go through shared memory and the eight slices are added
  // in order.  Each warp's weight vector is requested before x is staged.  Up to
  // kStageTokens tokens, x is staged in shared memory (and pair-interleaved for
  // phase 3); above, warps read their x slices from L2 and phase 3 stages the
  // token rows of each segment.
  const bool stage_all = T <= kStageTokens;
  {
    constexpr int kSliceVecs = kVecs / 8;  // uint4 per slice: 32 (H = 2048) or 16
    const int rows = E + (P.has_shared ? 1 : 0);
    const int rs = w >> 3, sl = w & 7;
    const bool vlane = lane < kSliceVecs;
    auto row_ptr = [&](int r) {
      return reinterpret_cast<const uint4*>(r < E ? P.wr + (int64_t)r * H : P.wg) + sl * kSliceVecs +
             lane;
    };
    int r = (int)blockIdx.x + rs * (int)gridDim.x;
    uint4 wv = make_uint4(0u, 0u, 0u, 0u);
    if (r < rows && vlane) wv = ld_stream(row_ptr(r));
    const uint4* xsrc = reinterpret_cast<const uint4*>(P.x);
    if (stage_all)
      for (int i = threadIdx.x; i < T * kVecs; i += kGemvThreads) {
        const int t = i / kVecs, q = i - t * kVecs;
        const uint4 v = ld_cached(xsrc + (int64_t)t * kVecs + q);
        xs[t * kVecs + swz(q)] = v;
        *reinterpret_cast<uint4*>(xp + t * kXpStride + q * 16) = pair_interleave(v);
      }
    if (P.has_shared && threadIdx.x == 0) {
      // the shared expert is always used: start pulling its weights into L2
      const AffineRef sw[3] = {P.gate[1], P.up[1], P.down[1]};
      const int64_t qbytes[3] = {(int64_t)I * H / 2, (int64_t)I * H / 2, (int64_t)H * I / 2};
      const int64_t sbytes[3] = {(int64_t)I * (H / 64) * 2, (int64_t)I * (H / 64) * 2,
                                 (int64_t)H * (I / 64) * 2};
#pragma unroll
      for (int m = 0; m < 3; ++m) {
        prefetch_l2_grid(sw[m].q, qbytes[m]);
        prefetch_l2_grid(sw[m].s, sbytes[m]);
        prefetch_l2_grid(sw[m].b, sbytes[m]);
      }
    }
    float* s_part = red;  // [2 rows][8 slices][kFusedMaxTokens]
    const int xq = sl * kSliceVecs + lane;  // this lane's x vector of the slice
    for (int pass = 0; pass * 2 * (int)gridDim.x < rows; ++pass) {
      if (pass > 0) {
        r = (int)blockIdx.x + (2 * pass + rs) * (int)gridDim.x;
        if (r < rows && vlane) wv = ld_stream(row_ptr(r));
      }
      __syncthreads();  // x staged; the previous pass is done with s_part
      if (r < rows) {
        float wf[8];
        bf16x8_to_f32(wv, wf);
        for (int t0 = 0; t0 < T; t0 += kStageTokens) {  // 16 tokens' sums at a time
          float acc[kStageTokens];
#pragma unroll
          for (int t = 0; t < kStageTokens; ++t) {
            acc[t] = 0.f;
            if (t0 + t < T && vlane) {
              float xf[8];
              bf16x8_to_f32(stage_all ? xs[t * kVecs + swz(xq)]
                                      : ld_cached(xsrc + (int64_t)(t0 + t) * kVecs + xq), xf);
#pragma unroll
              for (int i = 0; i < 8; ++i) acc[t] = __fmaf_rn(wf[i], xf[i], acc[t]);
            }
          }
#pragma unroll
          for (int t = 0; t < kStageTokens; ++t) {
            if (t0 + t < T) {
              const float v = warp_sum(acc[t]);
              if (lane == 0) s_part[(rs * 8 + sl) * kFusedMaxTokens + t0 + t] = v;
            }
          }
        }
      }
      __syncthreads();
      if (threadIdx.x < 2 * T) {
        const int k = threadIdx.x / T, t = threadIdx.x - k * T;
        const int rr = (int)blockIdx.x + (2 * pass + k) * (int)gridDim.x;
        if (rr < rows) {
          float v = 0.f;
#pragma unroll
          for (int s = 0; s < 8; ++s) v = __fadd_rn(v, s_part[(k * 8 + s) * kFusedMaxTokens + t]);
          if (rr < E) P.logits[(int64_t)t * E + rr] = __float2bfloat16_rn(v);
          else P.gate_logit[t] = __float2bfloat16_rn(v);
        }
      }
    }
  }
  if (!grid_barrier(P.barrier, 1, P.status, &s_flag)) return;

  // ---- phase 2: route + sort, redundantly in every block ----
  for (int i = threadIdx.x; i < T * E; i += kGemvThreads)
    s_logits[i] = __ushort_as_bfloat16(__ldcg(reinterpret_cast<const unsigned short*>(P.logits) + i));
  const int nw_assign = (N + 31) >> 5;  // warps holding assignments
  for (int i = threadIdx.x; i < nw_assign * kFusedMaxExperts / 4; i += kGemvThreads)
    reinterpret_cast<uint32_t*>(&s_wcnt[0][0])[i] = 0u;
  if (threadIdx.x < T)
    s_sg[threadIdx.x] =
        P.has_shared
            ? round_bf16(sigmoid_mlx(bf16_to_f32(__ldcg(reinterpret_cast<const unsigned short*>(P.gate_logit) + threadIdx.x))))
            : 0.f;
  __syncthreads();
  for (int tk = w; tk < T; tk += kGemvWarps)
    route_token<__nv_bfloat16, 8>(s_logits + tk * E, E, K, P.normalize, s_ids + tk * K, s_sc16 + tk * K);
  __syncthreads();
  // stable counting sort of the N assignments by expert: the rank of an
  // assignment among equal ids is its rank inside its warp (match_any) plus the
  // count of that id in earlier warps (per-warp counts, no atomics)
  int rank = 0;
  uint32_t my_id = 0xffffffffu;
  if (w < nw_assign) {
    if (threadIdx.x < N) {
      s_inv[threadIdx.x] = 0;  // an id >= E keeps slot row 0 (recorded, never used for output)
      my_id = s_ids[threadIdx.x];
      s_score[threadIdx.x] = __bfloat162float(s_sc16[threadIdx.x]);
      if (my_id >= (uint32_t)E) record_status(P.status, kDevBadExpertId);
      if (blockIdx.x == 0) {
        P.ids[threadIdx.x] = my_id;
        P.scores[threadIdx.x] = s_sc16[threadIdx.x];
      }
    }
    const uint32_t m = __match_any_sync(0xffffffffu, my_id);
    rank = __popc(m & lanemask_lt());
    if (my_id < (uint32_t)E && rank == 0) s_wcnt[w][my_id] = (uint8_t)__popc(m);
  }
  __syncthreads();
  if (my_id < (uint32_t)E)
    for (int v = 0; v < w; ++v) rank += s_wcnt[v][my_id];
  {
    // exclusive scans, over the block, of the E counts (thread e: expert e) and of
    // the non-empty experts; the active list follows expert order, then the
    // shared expert
    int c = 0;
    if ((int)threadIdx.x < E)
      for (int v = 0; v < nw_assign; ++v) c += s_wcnt[v][threadIdx.x];
    const int nz = c > 0 ? 1 : 0;
    int ic = c, inz = nz;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, ic, d);
      const int no = __shfl_up_sync(0xffffffffu, inz, d);
      if (lane >= d) {
        ic += o;
        inz += no;
      }
    }
    if (lane == 31) {
      s_wsum[w] = ic;
      s_wnz[w] = inz;
    }
    __syncthreads();
    int base = 0, nbase = 0, tot = 0, ntot = 0;
#pragma unroll
    for (int i = 0; i < kGemvWarps; ++i) {
      const int s = s_wsum[i], z = s_wnz[i];
      base += i < w ? s : 0;
      nbase += i < w ? z : 0;
      tot += s;
      ntot += z;
    }
    if ((int)threadIdx.x < E) {
      s_offs[threadIdx.x] = (uint32_t)(base + ic - c);
      if (nz) s_list[nbase + inz - 1] = (uint16_t)threadIdx.x;
    }
    if (threadIdx.x == 0) {
      s_offs[E] = (uint32_t)tot;
      s_offs[E + 1] = (uint32_t)(tot + (P.has_shared ? T : 0));
      int na = ntot;
      if (P.has_shared && T > 0) s_list[na++] = (uint16_t)E;
      s_nact = na;
    }
  }
  __syncthreads();
  if (w == 0 && T > kStageTokens) {
    // pass counts of the active segments, exclusive scan (block ranges by cost;
    // up to 16 tokens every segment is one pass)
    const int na = s_nact, C2 = (na + 31) / 32;
    int part = 0;
    for (int i = 0; i < C2; ++i) {
      const int idx = lane * C2 + i;
      if (idx < na) {
        const int sg = s_list[idx];
        part += (int)((s_offs[sg + 1] - s_offs[sg] + 15) / 16);
      }
    }
    int incl = part;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += o;
    }
    int run = incl - part;
    for (int i = 0; i < C2; ++i) {
      const int idx = lane * C2 + i;
      if (idx < na) {
        const int sg = s_list[idx];
        s_cum[idx] = run;
        run += (int)((s_offs[sg + 1] - s_offs[sg] + 15) / 16);
      }
    }
    if (lane == 31) s_cum[na] = incl;
  }
  if (threadIdx.x < N && my_id < (uint32_t)E) {
    const uint32_t pos = s_offs[my_id] + (uint32_t)rank;
    s_stok[pos] = threadIdx.x / K;
    s_inv[threadIdx.x] = pos;
  }
  if (P.has_shared && threadIdx.x < T) s_stok[s_offs[E] + threadIdx.x] = threadIdx.x;
  if (blockIdx.x == 0)
    for (int e = threadIdx.x; e < E + 2; e += kGemvThreads) P.offsets[e] = s_offs[e];
  __syncthreads();
  const int n_act = s_nact;
  // ---- phases 3 and 4: items and weight tiles ----
  // Gate/up item = (active segment, 32 features): their 32 gate and 32 up rows
  // against every token row of the segment; down item = (active segment, 64
  // output rows).  Warp w takes tile w & 3 (gate/up: gate rows of features
  // 0-15, 16-31, then up rows of the same) over K quarter w >> 2 on warp
  // tensor-core tiles; the quarters' partials are added in shared memory.  Each
  // block takes a contiguous share of the items; an item's weight rows are
  // requested before the previous item's epilogue (the first gate/up item's
  // before the L2 prefetch below, the first down item's before barrier 2).
  constexpr int kGQ3 = H / 256, kGQ4 = I / 256;  // 64-wide groups per K quarter
  const int g8 = lane >> 2, c4 = lane & 3;
  const int tile = w & 3, quarter = w >> 2;
  const int per_gu = I / 32, per_d = H / 64;
  int lo3, hi3, lo4, hi4;
  block_range(s_cum, s_list, s_offs, n_act, per_gu, stage_all, lo3, hi3);
  block_range(s_cum, s_list, s_offs, n_act, per_d, stage_all, lo4, hi4);
  TileRegs<kGQ3> R3;
  auto load3 = [&](int it) {
    const int seg = s_list[it / per_gu];
    const int sh = seg == E ? 1 : 0;
    const AffineRef W = tile < 2 ? (sh ? P.gate[1] : P.gate[0]) : (sh ? P.up[1] : P.up[0]);
    load_tile<kGQ3>(R3, W, sh ? 0 : seg, (it % per_gu) * 32 + (tile & 1) * 16 + g8, H,
                    quarter * kGQ3, c4);
  };
  if (lo3 < hi3) load3(lo3);
  // the experts are known: pull the rest of this block's gate/up rows (now) and
  // its down rows (once the first gate/up tile's own loads are served, after
  // its MMAs) into L2, one bulk prefetch per contiguous range (an item's codes,
  // scales or biases), so the loads of phases 3 and 4 do not each wait a full
  // HBM trip
  auto prefetch_items = [&](bool gate_up, bool down_rows) {
    const int n_gu = gate_up && hi3 - lo3 > 1 ? hi3 - lo3 - 1 : 0, n_d = down_rows ? hi4 - lo4 : 0;
    for (int i = threadIdx.x; i < n_gu * 6 + n_d * 3; i += kGemvThreads) {
      int seg, row0, rows, K, range;
      bool up = false, down = false;
      if (i < n_gu * 6) {
        const int it = lo3 + 1 + i / 6, m = i % 6;
        seg = s_list[it / per_gu];
        row0 = (it % per_gu) * 32;
        rows = 32;
        K = H;
        up = m >= 3;
        range = m % 3;
      } else {
        const int i2 = i - n_gu * 6;
        const int it = lo4 + i2 / 3;
        seg = s_list[it / per_d];
        row0 = (it % per_d) * 64;
        rows = 64;
        K = I;
        down = true;
        range = i2 % 3;
      }
      const int sh = seg == E ? 1 : 0;
      const AffineRef W = down ? (sh ? P.down[1] : P.down[0])
                               : (up ? (sh ? P.up[1] : P.up[0]) : (sh ? P.gate[1] : P.gate[0]));
      const int64_t ex = sh ? 0 : (int64_t)seg;
      if (range == 0)
        prefetch_l2_bulk(reinterpret_cast<const char*>(W.q) + q_row(W, ex, row0) * (K / 2),
                         (uint32_t)(rows * (K / 2)));
      else
        prefetch_l2_bulk(reinterpret_cast<const char*>(range == 1 ? W.s : W.b) +
                             sb_row(W, ex, row0) * (K / 64) * 2,
                         (uint32_t)(rows * (K / 64) * 2));
    }
  };
  prefetch_items(true, lo3 >= hi3);

  // ---- phase 3: gate/up + SwiGLU ----
  int xp_seg = -1;  // (T > kStageTokens) segment whose rows from xp_p sit in xp
  uint32_t xp_p = 0;
  const uint4* xsrc = reinterpret_cast<const uint4*>(P.x);
  for (int it = lo3; it < hi3; ++it) {
    const int seg = s_list[it / per_gu];
    const int fi = (it % per_gu) * 32;
    const uint32_t p0 = s_offs[seg], p1 = s_offs[seg + 1];
    for (uint32_t pb = p0; pb < p1; pb += kStageTokens) {
      const int n = (int)(p1 - pb < (uint32_t)kStageTokens ? p1 - pb : (uint32_t)kStageTokens);
      if (!stage_all && (seg != xp_seg || pb != xp_p)) {
        // every warp finished its previous MMAs before the last epilogue's barrier
        for (int i = threadIdx.x; i < n * kVecs; i += kGemvThreads) {
          const int j = i / kVecs, q = i - j * kVecs;
          *reinterpret_cast<uint4*>(xp + j * kXpStride + q * 16) =
              pair_interleave(ld_cached(xsrc + (int64_t)s_stok[pb + j] * kVecs + q));
        }
        xp_seg = seg;
        xp_p = pb;
        __syncthreads();
      }
      // B column g8 of chunk 0 / 1: sorted rows pb + g8 / pb + 8 + g8 (a valid row
      // stands in past n; its columns are not stored)
      const int j0 = g8 < n ? g8 : 0, j1 = g8 + 8 < n ? g8 + 8 : 0;
      const int b0 = stage_all ? (int)s_stok[pb + j0] : j0, b1 = stage_all ? (int)s_stok[pb + j1] : j1;
      const int off = quarter * kGQ3 * 128 + c4 * 32;
      float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
      tile_mma<kGQ3>(R3, xp + b0 * kXpStride + off, xp + b1 * kXpStride + off, n > 8, d0, d1);
      if (it == lo3 && pb == p0) prefetch_items(false, true);
      if (pb + kStageTokens >= p1 && it + 1 < hi3) load3(it + 1);
      __syncthreads();  // the previous epilogue is done with red
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        red[red_at(quarter, tile, 0, r, lane)] = d0[r];
        red[red_at(quarter, tile, 1, r, lane)] = d1[r];
      }
      __syncthreads();
      const int fl = threadIdx.x & 31, j = threadIdx.x >> 5;  // 32 features x kStageTokens rows
      if (j < n) {
        const float g = red_sum(red, fl >> 4, fl & 15, j);
        const float u = red_sum(red, 2 + (fl >> 4), fl & 15, j);
        P.act[(int64_t)(pb + j) * I + fi + fl] =
            __float2bfloat16_rn(swiglu_bf16(round_bf16(g), round_bf16(u)));
      }
      if (pb + kStageTokens >= p1) {
        // the item's act columns are stored: count it for its segment (release)
        __syncthreads();
        if (threadIdx.x == 0)
          asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(P.seg_done + seg) : "memory");
      }
    }
  }
  TileRegs<kGQ4> R4;
  auto load4 = [&](int it) {
    const int seg = s_list[it / per_d];
    const int sh = seg == E ? 1 : 0;
    load_tile<kGQ4>(R4, sh ? P.down[1] : P.down[0], sh ? 0 : seg,
                    (it % per_d) * 64 + tile * 16 + g8, I, quarter * kGQ4, c4);
  };
  if (lo4 < hi4) load4(lo4);

  // ---- phase 4: down ----
  // B = the segment's activation rows, staged (pair-interleaved) once for all
  // of the block's items on it.
  {
    constexpr int kAVecs = I / 8;
    const uint4* asrc = reinterpret_cast<const uint4*>(P.act);
    int staged_seg = -1;  // segment whose rows from staged_p sit in ap
    uint32_t staged_p = 0;
    int ready_seg = -1;   // segment whose gate/up items are all counted
    for (int it = lo4; it < hi4; ++it) {
      const int seg = s_list[it / per_d];
      const int r0 = (it % per_d) * 64;
      const uint32_t p0 = s_offs[seg], p1 = s_offs[seg + 1];
      for (uint32_t pb = p0; pb < p1; pb += kStageRows) {
        const int n = (int)(p1 - pb < (uint32_t)kStageRows ? p1 - pb : (uint32_t)kStageRows);
        const bool restage = seg != staged_seg || pb != staged_p;
        if (restage && seg != ready_seg && threadIdx.x == 0)
          s_ready = wait_count_geq(P.seg_done + seg, (uint32_t)per_gu, P.status);
        __syncthreads();  // the previous epilogue is done with red (and ap); the segment is ready
        if (restage && seg != ready_seg) {
          if (!s_ready) return;
          ready_seg = seg;
        }
        if (restage) {
          for (int i = threadIdx.x; i < n * kAVecs; i += kGemvThreads) {
            const int j = i / kAVecs, q = i - j * kAVecs;
            *reinterpret_cast<uint4*>(ap + j * kApStride + q * 16) =
                pair_interleave(__ldcg(asrc + (int64_t)(pb + j) * kAVecs + q));
          }
          staged_seg = seg;
          staged_p = pb;
          __syncthreads();
        }
        const int j0 = g8 < n ? g8 : 0, j1 = g8 + 8 < n ? g8 + 8 : 0;
        const int off = quarter * kGQ4 * 128 + c4 * 32;
        float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
        tile_mma<kGQ4>(R4, ap + j0 * kApStride + off, ap + j1 * kApStride + off, n > 8, d0, d1);
        if (pb + kStageRows >= p1 && it + 1 < hi4) load4(it + 1);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          red[red_at(quarter, tile, 0, r, lane)] = d0[r];
          red[red_at(quarter, tile, 1, r, lane)] = d1[r];
        }
        __syncthreads();
        const int rl = threadIdx.x & 63, jb = threadIdx.x >> 6;  // 64 rows x 8 (+8) tokens
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int j = jb + 8 * h;
          if (j < n)
            P.yrows[(int64_t)(pb + j) * H + r0 + rl] =
                __float2bfloat16_rn(red_sum(red, rl >> 4, rl & 15, j));
        }
      }
    }
  }
  if (!grid_barrier(P.barrier, 2, P.status, &s_flag)) return;
  // every block is past its counter waits: zero the counters for the next launch
  for (int i = gtid; i <= E; i += nthreads) P.seg_done[i] = 0;

  // ---- phase 5: weighted combine + gated shared expert ----
  {
    const uint4* rows = reinterpret_cast<const uint4*>(P.yrows);
    uint4* out = reinterpret_cast<uint4*>(P.out);
    for (int u = gtid; u < T * kVecs; u += nthreads) {
      const int t = u / kVecs, c = u - t * kVecs;
      out[u] = combine_chunk(rows, rows, kVecs, c, s_inv + t * K, s_score + t * K, K,
                             P.sorted != 0, P.has_shared ? (int64_t)(s_offs[E] + t) : -1, s_sg[t]);
    }
  }
  grid_exit(P.barrier);
}

}  // namespace

bool router_gemv_supported(int H) { return H == 1024 || H == 2048 || H == 4096; }

cudaError_t launch_router_gemv(const void* x, int64_t T, const void* wr, int E, int H, void* logits,
                               cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  const dim3 grid((unsigned)((E + kWarps - 1) / kWarps),
                  (unsigned)((T + kRouterTokens - 1) / kRouterTokens));
  const size_t smem = (size_t)kRouterTokens * H * 2;
  auto* xx = reinterpret_cast<const __nv_bfloat16*>(x);
  auto* ww = reinterpret_cast<const __nv_bfloat16*>(wr);
  auto* out = reinterpret_cast<__nv_bfloat16*>(logits);
  switch (H) {
    case 1024:
      router_gemv_kernel<4><<<grid, kThreads, smem, st>>>(xx, T, ww, E, out);
      break;
    case 2048:
      router_gemv_kernel<8><<<grid, kThreads, smem, st>>>(xx, T, ww, E, out);
      break;
    case 4096:
      cudaFuncSetAttribute(router_gemv_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem);
      router_gemv_kernel<16><<<grid, kThreads, smem, st>>>(xx, T, ww, E, out);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

bool decode_gemv_supported(int H, int I, int group, int bits) {
  return bits == 4 && group == 64 && (H == 1024 || H == 2048 || H == 4096) &&
         (I == 512 || I == 1024 || I == 2048) && I % kGemvWarps == 0 && H % (4 * kGemvWarps) == 0;
}

cudaError_t launch_decode_gate_up(const GroupedGemvDesc& d, int64_t max_active, cudaStream_t st) {
  if (d.rows_total == 0) return cudaSuccess;
  if (d.nseg > kMaxSegs - 1) return cudaErrorInvalidValue;
  const int grid = grid_for(max_active * (d.out_features / kGemvWarps));
  const size_t smem = (size_t)kRowChunkGU * d.in_features * 2;
  switch (d.in_features) {
    case 1024: decode_gate_up_kernel<1><<<grid, kGemvThreads, smem, st>>>(d); break;
    case 2048: decode_gate_up_kernel<2><<<grid, kGemvThreads, smem, st>>>(d); break;
    case 4096:
      cudaFuncSetAttribute(decode_gate_up_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem);
      decode_gate_up_kernel<4><<<grid, kGemvThreads, smem, st>>>(d);
      break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_decode_down(const GroupedGemvDesc& d, int64_t max_active, cudaStream_t st) {
  if (d.rows_total == 0) return cudaSuccess;
  if (d.nseg > kMaxSegs - 1) return cudaErrorInvalidValue;
  const int grid = grid_for(max_active * (d.out_features / (4 * kGemvWarps)));
  const size_t smem = (size_t)kRowChunk * d.in_features * 2;
  switch (d.in_features) {
    case 512: decode_down_kernel<1><<<grid, kGemvThreads, smem, st>>>(d); break;
    case 1024: decode_down_kernel<2><<<grid, kGemvThreads, smem, st>>>(d); break;
    case 2048: decode_down_kernel<4><<<grid, kGemvThreads, smem, st>>>(d); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace astro

namespace astro {

bool decode_fused_supported(int T, int H, int E, int K, int I) {
  return T >= 1 && T <= kFusedMaxTokens && E >= 1 && E <= kFusedMaxExperts && K >= 1 && K <= 32 &&
         T * K <= kFusedMaxAssign && (H == 1024 || H == 2048) && (I == 512 || I == 1024);
}

namespace {
template <int H, int I>
cudaError_t launch_fused_t(const FusedDecodeParams& p, cudaStream_t st) {
  auto kern = decode_fused_kernel<H, I>;
  const size_t smem = (size_t)fused_smem_bytes<H, I>();
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 0, per_sm = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kGemvThreads, smem)) !=
      cudaSuccess)
    return e;
  if (per_sm < 1) return cudaErrorCooperativeLaunchTooLarge;
  FusedDecodeParams arg = p;
  void* args[] = {&arg};
  return cudaLaunchCooperativeKernel((const void*)kern, dim3(sms), dim3(kGemvThreads), args, smem, st);
}
}  // namespace

cudaError_t launch_decode_fused(const DecodeFusedArgs& a, cudaStream_t st) {
  if (!decode_fused_supported(a.T, a.H, a.E, a.K, a.I)) return cudaErrorInvalidValue;
  const FusedDecodeParams p = FusedDecodeParams::from(a);
  if (a.H == 2048 && a.I == 512) return launch_fused_t<2048, 512>(p, st);
  if (a.H == 2048 && a.I == 1024) return launch_fused_t<2048, 1024>(p, st);
  if (a.H == 1024 && a.I == 512) return launch_fused_t<1024, 512>(p, st);
  return launch_fused_t<1024, 1024>(p, st);
}

}  // namespace astro
