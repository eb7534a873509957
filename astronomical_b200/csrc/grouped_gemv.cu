// grouped_gemv.cu -- grouped affine-quantised GEMV/GEMM on CUDA cores.
//
// Computes, for every sorted assignment row p of expert segment s,
//   y[row_out(p), f] = bf16( sum_k x[row_in(p), k] * dequant(W_s)[f, k] )
// (MLX gather_qmm with transpose=true, runtime-integration/src/mlx_quantized_operations.rs:100-157),
// or, in SwiGLU mode, act = swiglu(bf16(x.Wg[f]), bf16(x.Wu[f])) for the fused
// gate/up pair (qwen3_5_moe/model/resident_execution.rs:210-258).
//
// This is the memory-bound path: decode (a handful of rows per expert) and the
// generic fallback for every MLX affine profile (bits 2/3/4/5/6/8, group
// 32/64/128).  Each weight row is read once per tile of up to kRows rows of the
// same expert with 128-bit loads (4-bit) and reduced with warp shuffles; the
// tile's activation rows sit in shared memory.
#include "common.cuh"
#include "kernels.h"

namespace astro {

constexpr int kRows = 8;       // activation rows per tile
constexpr int kWarps = 8;

template <int BITS>
ASTRO_DEVINL void load_chunk(const uint32_t* __restrict__ row, int c, uint32_t (&w)[BITS]) {
  // chunk c = 32 elements = BITS words
  if constexpr (BITS == 4) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(row) + c);
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else if constexpr (BITS == 8) {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(row) + 2 * c);
    const uint4 b = __ldg(reinterpret_cast<const uint4*>(row) + 2 * c + 1);
    w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w; w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
  } else if constexpr (BITS == 2) {
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(row) + c);
    w[0] = v.x; w[1] = v.y;
  } else {
#pragma unroll
    for (int i = 0; i < BITS; ++i) w[i] = __ldg(row + (int64_t)c * BITS + i);
  }
}

template <int BITS>
ASTRO_DEVINL uint32_t code_at(const uint32_t (&w)[BITS], int j) {
  const int bit = j * BITS;
  const int wi = bit >> 5, b = bit & 31;
  uint64_t v = w[wi];
  if (b + BITS > 32) v |= (uint64_t)w[wi + 1] << 32;
  return (uint32_t)(v >> b) & ((1u << BITS) - 1u);
}

struct WRef {
  const uint32_t* q;
  const uint16_t* s;
  const uint16_t* b;
  int64_t expert_rows;  // rows per expert in this tensor
  int64_t row_offset;   // first row inside the expert (the up half of a fused tensor)
};

struct GroupedArgs {
  const __nv_bfloat16* x;
  const uint32_t* x_rows;    // sorted position -> activation row (nullptr: identity)
  int64_t x_limit;           // number of activation rows (bounds check)
  int in_features;
  const uint32_t* seg_offsets;  // [nseg + 1]
  int nseg;
  int shared_seg;            // segment using the shared weights (-1: none)
  WRef wa[2], wb[2];         // [routed, shared]; wb only for SwiGLU
  int out_features, group;
  __nv_bfloat16* y;
  const uint32_t* y_rows;    // sorted position -> output row (nullptr: identity)
  int64_t y_limit;           // number of output rows (bounds check)
  int64_t ldy;
  uint32_t* status;
};

// Dot of one weight row with the tile's rows.  Lanes of a row-group split the
// 32-element chunks of the row; partial sums stay per lane until the caller
// reduces them.
template <int BITS>
ASTRO_DEVINL void row_dot(const uint32_t* __restrict__ wrow, const uint16_t* __restrict__ srow,
                          const uint16_t* __restrict__ brow, int chunks, int group, int sub,
                          int sub_lanes, const __nv_bfloat16* __restrict__ xs, int in_features,
                          int nrows, float (&acc)[kRows]) {
  for (int c = sub; c < chunks; c += sub_lanes) {
    uint32_t w[BITS];
    load_chunk<BITS>(wrow, c, w);
    const int g = (c * 32) / group;
    const float s = bf16_to_f32(__ldg(srow + g)), b = bf16_to_f32(__ldg(brow + g));
    float wv[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) wv[j] = round_bf16(__fmaf_rn(s, (float)code_at<BITS>(w, j), b));
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      if (r < nrows) {
        const uint4* xr = reinterpret_cast<const uint4*>(xs + (int64_t)r * in_features + c * 32);
        float a = acc[r];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 v = xr[q];
          const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            a = __fmaf_rn(__uint_as_float(vv[h] << 16), wv[q * 8 + 2 * h], a);
            a = __fmaf_rn(__uint_as_float(vv[h] & 0xffff0000u), wv[q * 8 + 2 * h + 1], a);
          }
        }
        acc[r] = a;
      }
    }
  }
}

template <int BITS, bool SWIGLU>
__global__ void __launch_bounds__(kWarps * 32) grouped_gemv_kernel(GroupedArgs A, int feats_per_block) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem_raw);  // [kRows][in]
  __shared__ int tile_prefix[1025];
  __shared__ int s_info[3];

  // locate (segment, row chunk) from blockIdx.x via the per-segment tile counts
  if (threadIdx.x < 32) {
    int carry = 0;
    for (int base = 0; base < A.nseg; base += 32) {
      const int s = base + threadIdx.x;
      int c = 0;
      if (s < A.nseg) {
        const int cnt = (int)(A.seg_offsets[s + 1] - A.seg_offsets[s]);
        c = (cnt + kRows - 1) / kRows;
      }
      int incl = c;
#pragma unroll
      for (int m = 1; m < 32; m <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, incl, m);
        if (threadIdx.x >= m) incl += o;
      }
      if (s < A.nseg) tile_prefix[s] = carry + incl - c;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (threadIdx.x == 0) tile_prefix[A.nseg] = carry;
  }
  __syncthreads();
  const int tile = blockIdx.x;
  if (tile >= tile_prefix[A.nseg]) return;
  if (threadIdx.x == 0) {
    int lo = 0, hi = A.nseg - 1;  // last s with prefix[s] <= tile
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (tile_prefix[mid] <= tile) lo = mid; else hi = mid - 1;
    }
    s_info[0] = lo;
    s_info[1] = (int)A.seg_offsets[lo] + (tile - tile_prefix[lo]) * kRows;
    const int end = (int)A.seg_offsets[lo + 1];
    s_info[2] = min(kRows, end - s_info[1]);
  }
  __syncthreads();
  const int seg = s_info[0], p0 = s_info[1], nrows = s_info[2];
  const int in = A.in_features;

  // stage the tile's activation rows
  const int cpr = in / 8;
  for (int i = threadIdx.x; i < nrows * cpr; i += blockDim.x) {
    const int r = i / cpr, c = i - r * cpr;
    const int64_t src = A.x_rows ? (int64_t)A.x_rows[p0 + r] : (int64_t)(p0 + r);
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (src < A.x_limit) v = reinterpret_cast<const uint4*>(A.x + src * in)[c];
    else if (c == 0) record_status(A.status, kDevBadShape);
    reinterpret_cast<uint4*>(xs)[(int64_t)r * cpr + c] = v;
  }
  __syncthreads();

  const bool shared = (seg == A.shared_seg);
  const int wsel = shared ? 1 : 0;
  const int64_t e = shared ? 0 : seg;
  const WRef wa = A.wa[wsel];
  const WRef wb = A.wb[wsel];
  const int words = in * BITS / 32;
  const int groups = in / A.group;
  const int chunks = in / 32;
  // lanes per weight row: 32 when the row has >= 32 chunks, else the largest
  // power of two <= chunks (rows are then processed several per warp)
  int sub_lanes = 32;
  while (sub_lanes > chunks && sub_lanes > 1) sub_lanes >>= 1;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rows_per_warp = 32 / sub_lanes;
  const int sub = lane % sub_lanes, slot = lane / sub_lanes;
  const int f_begin = blockIdx.y * feats_per_block;
  const int f_end = min(A.out_features, f_begin + feats_per_block);

  for (int f0 = f_begin + warp * rows_per_warp; f0 < f_end; f0 += kWarps * rows_per_warp) {
    const int f = f0 + slot;
    const bool fok = f < f_end;
    float acc_a[kRows], acc_b[kRows];
#pragma unroll
    for (int r = 0; r < kRows; ++r) { acc_a[r] = 0.f; acc_b[r] = 0.f; }
    if (fok) {
      const int64_t ra = e * wa.expert_rows + wa.row_offset + f;
      row_dot<BITS>(wa.q + ra * words, wa.s + ra * groups, wa.b + ra * groups, chunks, A.group,
                    sub, sub_lanes, xs, in, nrows, acc_a);
      if constexpr (SWIGLU) {
        const int64_t rb = e * wb.expert_rows + wb.row_offset + f;
        row_dot<BITS>(wb.q + rb * words, wb.s + rb * groups, wb.b + rb * groups, chunks, A.group,
                      sub, sub_lanes, xs, in, nrows, acc_b);
      }
    }
    // reduce over the sub_lanes lanes of this row (butterfly inside the group)
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      for (int m = sub_lanes >> 1; m >= 1; m >>= 1) {
        acc_a[r] = __fadd_rn(acc_a[r], __shfl_xor_sync(0xffffffffu, acc_a[r], m));
        if constexpr (SWIGLU) acc_b[r] = __fadd_rn(acc_b[r], __shfl_xor_sync(0xffffffffu, acc_b[r], m));
      }
    }
    if (fok) {
      // after the butterfly every lane of the group holds all sums; row r is
      // written by lane (r mod sub_lanes) of the group
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        if (r < nrows && (r % sub_lanes) == sub) {
          const int p = p0 + r;
          const int64_t orow = A.y_rows ? (int64_t)A.y_rows[p] : (int64_t)p;
          if (orow >= A.y_limit) {
            record_status(A.status, kDevBadShape);
          } else {
            float v;
            if constexpr (SWIGLU) v = swiglu_bf16(round_bf16(acc_a[r]), round_bf16(acc_b[r]));
            else v = acc_a[r];
            A.y[orow * A.ldy + f] = __float2bfloat16_rn(v);
          }
        }
      }
    }
  }
}

template <int BITS, bool SW>
static cudaError_t launch_gemv_t(const GroupedArgs& A, int64_t max_tiles, cudaStream_t st) {
  const size_t smem = sizeof(__nv_bfloat16) * kRows * (size_t)A.in_features;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(grouped_gemv_kernel<BITS, SW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
  // feature block: enough blocks to cover the machine when there are few tiles
  int fpb = 64;
  while (fpb > 8 && max_tiles * ((A.out_features + fpb - 1) / fpb) < 148 * 4) fpb >>= 1;
  const dim3 grid((unsigned)max_tiles, (unsigned)((A.out_features + fpb - 1) / fpb));
  grouped_gemv_kernel<BITS, SW><<<grid, kWarps * 32, smem, st>>>(A, fpb);
  return cudaGetLastError();
}

template <bool SW>
static cudaError_t launch_gemv_bits(int bits, const GroupedArgs& A, int64_t max_tiles,
                                    cudaStream_t st) {
  switch (bits) {
    case 2: return launch_gemv_t<2, SW>(A, max_tiles, st);
    case 3: return launch_gemv_t<3, SW>(A, max_tiles, st);
    case 4: return launch_gemv_t<4, SW>(A, max_tiles, st);
    case 5: return launch_gemv_t<5, SW>(A, max_tiles, st);
    case 6: return launch_gemv_t<6, SW>(A, max_tiles, st);
    case 8: return launch_gemv_t<8, SW>(A, max_tiles, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_grouped_gemv(const GroupedGemvDesc& d, cudaStream_t st) {
  if (d.rows_total == 0 || d.out_features == 0) return cudaSuccess;
  if (d.nseg > 1024 || d.in_features % 32 != 0 || d.in_features % d.group != 0)
    return cudaErrorInvalidValue;
  GroupedArgs A;
  A.x = (const __nv_bfloat16*)d.x;
  A.x_rows = d.x_rows;
  A.x_limit = d.x_limit;
  A.in_features = d.in_features;
  A.seg_offsets = d.seg_offsets;
  A.nseg = d.nseg;
  A.shared_seg = d.shared_seg;
  for (int i = 0; i < 2; ++i) {
    A.wa[i] = WRef{(const uint32_t*)d.wa[i].q, (const uint16_t*)d.wa[i].s,
                   (const uint16_t*)d.wa[i].b, d.wa[i].expert_rows, d.wa[i].row_offset};
    A.wb[i] = WRef{(const uint32_t*)d.wb[i].q, (const uint16_t*)d.wb[i].s,
                   (const uint16_t*)d.wb[i].b, d.wb[i].expert_rows, d.wb[i].row_offset};
  }
  A.out_features = d.out_features;
  A.group = d.group;
  A.y = (__nv_bfloat16*)d.y;
  A.y_rows = d.y_rows;
  A.y_limit = d.y_limit;
  A.ldy = d.ldy;
  A.status = d.status;
  const int64_t max_tiles = (d.rows_total + kRows - 1) / kRows + d.nseg;
  return d.swiglu ? launch_gemv_bits<true>(d.bits, A, max_tiles, st)
                  : launch_gemv_bits<false>(d.bits, A, max_tiles, st);
}

}  // namespace astro
