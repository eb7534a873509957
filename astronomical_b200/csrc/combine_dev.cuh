// combine_dev.cuh -- one 8-element chunk of the block's weighted combine,
// shared by the combine kernel and the fused decode kernel.
//
// Sorted (weighted_sum.rs:16-33): acc = sum_k fma(float(row_k), score_k, acc) in
// slot order.  Unsorted (weighted_sum.rs:94-120): acc += bf16(row_k * score_k).
// With the shared expert (output_combination.rs:34-43):
//   out = bf16(bf16(acc) + bf16(shared * sg)),  sg = bf16(sigmoid(gate_logit)).
// Laguna (laguna/moe/resident.rs:60-100; fp32 scores, so the unsorted product
// stays fp32): routed = bf16(bf16(acc) * factor) with factor already rounded to
// bf16 (multiply_scalar casts the scalar to the array's dtype), then
//   out = bf16(routed + shared) with an ungated shared expert.
#pragma once

#include "common.cuh"

namespace astro {

constexpr int kCombineSlots = 8;  // slot rows whose loads are issued together

// rows: bf16 expert rows as uint4 [*, chunks]; slot_rows / slot_scores: the
// token's K (row, score) pairs; the shared expert's row is shared_rows[shared_row]
// (shared_row < 0: no shared expert).  Row loads bypass L1 (the rows may have
// been written earlier in the same kernel).
ASTRO_DEVINL uint4 combine_chunk(const uint4* rows, const uint4* shared_rows, int chunks, int c,
                                 const uint32_t* slot_rows, const float* slot_scores, int K,
                                 bool sorted, int64_t shared_row, float sg, bool laguna = false,
                                 float factor = 1.0f) {
  uint4 sh = make_uint4(0, 0, 0, 0);
  if (shared_row >= 0) sh = __ldcg(shared_rows + shared_row * chunks + c);
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
  for (int k0 = 0; k0 < K; k0 += kCombineSlots) {
    uint4 v[kCombineSlots];
#pragma unroll
    for (int kk = 0; kk < kCombineSlots; ++kk)
      if (k0 + kk < K) v[kk] = __ldcg(rows + (int64_t)slot_rows[k0 + kk] * chunks + c);
#pragma unroll
    for (int kk = 0; kk < kCombineSlots; ++kk) {
      if (k0 + kk >= K) break;
      const float s = slot_scores[k0 + kk];
      const uint32_t vv[4] = {v[kk].x, v[kk].y, v[kk].z, v[kk].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float lo = __uint_as_float(vv[j] << 16), hi = __uint_as_float(vv[j] & 0xffff0000u);
        if (sorted) {
          acc[2 * j] = __fmaf_rn(lo, s, acc[2 * j]);
          acc[2 * j + 1] = __fmaf_rn(hi, s, acc[2 * j + 1]);
        } else if (laguna) {
          acc[2 * j] = __fadd_rn(acc[2 * j], __fmul_rn(lo, s));
          acc[2 * j + 1] = __fadd_rn(acc[2 * j + 1], __fmul_rn(hi, s));
        } else {
          acc[2 * j] = __fadd_rn(acc[2 * j], round_bf16(__fmul_rn(lo, s)));
          acc[2 * j + 1] = __fadd_rn(acc[2 * j + 1], round_bf16(__fmul_rn(hi, s)));
        }
      }
    }
  }
  uint32_t o[4];
  if (laguna) {
    const uint32_t vv[4] = {sh.x, sh.y, sh.z, sh.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float y0 = round_bf16(__fmul_rn(round_bf16(acc[2 * j]), factor));
      float y1 = round_bf16(__fmul_rn(round_bf16(acc[2 * j + 1]), factor));
      if (shared_row >= 0) {
        y0 = __fadd_rn(y0, __uint_as_float(vv[j] << 16));
        y1 = __fadd_rn(y1, __uint_as_float(vv[j] & 0xffff0000u));
      }
      o[j] = (uint32_t)f32_to_bf16(y0) | ((uint32_t)f32_to_bf16(y1) << 16);
    }
  } else if (shared_row >= 0) {
    const uint32_t vv[4] = {sh.x, sh.y, sh.z, sh.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float lo = __uint_as_float(vv[j] << 16), hi = __uint_as_float(vv[j] & 0xffff0000u);
      const float y0 = __fadd_rn(round_bf16(acc[2 * j]), round_bf16(__fmul_rn(lo, sg)));
      const float y1 = __fadd_rn(round_bf16(acc[2 * j + 1]), round_bf16(__fmul_rn(hi, sg)));
      o[j] = (uint32_t)f32_to_bf16(y0) | ((uint32_t)f32_to_bf16(y1) << 16);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      o[j] = (uint32_t)f32_to_bf16(acc[2 * j]) | ((uint32_t)f32_to_bf16(acc[2 * j + 1]) << 16);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

}  // namespace astro
