// numerics_check.cu -- exhaustive device checks of the packed arithmetic the
// tcgen05 gate/up epilogue uses in place of the scalar, oracle-matching steps
// (common.cuh): each kernel walks its whole input space on the GPU and counts
// the inputs where the fast form and the reference form differ bit-wise (two
// NaNs count as equal).  Test hook behind astro_moe_numerics_check.
#include <cuda_bf16.h>

#include "astro_moe.h"
#include "common.cuh"
#include "kernels.h"

namespace astro {
namespace {

ASTRO_DEVINL bool same_f32(uint32_t a, uint32_t b) {
  if (a == b) return true;
  return (a & 0x7fffffffu) > 0x7f800000u && (b & 0x7fffffffu) > 0x7f800000u;
}
ASTRO_DEVINL bool same_bf16(uint32_t a, uint32_t b) {
  a &= 0xffffu;
  b &= 0xffffu;
  if (a == b) return true;
  return (a & 0x7fffu) > 0x7f80u && (b & 0x7fffu) > 0x7f80u;
}

ASTRO_DEVINL void miss(unsigned long long* count, uint32_t* first, uint64_t i) {
  atomicAdd(count, 1ull);
  atomicMin(first, (uint32_t)(i > 0xffffffffull ? 0xffffffffull : i));
}

// 0: rcp_1to2(d) == __frcp_rn(d) for every fp32 d in [1, 2]
// 1: expf_cw_nonpos(x) == expf_cw(x) for every fp32 x with the sign bit set, and +0
// 2: mul.rn.bf16x2 == bf16(fp32 product) for every pair of bf16
// 3: swiglu_bf16x2 == swiglu_bf16 for every (gate, up) pair of bf16, the second
//    lane fed fp32 accumulators that differ from the first below bf16 precision
//    (including exact ties)
__global__ void numerics_check_kernel(int which, unsigned long long* count, uint32_t* first) {
  const uint64_t n = which == 0 ? (1ull << 23) + 1 : which == 1 ? (1ull << 31) + 1 : 1ull << 32;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    if (which == 0) {
      const float d = __uint_as_float(0x3f800000u + (uint32_t)i);
      if (!same_f32(__float_as_uint(rcp_1to2(d)), __float_as_uint(__frcp_rn(d)))) miss(count, first, i);
    } else if (which == 1) {
      const float x = (i == (1ull << 31)) ? 0.0f : __uint_as_float(0x80000000u | (uint32_t)i);
      if (!same_f32(__float_as_uint(expf_cw_nonpos(x)), __float_as_uint(expf_cw(x))))
        miss(count, first, i);
    } else if (which == 2) {
      const uint16_t a = (uint16_t)(i >> 16), b = (uint16_t)i;
      const __nv_bfloat162 p =
          __hmul2(__bfloat162bfloat162(__ushort_as_bfloat16(a)), __bfloat162bfloat162(__ushort_as_bfloat16(b)));
      const uint16_t want = f32_to_bf16(__fmul_rn(bf16_to_f32(a), bf16_to_f32(b)));
      if (!same_bf16(__bfloat16_as_ushort(p.x), want)) miss(count, first, i);
    } else {
      const uint16_t gh = (uint16_t)(i >> 16), uh = (uint16_t)i;
      const float g = bf16_to_f32(gh), u = bf16_to_f32(uh);
      const float g1 = __uint_as_float(__float_as_uint(g) + 0x3fffu * (uint32_t)((i >> 7) & 1));
      const float u1 = __uint_as_float(__float_as_uint(u) + 0x4000u * (uint32_t)((i >> 9) & 1));
      const __nv_bfloat162 o =
          swiglu_bf16x2(__floats2bfloat162_rn(g, g1), __floats2bfloat162_rn(u, u1));
      const uint16_t w0 = f32_to_bf16(swiglu_bf16(round_bf16(g), round_bf16(u)));
      const uint16_t w1 = f32_to_bf16(swiglu_bf16(round_bf16(g1), round_bf16(u1)));
      if (!same_bf16(__bfloat16_as_ushort(o.x), w0) || !same_bf16(__bfloat16_as_ushort(o.y), w1))
        miss(count, first, i);
    }
  }
}

}  // namespace
}  // namespace astro

extern "C" int astro_moe_numerics_check(int32_t which, unsigned long long* mismatches,
                                        uint32_t* first_index, void* stream) {
  if (which < 0 || which > 3)
    return astro::set_last_error(ASTRO_MOE_ERR_INVALID_ARGUMENT, "numerics_check: `which` must be 0..3");
  if (!mismatches || !first_index)
    return astro::set_last_error(ASTRO_MOE_ERR_INVALID_ARGUMENT,
                                 "numerics_check: mismatches and first_index are required");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(mismatches, 0, sizeof(unsigned long long), st);
  if (e == cudaSuccess) e = cudaMemsetAsync(first_index, 0xff, sizeof(uint32_t), st);
  if (e == cudaSuccess) {
    astro::numerics_check_kernel<<<148 * 8, 256, 0, st>>>(which, mismatches, first_index);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return astro::set_last_error(ASTRO_MOE_ERR_CUDA, cudaGetErrorString(e));
  return ASTRO_MOE_OK;
}
