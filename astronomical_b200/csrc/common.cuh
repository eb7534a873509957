// common.cuh -- device numerics and small utilities shared by every kernel of
// libastro_moe.  The scalar numerics (bf16 rounding, exp, sigmoid, SwiGLU) are
// evaluated with explicitly rounded intrinsics in the same step order as the
// CPU restatement, so elementwise results are bit-identical to it.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define ASTRO_DEVINL __device__ __forceinline__

namespace astro {

// dtype codes of the C ABI
enum DType : int { kBF16 = 1, kF16 = 2, kF32 = 3 };

// Device-side status word bits (written by kernels, read by the host after a
// synchronising call).  No kernel traps; a failed check records a bit and the
// kernel skips the offending access.
enum DeviceStatus : uint32_t {
  kDevOk = 0,
  kDevBadExpertId = 1u << 0,
  kDevWaitTimeout = 1u << 1,
  kDevBadShape = 1u << 2,
};

ASTRO_DEVINL float bf16_to_f32(uint16_t h) { return __uint_as_float(((uint32_t)h) << 16); }
ASTRO_DEVINL uint16_t f32_to_bf16(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
ASTRO_DEVINL float round_bf16(float f) { return bf16_to_f32(f32_to_bf16(f)); }

template <typename T> struct Num;
template <> struct Num<float> {
  static ASTRO_DEVINL float load(const float* p, int64_t i) { return p[i]; }
  static ASTRO_DEVINL void store(float* p, int64_t i, float v) { p[i] = v; }
  static ASTRO_DEVINL float round(float v) { return v; }
};
template <> struct Num<__nv_bfloat16> {
  static ASTRO_DEVINL float load(const __nv_bfloat16* p, int64_t i) {
    return __bfloat162float(p[i]);
  }
  static ASTRO_DEVINL void store(__nv_bfloat16* p, int64_t i, float v) {
    p[i] = __float2bfloat16_rn(v);
  }
  static ASTRO_DEVINL float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
};
template <> struct Num<__half> {
  static ASTRO_DEVINL float load(const __half* p, int64_t i) { return __half2float(p[i]); }
  static ASTRO_DEVINL void store(__half* p, int64_t i, float v) { p[i] = __float2half_rn(v); }
  static ASTRO_DEVINL float round(float v) { return __half2float(__float2half_rn(v)); }
};

// e^x: Cody-Waite reduction with a 12-significant-bit head of ln2, degree-7
// Taylor polynomial by Horner with fused multiply-adds, exact scaling by 2^n.
// Results below ~1.6e-38 flush to zero.  Same steps as ao_expf in the oracle.
ASTRO_DEVINL float expf_cw(float x) {
  if (x != x) return x;
  if (x > 88.72283172607421875f) return __int_as_float(0x7f800000);
  if (x < -87.0f) return 0.0f;
  const float n = rintf(__fmul_rn(x, 1.44269502162933349609375f));
  float r = __fmaf_rn(-n, 0.693115234375f, x);
  r = __fmaf_rn(-n, __uint_as_float(0x3805fdf4u), r);
  float p = __uint_as_float(0x39500d01u);
  p = __fmaf_rn(p, r, __uint_as_float(0x3ab60b61u));
  p = __fmaf_rn(p, r, __uint_as_float(0x3c088889u));
  p = __fmaf_rn(p, r, __uint_as_float(0x3d2aaaabu));
  p = __fmaf_rn(p, r, __uint_as_float(0x3e2aaaabu));
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  int ni = (int)n;
  if (ni > 127) {
    p = __fmul_rn(p, 2.0f);
    ni -= 1;
  }
  return __fmul_rn(p, __uint_as_float((uint32_t)(ni + 127) << 23));
}

// MLX sigmoid form: y = 1/(1+e^-|x|); x < 0 gives 1 - y.  The correctly rounded
// reciprocal equals the correctly rounded quotient 1/d, so this matches an IEEE
// division bit for bit.
// 1 / (1 + e^-x) in fp32 (the Laguna router's CPU formula,
// laguna/moe/router_selection.rs sigmoid); same steps as ao_sigmoid_plainf.
ASTRO_DEVINL float sigmoid_plain(float x) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf_cw(-x)));
}

// tanh(x) = s * (1 - 2 / (e^(2|x|) + 1)), s = sign(x), with the exp above (defined
// here; same steps as ao_tanhf).
ASTRO_DEVINL float tanh_cw(float x) {
  const float a = fabsf(x);
  const float t = __fsub_rn(1.0f, __fdiv_rn(2.0f, __fadd_rn(expf_cw(__fmul_rn(2.0f, a)), 1.0f)));
  return x < 0.0f ? -t : t;
}

ASTRO_DEVINL float sigmoid_mlx(float x) {
  const float y = __frcp_rn(__fadd_rn(1.0f, expf_cw(-fabsf(x))));
  return (x < 0.0f) ? __fsub_rn(1.0f, y) : y;
}

// gate * sigmoid(gate) * up with each intermediate rounded to bf16 (inputs are
// already bf16 values held in fp32).
ASTRO_DEVINL float swiglu_bf16(float g, float u) {
  const float s = round_bf16(sigmoid_mlx(g));
  const float a = round_bf16(__fmul_rn(g, s));
  return round_bf16(__fmul_rn(a, u));
}

// K order of the tcgen05 grouped GEMMs' operands inside every 8-element chunk:
// position p holds element 0,4,1,5,2,6,3,7 -- the order in which the int4 codes of
// one packed word leave the bf16 conversion, so the dequantisers need no byte
// permutes.  Token rows (B of gate/up) and activations (B of down) are stored in
// this order; a K step of 16 covers two whole chunks, and a tensor-core step sums
// its 16 products exactly before rounding, so the results are unchanged.
// perm8_bf16 reorders 8 bf16 held in a uint4 (v.x = elements 0,1 ... v.w = 6,7).
ASTRO_DEVINL uint4 perm8_bf16(uint4 v) {
  uint4 o;
  o.x = __byte_perm(v.x, v.z, 0x5410);  // (e0, e4)
  o.y = __byte_perm(v.x, v.z, 0x7632);  // (e1, e5)
  o.z = __byte_perm(v.y, v.w, 0x5410);  // (e2, e6)
  o.w = __byte_perm(v.y, v.w, 0x7632);  // (e3, e7)
  return o;
}
// position of element e (0..7) of a chunk in that order
ASTRO_DEVINL int perm8_pos(int e) { return 2 * (e & 3) + (e >> 2); }

// expf_cw for x <= 0 (and NaN) without its branches: the same steps, the
// underflow case selected at the end (the overflow and 2^128 cases cannot occur).
ASTRO_DEVINL float expf_cw_nonpos(float x) {
  const float n = rintf(__fmul_rn(x, 1.44269502162933349609375f));
  float r = __fmaf_rn(-n, 0.693115234375f, x);
  r = __fmaf_rn(-n, __uint_as_float(0x3805fdf4u), r);
  float p = __uint_as_float(0x39500d01u);
  p = __fmaf_rn(p, r, __uint_as_float(0x3ab60b61u));
  p = __fmaf_rn(p, r, __uint_as_float(0x3c088889u));
  p = __fmaf_rn(p, r, __uint_as_float(0x3d2aaaabu));
  p = __fmaf_rn(p, r, __uint_as_float(0x3e2aaaabu));
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const float v = __fmul_rn(p, __uint_as_float((uint32_t)((int)n + 127) << 23));
  return (x < -87.0f) ? 0.0f : v;
}

// Correctly rounded 1/d for d in [1, 2]: one Newton step from the hardware
// approximation with an exact FMA residual (Markstein, IBM J. Res. Dev. 34(1),
// 1990).  Checked against __frcp_rn for every fp32 in [1, 2] on the B200.
ASTRO_DEVINL float rcp_1to2(float d) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(d));
  const float e = __fmaf_rn(-d, y, 1.0f);
  return __fmaf_rn(e, y, y);
}

// swiglu_bf16 of two (gate, up) pairs given as fp32 accumulators, packed: the
// bf16 roundings of the inputs and of sigmoid as one cvt.rn.bf16x2 each, and the
// two products as mul.rn.bf16x2 (a product of two bf16 values is exact in fp32,
// so its bf16 rounding is the fp32 path's).  Bit-identical to swiglu_bf16 for
// all 2^32 (gate, up) bf16 pairs (checked on the B200).  Returns (first, second)
// in the low / high half.
ASTRO_DEVINL __nv_bfloat162 swiglu_bf16x2(__nv_bfloat162 G, __nv_bfloat162 U) {
  const uint32_t gb = *reinterpret_cast<const uint32_t*>(&G);
  const float g0 = __uint_as_float(gb << 16), g1 = __uint_as_float(gb & 0xffff0000u);
  const float y0 = rcp_1to2(__fadd_rn(1.0f, expf_cw_nonpos(-fabsf(g0))));
  const float y1 = rcp_1to2(__fadd_rn(1.0f, expf_cw_nonpos(-fabsf(g1))));
  const float s0 = g0 < 0.0f ? __fsub_rn(1.0f, y0) : y0;
  const float s1 = g1 < 0.0f ? __fsub_rn(1.0f, y1) : y1;
  return __hmul2(__hmul2(G, __floats2bfloat162_rn(s0, s1)), U);
}

ASTRO_DEVINL void record_status(uint32_t* status, uint32_t bits) {
  if (status) atomicOr(status, bits);
}

// Waits (acquire loads, polled) until *c >= target for at most limit_ns of
// %globaltimer time; on timeout records kDevWaitTimeout and returns 0.  The
// fused decode kernel's per-segment completion wait; astro_moe_wait_probe runs
// it alone so a test can make it run out.
ASTRO_DEVINL int wait_count_geq(const uint32_t* c, uint32_t target, uint32_t* status,
                                uint64_t limit_ns = 2000000000ull) {
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  uint32_t spins = 0;
  while (true) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(c) : "memory");
    if (v >= target) return 1;
    if ((++spins & 255u) == 0) {
      uint64_t t1;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
      if (t1 - t0 > limit_ns) {
        record_status(status, kDevWaitTimeout);
        return 0;
      }
    }
  }
}

ASTRO_DEVINL uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

}  // namespace astro
