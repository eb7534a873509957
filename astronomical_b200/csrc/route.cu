// route.cu -- router softmax / top-K / renormalisation, one warp per token.
//
// Replaces qwen3_5_moe_route_experts (qwen3_5_moe/model/routing.rs:16-49):
// softmax(precise) over E in fp32 with probabilities rounded to the logits
// dtype, argpartition + take_along_axis for the K largest, and (norm_topk_prob)
// sum/divide.  The K winners are ordered by (probability desc, expert id asc).
//
// Reduction order (shared with the CPU restatement): lane l owns experts
// [l*C, min(E,(l+1)*C)), C = ceil(E/32), sums its exp values in index order;
// the 32 partial sums meet in a butterfly over xor distances 16..1.  The exp is
// expf_cw (common.cuh), so bf16 probabilities -- and therefore the selected ids --
// are bit-identical to the oracle given the same logits.
//
// Optionally the same warp computes the shared-expert gate logit
// bf16(x[t] . wg) (resident_execution.rs:384-388) so the block needs no extra
// pass over the hidden states for it.
#include "common.cuh"
#include "kernels.h"
#include "route_dev.cuh"

namespace astro {

template <typename T, int CMAX>
__global__ void __launch_bounds__(256, CMAX <= 16 ? 4 : 1) route_experts_kernel(
    const T* __restrict__ logits, int64_t tokens, int E, int K, int normalize,
    uint32_t* __restrict__ out_ids, T* __restrict__ out_scores,
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ wg, int H,
    __nv_bfloat16* __restrict__ gate_logit) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= tokens) return;
  // bf16(x[t] . wg): 16-byte chunks c = lane, lane + 32, ... in one fp32 fma chain
  // per lane, then a butterfly.  The token's first kGateBatch chunks per lane are
  // loaded before the routing so that their latency overlaps it (the 4 KB of
  // gate weights are shared by every warp and stay in L1).
  constexpr int kGateBatch = CMAX <= 8 ? 8 : 4;
  const int nch = gate_logit != nullptr ? H / 8 : 0;
  const uint4* xr = reinterpret_cast<const uint4*>(x + t * (int64_t)H);
  const uint4* wr = reinterpret_cast<const uint4*>(wg);
  uint4 xa[kGateBatch];
  auto load_batch = [&](int base) {
#pragma unroll
    for (int j = 0; j < kGateBatch; ++j) {
      const int c = base + j * 32 + lane;
      if (c < nch) xa[j] = xr[c];
    }
  };
  load_batch(0);
  route_token<T, CMAX>(logits + t * E, E, K, normalize, out_ids + t * K, out_scores + t * K);

  if (gate_logit != nullptr) {
    float acc = 0.0f;
    for (int base = 0; base < nch; base += 32 * kGateBatch) {
      if (base > 0) load_batch(base);
#pragma unroll
      for (int j = 0; j < kGateBatch; ++j) {
        const int c = base + j * 32 + lane;
        if (c >= nch) break;
        const uint4 w = __ldg(wr + c);
        const uint32_t av[4] = {xa[j].x, xa[j].y, xa[j].z, xa[j].w};
        const uint32_t bv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          acc = __fmaf_rn(__uint_as_float(av[i] << 16), __uint_as_float(bv[i] << 16), acc);
          acc = __fmaf_rn(__uint_as_float(av[i] & 0xffff0000u),
                          __uint_as_float(bv[i] & 0xffff0000u), acc);
        }
      }
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, m));
    if (lane == 0) gate_logit[t] = __float2bfloat16_rn(acc);
  }
}

template <typename T>
static cudaError_t launch_route_t(const void* logits, int64_t tokens, int E, int K, int normalize,
                                  uint32_t* ids, void* scores, const void* x, const void* wg,
                                  int H, void* gate_logit, cudaStream_t st) {
  if (tokens == 0) return cudaSuccess;
  const int warps = 8;
  const dim3 grid((unsigned)((tokens + warps - 1) / warps)), block(warps * 32);
  const int C = (E + 31) / 32;
  auto args = [&](auto kern) {
    kern<<<grid, block, 0, st>>>((const T*)logits, tokens, E, K, normalize, ids, (T*)scores,
                                 (const __nv_bfloat16*)x, (const __nv_bfloat16*)wg, H,
                                 (__nv_bfloat16*)gate_logit);
  };
  if (C <= 4) args(route_experts_kernel<T, 4>);
  else if (C <= 8) args(route_experts_kernel<T, 8>);
  else if (C <= 16) args(route_experts_kernel<T, 16>);
  else args(route_experts_kernel<T, 32>);
  return cudaGetLastError();
}

cudaError_t launch_route_experts(const void* logits, int dtype, int64_t tokens, int E, int K,
                                 int normalize, uint32_t* ids, void* scores, const void* x,
                                 const void* wg, int H, void* gate_logit, cudaStream_t st) {
  switch (dtype) {
    case kBF16:
      return launch_route_t<__nv_bfloat16>(logits, tokens, E, K, normalize, ids, scores, x, wg, H,
                                           gate_logit, st);
    case kF16:
      return launch_route_t<__half>(logits, tokens, E, K, normalize, ids, scores, x, wg, H,
                                    gate_logit, st);
    default:
      return launch_route_t<float>(logits, tokens, E, K, normalize, ids, scores, x, wg, H,
                                   gate_logit, st);
  }
}

// Laguna routing, one warp per token (route_token_laguna).
template <typename T, int CMAX>
__global__ void __launch_bounds__(256) route_laguna_kernel(
    const T* __restrict__ logits, int64_t tokens, int E, int K, float softcap,
    const float* __restrict__ bias, int normalize, uint32_t* __restrict__ out_ids,
    float* __restrict__ out_scores) {
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= tokens) return;
  route_token_laguna<T, CMAX>(logits + t * E, E, K, softcap, bias, normalize, out_ids + t * K,
                              out_scores + t * K);
}

template <typename T>
static cudaError_t launch_laguna_t(const void* logits, int64_t tokens, int E, int K, float softcap,
                                   const float* bias, int normalize, uint32_t* ids, float* scores,
                                   cudaStream_t st) {
  if (tokens == 0) return cudaSuccess;
  const int warps = 8;
  const dim3 grid((unsigned)((tokens + warps - 1) / warps)), block(warps * 32);
  const int C = (E + 31) / 32;
  auto run = [&](auto kern) {
    kern<<<grid, block, 0, st>>>((const T*)logits, tokens, E, K, softcap, bias, normalize, ids,
                                 scores);
  };
  if (C <= 4) run(route_laguna_kernel<T, 4>);
  else if (C <= 8) run(route_laguna_kernel<T, 8>);
  else if (C <= 16) run(route_laguna_kernel<T, 16>);
  else run(route_laguna_kernel<T, 32>);
  return cudaGetLastError();
}

cudaError_t launch_route_laguna(const void* logits, int dtype, int64_t tokens, int E, int K,
                                float softcap, const float* bias, int normalize, uint32_t* ids,
                                float* scores, cudaStream_t st) {
  switch (dtype) {
    case kBF16:
      return launch_laguna_t<__nv_bfloat16>(logits, tokens, E, K, softcap, bias, normalize, ids,
                                            scores, st);
    case kF16:
      return launch_laguna_t<__half>(logits, tokens, E, K, softcap, bias, normalize, ids, scores, st);
    default:
      return launch_laguna_t<float>(logits, tokens, E, K, softcap, bias, normalize, ids, scores, st);
  }
}

// ---------------------------------------------------------------------------
// Dense bf16 projection out[r, c] = bf16(sum_k x[r,k] w[c,k]) for the router
// when the tensor-core path is not used (portable SIMT tile kernel: 64x64
// output tile, K step 32, fp32 accumulation).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) dense_nt_simt_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w, int64_t rows,
    int cols, int depth, __nv_bfloat16* __restrict__ out, int ldo) {
  __shared__ float xs[32][65];
  __shared__ float ws[32][65];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t r0 = (int64_t)blockIdx.y * 64;
  const int c0 = blockIdx.x * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < depth; k0 += 32) {
    for (int i = threadIdx.x; i < 64 * 32; i += 256) {
      const int rr = i / 32, kk = i % 32;
      const int64_t gr = r0 + rr;
      const int gc = c0 + rr;
      xs[kk][rr] = (gr < rows && k0 + kk < depth) ? __bfloat162float(x[gr * depth + k0 + kk]) : 0.f;
      ws[kk][rr] = (gc < cols && k0 + kk < depth) ? __bfloat162float(w[(int64_t)gc * depth + k0 + kk])
                                                  : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < 32; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = xs[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = ws[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t gr = r0 + ty * 4 + i;
      const int gc = c0 + tx * 4 + j;
      if (gr < rows && gc < cols) out[gr * ldo + gc] = __float2bfloat16_rn(acc[i][j]);
    }
}

cudaError_t launch_dense_nt_simt(const void* x, const void* w, int64_t rows, int cols, int depth,
                                 void* out, int ldo, cudaStream_t st) {
  if (rows == 0 || cols == 0) return cudaSuccess;
  const dim3 grid((cols + 63) / 64, (unsigned)((rows + 63) / 64));
  dense_nt_simt_kernel<<<grid, 256, 0, st>>>((const __nv_bfloat16*)x, (const __nv_bfloat16*)w,
                                             rows, cols, depth, (__nv_bfloat16*)out, ldo);
  return cudaGetLastError();
}

}  // namespace astro
