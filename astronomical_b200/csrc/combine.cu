// combine.cu -- router-weighted reduction of expert rows, fused with the
// sigmoid-gated shared expert, plus the standalone elementwise stages.
//
// Sorted path: the custom kernel of sparse_experts/weighted_sum.rs:16-33
//   acc = sum_k fma(float(rows[inverse[t*K+k]][d]), float(score[t*K+k]), acc)
//   in slot order, cast to the activation dtype.
// Unsorted path (assignment count < 64): weighted_sum.rs:94-120, the product is
//   formed in the promoted dtype (bf16 x bf16 -> bf16) and summed in fp32.
// Shared combination (qwen3_5_moe/model/output_combination.rs:34-43 and the
// compiled graph runtime-integration/src/mlx_compiled_sparse_shared_expert_combination.rs):
//   out = bf16(sparse + bf16(shared * bf16(sigmoid(gate_logit)))).
// Every step rounds where MLX's dtypes round, so the result depends on the
// expert rows only through their bf16 values: deterministic, no atomics.
#include "combine_dev.cuh"
#include "common.cuh"
#include "kernels.h"

namespace astro {

// Block path: rows bf16 [*, H]; per token t, the K routed rows are found through
// `inverse` (slot -> row), the shared row is shared_base + t.  8 elements per
// thread, 16-byte loads.  The token's slot rows and scores are staged in shared
// memory first and combine_chunk issues the row loads of 8 slots before using
// any, so a token costs two dependent memory round trips, not 2K.
__global__ void __launch_bounds__(256) block_combine_kernel(
    const uint4* __restrict__ rows, const uint4* __restrict__ shared_rows,
    const uint32_t* __restrict__ inverse, const __nv_bfloat16* __restrict__ scores,
    const __nv_bfloat16* __restrict__ gate_logit, int64_t shared_base, int64_t tokens, int K,
    int H, int sorted, uint4* __restrict__ out, const float* __restrict__ scores_f32,
    int has_shared, float factor) {
  __shared__ uint32_t s_row[32];
  __shared__ float s_score[32];
  const int chunks = H >> 3;
  const bool laguna = scores_f32 != nullptr;
  for (int64_t t = blockIdx.x; t < tokens; t += gridDim.x) {
    if (threadIdx.x < K) {
      s_row[threadIdx.x] = __ldg(inverse + t * K + threadIdx.x);
      s_score[threadIdx.x] = laguna ? scores_f32[t * K + threadIdx.x]
                                    : __bfloat162float(scores[t * K + threadIdx.x]);
    }
    float sg = 0.f;
    if (gate_logit) sg = round_bf16(sigmoid_mlx(__bfloat162float(gate_logit[t])));
    __syncthreads();
    for (int c = threadIdx.x; c < chunks; c += blockDim.x)
      out[t * chunks + c] = combine_chunk(rows, shared_rows, chunks, c, s_row, s_score, K,
                                          sorted != 0, has_shared ? shared_base + t : -1, sg,
                                          laguna, factor);
    __syncthreads();  // s_row / s_score are rewritten for the next token
  }
}

cudaError_t launch_block_combine(const void* rows, const uint32_t* inverse, const void* scores,
                                 const void* gate_logit, int64_t shared_base, int64_t tokens,
                                 int K, int H, int sorted, void* out, cudaStream_t st,
                                 const float* scores_f32, int has_shared, float factor) {
  if (tokens == 0) return cudaSuccess;
  int64_t blocks = tokens < 148 * 64 ? tokens : 148 * 64;
  const int threads = (H / 8) < 256 ? ((H / 8 + 31) / 32) * 32 : 256;
  block_combine_kernel<<<(unsigned)blocks, threads, 0, st>>>(
      (const uint4*)rows, (const uint4*)rows, inverse, (const __nv_bfloat16*)scores,
      (const __nv_bfloat16*)gate_logit, shared_base, tokens, K, H, sorted, (uint4*)out,
      scores_f32, has_shared < 0 ? (gate_logit != nullptr) : has_shared, factor);
  return cudaGetLastError();
}

cudaError_t launch_block_combine_split(const void* rows, const void* shared_rows,
                                       const uint32_t* inverse, const void* scores,
                                       const void* gate_logit, int64_t tokens, int K, int H,
                                       int sorted, void* out, cudaStream_t st) {
  if (tokens == 0) return cudaSuccess;
  int64_t blocks = tokens < 148 * 64 ? tokens : 148 * 64;
  const int threads = (H / 8) < 256 ? ((H / 8 + 31) / 32) * 32 : 256;
  block_combine_kernel<<<(unsigned)blocks, threads, 0, st>>>(
      (const uint4*)rows, (const uint4*)shared_rows, inverse, (const __nv_bfloat16*)scores,
      (const __nv_bfloat16*)gate_logit, 0, tokens, K, H, sorted, (uint4*)out, nullptr,
      gate_logit != nullptr, 1.0f);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Standalone stages with the reference's dtype freedom (f32 / f16 / bf16).
// ---------------------------------------------------------------------------
template <typename TO, typename TS>
__global__ void sorted_weighted_sum_kernel(const TO* __restrict__ rows,
                                           const uint32_t* __restrict__ inverse,
                                           const TS* __restrict__ scores, int64_t tokens, int K,
                                           int64_t dim, TO* __restrict__ out) {
  const int64_t total = tokens * dim;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / dim, d = i - t * dim;
    float acc = 0.f;
    for (int k = 0; k < K; ++k) {
      const int64_t a = t * K + k;
      acc = __fmaf_rn(Num<TO>::load(rows, (int64_t)inverse[a] * dim + d), Num<TS>::load(scores, a),
                      acc);
    }
    Num<TO>::store(out, i, acc);
  }
}

template <typename TO, typename TS, typename TP>
__global__ void unsorted_weighted_sum_kernel(const TO* __restrict__ outputs,
                                             const TS* __restrict__ scores, int64_t tokens, int K,
                                             int64_t dim, TO* __restrict__ out) {
  const int64_t total = tokens * dim;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / dim, d = i - t * dim;
    float acc = 0.f;
    for (int k = 0; k < K; ++k) {
      const float p = __fmul_rn(Num<TO>::load(outputs, (t * K + k) * dim + d),
                                Num<TS>::load(scores, t * K + k));
      acc = __fadd_rn(acc, Num<TP>::round(p));
    }
    Num<TO>::store(out, i, acc);
  }
}

static unsigned grid_for(int64_t total) {
  int64_t b = (total + 255) / 256;
  if (b > 148 * 32) b = 148 * 32;
  return (unsigned)(b > 0 ? b : 1);
}

template <typename TO>
static cudaError_t sws_t(const void* rows, const uint32_t* inv, const void* scores, int sdt,
                         int64_t T, int K, int64_t D, void* out, cudaStream_t st) {
  const unsigned g = grid_for(T * D);
  if (sdt == kF32)
    sorted_weighted_sum_kernel<TO, float><<<g, 256, 0, st>>>((const TO*)rows, inv,
                                                             (const float*)scores, T, K, D, (TO*)out);
  else if (sdt == kF16)
    sorted_weighted_sum_kernel<TO, __half><<<g, 256, 0, st>>>((const TO*)rows, inv,
                                                              (const __half*)scores, T, K, D,
                                                              (TO*)out);
  else
    sorted_weighted_sum_kernel<TO, __nv_bfloat16><<<g, 256, 0, st>>>(
        (const TO*)rows, inv, (const __nv_bfloat16*)scores, T, K, D, (TO*)out);
  return cudaGetLastError();
}

cudaError_t launch_sorted_weighted_sum(const void* rows, int out_dtype, const uint32_t* inverse,
                                       const void* scores, int score_dtype, int64_t tokens, int K,
                                       int64_t dim, void* out, cudaStream_t st) {
  if (tokens * dim == 0) return cudaSuccess;
  if (out_dtype == kF32) return sws_t<float>(rows, inverse, scores, score_dtype, tokens, K, dim, out, st);
  if (out_dtype == kF16) return sws_t<__half>(rows, inverse, scores, score_dtype, tokens, K, dim, out, st);
  return sws_t<__nv_bfloat16>(rows, inverse, scores, score_dtype, tokens, K, dim, out, st);
}

template <typename TO, typename TS>
static cudaError_t uws_t(const void* rows, const void* scores, int64_t T, int K, int64_t D,
                         void* out, cudaStream_t st) {
  const unsigned g = grid_for(T * D);
  // promoted product dtype: f32 if either side is f32, the common 16-bit type otherwise
  constexpr bool f32p = std::is_same<TO, float>::value || std::is_same<TS, float>::value ||
                        !std::is_same<TO, TS>::value;
  using TP = typename std::conditional<f32p, float, TO>::type;
  unsorted_weighted_sum_kernel<TO, TS, TP><<<g, 256, 0, st>>>((const TO*)rows, (const TS*)scores,
                                                              T, K, D, (TO*)out);
  return cudaGetLastError();
}

template <typename TO>
static cudaError_t uws_s(const void* rows, const void* scores, int sdt, int64_t T, int K, int64_t D,
                         void* out, cudaStream_t st) {
  if (sdt == kF32) return uws_t<TO, float>(rows, scores, T, K, D, out, st);
  if (sdt == kF16) return uws_t<TO, __half>(rows, scores, T, K, D, out, st);
  return uws_t<TO, __nv_bfloat16>(rows, scores, T, K, D, out, st);
}

cudaError_t launch_unsorted_weighted_sum(const void* outputs, int out_dtype, const void* scores,
                                         int score_dtype, int64_t tokens, int K, int64_t dim,
                                         void* out, cudaStream_t st) {
  if (tokens * dim == 0) return cudaSuccess;
  if (out_dtype == kF32) return uws_s<float>(outputs, scores, score_dtype, tokens, K, dim, out, st);
  if (out_dtype == kF16) return uws_s<__half>(outputs, scores, score_dtype, tokens, K, dim, out, st);
  return uws_s<__nv_bfloat16>(outputs, scores, score_dtype, tokens, K, dim, out, st);
}

template <typename T>
__global__ void combine_shared_kernel(const T* __restrict__ sparse, const T* __restrict__ shared,
                                      const T* __restrict__ gate, int64_t tokens, int64_t dim,
                                      T* __restrict__ out) {
  const int64_t total = tokens * dim;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / dim;
    const float g = Num<T>::round(sigmoid_mlx(Num<T>::load(gate, t)));
    const float prod = Num<T>::round(__fmul_rn(Num<T>::load(shared, i), g));
    Num<T>::store(out, i, __fadd_rn(Num<T>::load(sparse, i), prod));
  }
}

cudaError_t launch_combine_shared(const void* sparse, const void* shared, const void* gate,
                                  int dtype, int64_t tokens, int64_t dim, void* out,
                                  cudaStream_t st) {
  if (tokens * dim == 0) return cudaSuccess;
  const unsigned g = grid_for(tokens * dim);
  if (dtype == kF32)
    combine_shared_kernel<float><<<g, 256, 0, st>>>((const float*)sparse, (const float*)shared,
                                                    (const float*)gate, tokens, dim, (float*)out);
  else if (dtype == kF16)
    combine_shared_kernel<__half><<<g, 256, 0, st>>>((const __half*)sparse, (const __half*)shared,
                                                     (const __half*)gate, tokens, dim, (__half*)out);
  else
    combine_shared_kernel<__nv_bfloat16><<<g, 256, 0, st>>>(
        (const __nv_bfloat16*)sparse, (const __nv_bfloat16*)shared, (const __nv_bfloat16*)gate,
        tokens, dim, (__nv_bfloat16*)out);
  return cudaGetLastError();
}

__global__ void swiglu_kernel(const __nv_bfloat16* __restrict__ gate,
                              const __nv_bfloat16* __restrict__ up, int64_t n,
                              __nv_bfloat16* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = __float2bfloat16_rn(swiglu_bf16(__bfloat162float(gate[i]), __bfloat162float(up[i])));
}

cudaError_t launch_swiglu(const void* gate, const void* up, int64_t n, void* out, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  swiglu_kernel<<<grid_for(n), 256, 0, st>>>((const __nv_bfloat16*)gate,
                                             (const __nv_bfloat16*)up, n, (__nv_bfloat16*)out);
  return cudaGetLastError();
}

// Numerics probe used by the parity tests: exp / sigmoid on the device.
__global__ void numerics_probe_kernel(const float* __restrict__ x, int64_t n, int which,
                                      float* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = which == 0 ? expf_cw(x[i]) : sigmoid_mlx(x[i]);
}

cudaError_t launch_numerics_probe(const float* x, int64_t n, int which, float* out,
                                  cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  numerics_probe_kernel<<<grid_for(n), 256, 0, st>>>(x, n, which, out);
  return cudaGetLastError();
}

}  // namespace astro
