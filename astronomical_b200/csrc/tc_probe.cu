// tc_probe.cu -- one tensor-core accumulation, exposed for checking its arithmetic.
//
// The CPU restatement of the MoE block (oracle/) reproduces the GPU kernels bit
// for bit by modelling the tensor cores' fp32 accumulation (ao_tc_step); these
// kernels run D = C + A.B^T on given operands with the two instructions the
// library's GEMMs use (tcgen05.mma kind::f16 with A and B in shared memory, and
// mma.sync m16n8k16), so a test can hold that model against the hardware on any
// inputs.  Not on any hot path.
#include <cstdio>

#include "astro_moe.h"
#include "common.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace astro {
namespace {

constexpr int kTileA = 128 * 128;  // bytes of one 64-wide K tile of A (128 rows)

// byte offset of element (row r, k) in a K-major tile of 128-byte rows with the
// 128-byte swizzle (8-row atoms of 1024 bytes; 16-byte chunk c of row r at c ^ (r & 7))
__device__ __forceinline__ int swz_off(int r, int k) {
  const int atom = r >> 3, rr = r & 7, chunk = k >> 3;
  return atom * 1024 + rr * 128 + ((chunk ^ rr) << 4) + ((k & 7) << 1);
}

// One problem per CTA (128 threads): A [128][K], B [N][K] staged in shared
// memory, C written into the TMEM accumulator (use_c), K/16 MMAs in order.
__global__ void __launch_bounds__(128) tc_probe_kernel(const uint16_t* A, const uint16_t* B,
                                                       const float* C, float* D, int N, int nk16,
                                                       int use_c, uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u);
  __shared__ uint64_t bar;
  __shared__ uint32_t tbase;
  __shared__ int abort_flag;
  const int prob = blockIdx.x;
  const int K = nk16 * 16;
  const int ntiles = (K + 63) / 64;
  uint8_t* sa = smem;                    // ntiles x 16 KB
  uint8_t* sb = smem + ntiles * kTileA;  // ntiles x N x 128 B
  const uint16_t* a = A + (size_t)prob * 128 * K;
  const uint16_t* b = B + (size_t)prob * N * K;
  for (int i = threadIdx.x; i < 128 * ntiles * 64; i += 128) {
    const int r = i / (ntiles * 64), kk = i % (ntiles * 64);
    *reinterpret_cast<uint16_t*>(sa + (kk / 64) * kTileA + swz_off(r, kk % 64)) =
        kk < K ? a[r * K + kk] : 0;
  }
  for (int i = threadIdx.x; i < N * ntiles * 64; i += 128) {
    const int r = i / (ntiles * 64), kk = i % (ntiles * 64);
    *reinterpret_cast<uint16_t*>(sb + (kk / 64) * N * 128 + swz_off(r, kk % 64)) =
        kk < K ? b[r * K + kk] : 0;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    abort_flag = 0;
    tc::fence_mbar_init();
  }
  if (warp == 0) tc::tmem_alloc(&tbase, 32);
  tc::fence_proxy_async_smem();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tm = tbase;
  const int row = warp * 32 + lane;
  const uint32_t lanes = (uint32_t)(warp * 32) << 16;
  if (use_c) {
    uint32_t v[32];
    for (int c = 0; c < 32; ++c)
      v[c] = c < N ? __float_as_uint(C[((size_t)prob * 128 + row) * N + c]) : 0u;
    tc::tmem_st32(tm + lanes, v);
    tc::tmem_st_wait();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (threadIdx.x == 0) {
    const uint32_t idesc = tc::idesc_bf16(128, N);
    for (int k16 = 0; k16 < nk16; ++k16) {
      const int t = k16 >> 2, s = k16 & 3;
      const uint64_t ad = tc::sdesc_sw128(tc::smem_u32(sa + t * kTileA)) + (uint64_t)(2 * s);
      const uint64_t bd = tc::sdesc_sw128(tc::smem_u32(sb + t * N * 128)) + (uint64_t)(2 * s);
      tc::mma_bf16(tm, ad, bd, idesc, (k16 > 0 || use_c) ? 1u : 0u);
    }
    tc::mma_commit(&bar);
  }
  __syncwarp();
  const bool ok = tc::mbar_wait(&bar, 0, (volatile int*)&abort_flag, status, 1000000000ull);
  tc::tc_fence_after();
  if (ok) {
    uint32_t v0[16], v1[16];
    tc::tmem_ld16(tm + lanes, v0);
    tc::tmem_ld_wait16(v0);
    tc::tmem_ld16(tm + lanes + 16, v1);
    tc::tmem_ld_wait16(v1);
    for (int c = 0; c < N && c < 16; ++c)
      D[((size_t)prob * 128 + row) * N + c] = __uint_as_float(v0[c]);
    for (int c = 16; c < N; ++c) D[((size_t)prob * 128 + row) * N + c] = __uint_as_float(v1[c - 16]);
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_relinquish();
    tc::tmem_dealloc(tm, 32);
  }
}

// One problem per warp: A [16][K], B [8][K] (B^T), C/D [16][8]; K/16 mma.sync in order.
__global__ void mma_probe_kernel(const uint16_t* A, const uint16_t* B, const float* C, float* D,
                                 int P, int nk16) {
  const int prob = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  if (prob >= P) return;
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int K = nk16 * 16;
  const uint16_t* a = A + (size_t)prob * 16 * K;
  const uint16_t* b = B + (size_t)prob * 8 * K;
  const float* c = C + (size_t)prob * 128;
  float d0 = c[g * 8 + 2 * t], d1 = c[g * 8 + 2 * t + 1];
  float d2 = c[(g + 8) * 8 + 2 * t], d3 = c[(g + 8) * 8 + 2 * t + 1];
  auto pk = [](uint16_t lo, uint16_t hi) { return (uint32_t)lo | ((uint32_t)hi << 16); };
  for (int kb = 0; kb < nk16; ++kb) {
    const int k0 = kb * 16 + 2 * t;
    const uint32_t a0 = pk(a[g * K + k0], a[g * K + k0 + 1]);
    const uint32_t a1 = pk(a[(g + 8) * K + k0], a[(g + 8) * K + k0 + 1]);
    const uint32_t a2 = pk(a[g * K + k0 + 8], a[g * K + k0 + 9]);
    const uint32_t a3 = pk(a[(g + 8) * K + k0 + 8], a[(g + 8) * K + k0 + 9]);
    const uint32_t b0 = pk(b[g * K + k0], b[g * K + k0 + 1]);
    const uint32_t b1 = pk(b[g * K + k0 + 8], b[g * K + k0 + 9]);
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d0), "+f"(d1), "+f"(d2), "+f"(d3)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  float* d = D + (size_t)prob * 128;
  d[g * 8 + 2 * t] = d0;
  d[g * 8 + 2 * t + 1] = d1;
  d[(g + 8) * 8 + 2 * t] = d2;
  d[(g + 8) * 8 + 2 * t + 1] = d3;
}

}  // namespace
}  // namespace astro

using namespace astro;

extern "C" int astro_moe_tensor_core_probe(int32_t instruction, const void* a, const void* b,
                                           const float* c, float* d, int64_t problems, int32_t n,
                                           int32_t k16, int32_t accumulate, uint32_t* device_status,
                                           void* stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (problems < 0 || problems > 65535 || k16 < 1)
    return set_last_error(ASTRO_MOE_ERR_INVALID_ARGUMENT, "tensor-core probe: invalid shape");
  if (instruction == 0 && ((n != 16 && n != 32) || k16 > 16 || !device_status))
    return set_last_error(ASTRO_MOE_ERR_INVALID_ARGUMENT,
                          "tensor-core probe: tcgen05 takes n in {16, 32}, k16 <= 16 and a status word");
  if (instruction == 1 && (n != 8 || k16 > 64))
    return set_last_error(ASTRO_MOE_ERR_INVALID_ARGUMENT,
                          "tensor-core probe: mma.sync takes n = 8 and k16 <= 64");
  if (instruction != 0 && instruction != 1)
    return set_last_error(ASTRO_MOE_ERR_INVALID_ARGUMENT, "tensor-core probe: unknown instruction");
  if (problems == 0) return ASTRO_MOE_OK;
  if (!a || !b || !c || !d)
    return set_last_error(ASTRO_MOE_ERR_INVALID_ARGUMENT, "tensor-core probe: null array");
  if (instruction == 0) {
    const int ntiles = (k16 * 16 + 63) / 64;
    const int smem = ntiles * kTileA + ntiles * n * 128 + 1024;
    cudaFuncSetAttribute(tc_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    tc_probe_kernel<<<(unsigned)problems, 128, smem, st>>>(
        (const uint16_t*)a, (const uint16_t*)b, c, d, n, k16, accumulate ? 1 : 0, device_status);
  } else {
    const int threads = 256;
    const int64_t blocks = (problems * 32 + threads - 1) / threads;
    mma_probe_kernel<<<(unsigned)blocks, threads, 0, st>>>((const uint16_t*)a, (const uint16_t*)b,
                                                           c, d, (int)problems, k16);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    char buf[256];
    snprintf(buf, sizeof(buf), "tensor-core probe: %s", cudaGetErrorString(e));
    return set_last_error(ASTRO_MOE_ERR_CUDA, buf);
  }
  return ASTRO_MOE_OK;
}
