// moe_gemm.cu -- tcgen05 grouped GEMM (placeholder until the tensor-core
// kernels land: every layer takes the CUDA-core path).
#include "moe_gemm.h"

namespace astro {

int moe_gemm_plan(const astro_moe_layer_weights& w, MoeGemmPlan* plan) {
  plan->ok = false;
  plan->w = w;
  return 0;
}
void moe_gemm_release(MoeGemmPlan& plan) { plan.ok = false; }
bool moe_gemm_enabled(const MoeGemmPlan& plan, int opt) { return plan.ok && opt >= 0; }
size_t moe_gemm_scratch_bytes() { return 256; }
cudaError_t moe_gemm_router(const MoeGemmPlan&, const void*, int64_t, void*, void*, cudaStream_t) {
  return cudaErrorNotSupported;
}
cudaError_t moe_gemm_gate_up(const MoeGemmPlan&, const void*, int64_t, const uint32_t*, void*, void*,
                             cudaStream_t) {
  return cudaErrorNotSupported;
}
cudaError_t moe_gemm_down(const MoeGemmPlan&, const void*, int64_t, const uint32_t*, void*, void*,
                          cudaStream_t) {
  return cudaErrorNotSupported;
}

}  // namespace astro
