// moe_gemm.h -- interface of the tcgen05 grouped GEMM path (moe_gemm.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "astro_moe.h"

namespace astro {

// Per-layer tensor-core plan: TMA descriptors over the borrowed MLX-layout
// weights.  `ok` is false when the layer's profile is not handled by the
// tensor-core kernels (anything but 4-bit, group 64, bf16 scales).
struct MoeGemmPlan {
  bool ok = false;
  void* dev = nullptr;  // device copy of the kernel parameter blocks
  astro_moe_layer_weights w{};
};

// The routed experts of a paged layer: a device pool of `slots` pages of
// page_bytes each; inside a page, projection m (gate, up, down) has its packed
// codes at off_q[m], scales at off_s[m] and biases at off_b[m].  The kernels
// then read routed segment e from slot slot_of[e] (a device table passed per
// call).
struct PagedStacks {
  const char* pool = nullptr;
  int64_t slots = 0, page_bytes = 0;
  int64_t off_q[3] = {0, 0, 0}, off_s[3] = {0, 0, 0}, off_b[3] = {0, 0, 0};
};

// router_rows > 0: the router projection has this many output rows (all experts
// of an expert-parallel layer) while w.experts counts the stacked local experts.
// paged != nullptr: the routed experts are pages of that pool (w's gate, up and
// down are ignored).
int moe_gemm_plan(const astro_moe_layer_weights& w, MoeGemmPlan* plan, int router_rows = 0,
                  const PagedStacks* paged = nullptr);
void moe_gemm_release(MoeGemmPlan& plan);
bool moe_gemm_enabled(const MoeGemmPlan& plan, int use_tensor_cores_option);
size_t moe_gemm_scratch_bytes();

cudaError_t moe_gemm_router(const MoeGemmPlan& plan, const void* x, int64_t tokens, void* logits,
                            void* scratch, uint32_t* status, cudaStream_t st);
// slot_of: a paged plan's device table routed segment -> slot (required there)
cudaError_t moe_gemm_gate_up(const MoeGemmPlan& plan, const void* states, int64_t rows,
                             const uint32_t* offsets, void* act, void* scratch, uint32_t* status,
                             cudaStream_t st, const uint32_t* slot_of = nullptr);
cudaError_t moe_gemm_down(const MoeGemmPlan& plan, const void* act, int64_t rows,
                          const uint32_t* offsets, void* yrows, void* scratch, uint32_t* status,
                          cudaStream_t st, const uint32_t* slot_of = nullptr);

}  // namespace astro
