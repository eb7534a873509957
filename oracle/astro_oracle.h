/*
 * astro_oracle.h -- CPU restatement of Astronomical's sorted mixture-of-experts
 * block (the Qwen3.5-MoE resident path), used ONLY as the parity checker by the
 * tests, by __graft_entry__.smoke() and by the CPU baseline leg of bench.py.
 * Nothing in the product links or calls this library.
 *
 * Every function follows the reference's op sequence (paths relative to the
 * reference project root) with the dtype boundaries of the MLX 0.32.1 calls the
 * reference makes.  Where MLX leaves a choice open (reduction order, tie order
 * of argpartition, rounding of the dequantised weight) the choice is fixed here
 * and the CUDA kernels follow the same definition; each such choice is marked
 * "defined here" in the comments.
 *
 * Parity pins: the known-answer tests of the reference (routing, sort, inverse
 * permutation, weighted sum, affine qmm / gather_qmm, SwiGLU) are ported as data
 * in tests/test_oracle_kat.py and checked against these functions.
 */
#ifndef ASTRO_ORACLE_H
#define ASTRO_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes, identical to ASTRO_MOE_DTYPE_* in include/astro_moe.h */
enum { AO_BF16 = 1, AO_F16 = 2, AO_F32 = 3 };

/* status codes, identical to ASTRO_MOE_* in include/astro_moe.h */
enum {
  AO_OK = 0,
  AO_ERR_INVALID_ARGUMENT = 1,
  AO_ERR_DUPLICATE_SLOT = 8,
  AO_ERR_OUT_OF_RANGE_SLOT = 9
};

/* ---- scalar numerics shared (step for step) with the CUDA kernels ---- */
uint16_t ao_f32_to_bf16(float f);         /* round to nearest even */
float ao_bf16_to_f32(uint16_t h);
float ao_expf(float x);                   /* Cody-Waite reduction + Taylor(7) */
float ao_sigmoidf(float x);               /* MLX's |x| form, see .c */
void ao_expf_batch(const float* x, int64_t n, float* out);

/* a1: router / shared-gate projection, bf16 x bf16 -> fp32 accumulate -> bf16.
 * qwen3_5_moe/model/forward.rs:52-93 (matmul with the transposed gate weight). */
void ao_matmul_bf16_nt(const uint16_t* x, const uint16_t* w, int64_t rows, int64_t cols,
                       int64_t depth, uint16_t* out);

/* a2: qwen3_5_moe_route_experts, qwen3_5_moe/model/routing.rs:16-49. */
int ao_route_experts(const void* logits, int dtype, int64_t tokens, int experts, int top_k,
                     int normalize, uint32_t* out_ids, void* out_scores);

/* a3: sort_expert_assignments, sparse_experts/assignment_sort.rs:36-97.
 * expert_offsets has experts+1 entries (exclusive scan of the histogram). */
int ao_sort_expert_assignments(const uint32_t* ids, int64_t tokens, int top_k, int experts,
                               uint32_t* sorted_order, uint32_t* inverse_order,
                               uint32_t* sorted_ids, uint32_t* sorted_tokens,
                               uint32_t* expert_offsets);

/* sparse_experts/assignment_permutation.rs:10-41 */
int ao_invert_assignment_order(const uint32_t* sorted_order, int64_t n, uint32_t* inverse_order);

/* MLX affine dequantize (w = scale*q + bias), rows x in_features -> bf16.
 * runtime-integration/src/mlx_quantized_operations.rs:5-47. */
int ao_dequantize_affine(const uint32_t* packed, const uint16_t* scales, const uint16_t* biases,
                         int64_t rows, int in_features, int group, int bits, uint16_t* out);

/* a4/a6: gather_qmm (transpose=true), mlx_quantized_operations.rs:100-157.
 * Output row n = x[lhs_rows[n]] . dequant(W[rhs_experts[n]])^T.  lhs_rows NULL
 * means identity; rhs_experts NULL means expert 0 (quantized_matmul, :49-98). */
int ao_gather_qmm(const uint16_t* x, const uint32_t* lhs_rows, const uint32_t* rhs_experts,
                  int64_t n_rows, int in_features, const uint32_t* packed,
                  const uint16_t* scales, const uint16_t* biases, int experts,
                  int out_features, int group, int bits, uint16_t* y);

/* a5: compiled SwiGLU, runtime-integration/src/mlx_compiled_swiglu.rs:44-89 */
void ao_swiglu(const uint16_t* gate, const uint16_t* up, int64_t n, uint16_t* out);

/* a7: sorted weighted sum (custom kernel source sparse_experts/weighted_sum.rs:16-33). */
int ao_sorted_expert_weighted_sum(const void* sorted_outputs, int out_dtype,
                                  const uint32_t* inverse_order, const void* scores,
                                  int score_dtype, int64_t tokens, int top_k, int64_t dim,
                                  void* out);

/* a7: unsorted weighted sum, sparse_experts/weighted_sum.rs:94-120 */
int ao_unsorted_expert_weighted_sum(const void* outputs, int out_dtype, const void* scores,
                                    int score_dtype, int64_t tokens, int top_k, int64_t dim,
                                    void* out);

/* a8: sparse + sigmoid(gate) * shared, qwen3_5_moe/model/output_combination.rs:34-43 */
void ao_combine_sparse_and_shared(const void* sparse, const void* shared, const void* gate_logits,
                                  int dtype, int64_t tokens, int64_t dim, void* out);

/* a9: the whole resident block (qwen3_5_moe/model/resident_execution.rs:70-143 and
 * :352-400).  Weights are in MLX layout: packed [E, out, in*bits/32] u32, scales and
 * biases [E, out, in/group] bf16.  shared_intermediate == 0 means no shared expert. */
typedef struct {
  int hidden, experts, top_k, intermediate, shared_intermediate, group, bits, normalize;
  const uint16_t* router_w;                                  /* [E, H] bf16 */
  const uint32_t* gate_q; const uint16_t* gate_s; const uint16_t* gate_b; /* [E, I, .] */
  const uint32_t* up_q;   const uint16_t* up_s;   const uint16_t* up_b;   /* [E, I, .] */
  const uint32_t* down_q; const uint16_t* down_s; const uint16_t* down_b; /* [E, H, .] */
  const uint32_t* sgate_q; const uint16_t* sgate_s; const uint16_t* sgate_b; /* [Is, .] */
  const uint32_t* sup_q;   const uint16_t* sup_s;   const uint16_t* sup_b;   /* [Is, .] */
  const uint32_t* sdown_q; const uint16_t* sdown_s; const uint16_t* sdown_b; /* [H, .] */
  const uint16_t* shared_gate_w;                             /* [1, H] bf16 */
} ao_block_weights;

/* Runs the block for the tokens listed in token_subset (NULL = all tokens).  The
 * sorted/unsorted decision uses the FULL assignment count tokens*top_k
 * (routing.rs:13, resident_execution.rs:86-96), so a subset run reproduces the
 * rows of the full run.  logits_override (bf16 [tokens, E], may be NULL) replaces
 * the router projection.  ids/scores/out are indexed by the subset position. */
int ao_moe_block_forward(const ao_block_weights* w, const uint16_t* x, int64_t tokens,
                         const int64_t* token_subset, int64_t n_subset,
                         const uint16_t* logits_override, uint16_t* out,
                         uint32_t* out_ids, uint16_t* out_scores, int num_threads);

/* Same, also returning the two bf16 terms of the final addition (the routed
 * weighted sum and the gated shared-expert output; zero without a shared
 * expert), used to scale output tolerances. */
int ao_moe_block_forward_terms(const ao_block_weights* w, const uint16_t* x, int64_t tokens,
                               const int64_t* token_subset, int64_t n_subset,
                               const uint16_t* logits_override, uint16_t* out,
                               uint32_t* out_ids, uint16_t* out_scores, uint16_t* out_sparse,
                               uint16_t* out_shared_gated, int num_threads);

#ifdef __cplusplus
}
#endif
#endif
