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

/* Accumulation arithmetic of one dot product (fp32 accumulator, bf16-valued
 * operands).  MLX leaves the order of a projection's reduction open, so it is
 * defined here: AO_DOT_SEQ is the canonical order (sequential fmaf in k order);
 * every other mode is the exact arithmetic of one CUDA kernel of the library,
 * so that each GPU path can be checked bit for bit:
 *   AO_DOT_TC           tensor-core steps over 16 consecutive k, in k order
 *                       (tcgen05.mma kind::f16: the grouped GEMMs and the router
 *                       GEMM); the step is ao_tc_step below;
 *   AO_DOT_TC_QUARTERS  the fused decode kernel's warp tiles (mma.sync): four K
 *                       quarters, each a chain of tensor-core steps over the
 *                       16-element sets {16c + 8(s>>1) + 2(s&1) + {0,1,4,5}} of
 *                       each 64-wide group (s = 0..3), the quarters then added
 *                       in order;
 *   AO_DOT_SLICES8      the router GEMV / fused router: 8 K slices, lane l of 32
 *                       taking 8-element vectors l, l+32, .. of a slice (fmaf in
 *                       order), a butterfly over the lanes, the slices added in
 *                       order;
 *   AO_DOT_LANES8       the routing kernel's shared-gate dot: lane l of 32 taking
 *                       8-element chunks l, l+32, .. (fmaf in order), butterfly;
 *   AO_DOT_DECODE32/16  the decode GEMVs: L = 32 (gate/up) or 16 (down) lanes,
 *                       lane l taking elements [32L s + 32 l, +32) of step s as
 *                       four chunks of 8 in the order 0,4,1,5,2,6,3,7, butterfly;
 *   AO_DOT_CHUNK32      the grouped GEMV: L = min(32, largest power of two <=
 *                       K/32) lanes, lane l taking 32-element chunks l, l+L, ..
 *                       in order, butterfly.
 * A butterfly over L lanes adds partial[l] + partial[l ^ m] for m = L/2 .. 1. */
enum {
  AO_DOT_SEQ = 0,
  AO_DOT_TC = 1,
  AO_DOT_TC_QUARTERS = 2,
  AO_DOT_SLICES8 = 3,
  AO_DOT_LANES8 = 4,
  AO_DOT_DECODE32 = 5,
  AO_DOT_DECODE16 = 6,
  AO_DOT_CHUNK32 = 7
};

/* One kind::f16 tensor-core accumulation step with bf16 operands and an fp32
 * accumulator, D = C + sum_k a_k b_k over 16 products, as measured on B200 for
 * both tcgen05.mma and mma.sync (tests/test_gpu_tensor_core_model.py checks it
 * against the hardware, tests/test_oracle_tc_model.py against recorded steps):
 * the products are exact; with emax the largest of e(a_k) + e(b_k) over the
 * non-zero products and e(C) (e = the unbiased exponent of the operand), every
 * product and C are truncated toward zero to a multiple of 2^(emax - 25),
 * summed exactly, and the sum is rounded toward zero to 24 significant bits.
 * Operands are normal or zero. */
float ao_tc_step(float c, const float* a, const float* b);

/* out[i] = the chain of n/16 tensor-core steps over a[i][.] and b[i][.] (k in
 * order) starting from c[i] (c NULL: from zero), for `count` independent dots. */
void ao_tc_chain_batch(const float* a, const float* b, const float* c, int64_t count, int64_t n,
                       float* out);

/* a = [n], b = [n] (bf16 values held in floats); returns the fp32 accumulator. */
float ao_dot(const float* a, const float* b, int64_t n, int mode);

/* a1: router / shared-gate projection, bf16 x bf16 -> fp32 accumulate -> bf16.
 * qwen3_5_moe/model/forward.rs:52-93 (matmul with the transposed gate weight).
 * ao_matmul_bf16_nt_mode takes the accumulation mode (ao_matmul_bf16_nt: SEQ). */
void ao_matmul_bf16_nt(const uint16_t* x, const uint16_t* w, int64_t rows, int64_t cols,
                       int64_t depth, uint16_t* out);
void ao_matmul_bf16_nt_mode(const uint16_t* x, const uint16_t* w, int64_t rows, int64_t cols,
                            int64_t depth, int mode, uint16_t* out);

/* a2: qwen3_5_moe_route_experts, qwen3_5_moe/model/routing.rs:16-49. */
int ao_route_experts(const void* logits, int dtype, int64_t tokens, int experts, int top_k,
                     int normalize, uint32_t* out_ids, void* out_scores);

/* f4: Laguna router, laguna/moe/router_selection.rs:47-107 (the authoritative CPU
 * formula of laguna/moe/router.rs:11-60): score = sigmoid(l), l = softcap *
 * tanh(logit / softcap) when softcap > 0; selection = score + bias[e] (bias may
 * be NULL); top-K by (selection desc, id asc; IEEE total order); the winners'
 * original scores, divided by their slot-order sum when normalize and sum > 0.
 * exp, sigmoid and tanh are ao_expf, ao_sigmoid_plainf and ao_tanhf (defined
 * here; the kernel evaluates the same steps).  scores fp32 [tokens, K]. */
float ao_sigmoid_plainf(float x);         /* 1 / (1 + e^-x) */
float ao_tanhf(float x);                  /* sign(x) * (1 - 2 / (e^(2|x|) + 1)) */
int ao_route_laguna_experts(const void* logits, int dtype, int64_t tokens, int experts, int top_k,
                            const float* bias, float softcap, int normalize, uint32_t* out_ids,
                            float* out_scores);

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
  /* Each projection's own quantisation (Qwen3_5AffineWeights::Quantized carries
   * its bits and group size, qwen3_5/model/decoder_layer_weights.rs:15-26):
   * gate, up, down, shared gate, shared up, shared down; 0 = `bits` / `group`. */
  int proj_bits[6], proj_group[6];
  /* Affine router (Qwen3_5MoERouterGateWeights::Affine, feed_forward_weights.rs:10-14):
   * used when router_bits > 0, router_w is then ignored.  [E, H*bits/32] codes,
   * [E, H/group] scales and biases. */
  const uint32_t* router_q; const uint16_t* router_s; const uint16_t* router_b;
  int router_bits, router_group;
  /* Affine shared-expert output gate, used when shared_gate_bits > 0. */
  const uint32_t* shared_gate_q; const uint16_t* shared_gate_s; const uint16_t* shared_gate_b;
  int shared_gate_bits, shared_gate_group;
  /* Accumulation modes (AO_DOT_*): router, shared-gate logit, routed gate/up,
   * routed down, shared gate/up, shared down. */
  int arith[6];
  /* Router family: 0 Qwen (softmax, bf16 scores, sigmoid-gated shared expert);
   * 1 Laguna (laguna/moe/resident.rs:60-100): ao_route_laguna_experts with the
   * fields below, fp32 scores, the routed sum times bf16(routed_scaling_factor)
   * (<= 0: 1) rounded to bf16, plus the ungated shared expert.  out_scores of
   * the block functions are bf16 for 0 and fp32 for 1. */
  int router_kind;
  float router_logit_softcap;
  float routed_scaling_factor;
  const float* router_correction_bias;
} ao_block_weights;

/* Runs the block for the tokens listed in token_subset (NULL = all tokens).  The
 * sorted/unsorted decision uses the FULL assignment count tokens*top_k
 * (routing.rs:13, resident_execution.rs:86-96), so a subset run reproduces the
 * rows of the full run.  logits_override (bf16 [tokens, E], may be NULL) replaces
 * the router projection.  ids/scores/out are indexed by the subset position. */
int ao_moe_block_forward(const ao_block_weights* w, const uint16_t* x, int64_t tokens,
                         const int64_t* token_subset, int64_t n_subset,
                         const uint16_t* logits_override, uint16_t* out,
                         uint32_t* out_ids, void* out_scores, int num_threads);

/* Same, also returning the two bf16 terms of the final addition (the routed
 * weighted sum and the gated shared-expert output; zero without a shared
 * expert), used to scale output tolerances. */
int ao_moe_block_forward_terms(const ao_block_weights* w, const uint16_t* x, int64_t tokens,
                               const int64_t* token_subset, int64_t n_subset,
                               const uint16_t* logits_override, uint16_t* out,
                               uint32_t* out_ids, void* out_scores, uint16_t* out_sparse,
                               uint16_t* out_shared_gated, int num_threads);

#ifdef __cplusplus
}
#endif
#endif
