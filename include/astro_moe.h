/*
 * astro_moe.h -- C ABI of libastro_moe, the B200 (sm_100a) implementation of
 * Astronomical's sorted mixture-of-experts block.
 *
 * Conventions (mirroring the MLX-C convention the reference binds through
 * crates/runtime-integration/src/mlx_runtime/error_handling.rs:19-60):
 *   - every entry point returns an int status (ASTRO_MOE_OK == 0); the message
 *     of the last failure on the calling thread is astro_moe_last_error();
 *   - array arguments are caller-owned DEVICE pointers unless the name says
 *     host; calls are stream-ordered and asynchronous on the given cudaStream_t
 *     (passed as void*, NULL = the legacy default stream);
 *   - geometry is validated on the host before any kernel runs (as
 *     sparse_experts/error.rs:1-22 does); index errors found on the device
 *     (expert id >= E, bad row) are recorded in a per-device status word, read
 *     with astro_moe_device_status(), and the offending access is skipped;
 *   - weights are borrowed, never copied (StackedExpertProjection<'a>,
 *     sparse_experts/gathered_projection.rs:45-71): the caller keeps them alive.
 *
 * Weight layout is MLX's affine layout, unchanged, so checkpoints drop in:
 * packed uint32 [E, out, in*bits/32] with element j of a row at bit j*bits of
 * the row's little-endian bit stream, scales/biases bf16 [E, out, in/group],
 * w = scale * q + bias.  Paths below are relative to the reference project root.
 */
#ifndef ASTRO_MOE_H
#define ASTRO_MOE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ASTRO_MOE_ABI_VERSION 2

enum {
  ASTRO_MOE_OK = 0,
  ASTRO_MOE_ERR_INVALID_ARGUMENT = 1, /* MlxRuntimeError::RuntimeOperation, geometry */
  ASTRO_MOE_ERR_CUDA = 2,
  ASTRO_MOE_ERR_OUT_OF_MEMORY = 3,
  ASTRO_MOE_ERR_UNSUPPORTED = 4,
  ASTRO_MOE_ERR_DEVICE_STATUS = 5,    /* a kernel recorded a bad index or a wait timeout */
  ASTRO_MOE_ERR_NOT_REGISTERED = 6,
  ASTRO_MOE_ERR_NCCL = 7,
  ASTRO_MOE_ERR_DUPLICATE_SLOT = 8,   /* assignment_permutation.rs:26-31 */
  ASTRO_MOE_ERR_OUT_OF_RANGE_SLOT = 9,/* assignment_permutation.rs:20-25 */
  ASTRO_MOE_ERR_MEMORY_LIMIT = 10     /* MlxRuntimeError::ActiveMemoryLimitExceeded, mlx_runtime_types.rs:129-133 */
};

enum { ASTRO_MOE_DTYPE_BF16 = 1, ASTRO_MOE_DTYPE_F16 = 2, ASTRO_MOE_DTYPE_F32 = 3 };

/* device status bits (astro_moe_device_status) */
enum {
  ASTRO_MOE_DEVICE_BAD_EXPERT_ID = 1,
  ASTRO_MOE_DEVICE_WAIT_TIMEOUT = 2,
  ASTRO_MOE_DEVICE_BAD_SHAPE = 4
};

/* No counterpart in the reference.  One tensor-core accumulation on given
 * operands, for checking the arithmetic the CPU restatement models (not on any
 * hot path): d = c + a . b^T in fp32 with bf16 a and b, per problem.
 *   instruction 0: tcgen05.mma kind::f16 (M = 128, N = n in {16, 32}, K = 16*k16,
 *     k16 <= 16); a bf16 [problems][128][K], b bf16 [problems][n][K], c and d fp32
 *     [problems][128][n]; accumulate = 0 starts from zero (c unused);
 *     device_status (required) receives ASTRO_MOE_DEVICE_WAIT_TIMEOUT if the MMAs
 *     do not complete within 1 s.
 *   instruction 1: mma.sync m16n8k16 (n = 8, K = 16*k16, k16 <= 64); a [problems][16][K],
 *     b [problems][8][K], c and d [problems][16][8]; always starts from c.
 * K steps are issued in order, 16 at a time. */
int astro_moe_tensor_core_probe(int32_t instruction, const void* a, const void* b, const float* c,
                                float* d, int64_t problems, int32_t n, int32_t k16,
                                int32_t accumulate, uint32_t* device_status, void* stream);

/* No counterpart in the reference.  Runs one of the library's bounded device
 * waits alone, for failure tests that make a wait run out without faulting or
 * hanging the GPU: kind 0 polls *flag >= target (the fused decode kernel's
 * completion-counter wait), kind 1 waits on an mbarrier that expects two
 * arrivals and receives min(target, 2) (the tcgen05 GEMMs' pipeline wait).  A
 * wait that does not complete within limit_ns (<= 2 s) records
 * ASTRO_MOE_DEVICE_WAIT_TIMEOUT in the caller's device_status word and gives
 * up; *result (device) is 1 when the wait completed, 0 when it ran out. */
int astro_moe_wait_probe(int32_t kind, const uint32_t* flag, uint32_t target, int64_t limit_ns,
                         uint32_t* device_status, uint32_t* result, void* stream);

/* No counterpart in the reference.  Exhaustive device check of the packed
 * arithmetic the tcgen05 gate/up epilogue uses in place of the scalar steps that
 * match the CPU restatement: which 0 = the reciprocal of [1, 2] (every fp32),
 * 1 = exp of x <= 0 (every fp32), 2 = bf16x2 multiply against the rounded fp32
 * product (every pair of bf16), 3 = the packed SwiGLU against the scalar one
 * (every (gate, up) pair of bf16).  Device outputs: *mismatches (uint64) counts
 * the inputs whose results differ bit-wise (NaN == NaN), *first_index the
 * smallest such input index (0xffffffff when none).  Asynchronous on `stream`. */
int astro_moe_numerics_check(int32_t which, unsigned long long* mismatches,
                             uint32_t* first_index, void* stream);

/* Thread-local message of the last failed call; replaces the handler installed
 * by crates/runtime-integration/src/mlx_runtime/error_handling.rs:10-44. */
const char* astro_moe_last_error(void);
int astro_moe_abi_version(void);

/* Reads (and with reset != 0 clears) the device status word of `device`;
 * synchronises that device first. */
int astro_moe_device_status(int32_t device, uint32_t* status, int32_t reset);

/* ------------------------------------------------------------------------ */
/* Stage entry points: one per MlxRuntime call the reference's MoE path makes */
/* ------------------------------------------------------------------------ */

/* qwen3_5_moe_route_experts, crates/model-serving/src/qwen3_5_moe/model/routing.rs:16-49
 * (softmax_axis mlx_operations.rs:314, argpartition_axis :364, take_along_axis,
 * sum/divide).  router_logits [tokens, experts] of `dtype`; selected_indices
 * uint32 [tokens, top_k]; selected_scores [tokens, top_k] of `dtype`.  The K
 * winners are ordered by (probability desc, expert id asc).  top_k <= 32,
 * experts <= 1024. */
int astro_moe_route_experts(const void* router_logits, int32_t dtype, int64_t tokens,
                            int32_t experts, int32_t top_k, int32_t normalize,
                            uint32_t* selected_indices, void* selected_scores, void* stream);

/* route_laguna_experts, crates/model-serving/src/laguna/moe/router.rs:11-60 (CPU
 * owner laguna/moe/router_selection.rs:47-107): per token, score = sigmoid(l) in
 * fp32 with l = softcap * tanh(logit / softcap) when router_logit_softcap > 0
 * (else the logit); selection = score + correction_bias[e] (fp32 [experts], may
 * be NULL) ranks the experts, the K largest by (selection desc, expert id asc)
 * are selected, and their original scores are gathered, divided by their sum
 * (slot order) when normalize != 0 and that sum is > 0.  selected_scores fp32
 * [tokens, top_k].  top_k <= 32, experts <= 1024. */
int astro_moe_route_laguna_experts(const void* router_logits, int32_t dtype, int64_t tokens,
                                   int32_t experts, int32_t top_k, const float* correction_bias,
                                   double router_logit_softcap, int32_t normalize,
                                   uint32_t* selected_indices, float* selected_scores,
                                   void* stream);

/* sort_expert_assignments, crates/model-serving/src/sparse_experts/assignment_sort.rs:36-97
 * (argsort_axis mlx_operations.rs:377 twice, floor_divide :178).  Stable.  Any
 * output pointer may be NULL.  expert_offsets has experts+1 entries (the
 * per-expert row ranges gather_qmm derives internally).  experts <= 1024. */
int astro_moe_sort_expert_assignments(const uint32_t* selected_indices, int64_t tokens,
                                      int32_t top_k, int32_t experts, uint32_t* sorted_order,
                                      uint32_t* inverse_order, uint32_t* sorted_indices,
                                      uint32_t* sorted_tokens, uint32_t* expert_offsets,
                                      void* stream);

/* No counterpart in the reference.  The same sort for callers that cannot
 * allocate device memory: a process whose own caching allocator has reserved
 * all of HBM (cudaMalloc/cudaMallocAsync would fail), or a latency-bound loop
 * that cannot accept the device synchronisation cudaMalloc/cudaFree may cause.
 * Outputs equal astro_moe_sort_expert_assignments's.  Its scratch is a fixed
 * ASTRO_MOE_NO_ALLOC_SCRATCH_BYTES (256 KiB) device array per GPU, kept until
 * the process exits: a call needs 4*experts*ceil(tokens*top_k/2048) bytes, plus
 * 4*(experts+1) when expert_offsets is NULL, and larger calls fail with
 * ASTRO_MOE_ERR_UNSUPPORTED before any work is queued.  Nothing in the array
 * must start at zero.  All calls on a device share the array: calls whose
 * kernels overlap on the GPU race, so order them on one stream.  The first call
 * in each CUDA context (normally a device's primary context, with that device
 * current) looks up the array's device address and keeps it for that context
 * only (so it is looked up again after a cudaDeviceReset or in another
 * context); make that first call before any stream capture.  device_status is an
 * optional caller-owned device word that receives ASTRO_MOE_DEVICE_BAD_EXPERT_ID
 * (OR'ed in) for ids >= experts; NULL records nothing.  Such ids are skipped. */
#define ASTRO_MOE_NO_ALLOC_SCRATCH_BYTES 262144
int astro_moe_sort_expert_assignments_no_alloc(const uint32_t* selected_indices, int64_t tokens,
                                               int32_t top_k, int32_t experts,
                                               uint32_t* sorted_order, uint32_t* inverse_order,
                                               uint32_t* sorted_indices, uint32_t* sorted_tokens,
                                               uint32_t* expert_offsets, uint32_t* device_status,
                                               void* stream);

/* take_axis(states, rows, 0), crates/runtime-integration/src/mlx_shape_operations.rs:34
 * as used at assignment_sort.rs:88: out[p] = states[rows[p]] (bf16 rows of
 * `hidden` elements, hidden % 8 == 0). */
int astro_moe_take_rows(const void* states, int64_t state_rows, int32_t hidden,
                        const uint32_t* rows, int64_t n, void* out, void* stream);

/* MlxRuntime::gather_quantized_matmul_affine,
 * crates/runtime-integration/src/mlx_quantized_operations.rs:100-157 (transpose=true,
 * validation :226-330).  out[n] = activations[lhs_indices[n]] .
 * dequant(W[rhs_indices[n]])^T; lhs_indices NULL = identity, rhs_indices NULL
 * = expert 0.  activations bf16 [activation_rows, in_features]; out bf16
 * [n_rows, out_features].  sorted_indices != 0 promises ascending rhs indices
 * (gathered_projection.rs:24-38); otherwise rows are grouped internally.
 * group_size in {32,64,128}, bits in {2,3,4,5,6,8}. */
int astro_moe_gather_qmm(const void* activations, int64_t activation_rows, int32_t in_features,
                         const uint32_t* lhs_indices, const uint32_t* rhs_indices, int64_t n_rows,
                         const uint32_t* packed, const void* scales, const void* biases,
                         int32_t experts, int32_t out_features, int32_t group_size, int32_t bits,
                         int32_t sorted_indices, void* out, void* stream);

/* MlxRuntime::quantized_matmul_affine, mlx_quantized_operations.rs:49-98
 * (transpose=true): out = activations . dequant(W)^T. */
int astro_moe_quantized_matmul(const void* activations, int64_t rows, int32_t in_features,
                               const uint32_t* packed, const void* scales, const void* biases,
                               int32_t out_features, int32_t group_size, int32_t bits, void* out,
                               void* stream);

/* MLX affine dequantize, crates/runtime-integration/src/mlx_quantized_operations.rs:5-47:
 * out[r, j] = bf16(scale[r, j/group] * q[r, j] + bias[r, j/group]) for `rows`
 * rows of in_features elements (MLX layout, any supported bits / group). */
int astro_moe_dequantize_affine(const uint32_t* packed, const void* scales, const void* biases,
                                int64_t rows, int32_t in_features, int32_t group_size,
                                int32_t bits, void* out, void* stream);

/* MlxRuntime::apply_compiled_swiglu, crates/runtime-integration/src/mlx_compiled_swiglu.rs:32-89:
 * out = gate * sigmoid(gate) * up, bf16, n elements. */
int astro_moe_swiglu(const void* gate, const void* up, int64_t n, void* out, void* stream);

/* sorted_expert_weighted_sum, crates/model-serving/src/sparse_experts/weighted_sum.rs:75-190
 * (kernel source :16-33).  sorted_outputs [tokens*top_k, dim] and out
 * [tokens, dim] of output_dtype; scores [tokens, top_k] of score_dtype. */
int astro_moe_sorted_expert_weighted_sum(const void* sorted_outputs, int32_t output_dtype,
                                         const uint32_t* inverse_order, const void* scores,
                                         int32_t score_dtype, int64_t tokens, int32_t top_k,
                                         int64_t dim, void* out, void* stream);

/* unsorted_expert_weighted_sum, weighted_sum.rs:46-60 and :94-120.
 * outputs [tokens, top_k, dim]. */
int astro_moe_unsorted_expert_weighted_sum(const void* outputs, int32_t output_dtype,
                                           const void* scores, int32_t score_dtype,
                                           int64_t tokens, int32_t top_k, int64_t dim, void* out,
                                           void* stream);

/* combine_sparse_and_shared_experts, crates/model-serving/src/qwen3_5_moe/model/output_combination.rs:34-43,
 * and the compiled graph runtime-integration/src/mlx_compiled_sparse_shared_expert_combination.rs:9-75:
 * out = sparse + sigmoid(gate_logits) * shared; gate_logits [tokens, 1]. */
int astro_moe_combine_sparse_and_shared(const void* sparse, const void* shared,
                                        const void* gate_logits, int32_t dtype, int64_t tokens,
                                        int64_t dim, void* out, void* stream);

/* invert_assignment_order, crates/model-serving/src/sparse_experts/assignment_permutation.rs:10-41.
 * HOST arrays; returns ASTRO_MOE_ERR_DUPLICATE_SLOT / _OUT_OF_RANGE_SLOT. */
int astro_moe_invert_assignment_order(const uint32_t* host_sorted_order, int64_t n,
                                      uint32_t* host_inverse_order);

/* ------------------------------------------------------------------------ */
/* Block level: Qwen3_5Model::forward_qwen3_5_moe, resident branch            */
/* (crates/model-serving/src/qwen3_5_moe/model/forward.rs:19-28, :111-127;    */
/*  resident_execution.rs:70-143, :352-400)                                  */
/* ------------------------------------------------------------------------ */

typedef struct astro_moe_ctx astro_moe_ctx;

typedef struct {
  int64_t max_tokens;        /* workspace is sized for this many tokens per call */
  int32_t sorted_threshold;  /* 0 = 64, MINIMUM_SORTED_EXPERT_ASSIGNMENTS (routing.rs:13) */
  int32_t use_tensor_cores;  /* 0 = auto (tcgen05 path for 4-bit g64), -1 = never */
  int64_t decode_max_tokens; /* batches of at most this many tokens take the decode
                                path (4-bit g64 layers); 0 = 48 where the fused
                                decode kernel applies, else 8; -1 = never */
  int64_t decode_fused;      /* decode batches of <= 64 tokens run as one cooperative
                                kernel; 0 = auto, -1 = never (separate kernels) */
  int64_t reserved[4];
} astro_moe_options;

/* One stacked affine projection in MLX layout (Qwen3_5AffineWeights::Quantized,
 * qwen3_5/model/decoder_layer_weights.rs:15-26), with its own bit width and
 * group size as each reference module carries them (0 = the layer's). */
typedef struct {
  const uint32_t* packed;
  const void* scales;  /* bf16 */
  const void* biases;  /* bf16 */
  int32_t bits;        /* 2, 3, 4, 5, 6 or 8; 0 = astro_moe_layer_weights.bits */
  int32_t group_size;  /* 32, 64 or 128; 0 = astro_moe_layer_weights.group_size */
} astro_moe_affine;

/* Qwen3_5MoEFeedForwardWeights (qwen3_5_moe/model/feed_forward_weights.rs:16-24)
 * plus the resident expert stacks (expert_residency).  With gate_up_fused the
 * `gate` tensor is the [E, 2I, .] concatenation of resident_gate_up_fusion.rs:221-260
 * (gate rows first) and `up` is ignored.  shared_intermediate == 0: no shared expert.
 *
 * Quantisation: `bits` / `group_size` are the defaults; each astro_moe_affine may
 * carry its own.  gate and up must share theirs, and so must the shared gate and
 * shared up.  The tcgen05 and decode kernels serve 4-bit group-64 experts; other
 * profiles run on the CUDA-core grouped GEMV.  A shared expert quantised unlike
 * the routed experts runs as its own launches.
 *
 * Router (Qwen3_5MoERouterGateWeights, feed_forward_weights.rs:10-14): a bf16
 * `router_weight`, or NULL with `router_affine` set (the Affine variant, which the
 * reference runs through quantized_linear, forward.rs:53-58).  The shared-expert
 * output gate likewise: bf16 `shared_expert_gate`, or NULL with
 * `shared_expert_gate_affine`.  An affine router or gate is dequantised once at
 * registration into a bf16 copy the context owns (w = bf16(scale * q + bias), the
 * weight MLX's quantized matmul multiplies; 2*E*H bytes for the router); every
 * call then runs the dense router kernels on it. */
typedef struct {
  int32_t hidden, experts, top_k, intermediate, shared_intermediate;
  int32_t group_size, bits, normalize_top_k, gate_up_fused;
  const void* router_weight;       /* bf16 [E, H] (Qwen3_5MoERouterGateWeights::Unquantized) */
  astro_moe_affine gate, up;       /* [E, I, H*bits/32] */
  astro_moe_affine down;           /* [E, H, I*bits/32] */
  astro_moe_affine shared_gate, shared_up; /* [Is, H*bits/32] */
  astro_moe_affine shared_down;    /* [H, Is*bits/32] */
  const void* shared_expert_gate;  /* bf16 [1, H] */
  astro_moe_affine router_affine;            /* [E, H*bits/32] when router_weight is NULL */
  astro_moe_affine shared_expert_gate_affine; /* [1, H*bits/32] when shared_expert_gate is NULL */
  /* Router family.  ASTRO_MOE_ROUTER_SOFTMAX: Qwen3.5/3.6 (softmax top-K, bf16
   * scores, sigmoid-gated shared expert).  ASTRO_MOE_ROUTER_SIGMOID: Laguna
   * (laguna/moe/resident.rs:60-100): astro_moe_route_laguna_experts with the
   * fields below, fp32 scores, the routed sum times routed_scaling_factor
   * (0 = 1), and an ungated shared expert (shared_expert_gate unused). */
  int32_t router_kind;
  float router_logit_softcap;          /* Laguna: > 0 applies softcap * tanh(logit / softcap) */
  float routed_scaling_factor;         /* Laguna */
  const float* router_correction_bias; /* Laguna: fp32 [E] or NULL */
} astro_moe_layer_weights;

enum { ASTRO_MOE_ROUTER_SOFTMAX = 0, ASTRO_MOE_ROUTER_SIGMOID = 1 };

/* Optional device outputs of one block call, for parity checks. */
typedef struct {
  void* router_logits;        /* bf16 [tokens, E] */
  uint32_t* selected_indices; /* [tokens, K] */
  void* selected_scores;      /* bf16 [tokens, K] (fp32 for a Laguna router) */
  uint32_t* expert_offsets;   /* [E + 2] (segment E = shared expert rows) */
} astro_moe_block_taps;

int astro_moe_ctx_create(int32_t device, void* stream, const astro_moe_options* options,
                         astro_moe_ctx** out_ctx);
int astro_moe_ctx_destroy(astro_moe_ctx* ctx);
int astro_moe_ctx_set_stream(astro_moe_ctx* ctx, void* stream);
/* synchronises the context stream and turns a non-zero device status into
 * ASTRO_MOE_ERR_DEVICE_STATUS */
int astro_moe_ctx_synchronize(astro_moe_ctx* ctx);

/* Borrows the weights of one decoder layer (bind_qwen3_5_moe_feed_forward_weights,
 * feed_forward_weights.rs:50-84); validates every shape. */
int astro_moe_register_layer(astro_moe_ctx* ctx, int32_t layer,
                             const astro_moe_layer_weights* weights);

/* forward_qwen3_5_moe: hidden_states bf16 [tokens, H] -> out bf16 [tokens, H]. */
int astro_moe_block_forward(astro_moe_ctx* ctx, int32_t layer, const void* hidden_states,
                            int64_t tokens, void* out);
int astro_moe_block_forward_taps(astro_moe_ctx* ctx, int32_t layer, const void* hidden_states,
                                 int64_t tokens, void* out, const astro_moe_block_taps* taps);
/* Per-stage device time of block calls, measured with CUDA events on the context
 * stream (a fused decode call is one kernel; its time is reported as gate_up_ms); the stage names follow PerformanceOperation
 * (crates/model-serving/src/performance_attribution/catalog.rs:89-92), which in
 * the reference times only host graph construction. */
typedef struct {
  int64_t calls;                     /* block calls measured */
  int64_t kernel_launches;           /* kernels those calls launched */
  double router_projection_ms;
  double assignment_preparation_ms;  /* ExpertAssignmentPreparation: route, sort, row gather */
  double gate_up_ms;                 /* GatheredExpertExecution: gate/up projection + SwiGLU */
  double down_ms;                    /* GatheredExpertExecution: down projection */
  double weighted_reduction_ms;      /* ExpertWeightedReduction, fused with the shared expert */
} astro_moe_attribution;

/* Kernels that the last block call of a context ran, stage by stage (no
 * counterpart in the reference, whose MLX graph hides its kernels).  A stage's
 * accumulation order follows from its kernel, which is what the parity tests
 * use to pick the matching arithmetic of the CPU restatement. */
enum {
  ASTRO_MOE_KERNEL_NONE = 0,
  ASTRO_MOE_KERNEL_TCGEN05_GEMM = 1,  /* tcgen05 grouped GEMM / router GEMM */
  ASTRO_MOE_KERNEL_FUSED_DECODE = 2,  /* the cooperative decode kernel (mma.sync tiles) */
  ASTRO_MOE_KERNEL_DECODE_GEMV = 3,   /* the separate decode GEMVs */
  ASTRO_MOE_KERNEL_GROUPED_GEMV = 4,  /* the CUDA-core grouped GEMV (every bits / group) */
  ASTRO_MOE_KERNEL_ROUTER_GEMV = 5,   /* the router GEMV (small batches) */
  ASTRO_MOE_KERNEL_SIMT_GEMM = 6,     /* the CUDA-core dense GEMM */
  ASTRO_MOE_KERNEL_ROUTE = 7          /* the routing kernel (shared-expert gate dot) */
};
typedef struct {
  int32_t router;         /* router logits */
  int32_t gate_logit;     /* shared-expert gate logit (NONE without a shared expert) */
  int32_t experts;        /* routed gate/up + SwiGLU and down projections */
  int32_t shared_expert;  /* shared expert's projections (NONE without one) */
} astro_moe_block_path;
int astro_moe_ctx_last_block_path(astro_moe_ctx* ctx, astro_moe_block_path* out);

int astro_moe_ctx_set_attribution(astro_moe_ctx* ctx, int32_t enabled);
/* Synchronises, adds up the pending measurements and optionally resets them. */
int astro_moe_ctx_read_attribution(astro_moe_ctx* ctx, astro_moe_attribution* out, int32_t reset);

/* Same with HOST buffers: copies in, runs, copies out, synchronises. */
int astro_moe_block_forward_host(astro_moe_ctx* ctx, int32_t layer, const void* host_hidden,
                                 int64_t tokens, void* host_out);

/* Same with HOST buffers (pinned for overlap), without synchronising: the input
 * goes up on an upload stream, the block runs on the context stream, the output
 * comes down on a download stream, through two staging slots that alternate
 * between calls, so call i's download and call i+1's upload overlap call i+1's
 * block.  host_out is written when astro_moe_host_synchronize returns; the
 * caller keeps both host buffers of a call untouched until then. */
int astro_moe_block_forward_host_async(astro_moe_ctx* ctx, int32_t layer, const void* host_hidden,
                                       int64_t tokens, void* host_out);
int astro_moe_host_synchronize(astro_moe_ctx* ctx);

/* ------------------------------------------------------------------------ */
/* Expert parallelism over the GPUs of one node.  No counterpart in the       */
/* reference (MLX runs the block on one device); it splits the same block      */
/* (forward.rs:19-127) so that rank r of `world` holds experts                 */
/* [r*E/world, (r+1)*E/world) and tokens stay data-parallel.  One layer call    */
/* is dispatch -> (caller's all-to-all of rows) -> experts -> (all-to-all back) */
/* -> combine, all stream-ordered on the context stream; the caller moves the   */
/* rows (NCCL) between the calls.  One layer may be in flight per context.      */
/* ------------------------------------------------------------------------ */

/* `weights` describes the whole layer for routing (experts = all experts,
 * router_weight [experts, H], shared expert and its gate), but gate/up/down hold
 * only this rank's experts [expert_first, expert_first + expert_count) as
 * stacks of expert_count experts (MLX layout). */
int astro_moe_ep_register_layer(astro_moe_ctx* ctx, int32_t layer,
                                const astro_moe_layer_weights* weights, int32_t expert_first,
                                int32_t expert_count);

/* Router, routing and the stable sort of this rank's tokens over ALL experts,
 * then the gather of the sorted token rows: send_rows bf16 [tokens*top_k, H]
 * in expert order, so the rows for each rank's experts are contiguous;
 * expert_offsets uint32 [experts + 1] (device).  The routing is kept in the
 * context for astro_moe_ep_combine. */
int astro_moe_ep_dispatch(astro_moe_ctx* ctx, int32_t layer, const void* hidden_states,
                          int64_t tokens, void* send_rows, uint32_t* expert_offsets);

/* Runs this rank's experts on the rows received from all `world` ranks:
 * recv_rows bf16 [recv_total, H], source-major and, within a source, in expert
 * order; recv_counts uint32 [world][expert_count] (device) are the per-source,
 * per-expert row counts (recv_total = their sum, host value).  out_rows bf16
 * [recv_total, H] receives the expert outputs in the received order.  The
 * shared expert runs here on this rank's own `tokens` hidden states and is
 * kept for the combine. */
int astro_moe_ep_experts(astro_moe_ctx* ctx, int32_t layer, const void* recv_rows,
                         const uint32_t* recv_counts, int32_t world, int64_t recv_total,
                         const void* hidden_states, int64_t tokens, void* out_rows);

/* returned_rows bf16 [tokens*top_k, H]: the expert outputs of send_rows, in
 * send order (NULL: the peer exchange's return buffer).  out bf16 [tokens, H] =
 * router-weighted sum + gated shared expert, the same arithmetic as
 * astro_moe_block_forward. */
int astro_moe_ep_combine(astro_moe_ctx* ctx, int32_t layer, const void* returned_rows,
                         int64_t tokens, void* out);

/* Peer-memory exchange (world <= 8 GPUs of one node with peer access): the
 * dispatch gather stores rows straight into the destination rank's receive
 * buffer, and the expert side stores outputs straight into the source rank's
 * return buffer, over NVLink.  No kernel waits on another GPU: between push and
 * experts, and between experts and combine, the caller orders all ranks with a
 * stream-ordered collective (e.g. a one-element NCCL all-reduce).
 *
 * create: allocates this rank's receive buffer (recv_rows rows of H bf16; size
 * it for the most rows any rank can receive, world * tokens * top_k), return
 * buffer (return_rows >= tokens * top_k) and count mailbox, and writes their
 * three IPC handles (3 x 64 bytes) to handles_out.  connect: all_handles = every
 * rank's handles, in rank order (world x 3 x 64 bytes); opens the peers' buffers. */
int astro_moe_ep_exchange_create(astro_moe_ctx* ctx, int32_t world, int32_t rank, int32_t hidden,
                                 int64_t recv_rows, int64_t return_rows, void* handles_out);
int astro_moe_ep_exchange_connect(astro_moe_ctx* ctx, const void* all_handles);
int astro_moe_ep_exchange_buffers(astro_moe_ctx* ctx, void** recv_buffer, void** return_buffer);

/* astro_moe_ep_dispatch without the gather: router, routing and sort. */
int astro_moe_ep_route(astro_moe_ctx* ctx, int32_t layer, const void* hidden_states,
                       int64_t tokens, uint32_t* expert_offsets);

/* Gathers the sorted rows and stores the rows for rank d into d's receive buffer
 * from row dest_offsets[d]; this rank's rows for d start at sorted position
 * send_starts[d] (HOST arrays of world entries). */
int astro_moe_ep_push(astro_moe_ctx* ctx, int32_t layer, const void* hidden_states,
                      int64_t tokens, const int64_t* send_starts, const int64_t* dest_offsets);

/* astro_moe_ep_experts on this rank's receive buffer (recv_total rows; source
 * s's rows start at received row recv_starts[s]); the outputs of source s are
 * stored into s's return buffer from row return_offsets[s] (HOST arrays). */
int astro_moe_ep_experts_push(astro_moe_ctx* ctx, int32_t layer, const uint32_t* recv_counts,
                              int64_t recv_total, const void* hidden_states, int64_t tokens,
                              const int64_t* recv_starts, const int64_t* return_offsets);

/* Device-planned variant (no host synchronisation in a layer): after
 * astro_moe_ep_route, post_counts stores this rank's per-expert counts and
 * per-rank totals into every rank's count mailbox; after an all-rank ordering
 * collective, push_dev stores the rows (placements computed on the device from
 * the mailbox), and after another, experts_dev runs the experts over this rank's
 * whole receive buffer capacity (bounds read on the device) and stores the
 * outputs back; after a third, astro_moe_ep_combine(returned_rows = NULL). */
int astro_moe_ep_post_counts(astro_moe_ctx* ctx, int32_t layer, const uint32_t* expert_offsets);
int astro_moe_ep_push_dev(astro_moe_ctx* ctx, int32_t layer, const void* hidden_states,
                          int64_t tokens);
int astro_moe_ep_experts_dev(astro_moe_ctx* ctx, int32_t layer, const void* hidden_states,
                             int64_t tokens);
/* The last layer's [world][world] send matrix (rows rank s sent rank d);
 * synchronises the context stream. */
int astro_moe_ep_exchange_counts(astro_moe_ctx* ctx, uint32_t* host_matrix);

/* ------------------------------------------------------------------------ */
/* Expert paging (config 4): Qwen3_5ExpertPager and the paged branch of        */
/* forward_qwen3_5_moe (qwen3_5_moe/expert_paging/expert_pager/mod.rs:55-224,  */
/* model/forward.rs:229-312, split_page_route.rs:10-60).  The reference reads  */
/* missing expert pages from SSD; here every page lives in pinned host memory  */
/* and an HBM page cache under a byte ceiling keeps the recently used ones      */
/* (LRU), filled by cudaMemcpyAsync on the pager's own copy stream.            */
/* ------------------------------------------------------------------------ */
typedef struct astro_moe_pager astro_moe_pager;

/* Bytes of one expert page: gate, up and down codes, then their scales and
 * biases, each in MLX layout (see astro_moe_pager_create). */
int64_t astro_moe_page_bytes(int32_t hidden, int32_t intermediate, int32_t group_size,
                             int32_t bits);

/* host_pages: PINNED host memory holding layers * experts pages, page
 * (layer, expert) at byte (layer * experts + expert) * page_bytes; a page is
 *   gate codes uint32 [I, H*bits/32] | up codes [I, H*bits/32] |
 *   down codes [H, I*bits/32] | gate scales bf16 [I, H/group] | gate biases |
 *   up scales | up biases | down scales [H, I/group] | down biases.
 * cache_bytes: the HBM ceiling of the page cache (whole pages).  4-bit, group 64. */
int astro_moe_pager_create(astro_moe_ctx* ctx, int32_t layers, int32_t experts, int32_t hidden,
                           int32_t intermediate, int32_t group_size, int32_t bits,
                           const void* host_pages, int64_t cache_bytes, astro_moe_pager** out);
int astro_moe_pager_destroy(astro_moe_pager* pager);

typedef struct {
  int64_t lookups;          /* (layer, expert) pages a block call needed */
  int64_t hits;
  int64_t misses;
  int64_t evictions;
  int64_t bytes_h2d;        /* page bytes copied host -> HBM */
  double copy_ms;           /* device time of those copies (copy-stream events) */
  int64_t resident_pages;
  int64_t capacity_pages;
  int64_t calls;            /* paged block calls */
  int64_t split_calls;      /* ... that copied pages in, so ran the copied experts' second launch */
  int64_t copy_failures;    /* page copies that failed (the call returned an error) */
} astro_moe_pager_stats;

/* Retention policy of the page cache.  LRU (default): a miss evicts the least
 * recently used page.  DEMAND: the pager counts the routed assignments every
 * (layer, expert) page has received (the reference's demand evidence,
 * expert_paging/retained_expert_layer_cache.rs:35-64, :277-311) and a miss evicts
 * the page with the least demand (ties: least recently used), so pages routed
 * often stay resident while a cyclic pass over the layers would make LRU evict
 * exactly the pages the next layers need.  Neither policy copies a page a call
 * does not route to, nor evicts one the current call needs. */
enum { ASTRO_MOE_PAGER_LRU = 0, ASTRO_MOE_PAGER_DEMAND = 1 };
int astro_moe_pager_set_policy(astro_moe_pager* pager, int32_t policy);

/* Host-side fault injection for failure tests: the next `count` page copies are
 * not issued and report a failure as a failed cudaMemcpyAsync would, so the
 * paged call returns ASTRO_MOE_ERR_CUDA without writing its output and the
 * cache holds no page for the failed experts (a later call copies them again). */
int astro_moe_pager_inject_copy_failures(astro_moe_pager* pager, int64_t count);
/* Synchronises the pager's copy stream; reset != 0 clears the counters. */
int astro_moe_pager_read_stats(astro_moe_pager* pager, astro_moe_pager_stats* out, int32_t reset);

/* A paged layer: `weights` supplies the router, the shared expert and its gate
 * (resident); gate/up/down are ignored -- the routed experts are the pager's
 * pages of `layer`. */
int astro_moe_register_paged_layer(astro_moe_ctx* ctx, int32_t layer,
                                   const astro_moe_layer_weights* weights,
                                   astro_moe_pager* pager);

/* forward_qwen3_5_moe for a paged layer: routes, reads the routed experts back
 * to the host (one stream synchronisation, as the reference's pager does),
 * admits the missing pages, and runs the experts from the cache.  Up to 64
 * tokens (decode, forward.rs:229-312) the resident experts are computed while
 * the missing pages copy; more tokens (prefill, the reference's layer streaming,
 * expert_pager/rust_layer_streaming.rs:8-11) bring in every routed page first
 * and run the tcgen05 grouped GEMMs over the cache.  A call that routes to more
 * pages than the cache holds returns ASTRO_MOE_ERR_MEMORY_LIMIT (a call never
 * evicts its own pages). */
int astro_moe_paged_block_forward(astro_moe_ctx* ctx, int32_t layer, const void* hidden_states,
                                  int64_t tokens, void* out);

#ifdef __cplusplus
}
#endif
#endif
