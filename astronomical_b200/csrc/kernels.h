// kernels.h -- internal launch interface between the C ABI (api.cu) and the
// kernels.  Not installed; the public boundary is include/astro_moe.h.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace astro {

cudaError_t launch_route_experts(const void* logits, int dtype, int64_t tokens, int E, int K,
                                 int normalize, uint32_t* ids, void* scores, const void* x,
                                 const void* wg, int H, void* gate_logit, cudaStream_t st);

cudaError_t launch_dense_nt_simt(const void* x, const void* w, int64_t rows, int cols, int depth,
                                 void* out, int ldo, cudaStream_t st);

// scratch: sort_scratch_bytes(tokens * K, E) bytes of device memory
size_t sort_scratch_bytes(int64_t n, int E);
// kernels one launch_sort_assignments call issues (1 when all n fit one tile)
int sort_launch_count(int64_t n);
cudaError_t launch_sort_assignments(const uint32_t* ids, int64_t tokens, int K, int E,
                                    int64_t shared_rows, uint32_t* sorted_order,
                                    uint32_t* inverse_order, uint32_t* sorted_ids,
                                    uint32_t* sorted_tokens, uint32_t* offsets, uint32_t* status,
                                    void* scratch, cudaStream_t st);

// rows == nullptr: row p; perm8: rows stored in the tcgen05 grouped GEMMs' K
// order (perm8_bf16 in common.cuh)
cudaError_t launch_take_rows(const void* src, int64_t src_rows, const uint32_t* rows, int64_t n,
                             int hidden, void* out, uint32_t* status, cudaStream_t st,
                             bool perm8 = false);

// scores_f32 != nullptr: the Laguna combination (fp32 scores, routed sum times
// `factor` -- already bf16-rounded -- and an ungated shared expert when has_shared);
// has_shared < 0: a shared expert iff gate_logit is given (the Qwen combination).
cudaError_t launch_block_combine(const void* rows, const uint32_t* inverse, const void* scores,
                                 const void* gate_logit, int64_t shared_base, int64_t tokens,
                                 int K, int H, int sorted, void* out, cudaStream_t st,
                                 const float* scores_f32 = nullptr, int has_shared = -1,
                                 float factor = 1.0f);

// Same with the shared expert's rows in their own array: shared_rows[t] (row t
// of the token), routed rows through `inverse` into `rows`.
cudaError_t launch_block_combine_split(const void* rows, const void* shared_rows,
                                       const uint32_t* inverse, const void* scores,
                                       const void* gate_logit, int64_t tokens, int K, int H,
                                       int sorted, void* out, cudaStream_t st);

cudaError_t launch_sorted_weighted_sum(const void* rows, int out_dtype, const uint32_t* inverse,
                                       const void* scores, int score_dtype, int64_t tokens, int K,
                                       int64_t dim, void* out, cudaStream_t st);

cudaError_t launch_unsorted_weighted_sum(const void* outputs, int out_dtype, const void* scores,
                                         int score_dtype, int64_t tokens, int K, int64_t dim,
                                         void* out, cudaStream_t st);

cudaError_t launch_combine_shared(const void* sparse, const void* shared, const void* gate,
                                  int dtype, int64_t tokens, int64_t dim, void* out,
                                  cudaStream_t st);

cudaError_t launch_swiglu(const void* gate, const void* up, int64_t n, void* out, cudaStream_t st);

cudaError_t launch_numerics_probe(const float* x, int64_t n, int which, float* out,
                                  cudaStream_t st);

// One stacked affine tensor seen as rows: row (e, f) = e * expert_rows + row_offset + f
// of the packed codes, e * sb_expert_rows + row_offset + f of the scales and
// biases.  sb_expert_rows == 0 means expert_rows (MLX stacks); page-major expert
// pages (expert paging), where one expert's tensors share one contiguous page,
// stride the codes and the scales by different row counts.  The decode GEMVs and
// the fused decode kernel honour sb_expert_rows; the other kernels take MLX
// stacks only.
struct AffineRef {
  const void* q = nullptr;  // uint32 packed
  const void* s = nullptr;  // bf16 scales
  const void* b = nullptr;  // bf16 biases
  int64_t expert_rows = 0;
  int64_t row_offset = 0;
  int64_t sb_expert_rows = 0;
};

struct GroupedGemvDesc {
  const void* x = nullptr;           // bf16 activations
  const uint32_t* x_rows = nullptr;  // sorted position -> activation row
  int64_t x_limit = 0;               // activation rows available
  int in_features = 0;
  const uint32_t* seg_offsets = nullptr;  // [nseg + 1], device
  int nseg = 0;
  int shared_seg = -1;
  int64_t rows_total = 0;            // upper bound on seg_offsets[nseg]
  AffineRef wa[2], wb[2];            // [routed, shared]; wb for SwiGLU mode
  int out_features = 0, group = 64, bits = 4;
  bool swiglu = false;
  void* y = nullptr;
  const uint32_t* y_rows = nullptr;  // sorted position -> output row
  int64_t y_limit = 0;               // output rows available
  int64_t ldy = 0;
  uint32_t* status = nullptr;
  // decode GEMVs only: routed segment e reads expert slot slot_of[e] of wa/wb
  // (expert paging); nullptr = slot e.  A slot of kSlotElsewhere leaves the
  // segment to another launch, and skip_shared leaves the shared expert to one.
  const uint32_t* slot_of = nullptr;
  bool skip_shared = false;
};
constexpr uint32_t kSlotElsewhere = 0xffffffffu;

cudaError_t launch_grouped_gemv(const GroupedGemvDesc& d, cudaStream_t st);

// Small-batch kernels (decode.cu).  Router GEMV: logits [T, E] bf16 = x [T, H] .
// Wr [E, H]^T for H in {1024, 2048, 4096}; x and Wr 16-byte aligned.
bool router_gemv_supported(int H);
cudaError_t launch_router_gemv(const void* x, int64_t T, const void* wr, int E, int H, void* logits,
                               cudaStream_t st);
// Gathered int4 g64 GEMVs over the non-empty segments of d.seg_offsets
// (max_active bounds their number): gate/up writes SwiGLU(gate, up) rows
// (d.wa = gate, d.wb = up, in_features 1024/2048/4096); down reads rows of
// d.x by sorted position (in_features 512/1024/2048).
bool decode_gemv_supported(int H, int I, int group, int bits);
cudaError_t launch_decode_gate_up(const GroupedGemvDesc& d, int64_t max_active, cudaStream_t st);
cudaError_t launch_decode_down(const GroupedGemvDesc& d, int64_t max_active, cudaStream_t st);

// Fused decode block (decode.cu): router, route, sort, gate/up, down and
// combine of T <= 64 tokens in one cooperative launch (one block per SM; grid
// barriers after the router and the down projection, per-segment completion
// counters between gate/up and down).  `barrier` (two words) and `seg_done`
// (E + 1 words) must be zero before the first launch; the kernel leaves them
// zero.  Returns cudaErrorCooperativeLaunchTooLarge when the device cannot hold
// the grid.
struct DecodeFusedArgs {
  const void* x = nullptr;  // bf16 [T, H]
  int T = 0, H = 0, E = 0, K = 0, I = 0, normalize = 1, sorted = 0, has_shared = 0;
  const void* wr = nullptr;  // bf16 [E, H]
  const void* wg = nullptr;  // bf16 [H]
  AffineRef gate[2], up[2], down[2];  // [routed, shared]
  void* logits = nullptr;
  void* gate_logit = nullptr;
  uint32_t* ids = nullptr;
  void* scores = nullptr;
  uint32_t* offsets = nullptr;
  void* act = nullptr;
  void* yrows = nullptr;
  void* out = nullptr;
  uint32_t* barrier = nullptr;
  uint32_t* seg_done = nullptr;  // [E + 1] gate/up items done per segment, zero between launches
  uint32_t* status = nullptr;
};
bool decode_fused_supported(int T, int H, int E, int K, int I);
cudaError_t launch_decode_fused(const DecodeFusedArgs& a, cudaStream_t st);

cudaError_t launch_offsets_from_sorted(const uint32_t* ids, int64_t n, int E, uint32_t* offsets,
                                       uint32_t* status, cudaStream_t st);
cudaError_t launch_route_laguna(const void* logits, int dtype, int64_t tokens, int E, int K,
                                float softcap, const float* bias, int normalize, uint32_t* ids,
                                float* scores, cudaStream_t st);
cudaError_t launch_dequantize_affine(const uint32_t* packed, const void* scales,
                                     const void* biases, int64_t rows, int in_features, int group,
                                     int bits, void* out, cudaStream_t st);
cudaError_t launch_compose_rows(const uint32_t* lhs, const uint32_t* order, int64_t n,
                                uint32_t* rows_out, cudaStream_t st);

// Expert parallelism (ep.cu): from the received counts [world][El] (device),
// the (source, expert) run starts in received and expert-major order, the
// expert-major offsets [El + 2] (segment El: shared_rows rows), and the row maps
// dest[received q] = expert-major position, src_of[dest[q]] = q.
cudaError_t launch_ep_permutation(const uint32_t* counts, int world, int El, int shared_rows,
                                  uint32_t* src_start, uint32_t* exp_start, uint32_t* offsets,
                                  uint32_t* dest, uint32_t* src_of, cudaStream_t st);

// Peer-memory exchange (ep.cu).  Up to kMaxPeers ranks.  push: sorted row p goes
// to rank d = sorted_ids[p] / El, row peer_offs[d] + p - starts[d] of its receive
// buffer.  return: received row q of source s (starts[s] <= q < starts[s+1])
// takes yrows[dest[q]] to row peer_offs[s] + q - starts[s] of s's return buffer.
constexpr int kMaxPeers = 8;
cudaError_t launch_ep_push_rows(const void* x, int64_t x_rows, const uint32_t* stok,
                                const uint32_t* sids, int64_t n, int El, int world, int H,
                                void* const* peer_bases, const int64_t* peer_cap_rows,
                                const int64_t* peer_offs, const int64_t* starts, uint32_t* status,
                                cudaStream_t st);
cudaError_t launch_ep_return_rows(const void* yrows, int64_t y_rows, const uint32_t* dest,
                                  int64_t n, int world, int H, void* const* peer_bases,
                                  const int64_t* peer_cap_rows, const int64_t* peer_offs,
                                  const int64_t* starts, uint32_t* status, cudaStream_t st);

// Device-planned peer exchange (ep.cu).  Mailbox of every rank: uint32
// [world][El] per-expert counts it receives, then the [world][world] send matrix.
cudaError_t launch_ep_post_counts(const uint32_t* offsets, int El, int world, int me,
                                  void* const* mailboxes, int stride, cudaStream_t st);
// counts [world][cstride] (the first El of each row used)
cudaError_t launch_ep_permutation_strided(const uint32_t* counts, int cstride, int world, int El,
                                          int shared_rows, int64_t cap, uint32_t* src_start,
                                          uint32_t* exp_start, uint32_t* offsets, uint32_t* dest,
                                          uint32_t* src_of, cudaStream_t st);
cudaError_t launch_ep_push_rows_dev(const void* x, int64_t x_rows, const uint32_t* stok,
                                    const uint32_t* sids, int64_t n, int El, int world, int me,
                                    int H, const uint32_t* M, void* const* peer_recv,
                                    int64_t cap_rows, uint32_t* status, cudaStream_t st);
cudaError_t launch_ep_gather_states(const void* recv, const uint32_t* src_of, const void* x,
                                    int64_t T, int world, int me, int H, const uint32_t* M,
                                    int64_t cap_rows, void* states, uint32_t* status,
                                    cudaStream_t st, bool perm8 = false);
cudaError_t launch_ep_return_rows_dev(const void* yrows, int64_t y_rows, const uint32_t* dest,
                                      int world, int me, int H, const uint32_t* M,
                                      void* const* peer_ret, int64_t cap_rows, uint32_t* status,
                                      cudaStream_t st);

cudaError_t launch_ep_copy_shared_rows(const void* yrows, int64_t y_rows, int world, int me,
                                       int64_t T, int H, const uint32_t* M, void* out,
                                       cudaStream_t st);

// Sets the calling thread's astro_moe_last_error() message and returns `status`
// (for entry points defined outside api.cu).
int set_last_error(int status, const char* message);

}  // namespace astro
