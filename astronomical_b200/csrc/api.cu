// api.cu -- the C ABI (include/astro_moe.h): validation, error reporting, the
// block context and the orchestration of one MoE block.
//
// Host-side mirror of the reference operator: astro_moe_block_forward plays the
// role of Qwen3_5Model::forward_qwen3_5_moe's resident branch
// (crates/model-serving/src/qwen3_5_moe/model/forward.rs:19-127 and
// resident_execution.rs:70-143): route once, sort the assignments (always on the
// device -- the sort only permutes rows, so it never changes a row's value), run
// the gathered gate/up projection with SwiGLU, the gathered down projection, and
// the weighted combine with the shared expert.  The reference's sorted/unsorted
// switch (routing.rs:13, assignment count >= 64) still selects the weighted-sum
// arithmetic, exactly as in the reference.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <list>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "astro_moe.h"
#include "kernels.h"
#include "moe_gemm.h"

namespace {

thread_local std::string g_last_error;

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  if (e == cudaErrorMemoryAllocation)
    return fail(ASTRO_MOE_ERR_OUT_OF_MEMORY, "%s: %s", what, cudaGetErrorString(e));
  return fail(ASTRO_MOE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define CK(expr, what)                              \
  do {                                              \
    cudaError_t _e = (expr);                        \
    if (_e != cudaSuccess) return cuda_fail(_e, what); \
  } while (0)

inline cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }

bool valid_dtype(int d) {
  return d == ASTRO_MOE_DTYPE_BF16 || d == ASTRO_MOE_DTYPE_F16 || d == ASTRO_MOE_DTYPE_F32;
}
bool valid_group(int g) { return g == 32 || g == 64 || g == 128; }
bool valid_bits(int b) { return b == 2 || b == 3 || b == 4 || b == 5 || b == 6 || b == 8; }

// affine profile check, mlx_quantized_operations.rs:226-330 (in_features here is
// the unpacked width; rows of 32 elements are the unit of the kernels)
int check_affine(const char* op, int64_t in_features, int group, int bits) {
  if (!valid_group(group)) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: affine group size must be 32, 64, or 128", op);
  if (!valid_bits(bits)) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: affine bit width must be 2, 3, 4, 5, 6, or 8", op);
  if (in_features <= 0 || in_features % group != 0)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: input width %lld is not a multiple of the group size", op, (long long)in_features);
  if (in_features % 32 != 0)
    return fail(ASTRO_MOE_ERR_UNSUPPORTED, "%s: input width must be a multiple of 32", op);
  return ASTRO_MOE_OK;
}

// per-device status word and scratch
struct DeviceState {
  uint32_t* status = nullptr;
};
std::mutex g_dev_mu;
std::map<int, DeviceState> g_dev;

int device_status_ptr(uint32_t** out) {
  int dev = 0;
  CK(cudaGetDevice(&dev), "cudaGetDevice");
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceState& ds = g_dev[dev];
  if (!ds.status) {
    CK(cudaMalloc(&ds.status, sizeof(uint32_t)), "cudaMalloc(status)");
    CK(cudaMemset(ds.status, 0, sizeof(uint32_t)), "cudaMemset(status)");
  }
  *out = ds.status;
  return ASTRO_MOE_OK;
}

}  // namespace

// ===========================================================================
// context
// ===========================================================================
struct LayerState {
  astro_moe_layer_weights w{};
  bool registered = false;
  astro::MoeGemmPlan gemm{};  // tensor-core plan (TMA descriptors), when eligible
  bool decode_ok = false;     // the small-batch GEMVs cover this layer's geometry
  bool fused_ok = false;      // ... and scale / bias rows suit the fused decode kernel's vector loads
  bool router_gemv_ok = false;
  // expert-parallel layer: w.experts counts the local stacks, ep_total all experts
  bool ep = false;
  int ep_first = 0, ep_total = 0;
  // paged layer: routed experts come from the pager's pages of this layer
  astro_moe_pager* pager = nullptr;
  // quantisation {bits, group} of gate, up, down, shared gate, shared up, shared down
  int qbits[6] = {}, qgroup[6] = {};
  // shared expert quantised unlike the routed experts: it runs as its own launches
  bool shared_separate = false;
  // bf16 copies of an affine router / shared-expert gate, dequantised at registration
  void* router_dense = nullptr;
  void* sgate_dense = nullptr;
};

void release_layer(LayerState& L) {
  astro::moe_gemm_release(L.gemm);
  if (L.router_dense) cudaFree(L.router_dense);
  if (L.sgate_dense) cudaFree(L.sgate_dense);
  L.router_dense = L.sgate_dense = nullptr;
}

// Grow-only device buffer (synchronises the stream before replacing memory).
struct DevBuf {
  void* p = nullptr;
  size_t bytes = 0;
};

struct astro_moe_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  astro_moe_options opt{};
  std::map<int, LayerState> layers;
  uint32_t* status = nullptr;
  // workspace
  void* ws = nullptr;
  size_t ws_bytes = 0;
  void* io = nullptr;  // device staging for the host-buffer entry point
  size_t io_bytes = 0;
  // asynchronous host-buffer calls: two staging slots (input + output each), an
  // upload and a download stream, and per slot the events that order them
  void* aio[2] = {nullptr, nullptr};
  size_t aio_bytes = 0;
  cudaStream_t up = nullptr, down = nullptr;
  cudaEvent_t ev_in[2] = {}, ev_done[2] = {}, ev_out[2] = {};
  bool ev_out_used[2] = {false, false}, ev_done_used[2] = {false, false};
  int aio_next = 0;
  // stage attribution
  bool attribution = false;
  std::vector<cudaEvent_t> event_pool;
  std::vector<std::vector<cudaEvent_t>> pending;  // 6 events per measured call
  astro_moe_attribution acc{};
  int64_t launches = 0;
  astro_moe_block_path last_path{};
  // expert-parallel block in flight (dispatch -> experts -> combine)
  DevBuf ep_disp, ep_exp, ep_shared;
  int ep_layer = -1;
  int64_t ep_tokens = -1;
  // peer-memory exchange: this rank's receive / return buffers and every rank's
  // mapping of them (index = rank)
  int xr_world = 0, xr_rank = -1;
  void* xr_recv = nullptr;
  void* xr_ret = nullptr;
  int64_t xr_recv_rows = 0, xr_ret_rows = 0;
  void* xr_peer_recv[astro::kMaxPeers] = {};
  void* xr_peer_ret[astro::kMaxPeers] = {};
  // count mailbox: uint32 [world][kMailboxExperts] received per-expert counts, then
  // the [world][world] send matrix
  void* xr_mbox = nullptr;
  void* xr_peer_mbox[astro::kMaxPeers] = {};
  bool xr_connected = false;
};

// Expert page cache: pinned host pages, HBM slots, LRU over slots (host side).
struct astro_moe_pager {
  int device = 0;
  int layers = 0, E = 0, H = 0, I = 0, group = 64, bits = 4;
  int64_t page_bytes = 0;
  // byte offsets of the nine tensors inside a page
  int64_t off_q[3] = {0, 0, 0}, off_s[3] = {0, 0, 0}, off_b[3] = {0, 0, 0};
  const char* host = nullptr;
  char* pool = nullptr;
  int64_t slots = 0, used = 0;
  std::vector<int32_t> slot_of_page;   // [layers * E] -> slot or -1
  std::vector<int64_t> page_of_slot;   // [slots] -> page or -1
  std::vector<int64_t> last_call;      // [slots] call that last needed the slot
  std::list<int64_t> lru;              // slots, most recently used first
  std::vector<std::list<int64_t>::iterator> lru_pos;
  int64_t call = 0;
  cudaStream_t copy = nullptr;
  cudaEvent_t ready = nullptr;
  uint32_t* h_offsets = nullptr;  // pinned [E + 2]
  // slot tables of the two launches of a paged layer: [0, E) the experts whose
  // pages were resident (computed while the missing pages copy), [E, 2E) the
  // experts whose pages were copied in; kSlotElsewhere marks the other launch's
  uint32_t* h_table = nullptr;    // pinned [2E]
  uint32_t* d_table = nullptr;    // device [2E]
  std::vector<uint8_t> missed;    // [E] this call copied the expert's page
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> pending, spare;
  astro_moe_pager_stats st{};
  // retention policy (ASTRO_MOE_PAGER_*) and, for the demand policy, the routed
  // assignments each page has received (expert_paging/retained_expert_layer_cache.rs
  // record_expert_demand): the eviction victim is the slot whose page has the
  // least demand (ties: least recently used) among those the call does not need
  int policy = ASTRO_MOE_PAGER_LRU;
  std::vector<uint64_t> demand;   // [layers * E]
  // host-side fault injection: the next n page copies report a failure instead
  // of being issued (the failure tests' simulated H2D copy error)
  int64_t inject_copy_failures = 0;
};

namespace {

// fused decode synchronisation words at workspace offset 0: the grid barrier's
// two words, then (from word 64) one completion counter per expert segment
constexpr size_t kFusedSyncBytes = 2048;
constexpr int kFusedSegDoneWord = 64;
static_assert((kFusedSyncBytes / 4 - kFusedSegDoneWord) >= 257,
              "a counter per segment of the fused decode kernel (<= 256 experts + shared)");

struct BlockWorkspace {
  uint32_t* barrier;  // fused decode grid barrier; first in the workspace (fixed address)
  uint16_t* logits;
  uint32_t* ids;
  uint16_t* scores;
  uint16_t* gate_logit;
  uint32_t* order;
  uint32_t* inverse;
  uint32_t* sids;
  uint32_t* stok;
  uint32_t* offsets;
  void* sort_scratch;
  uint16_t* states;  // gathered activation rows [rows, H] (tensor-core path)
  uint16_t* act;     // [rows, I]
  uint16_t* yrows;   // [rows, H]
  void* gemm_scratch;
};

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

size_t plan_workspace(const astro_moe_layer_weights& w, int64_t T, BlockWorkspace* out,
                      char* base) {
  const int64_t H = w.hidden, E = w.experts, K = w.top_k;
  const int64_t Imax = w.intermediate;
  const int64_t N = T * K;
  const int64_t rows = N + (w.shared_intermediate > 0 ? T : 0);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    char* p = base ? base + off : nullptr;
    off = align_up(off + bytes, 256);
    return p;
  };
  BlockWorkspace b{};
  b.barrier = (uint32_t*)take(kFusedSyncBytes);
  b.logits = (uint16_t*)take(sizeof(uint16_t) * T * E);
  b.ids = (uint32_t*)take(sizeof(uint32_t) * N);
  b.scores = (uint16_t*)take(sizeof(float) * N);  // bf16 scores, or fp32 for a Laguna router
  b.gate_logit = (uint16_t*)take(sizeof(uint16_t) * T);
  b.order = (uint32_t*)take(sizeof(uint32_t) * N);
  b.inverse = (uint32_t*)take(sizeof(uint32_t) * N);
  b.sids = (uint32_t*)take(sizeof(uint32_t) * rows);
  b.stok = (uint32_t*)take(sizeof(uint32_t) * rows);
  b.offsets = (uint32_t*)take(sizeof(uint32_t) * (E + 2));
  b.sort_scratch = take(astro::sort_scratch_bytes(N, (int)E));
  b.states = (uint16_t*)take(sizeof(uint16_t) * rows * H);
  b.act = (uint16_t*)take(sizeof(uint16_t) * rows * Imax);
  b.yrows = (uint16_t*)take(sizeof(uint16_t) * rows * H);
  b.gemm_scratch = take(astro::moe_gemm_scratch_bytes());
  if (out) *out = b;
  return off;
}

int ensure_ws(astro_moe_ctx* ctx, size_t bytes) {
  if (ctx->ws_bytes >= bytes) return ASTRO_MOE_OK;
  if (ctx->ws) {
    CK(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    cudaFree(ctx->ws);
    ctx->ws = nullptr;
    ctx->ws_bytes = 0;
  }
  CK(cudaMalloc(&ctx->ws, bytes), "cudaMalloc(workspace)");
  ctx->ws_bytes = bytes;
  // the fused decode kernel's barrier words and segment counters (workspace
  // offset 0) start at zero; the kernel leaves them zero
  CK(cudaMemset(ctx->ws, 0, kFusedSyncBytes), "cudaMemset(workspace barrier)");
  return ASTRO_MOE_OK;
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) == cudaSuccess && prev != dev) cudaSetDevice(dev);
    else prev = -1;
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

int validate_affine_tensor(const char* name, const astro_moe_affine& a) {
  if (!a.packed || !a.scales || !a.biases)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "register layer: %s has a null pointer", name);
  if ((reinterpret_cast<uintptr_t>(a.packed) & 15u) != 0)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "register layer: %s packed weights must be 16-byte aligned", name);
  return ASTRO_MOE_OK;
}

cudaEvent_t take_event(astro_moe_ctx* ctx) {
  if (!ctx->event_pool.empty()) {
    cudaEvent_t e = ctx->event_pool.back();
    ctx->event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

struct StageMarks {
  astro_moe_ctx* ctx;
  std::vector<cudaEvent_t> ev;
  explicit StageMarks(astro_moe_ctx* c) : ctx(c) {}
  void mark() {
    if (!ctx->attribution) return;
    cudaEvent_t e = take_event(ctx);
    cudaEventRecord(e, ctx->stream);
    ev.push_back(e);
  }
  // forgets the last n marks (recorded before a launch that did not happen)
  void drop(size_t n) {
    while (n-- > 0 && !ev.empty()) {
      ctx->event_pool.push_back(ev.back());
      ev.pop_back();
    }
  }
  void commit() {
    if (ctx->attribution && ev.size() == 6) ctx->pending.push_back(ev);
    else for (auto e : ev) ctx->event_pool.push_back(e);
    ev.clear();
  }
};

// Stacked projections of a layer as row views: [routed, shared] gate, up, down.
void fill_projections(const astro_moe_layer_weights& w, astro::AffineRef (&gate)[2],
                      astro::AffineRef (&up)[2], astro::AffineRef (&down)[2]) {
  const int64_t I = w.intermediate, Is = w.shared_intermediate, H = w.hidden;
  if (w.gate_up_fused) {
    gate[0] = astro::AffineRef{w.gate.packed, w.gate.scales, w.gate.biases, 2 * I, 0};
    up[0] = astro::AffineRef{w.gate.packed, w.gate.scales, w.gate.biases, 2 * I, I};
  } else {
    gate[0] = astro::AffineRef{w.gate.packed, w.gate.scales, w.gate.biases, I, 0};
    up[0] = astro::AffineRef{w.up.packed, w.up.scales, w.up.biases, I, 0};
  }
  down[0] = astro::AffineRef{w.down.packed, w.down.scales, w.down.biases, H, 0};
  gate[1] = up[1] = down[1] = astro::AffineRef{};
  if (Is > 0) {
    gate[1] = astro::AffineRef{w.shared_gate.packed, w.shared_gate.scales, w.shared_gate.biases, Is, 0};
    up[1] = astro::AffineRef{w.shared_up.packed, w.shared_up.scales, w.shared_up.biases, Is, 0};
    down[1] = astro::AffineRef{w.shared_down.packed, w.shared_down.scales, w.shared_down.biases, H, 0};
  }
}

// Copies the requested intermediate arrays of a block call to the caller's taps.
int copy_taps(astro_moe_ctx* ctx, const BlockWorkspace& b, int64_t T, int E, int K,
              bool has_shared, const astro_moe_block_taps* taps, size_t score_bytes = 2) {
  if (!taps) return ASTRO_MOE_OK;
  cudaStream_t st = ctx->stream;
  const int64_t N = T * K;
  {
    if (taps->router_logits)
      CK(cudaMemcpyAsync(taps->router_logits, b.logits, sizeof(uint16_t) * T * E,
                         cudaMemcpyDeviceToDevice, st), "taps");
    if (taps->selected_indices)
      CK(cudaMemcpyAsync(taps->selected_indices, b.ids, sizeof(uint32_t) * N,
                         cudaMemcpyDeviceToDevice, st), "taps");
    if (taps->selected_scores)
      CK(cudaMemcpyAsync(taps->selected_scores, b.scores, score_bytes * N,
                         cudaMemcpyDeviceToDevice, st), "taps");
    if (taps->expert_offsets)
      CK(cudaMemcpyAsync(taps->expert_offsets, b.offsets,
                         sizeof(uint32_t) * (E + (has_shared ? 2 : 1)), cudaMemcpyDeviceToDevice, st),
         "taps");
  }
  return ASTRO_MOE_OK;
}

// experts per rank a count mailbox holds
constexpr int kMailboxExperts = 1024;

// batches up to this many tokens take the decode path unless the options say
// otherwise: the fused decode kernel where its shapes apply (it takes up to 64
// tokens when asked; above 16 it restages and re-dequantises per 16 token rows
// of a segment: level with the grouped GEMMs at 32 tokens, 88 us per layer,
// ahead at 48, 97 against 109, behind at 64, 125 against 108), else the
// separate decode GEMVs
constexpr int64_t kDefaultFusedTokens = 48;
constexpr int64_t kDefaultDecodeTokens = 8;
// batches up to this many tokens compute router logits with the router GEMV
constexpr int64_t kRouterGemvTokens = 64;
// a paged call of more tokens brings in all its pages first (prefill)
constexpr int64_t kPagedDecodeTokens = 64;

int run_block(astro_moe_ctx* ctx, LayerState& L, const void* x, int64_t T, void* out,
              const astro_moe_block_taps* taps) {
  const astro_moe_layer_weights& w = L.w;
  const int H = w.hidden, E = w.experts, K = w.top_k, I = w.intermediate;
  const int Is = w.shared_intermediate;
  const bool has_shared = Is > 0;
  cudaStream_t st = ctx->stream;
  if (T == 0) return ASTRO_MOE_OK;
  const size_t need = plan_workspace(w, T, nullptr, nullptr);
  if (int rc = ensure_ws(ctx, need)) return rc;
  BlockWorkspace b{};
  plan_workspace(w, T, &b, (char*)ctx->ws);
  const int64_t N = T * K;
  const int64_t rows = N + (has_shared ? T : 0);
  const int threshold = ctx->opt.sorted_threshold > 0 ? ctx->opt.sorted_threshold : 64;
  const bool sorted_semantics = N >= threshold;

  StageMarks marks(ctx);
  marks.mark();
  // a1: router projection
  const bool x_aligned = (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
  const bool fused_shape = ctx->opt.decode_fused >= 0 && L.fused_ok &&
                           astro::decode_fused_supported((int)T, H, E, K, I) &&
                           w.shared_intermediate == (has_shared ? I : 0);
  const int64_t decode_max =
      ctx->opt.decode_max_tokens != 0 ? ctx->opt.decode_max_tokens
                                      : (fused_shape ? kDefaultFusedTokens : kDefaultDecodeTokens);
  // small batches: GEMVs over the active experts (HBM-bound); otherwise the
  // tcgen05 grouped GEMMs, or the CUDA-core grouped GEMV when those are off
  const bool use_decode = decode_max > 0 && T <= decode_max && x_aligned && L.decode_ok;
  const bool use_tc = !use_decode && astro::moe_gemm_enabled(L.gemm, ctx->opt.use_tensor_cores) &&
                      x_aligned;
  const bool router_gemv = T <= kRouterGemvTokens && x_aligned && L.router_gemv_ok;
  const bool laguna = w.router_kind == ASTRO_MOE_ROUTER_SIGMOID;
  const bool gated_shared = has_shared && !laguna;
  const size_t score_bytes = laguna ? sizeof(float) : sizeof(uint16_t);
  const bool try_fused = use_decode && fused_shape && !laguna;
  if (try_fused) {
    astro::DecodeFusedArgs a;
    a.x = x;
    a.T = (int)T;
    a.H = H;
    a.E = E;
    a.K = K;
    a.I = I;
    a.normalize = w.normalize_top_k;
    a.sorted = sorted_semantics ? 1 : 0;
    a.has_shared = has_shared ? 1 : 0;
    a.wr = w.router_weight;
    a.wg = w.shared_expert_gate;
    fill_projections(w, a.gate, a.up, a.down);
    a.logits = b.logits;
    a.gate_logit = b.gate_logit;
    a.ids = b.ids;
    a.scores = b.scores;
    a.offsets = b.offsets;
    a.act = b.act;
    a.yrows = b.yrows;
    a.out = out;
    a.barrier = b.barrier;
    a.seg_done = b.barrier + kFusedSegDoneWord;
    a.status = ctx->status;
    // one kernel: its whole time is reported under gate_up_ms
    marks.mark();
    marks.mark();
    const cudaError_t e = astro::launch_decode_fused(a, st);
    if (e == cudaSuccess) {
      ctx->launches += 1;
      ctx->last_path.router = ASTRO_MOE_KERNEL_FUSED_DECODE;
      ctx->last_path.gate_logit = has_shared ? ASTRO_MOE_KERNEL_FUSED_DECODE : ASTRO_MOE_KERNEL_NONE;
      ctx->last_path.experts = ASTRO_MOE_KERNEL_FUSED_DECODE;
      ctx->last_path.shared_expert = has_shared ? ASTRO_MOE_KERNEL_FUSED_DECODE : ASTRO_MOE_KERNEL_NONE;
      marks.mark();
      marks.mark();
      marks.mark();
      marks.commit();
      if (ctx->attribution) ctx->acc.calls += 1;
      return copy_taps(ctx, b, T, E, K, has_shared, taps);
    }
    if (e != cudaErrorCooperativeLaunchTooLarge && e != cudaErrorNotSupported) {
      return cuda_fail(e, "fused decode block");
    }
    cudaGetLastError();  // the device cannot co-schedule the grid: unfused kernels below
    marks.drop(2);
  }
  ctx->launches += 3 + astro::sort_launch_count(N) + (use_tc ? 3 : 2);
  {
    const int ek = use_tc ? ASTRO_MOE_KERNEL_TCGEN05_GEMM
                          : (use_decode ? ASTRO_MOE_KERNEL_DECODE_GEMV : ASTRO_MOE_KERNEL_GROUPED_GEMV);
    ctx->last_path.router = router_gemv ? ASTRO_MOE_KERNEL_ROUTER_GEMV
                                        : (use_tc ? ASTRO_MOE_KERNEL_TCGEN05_GEMM : ASTRO_MOE_KERNEL_SIMT_GEMM);
    ctx->last_path.gate_logit = gated_shared ? ASTRO_MOE_KERNEL_ROUTE : ASTRO_MOE_KERNEL_NONE;
    ctx->last_path.experts = ek;
    ctx->last_path.shared_expert =
        has_shared ? (L.shared_separate ? ASTRO_MOE_KERNEL_GROUPED_GEMV : ek) : ASTRO_MOE_KERNEL_NONE;
  }
  if (L.shared_separate) ctx->launches += 2;
  if (router_gemv) {
    CK(astro::launch_router_gemv(x, T, w.router_weight, E, H, b.logits, st), "router projection");
  } else if (use_tc) {
    CK(astro::moe_gemm_router(L.gemm, x, T, b.logits, b.gemm_scratch, ctx->status, st),
       "router projection");
  } else {
    CK(astro::launch_dense_nt_simt(x, w.router_weight, T, E, H, b.logits, E, st), "router projection");
  }
  marks.mark();
  // a2: route (+ shared-expert gate logit); Laguna: sigmoid routing, fp32 scores
  if (laguna) {
    CK(astro::launch_route_laguna(b.logits, ASTRO_MOE_DTYPE_BF16, T, E, K, w.router_logit_softcap,
                                  w.router_correction_bias, w.normalize_top_k, b.ids,
                                  reinterpret_cast<float*>(b.scores), st),
       "route Laguna experts");
  } else {
    CK(astro::launch_route_experts(b.logits, ASTRO_MOE_DTYPE_BF16, T, E, K, w.normalize_top_k,
                                   b.ids, b.scores, x, has_shared ? w.shared_expert_gate : nullptr,
                                   H, has_shared ? b.gate_logit : nullptr, st),
       "route experts");
  }
  // a3: sort (+ shared segment E)
  CK(astro::launch_sort_assignments(b.ids, T, K, E, has_shared ? T : 0, b.order, b.inverse,
                                    b.sids, b.stok, b.offsets, ctx->status, b.sort_scratch, st),
     "sort expert assignments");

  if (use_tc) {
    // a4-a6 on tcgen05: gather rows, gate/up + SwiGLU, down
    // token rows in the grouped GEMMs' K order (perm8_bf16)
    CK(astro::launch_take_rows(x, T, b.stok, rows, H, b.states, ctx->status, st, true),
       "take rows");
    marks.mark();
    CK(astro::moe_gemm_gate_up(L.gemm, b.states, rows, b.offsets, b.act, b.gemm_scratch,
                               ctx->status, st),
       "gate/up projection");
    marks.mark();
    CK(astro::moe_gemm_down(L.gemm, b.act, rows, b.offsets, b.yrows, b.gemm_scratch,
                            ctx->status, st),
       "down projection");
  } else {
    marks.mark();
    // a4-a6 on CUDA cores: the decode GEMVs, or the grouped GEMV tiles; the shared
    // expert is segment E
    astro::GroupedGemvDesc d;
    d.x = x;
    d.x_rows = b.stok;
    d.x_limit = T;
    d.in_features = H;
    d.seg_offsets = b.offsets;
    d.nseg = E + (has_shared && !L.shared_separate ? 1 : 0);
    d.shared_seg = has_shared && !L.shared_separate ? E : -1;
    d.rows_total = rows;
    if (w.gate_up_fused) {
      d.wa[0] = astro::AffineRef{w.gate.packed, w.gate.scales, w.gate.biases, 2LL * I, 0};
      d.wb[0] = astro::AffineRef{w.gate.packed, w.gate.scales, w.gate.biases, 2LL * I, I};
    } else {
      d.wa[0] = astro::AffineRef{w.gate.packed, w.gate.scales, w.gate.biases, I, 0};
      d.wb[0] = astro::AffineRef{w.up.packed, w.up.scales, w.up.biases, I, 0};
    }
    if (has_shared) {
      d.wa[1] = astro::AffineRef{w.shared_gate.packed, w.shared_gate.scales, w.shared_gate.biases, Is, 0};
      d.wb[1] = astro::AffineRef{w.shared_up.packed, w.shared_up.scales, w.shared_up.biases, Is, 0};
    }
    d.out_features = I;
    d.group = L.qgroup[0];
    d.bits = L.qbits[0];
    d.swiglu = true;
    d.y = b.act;
    d.y_limit = rows;
    d.ldy = I;
    d.status = ctx->status;
    const int64_t max_active = (N < E ? N : E) + (has_shared ? 1 : 0);
    if (use_decode) {
      CK(astro::launch_decode_gate_up(d, max_active, st), "gate/up projection");
    } else {
      CK(astro::launch_grouped_gemv(d, st), "gate/up projection");
    }
    marks.mark();
    astro::GroupedGemvDesc dd = d;
    dd.x = b.act;
    dd.x_rows = nullptr;
    dd.x_limit = rows;
    dd.in_features = I;
    dd.wa[0] = astro::AffineRef{w.down.packed, w.down.scales, w.down.biases, H, 0};
    if (has_shared)
      dd.wa[1] = astro::AffineRef{w.shared_down.packed, w.shared_down.scales, w.shared_down.biases, H, 0};
    dd.wb[0] = dd.wb[1] = astro::AffineRef{};
    dd.out_features = H;
    dd.group = L.qgroup[2];
    dd.bits = L.qbits[2];
    dd.swiglu = false;
    dd.y = b.yrows;
    dd.ldy = H;
    if (use_decode) {
      CK(astro::launch_decode_down(dd, max_active, st), "down projection");
    } else {
      CK(astro::launch_grouped_gemv(dd, st), "down projection");
    }
  }
  if (L.shared_separate) {
    // a shared expert quantised unlike the routed experts: its own grouped-GEMV
    // launches over its rows [N, N + T) (segment E of the sort), same outputs
    astro::GroupedGemvDesc d;
    d.x = x;
    d.x_rows = b.stok;
    d.x_limit = T;
    d.in_features = H;
    d.seg_offsets = b.offsets + E;
    d.nseg = 1;
    d.shared_seg = 0;
    d.rows_total = rows;
    d.wa[1] = astro::AffineRef{w.shared_gate.packed, w.shared_gate.scales, w.shared_gate.biases, Is, 0};
    d.wb[1] = astro::AffineRef{w.shared_up.packed, w.shared_up.scales, w.shared_up.biases, Is, 0};
    d.out_features = I;
    d.group = L.qgroup[3];
    d.bits = L.qbits[3];
    d.swiglu = true;
    d.y = b.act;
    d.y_limit = rows;
    d.ldy = I;
    d.status = ctx->status;
    CK(astro::launch_grouped_gemv(d, st), "shared expert gate/up projection");
    astro::GroupedGemvDesc dd = d;
    dd.x = b.act;
    dd.x_rows = nullptr;
    dd.x_limit = rows;
    dd.in_features = I;
    dd.wa[1] = astro::AffineRef{w.shared_down.packed, w.shared_down.scales, w.shared_down.biases, H, 0};
    dd.wb[1] = astro::AffineRef{};
    dd.out_features = H;
    dd.group = L.qgroup[5];
    dd.bits = L.qbits[5];
    dd.swiglu = false;
    dd.y = b.yrows;
    dd.ldy = H;
    CK(astro::launch_grouped_gemv(dd, st), "shared expert down projection");
  }
  marks.mark();
  // a7 + a8: weighted sum fused with the shared expert and its gate
  if (laguna) {
    const float f = w.routed_scaling_factor > 0.0f ? w.routed_scaling_factor : 1.0f;
    CK(astro::launch_block_combine(b.yrows, b.inverse, nullptr, nullptr, N, T, K, H,
                                   sorted_semantics ? 1 : 0, out, st,
                                   reinterpret_cast<const float*>(b.scores), has_shared ? 1 : 0,
                                   __bfloat162float(__float2bfloat16_rn(f))),
       "weighted combine");
  } else {
    CK(astro::launch_block_combine(b.yrows, b.inverse, b.scores, has_shared ? b.gate_logit : nullptr,
                                   N, T, K, H, sorted_semantics ? 1 : 0, out, st),
       "weighted combine");
  }
  marks.mark();
  marks.commit();
  if (ctx->attribution) ctx->acc.calls += 1;
  return copy_taps(ctx, b, T, E, K, has_shared, taps, score_bytes);
}

// geometry and pointer checks of one layer's weights (register_layer and the
// expert-parallel registration)
// {bits, group} of a projection: its own when set, else the layer's
void eff_quant(const astro_moe_affine& a, const astro_moe_layer_weights& w, int* bits, int* group) {
  *bits = a.bits > 0 ? a.bits : w.bits;
  *group = a.group_size > 0 ? a.group_size : w.group_size;
}

// quantisation of gate, up, down, shared gate, shared up, shared down
void layer_quant(const astro_moe_layer_weights& w, int (&bits)[6], int (&group)[6]) {
  eff_quant(w.gate, w, &bits[0], &group[0]);
  if (w.gate_up_fused) {
    bits[1] = bits[0];
    group[1] = group[0];
  } else {
    eff_quant(w.up, w, &bits[1], &group[1]);
  }
  eff_quant(w.down, w, &bits[2], &group[2]);
  eff_quant(w.shared_gate, w, &bits[3], &group[3]);
  eff_quant(w.shared_up, w, &bits[4], &group[4]);
  eff_quant(w.shared_down, w, &bits[5], &group[5]);
}

// geometry and pointer checks of one layer's weights (register_layer and the
// expert-parallel registration); routed_stacks = false skips the routed expert
// stacks (a paged layer's come from its pages)
int validate_layer(const char* op, const astro_moe_layer_weights* w, bool routed_stacks = true) {
  if (w->hidden <= 0 || w->experts <= 0 || w->top_k <= 0 || w->top_k > w->experts ||
      w->intermediate <= 0 || w->shared_intermediate < 0)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: invalid geometry", op);
  if (w->top_k > 32 || w->experts > 1024)
    return fail(ASTRO_MOE_ERR_UNSUPPORTED, "%s: top_k <= 32 and experts <= 1024 are supported", op);
  if (w->hidden % 8 != 0) return fail(ASTRO_MOE_ERR_UNSUPPORTED, "%s: hidden must be a multiple of 8", op);
  int qb[6], qg[6];
  layer_quant(*w, qb, qg);
  if (routed_stacks) {
    if (int rc = check_affine(op, w->hidden, qg[0], qb[0])) return rc;
    if (int rc = check_affine(op, w->hidden, qg[1], qb[1])) return rc;
    if (int rc = check_affine(op, w->intermediate, qg[2], qb[2])) return rc;
    if (qb[0] != qb[1] || qg[0] != qg[1])
      return fail(ASTRO_MOE_ERR_UNSUPPORTED,
                  "%s: the gate and up projections must share their bits and group size", op);
  }
  const bool has_shared = w->shared_intermediate > 0;
  if (has_shared) {
    if (int rc = check_affine(op, w->hidden, qg[3], qb[3])) return rc;
    if (int rc = check_affine(op, w->hidden, qg[4], qb[4])) return rc;
    if (int rc = check_affine(op, w->shared_intermediate, qg[5], qb[5])) return rc;
    if (qb[3] != qb[4] || qg[3] != qg[4])
      return fail(ASTRO_MOE_ERR_UNSUPPORTED,
                  "%s: the shared gate and shared up projections must share their bits and group size", op);
  }
  if (w->shared_intermediate != 0 && w->shared_intermediate != w->intermediate)
    return fail(ASTRO_MOE_ERR_UNSUPPORTED,
                "%s: the shared expert must have the routed intermediate width (or be absent)", op);
  if (w->router_kind != ASTRO_MOE_ROUTER_SOFTMAX && w->router_kind != ASTRO_MOE_ROUTER_SIGMOID)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: unknown router kind %d", op, (int)w->router_kind);
  if (w->router_kind == ASTRO_MOE_ROUTER_SIGMOID &&
      (w->router_logit_softcap != w->router_logit_softcap || w->router_logit_softcap < 0.0f ||
       w->routed_scaling_factor != w->routed_scaling_factor || w->routed_scaling_factor < 0.0f))
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT,
                "%s: the Laguna softcap and routed scaling factor must be >= 0", op);
  if (!w->router_weight) {
    if (!w->router_affine.packed)
      return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null router weight (bf16 or affine)", op);
    if (int rc = validate_affine_tensor("affine router", w->router_affine)) return rc;
    int rb, rg;
    eff_quant(w->router_affine, *w, &rb, &rg);
    if (int rc = check_affine(op, w->hidden, rg, rb)) return rc;
  }
  if (routed_stacks) {
    if (int rc = validate_affine_tensor("gate", w->gate)) return rc;
    if (!w->gate_up_fused)
      if (int rc = validate_affine_tensor("up", w->up)) return rc;
    if (int rc = validate_affine_tensor("down", w->down)) return rc;
  }
  if (has_shared) {
    if (int rc = validate_affine_tensor("shared gate", w->shared_gate)) return rc;
    if (int rc = validate_affine_tensor("shared up", w->shared_up)) return rc;
    if (int rc = validate_affine_tensor("shared down", w->shared_down)) return rc;
    if (!w->shared_expert_gate && w->router_kind == ASTRO_MOE_ROUTER_SOFTMAX) {
      if (!w->shared_expert_gate_affine.packed)
        return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null shared expert gate (bf16 or affine)", op);
      if (int rc = validate_affine_tensor("affine shared expert gate", w->shared_expert_gate_affine))
        return rc;
      int gb, gg;
      eff_quant(w->shared_expert_gate_affine, *w, &gb, &gg);
      if (int rc = check_affine(op, w->hidden, gg, gb)) return rc;
    }
  }
  return ASTRO_MOE_OK;
}

// Takes a validated layer into L: per-projection quantisation, bf16 copies of an
// affine router / shared-expert gate (router_rows rows of the router), and the
// weights the kernels read (L.w: dense router and gate pointers, bits / group of
// the routed gate/up).  Synchronises the context stream after any dequantisation.
int resolve_layer(astro_moe_ctx* ctx, const astro_moe_layer_weights* in, int router_rows,
                  LayerState& L) {
  release_layer(L);
  L.w = *in;
  layer_quant(*in, L.qbits, L.qgroup);
  L.w.bits = L.qbits[0];
  L.w.group_size = L.qgroup[0];
  const bool has_shared = in->shared_intermediate > 0;
  L.shared_separate = has_shared && (L.qbits[3] != L.qbits[0] || L.qgroup[3] != L.qgroup[0] ||
                                     L.qbits[5] != L.qbits[2] || L.qgroup[5] != L.qgroup[2]);
  bool sync = false;
  if (!in->router_weight) {
    int rb, rg;
    eff_quant(in->router_affine, *in, &rb, &rg);
    CK(cudaMalloc(&L.router_dense, sizeof(uint16_t) * (size_t)router_rows * in->hidden),
       "cudaMalloc(dequantised router)");
    CK(astro::launch_dequantize_affine(in->router_affine.packed, in->router_affine.scales,
                                       in->router_affine.biases, router_rows, in->hidden, rg, rb,
                                       L.router_dense, ctx->stream),
       "dequantise router");
    L.w.router_weight = L.router_dense;
    sync = true;
  }
  if (has_shared && !in->shared_expert_gate && in->router_kind == ASTRO_MOE_ROUTER_SOFTMAX) {
    int gb, gg;
    eff_quant(in->shared_expert_gate_affine, *in, &gb, &gg);
    CK(cudaMalloc(&L.sgate_dense, sizeof(uint16_t) * (size_t)in->hidden),
       "cudaMalloc(dequantised shared expert gate)");
    CK(astro::launch_dequantize_affine(in->shared_expert_gate_affine.packed,
                                       in->shared_expert_gate_affine.scales,
                                       in->shared_expert_gate_affine.biases, 1, in->hidden, gg, gb,
                                       L.sgate_dense, ctx->stream),
       "dequantise shared expert gate");
    L.w.shared_expert_gate = L.sgate_dense;
    sync = true;
  }
  if (sync) CK(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
  return ASTRO_MOE_OK;
}

// every projection in [first, last] is 4-bit, group 64 (the tcgen05 / decode kernels)
bool q4g64(const LayerState& L, int first, int last) {
  for (int i = first; i <= last; ++i)
    if (L.qbits[i] != 4 || L.qgroup[i] != 64) return false;
  return true;
}

int devbuf_ensure(astro_moe_ctx* ctx, DevBuf& b, size_t bytes) {
  if (b.bytes >= bytes) return ASTRO_MOE_OK;
  if (b.p) {
    CK(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    cudaFree(b.p);
    b.p = nullptr;
    b.bytes = 0;
  }
  CK(cudaMalloc(&b.p, bytes), "cudaMalloc(expert-parallel buffers)");
  b.bytes = bytes;
  return ASTRO_MOE_OK;
}

// dispatch-side arrays of an expert-parallel layer for T tokens
struct EpDispatch {
  uint16_t* logits;
  uint32_t* ids;
  uint16_t* scores;
  uint16_t* gate_logit;
  uint32_t* order;
  uint32_t* inverse;
  uint32_t* sids;
  uint32_t* stok;
  void* sort_scratch;
};
size_t plan_ep_dispatch(int64_t T, int E, int K, EpDispatch* out, char* base) {
  const int64_t N = T * K;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    char* p = base ? base + off : nullptr;
    off = align_up(off + bytes, 256);
    return p;
  };
  EpDispatch d{};
  d.logits = (uint16_t*)take(sizeof(uint16_t) * T * E);
  d.ids = (uint32_t*)take(sizeof(uint32_t) * N);
  d.scores = (uint16_t*)take(sizeof(uint16_t) * N);
  d.gate_logit = (uint16_t*)take(sizeof(uint16_t) * T);
  d.order = (uint32_t*)take(sizeof(uint32_t) * N);
  d.inverse = (uint32_t*)take(sizeof(uint32_t) * N);
  d.sids = (uint32_t*)take(sizeof(uint32_t) * N);
  d.stok = (uint32_t*)take(sizeof(uint32_t) * N);
  d.sort_scratch = take(astro::sort_scratch_bytes(N, E));
  if (out) *out = d;
  return off;
}

// expert-side arrays for `rows` expert-major rows (received + shared)
struct EpExperts {
  uint16_t* states;
  uint16_t* act;
  uint16_t* yrows;
  uint32_t* src_start;
  uint32_t* exp_start;
  uint32_t* offsets;
  uint32_t* dest;
  uint32_t* src_of;
  void* gemm_scratch;
};
size_t plan_ep_experts(int64_t rows, int64_t n_recv, int H, int I, int runs, int El, EpExperts* out,
                       char* base) {
  size_t off = 0;
  auto take = [&](size_t bytes) {
    char* p = base ? base + off : nullptr;
    off = align_up(off + bytes, 256);
    return p;
  };
  EpExperts e{};
  e.states = (uint16_t*)take(sizeof(uint16_t) * rows * H);
  e.act = (uint16_t*)take(sizeof(uint16_t) * rows * I);
  e.yrows = (uint16_t*)take(sizeof(uint16_t) * rows * H);
  e.src_start = (uint32_t*)take(sizeof(uint32_t) * runs);
  e.exp_start = (uint32_t*)take(sizeof(uint32_t) * runs);
  e.offsets = (uint32_t*)take(sizeof(uint32_t) * (El + 2));
  e.dest = (uint32_t*)take(sizeof(uint32_t) * (n_recv > 0 ? n_recv : 1));
  e.src_of = (uint32_t*)take(sizeof(uint32_t) * (n_recv > 0 ? n_recv : 1));
  e.gemm_scratch = take(astro::moe_gemm_scratch_bytes());
  if (out) *out = e;
  return off;
}

int ep_layer(astro_moe_ctx* ctx, int32_t layer, const char* op, LayerState** out) {
  if (!ctx) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null ctx", op);
  auto it = ctx->layers.find(layer);
  if (it == ctx->layers.end() || !it->second.registered)
    return fail(ASTRO_MOE_ERR_NOT_REGISTERED, "%s: layer %d is not registered", op, layer);
  if (!it->second.ep)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: layer %d is not an expert-parallel layer", op, layer);
  *out = &it->second;
  return ASTRO_MOE_OK;
}

// page-major view of the pager's pool as stacked tensors (slot = expert index)
astro::AffineRef pool_ref(const astro_moe_pager* pg, int m, int64_t code_row_bytes, int64_t sb_row_bytes) {
  astro::AffineRef r;
  r.q = pg->pool + pg->off_q[m];
  r.s = pg->pool + pg->off_s[m];
  r.b = pg->pool + pg->off_b[m];
  r.expert_rows = pg->page_bytes / code_row_bytes;
  r.sb_expert_rows = pg->page_bytes / sb_row_bytes;
  r.row_offset = 0;
  return r;
}

// LRU admission of the experts one block call routes to; returns the number of
// page copies issued on the pager's copy stream.
// Victim slot for a miss once the cache is full, by the pager's policy; never a
// slot the current call has touched (its experts run from it).
int64_t pick_victim(astro_moe_pager* pg) {
  if (pg->policy == ASTRO_MOE_PAGER_DEMAND) {
    // least demand, then least recently used: walk the LRU list from its tail
    int64_t best = -1;
    uint64_t best_d = 0;
    for (auto it = pg->lru.rbegin(); it != pg->lru.rend(); ++it) {
      const int64_t sl = *it;
      if (pg->last_call[sl] == pg->call) continue;
      if (pg->page_of_slot[sl] < 0) return sl;  // holds no page (a failed copy)
      const uint64_t d = pg->demand[pg->page_of_slot[sl]];
      if (best < 0 || d < best_d) {
        best = sl;
        best_d = d;
        if (d == 0) break;
      }
    }
    if (best >= 0) return best;
  }
  auto it = pg->lru.end();
  do {
    --it;
  } while (pg->last_call[*it] == pg->call && it != pg->lru.begin());
  return *it;
}

int64_t admit_pages(astro_moe_pager* pg, int layer, const uint32_t* offs, int* failed) {
  *failed = 0;
  // one call's pages must all fit: a page this call routes to is never evicted
  // by it
  int64_t needed = 0;
  for (int e = 0; e < pg->E; ++e) needed += offs[e + 1] > offs[e] ? 1 : 0;
  if (needed > pg->slots) {
    *failed = 2;
    return needed;
  }
  pg->call += 1;
  int64_t copies = 0;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  for (int e = 0; e < pg->E; ++e) {
    pg->h_table[e] = 0;
    pg->missed[e] = 0;
    if (offs[e + 1] <= offs[e]) continue;
    const int64_t page = (int64_t)layer * pg->E + e;
    pg->st.lookups += 1;
    pg->demand[page] += offs[e + 1] - offs[e];
    int64_t slot = pg->slot_of_page[page];
    if (slot >= 0) {
      pg->st.hits += 1;
      pg->lru.splice(pg->lru.begin(), pg->lru, pg->lru_pos[slot]);
    } else {
      pg->st.misses += 1;
      if (pg->used < pg->slots) {
        slot = pg->used++;
        pg->lru.push_front(slot);
        pg->lru_pos[slot] = pg->lru.begin();
      } else {
        slot = pick_victim(pg);
        if (pg->page_of_slot[slot] >= 0) {
          pg->slot_of_page[pg->page_of_slot[slot]] = -1;
          pg->st.evictions += 1;
        }
        pg->page_of_slot[slot] = -1;
        pg->lru.splice(pg->lru.begin(), pg->lru, pg->lru_pos[slot]);
      }
      pg->slot_of_page[page] = (int32_t)slot;
      pg->page_of_slot[slot] = page;
      if (copies == 0) {
        if (pg->spare.empty()) {
          cudaEventCreate(&e0);
          cudaEventCreate(&e1);
        } else {
          e0 = pg->spare.back().first;
          e1 = pg->spare.back().second;
          pg->spare.pop_back();
        }
        cudaEventRecord(e0, pg->copy);
      }
      cudaError_t ce = cudaErrorInvalidValue;
      if (pg->inject_copy_failures > 0) {
        pg->inject_copy_failures -= 1;
      } else {
        ce = cudaMemcpyAsync(pg->pool + slot * pg->page_bytes, pg->host + page * pg->page_bytes,
                             (size_t)pg->page_bytes, cudaMemcpyHostToDevice, pg->copy);
      }
      if (ce != cudaSuccess) {
        // the page never arrived: the slot holds no page, the call fails
        pg->slot_of_page[page] = -1;
        pg->page_of_slot[slot] = -1;
        pg->st.copy_failures += 1;
        *failed = 1;
      } else {
        pg->st.bytes_h2d += pg->page_bytes;
      }
      copies += 1;
      pg->missed[e] = 1;
    }
    pg->last_call[slot] = pg->call;
    pg->h_table[e] = (uint32_t)slot;
  }
  // a slot that this call touched is never evicted by it, so the resident
  // experts' slots stay valid while the copies land
  for (int e = 0; e < pg->E; ++e) {
    const uint32_t slot = pg->h_table[e];
    pg->h_table[pg->E + e] = pg->missed[e] ? slot : astro::kSlotElsewhere;
    if (pg->missed[e]) pg->h_table[e] = astro::kSlotElsewhere;
  }
  if (copies) {
    cudaEventRecord(e1, pg->copy);
    pg->pending.emplace_back(e0, e1);
  }
  pg->st.resident_pages = pg->used;
  return copies;
}

int run_paged_block(astro_moe_ctx* ctx, LayerState& L, int layer, const void* x, int64_t T, void* out) {
  const char* op = "paged block forward";
  astro_moe_pager* pg = L.pager;
  const astro_moe_layer_weights& w = L.w;
  const int H = w.hidden, E = w.experts, K = w.top_k, I = w.intermediate;
  const bool has_shared = w.shared_intermediate > 0;
  cudaStream_t st = ctx->stream;
  if (T == 0) return ASTRO_MOE_OK;
  const size_t need = plan_workspace(w, T, nullptr, nullptr);
  if (int rc = ensure_ws(ctx, need)) return rc;
  BlockWorkspace b{};
  plan_workspace(w, T, &b, (char*)ctx->ws);
  const int64_t N = T * K;
  const int64_t rows = N + (has_shared ? T : 0);
  const int threshold = ctx->opt.sorted_threshold > 0 ? ctx->opt.sorted_threshold : 64;
  // more than kPagedDecodeTokens tokens (prefill): the whole call's pages are
  // brought in, then the tcgen05 grouped GEMMs read them through the slot table,
  // exactly as the resident block computes (its router included)
  const bool prefill = T > kPagedDecodeTokens &&
                       astro::moe_gemm_enabled(L.gemm, ctx->opt.use_tensor_cores);
  const bool router_gemv = !prefill && L.router_gemv_ok;
  ctx->last_path.router = router_gemv ? ASTRO_MOE_KERNEL_ROUTER_GEMV
                                      : (prefill ? ASTRO_MOE_KERNEL_TCGEN05_GEMM : ASTRO_MOE_KERNEL_SIMT_GEMM);
  ctx->last_path.gate_logit = has_shared ? ASTRO_MOE_KERNEL_ROUTE : ASTRO_MOE_KERNEL_NONE;
  ctx->last_path.experts = prefill ? ASTRO_MOE_KERNEL_TCGEN05_GEMM : ASTRO_MOE_KERNEL_DECODE_GEMV;
  ctx->last_path.shared_expert = has_shared ? ctx->last_path.experts : ASTRO_MOE_KERNEL_NONE;
  if (router_gemv) {
    CK(astro::launch_router_gemv(x, T, w.router_weight, E, H, b.logits, st), "router projection");
  } else if (prefill) {
    CK(astro::moe_gemm_router(L.gemm, x, T, b.logits, b.gemm_scratch, ctx->status, st),
       "router projection");
  } else {
    CK(astro::launch_dense_nt_simt(x, w.router_weight, T, E, H, b.logits, E, st), "router projection");
  }
  CK(astro::launch_route_experts(b.logits, ASTRO_MOE_DTYPE_BF16, T, E, K, w.normalize_top_k, b.ids,
                                 b.scores, x, has_shared ? w.shared_expert_gate : nullptr, H,
                                 has_shared ? b.gate_logit : nullptr, st),
     "route experts");
  CK(astro::launch_sort_assignments(b.ids, T, K, E, has_shared ? T : 0, b.order, b.inverse, b.sids,
                                    b.stok, b.offsets, ctx->status, b.sort_scratch, st),
     "sort expert assignments");
  // the routed experts, back on the host (the reference's pager syncs here too)
  CK(cudaMemcpyAsync(pg->h_offsets, b.offsets, sizeof(uint32_t) * (E + 2), cudaMemcpyDeviceToHost, st),
     "read back expert offsets");
  CK(cudaStreamSynchronize(st), "cudaStreamSynchronize");
  int copy_failed = 0;
  const int64_t copies = admit_pages(pg, layer, pg->h_offsets, &copy_failed);
  if (copy_failed == 2)
    return fail(ASTRO_MOE_ERR_MEMORY_LIMIT,
                "%s: the cache of %lld pages cannot hold the %lld expert pages this call routes to "
                "(layer %d)",
                op, (long long)pg->slots, (long long)copies, layer);
  if (copy_failed) {
    // a routed expert's page did not reach HBM: nothing reads the cache this
    // call (the issued copies finish on the copy stream and stay valid)
    pg->st.calls += 1;
    return fail(ASTRO_MOE_ERR_CUDA,
                "%s: an expert page copy to HBM failed (layer %d); no output was written", op, layer);
  }
  if (prefill) {
    // one table, every routed expert's slot; the GEMMs start once the copies
    // have landed
    for (int e = 0; e < E; ++e)
      if (pg->h_table[e] == astro::kSlotElsewhere) pg->h_table[e] = pg->h_table[E + e];
    CK(cudaMemcpyAsync(pg->d_table, pg->h_table, sizeof(uint32_t) * E, cudaMemcpyHostToDevice, st),
       "slot table");
    if (copies) {
      CK(cudaEventRecord(pg->ready, pg->copy), op);
      CK(cudaStreamWaitEvent(st, pg->ready, 0), op);
    }
    CK(astro::launch_take_rows(x, T, b.stok, rows, H, b.states, ctx->status, st, true), "take rows");
    CK(astro::moe_gemm_gate_up(L.gemm, b.states, rows, b.offsets, b.act, b.gemm_scratch, ctx->status,
                               st, pg->d_table),
       "gate/up projection");
    CK(astro::moe_gemm_down(L.gemm, b.act, rows, b.offsets, b.yrows, b.gemm_scratch, ctx->status,
                            st, pg->d_table),
       "down projection");
    CK(astro::launch_block_combine(b.yrows, b.inverse, b.scores, has_shared ? b.gate_logit : nullptr,
                                   N, T, K, H, N >= threshold ? 1 : 0, out, st),
       "weighted combine");
    ctx->launches += 8 + astro::sort_launch_count(N);
    pg->st.calls += 1;
    return ASTRO_MOE_OK;
  }
  // the slot tables travel on the compute stream (the next layer's read-back
  // sync covers them before the host rewrites the pinned copy); the experts whose
  // pages are resident are computed while the missing pages copy
  CK(cudaMemcpyAsync(pg->d_table, pg->h_table, sizeof(uint32_t) * 2 * E, cudaMemcpyHostToDevice, st),
     "slot tables");
  if (copies) CK(cudaEventRecord(pg->ready, pg->copy), op);
  astro::GroupedGemvDesc d;
  d.x = x;
  d.x_rows = b.stok;
  d.x_limit = T;
  d.in_features = H;
  d.seg_offsets = b.offsets;
  d.nseg = E + (has_shared ? 1 : 0);
  d.shared_seg = has_shared ? E : -1;
  d.rows_total = rows;
  astro::AffineRef g[2], u[2], dn[2];
  fill_projections(w, g, u, dn);  // shared expert refs (the routed ones are replaced)
  d.wa[0] = pool_ref(pg, 0, (int64_t)H * pg->bits / 8, (int64_t)(H / pg->group) * 2);
  d.wb[0] = pool_ref(pg, 1, (int64_t)H * pg->bits / 8, (int64_t)(H / pg->group) * 2);
  d.wa[1] = g[1];
  d.wb[1] = u[1];
  d.out_features = I;
  d.group = w.group_size;
  d.bits = w.bits;
  d.swiglu = true;
  d.y = b.act;
  d.y_limit = rows;
  d.ldy = I;
  d.status = ctx->status;
  d.slot_of = pg->d_table;
  const int64_t max_active = (N < E ? N : E) + (has_shared ? 1 : 0);
  astro::GroupedGemvDesc dd = d;
  dd.x = b.act;
  dd.x_rows = nullptr;
  dd.x_limit = rows;
  dd.in_features = I;
  dd.wa[0] = pool_ref(pg, 2, (int64_t)I * pg->bits / 8, (int64_t)(I / pg->group) * 2);
  dd.wa[1] = dn[1];
  dd.wb[0] = dd.wb[1] = astro::AffineRef{};
  dd.out_features = H;
  dd.swiglu = false;
  dd.y = b.yrows;
  dd.ldy = H;
  // resident experts and the shared expert, then (after the copies) the rest
  CK(astro::launch_decode_gate_up(d, max_active, st), "gate/up projection");
  CK(astro::launch_decode_down(dd, max_active, st), "down projection");
  if (copies) {
    CK(cudaStreamWaitEvent(st, pg->ready, 0), op);
    d.slot_of = dd.slot_of = pg->d_table + E;
    d.skip_shared = dd.skip_shared = true;
    CK(astro::launch_decode_gate_up(d, max_active, st), "gate/up projection (copied pages)");
    CK(astro::launch_decode_down(dd, max_active, st), "down projection (copied pages)");
  }
  CK(astro::launch_block_combine(b.yrows, b.inverse, b.scores, has_shared ? b.gate_logit : nullptr,
                                 N, T, K, H, N >= threshold ? 1 : 0, out, st),
     "weighted combine");
  ctx->launches += 6 + (copies ? 2 : 0) + astro::sort_launch_count(N);
  pg->st.calls += 1;
  if (copies) pg->st.split_calls += 1;
  return ASTRO_MOE_OK;
}

}  // namespace

int astro::set_last_error(int status, const char* message) {
  g_last_error = message;
  return status;
}

extern "C" {

const char* astro_moe_last_error(void) { return g_last_error.c_str(); }
int astro_moe_abi_version(void) { return ASTRO_MOE_ABI_VERSION; }

int astro_moe_device_status(int32_t device, uint32_t* status, int32_t reset) {
  if (!status) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "device status: null output");
  DeviceGuard g(device);
  uint32_t* p = nullptr;
  if (int rc = device_status_ptr(&p)) return rc;
  CK(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  CK(cudaMemcpy(status, p, sizeof(uint32_t), cudaMemcpyDeviceToHost), "read device status");
  if (reset) CK(cudaMemset(p, 0, sizeof(uint32_t)), "reset device status");
  return ASTRO_MOE_OK;
}

int astro_moe_route_experts(const void* logits, int32_t dtype, int64_t tokens, int32_t experts,
                            int32_t top_k, int32_t normalize, uint32_t* ids, void* scores,
                            void* stream) {
  const char* op = "route Qwen3.5-MoE sparse experts";
  if (!valid_dtype(dtype))
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: router logits must use float16, bfloat16, or float32", op);
  if (tokens < 0) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: negative token count", op);
  if (experts <= 0 || top_k <= 0 || top_k > experts)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT,
                "%s: selected expert count must be positive and no larger than the router dimension", op);
  if (top_k > 32 || experts > 1024)
    return fail(ASTRO_MOE_ERR_UNSUPPORTED, "%s: top_k <= 32 and experts <= 1024 are supported", op);
  if (tokens > 0 && (!logits || !ids || !scores))
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null array", op);
  CK(astro::launch_route_experts(logits, dtype, tokens, experts, top_k, normalize, ids, scores,
                                 nullptr, nullptr, 0, nullptr, S(stream)),
     op);
  return ASTRO_MOE_OK;
}

int astro_moe_route_laguna_experts(const void* logits, int32_t dtype, int64_t tokens,
                                   int32_t experts, int32_t top_k, const float* correction_bias,
                                   double router_logit_softcap, int32_t normalize, uint32_t* ids,
                                   float* scores, void* stream) {
  const char* op = "route Laguna experts";
  if (!valid_dtype(dtype))
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: router logits must use float16, bfloat16, or float32", op);
  // validate_router_geometry, laguna/moe/router_selection.rs:127-150
  if (tokens < 0 || experts <= 0 || top_k <= 0 || top_k > experts ||
      router_logit_softcap != router_logit_softcap || router_logit_softcap < 0.0)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT,
                "%s: Laguna router logits, top-K, and softcap must describe a valid selection", op);
  if (top_k > 32 || experts > 1024)
    return fail(ASTRO_MOE_ERR_UNSUPPORTED, "%s: top_k <= 32 and experts <= 1024 are supported", op);
  if (tokens > 0 && (!logits || !ids || !scores))
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null array", op);
  CK(astro::launch_route_laguna(logits, dtype, tokens, experts, top_k, (float)router_logit_softcap,
                                correction_bias, normalize, ids, scores, S(stream)),
     op);
  return ASTRO_MOE_OK;
}

int astro_moe_sort_expert_assignments(const uint32_t* ids, int64_t tokens, int32_t top_k,
                                      int32_t experts, uint32_t* sorted_order,
                                      uint32_t* inverse_order, uint32_t* sorted_ids,
                                      uint32_t* sorted_tokens, uint32_t* expert_offsets,
                                      void* stream) {
  const char* op = "sort stacked expert assignments";
  if (tokens < 0 || top_k < 0 || experts <= 0)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: expert assignments have invalid shapes", op);
  if (experts > 1024) return fail(ASTRO_MOE_ERR_UNSUPPORTED, "%s: experts <= 1024 are supported", op);
  if (tokens * (int64_t)top_k > 0xffffffffLL)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: expert assignment count exceeds the integer range", op);
  if (tokens * top_k > 0 && !ids) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null ids", op);
  uint32_t* status = nullptr;
  if (int rc = device_status_ptr(&status)) return rc;
  const int64_t n = tokens * (int64_t)top_k;
  const size_t scratch_bytes = astro::sort_scratch_bytes(n, experts);
  char* tmp = nullptr;
  CK(cudaMallocAsync((void**)&tmp, scratch_bytes + sizeof(uint32_t) * (experts + 1), S(stream)),
     "cudaMallocAsync");
  uint32_t* offs = expert_offsets ? expert_offsets : (uint32_t*)(tmp + scratch_bytes);
  CK(astro::launch_sort_assignments(ids, tokens, top_k, experts, 0, sorted_order, inverse_order,
                                    sorted_ids, sorted_tokens, offs, status, tmp, S(stream)),
     op);
  CK(cudaFreeAsync(tmp, S(stream)), "cudaFreeAsync");
  return ASTRO_MOE_OK;
}

int astro_moe_take_rows(const void* states, int64_t state_rows, int32_t hidden,
                        const uint32_t* rows, int64_t n, void* out, void* stream) {
  if (hidden <= 0 || hidden % 8 != 0 || n < 0 || state_rows < 0)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "take rows: hidden must be a positive multiple of 8");
  uint32_t* status = nullptr;
  if (int rc = device_status_ptr(&status)) return rc;
  CK(astro::launch_take_rows(states, state_rows, rows, n, hidden, out, status, S(stream)), "take rows");
  return ASTRO_MOE_OK;
}

int astro_moe_gather_qmm(const void* x, int64_t x_rows, int32_t in_features,
                         const uint32_t* lhs, const uint32_t* rhs, int64_t n_rows,
                         const uint32_t* packed, const void* scales, const void* biases,
                         int32_t experts, int32_t out_features, int32_t group, int32_t bits,
                         int32_t sorted_indices, void* out, void* stream) {
  const char* op = "build affine gather_qmm";
  if (int rc = check_affine(op, in_features, group, bits)) return rc;
  if (n_rows < 0 || x_rows < 0 || experts <= 0 || out_features <= 0)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: invalid shapes", op);
  if (experts > 1024) return fail(ASTRO_MOE_ERR_UNSUPPORTED, "%s: experts <= 1024 are supported", op);
  if (n_rows == 0) return ASTRO_MOE_OK;
  if (!x || !packed || !scales || !biases || !out)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null array", op);
  if (!lhs && x_rows < n_rows)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: activation rows do not cover the assignments", op);
  uint32_t* status = nullptr;
  if (int rc = device_status_ptr(&status)) return rc;
  cudaStream_t st = S(stream);
  astro::GroupedGemvDesc d;
  d.x = x;
  d.x_limit = x_rows;
  d.in_features = in_features;
  d.wa[0] = astro::AffineRef{packed, scales, biases, out_features, 0};
  d.out_features = out_features;
  d.group = group;
  d.bits = bits;
  d.y = out;
  d.y_limit = n_rows;
  d.ldy = out_features;
  d.status = status;
  d.rows_total = n_rows;
  uint32_t* buf = nullptr;
  if (!rhs) {
    // single expert: one segment [0, n)
    CK(cudaMallocAsync(&buf, sizeof(uint32_t) * 2, st), "cudaMallocAsync");
    const uint32_t h[2] = {0u, (uint32_t)n_rows};
    CK(cudaMemcpyAsync(buf, h, sizeof(h), cudaMemcpyHostToDevice, st), "copy offsets");
    CK(cudaStreamSynchronize(st), "sync");  // h is a stack array
    d.seg_offsets = buf;
    d.nseg = 1;
    d.x_rows = lhs;
  } else if (sorted_indices) {
    CK(cudaMallocAsync(&buf, sizeof(uint32_t) * (experts + 1), st), "cudaMallocAsync");
    CK(astro::launch_offsets_from_sorted(rhs, n_rows, experts, buf, status, st), op);
    d.seg_offsets = buf;
    d.nseg = experts;
    d.x_rows = lhs;
  } else {
    // group rows by expert with the stable sort, gather through the order and
    // write every result back to its original row
    const size_t n = (size_t)n_rows;
    const size_t sb = astro::sort_scratch_bytes(n_rows, experts);
    CK(cudaMallocAsync(&buf, sizeof(uint32_t) * (2 * n + experts + 1) + sb, st), "cudaMallocAsync");
    uint32_t* order = buf;
    uint32_t* xr = buf + n;
    uint32_t* offs = buf + 2 * n;
    void* sscratch = buf + 2 * n + experts + 1;
    CK(astro::launch_sort_assignments(rhs, n_rows, 1, experts, 0, order, nullptr, nullptr, nullptr,
                                      offs, status, sscratch, st),
       op);
    CK(astro::launch_compose_rows(lhs, order, n_rows, xr, st), op);
    d.seg_offsets = offs;
    d.nseg = experts;
    d.x_rows = xr;
    d.y_rows = order;
  }
  CK(astro::launch_grouped_gemv(d, st), op);
  CK(cudaFreeAsync(buf, st), "cudaFreeAsync");
  return ASTRO_MOE_OK;
}

int astro_moe_quantized_matmul(const void* x, int64_t rows, int32_t in_features,
                               const uint32_t* packed, const void* scales, const void* biases,
                               int32_t out_features, int32_t group, int32_t bits, void* out,
                               void* stream) {
  return astro_moe_gather_qmm(x, rows, in_features, nullptr, nullptr, rows, packed, scales, biases,
                              1, out_features, group, bits, 1, out, stream);
}

int astro_moe_dequantize_affine(const uint32_t* packed, const void* scales, const void* biases,
                                int64_t rows, int32_t in_features, int32_t group_size,
                                int32_t bits, void* out, void* stream) {
  const char* op = "dequantize affine";
  if (rows < 0) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: negative row count", op);
  if (int rc = check_affine(op, in_features, group_size, bits)) return rc;
  if (rows > 0 && (!packed || !scales || !biases || !out))
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null array", op);
  CK(astro::launch_dequantize_affine(packed, scales, biases, rows, in_features, group_size, bits, out,
                                     S(stream)),
     op);
  return ASTRO_MOE_OK;
}

int astro_moe_swiglu(const void* gate, const void* up, int64_t n, void* out, void* stream) {
  if (n < 0) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "apply a compiled MLX SwiGLU graph: negative size");
  CK(astro::launch_swiglu(gate, up, n, out, S(stream)), "apply a compiled MLX SwiGLU graph");
  return ASTRO_MOE_OK;
}

int astro_moe_sorted_expert_weighted_sum(const void* sorted_outputs, int32_t out_dtype,
                                         const uint32_t* inverse, const void* scores,
                                         int32_t score_dtype, int64_t tokens, int32_t top_k,
                                         int64_t dim, void* out, void* stream) {
  const char* op = "reduce stacked expert outputs";
  if (!valid_dtype(out_dtype) || !valid_dtype(score_dtype) || tokens < 0 || top_k < 0 || dim < 0)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT,
                "%s: sorted expert outputs, inverse order, and scores have invalid shapes or dtypes", op);
  CK(astro::launch_sorted_weighted_sum(sorted_outputs, out_dtype, inverse, scores, score_dtype,
                                       tokens, top_k, dim, out, S(stream)),
     op);
  return ASTRO_MOE_OK;
}

int astro_moe_unsorted_expert_weighted_sum(const void* outputs, int32_t out_dtype,
                                           const void* scores, int32_t score_dtype,
                                           int64_t tokens, int32_t top_k, int64_t dim, void* out,
                                           void* stream) {
  const char* op = "reduce stacked expert outputs";
  if (!valid_dtype(out_dtype) || !valid_dtype(score_dtype) || tokens < 0 || top_k < 0 || dim < 0)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT,
                "%s: unsorted expert outputs and scores must include an assignment axis", op);
  if (top_k == 0) {
    // empty reduction: zeros (weighted_sum.rs:172-188, empty_weighted_outputs)
    const size_t es = out_dtype == ASTRO_MOE_DTYPE_F32 ? 4 : 2;
    CK(cudaMemsetAsync(out, 0, es * (size_t)(tokens * dim), S(stream)), op);
    return ASTRO_MOE_OK;
  }
  CK(astro::launch_unsorted_weighted_sum(outputs, out_dtype, scores, score_dtype, tokens, top_k,
                                         dim, out, S(stream)),
     op);
  return ASTRO_MOE_OK;
}

int astro_moe_combine_sparse_and_shared(const void* sparse, const void* shared,
                                        const void* gate_logits, int32_t dtype, int64_t tokens,
                                        int64_t dim, void* out, void* stream) {
  const char* op = "combine Qwen3.5-MoE sparse and shared experts";
  if (!valid_dtype(dtype) || tokens < 0 || dim < 0)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: invalid shapes", op);
  CK(astro::launch_combine_shared(sparse, shared, gate_logits, dtype, tokens, dim, out, S(stream)), op);
  return ASTRO_MOE_OK;
}

int astro_moe_invert_assignment_order(const uint32_t* order, int64_t n, uint32_t* inverse) {
  if (n < 0 || n > 0xffffffffLL)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "assignment permutation length exceeds u32");
  std::vector<unsigned char> seen((size_t)n, 0);
  for (int64_t s = 0; s < n; ++s) {
    const uint32_t o = order[s];
    if ((int64_t)o >= n)
      return fail(ASTRO_MOE_ERR_OUT_OF_RANGE_SLOT, "assignment permutation contains an out-of-range slot");
    if (seen[o]) return fail(ASTRO_MOE_ERR_DUPLICATE_SLOT, "assignment permutation contains a duplicate slot");
    seen[o] = 1;
    inverse[o] = (uint32_t)s;
  }
  return ASTRO_MOE_OK;
}

// ---------------------------------------------------------------------------
// context API
// ---------------------------------------------------------------------------
int astro_moe_ctx_create(int32_t device, void* stream, const astro_moe_options* options,
                         astro_moe_ctx** out_ctx) {
  if (!out_ctx) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "ctx create: null output");
  int ndev = 0;
  CK(cudaGetDeviceCount(&ndev), "cudaGetDeviceCount");
  if (device < 0 || device >= ndev)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "ctx create: device %d out of range", device);
  DeviceGuard g(device);
  auto* ctx = new astro_moe_ctx();
  ctx->device = device;
  ctx->stream = S(stream);
  if (options) ctx->opt = *options;
  if (int rc = device_status_ptr(&ctx->status)) {
    delete ctx;
    return rc;
  }
  *out_ctx = ctx;
  return ASTRO_MOE_OK;
}

int astro_moe_ctx_destroy(astro_moe_ctx* ctx) {
  if (!ctx) return ASTRO_MOE_OK;
  DeviceGuard g(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  for (auto& kv : ctx->layers) release_layer(kv.second);
  for (auto& ev : ctx->pending)
    for (auto e : ev) cudaEventDestroy(e);
  for (auto e : ctx->event_pool) cudaEventDestroy(e);
  if (ctx->ws) cudaFree(ctx->ws);
  if (ctx->io) cudaFree(ctx->io);
  if (ctx->up) cudaStreamSynchronize(ctx->up);
  if (ctx->down) cudaStreamSynchronize(ctx->down);
  for (int i = 0; i < 2; ++i) {
    if (ctx->aio[i]) cudaFree(ctx->aio[i]);
    if (ctx->ev_in[i]) cudaEventDestroy(ctx->ev_in[i]);
    if (ctx->ev_done[i]) cudaEventDestroy(ctx->ev_done[i]);
    if (ctx->ev_out[i]) cudaEventDestroy(ctx->ev_out[i]);
  }
  if (ctx->up) cudaStreamDestroy(ctx->up);
  if (ctx->down) cudaStreamDestroy(ctx->down);
  if (ctx->ep_disp.p) cudaFree(ctx->ep_disp.p);
  if (ctx->ep_exp.p) cudaFree(ctx->ep_exp.p);
  if (ctx->ep_shared.p) cudaFree(ctx->ep_shared.p);
  for (int r = 0; r < ctx->xr_world; ++r) {
    if (r == ctx->xr_rank) continue;
    if (ctx->xr_peer_recv[r]) cudaIpcCloseMemHandle(ctx->xr_peer_recv[r]);
    if (ctx->xr_peer_ret[r]) cudaIpcCloseMemHandle(ctx->xr_peer_ret[r]);
    if (ctx->xr_peer_mbox[r]) cudaIpcCloseMemHandle(ctx->xr_peer_mbox[r]);
  }
  if (ctx->xr_recv) cudaFree(ctx->xr_recv);
  if (ctx->xr_ret) cudaFree(ctx->xr_ret);
  if (ctx->xr_mbox) cudaFree(ctx->xr_mbox);
  delete ctx;
  return ASTRO_MOE_OK;
}

int astro_moe_ctx_set_stream(astro_moe_ctx* ctx, void* stream) {
  if (!ctx) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "ctx: null");
  ctx->stream = S(stream);
  return ASTRO_MOE_OK;
}

int astro_moe_ctx_synchronize(astro_moe_ctx* ctx) {
  if (!ctx) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "ctx: null");
  DeviceGuard g(ctx->device);
  CK(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
  uint32_t st = 0;
  CK(cudaMemcpy(&st, ctx->status, sizeof(st), cudaMemcpyDeviceToHost), "read device status");
  if (st) {
    cudaMemset(ctx->status, 0, sizeof(uint32_t));
    return fail(ASTRO_MOE_ERR_DEVICE_STATUS, "device status 0x%x (1: expert id out of range, 2: wait timeout, 4: bad row)", st);
  }
  return ASTRO_MOE_OK;
}

int astro_moe_register_layer(astro_moe_ctx* ctx, int32_t layer, const astro_moe_layer_weights* w) {
  const char* op = "register layer";
  if (!ctx || !w) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null argument", op);
  if (layer < 0) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: negative layer index", op);
  if (int rc = validate_layer(op, w)) return rc;
  DeviceGuard g(ctx->device);
  LayerState& L = ctx->layers[layer];
  L.registered = false;
  if (int rc = resolve_layer(ctx, w, w->experts, L)) return rc;
  const bool has_shared = w->shared_intermediate > 0;
  // the tcgen05 kernels: routed experts 4-bit g64 (and the shared expert too, or
  // it runs separately); the plan covers the shared expert only when it is a
  // segment of the same launches
  const bool routed_q4 = q4g64(L, 0, 2);
  const bool shared_q4 = !has_shared || q4g64(L, 3, 5);
  if (routed_q4 && (shared_q4 || L.shared_separate)) {
    astro_moe_layer_weights view = L.w;
    if (L.shared_separate) view.shared_intermediate = 0;
    if (int st = astro::moe_gemm_plan(view, &L.gemm))
      return fail(ASTRO_MOE_ERR_CUDA, "%s: tensor-core plan failed (%d)", op, st);
  }
  L.registered = true;
  auto aligned16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  bool weights_aligned = aligned16(w->gate.packed) && aligned16(w->down.packed) &&
                         (w->gate_up_fused || aligned16(w->up.packed));
  if (has_shared)
    weights_aligned = weights_aligned && aligned16(w->shared_gate.packed) &&
                      aligned16(w->shared_up.packed) && aligned16(w->shared_down.packed);
  L.decode_ok = weights_aligned && routed_q4 && shared_q4 && !L.shared_separate &&
                astro::decode_gemv_supported(w->hidden, w->intermediate, 64, 4);
  L.router_gemv_ok = aligned16(L.w.router_weight) && astro::router_gemv_supported(w->hidden);
  // the fused decode kernel reads each row's scales and biases of a K quarter as
  // one vector of up to 16 bytes
  bool sb_aligned = aligned16(w->gate.scales) && aligned16(w->gate.biases) &&
                    aligned16(w->down.scales) && aligned16(w->down.biases) &&
                    (w->gate_up_fused || (aligned16(w->up.scales) && aligned16(w->up.biases)));
  if (has_shared)
    sb_aligned = sb_aligned && aligned16(w->shared_gate.scales) && aligned16(w->shared_gate.biases) &&
                 aligned16(w->shared_up.scales) && aligned16(w->shared_up.biases) &&
                 aligned16(w->shared_down.scales) && aligned16(w->shared_down.biases);
  L.fused_ok = L.decode_ok && sb_aligned;
  return ASTRO_MOE_OK;
}

int astro_moe_block_forward_taps(astro_moe_ctx* ctx, int32_t layer, const void* x, int64_t T,
                                 void* out, const astro_moe_block_taps* taps) {
  if (!ctx) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "block forward: null ctx");
  auto it = ctx->layers.find(layer);
  if (it == ctx->layers.end() || !it->second.registered)
    return fail(ASTRO_MOE_ERR_NOT_REGISTERED, "block forward: layer %d is not registered", layer);
  if (it->second.ep)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT,
                "block forward: layer %d is expert-parallel (use astro_moe_ep_dispatch/experts/combine)", layer);
  if (it->second.pager)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT,
                "block forward: layer %d is paged (use astro_moe_paged_block_forward)", layer);
  if (T < 0) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "block forward: negative token count");
  if (T * (int64_t)it->second.w.top_k + T > 0x7fffffffLL)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "block forward: too many tokens");
  if (T > 0 && (!x || !out)) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "block forward: null array");
  DeviceGuard g(ctx->device);
  return run_block(ctx, it->second, x, T, out, taps);
}

int astro_moe_block_forward(astro_moe_ctx* ctx, int32_t layer, const void* x, int64_t T, void* out) {
  return astro_moe_block_forward_taps(ctx, layer, x, T, out, nullptr);
}

int astro_moe_ctx_last_block_path(astro_moe_ctx* ctx, astro_moe_block_path* out) {
  if (!ctx || !out) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "last block path: null argument");
  *out = ctx->last_path;
  return ASTRO_MOE_OK;
}

int astro_moe_ctx_set_attribution(astro_moe_ctx* ctx, int32_t enabled) {
  if (!ctx) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "ctx: null");
  ctx->attribution = enabled != 0;
  return ASTRO_MOE_OK;
}

int astro_moe_ctx_read_attribution(astro_moe_ctx* ctx, astro_moe_attribution* out, int32_t reset) {
  if (!ctx || !out) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "attribution: null argument");
  DeviceGuard g(ctx->device);
  CK(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
  for (auto& ev : ctx->pending) {
    float ms[5] = {0, 0, 0, 0, 0};
    for (int i = 0; i < 5; ++i) cudaEventElapsedTime(&ms[i], ev[i], ev[i + 1]);
    ctx->acc.router_projection_ms += ms[0];
    ctx->acc.assignment_preparation_ms += ms[1];
    ctx->acc.gate_up_ms += ms[2];
    ctx->acc.down_ms += ms[3];
    ctx->acc.weighted_reduction_ms += ms[4];
    for (auto e : ev) ctx->event_pool.push_back(e);
  }
  ctx->pending.clear();
  *out = ctx->acc;
  out->kernel_launches = ctx->launches;
  if (reset) {
    ctx->acc = astro_moe_attribution{};
    ctx->launches = 0;
  }
  return ASTRO_MOE_OK;
}

int astro_moe_block_forward_host(astro_moe_ctx* ctx, int32_t layer, const void* host_x, int64_t T,
                                 void* host_out) {
  if (!ctx) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "block forward: null ctx");
  auto it = ctx->layers.find(layer);
  if (it == ctx->layers.end() || !it->second.registered)
    return fail(ASTRO_MOE_ERR_NOT_REGISTERED, "block forward: layer %d is not registered", layer);
  if (it->second.ep || it->second.pager)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "block forward: layer %d is expert-parallel or paged", layer);
  if (T <= 0) return T == 0 ? ASTRO_MOE_OK : fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "negative tokens");
  DeviceGuard g(ctx->device);
  const size_t bytes = sizeof(uint16_t) * (size_t)T * it->second.w.hidden;
  if (ctx->io_bytes < 2 * bytes) {
    if (ctx->io) {
      CK(cudaStreamSynchronize(ctx->stream), "sync");
      cudaFree(ctx->io);
    }
    ctx->io = nullptr;
    ctx->io_bytes = 0;
    CK(cudaMalloc(&ctx->io, 2 * bytes), "cudaMalloc(io)");
    ctx->io_bytes = 2 * bytes;
  }
  char* dx = (char*)ctx->io;
  char* dy = dx + bytes;
  CK(cudaMemcpyAsync(dx, host_x, bytes, cudaMemcpyHostToDevice, ctx->stream), "copy hidden states in");
  if (int rc = run_block(ctx, it->second, dx, T, dy, nullptr)) return rc;
  CK(cudaMemcpyAsync(host_out, dy, bytes, cudaMemcpyDeviceToHost, ctx->stream), "copy output out");
  return astro_moe_ctx_synchronize(ctx);
}


// ===========================================================================
// expert parallelism
// ===========================================================================
int astro_moe_ep_register_layer(astro_moe_ctx* ctx, int32_t layer, const astro_moe_layer_weights* w,
                                int32_t expert_first, int32_t expert_count) {
  const char* op = "register expert-parallel layer";
  if (!ctx || !w) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null argument", op);
  if (layer < 0) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: negative layer index", op);
  if (int rc = validate_layer(op, w)) return rc;
  if (expert_first < 0 || expert_count < 1 || expert_first + expert_count > w->experts)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: local experts [%d, %d) outside [0, %d)", op,
                expert_first, expert_first + expert_count, w->experts);
  DeviceGuard g(ctx->device);
  LayerState& L = ctx->layers[layer];
  L.registered = false;
  if (int rc = resolve_layer(ctx, w, w->experts, L)) return rc;
  if (L.shared_separate)
    return fail(ASTRO_MOE_ERR_UNSUPPORTED,
                "%s: the shared expert must share the routed experts' quantisation here", op);
  if (w->router_kind != ASTRO_MOE_ROUTER_SOFTMAX)
    return fail(ASTRO_MOE_ERR_UNSUPPORTED, "%s: expert parallelism takes the softmax router", op);
  L.w.experts = expert_count;
  L.ep = true;
  L.ep_first = expert_first;
  L.ep_total = w->experts;
  L.decode_ok = false;
  L.fused_ok = false;
  if (q4g64(L, 0, 2) && (w->shared_intermediate == 0 || q4g64(L, 3, 5)))
    if (int st = astro::moe_gemm_plan(L.w, &L.gemm, w->experts))
      return fail(ASTRO_MOE_ERR_CUDA, "%s: tensor-core plan failed (%d)", op, st);
  L.registered = true;
  L.router_gemv_ok = (reinterpret_cast<uintptr_t>(L.w.router_weight) & 15u) == 0 &&
                     astro::router_gemv_supported(w->hidden);
  return ASTRO_MOE_OK;
}

int astro_moe_ep_dispatch(astro_moe_ctx* ctx, int32_t layer, const void* x, int64_t T,
                          void* send_rows, uint32_t* expert_offsets) {
  const char* op = "expert-parallel dispatch";
  LayerState* Lp = nullptr;
  if (int rc = ep_layer(ctx, layer, op, &Lp)) return rc;
  LayerState& L = *Lp;
  const astro_moe_layer_weights& w = L.w;
  const int H = w.hidden, E = L.ep_total, K = w.top_k;
  if (T < 0 || T * (int64_t)K > 0x7fffffffLL)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: invalid token count", op);
  if (T > 0 && (!x || !send_rows || !expert_offsets))
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null array", op);
  if ((reinterpret_cast<uintptr_t>(x) & 15u) != 0)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: hidden states must be 16-byte aligned", op);
  DeviceGuard g(ctx->device);
  cudaStream_t st = ctx->stream;
  const bool has_shared = w.shared_intermediate > 0;
  EpDispatch d{};
  if (int rc = devbuf_ensure(ctx, ctx->ep_disp, plan_ep_dispatch(T > 0 ? T : 1, E, K, nullptr, nullptr)))
    return rc;
  plan_ep_dispatch(T > 0 ? T : 1, E, K, &d, (char*)ctx->ep_disp.p);
  ctx->ep_layer = layer;
  ctx->ep_tokens = T;
  if (T == 0) {
    CK(cudaMemsetAsync(expert_offsets, 0, sizeof(uint32_t) * (E + 1), st), op);
    return ASTRO_MOE_OK;
  }
  if (T <= kRouterGemvTokens && L.router_gemv_ok) {
    CK(astro::launch_router_gemv(x, T, w.router_weight, E, H, d.logits, st), "router projection");
  } else if (astro::moe_gemm_enabled(L.gemm, ctx->opt.use_tensor_cores)) {
    CK(astro::moe_gemm_router(L.gemm, x, T, d.logits, nullptr, ctx->status, st), "router projection");
  } else {
    CK(astro::launch_dense_nt_simt(x, w.router_weight, T, E, H, d.logits, E, st), "router projection");
  }
  CK(astro::launch_route_experts(d.logits, ASTRO_MOE_DTYPE_BF16, T, E, K, w.normalize_top_k, d.ids,
                                 d.scores, x, has_shared ? w.shared_expert_gate : nullptr, H,
                                 has_shared ? d.gate_logit : nullptr, st),
     "route experts");
  CK(astro::launch_sort_assignments(d.ids, T, K, E, 0, d.order, d.inverse, d.sids, d.stok,
                                    expert_offsets, ctx->status, d.sort_scratch, st),
     "sort expert assignments");
  CK(astro::launch_take_rows(x, T, d.stok, T * K, H, send_rows, ctx->status, st), "gather rows");
  ctx->launches += 3 + astro::sort_launch_count(T * K);
  return ASTRO_MOE_OK;
}

// Expert side of an expert-parallel layer up to the expert-major outputs (in
// ctx->ep_exp: yrows, dest) and the shared-expert rows (ctx->ep_shared).
static int ep_experts_compute(astro_moe_ctx* ctx, int32_t layer, const char* op,
                              const void* recv_rows, const uint32_t* recv_counts, int32_t world,
                              int64_t recv_total, const void* x, int64_t T) {
  LayerState* Lp = nullptr;
  if (int rc = ep_layer(ctx, layer, op, &Lp)) return rc;
  LayerState& L = *Lp;
  const astro_moe_layer_weights& w = L.w;
  const int H = w.hidden, El = w.experts, I = w.intermediate;
  if (world < 1 || world * El > 2048)
    return fail(ASTRO_MOE_ERR_UNSUPPORTED, "%s: world * local experts must be <= 2048", op);
  if (recv_total < 0 || T < 0 || recv_total + T > 0x7fffffffLL)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: invalid row counts", op);
  if (!recv_counts || (recv_total > 0 && !recv_rows) || (T > 0 && !x))
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null array", op);
  DeviceGuard g(ctx->device);
  cudaStream_t st = ctx->stream;
  const bool has_shared = w.shared_intermediate > 0;
  const int64_t shared_rows = has_shared ? T : 0;
  const int64_t rows = recv_total + shared_rows;
  EpExperts e{};
  if (int rc = devbuf_ensure(ctx, ctx->ep_exp,
                             plan_ep_experts(rows, recv_total, H, I, world * El, El, nullptr, nullptr)))
    return rc;
  plan_ep_experts(rows, recv_total, H, I, world * El, El, &e, (char*)ctx->ep_exp.p);
  if (has_shared)
    if (int rc = devbuf_ensure(ctx, ctx->ep_shared, sizeof(uint16_t) * (size_t)(T > 0 ? T : 1) * H))
      return rc;
  CK(astro::launch_ep_permutation(recv_counts, world, El, (int)shared_rows, e.src_start, e.exp_start,
                                  e.offsets, e.dest, e.src_of, st),
     "expert-major permutation");
  // the tcgen05 GEMMs take their token rows in K order perm8_bf16
  const bool perm8 = astro::moe_gemm_enabled(L.gemm, ctx->opt.use_tensor_cores);
  CK(astro::launch_take_rows(recv_rows, recv_total, e.src_of, recv_total, H, e.states, ctx->status,
                             st, perm8),
     "expert-major rows");
  if (shared_rows > 0)
    CK(astro::launch_take_rows(x, shared_rows, nullptr, shared_rows, H, e.states + recv_total * H,
                               ctx->status, st, perm8),
       "shared-expert rows");
  ctx->launches += 3;
  if (rows > 0) {
    if (astro::moe_gemm_enabled(L.gemm, ctx->opt.use_tensor_cores)) {
      CK(astro::moe_gemm_gate_up(L.gemm, e.states, rows, e.offsets, e.act, e.gemm_scratch,
                                 ctx->status, st),
         "gate/up projection");
      CK(astro::moe_gemm_down(L.gemm, e.act, rows, e.offsets, e.yrows, e.gemm_scratch, ctx->status,
                              st),
         "down projection");
    } else {
      astro::GroupedGemvDesc d;
      d.x = e.states;
      d.x_limit = rows;
      d.in_features = H;
      d.seg_offsets = e.offsets;
      d.nseg = El + (has_shared ? 1 : 0);
      d.shared_seg = has_shared ? El : -1;
      d.rows_total = rows;
      astro::AffineRef down[2];
      fill_projections(w, d.wa, d.wb, down);
      d.out_features = I;
      d.group = L.qgroup[0];
      d.bits = L.qbits[0];
      d.swiglu = true;
      d.y = e.act;
      d.y_limit = rows;
      d.ldy = I;
      d.status = ctx->status;
      CK(astro::launch_grouped_gemv(d, st), "gate/up projection");
      astro::GroupedGemvDesc dd = d;
      dd.x = e.act;
      dd.in_features = I;
      dd.wa[0] = down[0];
      dd.wa[1] = down[1];
      dd.wb[0] = dd.wb[1] = astro::AffineRef{};
      dd.out_features = H;
      dd.group = L.qgroup[2];
      dd.bits = L.qbits[2];
      dd.swiglu = false;
      dd.y = e.yrows;
      dd.ldy = H;
      CK(astro::launch_grouped_gemv(dd, st), "down projection");
    }
    ctx->launches += 2;
  }
  if (shared_rows > 0)
    CK(cudaMemcpyAsync(ctx->ep_shared.p, e.yrows + recv_total * H, sizeof(uint16_t) * shared_rows * H,
                       cudaMemcpyDeviceToDevice, st),
       "shared-expert rows");
  return ASTRO_MOE_OK;
}

int astro_moe_ep_experts(astro_moe_ctx* ctx, int32_t layer, const void* recv_rows,
                         const uint32_t* recv_counts, int32_t world, int64_t recv_total,
                         const void* x, int64_t T, void* out_rows) {
  const char* op = "expert-parallel experts";
  if (recv_total > 0 && !out_rows) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null array", op);
  if (int rc = ep_experts_compute(ctx, layer, op, recv_rows, recv_counts, world, recv_total, x, T))
    return rc;
  const astro_moe_layer_weights& w = ctx->layers[layer].w;
  const int64_t rows = recv_total + (w.shared_intermediate > 0 ? T : 0);
  EpExperts e{};
  plan_ep_experts(rows, recv_total, w.hidden, w.intermediate, world * w.experts, w.experts, &e,
                  (char*)ctx->ep_exp.p);
  DeviceGuard g(ctx->device);
  CK(astro::launch_take_rows(e.yrows, rows, e.dest, recv_total, w.hidden, out_rows, ctx->status,
                             ctx->stream),
     "received order");
  ctx->launches += 1;
  return ASTRO_MOE_OK;
}

int astro_moe_ep_combine(astro_moe_ctx* ctx, int32_t layer, const void* returned_rows, int64_t T,
                         void* out) {
  const char* op = "expert-parallel combine";
  LayerState* Lp = nullptr;
  if (int rc = ep_layer(ctx, layer, op, &Lp)) return rc;
  const astro_moe_layer_weights& w = Lp->w;
  if (ctx->ep_layer != layer || ctx->ep_tokens != T)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT,
                "%s: layer %d with %lld tokens does not match the dispatch in flight", op, layer,
                (long long)T);
  if (T == 0) return ASTRO_MOE_OK;
  if (!returned_rows) returned_rows = ctx->xr_ret;  // rows returned by the peer exchange
  if (!returned_rows || !out) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null array", op);
  const int H = w.hidden, E = Lp->ep_total, K = w.top_k;
  const bool has_shared = w.shared_intermediate > 0;
  DeviceGuard g(ctx->device);
  EpDispatch d{};
  plan_ep_dispatch(T, E, K, &d, (char*)ctx->ep_disp.p);
  const int threshold = ctx->opt.sorted_threshold > 0 ? ctx->opt.sorted_threshold : 64;
  CK(astro::launch_block_combine_split(returned_rows, has_shared ? ctx->ep_shared.p : returned_rows,
                                       d.inverse, d.scores, has_shared ? d.gate_logit : nullptr, T, K,
                                       H, T * K >= threshold ? 1 : 0, out, ctx->stream),
     "weighted combine");
  ctx->launches += 1;
  return ASTRO_MOE_OK;
}


// ===========================================================================
// expert paging
// ===========================================================================
int64_t astro_moe_page_bytes(int32_t H, int32_t I, int32_t G, int32_t bits) {
  if (H <= 0 || I <= 0 || G <= 0 || bits <= 0 || H % G || I % G) return 0;
  return (3LL * I * H) * bits / 8 + (2LL * I * (H / G) + (int64_t)H * (I / G)) * 2 * 2;
}

int astro_moe_pager_create(astro_moe_ctx* ctx, int32_t layers, int32_t experts, int32_t H,
                           int32_t I, int32_t G, int32_t bits, const void* host_pages,
                           int64_t cache_bytes, astro_moe_pager** out) {
  const char* op = "pager create";
  if (!ctx || !out || !host_pages) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null argument", op);
  if (layers <= 0 || experts <= 0 || experts > 1024)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: invalid layer or expert count", op);
  if (bits != 4 || G != 64 || !astro::decode_gemv_supported(H, I, G, bits))
    return fail(ASTRO_MOE_ERR_UNSUPPORTED, "%s: paged experts need 4-bit, group-64 layers of a decode-kernel shape", op);
  const int64_t page = astro_moe_page_bytes(H, I, G, bits);
  const int64_t rq_h = (int64_t)H * bits / 8, rs_h = (int64_t)(H / G) * 2;
  const int64_t rq_i = (int64_t)I * bits / 8, rs_i = (int64_t)(I / G) * 2;
  if (page % rq_h || page % rs_h || page % rq_i || page % rs_i || page % 16)
    return fail(ASTRO_MOE_ERR_UNSUPPORTED, "%s: page size does not tile the expert rows", op);
  const int64_t slots = cache_bytes / page;
  if (slots < 1)
    return fail(ASTRO_MOE_ERR_MEMORY_LIMIT,
                "%s: the cache ceiling of %lld bytes holds no %lld-byte expert page", op,
                (long long)cache_bytes, (long long)page);
  DeviceGuard g(ctx->device);
  cudaPointerAttributes attr{};
  CK(cudaPointerGetAttributes(&attr, host_pages), "cudaPointerGetAttributes");
  if (attr.type != cudaMemoryTypeHost)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: host_pages must be pinned host memory", op);
  auto* pg = new astro_moe_pager();
  pg->device = ctx->device;
  pg->layers = layers;
  pg->E = experts;
  pg->H = H;
  pg->I = I;
  pg->group = G;
  pg->bits = bits;
  pg->page_bytes = page;
  const int64_t cq = (int64_t)I * rq_h, cd = (int64_t)H * rq_i;
  const int64_t cs = (int64_t)I * rs_h, cds = (int64_t)H * rs_i;
  pg->off_q[0] = 0;
  pg->off_q[1] = cq;
  pg->off_q[2] = 2 * cq;
  pg->off_s[0] = 2 * cq + cd;
  pg->off_b[0] = pg->off_s[0] + cs;
  pg->off_s[1] = pg->off_b[0] + cs;
  pg->off_b[1] = pg->off_s[1] + cs;
  pg->off_s[2] = pg->off_b[1] + cs;
  pg->off_b[2] = pg->off_s[2] + cds;
  pg->host = static_cast<const char*>(host_pages);
  pg->slots = slots;
  pg->slot_of_page.assign((size_t)layers * experts, -1);
  pg->demand.assign((size_t)layers * experts, 0);
  pg->page_of_slot.assign((size_t)slots, -1);
  pg->last_call.assign((size_t)slots, -1);
  pg->missed.assign((size_t)experts, 0);
  pg->lru_pos.resize((size_t)slots);
  pg->st.capacity_pages = slots;
  auto cleanup = [&](cudaError_t e, const char* what) {
    if (pg->pool) cudaFree(pg->pool);
    if (pg->d_table) cudaFree(pg->d_table);
    if (pg->h_table) cudaFreeHost(pg->h_table);
    if (pg->h_offsets) cudaFreeHost(pg->h_offsets);
    if (pg->ready) cudaEventDestroy(pg->ready);
    if (pg->copy) cudaStreamDestroy(pg->copy);
    delete pg;
    return cuda_fail(e, what);
  };
  cudaError_t e;
  if ((e = cudaMalloc(&pg->pool, (size_t)(slots * page))) != cudaSuccess) return cleanup(e, "cudaMalloc(page cache)");
  if ((e = cudaMalloc(&pg->d_table, sizeof(uint32_t) * 2 * experts)) != cudaSuccess) return cleanup(e, "cudaMalloc(slot table)");
  if ((e = cudaHostAlloc(&pg->h_table, sizeof(uint32_t) * 2 * experts, cudaHostAllocDefault)) != cudaSuccess)
    return cleanup(e, "cudaHostAlloc(slot table)");
  if ((e = cudaHostAlloc(&pg->h_offsets, sizeof(uint32_t) * (experts + 2), cudaHostAllocDefault)) != cudaSuccess)
    return cleanup(e, "cudaHostAlloc(offsets)");
  if ((e = cudaEventCreateWithFlags(&pg->ready, cudaEventDisableTiming)) != cudaSuccess) return cleanup(e, "cudaEventCreate");
  if ((e = cudaStreamCreateWithFlags(&pg->copy, cudaStreamNonBlocking)) != cudaSuccess) return cleanup(e, "cudaStreamCreate");
  *out = pg;
  return ASTRO_MOE_OK;
}

int astro_moe_pager_set_policy(astro_moe_pager* pg, int32_t policy) {
  if (!pg) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "pager set policy: null pager");
  if (policy != ASTRO_MOE_PAGER_LRU && policy != ASTRO_MOE_PAGER_DEMAND)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "pager set policy: unknown policy %d", (int)policy);
  pg->policy = policy;
  return ASTRO_MOE_OK;
}

int astro_moe_pager_inject_copy_failures(astro_moe_pager* pg, int64_t count) {
  if (!pg || count < 0)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "pager inject copy failures: invalid argument");
  pg->inject_copy_failures = count;
  return ASTRO_MOE_OK;
}

int astro_moe_pager_destroy(astro_moe_pager* pg) {
  if (!pg) return ASTRO_MOE_OK;
  DeviceGuard g(pg->device);
  cudaStreamSynchronize(pg->copy);
  for (auto& p : pg->pending) {
    cudaEventDestroy(p.first);
    cudaEventDestroy(p.second);
  }
  for (auto& p : pg->spare) {
    cudaEventDestroy(p.first);
    cudaEventDestroy(p.second);
  }
  cudaFree(pg->pool);
  cudaFree(pg->d_table);
  cudaFreeHost(pg->h_table);
  cudaFreeHost(pg->h_offsets);
  cudaEventDestroy(pg->ready);
  cudaStreamDestroy(pg->copy);
  delete pg;
  return ASTRO_MOE_OK;
}

int astro_moe_pager_read_stats(astro_moe_pager* pg, astro_moe_pager_stats* out, int32_t reset) {
  if (!pg || !out) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "pager stats: null argument");
  DeviceGuard g(pg->device);
  CK(cudaStreamSynchronize(pg->copy), "cudaStreamSynchronize");
  for (auto& p : pg->pending) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, p.first, p.second);
    pg->st.copy_ms += ms;
    pg->spare.push_back(p);
  }
  pg->pending.clear();
  *out = pg->st;
  if (reset) {
    const int64_t res = pg->st.resident_pages, cap = pg->st.capacity_pages;
    pg->st = astro_moe_pager_stats{};
    pg->st.resident_pages = res;
    pg->st.capacity_pages = cap;
  }
  return ASTRO_MOE_OK;
}

int astro_moe_register_paged_layer(astro_moe_ctx* ctx, int32_t layer, const astro_moe_layer_weights* w,
                                   astro_moe_pager* pg) {
  const char* op = "register paged layer";
  if (!ctx || !w || !pg) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null argument", op);
  if (layer < 0 || layer >= pg->layers)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: layer %d outside the pager's %d layers", op, layer, pg->layers);
  if (w->experts != pg->E || w->hidden != pg->H || w->intermediate != pg->I ||
      w->group_size != pg->group || w->bits != pg->bits)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: layer geometry differs from the pager's pages", op);
  if (int rc = validate_layer(op, w, /*routed_stacks=*/false)) return rc;
  if (w->router_kind != ASTRO_MOE_ROUTER_SOFTMAX)
    return fail(ASTRO_MOE_ERR_UNSUPPORTED, "%s: paged layers take the softmax router", op);
  DeviceGuard g(ctx->device);
  LayerState& L = ctx->layers[layer];
  release_layer(L);
  L = LayerState{};
  astro_moe_layer_weights pw = *w;
  pw.gate = pw.up = pw.down = astro_moe_affine{};  // the routed experts are the pages
  pw.gate_up_fused = 0;
  if (int rc = resolve_layer(ctx, &pw, w->experts, L)) return rc;
  if (w->shared_intermediate > 0 && !q4g64(L, 3, 5))
    return fail(ASTRO_MOE_ERR_UNSUPPORTED,
                "%s: a paged layer's shared expert must be 4-bit with group 64 (the decode kernels)", op);
  L.shared_separate = false;
  L.registered = true;
  L.pager = pg;
  L.router_gemv_ok = (reinterpret_cast<uintptr_t>(L.w.router_weight) & 15u) == 0 &&
                     astro::router_gemv_supported(w->hidden);
  // prefill: the tcgen05 grouped GEMMs over the page pool (the routed experts'
  // tensors are located inside each page); not eligible -> the decode kernels
  astro::PagedStacks ps;
  ps.pool = pg->pool;
  ps.slots = pg->slots;
  ps.page_bytes = pg->page_bytes;
  for (int m = 0; m < 3; ++m) {
    ps.off_q[m] = pg->off_q[m];
    ps.off_s[m] = pg->off_s[m];
    ps.off_b[m] = pg->off_b[m];
  }
  astro::moe_gemm_plan(L.w, &L.gemm, 0, &ps);
  return ASTRO_MOE_OK;
}

int astro_moe_paged_block_forward(astro_moe_ctx* ctx, int32_t layer, const void* x, int64_t T,
                                  void* out) {
  const char* op = "paged block forward";
  if (!ctx) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null ctx", op);
  auto it = ctx->layers.find(layer);
  if (it == ctx->layers.end() || !it->second.registered || !it->second.pager)
    return fail(ASTRO_MOE_ERR_NOT_REGISTERED, "%s: layer %d is not a registered paged layer", op, layer);
  if (T < 0) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: negative token count", op);
  if (T * (int64_t)it->second.w.top_k + T > 0x7fffffffLL)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: too many tokens", op);
  if (T > 0 && (!x || !out)) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null array", op);
  if ((reinterpret_cast<uintptr_t>(x) & 15u) != 0)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: hidden states must be 16-byte aligned", op);
  DeviceGuard g(ctx->device);
  return run_paged_block(ctx, it->second, layer, x, T, out);
}


// --- peer-memory exchange -------------------------------------------------
int astro_moe_ep_exchange_create(astro_moe_ctx* ctx, int32_t world, int32_t rank, int32_t hidden,
                                 int64_t recv_rows, int64_t return_rows, void* handles_out) {
  const char* op = "expert-parallel exchange create";
  if (!ctx || !handles_out) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null argument", op);
  if (world < 2 || world > astro::kMaxPeers || rank < 0 || rank >= world)
    return fail(ASTRO_MOE_ERR_UNSUPPORTED, "%s: 2 <= world <= %d", op, astro::kMaxPeers);
  if (hidden <= 0 || hidden % 8 || recv_rows <= 0 || return_rows <= 0)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: invalid sizes", op);
  if (ctx->xr_recv) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: already created", op);
  DeviceGuard g(ctx->device);
  CK(cudaMalloc(&ctx->xr_recv, sizeof(uint16_t) * (size_t)recv_rows * hidden), "cudaMalloc(receive buffer)");
  CK(cudaMalloc(&ctx->xr_ret, sizeof(uint16_t) * (size_t)return_rows * hidden), "cudaMalloc(return buffer)");
  CK(cudaMalloc(&ctx->xr_mbox, sizeof(uint32_t) * (size_t)world * (kMailboxExperts + world)),
     "cudaMalloc(count mailbox)");
  cudaIpcMemHandle_t h[3];
  CK(cudaIpcGetMemHandle(&h[0], ctx->xr_recv), "cudaIpcGetMemHandle");
  CK(cudaIpcGetMemHandle(&h[1], ctx->xr_ret), "cudaIpcGetMemHandle");
  CK(cudaIpcGetMemHandle(&h[2], ctx->xr_mbox), "cudaIpcGetMemHandle");
  std::memcpy(handles_out, h, sizeof(h));
  ctx->xr_world = world;
  ctx->xr_rank = rank;
  ctx->xr_recv_rows = recv_rows;
  ctx->xr_ret_rows = return_rows;
  return ASTRO_MOE_OK;
}

int astro_moe_ep_exchange_connect(astro_moe_ctx* ctx, const void* all_handles) {
  const char* op = "expert-parallel exchange connect";
  if (!ctx || !all_handles) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null argument", op);
  if (!ctx->xr_recv) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: create the exchange first", op);
  if (ctx->xr_connected) return ASTRO_MOE_OK;
  DeviceGuard g(ctx->device);
  const auto* h = static_cast<const cudaIpcMemHandle_t*>(all_handles);
  for (int r = 0; r < ctx->xr_world; ++r) {
    if (r == ctx->xr_rank) {
      ctx->xr_peer_recv[r] = ctx->xr_recv;
      ctx->xr_peer_ret[r] = ctx->xr_ret;
      ctx->xr_peer_mbox[r] = ctx->xr_mbox;
      continue;
    }
    CK(cudaIpcOpenMemHandle(&ctx->xr_peer_recv[r], h[3 * r], cudaIpcMemLazyEnablePeerAccess),
       "cudaIpcOpenMemHandle(receive buffer)");
    CK(cudaIpcOpenMemHandle(&ctx->xr_peer_ret[r], h[3 * r + 1], cudaIpcMemLazyEnablePeerAccess),
       "cudaIpcOpenMemHandle(return buffer)");
    CK(cudaIpcOpenMemHandle(&ctx->xr_peer_mbox[r], h[3 * r + 2], cudaIpcMemLazyEnablePeerAccess),
       "cudaIpcOpenMemHandle(count mailbox)");
  }
  ctx->xr_connected = true;
  return ASTRO_MOE_OK;
}

int astro_moe_ep_route(astro_moe_ctx* ctx, int32_t layer, const void* x, int64_t T,
                       uint32_t* expert_offsets) {
  // the dispatch without its gather: rows go out with astro_moe_ep_push
  const char* op = "expert-parallel route";
  LayerState* Lp = nullptr;
  if (int rc = ep_layer(ctx, layer, op, &Lp)) return rc;
  LayerState& L = *Lp;
  const astro_moe_layer_weights& w = L.w;
  const int H = w.hidden, E = L.ep_total, K = w.top_k;
  if (T < 0 || T * (int64_t)K > 0x7fffffffLL)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: invalid token count", op);
  if (T > 0 && (!x || !expert_offsets)) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null array", op);
  if ((reinterpret_cast<uintptr_t>(x) & 15u) != 0)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: hidden states must be 16-byte aligned", op);
  DeviceGuard g(ctx->device);
  cudaStream_t st = ctx->stream;
  const bool has_shared = w.shared_intermediate > 0;
  EpDispatch d{};
  if (int rc = devbuf_ensure(ctx, ctx->ep_disp, plan_ep_dispatch(T > 0 ? T : 1, E, K, nullptr, nullptr)))
    return rc;
  plan_ep_dispatch(T > 0 ? T : 1, E, K, &d, (char*)ctx->ep_disp.p);
  ctx->ep_layer = layer;
  ctx->ep_tokens = T;
  if (T == 0) {
    CK(cudaMemsetAsync(expert_offsets, 0, sizeof(uint32_t) * (E + 1), st), op);
    return ASTRO_MOE_OK;
  }
  if (T <= kRouterGemvTokens && L.router_gemv_ok) {
    CK(astro::launch_router_gemv(x, T, w.router_weight, E, H, d.logits, st), "router projection");
  } else if (astro::moe_gemm_enabled(L.gemm, ctx->opt.use_tensor_cores)) {
    CK(astro::moe_gemm_router(L.gemm, x, T, d.logits, nullptr, ctx->status, st), "router projection");
  } else {
    CK(astro::launch_dense_nt_simt(x, w.router_weight, T, E, H, d.logits, E, st), "router projection");
  }
  CK(astro::launch_route_experts(d.logits, ASTRO_MOE_DTYPE_BF16, T, E, K, w.normalize_top_k, d.ids,
                                 d.scores, x, has_shared ? w.shared_expert_gate : nullptr, H,
                                 has_shared ? d.gate_logit : nullptr, st),
     "route experts");
  CK(astro::launch_sort_assignments(d.ids, T, K, E, 0, d.order, d.inverse, d.sids, d.stok,
                                    expert_offsets, ctx->status, d.sort_scratch, st),
     "sort expert assignments");
  ctx->launches += 2 + astro::sort_launch_count(T * K);
  return ASTRO_MOE_OK;
}

int astro_moe_ep_push(astro_moe_ctx* ctx, int32_t layer, const void* x, int64_t T,
                      const int64_t* send_starts, const int64_t* dest_offsets) {
  const char* op = "expert-parallel push";
  LayerState* Lp = nullptr;
  if (int rc = ep_layer(ctx, layer, op, &Lp)) return rc;
  if (!ctx->xr_connected) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: exchange not connected", op);
  if (ctx->ep_layer != layer || ctx->ep_tokens != T)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: does not match the routing in flight", op);
  if (T == 0) return ASTRO_MOE_OK;
  if (!x || !send_starts || !dest_offsets) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null array", op);
  const astro_moe_layer_weights& w = Lp->w;
  const int E = Lp->ep_total, K = w.top_k, El = w.experts;
  DeviceGuard g(ctx->device);
  EpDispatch d{};
  plan_ep_dispatch(T, E, K, &d, (char*)ctx->ep_disp.p);
  int64_t caps[astro::kMaxPeers];
  for (int r = 0; r < ctx->xr_world; ++r) caps[r] = ctx->xr_recv_rows;
  CK(astro::launch_ep_push_rows(x, T, d.stok, d.sids, T * K, El, ctx->xr_world, w.hidden,
                                ctx->xr_peer_recv, caps, dest_offsets, send_starts, ctx->status,
                                ctx->stream),
     op);
  ctx->launches += 1;
  return ASTRO_MOE_OK;
}

int astro_moe_ep_experts_push(astro_moe_ctx* ctx, int32_t layer, const uint32_t* recv_counts,
                              int64_t recv_total, const void* x, int64_t T,
                              const int64_t* recv_starts, const int64_t* return_offsets) {
  const char* op = "expert-parallel experts (peer return)";
  if (!ctx) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null ctx", op);
  if (!ctx->xr_connected) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: exchange not connected", op);
  if (recv_total > ctx->xr_recv_rows)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: %lld received rows exceed the receive buffer", op,
                (long long)recv_total);
  if (!recv_starts || !return_offsets) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null array", op);
  // the expert arithmetic reads the receive buffer; outputs land in ep_exp.yrows
  // in expert-major order, then travel back by the peer return kernel
  if (int rc = ep_experts_compute(ctx, layer, op, ctx->xr_recv, recv_counts, ctx->xr_world,
                                  recv_total, x, T))
    return rc;
  LayerState* Lp = nullptr;
  ep_layer(ctx, layer, op, &Lp);
  const astro_moe_layer_weights& w = Lp->w;
  EpExperts e{};
  const int64_t rows = recv_total + (w.shared_intermediate > 0 ? T : 0);
  plan_ep_experts(rows, recv_total, w.hidden, w.intermediate, ctx->xr_world * w.experts, w.experts,
                  &e, (char*)ctx->ep_exp.p);
  int64_t caps[astro::kMaxPeers];
  for (int r = 0; r < ctx->xr_world; ++r) caps[r] = ctx->xr_ret_rows;
  DeviceGuard g(ctx->device);
  CK(astro::launch_ep_return_rows(e.yrows, rows, e.dest, recv_total, ctx->xr_world, w.hidden,
                                  ctx->xr_peer_ret, caps, return_offsets, recv_starts, ctx->status,
                                  ctx->stream),
     op);
  ctx->launches += 1;
  return ASTRO_MOE_OK;
}

int astro_moe_ep_exchange_buffers(astro_moe_ctx* ctx, void** recv, void** ret) {
  if (!ctx) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "exchange buffers: null ctx");
  if (recv) *recv = ctx->xr_recv;
  if (ret) *ret = ctx->xr_ret;
  return ASTRO_MOE_OK;
}


// --- device-planned peer exchange (no host synchronisation) -----------------
static int ep_dev_check(astro_moe_ctx* ctx, int32_t layer, const char* op, LayerState** Lp) {
  if (int rc = ep_layer(ctx, layer, op, Lp)) return rc;
  if (!ctx->xr_connected) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: exchange not connected", op);
  if ((*Lp)->w.experts > kMailboxExperts)
    return fail(ASTRO_MOE_ERR_UNSUPPORTED, "%s: more than %d experts per rank", op, kMailboxExperts);
  return ASTRO_MOE_OK;
}

static const uint32_t* mailbox_matrix(astro_moe_ctx* ctx) {
  return static_cast<const uint32_t*>(ctx->xr_mbox) + (size_t)ctx->xr_world * kMailboxExperts;
}

int astro_moe_ep_post_counts(astro_moe_ctx* ctx, int32_t layer, const uint32_t* expert_offsets) {
  const char* op = "expert-parallel post counts";
  LayerState* Lp = nullptr;
  if (int rc = ep_dev_check(ctx, layer, op, &Lp)) return rc;
  if (!expert_offsets) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null offsets", op);
  DeviceGuard g(ctx->device);
  // mailbox rows are [world][kMailboxExperts]; the send matrix follows them
  const int El = Lp->w.experts;
  void* boxes[astro::kMaxPeers];
  for (int r = 0; r < ctx->xr_world; ++r) boxes[r] = ctx->xr_peer_mbox[r];
  CK(astro::launch_ep_post_counts(expert_offsets, El, ctx->xr_world, ctx->xr_rank, boxes,
                                  kMailboxExperts, ctx->stream),
     op);
  ctx->launches += 1;
  return ASTRO_MOE_OK;
}

int astro_moe_ep_push_dev(astro_moe_ctx* ctx, int32_t layer, const void* x, int64_t T) {
  const char* op = "expert-parallel push (device-planned)";
  LayerState* Lp = nullptr;
  if (int rc = ep_dev_check(ctx, layer, op, &Lp)) return rc;
  if (ctx->ep_layer != layer || ctx->ep_tokens != T)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: does not match the routing in flight", op);
  if (T == 0) return ASTRO_MOE_OK;
  const astro_moe_layer_weights& w = Lp->w;
  const int E = Lp->ep_total, K = w.top_k;
  DeviceGuard g(ctx->device);
  EpDispatch d{};
  plan_ep_dispatch(T, E, K, &d, (char*)ctx->ep_disp.p);
  CK(astro::launch_ep_push_rows_dev(x, T, d.stok, d.sids, T * K, w.experts, ctx->xr_world,
                                    ctx->xr_rank, w.hidden, mailbox_matrix(ctx), ctx->xr_peer_recv,
                                    ctx->xr_recv_rows, ctx->status, ctx->stream),
     op);
  ctx->launches += 1;
  return ASTRO_MOE_OK;
}

int astro_moe_ep_experts_dev(astro_moe_ctx* ctx, int32_t layer, const void* x, int64_t T) {
  const char* op = "expert-parallel experts (device-planned)";
  LayerState* Lp = nullptr;
  if (int rc = ep_dev_check(ctx, layer, op, &Lp)) return rc;
  LayerState& L = *Lp;
  const astro_moe_layer_weights& w = L.w;
  const int H = w.hidden, El = w.experts, I = w.intermediate, W = ctx->xr_world;
  const bool has_shared = w.shared_intermediate > 0;
  if (T < 0 || (T > 0 && !x)) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: invalid tokens", op);
  const int64_t n_cap = ctx->xr_recv_rows;  // every row this rank can receive
  const int64_t shared_rows = has_shared ? T : 0;
  const int64_t rows_cap = n_cap + shared_rows;
  DeviceGuard g(ctx->device);
  cudaStream_t st = ctx->stream;
  EpExperts e{};
  if (int rc = devbuf_ensure(ctx, ctx->ep_exp, plan_ep_experts(rows_cap, n_cap, H, I, W * El, El,
                                                               nullptr, nullptr)))
    return rc;
  plan_ep_experts(rows_cap, n_cap, H, I, W * El, El, &e, (char*)ctx->ep_exp.p);
  if (has_shared)
    if (int rc = devbuf_ensure(ctx, ctx->ep_shared, sizeof(uint16_t) * (size_t)(T > 0 ? T : 1) * H))
      return rc;
  const uint32_t* counts = static_cast<const uint32_t*>(ctx->xr_mbox);  // [W][kMailboxExperts]
  CK(astro::launch_ep_permutation_strided(counts, kMailboxExperts, W, El, (int)shared_rows, n_cap,
                                          e.src_start, e.exp_start, e.offsets, e.dest, e.src_of, st),
     "expert-major permutation");
  CK(astro::launch_ep_gather_states(ctx->xr_recv, e.src_of, x, shared_rows, W, ctx->xr_rank, H,
                                    mailbox_matrix(ctx), n_cap, e.states, ctx->status, st,
                                    astro::moe_gemm_enabled(L.gemm, ctx->opt.use_tensor_cores)),
     "expert-major rows");
  if (astro::moe_gemm_enabled(L.gemm, ctx->opt.use_tensor_cores)) {
    CK(astro::moe_gemm_gate_up(L.gemm, e.states, rows_cap, e.offsets, e.act, e.gemm_scratch,
                               ctx->status, st),
       "gate/up projection");
    CK(astro::moe_gemm_down(L.gemm, e.act, rows_cap, e.offsets, e.yrows, e.gemm_scratch, ctx->status,
                            st),
       "down projection");
  } else {
    astro::GroupedGemvDesc dsc;
    dsc.x = e.states;
    dsc.x_limit = rows_cap;
    dsc.in_features = H;
    dsc.seg_offsets = e.offsets;
    dsc.nseg = El + (has_shared ? 1 : 0);
    dsc.shared_seg = has_shared ? El : -1;
    dsc.rows_total = rows_cap;
    astro::AffineRef down[2];
    fill_projections(w, dsc.wa, dsc.wb, down);
    dsc.out_features = I;
    dsc.group = L.qgroup[0];
    dsc.bits = L.qbits[0];
    dsc.swiglu = true;
    dsc.y = e.act;
    dsc.y_limit = rows_cap;
    dsc.ldy = I;
    dsc.status = ctx->status;
    CK(astro::launch_grouped_gemv(dsc, st), "gate/up projection");
    astro::GroupedGemvDesc dd = dsc;
    dd.x = e.act;
    dd.in_features = I;
    dd.wa[0] = down[0];
    dd.wa[1] = down[1];
    dd.wb[0] = dd.wb[1] = astro::AffineRef{};
    dd.out_features = H;
    dd.group = L.qgroup[2];
    dd.bits = L.qbits[2];
    dd.swiglu = false;
    dd.y = e.yrows;
    dd.ldy = H;
    CK(astro::launch_grouped_gemv(dd, st), "down projection");
  }
  CK(astro::launch_ep_return_rows_dev(e.yrows, rows_cap, e.dest, W, ctx->xr_rank, H,
                                      mailbox_matrix(ctx), ctx->xr_peer_ret, ctx->xr_ret_rows,
                                      ctx->status, st),
     "return rows");
  if (has_shared)
    CK(astro::launch_ep_copy_shared_rows(e.yrows, rows_cap, W, ctx->xr_rank, T, H,
                                         mailbox_matrix(ctx), ctx->ep_shared.p, st),
       "shared-expert rows");
  ctx->launches += 7;
  return ASTRO_MOE_OK;
}

int astro_moe_ep_exchange_counts(astro_moe_ctx* ctx, uint32_t* host_matrix) {
  if (!ctx || !host_matrix || !ctx->xr_mbox)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "exchange counts: no exchange");
  DeviceGuard g(ctx->device);
  CK(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
  CK(cudaMemcpy(host_matrix, mailbox_matrix(ctx), sizeof(uint32_t) * ctx->xr_world * ctx->xr_world,
                cudaMemcpyDeviceToHost),
     "read count matrix");
  return ASTRO_MOE_OK;
}


// --- asynchronous host-buffer calls ------------------------------------------
int astro_moe_block_forward_host_async(astro_moe_ctx* ctx, int32_t layer, const void* host_x,
                                       int64_t T, void* host_out) {
  const char* op = "block forward (host, async)";
  if (!ctx) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null ctx", op);
  auto it = ctx->layers.find(layer);
  if (it == ctx->layers.end() || !it->second.registered)
    return fail(ASTRO_MOE_ERR_NOT_REGISTERED, "%s: layer %d is not registered", op, layer);
  if (it->second.ep || it->second.pager)
    return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: layer %d is expert-parallel or paged", op, layer);
  if (T < 0) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: negative tokens", op);
  if (T == 0) return ASTRO_MOE_OK;
  if (!host_x || !host_out) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null buffer", op);
  DeviceGuard g(ctx->device);
  const size_t bytes = sizeof(uint16_t) * (size_t)T * it->second.w.hidden;
  if (!ctx->up) {
    CK(cudaStreamCreateWithFlags(&ctx->up, cudaStreamNonBlocking), "cudaStreamCreate");
    CK(cudaStreamCreateWithFlags(&ctx->down, cudaStreamNonBlocking), "cudaStreamCreate");
    for (int i = 0; i < 2; ++i) {
      CK(cudaEventCreateWithFlags(&ctx->ev_in[i], cudaEventDisableTiming), "cudaEventCreate");
      CK(cudaEventCreateWithFlags(&ctx->ev_done[i], cudaEventDisableTiming), "cudaEventCreate");
      CK(cudaEventCreateWithFlags(&ctx->ev_out[i], cudaEventDisableTiming), "cudaEventCreate");
    }
  }
  if (ctx->aio_bytes < 2 * bytes) {
    CK(cudaStreamSynchronize(ctx->up), "sync");
    CK(cudaStreamSynchronize(ctx->down), "sync");
    CK(cudaStreamSynchronize(ctx->stream), "sync");
    for (int i = 0; i < 2; ++i) {
      if (ctx->aio[i]) cudaFree(ctx->aio[i]);
      ctx->aio[i] = nullptr;
    }
    ctx->aio_bytes = 0;
    for (int i = 0; i < 2; ++i) CK(cudaMalloc(&ctx->aio[i], 2 * bytes), "cudaMalloc(async staging)");
    ctx->aio_bytes = 2 * bytes;
  }
  const int slot = ctx->aio_next;
  ctx->aio_next ^= 1;
  char* dx = (char*)ctx->aio[slot];
  char* dy = dx + bytes;
  // the slot's input may be overwritten once the block two calls ago read it
  if (ctx->ev_done_used[slot]) CK(cudaStreamWaitEvent(ctx->up, ctx->ev_done[slot], 0), op);
  CK(cudaMemcpyAsync(dx, host_x, bytes, cudaMemcpyHostToDevice, ctx->up), "copy hidden states in");
  CK(cudaEventRecord(ctx->ev_in[slot], ctx->up), op);
  CK(cudaStreamWaitEvent(ctx->stream, ctx->ev_in[slot], 0), op);
  // ... and its output once the download two calls ago finished
  if (ctx->ev_out_used[slot]) CK(cudaStreamWaitEvent(ctx->stream, ctx->ev_out[slot], 0), op);
  if (int rc = run_block(ctx, it->second, dx, T, dy, nullptr)) return rc;
  CK(cudaEventRecord(ctx->ev_done[slot], ctx->stream), op);
  ctx->ev_done_used[slot] = true;
  CK(cudaStreamWaitEvent(ctx->down, ctx->ev_done[slot], 0), op);
  CK(cudaMemcpyAsync(host_out, dy, bytes, cudaMemcpyDeviceToHost, ctx->down), "copy output out");
  CK(cudaEventRecord(ctx->ev_out[slot], ctx->down), op);
  ctx->ev_out_used[slot] = true;
  return ASTRO_MOE_OK;
}

int astro_moe_host_synchronize(astro_moe_ctx* ctx) {
  if (!ctx) return fail(ASTRO_MOE_ERR_INVALID_ARGUMENT, "synchronize: null ctx");
  DeviceGuard g(ctx->device);
  if (ctx->up) CK(cudaStreamSynchronize(ctx->up), "cudaStreamSynchronize");
  if (ctx->down) CK(cudaStreamSynchronize(ctx->down), "cudaStreamSynchronize");
  return astro_moe_ctx_synchronize(ctx);
}

}  // extern "C"
