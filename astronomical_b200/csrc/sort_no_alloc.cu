// sort_no_alloc.cu -- astro_moe_sort_expert_assignments_no_alloc: the stable
// expert-assignment sort with its scratch in a fixed, file-scope device array
// instead of memory allocated per call.
//
// Who needs it: callers that cannot call cudaMalloc, cudaMallocAsync or
// cudaFree on the device.  A serving process whose own caching allocator has
// reserved all of HBM leaves nothing for the CUDA allocator, so an allocating
// call fails with out-of-memory; a latency-bound decode loop cannot accept the
// device-wide synchronisation cudaMalloc/cudaFree may perform; code embedded in
// a host framework may be forbidden to allocate outside that framework's pool.
// Such callers own every input and output buffer and pass them in; the only
// scratch the sort needs (per-tile expert histograms, plus the expert offsets
// when the caller does not want them) lives in g_sort_scratch below.
//
// The array is kNoAllocScratchBytes (256 KiB) and every GPU that loads the
// library holds it until the process exits.  A call needs
// 4 * E * ceil(tokens * top_k / 2048) bytes of it, plus 4 * (E + 1) when
// expert_offsets is NULL; larger calls are rejected before any work is queued
// (with E = 256 that is about 522k assignments).
//
// Sharing: all calls on one device use the same array and it keeps whatever the
// last call wrote.  Nothing in it has to start at zero -- the histogram pass
// writes every entry the scatter pass reads, and the offsets are written in
// full -- so no clearing is queued.  Two calls whose kernels overlap on the GPU
// (unordered streams, or several host threads on one device) race on the array
// and produce wrong results; order such calls on one stream.
//
// Set-up: the first call in each CUDA context -- normally a device's primary
// context, with that device current -- looks up the array's device address with
// cudaGetSymbolAddress (the host-side symbol is only a stand-in and must never
// reach a kernel) and keeps it for that context, keyed by the context's unique
// id (cuCtxGetId), so a kept address never outlives its context: after a
// cudaDeviceReset, or in another context the caller makes current, the next
// call looks it up again.  The first call in a context should come before any
// stream capture on it.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <map>
#include <mutex>

#include "astro_moe.h"
#include "kernels.h"

namespace {

constexpr size_t kNoAllocScratchBytes = ASTRO_MOE_NO_ALLOC_SCRATCH_BYTES;

static __device__ __align__(256) unsigned char g_sort_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
std::map<unsigned long long, void*> g_scratch_addr;  // context id -> address of g_sort_scratch

int failf(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int failf(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return astro::set_last_error(status, buf);
}

int cuda_failf(cudaError_t e, const char* what) {
  return failf(ASTRO_MOE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Unique id of the current CUDA context, or 0 when none is current or the
// driver does not report ids.
unsigned long long current_context_id() {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrent>(p);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetId>(p);
  });
  if (!get_current || !get_id) return 0;
  CUcontext c = nullptr;
  unsigned long long id = 0;
  if (get_current(&c) != CUDA_SUCCESS || !c || get_id(c, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Device address of g_sort_scratch in the current context: kept per context
// (looked up with cudaGetSymbolAddress on the first call in a context, which
// also makes the device's primary context current if none is); looked up on
// every call when the context cannot be identified.
int scratch_address(void** out) {
  const unsigned long long id = current_context_id();
  if (id != 0) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_scratch_addr.find(id);
    if (it != g_scratch_addr.end()) {
      *out = it->second;
      return ASTRO_MOE_OK;
    }
  }
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_sort_scratch);
  if (e != cudaSuccess) return cuda_failf(e, "cudaGetSymbolAddress(no-alloc sort scratch)");
  if (!p) return failf(ASTRO_MOE_ERR_CUDA, "cudaGetSymbolAddress returned a null address");
  const unsigned long long id2 = current_context_id();
  if (id2 != 0) {
    std::lock_guard<std::mutex> lk(g_mu);
    g_scratch_addr[id2] = p;
  }
  *out = p;
  return ASTRO_MOE_OK;
}

}  // namespace

extern "C" int astro_moe_sort_expert_assignments_no_alloc(
    const uint32_t* ids, int64_t tokens, int32_t top_k, int32_t experts, uint32_t* sorted_order,
    uint32_t* inverse_order, uint32_t* sorted_ids, uint32_t* sorted_tokens,
    uint32_t* expert_offsets, uint32_t* device_status, void* stream) {
  const char* op = "sort stacked expert assignments (no-alloc)";
  if (tokens < 0 || top_k < 0 || experts <= 0)
    return failf(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: expert assignments have invalid shapes", op);
  if (experts > 1024)
    return failf(ASTRO_MOE_ERR_UNSUPPORTED, "%s: experts <= 1024 are supported", op);
  if (tokens * (int64_t)top_k > 0xffffffffLL)
    return failf(ASTRO_MOE_ERR_INVALID_ARGUMENT,
                 "%s: expert assignment count exceeds the integer range", op);
  const int64_t n = tokens * (int64_t)top_k;
  if (n > 0 && !ids) return failf(ASTRO_MOE_ERR_INVALID_ARGUMENT, "%s: null ids", op);
  const size_t hist_bytes = astro::sort_scratch_bytes(n, experts);
  const size_t offs_bytes = expert_offsets ? 0 : sizeof(uint32_t) * (size_t)(experts + 1);
  if (hist_bytes + offs_bytes > kNoAllocScratchBytes)
    return failf(ASTRO_MOE_ERR_UNSUPPORTED,
                 "%s: %lld assignments over %d experts need %zu bytes of scratch, more than the "
                 "%zu-byte static array holds; astro_moe_sort_expert_assignments "
                 "(which allocates its scratch) has no such limit",
                 op, (long long)n, (int)experts, hist_bytes + offs_bytes, kNoAllocScratchBytes);
  void* scratch = nullptr;
  if (int rc = scratch_address(&scratch)) return rc;
  char* base = static_cast<char*>(scratch);
  uint32_t* offs = expert_offsets ? expert_offsets : reinterpret_cast<uint32_t*>(base + hist_bytes);
  cudaError_t e = astro::launch_sort_assignments(
      ids, tokens, top_k, experts, 0, sorted_order, inverse_order, sorted_ids, sorted_tokens, offs,
      device_status, scratch, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_failf(e, op);
  return ASTRO_MOE_OK;
}
