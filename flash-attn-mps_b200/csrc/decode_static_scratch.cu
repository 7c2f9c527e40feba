// Split-KV paged decode for callers that cannot allocate device memory.
//
// fa_attention_fwd needs a caller-provided workspace for the split-KV
// partials (sized by fa_attention_workspace_size). Some callers cannot
// provide one: hosts that reach this library through a C FFI holding only raw
// pointers handed out by another framework's allocator, processes whose whole
// device memory budget is pre-reserved by a pool they do not control, and
// latency-critical decode loops that must never call cudaMalloc (it can
// synchronise the device). fa_decode_fwd_noalloc serves them: the split
// partials live in the file-scope static device array below, so the call
// itself allocates nothing.
//
// Contract of the static scratch:
//   * Its size is fixed at kStaticScratchBytes (32 MiB); every GPU on which
//     the library's module is loaded holds it until the process exits.
//   * When the library chooses the split count (num_splits == 0) it lowers
//     that count until the partials fit (one split needs no partials at all).
//     An explicit num_splits whose partials would not fit is rejected with
//     FA_ERR_INVALID before anything is launched (lower num_splits, or use
//     fa_attention_fwd with a caller workspace).
//   * All calls on a device share the one array and it keeps the previous
//     call's contents. The split partials need no clearing: every split of
//     every (token, head) writes its partial output and LSE before the merge
//     reads them. The one value that must start at zero -- the work counter of
//     the persistent tensor-core kernel, which a num_splits == 1 (batch-
//     invariant) call runs -- is zeroed on the stream by that launch itself.
//     Calls whose GPU work overlaps (different streams without ordering, or
//     concurrent host threads on different streams) race on the array.
//   * The first call on a device resolves the array's device address with
//     cudaGetSymbolAddress (this may load the module on that device); make
//     that first call before any stream capture begins. The address is cached
//     per device together with the CUDA context that was current when it was
//     resolved; a call under another context (a driver-API context, or the
//     primary context re-created after cudaDeviceReset) resolves it again.
#include <cudaTypedefs.h>

#include <mutex>

#include "kernels.cuh"

namespace fab {
namespace {

constexpr size_t kStaticScratchBytes = size_t(32) << 20;
constexpr int kMaxDevices = 256;

static __device__ __align__(256) uint8_t g_decode_scratch[kStaticScratchBytes];

struct ScratchAddress {
  CUcontext context;  // current context when `ptr` was resolved
  void* ptr;
};
std::mutex g_scratch_mutex;
ScratchAddress g_scratch_address[kMaxDevices] = {};

// The calling thread's current CUDA context (nullptr when the driver entry
// point is unavailable; the address is then cached per device only).
CUcontext current_context() {
  static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(ptr);
  });
  CUcontext ctx = nullptr;
  if (fn == nullptr || fn(&ctx) != CUDA_SUCCESS) return nullptr;
  return ctx;
}

// Device address of g_decode_scratch on the current device (host code must not
// use the symbol itself: on the host it is only a stand-in).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(FA_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(FA_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  const CUcontext ctx = current_context();
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  ScratchAddress& slot = g_scratch_address[dev];
  if (slot.ptr == nullptr || slot.context != ctx) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_decode_scratch);
    if (e != cudaSuccess || ptr == nullptr)
      return fail(FA_ERR_CUDA, "cudaGetSymbolAddress(static decode scratch): %s", cudaGetErrorString(e));
    // Read the context again: resolving may have made the primary context
    // current on a thread that had none.
    slot.context = current_context();
    slot.ptr = ptr;
  }
  *out = slot.ptr;
  return FA_OK;
}

}  // namespace
}  // namespace fab

using namespace fab;

extern "C" int fa_decode_fwd_noalloc(const fa_attention_args* args, void* stream) {
  FAB_CHECK_ARG(args != nullptr, "null arguments");
  FAB_CHECK_ARG(args->max_seqlen_q == 1 && !args->deterministic && args->alibi_slopes.ptr == nullptr &&
                    args->mask_kind == 0,
                "fa_decode_fwd_noalloc serves single-query decode only "
                "(max_seqlen_q == 1, no ALiBi, no mask, not deterministic)");
  // A library-chosen split count is lowered until its partials fit.
  const size_t cap = args->num_splits == 0 ? kStaticScratchBytes : 0;
  size_t need = 0;
  int rc = attention_workspace_capped(args, &need, cap);
  if (rc) return rc;
  if (need > kStaticScratchBytes)
    return fail(FA_ERR_INVALID,
                "split-KV partials need %zu bytes but the static scratch of fa_decode_fwd_noalloc "
                "holds %zu; lower num_splits or use fa_attention_fwd with a caller workspace",
                need, kStaticScratchBytes);
  fa_attention_args local = *args;
  local.workspace = fa_tensor{};
  if (need > 0) {
    void* ptr = nullptr;
    rc = scratch_address(&ptr);
    if (rc) return rc;
    local.workspace.ptr = ptr;
    local.workspace.dtype = FA_U8;
    local.workspace.ndim = 1;
    local.workspace.shape[0] = (int64_t)kStaticScratchBytes;
    local.workspace.stride[0] = 1;
  }
  return attention_fwd_capped(&local, stream, cap);
}
