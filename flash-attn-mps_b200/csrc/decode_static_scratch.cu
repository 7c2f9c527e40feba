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
//   * Requests whose split partials would not fit are rejected with
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
//     that first call before any stream capture begins.
#include <mutex>

#include "kernels.cuh"

namespace fab {
namespace {

constexpr size_t kStaticScratchBytes = size_t(32) << 20;
constexpr int kMaxDevices = 256;

static __device__ __align__(256) uint8_t g_decode_scratch[kStaticScratchBytes];

std::mutex g_scratch_mutex;
void* g_scratch_address[kMaxDevices] = {nullptr};

// Device address of g_decode_scratch on the current device (host code must not
// use the symbol itself: on the host it is only a stand-in).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(FA_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(FA_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_address[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_decode_scratch);
    if (e != cudaSuccess || ptr == nullptr)
      return fail(FA_ERR_CUDA, "cudaGetSymbolAddress(static decode scratch): %s", cudaGetErrorString(e));
    g_scratch_address[dev] = ptr;
  }
  *out = g_scratch_address[dev];
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
  size_t need = 0;
  int rc = fa_attention_workspace_size(args, &need);
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
  return fa_attention_fwd(&local, stream);
}
