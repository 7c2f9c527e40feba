// tcgen05/TMEM/TMA prefill kernel (placeholder until the kernel lands).
#include "kernels.cuh"

namespace fab {
int prefill_sm100_supported(const AttnParams&) { return 0; }
int launch_prefill_sm100(const AttnParams&, cudaStream_t) {
  return fail(FA_ERR_UNSUPPORTED, "tcgen05 prefill kernel not available");
}
}  // namespace fab
