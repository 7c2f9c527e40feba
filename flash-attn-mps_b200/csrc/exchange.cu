// KV-sharded decode: the exchange of the ranks' partial states over NVLink
// peer memory, in place of an NCCL all-gather.
//
// Each rank owns a gather buffer in symmetric memory (the same allocation
// mapped into every rank's address space): two parities x N slots of one
// packed fp32 row [B*Hq*Dv | Hq*B] (the rank's partial output and LSE), then a
// small flag array. A decode step with epoch e (1, 2, ...):
//   1. the local decode writes this rank's row into its own slot
//      (parity e & 1, slot rank) of its own buffer;
//   2. fa_shard_push copies that row into slot `rank` of every peer's buffer
//      (16-byte peer stores over NVLink / NVSwitch); the last CTA to finish
//      fences at system scope and raises flag[rank] = e on every peer;
//   3. fa_shard_wait spins (bounded) until flag[p] >= e for every peer p on
//      this rank;
//   4. the N-way merge kernel combines the N slots of parity e & 1.
// Two parities make the buffer safe to reuse: a rank can start step e+1 only
// after every peer has pushed step e, so no rank is ever more than one step
// ahead of another's reads. No TMA and no NVSwitch reductions: plain peer
// stores and loads.
// A wait that gives up sets g_exchange_timeout (fa_pipeline_timeouts bit 2)
// and returns; the merged outputs of that step are then undefined.
#include <algorithm>

#include "kernels.cuh"

namespace fab {
namespace {

__device__ int g_exchange_timeout;

constexpr int kPushThreads = 256;

// Slot `slot` of parity `par` in a gather buffer of `world` slots per parity.
__device__ __forceinline__ uint4* slot_ptr(void* buf, int par, int world, int slot, int64_t row16) {
  return reinterpret_cast<uint4*>(buf) + ((int64_t)par * world + slot) * row16;
}

__global__ void __launch_bounds__(kPushThreads)
    shard_push_kernel(const uint4* __restrict__ row, int64_t row16, fa_peer_buffers peers, int world, int rank,
                      uint32_t epoch) {
  const int par = (int)(epoch & 1u);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < row16; i += stride) {
    const uint4 v = __ldg(row + i);
#pragma unroll 1
    for (int p = 0; p < world; ++p)
      if (p != rank) slot_ptr(peers.slots[p], par, world, rank, row16)[i] = v;
  }
  // Last CTA: every CTA's peer stores are ordered before its counter update;
  // the last one then publishes this rank's row to every peer.
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* counter = peers.flags[rank] + FA_MAX_PEERS;
    const uint32_t done = atomicAdd(counter, 1u);
    if (done == gridDim.x - 1) {
      *counter = 0u;
      __threadfence_system();
      for (int p = 0; p < world; ++p) {
        if (p == rank) continue;
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(peers.flags[p] + rank), "r"(epoch) : "memory");
      }
    }
  }
}

__global__ void shard_wait_kernel(fa_peer_buffers peers, int world, int rank, uint32_t epoch) {
  // Lane p < world waits for rank p's flag on this rank.
  const int p = threadIdx.x;
  bool ok = true;
  if (p < world && p != rank) {
    const uint32_t* flag = peers.flags[rank] + p;
    uint32_t v = 0;
    long long spins = 0;
    while (true) {
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
      // Epochs only grow; the signed difference survives wrap-around.
      if ((int32_t)(v - epoch) >= 0) break;
      if (++spins > (1LL << 22)) {
        ok = false;
        break;
      }
      __nanosleep(64);
    }
  }
  if (!ok) atomicExch(&g_exchange_timeout, 1);
  __threadfence_system();
}

int check_peers(const fa_peer_buffers* peers, int world, int rank) {
  FAB_CHECK_ARG(peers != nullptr, "peer buffers are required");
  FAB_CHECK_ARG(world >= 2 && world <= FA_MAX_PEERS, "world size must be in [2, FA_MAX_PEERS]");
  FAB_CHECK_ARG(rank >= 0 && rank < world, "rank must be in [0, world)");
  for (int p = 0; p < world; ++p) {
    FAB_CHECK_ARG(peers->slots[p] != nullptr && peers->flags[p] != nullptr, "every rank needs a buffer and flags");
    FAB_CHECK_ARG(((uintptr_t)peers->slots[p] & 15u) == 0, "gather buffers must be 16-byte aligned");
    FAB_CHECK_ARG(((uintptr_t)peers->flags[p] & 3u) == 0, "flag arrays must be 4-byte aligned");
  }
  return FA_OK;
}

}  // namespace

int exchange_timeout_flag(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_exchange_timeout, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_exchange_timeout, &zero, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

}  // namespace fab

using namespace fab;

extern "C" int fa_shard_push(const fa_tensor* row, const fa_peer_buffers* peers, int32_t world, int32_t rank,
                             uint32_t epoch, void* stream) {
  int rc = check_peers(peers, world, rank);
  if (rc) return rc;
  FAB_CHECK_ARG(row != nullptr && present(*row) && row->dtype == FA_F32 && row->ndim == 1 && row->stride[0] == 1,
                "row must be a contiguous float32 vector");
  FAB_CHECK_ARG(row->shape[0] % 4 == 0 && ((uintptr_t)row->ptr & 15u) == 0,
                "row length must be a multiple of 4 floats, 16-byte aligned");
  FAB_CHECK_ARG(epoch != 0, "epochs start at 1");
  const int64_t row16 = row->shape[0] / 4;
  if (row16 == 0) return FA_OK;
  const int64_t blocks_needed = (row16 + kPushThreads - 1) / kPushThreads;
  const int grid = (int)std::min<int64_t>(blocks_needed, (int64_t)sm_count() * 2);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  shard_push_kernel<<<grid, kPushThreads, 0, st>>>(reinterpret_cast<const uint4*>(row->ptr), row16, *peers, world,
                                                   rank, epoch);
  note_launch();
  FAB_LAUNCH_CHECK("shard push launch");
  return FA_OK;
}

extern "C" int fa_shard_wait(const fa_peer_buffers* peers, int32_t world, int32_t rank, uint32_t epoch,
                             void* stream) {
  int rc = check_peers(peers, world, rank);
  if (rc) return rc;
  FAB_CHECK_ARG(epoch != 0, "epochs start at 1");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  shard_wait_kernel<<<1, 32, 0, st>>>(*peers, world, rank, epoch);
  note_launch();
  FAB_LAUNCH_CHECK("shard wait launch");
  return FA_OK;
}
