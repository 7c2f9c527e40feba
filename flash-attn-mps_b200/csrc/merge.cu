// Stable log-sum-exp merges of attention states (bandwidth kernels).
//
//   merge_pair      reference kernels/merge.metal:9-28, host _merge.py:20-41
//   merge_partials  reference kernels/merge.metal:30-58 and
//                   kernels/attention_decode.metal:151-207, host _merge.py:44-57
//
// One warp owns one (token, head) row: lane 0..S-1 reads the split LSEs, the
// weights are reduced with warp shuffles, and the lanes stride over the head
// dimension, so each row's payload is read once with coalesced accesses. A
// row's LSE is read by every lane before any lane writes, which keeps the
// in-place pairwise merge (out/out_lse aliasing the left state) safe.
#include "common.cuh"
#include "kernels.cuh"

namespace fab {

namespace {

struct PairArgs {
  void* out; const void* left; const void* right;
  const float* llse; const float* rlse; float* olse;
  int64_t os0, os1, os2, ls0, ls1, ls2, rs0, rs1, rs2;
  int64_t lls0, lls1, rls0, rls1, ols0, ols1;
  int32_t T, H, D, dtype, has_olse;
};

__device__ __forceinline__ float pair_weight(float x, float maximum) {
  if (maximum == -INFINITY) return 0.f;
  if (maximum == INFINITY) return x == maximum ? 1.f : 0.f;
  return expf(x - maximum);
}

__global__ void __launch_bounds__(256) merge_pair_kernel(PairArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)a.T * a.H;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows;
       row += warps) {
    const int64_t t = row / a.H, h = row % a.H;
    const float la = a.llse[h * a.lls0 + t * a.lls1];
    const float lb = a.rlse[h * a.rls0 + t * a.rls1];
    __syncwarp();
    const float maximum = fmaxf(la, lb);
    const bool empty = maximum == -INFINITY;
    const float wa = pair_weight(la, maximum), wb = pair_weight(lb, maximum);
    const float total = wa + wb;
    for (int d = lane; d < a.D; d += 32) {
      float value = 0.f;
      if (wa > 0.f) value += wa * load_float(a.left, a.dtype, t * a.ls0 + h * a.ls1 + d * a.ls2);
      if (wb > 0.f) value += wb * load_float(a.right, a.dtype, t * a.rs0 + h * a.rs1 + d * a.rs2);
      if (!empty) value /= total;
      store_float(a.out, a.dtype, t * a.os0 + h * a.os1 + d * a.os2, value);
    }
    if (a.has_olse && lane == 0)
      a.olse[h * a.ols0 + t * a.ols1] = empty ? -INFINITY : maximum + logf(total);
  }
}

}  // namespace

// N-way merge, also the combine step of split-KV attention and of the
// multi-GPU KV-sharded decode.
__global__ void __launch_bounds__(256) merge_partials_kernel(MergePartialsArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)a.T * a.H;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows;
       row += warps) {
    const int64_t t = row / a.H, h = row % a.H;
    float maximum = -INFINITY;
    for (int s = lane; s < a.S; s += 32) maximum = fmaxf(maximum, a.lse[s * a.ls0 + h * a.ls1 + t * a.ls2]);
    maximum = warp_max(maximum);
    const bool empty = maximum == -INFINITY;
    float denominator = 0.f;
    if (!empty)
      for (int s = lane; s < a.S; s += 32)
        denominator += pair_weight(a.lse[s * a.ls0 + h * a.ls1 + t * a.ls2], maximum);
    denominator = warp_sum(denominator);
    const float inverse = empty ? 0.f : 1.f / denominator;
    for (int d0 = 0; d0 < a.D; d0 += 32) {
      const int d = d0 + lane;
      float value = 0.f;
      if (!empty) {
        for (int s0 = 0; s0 < a.S; s0 += 32) {
          const int sl = s0 + lane;
          const float w = sl < a.S ? pair_weight(a.lse[sl * a.ls0 + h * a.ls1 + t * a.ls2], maximum) : 0.f;
          const int count = min(32, a.S - s0);
          for (int j = 0; j < count; ++j) {
            const float wj = __shfl_sync(0xffffffffu, w, j);
            if (wj > 0.f && d < a.D)
              value = fmaf(wj, load_float(a.partial, a.pdtype, (s0 + j) * a.ps0 + t * a.ps1 + h * a.ps2 + d * a.ps3), value);
          }
        }
        value *= inverse;
      }
      if (d < a.D) store_float(a.out, a.odtype, t * a.os0 + h * a.os1 + d * a.os2, value);
    }
    if (lane == 0 && a.out_lse)
      a.out_lse[h * a.ols0 + t * a.ols1] = empty ? -INFINITY : maximum + logf(denominator);
  }
}

int launch_merge_partials(const MergePartialsArgs& a, cudaStream_t stream) {
  const int64_t rows = (int64_t)a.T * a.H;
  if (rows == 0) return FA_OK;
  int64_t blocks = (rows + 7) / 8;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  merge_partials_kernel<<<(unsigned)blocks, 256, 0, stream>>>(a);
  note_launch();
  FAB_LAUNCH_CHECK("merge_partials launch");
  return FA_OK;
}

}  // namespace fab

using namespace fab;

extern "C" int fa_merge_attn_states(const fa_tensor* out, const fa_tensor* left,
                                    const fa_tensor* left_lse, const fa_tensor* right,
                                    const fa_tensor* right_lse, const fa_tensor* out_lse,
                                    void* stream) {
  FAB_CHECK_ARG(present(out) && present(left) && present(right) && present(left_lse) &&
                    present(right_lse), "merge_attn_states requires both states and out");
  FAB_CHECK_ARG(out->ndim == 3 && left->ndim == 3 && right->ndim == 3,
                "output states must have matching [tokens, heads, dim] shapes");
  for (int i = 0; i < 3; ++i)
    FAB_CHECK_ARG(left->shape[i] == out->shape[i] && right->shape[i] == out->shape[i],
                  "output states must have matching [tokens, heads, dim] shapes");
  FAB_CHECK_ARG(left->dtype == out->dtype && right->dtype == out->dtype && is_float(out->dtype),
                "output state dtypes must match");
  const fa_tensor* lses[3] = {left_lse, right_lse, present(out_lse) ? out_lse : nullptr};
  for (const fa_tensor* l : lses)
    if (l)
      FAB_CHECK_ARG(l->ndim == 2 && l->dtype == FA_F32 && l->shape[0] == out->shape[1] &&
                        l->shape[1] == out->shape[0], "LSE tensors must be float32 [heads, tokens]");
  PairArgs a{};
  a.out = out->ptr; a.left = left->ptr; a.right = right->ptr;
  a.llse = reinterpret_cast<const float*>(left_lse->ptr);
  a.rlse = reinterpret_cast<const float*>(right_lse->ptr);
  a.os0 = out->stride[0]; a.os1 = out->stride[1]; a.os2 = out->stride[2];
  a.ls0 = left->stride[0]; a.ls1 = left->stride[1]; a.ls2 = left->stride[2];
  a.rs0 = right->stride[0]; a.rs1 = right->stride[1]; a.rs2 = right->stride[2];
  a.lls0 = left_lse->stride[0]; a.lls1 = left_lse->stride[1];
  a.rls0 = right_lse->stride[0]; a.rls1 = right_lse->stride[1];
  a.has_olse = present(out_lse);
  if (a.has_olse) {
    a.olse = reinterpret_cast<float*>(out_lse->ptr);
    a.ols0 = out_lse->stride[0]; a.ols1 = out_lse->stride[1];
  }
  a.T = (int32_t)out->shape[0]; a.H = (int32_t)out->shape[1]; a.D = (int32_t)out->shape[2];
  a.dtype = out->dtype;
  const int64_t rows = (int64_t)a.T * a.H;
  if (rows == 0 || a.D == 0) return FA_OK;
  int64_t blocks = (rows + 7) / 8;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  merge_pair_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  note_launch();
  FAB_LAUNCH_CHECK("merge_attn_states launch");
  return FA_OK;
}

extern "C" int fa_merge_partials(const fa_tensor* partial, const fa_tensor* partial_lse,
                                 const fa_tensor* out, const fa_tensor* out_lse, void* stream) {
  FAB_CHECK_ARG(present(partial) && present(partial_lse) && present(out),
                "merge_partials requires partials, their LSE and out");
  FAB_CHECK_ARG(partial->ndim == 4 && partial_lse->ndim == 3 &&
                    partial_lse->shape[0] == partial->shape[0] &&
                    partial_lse->shape[1] == partial->shape[2] &&
                    partial_lse->shape[2] == partial->shape[1],
                "partial states require [splits,tokens,heads,dim] and [splits,heads,tokens]");
  FAB_CHECK_ARG(partial_lse->dtype == FA_F32, "partial LSE must be float32");
  FAB_CHECK_ARG(is_float(partial->dtype) && is_float(out->dtype), "partials and out must be float");
  FAB_CHECK_ARG(out->ndim == 3 && out->shape[0] == partial->shape[1] &&
                    out->shape[1] == partial->shape[2] && out->shape[2] == partial->shape[3],
                "out must be [tokens, heads, dim]");
  MergePartialsArgs a{};
  a.partial = partial->ptr; a.pdtype = partial->dtype;
  for (int i = 0; i < 4; ++i) (&a.ps0)[i] = partial->stride[i];
  a.lse = reinterpret_cast<const float*>(partial_lse->ptr);
  a.ls0 = partial_lse->stride[0]; a.ls1 = partial_lse->stride[1]; a.ls2 = partial_lse->stride[2];
  a.out = out->ptr; a.odtype = out->dtype;
  a.os0 = out->stride[0]; a.os1 = out->stride[1]; a.os2 = out->stride[2];
  if (present(out_lse)) {
    FAB_CHECK_ARG(out_lse->ndim == 2 && out_lse->dtype == FA_F32 &&
                      out_lse->shape[0] == out->shape[1] && out_lse->shape[1] == out->shape[0],
                  "out_lse must be float32 [heads, tokens]");
    a.out_lse = reinterpret_cast<float*>(out_lse->ptr);
    a.ols0 = out_lse->stride[0]; a.ols1 = out_lse->stride[1];
  }
  a.S = (int32_t)partial->shape[0]; a.T = (int32_t)partial->shape[1];
  a.H = (int32_t)partial->shape[2]; a.D = (int32_t)partial->shape[3];
  return launch_merge_partials(a, reinterpret_cast<cudaStream_t>(stream));
}
