// Internal launch interfaces shared by the attention kernels and the dispatcher.
#pragma once

#include "common.cuh"

namespace fab {

struct MergePartialsArgs {
  const void* partial; int32_t pdtype;
  int64_t ps0, ps1, ps2, ps3;      // [S,T,H,D]
  const float* lse; int64_t ls0, ls1, ls2;  // [S,H,T]
  void* out; int32_t odtype; int64_t os0, os1, os2;  // [T,H,D]
  float* out_lse; int64_t ols0, ols1;  // [H,T]
  int32_t S, T, H, D;
};
int launch_merge_partials(const MergePartialsArgs& a, cudaStream_t stream);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda
// link dependency). rank <= 5; strides in bytes for dims 1..rank-1.
bool tensor_map_available();
int encode_tensor_map(void* map, int dtype, int rank, const void* ptr, const uint64_t* dims,
                      const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128);

// Flattened attention parameters: device pointers, element strides and
// feature flags. Mirrors the reference's parameter vector
// (flash_attn_mps/_attention.py:10-16 _META, filled at 183-213).
struct AttnParams {
  const void* q; const void* k; const void* v;
  int32_t qt, kt, vt;              // element dtypes (FA_*)
  int64_t qs0, qs1, qs2;           // q [T,H,D]
  int64_t ks0, ks1, ks2, ks3;      // k paged [N,P,H,D] / packed [-,T,H,D] (ks0 unused)
  int64_t vs0, vs1, vs2, vs3;
  // Final output (or, with splits > 1, fp32 partials [S,T,H,Dv] at `part`).
  void* out; int32_t ot; int64_t os0, os1, os2;
  float* lse; int64_t ls0, ls1;    // [H,T]
  float* part; float* part_lse;    // split workspace (contiguous) or null
  void* scratch;                   // prefill: work counter (zeroed before launch)
  const int32_t* cu_q; int64_t cq0;
  const int32_t* cu_k; int64_t ck0;
  const int32_t* used; int64_t u0;
  const int32_t* table; int64_t bt0, bt1;
  const int32_t* leftpad; int64_t lp0;
  const uint8_t* causal_b; int64_t ca0;
  const float* alibi; int64_t a0, a1;
  const void* sinks; int32_t sink_t; int64_t si0;
  const float* qd; int64_t qd0, qd1;
  const float* kd; int64_t kd0, kd1;
  const float* vd; int64_t vd0, vd1;
  const int32_t* mr; int64_t mr0, mr1;   // mask kind 1 ranges [T,2]
  const int32_t* mp; int64_t mp0;        // mask kind 2 prefix [B]
  const int32_t* mw;                      // mask kind 2 window [1]
  int64_t k_rows;                        // packed K/V: rows of the K/V tensors
  int64_t k_pages, bt_cols;              // paged K/V: pages in the cache, block_table columns
  // Context parallelism: local key j is global position j * cp_n + cp_r;
  // cp_tot[b] is the global KV length (queries sit at its end). cp_n <= 1: off.
  const int32_t* cp_tot; int64_t ct0;
  int32_t cp_n, cp_r;
  int32_t T, B, HQ, HK, DQ, DV, page;
  int32_t paged, causal, dynamic, win_l, win_r;
  int32_t mask, mask_win, clamp, splits, max_q, max_k;
  float scale, softcap;
};

// Generic SIMT kernel: every feature, dtype and head dimension (1..512).
int launch_generic_attention(const AttnParams& p, cudaStream_t stream);

// Tensor-core paged/packed decode (one query per request). Returns
// FA_ERR_UNSUPPORTED when the arguments fall outside its envelope.
int decode_mma_supported(const AttnParams& p);
int launch_decode_mma(const AttnParams& p, int splits, int span, cudaStream_t stream);
int decode_default_splits(const AttnParams& p, int* span);

// tcgen05/TMEM/TMA prefill kernel.
int prefill_sm100_supported(const AttnParams& p);
int launch_prefill_sm100(const AttnParams& p, cudaStream_t stream);
int mma_attention_supported(const AttnParams& p);
int launch_mma_attention(const AttnParams& p, cudaStream_t stream);
// FP8 E4M3 K/V prefill on the tcgen05 kernel through an exact 16-bit copy of
// the K/V rows (kv_dequant.cu): rows of that copy, the prefill's view of it
// (false when the prefill cannot take it), and the conversion launch.
int64_t fp8_prefill_rows(const AttnParams& p);
bool fp8_prefill_view(const AttnParams& p, AttnParams* view);
int launch_kv_dequant(const AttnParams& p, void* k_out, void* v_out, int32_t* cu_out, int32_t* used_out,
                      cudaStream_t stream);
// fa_attention_workspace_size / fa_attention_fwd with a bound on the split
// partials: part_cap > 0 lowers a library-chosen decode split count until its
// partials fit in part_cap bytes (0 = no bound, the public behaviour).
int attention_workspace_capped(const fa_attention_args* a, size_t* bytes, size_t part_cap);
int attention_fwd_capped(const fa_attention_args* a, void* stream, size_t part_cap);
// Timed-out pipeline waits recorded by the prefill / TMA decode kernels on the
// current device (1 = some wait gave up, 0 = none, -1 = CUDA error).
int prefill_timeout_flag(bool clear);
int decode_timeout_flag(bool clear);
int exchange_timeout_flag(bool clear);

}  // namespace fab
