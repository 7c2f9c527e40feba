// Per-score feature semantics shared by the generic and the mma.sync
// attention kernels: K/V addressing (packed or paged) and the reference's
// allowed_key predicate (flash_attn_mps/kernels/attention.metal:29-45).
#pragma once

#include "kernels.cuh"

namespace fab {

__device__ __forceinline__ int64_t kv_offset(const AttnParams& p, int b, int64_t token, int kh,
                                             bool value) {
  const int64_t s0 = value ? p.vs0 : p.ks0, s1 = value ? p.vs1 : p.ks1, s2 = value ? p.vs2 : p.ks2;
  if (p.paged) {
    const int64_t page = token / p.page;
    const int64_t block = p.table[b * p.bt0 + page * p.bt1];
    return block * s0 + (token - page * p.page) * s1 + kh * s2;
  }
  return token * s1 + kh * s2;
}

// Global position of local key index t under context parallelism (identity
// without it), and the global KV length the queries are aligned to.
__device__ __forceinline__ int key_pos(const AttnParams& p, int t) { return p.cp_n > 1 ? t * p.cp_n + p.cp_r : t; }
__device__ __forceinline__ int kv_total(const AttnParams& p, int b, int k_len) {
  return p.cp_n > 1 ? p.cp_tot[b * p.ct0] : k_len;
}

// attention.metal:29-45
__device__ __forceinline__ bool allowed_key(const AttnParams& p, int b, int token, int q_abs,
                                            int64_t packed_q, bool causal) {
  const int diff = q_abs - token;
  if (p.mask == 1) {
    const bool local = diff >= 0 && (p.mask_win < 0 || diff < p.mask_win);
    const int lo = p.mr[packed_q * p.mr0], hi = p.mr[packed_q * p.mr0 + p.mr1];
    bool modality = lo >= 0 && token >= lo && token <= hi;
    if (p.clamp) modality = modality && (p.mask_win < 0 || diff < p.mask_win);
    return local || modality;
  }
  if (p.mask == 2) return diff >= 0 && (token < p.mp[b * p.mp0] || diff < p.mw[0]);
  return (!causal || diff >= 0) && (p.win_l < 0 || diff <= p.win_l) &&
         (p.win_r < 0 || -diff <= p.win_r);
}

}  // namespace fab
