/*
 * flash_attn_b200 — C ABI of the B200 (sm_100a) FlashAttention inference kernels.
 *
 * This is the drop-in boundary that replaces the reference's host dispatch
 * layer (SuperMarioYL/flash-attn-mps 0.1.0, directory flash_attn_mps/), whose
 * Python functions compile and launch Metal shaders. Each entry point below
 * names the reference function it replaces.
 *
 * Conventions
 *  - Every tensor is an fa_tensor: a device pointer plus shape and ELEMENT
 *    strides (not bytes), up to 4 dimensions. ptr == NULL means "absent".
 *  - The caller owns all memory, including the split-KV workspace sized by
 *    fa_attention_workspace_size(). The library never allocates or frees
 *    device memory and never synchronises the host.
 *  - Every launch is asynchronous on the caller's CUDA stream (a cudaStream_t
 *    passed as void*; NULL = legacy default stream).
 *  - Sequence metadata (cu_seqlens, seqused_k, block_table, slots) is read on
 *    the device only; the host never reads tensor values.
 *  - Return value: 0 = success, FA_ERR_INVALID = bad argument (nothing was
 *    launched), FA_ERR_UNSUPPORTED = valid but unsupported combination,
 *    FA_ERR_CUDA = a CUDA launch error. fa_last_error() gives the message of
 *    the calling thread's last failure.
 */
#ifndef FLASH_ATTN_B200_H
#define FLASH_ATTN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FA_B200_ABI_VERSION 2

enum {
  FA_OK = 0,
  FA_ERR_INVALID = 1,
  FA_ERR_UNSUPPORTED = 2,
  FA_ERR_CUDA = 3
};

/* Element types. FA_E4M3 is float8_e4m3fn storage (one byte). */
enum {
  FA_DTYPE_NONE = 0,
  FA_F16 = 1,
  FA_BF16 = 2,
  FA_F32 = 3,
  FA_E4M3 = 4,
  FA_I32 = 5,
  FA_I64 = 6,
  FA_BOOL = 7,
  FA_U8 = 8
};

typedef struct fa_tensor {
  void* ptr;
  int32_t dtype;
  int32_t ndim;
  int64_t shape[4];
  int64_t stride[4];
} fa_tensor;

/*
 * Arguments of one attention call. Field meanings follow the reference's
 * internal attention() (flash_attn_mps/_attention.py:88-94):
 *   q [Tq,Hq,Dq]; k/v packed [Tk,Hkv,Dq|Dv] or paged [N,P,Hkv,Dq|Dv];
 *   out [Tq,Hq,Dv] (f16/bf16/f32, any strides); lse [Hq,Tq] f32.
 * Query row i of a request with Sq queries and Sk keys sits at absolute
 * position i + Sk - Sq (lower-right causal, docs/contracts.md:32-37).
 */
typedef struct fa_attention_args {
  fa_tensor q, k, v, out, lse;
  fa_tensor cu_seqlens_q;   /* int32 [B+1] */
  fa_tensor cu_seqlens_k;   /* int32 [B+1] or absent */
  fa_tensor seqused_k;      /* int32 [B] or absent (exactly one of the two) */
  fa_tensor block_table;    /* int32 [B,pages] (paged K/V) or absent */
  fa_tensor leftpad_k;      /* int32 [B] or absent */
  fa_tensor causal_per_seq; /* bool [B] (dynamic causal) or absent */
  fa_tensor alibi_slopes;   /* f32 [Hq] or [B,Hq] or absent */
  fa_tensor s_aux;          /* sinks, [Hq] f16/bf16/f32, or absent */
  fa_tensor q_descale, k_descale, v_descale; /* f32 [B,Hkv] (zero strides allowed) */
  fa_tensor mask_aux0, mask_aux1; /* kind 1: ranges int32 [Tq,2], cu_q int32 [B+1];
                                     kind 2: prefix int32 [B], window int32 [1] */
  fa_tensor workspace;      /* uint8 [bytes] from fa_attention_workspace_size */
  int32_t batch;
  int32_t max_seqlen_q, max_seqlen_k;
  float softmax_scale;      /* resolved by the caller (reference default Dq^-0.5) */
  float softcap;            /* 0 disables; applied as cap*tanh(s/cap) before masking */
  int32_t causal;           /* static causal flag, ignored when causal_per_seq is set */
  int32_t window_left, window_right; /* -1 = unbounded */
  int32_t mask_kind;        /* 0 none, 1 mm-prefix, 2 rolling SWA */
  int32_t mask_window;      /* mm-prefix sliding window (-1 none) */
  int32_t mask_clamp;       /* mm-prefix: clamp the bidirectional range to the window */
  int32_t num_splits;       /* 0 = library chooses; >0 exact split-KV count */
  int32_t deterministic;    /* 1 = fixed batch-invariant reduction schedule */
  /* Context parallelism (vLLM DCP, ABI 2): this rank holds KV tokens
   * cp_rank, cp_rank + cp_world_size, ... of each sequence (local index j =
   * global position j * cp_world_size + cp_rank); causal, window, mask and
   * ALiBi positions are global, queries sit at the end of cp_tot_seqused_k
   * (int32 [B], the global KV lengths); sinks count on rank 0 only. The
   * caller merges the ranks' (out, lse). cp_world_size 0 or 1 = off. No
   * counterpart in the reference, which rejects these arguments
   * (flash_attn_mps/vllm.py:51-53). */
  fa_tensor cp_tot_seqused_k;
  int32_t cp_world_size, cp_rank;
} fa_attention_args;

/* Library ABI version (FA_B200_ABI_VERSION). */
int fa_abi_version(void);

/* Message of the calling thread's last failure ("" if none). */
const char* fa_last_error(void);

/*
 * Build identity: 16 hex digits hashing every compiled source file, header and
 * compiler flag the library was built from (flash-attn-mps_b200/build.py,
 * source_hash), so a caller can check that a prebuilt library matches the
 * sources it ships with. No counterpart in the reference, which compiles its
 * Metal shaders from source at first use.
 */
const char* fa_build_id(void);

/*
 * Pipeline wait time-outs on the current device since the last clear:
 * bit 0 = the tensor-core prefill kernels, bit 1 = the TMA paged-decode
 * kernel, bit 2 = the sharded-decode exchange (fa_shard_wait).
 * Every mbarrier wait in those kernels gives up after a bounded number of
 * polls, sets its bit and lets the CTA finish, so a stalled pipeline shows
 * up here instead of hanging the GPU; outputs of the affected launch are then
 * undefined. clear != 0 resets the bits. Synchronous (reads device memory);
 * returns -1 on a CUDA error. No counterpart in the reference, whose Metal
 * kernels have no asynchronous pipelines.
 */
int fa_pipeline_timeouts(int clear);

/*
 * Kernel launches this library has issued in the process so far: a host-side
 * counter incremented at every launch site. A launch recorded into a CUDA
 * graph counts once, at capture, not per replay. A diagnostic for benchmarks
 * (how many of the library's kernels a timed region ran); no counterpart in
 * the reference.
 */
uint64_t fa_kernel_launches(void);

/*
 * Bytes of device workspace fa_attention_fwd needs for these arguments
 * (split-KV partial outputs and LSEs). Host-only; reads no tensor values.
 * Replaces the partial-buffer allocation of flash_attn_mps/_attention.py:162-167
 * and _decode.py:88-91.
 */
int fa_attention_workspace_size(const fa_attention_args* args, size_t* bytes);

/*
 * Attention forward: dispatch (decode / tcgen05 prefill / generic), split-KV
 * and the LSE merge, writing out and lse.
 * Replaces flash_attn_mps/_attention.py:88-238 (attention) together with
 * flash_attn_mps/_decode.py:40-99 (decode_attention) which it routes to.
 */
int fa_attention_fwd(const fa_attention_args* args, void* stream);

/*
 * Single-query split-KV decode that allocates nothing: same arguments and
 * results as fa_attention_fwd on its decode route (max_seqlen_q == 1, no
 * ALiBi, no mask, not deterministic), but the split partials live in a static
 * 32 MiB device array inside the library instead of args->workspace (which is
 * ignored). For callers that cannot allocate device memory: FFI hosts holding
 * only raw pointers from another allocator, processes whose device memory is
 * pre-reserved by a pool they do not control, and decode loops that must not
 * call cudaMalloc. With num_splits == 0 the library's split count is lowered
 * until the partials fit in 32 MiB; an explicit num_splits whose partials
 * exceed 32 MiB fails with FA_ERR_INVALID before any launch. All calls on a
 * device share the array: calls whose GPU work overlaps race. The first call
 * on a device resolves the array's address (cudaGetSymbolAddress) and caches
 * it with the current CUDA context (another context resolves it again); make
 * that first call before any stream capture.
 * This entry point has no counterpart in the reference.
 */
int fa_decode_fwd_noalloc(const fa_attention_args* args, void* stream);

/*
 * Scatter new K and V rows [T,Hkv,D] into paged caches [N,P,Hkv,D] at
 * slot_mapping (int32/int64 [T]; slot < 0 or >= N*P is skipped). An FP8 E4M3
 * cache stores the saturating round-to-nearest-even code of x/scale[h]
 * (scale f32 scalar or [Hkv], absent = 1); other caches must match x's dtype
 * and receive a bit-exact copy. Either K or V side may be absent (ptr NULL).
 * Replaces flash_attn_mps/_cache.py:67-85 (store_kvcache) and its kernel
 * kernels/cache.metal:20-39.
 */
int fa_store_kvcache(const fa_tensor* key, const fa_tensor* value,
                     const fa_tensor* k_cache, const fa_tensor* v_cache,
                     const fa_tensor* slot_mapping,
                     const fa_tensor* k_scale, const fa_tensor* v_scale,
                     void* stream);

/*
 * Append new K/V [B,Snew,Hkv,D] at positions lengths[b]+j of a continuous
 * cache [Bcache,capacity,Hkv,D] (row cache_batch_idx[b] when given) or of a
 * paged cache through block_table [B,pages]; out-of-range rows, positions and
 * pages are skipped; lengths are not modified.
 * Replaces flash_attn_mps/_cache.py:99-127 (append_kvcache), kernel
 * kernels/cache.metal:41-56.
 */
int fa_append_kvcache(const fa_tensor* key, const fa_tensor* value,
                      const fa_tensor* k_cache, const fa_tensor* v_cache,
                      const fa_tensor* lengths, const fa_tensor* cache_batch_idx,
                      const fa_tensor* block_table,
                      const fa_tensor* k_scale, const fa_tensor* v_scale,
                      void* stream);

/*
 * Rotary position embedding of x [B,S,H,D] into out (same shape and dtype):
 * position lengths[b] (+ j when advance), cos/sin f32 [positions, rot/2],
 * interleaved or split-half pairs, dims beyond rot copied.
 * Replaces flash_attn_mps/_cache.py:130-155 (rotary), kernel
 * kernels/cache.metal:58-76.
 */
int fa_rotary(const fa_tensor* x, const fa_tensor* out,
              const fa_tensor* cos, const fa_tensor* sin,
              const fa_tensor* lengths, int32_t interleaved, int32_t advance,
              void* stream);

/*
 * Fused RoPE + cache append (what flash_attn_with_kvcache does with rotary
 * tables and new K/V, in one launch): the new key [B,S,Hkv,Dk] rotated at
 * lengths[b] + j and rounded to its dtype, then appended like
 * fa_append_kvcache (E4M3-quantised with k_scale for an FP8 cache); value
 * appended unchanged; q [B,Sq,H,D] (optional) rotated at lengths[b] (+ j when
 * advance_q) into q_out. cos/sin: [positions, rotary_dim/2] of any float
 * dtype. Results equal fa_rotary followed by fa_append_kvcache bit for bit.
 * No single counterpart in the reference: it fuses flash_attn_mps/_cache.py:
 * 130-155 (rotary, kernels/cache.metal:58-76) with _cache.py:99-127 (append,
 * kernels/cache.metal:41-56) as called from interface.py:231-307.
 */
int fa_rotary_append_kvcache(const fa_tensor* q, const fa_tensor* q_out,
                             const fa_tensor* key, const fa_tensor* value,
                             const fa_tensor* k_cache, const fa_tensor* v_cache,
                             const fa_tensor* lengths, const fa_tensor* cache_batch_idx,
                             const fa_tensor* block_table,
                             const fa_tensor* k_scale, const fa_tensor* v_scale,
                             const fa_tensor* cos, const fa_tensor* sin,
                             int32_t interleaved, int32_t advance_q, void* stream);

/*
 * Stable pairwise merge of two attention states: out [T,H,D] and out_lse
 * [H,T] (optional) may alias the left state.
 * Replaces flash_attn_mps/_merge.py:20-41 (merge_attn_states), kernel
 * kernels/merge.metal:9-28.
 */
int fa_merge_attn_states(const fa_tensor* out, const fa_tensor* left, const fa_tensor* left_lse,
                         const fa_tensor* right, const fa_tensor* right_lse,
                         const fa_tensor* out_lse, void* stream);

/*
 * N-way merge of split partials [S,T,H,D] (any float dtype, any strides) and
 * LSEs [S,H,T] f32 into out [T,H,D] (f16/bf16/f32, any strides) and
 * out_lse [H,T] f32.
 * Replaces flash_attn_mps/_merge.py:44-57 (_merge_partials), kernels
 * kernels/merge.metal:30-58 and kernels/attention_decode.metal:151-207.
 */
int fa_merge_partials(const fa_tensor* partial, const fa_tensor* partial_lse,
                      const fa_tensor* out, const fa_tensor* out_lse, void* stream);

/*
 * KV-sharded decode across GPUs: the exchange of the ranks' partial states over
 * NVLink peer memory (one process per GPU). Each rank owns a gather buffer
 * mapped into every rank's address space (symmetric memory): two parities x
 * world slots of one float32 row [B*Hq*Dv | Hq*B] (a rank's partial output and
 * LSE), and a flag array of 2*FA_MAX_PEERS uint32 (zero before the first
 * step). slots[p] / flags[p] are this process's device addresses of rank p's
 * buffer and flag array. Step epochs start at 1 and grow by 1; step e uses
 * parity e & 1, and its merge reads this rank's own buffer:
 *   fa_shard_push: copy this rank's row (already in its own slot `rank` of
 *     parity e & 1) into slot `rank` of every peer's buffer, then raise
 *     flags[rank] = e on every peer;
 *   fa_shard_wait: wait until every peer's flag on this rank reached e (a
 *     bounded wait: on a timeout bit 2 of fa_pipeline_timeouts is set).
 * Both are asynchronous on the caller's stream; between them and the merge no
 * host synchronisation is needed. No counterpart in the reference, which has
 * no distributed code (flash_attn_mps/vllm.py:5): it replaces an NCCL
 * all-gather of the partials in front of the N-way merge
 * (flash_attn_mps/_merge.py:44-57, kernels/merge.metal:30-58).
 */
#define FA_MAX_PEERS 8

typedef struct fa_peer_buffers {
  void* slots[FA_MAX_PEERS];
  uint32_t* flags[FA_MAX_PEERS];
} fa_peer_buffers;

int fa_shard_push(const fa_tensor* row, const fa_peer_buffers* peers, int32_t world, int32_t rank,
                  uint32_t epoch, void* stream);

int fa_shard_wait(const fa_peer_buffers* peers, int32_t world, int32_t rank, uint32_t epoch, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FLASH_ATTN_B200_H */
