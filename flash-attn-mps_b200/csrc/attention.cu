// Attention dispatch (host side of the C ABI): argument checks, kernel choice,
// split-KV planning and the partial merge.
//
// Routing follows the reference dispatcher (flash_attn_mps/_attention.py:88-238):
//   * one query per request, not deterministic, no ALiBi, no mask
//     -> decode (_attention.py:134-147 -> _decode.py:40-99): the tensor-core
//        decode kernel when its envelope fits, else the generic kernel;
//   * eligible dense/varlen prefill -> the tcgen05 kernel (the reference's
//     "fast" predicate, _attention.py:149-158);
//   * everything else -> the generic kernel with the reference's split rule
//     (_attention.py:159-161).
// The choice depends on shapes, dtypes, strides and flags only, never on
// tensor values or lengths beyond the caller's max_seqlen_*.
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>

#include "kernels.cuh"

namespace fab {

std::string& last_error() {
  thread_local std::string message;
  return message;
}

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  last_error() = buf;
  return code;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

namespace {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}
}  // namespace

bool tensor_map_available() { return encode_fn() != nullptr; }

int encode_tensor_map(void* map, int dtype, int rank, const void* ptr, const uint64_t* dims,
                      const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128) {
  auto fn = encode_fn();
  if (!fn) return fail(FA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  CUtensorMapDataType t = dtype == FA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                          : dtype == FA_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                            : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  cuuint64_t d[5];
  cuuint64_t st[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) st[i] = strides_bytes[i];
  }
  CUresult r = fn(reinterpret_cast<CUtensorMap*>(map), t, (cuuint32_t)rank, const_cast<void*>(ptr), d, st, bx, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return FA_OK;
}

namespace {

enum Route { kRouteGeneric = 0, kRouteDecode = 1, kRoutePrefill = 2, kRouteMma = 3, kRouteFp8Prefill = 4 };

// Workspace of the FP8 prefill route: work counter, 16-bit K and V copies,
// then (paged K/V) row starts [B+1] and lengths [B].
struct Fp8Layout {
  size_t kv_off, kv_bytes, cu_off, used_off, total;
};
Fp8Layout fp8_layout(const AttnParams& p) {
  auto up = [](size_t x) { return (x + 255) / 256 * 256; };
  Fp8Layout l{};
  l.kv_off = 256;
  l.kv_bytes = up((size_t)fp8_prefill_rows(p) * p.HK * p.DQ * 2);
  l.cu_off = l.kv_off + 2 * l.kv_bytes;
  l.used_off = l.cu_off + up((size_t)(p.B + 1) * 4);
  l.total = l.used_off + up((size_t)p.B * 4);
  return l;
}

struct Plan {
  int route;
  int splits;
  int span;          // decode only
  size_t part_bytes, lse_bytes;
};

int validate(const fa_attention_args* a) {
  FAB_CHECK_ARG(a != nullptr, "null arguments");
  const fa_tensor &q = a->q, &k = a->k, &v = a->v;
  FAB_CHECK_ARG(present(q) && present(k) && present(v) || q.shape[0] == 0,
                "q, k and v are required");
  FAB_CHECK_ARG(q.ndim == 3 && (k.ndim == 3 || k.ndim == 4) && v.ndim == k.ndim,
                "q must be packed 3-D; k/v must be packed 3-D or paged 4-D");
  for (const fa_tensor* t : {&q, &k, &v})
    FAB_CHECK_ARG(t->dtype == FA_F16 || t->dtype == FA_BF16 || t->dtype == FA_F32 || t->dtype == FA_E4M3,
                  "attention supports FP16, BF16, FP32 and FP8 E4M3FN");
  const int64_t dq = q.shape[2], dv = v.shape[v.ndim - 1];
  FAB_CHECK_ARG(dq >= 1 && dq <= 512 && dv >= 1 && dv <= 512,
                "query/key and value head dimensions must be in 1..512");
  for (int i = 0; i < k.ndim - 1; ++i)
    FAB_CHECK_ARG(k.shape[i] == v.shape[i], "key/value shapes must agree except for their last dimension");
  FAB_CHECK_ARG(k.shape[k.ndim - 1] == dq, "key/value shapes must agree except for their last dimension");
  const int64_t heads = q.shape[1], kh = k.shape[k.ndim - 2];
  FAB_CHECK_ARG(heads >= 1 && kh >= 1 && heads % kh == 0, "query heads must be a positive multiple of KV heads");
  FAB_CHECK_ARG((k.ndim == 4) == present(a->block_table),
                "paged 4-D KV requires block_table; packed 3-D KV does not");
  FAB_CHECK_ARG(present(a->cu_seqlens_k) || present(a->seqused_k), "cu_seqlens_k or seqused_k is required");
  FAB_CHECK_ARG(a->num_splits >= 0, "num_splits must be nonnegative");
  if (a->cp_world_size > 1) {
    FAB_CHECK_ARG(a->cp_rank >= 0 && a->cp_rank < a->cp_world_size, "cp_rank must be in [0, cp_world_size)");
    FAB_CHECK_ARG(present(a->cp_tot_seqused_k) && a->cp_tot_seqused_k.dtype == FA_I32 &&
                      a->cp_tot_seqused_k.ndim == 1 && a->cp_tot_seqused_k.shape[0] == a->batch,
                  "context parallelism needs cp_tot_seqused_k int32 [B]");
  }
  FAB_CHECK_ARG(present(a->out) && a->out.ndim == 3 && a->out.shape[0] == q.shape[0] &&
                    a->out.shape[1] == heads && a->out.shape[2] == dv,
                "out must have shape [total_q, query_heads, value_dim]");
  FAB_CHECK_ARG(is_float(a->out.dtype), "out must have FP16, BF16 or FP32 dtype");
  FAB_CHECK_ARG(present(a->lse) && a->lse.ndim == 2 && a->lse.dtype == FA_F32 &&
                    a->lse.shape[0] == heads && a->lse.shape[1] == q.shape[0],
                "lse must be float32 [heads, total_q]");
  if (q.shape[0] == 0) return FA_OK;
  FAB_CHECK_ARG(a->max_seqlen_q > 0 && a->max_seqlen_k >= 0,
                "nonempty q requires positive max_seqlen_q and nonnegative max_seqlen_k");
  FAB_CHECK_ARG(a->batch >= 1 && present(a->cu_seqlens_q) && a->cu_seqlens_q.dtype == FA_I32 &&
                    a->cu_seqlens_q.shape[0] == a->batch + 1,
                "cu_seqlens_q must contain at least two offsets");
  if (present(a->block_table))
    FAB_CHECK_ARG(a->block_table.dtype == FA_I32 && a->block_table.ndim == 2, "block_table must be int32 [B,P]");
  FAB_CHECK_ARG(a->mask_kind >= 0 && a->mask_kind <= 2, "unknown mask kind");
  if (a->mask_kind == 1)
    FAB_CHECK_ARG(present(a->mask_aux0) && a->mask_aux0.ndim == 2, "mask kind 1 needs query ranges [T,2]");
  if (a->mask_kind == 2)
    FAB_CHECK_ARG(present(a->mask_aux0) && present(a->mask_aux1), "mask kind 2 needs prefix and window");
  return FA_OK;
}

void fill_params(const fa_attention_args* a, AttnParams* p) {
  *p = AttnParams{};
  const fa_tensor &q = a->q, &k = a->k, &v = a->v;
  p->q = q.ptr; p->k = k.ptr; p->v = v.ptr;
  p->qt = q.dtype; p->kt = k.dtype; p->vt = v.dtype;
  p->qs0 = q.stride[0]; p->qs1 = q.stride[1]; p->qs2 = q.stride[2];
  if (k.ndim == 4) {
    p->ks0 = k.stride[0]; p->ks1 = k.stride[1]; p->ks2 = k.stride[2]; p->ks3 = k.stride[3];
    p->vs0 = v.stride[0]; p->vs1 = v.stride[1]; p->vs2 = v.stride[2]; p->vs3 = v.stride[3];
    p->page = (int32_t)k.shape[1];
    p->k_pages = k.shape[0];
    p->paged = 1;
  } else {
    p->ks1 = k.stride[0]; p->ks2 = k.stride[1]; p->ks3 = k.stride[2];
    p->k_rows = k.shape[0];
    p->vs1 = v.stride[0]; p->vs2 = v.stride[1]; p->vs3 = v.stride[2];
  }
  p->out = a->out.ptr; p->ot = a->out.dtype;
  p->os0 = a->out.stride[0]; p->os1 = a->out.stride[1]; p->os2 = a->out.stride[2];
  p->lse = reinterpret_cast<float*>(a->lse.ptr);
  p->ls0 = a->lse.stride[0]; p->ls1 = a->lse.stride[1];
  p->cu_q = reinterpret_cast<const int32_t*>(a->cu_seqlens_q.ptr); p->cq0 = a->cu_seqlens_q.stride[0];
  if (present(a->cu_seqlens_k)) { p->cu_k = reinterpret_cast<const int32_t*>(a->cu_seqlens_k.ptr); p->ck0 = a->cu_seqlens_k.stride[0]; }
  if (present(a->seqused_k)) { p->used = reinterpret_cast<const int32_t*>(a->seqused_k.ptr); p->u0 = a->seqused_k.stride[0]; }
  if (present(a->block_table)) {
    p->table = reinterpret_cast<const int32_t*>(a->block_table.ptr);
    p->bt0 = a->block_table.stride[0]; p->bt1 = a->block_table.stride[1];
    p->bt_cols = a->block_table.shape[1];
  }
  if (present(a->leftpad_k)) { p->leftpad = reinterpret_cast<const int32_t*>(a->leftpad_k.ptr); p->lp0 = a->leftpad_k.stride[0]; }
  if (present(a->causal_per_seq)) {
    p->causal_b = reinterpret_cast<const uint8_t*>(a->causal_per_seq.ptr);
    p->ca0 = a->causal_per_seq.stride[0];
    p->dynamic = 1;
  }
  if (present(a->alibi_slopes)) {
    p->alibi = reinterpret_cast<const float*>(a->alibi_slopes.ptr);
    if (a->alibi_slopes.ndim == 1) { p->a0 = 0; p->a1 = a->alibi_slopes.stride[0]; }
    else { p->a0 = a->alibi_slopes.stride[0]; p->a1 = a->alibi_slopes.stride[1]; }
  }
  if (present(a->s_aux)) { p->sinks = a->s_aux.ptr; p->sink_t = a->s_aux.dtype; p->si0 = a->s_aux.stride[0]; }
  auto descale = [](const fa_tensor& t, const float** ptr, int64_t* s0, int64_t* s1) {
    if (!present(t)) return;
    *ptr = reinterpret_cast<const float*>(t.ptr);
    *s0 = t.ndim == 2 ? t.stride[0] : 0;
    *s1 = t.ndim == 2 ? t.stride[1] : (t.ndim == 1 ? t.stride[0] : 0);
  };
  descale(a->q_descale, &p->qd, &p->qd0, &p->qd1);
  descale(a->k_descale, &p->kd, &p->kd0, &p->kd1);
  descale(a->v_descale, &p->vd, &p->vd0, &p->vd1);
  p->mask = a->mask_kind; p->mask_win = a->mask_window; p->clamp = a->mask_clamp;
  if (a->cp_world_size > 1) {
    p->cp_n = a->cp_world_size; p->cp_r = a->cp_rank;
    p->cp_tot = reinterpret_cast<const int32_t*>(a->cp_tot_seqused_k.ptr);
    p->ct0 = a->cp_tot_seqused_k.stride[0];
  }
  if (a->mask_kind == 1) {
    p->mr = reinterpret_cast<const int32_t*>(a->mask_aux0.ptr);
    p->mr0 = a->mask_aux0.stride[0]; p->mr1 = a->mask_aux0.stride[1];
  } else if (a->mask_kind == 2) {
    p->mp = reinterpret_cast<const int32_t*>(a->mask_aux0.ptr); p->mp0 = a->mask_aux0.stride[0];
    p->mw = reinterpret_cast<const int32_t*>(a->mask_aux1.ptr);
  }
  p->T = (int32_t)q.shape[0];
  p->B = a->batch;
  p->HQ = (int32_t)q.shape[1];
  p->HK = (int32_t)k.shape[k.ndim - 2];
  p->DQ = (int32_t)q.shape[2];
  p->DV = (int32_t)v.shape[v.ndim - 1];
  p->causal = a->causal;
  p->win_l = a->window_left; p->win_r = a->window_right;
  p->max_q = a->max_seqlen_q; p->max_k = a->max_seqlen_k;
  p->scale = a->softmax_scale; p->softcap = a->softcap;
  p->splits = 1;
}

// Bytes of split partials (outputs, then LSEs) for `splits` splits.
size_t split_part_bytes(const AttnParams& p, int splits) {
  return ((size_t)splits * p.T * p.HQ * p.DV * sizeof(float) + 255) / 256 * 256;
}
size_t split_lse_bytes(const AttnParams& p, int splits) {
  return ((size_t)splits * p.HQ * p.T * sizeof(float) + 255) / 256 * 256;
}

// part_cap > 0: when the library chooses a decode split count
// (num_splits == 0), lower it until the split partials fit in part_cap bytes
// (down to one split, which writes the outputs directly and needs none).
int make_plan(const fa_attention_args* a, const AttnParams& p, Plan* plan, size_t part_cap = 0) {
  *plan = Plan{kRouteGeneric, 1, 0, 0, 0};
  // Batch-invariant mode (deterministic, or num_splits == 1 as vLLM's
  // batch-invariant path passes it): the kernel choice depends on dtypes and
  // features only, never on the batch's max_seqlen_q, and every row reduces
  // its keys in one fixed order. The tensor-core prefill qualifies (a row's
  // key tiles depend only on its own request); otherwise the mma.sync or the
  // generic kernel with one split.
  const bool invariant = a->deterministic || a->num_splits == 1;
  if (invariant && prefill_sm100_supported(p)) {
    plan->route = kRoutePrefill;
    plan->part_bytes = 256;  // persistent-scheduler work counter
    return FA_OK;
  }
  const bool decode = a->max_seqlen_q == 1 && !present(a->alibi_slopes) && a->mask_kind == 0;
  if (invariant) {
    plan->splits = 1;  // generic or mma.sync kernel, one split
  } else if (decode) {
    const int eff = a->window_left >= 0 ? std::min(a->max_seqlen_k, a->window_left + 1) : a->max_seqlen_k;
    if (decode_mma_supported(p)) {
      plan->route = kRouteDecode;
      if (a->num_splits > 0) {
        plan->splits = a->num_splits;
        plan->span = std::max(1, (eff + a->num_splits - 1) / a->num_splits);
      } else {
        plan->splits = decode_default_splits(p, &plan->span);
      }
    } else {
      // _decode.py:63-64
      plan->splits = a->num_splits > 0 ? a->num_splits : std::max(1, std::min(32, (eff + 255) / 256));
    }
    if (part_cap > 0 && a->num_splits == 0) {
      while (plan->splits > 1 &&
             split_part_bytes(p, plan->splits) + split_lse_bytes(p, plan->splits) > part_cap)
        --plan->splits;
      if (plan->route == kRouteDecode) plan->span = std::max(1, (eff + plan->splits - 1) / plan->splits);
    }
  } else {
    AttnParams view;
    // (Single-query ALiBi calls keep the split-KV route of the kernels below.)
    if (a->num_splits == 0 && prefill_sm100_supported(p) && !(p.alibi && a->max_seqlen_q == 1)) {
      plan->route = kRoutePrefill;
      plan->splits = 1;
      plan->part_bytes = 256;  // persistent-scheduler work counter
      return FA_OK;
    } else if (a->num_splits == 0 && a->max_seqlen_q >= 128 && fp8_prefill_view(p, &view)) {
      // FP8 K/V with at least one full 128-row query tile: an exact 16-bit
      // copy of the K/V rows (3 bytes per element of extra traffic) turns the
      // call into the tcgen05 prefill's compute-bound work; shorter query
      // chunks stay on the mma.sync kernel, which reads the FP8 bytes directly.
      plan->route = kRouteFp8Prefill;
      plan->splits = 1;
      plan->part_bytes = fp8_layout(p).total;
      return FA_OK;
    } else {
      const bool vector = a->max_seqlen_q == 1 || std::max(p.DQ, p.DV) > 256;
      plan->splits = a->num_splits > 0 ? a->num_splits
                     : vector ? std::min(32, std::max(1, (a->max_seqlen_k + 255) / 256)) : 1;
    }
  }
  // f16/bf16 cases left to the generic kernel run on the mma.sync tensor-core
  // kernel when its head dims and strides fit (same splits, same semantics).
  if (plan->route == kRouteGeneric) {
    AttnParams q = p;
    q.splits = plan->splits;
    if (mma_attention_supported(q)) plan->route = kRouteMma;
  }
  if (plan->splits > 1) {
    plan->part_bytes = split_part_bytes(p, plan->splits);
    plan->lse_bytes = split_lse_bytes(p, plan->splits);
  }
  return FA_OK;
}

}  // namespace
}  // namespace fab

using namespace fab;

extern "C" int fa_abi_version(void) { return FA_B200_ABI_VERSION; }

extern "C" const char* fa_last_error(void) { return last_error().c_str(); }

namespace fab {
static std::atomic<unsigned long long> g_kernel_launches{0};
void note_launch() { g_kernel_launches.fetch_add(1, std::memory_order_relaxed); }
}  // namespace fab

extern "C" uint64_t fa_kernel_launches(void) { return fab::g_kernel_launches.load(std::memory_order_relaxed); }

extern "C" int fa_pipeline_timeouts(int clear) {
  const int a = fab::prefill_timeout_flag(clear != 0);
  const int b = fab::decode_timeout_flag(clear != 0);
  const int c = fab::exchange_timeout_flag(clear != 0);
  if (a < 0 || b < 0 || c < 0) return -1;
  return (a ? 1 : 0) | (b ? 2 : 0) | (c ? 4 : 0);
}

namespace fab {

int attention_workspace_capped(const fa_attention_args* a, size_t* bytes, size_t part_cap) {
  FAB_CHECK_ARG(bytes != nullptr, "bytes must not be null");
  *bytes = 0;
  int rc = validate(a);
  if (rc) return rc;
  if (a->q.shape[0] == 0) return FA_OK;
  AttnParams p;
  fill_params(a, &p);
  Plan plan;
  rc = make_plan(a, p, &plan, part_cap);
  if (rc) return rc;
  *bytes = plan.part_bytes + plan.lse_bytes;
  return FA_OK;
}

int attention_fwd_capped(const fa_attention_args* a, void* stream, size_t part_cap) {
  int rc = validate(a);
  if (rc) return rc;
  if (a->q.shape[0] == 0) return FA_OK;
  AttnParams p;
  fill_params(a, &p);
  Plan plan;
  rc = make_plan(a, p, &plan, part_cap);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (plan.route == kRoutePrefill || plan.route == kRouteFp8Prefill) {
    FAB_CHECK_ARG(present(a->workspace) && a->workspace.ndim >= 1 &&
                      (size_t)a->workspace.shape[0] * elem_size(a->workspace.dtype) >= plan.part_bytes,
                  "workspace smaller than fa_attention_workspace_size");
    FAB_CHECK_ARG(((uintptr_t)a->workspace.ptr & 255u) == 0 || plan.route == kRoutePrefill,
                  "workspace must be 256-byte aligned");
    p.scratch = a->workspace.ptr;
  }
  if (plan.route == kRouteFp8Prefill) {
    AttnParams view;
    if (!fp8_prefill_view(p, &view)) return fail(FA_ERR_INVALID, "FP8 prefill plan no longer applies");
    const Fp8Layout l = fp8_layout(p);
    uint8_t* ws = reinterpret_cast<uint8_t*>(a->workspace.ptr);
    int32_t* cu_out = p.paged ? reinterpret_cast<int32_t*>(ws + l.cu_off) : nullptr;
    int32_t* used_out = p.paged ? reinterpret_cast<int32_t*>(ws + l.used_off) : nullptr;
    rc = launch_kv_dequant(p, ws + l.kv_off, ws + l.kv_off + l.kv_bytes, cu_out, used_out, st);
    if (rc) return rc;
    view.k = ws + l.kv_off;
    view.v = ws + l.kv_off + l.kv_bytes;
    if (p.paged) {
      view.cu_k = cu_out; view.ck0 = 1;
      view.used = used_out; view.u0 = 1;
    }
    view.scratch = ws;
    view.splits = 1;
    return launch_prefill_sm100(view, st);
  }
  if (plan.splits > 1) {
    FAB_CHECK_ARG(present(a->workspace) && a->workspace.ndim >= 1 &&
                      (size_t)a->workspace.shape[0] * elem_size(a->workspace.dtype) >= plan.part_bytes + plan.lse_bytes,
                  "workspace smaller than fa_attention_workspace_size");
    uint8_t* ws = reinterpret_cast<uint8_t*>(a->workspace.ptr);
    FAB_CHECK_ARG(((uintptr_t)ws & 15u) == 0, "workspace must be 16-byte aligned");
    p.part = reinterpret_cast<float*>(ws);
    p.part_lse = reinterpret_cast<float*>(ws + plan.part_bytes);
  }
  p.splits = plan.splits;
  switch (plan.route) {
    case kRouteDecode: rc = launch_decode_mma(p, plan.splits, plan.span, st); break;
    case kRoutePrefill: rc = launch_prefill_sm100(p, st); break;
    case kRouteMma: rc = launch_mma_attention(p, st); break;
    default: rc = launch_generic_attention(p, st); break;
  }
  if (rc) return rc;
  if (plan.splits > 1) {
    MergePartialsArgs m{};
    m.partial = p.part; m.pdtype = FA_F32;
    m.ps0 = (int64_t)p.T * p.HQ * p.DV; m.ps1 = (int64_t)p.HQ * p.DV; m.ps2 = p.DV; m.ps3 = 1;
    m.lse = p.part_lse; m.ls0 = (int64_t)p.HQ * p.T; m.ls1 = p.T; m.ls2 = 1;
    m.out = a->out.ptr; m.odtype = a->out.dtype;
    m.os0 = a->out.stride[0]; m.os1 = a->out.stride[1]; m.os2 = a->out.stride[2];
    m.out_lse = reinterpret_cast<float*>(a->lse.ptr);
    m.ols0 = a->lse.stride[0]; m.ols1 = a->lse.stride[1];
    m.S = plan.splits; m.T = p.T; m.H = p.HQ; m.D = p.DV;
    rc = launch_merge_partials(m, st);
  }
  return rc;
}

}  // namespace fab

extern "C" int fa_attention_workspace_size(const fa_attention_args* a, size_t* bytes) {
  return fab::attention_workspace_capped(a, bytes, 0);
}

extern "C" int fa_attention_fwd(const fa_attention_args* a, void* stream) {
  return fab::attention_fwd_capped(a, stream, 0);
}
