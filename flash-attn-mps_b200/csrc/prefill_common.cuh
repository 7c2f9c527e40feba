// Shared pieces of the tcgen05 prefill kernels (prefill_sm100.cu: head dims up
// to 128, two query tiles per CTA; prefill_wide_sm100.cu: QK head dims 192/256,
// one query tile per CTA): kernel parameters, the work-item record, mask
// geometry, packed f32x2 arithmetic, the FMA-pipe exp2 and the tensor-map
// helpers.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "kernels.cuh"
#include "sm100.cuh"

namespace fab {
namespace pf {

using namespace sm100;

constexpr int BM = 128;                 // query rows per tile
constexpr int BN = 128;                 // keys per tile
constexpr int kRegion = 128 * 128;      // one 128-row x 64-element 16-bit box (bytes)
constexpr int kKVRegion = BN * 128;     // one BN-row x 64-element K/V box
constexpr int NWORK = 4;                // work-id ring slots
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: P stays <= 2^8 between rescales

struct PrefillParams {
  void* out; int64_t os0, os1;
  float* lse; int64_t ls0, ls1;
  const int32_t* cu_q; int64_t cq0;
  const int32_t* cu_k; int64_t ck0;
  const int32_t* used; int64_t u0;
  const uint8_t* causal_b; int64_t ca0;     // dynamic per-request causal flags
  const void* sinks; int32_t sink_t; int64_t si0;
  const float* qd; int64_t qd0, qd1;
  const float* kd; int64_t kd0, kd1;
  const float* vd; int64_t vd0, vd1;
  int* counter;                           // work counter, zero at launch
  const int32_t* table; int64_t bt0, bt1;  // paged K/V: block_table [B, bt_cols] (null for packed K/V)
  int32_t bt_cols, page_shift, box_rows;   // page = 1 << page_shift tokens, box_rows = min(page, 128)
  const float* alibi; int64_t al0, al1;    // ALiBi slopes [B,H] or [H] (ALIBI instantiation only)
  int32_t dim;                             // true head dim (<= HDIM; columns past it are TMA zero fill)
  int32_t head_pairs;                      // 1: tiles A/B = query heads h, h+1 of one row block; 0: row blocks r, r+1
  int32_t group_reqs;                      // requests per work-order group (their K/V share L2; B: one group)
  int32_t B, HQ, HK, n_pairs, causal, win_l, win_r;
  float scale, softcap;
};


// A bounded mbarrier wait taken by a whole warp (true only if every lane's
// wait succeeded); a timeout sets *flag.
__device__ __forceinline__ bool warp_wait_flag(uint32_t bar, uint32_t parity, int* flag) {
  bool ok = mbar_wait(bar, parity, flag);
  return __all_sync(0xffffffffu, ok);
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack_p(float a, float b) {
  if constexpr (BF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}
// ---- packed f32x2 arithmetic (sm_100 FFMA2 / FADD2) and an FMA-pipe exp2
__device__ __forceinline__ uint64_t f2pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max_nan(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ uint64_t fsub2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// 2^x for a pair, on the FMA pipe: x = n + f with n = rint(x) (round-to-
// nearest through the 1.5 * 2^23 shifter), 2^f by a minimax polynomial on
// [-1/2, 1/2] (Remez fit with the constant term pinned to 1, relative error
// 4.3e-4 at degree 3 -- below half a bf16 ulp -- and 5.4e-6 at degree 4 for
// f16 P; flash-attn-mps_b200/csrc/fit_exp2_poly.py), and 2^n added to the
// exponent field. x is clamped to >= -127 first (NaN kept), which makes
// 2^(-inf) exactly +0: n = -127, f = 0, p = 1.0 = 127 << 23. The constant
// pairs live in registers for the whole tile.
template <bool DEG3>
struct Exp2Poly {
  uint64_t magic, c1, c2, c3, c4, one;
  __device__ __forceinline__ Exp2Poly() {
    magic = f2pack(12582912.f, 12582912.f);
    one = f2pack(1.f, 1.f);
    if constexpr (DEG3) {
      c1 = f2pack(6.957671046e-01f, 6.957671046e-01f);
      c2 = f2pack(2.420305014e-01f, 2.420305014e-01f);
      c3 = f2pack(4.169750959e-02f, 4.169750959e-02f);
      c4 = 0;
    } else {
      c1 = f2pack(6.931053400e-01f, 6.931053400e-01f);
      c2 = f2pack(2.402216792e-01f, 2.402216792e-01f);
      c3 = f2pack(5.600578710e-02f, 5.600578710e-02f);
      c4 = f2pack(9.676037356e-03f, 9.676037356e-03f);
    }
  }
  __device__ __forceinline__ void operator()(uint64_t x2, float& p0, float& p1) const {
    float x0, x1;
    f2unpack(x2, x0, x1);
    in_range(f2pack(max_nan(x0, -127.f), max_nan(x1, -127.f)), p0, p1);
  }
  // x already within [-126, 126].
  __device__ __forceinline__ void in_range(uint64_t x2, float& p0, float& p1) const {
    const uint64_t t = fadd2(x2, magic);
    const uint64_t f = fsub2(x2, fsub2(t, magic));
    uint64_t q;
    if constexpr (DEG3) {
      q = ffma2(c3, f, c2);
    } else {
      q = ffma2(c4, f, c3);
      q = ffma2(q, f, c2);
    }
    q = ffma2(q, f, c1);
    q = ffma2(q, f, one);
    float q0, q1, t0, t1;
    f2unpack(q, q0, q1);
    f2unpack(t, t0, t1);
    p0 = __int_as_float(__float_as_int(q0) + (__float_as_int(t0) << 23));
    p1 = __int_as_float(__float_as_int(q1) + (__float_as_int(t1) << 23));
  }
};

// tanh from the identity tanh(y) = 1 - 2 / (e^(2y) + 1): one ex2, one rcp, one
// FFMA. Absolute error ~1e-6 over the whole range (saturates cleanly to +-1),
// which a softcap multiplies by the cap.
__device__ __forceinline__ float tanh_id(float y) {
  return fmaf(-2.f, rcp(1.f + ex2(y * 2.8853900817779268f)), 1.f);
}

// Softcap on the FMA pipe for bounded arguments: tanh(y) = y * Q(y^2) on
// |y| <= 3/4, Q a degree-4 minimax polynomial in y^2 with Q(0) = 1 (Remez fit,
// relative error 6.5e-7; float32 Horner 7.4e-7 relative, 4.6e-7 absolute --
// below the identity route's ~1.5e-6; flash-attn-mps_b200/csrc/fit_tanh_poly.py).
// With y = s * c (c = scale / cap) and cap * log2e * c = scale * log2e = sl2,
//   cap * log2e * tanh(s * c) = s * sl2 * Q(y^2):
// the score scale folds into Q's coefficients (y itself is formed first, so
// no coefficient depends on the cap and none can under- or overflow for an
// extreme cap). Two packed multiplies, four packed FMAs and the caller's
// final FMA per pair of scores, no MUFU operation.
constexpr float kSoftcapPolyY = 0.75f;
struct TanhPoly {
  uint64_t c2, k0, k1, k2, k3, k4;
  __device__ __forceinline__ TanhPoly(float sl2, float c) {
    c2 = f2pack(c, c);
    k0 = f2pack(sl2, sl2);
    const float a1 = sl2 * -3.332966864e-01f, a2 = sl2 * 1.326823682e-01f;
    const float a3 = sl2 * -5.027795583e-02f, a4 = sl2 * 1.310583670e-02f;
    k1 = f2pack(a1, a1);
    k2 = f2pack(a2, a2);
    k3 = f2pack(a3, a3);
    k4 = f2pack(a4, a4);
  }
  // cap * log2e * tanh(s * c) + add, for a pair of scores s.
  __device__ __forceinline__ uint64_t fma(uint64_t s2, uint64_t add2) const {
    const uint64_t y = fmul2(s2, c2);
    const uint64_t v = fmul2(y, y);
    uint64_t q = ffma2(k4, v, k3);
    q = ffma2(q, v, k2);
    q = ffma2(q, v, k1);
    q = ffma2(q, v, k0);
    return ffma2(s2, q, add2);
  }
};

// Largest |s| for which TanhPoly applies (|s * c| <= 3/4), for a positive
// finite c = scale / cap only (else -1: never). With c > 0 (and so every
// k_i's sign that of Q's coefficient) a masked score s = -inf gives y = -inf,
// v = +inf, Q = +inf (leading coefficient > 0) and s * sl2 * Q = -inf exactly,
// so 2^(logit - m) is exactly 0 without a select.
__device__ __forceinline__ float softcap_poly_limit(float c) {
  return (c > 0.f && c < INFINITY) ? kSoftcapPolyY / c : -1.f;
}

// Largest |s| of a score row, as 8 independent 3-input max chains (a NaN
// score, which only non-finite inputs produce, is ignored; an infinite one
// makes the bound infinite).
template <int N>
__device__ __forceinline__ float row_absmax(const uint32_t (&r)[N]) {
  float am8[8];
#pragma unroll
  for (int k8 = 0; k8 < 8; ++k8) am8[k8] = 0.f;
#pragma unroll
  for (int i = 0; i < N; i += 2)
    am8[(i >> 1) & 7] = max3(am8[(i >> 1) & 7], fabsf(__uint_as_float(r[i])), fabsf(__uint_as_float(r[i + 1])));
  return fmaxf(fmaxf(fmaxf(am8[0], am8[1]), fmaxf(am8[2], am8[3])),
               fmaxf(fmaxf(am8[4], am8[5]), fmaxf(am8[6], am8[7])));
}

// Visible key range [lo, hi] of the query at absolute position q_abs
// (lower-right causal, local window), clipped to [0, k_len).
struct KeyRange { int lo, hi; };
__device__ __forceinline__ KeyRange key_range(int q_abs, int k_len, bool causal, int win_l, int win_r) {
  int lo = win_l >= 0 ? max(0, q_abs - win_l) : 0;
  int hi = k_len - 1;
  if (causal) hi = min(hi, q_abs);
  if (win_r >= 0) hi = min(hi, q_abs + win_r);
  return {lo, hi};
}

// KV tiles [first, last) that a 128-row query tile starting at row0 touches.
__device__ __forceinline__ void tile_range(int row0, int q_len, int k_len, bool causal, int win_l, int win_r,
                                           int* first, int* last) {
  *first = *last = 0;
  if (row0 >= q_len || k_len <= 0) return;
  const int off = k_len - q_len;
  const KeyRange a = key_range(row0 + off, k_len, causal, win_l, win_r);
  const KeyRange z = key_range(min(row0 + BM, q_len) - 1 + off, k_len, causal, win_l, win_r);
  if (z.hi < a.lo || z.hi < 0) return;
  *first = a.lo / BN;
  *last = z.hi / BN + 1;
}

// One work item: two 128-row query tiles (A, B) of one request. When the
// query heads per KV head are even, A and B are the same row block of query
// heads h and h+1, which share their KV head: both see exactly the same key
// tiles (the same K/V loads, the same causal extent), so neither tile idles
// while the other finishes a diagonal or a short sequence. Otherwise A and B
// are row blocks r and r+1 of one head. Items are ordered by row-block index
// descending (the costliest causal tiles first), then head, then request.
// The TMA warp decodes each claimed item once (including its global reads:
// sequence offsets, lengths, causal flag, descales, sink) and publishes it in
// shared memory, so the MMA and softmax warps start an item without any
// global-memory round trip.
struct Item {
  int valid, b, h, kh, q_begin, q_len, k_begin, k_len, row_a, row_b, causal;
  int a0, a1, b0, b1, j_first, n_all;
  float qk_scale, vscale;
  int h_b;  // query head of tile B
};
constexpr int kItemWords = sizeof(Item) / 4;
static_assert(sizeof(Item) == 20 * 4, "Item is 20 words");

// Field-wise copies through the shared item ring (no address of a local Item
// is taken, so the item stays in registers).
__device__ __forceinline__ void item_store(volatile int* d, const Item& it) {
  d[0] = it.valid; d[1] = it.b; d[2] = it.h; d[3] = it.kh; d[4] = it.q_begin; d[5] = it.q_len;
  d[6] = it.k_begin; d[7] = it.k_len; d[8] = it.row_a; d[9] = it.row_b; d[10] = it.causal;
  d[11] = it.a0; d[12] = it.a1; d[13] = it.b0; d[14] = it.b1; d[15] = it.j_first; d[16] = it.n_all;
  d[17] = __float_as_int(it.qk_scale); d[18] = __float_as_int(it.vscale); d[19] = it.h_b;
}
// Five 16-byte shared loads (issued together) after the slot's full barrier.
__device__ __forceinline__ void item_load(const volatile int* d, Item& it) {
  int4 w[5];
#pragma unroll
  for (int i = 0; i < 5; ++i) {
    asm volatile("ld.shared.v4.s32 {%0, %1, %2, %3}, [%4];\n"
                 : "=r"(w[i].x), "=r"(w[i].y), "=r"(w[i].z), "=r"(w[i].w)
                 : "r"(smem_addr(const_cast<const int*>(d) + 4 * i))
                 : "memory");
  }
  it.valid = w[0].x; it.b = w[0].y; it.h = w[0].z; it.kh = w[0].w;
  it.q_begin = w[1].x; it.q_len = w[1].y; it.k_begin = w[1].z; it.k_len = w[1].w;
  it.row_a = w[2].x; it.row_b = w[2].y; it.causal = w[2].z; it.a0 = w[2].w;
  it.a1 = w[3].x; it.b0 = w[3].y; it.b1 = w[3].z; it.j_first = w[3].w;
  it.n_all = w[4].x; it.qk_scale = __int_as_float(w[4].y); it.vscale = __int_as_float(w[4].z);
  it.h_b = w[4].w;
}

// ------------------------------------------------------------- host helpers
// Paged [pages, page, heads, 128] cache -> 4-D map (dims, heads, token in page,
// page), box {64, 1, box_rows, 1}.
inline int make_page_map(CUtensorMap* map, const void* ptr, int dtype, int64_t dim, int64_t heads, int64_t page,
                  int64_t pages, int64_t s_page, int64_t s_tok, int64_t s_head, int box_rows) {
  const uint64_t dims[4] = {(uint64_t)dim, (uint64_t)heads, (uint64_t)page, (uint64_t)pages};
  const uint64_t strides[3] = {(uint64_t)(s_head * 2), (uint64_t)(s_tok * 2), (uint64_t)(s_page * 2)};
  const uint32_t box[4] = {64, 1, (uint32_t)box_rows, 1};
  return encode_tensor_map(map, dtype, 4, ptr, dims, strides, box, true);
}
// [rows, heads, 128] tensor with unit inner stride -> 3-D map, box {64, 1, 128}.
inline int make_map(CUtensorMap* map, const void* ptr, int dtype, int64_t dim, int64_t rows, int64_t heads,
             int64_t s_row, int64_t s_head, int box_rows = BM) {
  const uint64_t dims[3] = {(uint64_t)dim, (uint64_t)heads, (uint64_t)rows};
  const uint64_t strides[2] = {(uint64_t)(s_head * 2), (uint64_t)(s_row * 2)};
  const uint32_t box[3] = {64, 1, (uint32_t)box_rows};
  return encode_tensor_map(map, dtype, 3, ptr, dims, strides, box, true);
}

inline bool al16(const void* ptr) { return ((uintptr_t)ptr & 15u) == 0; }

// Requests per work-order group: as many as keep their K/V within about a
// third of the 126 MB L2 (Q tiles and output rows stream past it), so that
// the K/V tiles every row block and head of a request re-reads come from L2
// (config 2: DRAM reads 3.25 -> 0.81 GB per launch, +7 %).
constexpr int64_t kPrefillGroupBytes = 40ll << 20;
inline int prefill_group_reqs(const AttnParams& p) {
  const int64_t kv_req = (int64_t)p.max_k * p.HK * (p.DQ + p.DV) * 2;
  const int64_t g = kv_req > 0 ? kPrefillGroupBytes / kv_req : p.B;
  return (int)std::min<int64_t>(std::max<int64_t>(g, 1), std::max(p.B, 1));
}

}  // namespace pf

// Wide head dims (prefill_wide_sm100.cu): QK head dim 129..256, V head dim up
// to 256, one query tile per CTA. prefill_wide_dims: the head dims are in its
// range; prefill_wide_supported: also the features (no ALiBi).
bool prefill_wide_dims(const AttnParams& p);
int prefill_wide_supported(const AttnParams& p);
int launch_prefill_wide(const AttnParams& p, const pf::PrefillParams& pp, cudaStream_t stream);
int prefill_wide_timeout_flag(bool clear);

}  // namespace fab
