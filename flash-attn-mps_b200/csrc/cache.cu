// KV-cache bandwidth kernels: store_kvcache (slot scatter + FP8 E4M3
// quantisation), append_kvcache and rotary position embedding.
//
// Semantics follow the reference flash_attn_mps 0.1.0:
//   store   kernels/cache.metal:20-39, host _cache.py:67-85
//   append  kernels/cache.metal:41-56, host _cache.py:99-127
//   rotate  kernels/cache.metal:58-76, host _cache.py:130-155
// store_kvcache: a CTA row of threads covers the (head, 16-byte chunk) pairs of
// one token, CTA rows take successive tokens (grid-stride over tokens), so the
// slot lookup and page split happen once per token and a thread's head (and
// its FP8 reciprocal scale) stays fixed. FP8 quantisation computes x / scale
// correctly rounded without a division per element: with y = RN(1/scale),
// q = RN(x*y), r = x - q*scale (exact by FMA), RN(q + r*y) is the correctly
// rounded quotient (Markstein's theorem for FMA-based division); non-finite
// quotients take the IEEE division. Pairs are encoded with the packed
// cvt.rn.satfinite.e4m3x2.f32. append / rotary: one element or 16-byte vector
// per thread with a grid-stride loop.
#include <algorithm>
#include <type_traits>

#include "common.cuh"

namespace fab {
namespace {

struct StoreSide {
  const void* x;
  void* cache;
  int64_t xs0, xs1, xs2;          // x [T,H,D]
  int64_t cs0, cs1, cs2, cs3;     // cache [N,P,H,D]
  int64_t capacity;               // N*P
  const float* scale;             // FP8 only: [H] or scalar
  int64_t scale_stride;
  int32_t H, D, P;
  int32_t pshift;                 // log2(P) when P is a power of two, else -1
  int64_t tokens;
};

struct StoreArgs {
  StoreSide side[2];
  const void* slots;
  int32_t slot_dtype;
  int64_t slot_stride;
};

template <typename T> struct Vec16 { static constexpr int N = 16 / sizeof(T); };

// RN(x / s) for E4M3 encoding, given y = RN(1/s), with no division and no
// per-element branch: q = x*y is clamped to +-1e4 (every quotient beyond
// +-464 saturates to the same +-448 code; NaN propagates through the
// NaN-keeping min/max), Markstein's FMA correction then yields the correctly
// rounded quotient, and the sign of q is restored for an exact -0 quotient.
__device__ __forceinline__ float quotient_for_e4m3(float x, float s, float y) {
  float q = x * y;
  asm("max.NaN.f32 %0, %0, 0fC61C4000;\n\tmin.NaN.f32 %0, %0, 0f461C4000;" : "+f"(q));  // -1e4, 1e4
  const float r = fmaf(-q, s, x);
  return copysignf(fmaf(r, y, q), q);
}

// Two values -> two E4M3 codes (saturating round-to-nearest-even; the NaNs
// that reach here are the GPU's canonical positive NaN, encoded 0x7F).
__device__ __forceinline__ uint32_t e4m3x2_sat(float a, float b) {
  return (uint32_t)__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
}

// A 16-byte vector of VEC inputs as float32.
template <typename T>
__device__ __forceinline__ void vec_to_f32(const uint4& raw, float (&f)[16 / sizeof(T)]) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int i = 0; i < 4; ++i) f[i] = __uint_as_float(w[i]);
  } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      f[2 * i] = v.x;
      f[2 * i + 1] = v.y;
    }
  }
}

__device__ __forceinline__ int64_t page_of(int64_t slot, int P, int pshift) {
  if (pshift >= 0) return slot >> pshift;
  if (slot < 0x7fffffff) return (int64_t)((uint32_t)slot / (uint32_t)P);
  return slot / P;
}

// One 16-byte input vector (already loaded) of one (token, head) row.
template <typename T, bool FP8>
__device__ __forceinline__ void store_vector16(const StoreSide& s, const uint4& raw, int64_t dst, float scale,
                                               float rscale) {
  constexpr int VEC = 16 / sizeof(T);
  if constexpr (!FP8) {
    *reinterpret_cast<uint4*>(reinterpret_cast<T*>(s.cache) + dst) = raw;
  } else {
    uint8_t* cache = reinterpret_cast<uint8_t*>(s.cache);
    float f[VEC];
    vec_to_f32<T>(raw, f);
    uint32_t codes[VEC / 4];
#pragma unroll
    for (int i = 0; i < VEC / 4; ++i)
      codes[i] = e4m3x2_sat(quotient_for_e4m3(f[4 * i], scale, rscale), quotient_for_e4m3(f[4 * i + 1], scale, rscale)) |
                 (e4m3x2_sat(quotient_for_e4m3(f[4 * i + 2], scale, rscale),
                             quotient_for_e4m3(f[4 * i + 3], scale, rscale)) << 16);
    if constexpr (VEC == 8) {
      *reinterpret_cast<uint2*>(cache + dst) = make_uint2(codes[0], codes[1]);
    } else {
      *reinterpret_cast<uint32_t*>(cache + dst) = codes[0];
    }
  }
}

// Element-wise path (strided or unaligned rows).
template <typename T, bool FP8, int VEC>
__device__ __forceinline__ void store_scalar(const StoreSide& s, int64_t src, int64_t dst, float scale) {
  const T* x = reinterpret_cast<const T*>(s.x);
  for (int i = 0; i < VEC; ++i) {
    if constexpr (FP8)
      reinterpret_cast<uint8_t*>(s.cache)[dst + i * s.cs3] = float_to_e4m3_sat(__fdiv_rn((float)x[src + i * s.xs2], scale));
    else
      reinterpret_cast<T*>(s.cache)[dst + i * s.cs3] = x[src + i * s.xs2];
  }
}

// blockDim.x threads cover the H * D/VEC vectors of a token (looping when
// there are more), blockDim.y token rows per CTA; each thread carries kTokU
// tokens per step so that kTokU slot loads and then kTokU vector loads are in
// flight before the first conversion (the kernel is otherwise latency-bound).
constexpr int kTokU = 4;

template <typename T, bool FP8, int VEC>
__global__ void __launch_bounds__(256) store_kernel(StoreArgs a) {
  const StoreSide& s = a.side[blockIdx.y];
  if (s.x == nullptr) return;
  const int chunks = s.D / VEC;
  const int per_token = s.H * chunks;
  const int64_t rows = (int64_t)gridDim.x * blockDim.y;  // token rows in flight across the grid
  const int64_t tstep = rows * kTokU;
  for (int64_t t0 = (int64_t)blockIdx.x * blockDim.y + threadIdx.y; t0 < s.tokens; t0 += tstep) {
    int64_t dtok[kTokU], stok[kTokU];
#pragma unroll
    for (int u = 0; u < kTokU; ++u) {
      const int64_t t = t0 + u * rows;
      int64_t slot = -1;
      if (t < s.tokens) slot = load_index(a.slots, a.slot_dtype, t * a.slot_stride);
      if (slot < 0 || slot >= s.capacity) {
        dtok[u] = -1;
      } else {
        const int64_t block = page_of(slot, s.P, s.pshift), off = slot - block * s.P;
        dtok[u] = block * s.cs0 + off * s.cs1;
      }
      stok[u] = t * s.xs0;
    }
    for (int i = threadIdx.x; i < per_token; i += blockDim.x) {
      const int h = i / chunks, c = i - h * chunks;
      float scale = 1.f, rscale = 1.f;
      if constexpr (FP8) {
        if (s.scale) {
          scale = __ldg(s.scale + h * s.scale_stride);
          rscale = __frcp_rn(scale);
        }
      }
      const int64_t soff = h * s.xs1 + (int64_t)c * VEC * s.xs2, doff = h * s.cs2 + (int64_t)c * VEC * s.cs3;
      if constexpr (VEC * sizeof(T) == 16) {
        uint4 raw[kTokU];
#pragma unroll
        for (int u = 0; u < kTokU; ++u)
          if (dtok[u] >= 0) raw[u] = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(s.x) + stok[u] + soff));
#pragma unroll
        for (int u = 0; u < kTokU; ++u)
          if (dtok[u] >= 0) store_vector16<T, FP8>(s, raw[u], dtok[u] + doff, scale, rscale);
      } else {
#pragma unroll
        for (int u = 0; u < kTokU; ++u)
          if (dtok[u] >= 0) store_scalar<T, FP8, VEC>(s, stok[u] + soff, dtok[u] + doff, scale);
      }
    }
  }
}

// ---- warp-per-token-row store (16-bit inputs, unit inner strides)
//
// One warp owns one token row (H heads x D dims) at a time; lane L handles
// the 16-byte input vectors L, L+32, ... (NV per lane), whose head, source
// and destination offsets and FP8 scale constants are fixed for the whole
// launch and computed once. The source rows do not depend on the slots, so a
// warp issues the data loads of kRowU tokens together with their slot loads
// (one broadcast load per token) and only the stores wait on the slots.
// E4M3 quantisation per pair of elements: q = RN(x y) clamped to +-1e4,
// r = x - q s and RN(q + r y) (Markstein's correctly rounded quotient,
// y = RN(1/s)) with the products and sums as packed f32x2 operations, the sign
// of q kept for an exact zero, and cvt.rn.satfinite.e4m3x2.f32 encoding the
// pair. Scales that are zero, negative zero or non-finite, or
// whose reciprocal is not finite, take the IEEE division per element.
constexpr int kRowU = 2;

__device__ __forceinline__ uint64_t pk2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void upk2(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// copysign(min(|q|, 1e4), q) with NaN kept: every quotient beyond +-464
// saturates to the same +-448 code, and the bound keeps the exact correction
// below finite (an infinite q would turn it into NaN).
__device__ __forceinline__ float clamp_q(float q) {
  float d;
  asm("min.NaN.xorsign.abs.f32 %0, %1, 0f461C4000;" : "=f"(d) : "f"(q));
  return d;
}

template <typename T>
__device__ __forceinline__ void pair_to_f32(uint32_t w, float& lo, float& hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    lo = __uint_as_float(w << 16);
    hi = __uint_as_float(w & 0xFFFF0000u);
  } else {
    const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&w));
    lo = v.x;
    hi = v.y;
  }
}

struct RowScale {
  uint64_t s2n, y2;   // (-s, -s), (y, y) with y = RN(1/s)
  float s;
  bool fast;          // Markstein path valid for this scale
};

template <typename T>
__device__ __forceinline__ RowScale row_scale(float s) {
  RowScale r;
  const float y = __frcp_rn(s);
  r.s = s;
  r.fast = isfinite(s) && s != 0.f && isfinite(y) && y != 0.f;
  r.s2n = pk2(-s, -s);
  r.y2 = pk2(y, y);
  return r;
}

// 8 inputs (one 16-byte vector) -> 8 E4M3 codes of RN(x / s).
template <typename T>
__device__ __forceinline__ uint2 e4m3x8(const uint4& raw, const RowScale& rs) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
  uint32_t c16[4];
  if (rs.fast) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float x0, x1, q0, q1, d0, d1;
      pair_to_f32<T>(w[i], x0, x1);
      const uint64_t x2 = pk2(x0, x1);
      upk2(mul2(x2, rs.y2), q0, q1);
      const uint64_t q2 = pk2(clamp_q(q0), clamp_q(q1));
      const uint64_t r2 = fma2(q2, rs.s2n, x2);  // x - q s, exact
      upk2(fma2(r2, rs.y2, q2), d0, d1);
      upk2(q2, q0, q1);
      c16[i] = e4m3x2_sat(copysignf(d0, q0), copysignf(d1, q1));
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float x0, x1;
      pair_to_f32<T>(w[i], x0, x1);
      c16[i] = e4m3x2_sat(__fdiv_rn(x0, rs.s), __fdiv_rn(x1, rs.s));
    }
  }
  return make_uint2(c16[0] | (c16[1] << 16), c16[2] | (c16[3] << 16));
}

template <typename T, bool FP8, int NV>
__global__ void __launch_bounds__(256) store_row_kernel(StoreArgs a) {
  const StoreSide& s = a.side[blockIdx.y];
  if (s.x == nullptr) return;
  constexpr int VEC = 8;
  const int lane = threadIdx.x & 31;
  const int chunks = s.D / VEC;
  const int nvec = s.H * chunks;
  int32_t soff[NV], doff[NV];
  RowScale rsc[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int v = k * 32 + lane;
    const int h = v < nvec ? v / chunks : 0;
    const int c = v - h * chunks;
    soff[k] = v < nvec ? (int32_t)(h * s.xs1 + c * VEC) : -1;
    doff[k] = (int32_t)(h * s.cs2 + c * VEC);
    if constexpr (FP8) rsc[k] = row_scale<T>(s.scale ? __ldg(s.scale + h * s.scale_stride) : 1.f);
  }
  const T* x = reinterpret_cast<const T*>(s.x);
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < s.tokens;
       t += warps * kRowU) {
    int64_t slot[kRowU];
    uint4 raw[kRowU][NV];
#pragma unroll
    for (int u = 0; u < kRowU; ++u) {
      const int64_t tt = t + u * warps;
      slot[u] = tt < s.tokens ? load_index(a.slots, a.slot_dtype, tt * a.slot_stride) : -1;
#pragma unroll
      for (int k = 0; k < NV; ++k)
        if (tt < s.tokens && soff[k] >= 0)
          raw[u][k] = __ldg(reinterpret_cast<const uint4*>(x + tt * s.xs0 + soff[k]));
    }
#pragma unroll
    for (int u = 0; u < kRowU; ++u) {
      if (slot[u] < 0 || slot[u] >= s.capacity) continue;
      const int64_t block = page_of(slot[u], s.P, s.pshift), off = slot[u] - block * s.P;
      const int64_t drow = block * s.cs0 + off * s.cs1;
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        if (soff[k] < 0) continue;
        if constexpr (FP8) {
          *reinterpret_cast<uint2*>(reinterpret_cast<uint8_t*>(s.cache) + drow + doff[k]) =
              e4m3x8<T>(raw[u][k], rsc[k]);
        } else {
          *reinterpret_cast<uint4*>(reinterpret_cast<T*>(s.cache) + drow + doff[k]) = raw[u][k];
        }
      }
    }
  }
}

bool aligned(const void* p, int64_t bytes) { return ((uintptr_t)p % bytes) == 0; }

// One side (K or V) of a store call: shape checks and vector eligibility.
int prepare_side(const fa_tensor* x, const fa_tensor* cache, const fa_tensor* scale,
                 int64_t tokens, StoreSide* s, int* dtype, bool* fp8, bool* vec) {
  s->x = nullptr;
  if (!present(x)) return FA_OK;
  FAB_CHECK_ARG(present(cache), "cache is required for each provided K/V input");
  FAB_CHECK_ARG(x->ndim == 3 && cache->ndim == 4, "K/V must be [T,H,D] and caches [N,P,H,D]");
  FAB_CHECK_ARG(x->shape[0] == tokens, "slot_mapping must have one slot per token");
  FAB_CHECK_ARG(cache->shape[2] == x->shape[1] && cache->shape[3] == x->shape[2],
                "cache must have shape [blocks, block_size, heads, dim]");
  FAB_CHECK_ARG(is_float(x->dtype), "input dtype must be float16, bfloat16 or float32");
  *fp8 = cache->dtype == FA_E4M3;
  FAB_CHECK_ARG(*fp8 || cache->dtype == x->dtype, "cache dtype must match input or be float8_e4m3fn");
  *dtype = x->dtype;
  s->x = x->ptr;
  s->cache = cache->ptr;
  s->xs0 = x->stride[0]; s->xs1 = x->stride[1]; s->xs2 = x->stride[2];
  for (int i = 0; i < 4; ++i) (&s->cs0)[i] = cache->stride[i];
  s->H = (int32_t)x->shape[1];
  s->D = (int32_t)x->shape[2];
  s->P = (int32_t)cache->shape[1];
  s->capacity = cache->shape[0] * cache->shape[1];
  s->scale = nullptr;
  s->scale_stride = 0;
  if (*fp8 && present(scale)) {
    FAB_CHECK_ARG(scale->dtype == FA_F32, "scale must be float32");
    int64_t n = 1;
    for (int i = 0; i < scale->ndim; ++i) n *= scale->shape[i];
    FAB_CHECK_ARG(n == 1 || n == s->H, "scale must be scalar or have one value per KV head");
    s->scale = reinterpret_cast<const float*>(scale->ptr);
    s->scale_stride = n == 1 ? 0 : scale->stride[scale->ndim - 1];
  }
  const int esz = elem_size(x->dtype);
  const int v = 16 / esz;
  const int out_bytes = *fp8 ? v : 16;
  *vec = s->D % v == 0 && s->xs2 == 1 && cache->stride[3] == 1 &&
         aligned(x->ptr, 16) && aligned(cache->ptr, out_bytes) &&
         (s->xs0 * esz) % 16 == 0 && (s->xs1 * esz) % 16 == 0 &&
         (s->cs0 * (*fp8 ? 1 : esz)) % out_bytes == 0 && (s->cs1 * (*fp8 ? 1 : esz)) % out_bytes == 0 &&
         (s->cs2 * (*fp8 ? 1 : esz)) % out_bytes == 0;
  s->tokens = tokens;
  s->pshift = -1;
  for (int k = 0; k < 31; ++k)
    if ((1 << k) == s->P) s->pshift = k;
  return FA_OK;
}

// Vectors per lane of the row kernel for this side, or 0 when it does not apply
// (16-bit inputs, whole 16-byte vectors, a row of at most 32 * 8 vectors,
// offsets within a row below 2^31).
template <typename T>
int row_vectors(const StoreSide& s) {
  if (sizeof(T) != 2) return 0;
  const int64_t nvec = (int64_t)s.H * (s.D / 8);
  if (nvec <= 0 || nvec > 32 * 8) return 0;
  if ((int64_t)s.H * s.xs1 + s.D >= (1LL << 31) || (int64_t)s.H * s.cs2 + s.D >= (1LL << 31)) return 0;
  const int64_t nv = (nvec + 31) / 32;
  return nv <= 1 ? 1 : nv <= 2 ? 2 : nv <= 4 ? 4 : 8;
}

template <typename T, bool FP8>
void launch_store(const StoreArgs& a, bool vec, int sides, cudaStream_t stream) {
  const StoreSide& s0 = a.side[0].x ? a.side[0] : a.side[1];
  int nv = vec ? row_vectors<T>(s0) : 0;
  if (nv && a.side[0].x && a.side[1].x && row_vectors<T>(a.side[1]) != nv) nv = 0;
  if constexpr (sizeof(T) == 2) if (nv) {
    // One warp per token row, kRowU rows in flight per warp.
    int64_t blocks = (s0.tokens + 8 * kRowU - 1) / (8 * kRowU);
    const int64_t cap = (int64_t)sm_count() * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    dim3 grid((unsigned)blocks, (unsigned)sides);
    switch (nv) {
      case 1: store_row_kernel<T, FP8, 1><<<grid, 256, 0, stream>>>(a); break;
      case 2: store_row_kernel<T, FP8, 2><<<grid, 256, 0, stream>>>(a); break;
      case 4: store_row_kernel<T, FP8, 4><<<grid, 256, 0, stream>>>(a); break;
      default: store_row_kernel<T, FP8, 8><<<grid, 256, 0, stream>>>(a); break;
    }
    note_launch();
    return;
  }
  const int per_token = s0.H * (vec ? s0.D / Vec16<T>::N : s0.D);  // both sides share H, D
  int bx = (per_token + 31) / 32 * 32;
  if (bx > 256) bx = 256;
  const int by = 256 / bx;
  int64_t blocks = (s0.tokens + (int64_t)by * kTokU - 1) / ((int64_t)by * kTokU);
  const int64_t cap = (int64_t)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  dim3 grid((unsigned)blocks, (unsigned)sides), block((unsigned)bx, (unsigned)by);
  if (vec) store_kernel<T, FP8, Vec16<T>::N><<<grid, block, 0, stream>>>(a);
  else store_kernel<T, FP8, 1><<<grid, block, 0, stream>>>(a);
  note_launch();
}

int dispatch_store(const StoreArgs& a, int dtype, bool fp8, bool vec, int sides, cudaStream_t st) {
  switch (dtype) {
    case FA_F16: fp8 ? launch_store<__half, true>(a, vec, sides, st) : launch_store<__half, false>(a, vec, sides, st); break;
    case FA_BF16: fp8 ? launch_store<__nv_bfloat16, true>(a, vec, sides, st) : launch_store<__nv_bfloat16, false>(a, vec, sides, st); break;
    case FA_F32: fp8 ? launch_store<float, true>(a, vec, sides, st) : launch_store<float, false>(a, vec, sides, st); break;
    default: return fail(FA_ERR_INVALID, "unsupported input dtype");
  }
  FAB_LAUNCH_CHECK("store_kvcache launch");
  return FA_OK;
}

// ------------------------------------------------------------------ append
struct AppendSide {
  const void* x;
  void* cache;
  int64_t xs0, xs1, xs2, xs3;     // x [B,S,H,D]
  int64_t cs0, cs1, cs2, cs3;     // cache [rows|N, capacity|P, H, D]
  const float* scale;
  int64_t scale_stride;
  int32_t S, H, D;
  int32_t xdtype, fp8;
};

struct AppendArgs {
  AppendSide side[2];
  const int32_t* lengths; int64_t len_stride;
  const int32_t* batch_idx; int64_t bi_stride;
  const int32_t* table; int64_t bt0, bt1;
  int32_t paged, pages_per_seq, P, remap;
  int64_t blocks, rows;
  int64_t units;                  // B*S*H*D (max over sides)
};

__global__ void __launch_bounds__(256) append_kernel(AppendArgs a) {
  const AppendSide& s = a.side[blockIdx.y];
  if (s.x == nullptr) return;
  const int64_t total = a.units;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < total; u += step) {
    const int d = (int)(u % s.D);
    int64_t r = u / s.D;
    const int h = (int)(r % s.H); r /= s.H;
    const int j = (int)(r % s.S);
    const int64_t b = r / s.S;
    const int64_t row = a.remap ? (int64_t)a.batch_idx[b * a.bi_stride] : b;
    const int64_t pos = (int64_t)a.lengths[b * a.len_stride] + j;
    const int64_t capacity = a.paged ? (int64_t)a.pages_per_seq * a.P : a.P;
    if (row < 0 || row >= a.rows || pos < 0 || pos >= capacity) continue;
    const int64_t block = a.paged ? (int64_t)a.table[row * a.bt0 + (pos / a.P) * a.bt1] : row;
    const int64_t offset = a.paged ? pos % a.P : pos;
    if (block < 0 || block >= a.blocks) continue;
    const int64_t src = b * s.xs0 + j * s.xs1 + h * s.xs2 + d * s.xs3;
    const int64_t dst = block * s.cs0 + offset * s.cs1 + h * s.cs2 + d * s.cs3;
    if (s.fp8) {
      const float scale = s.scale ? s.scale[h * s.scale_stride] : 1.0f;
      reinterpret_cast<uint8_t*>(s.cache)[dst] =
          float_to_e4m3_sat(__fdiv_rn(load_float(s.x, s.xdtype, src), scale));
    } else if (s.xdtype == FA_F32) {
      reinterpret_cast<uint32_t*>(s.cache)[dst] = reinterpret_cast<const uint32_t*>(s.x)[src];
    } else {
      reinterpret_cast<uint16_t*>(s.cache)[dst] = reinterpret_cast<const uint16_t*>(s.x)[src];
    }
  }
}

// ------------------------------------------------------------------ rotary
struct RotaryArgs {
  const void* x; void* out;
  int64_t xs0, xs1, xs2, xs3;
  int64_t os0, os1, os2, os3;
  const float* cos; const float* sin; int64_t cs0, cs1, ss0, ss1;
  const int32_t* lengths; int64_t len_stride;
  int32_t S, H, D, half, interleaved, advance, dtype;
  int64_t units;
};

__global__ void __launch_bounds__(256) rotary_kernel(RotaryArgs a) {
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < a.units; u += step) {
    const int d = (int)(u % a.D);
    int64_t r = u / a.D;
    const int h = (int)(r % a.H); r /= a.H;
    const int j = (int)(r % a.S);
    const int64_t b = r / a.S;
    const int64_t src = b * a.xs0 + j * a.xs1 + h * a.xs2;
    const int64_t dst = b * a.os0 + j * a.os1 + h * a.os2 + d * a.os3;
    if (d >= 2 * a.half) {
      if (a.dtype == FA_F32)
        reinterpret_cast<uint32_t*>(a.out)[dst] = reinterpret_cast<const uint32_t*>(a.x)[src + d * a.xs3];
      else
        reinterpret_cast<uint16_t*>(a.out)[dst] = reinterpret_cast<const uint16_t*>(a.x)[src + d * a.xs3];
      continue;
    }
    const int pair = a.interleaved ? d / 2 : d % a.half;
    const bool second = a.interleaved ? (d & 1) : d >= a.half;
    const int other = a.interleaved ? (second ? d - 1 : d + 1) : (second ? d - a.half : d + a.half);
    const int64_t pos = (int64_t)a.lengths[b * a.len_stride] + (a.advance ? j : 0);
    const float c = a.cos[pos * a.cs0 + pair * a.cs1], s = a.sin[pos * a.ss0 + pair * a.ss1];
    const float x = load_float(a.x, a.dtype, src + d * a.xs3);
    const float y = load_float(a.x, a.dtype, src + other * a.xs3);
    // Same operation order as the reference (x*c and y*s rounded separately).
    const float ys = __fmul_rn(y, s);
    const float value = __fadd_rn(__fmul_rn(x, c), second ? ys : -ys);
    store_float(a.out, a.dtype, dst, value);
  }
}

// ------------------------------------------------- fused rotary + append
// Rotates the new K at lengths[b] + j, rounds it to K's dtype (what the
// separate rotary writes), appends it (E4M3-quantised for an FP8 cache),
// appends V, and rotates Q into q_out at lengths[b] (+ j when advance_q): the
// same values as rotary followed by append, in one pass (blockIdx.y = 0 K,
// 1 V, 2 Q). cos/sin may be any float dtype (read as float32).
struct RopeArgs {
  const void* cos; const void* sin; int32_t cdtype;
  int64_t cs0, cs1, ss0, ss1;
  int32_t half, interleaved, advance_q;
  int64_t batch;
  const void* q; void* q_out; int32_t qdtype, QS, QH, QD;
  int64_t qs0, qs1, qs2, qs3, qo0, qo1, qo2, qo3;
  int64_t q_units;
};

__device__ __forceinline__ float round_to(int dtype, float v) {
  if (dtype == FA_F16) return __half2float(__float2half_rn(v));
  if (dtype == FA_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  return v;
}

// Rotated value of element d of row `src` (element strides ds) at position pos.
__device__ __forceinline__ float rope_value(const RopeArgs& r, const void* x, int dtype, int64_t src, int64_t ds,
                                            int d, int64_t pos) {
  const int pair = r.interleaved ? d / 2 : d % r.half;
  const bool second = r.interleaved ? (d & 1) : d >= r.half;
  const int other = r.interleaved ? (second ? d - 1 : d + 1) : (second ? d - r.half : d + r.half);
  const float c = load_float(r.cos, r.cdtype, pos * r.cs0 + pair * r.cs1);
  const float sn = load_float(r.sin, r.cdtype, pos * r.ss0 + pair * r.ss1);
  const float xv = load_float(x, dtype, src + d * ds);
  const float yv = load_float(x, dtype, src + other * ds);
  const float ys = __fmul_rn(yv, sn);
  return __fadd_rn(__fmul_rn(xv, c), second ? ys : -ys);
}

__global__ void __launch_bounds__(256) rotary_append_kernel(AppendArgs a, RopeArgs r) {
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  if (blockIdx.y == 2) {
    for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < r.q_units; u += step) {
      const int d = (int)(u % r.QD);
      int64_t t = u / r.QD;
      const int h = (int)(t % r.QH); t /= r.QH;
      const int j = (int)(t % r.QS);
      const int64_t b = t / r.QS;
      const int64_t src = b * r.qs0 + j * r.qs1 + h * r.qs2;
      const int64_t dst = b * r.qo0 + j * r.qo1 + h * r.qo2 + d * r.qo3;
      const int64_t pos = (int64_t)a.lengths[b * a.len_stride] + (r.advance_q ? j : 0);
      const float value = d < 2 * r.half ? rope_value(r, r.q, r.qdtype, src, r.qs3, d, pos)
                                         : load_float(r.q, r.qdtype, src + d * r.qs3);
      store_float(r.q_out, r.qdtype, dst, value);
    }
    return;
  }
  const AppendSide& s = a.side[blockIdx.y];
  if (s.x == nullptr) return;
  const bool rotate = blockIdx.y == 0;
  const int64_t total = r.batch * s.S * (int64_t)s.H * s.D;
  for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < total; u += step) {
    const int d = (int)(u % s.D);
    int64_t t = u / s.D;
    const int h = (int)(t % s.H); t /= s.H;
    const int j = (int)(t % s.S);
    const int64_t b = t / s.S;
    const int64_t row = a.remap ? (int64_t)a.batch_idx[b * a.bi_stride] : b;
    const int64_t pos = (int64_t)a.lengths[b * a.len_stride] + j;
    const int64_t capacity = a.paged ? (int64_t)a.pages_per_seq * a.P : a.P;
    if (row < 0 || row >= a.rows || pos < 0 || pos >= capacity) continue;
    const int64_t block = a.paged ? (int64_t)a.table[row * a.bt0 + (pos / a.P) * a.bt1] : row;
    const int64_t offset = a.paged ? pos % a.P : pos;
    if (block < 0 || block >= a.blocks) continue;
    const int64_t src = b * s.xs0 + j * s.xs1 + h * s.xs2;
    const int64_t dst = block * s.cs0 + offset * s.cs1 + h * s.cs2 + d * s.cs3;
    const float value = rotate && d < 2 * r.half ? round_to(s.xdtype, rope_value(r, s.x, s.xdtype, src, s.xs3, d, pos))
                                                 : load_float(s.x, s.xdtype, src + d * s.xs3);
    if (s.fp8) {
      const float scale = s.scale ? s.scale[h * s.scale_stride] : 1.0f;
      reinterpret_cast<uint8_t*>(s.cache)[dst] = float_to_e4m3_sat(__fdiv_rn(value, scale));
    } else {
      store_float(s.cache, s.xdtype, dst, value);
    }
  }
}

int grid_for(int64_t units) {
  int64_t blocks = (units + 255) / 256;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  return (int)(blocks < 1 ? 1 : blocks);
}

// ------------------------------------------- vectorized RoPE + append
// The same element values as append_kernel / rotary_append_kernel (identical
// mul/add roundings, same skips) for 16-bit rows with unit inner stride:
// each thread moves one 16-byte vector of 8 elements of one head row, and a
// split-half rotation pairs the vector at e with the one at e + half. Sides:
// blockIdx.y 0 = K (rotated when `rotate`), 1 = V, 2 = Q (rotated into q_out).
struct VecSide {
  const uint8_t* x; uint8_t* dst;  // byte pointers (dst: cache, or q_out for Q)
  int64_t xs0, xs1, xs2;           // element strides of x [B,S,H,D]
  int64_t ds0, ds1, ds2;           // cache [N|rows, P|cap, H, D], or q_out [B,S,H,D]
  const float* scale; int64_t scale_stride;
  int32_t H, V, fp8, rotate;       // V = D / 8
  int32_t vshift;                  // log2(V), or -1 when V is not a power of two
};

struct VecArgs {
  VecSide side[3];
  const float* cos; const float* sin; int64_t cs0, ss0;
  int32_t half, interleaved, advance_q;
  const int32_t* lengths; int64_t len_stride;
  const int32_t* batch_idx; int64_t bi_stride;
  const int32_t* table; int64_t bt0, bt1;
  int32_t paged, pages_per_seq, P, remap, S;
  int32_t pshift;                  // log2(P), or -1 when P is not a power of two
  int64_t blocks, rows, tokens;
};

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
      f[2 * i] = t.x; f[2 * i + 1] = t.y;
    } else {
      const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      f[2 * i] = t.x; f[2 * i + 1] = t.y;
    }
  }
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      const __nv_bfloat162 t = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<const uint32_t*>(&t);
    } else {
      const __half2 t = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<const uint32_t*>(&t);
    }
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Store 8 values at element e of a destination row: RN to T, or (FP8 cache)
// the saturating E4M3 code of float(T-rounded value) / scale.
template <typename T>
__device__ __forceinline__ void put8(const VecSide& s, uint8_t* row, int e, const float (&f)[8], float scale) {
  if (!s.fp8) {
    *reinterpret_cast<uint4*>(row + (int64_t)e * sizeof(T)) = pack8<T>(f);
    return;
  }
  uint32_t w[2] = {0u, 0u};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float v = std::is_same<T, __nv_bfloat16>::value ? __bfloat162float(__float2bfloat16_rn(f[i]))
                                                           : __half2float(__float2half_rn(f[i]));
    w[i >> 2] |= (uint32_t)float_to_e4m3_sat(__fdiv_rn(v, scale)) << ((i & 3) * 8);
  }
  *reinterpret_cast<uint2*>(row + e) = make_uint2(w[0], w[1]);
}

template <typename T>
__global__ void __launch_bounds__(128) rope_append_vec_kernel(VecArgs a) {
  const int which = blockIdx.y;
  const VecSide& s = a.side[which];
  if (s.x == nullptr) return;
  const int units = s.H * s.V;
  const int64_t dst_elt = which != 2 && s.fp8 ? 1 : (int64_t)sizeof(T);
  // One token row (all heads) per block iteration: the row geometry (request,
  // position, page) is computed once per token, heads and vectors by shifts.
  for (int64_t tok = blockIdx.x; tok < a.tokens; tok += gridDim.x) {
    const int64_t b = tok <= 0x7fffffff ? (int64_t)((uint32_t)tok / (uint32_t)a.S) : tok / a.S;
    const int j = (int)(tok - b * a.S);
    const int64_t len = a.lengths[b * a.len_stride];
    int64_t pos;
    uint8_t* out_tok;
    if (which == 2) {
      pos = len + (a.advance_q ? j : 0);
      out_tok = s.dst + (b * s.ds0 + j * s.ds1) * dst_elt;
    } else {
      pos = len + j;
      const int64_t row = a.remap ? (int64_t)a.batch_idx[b * a.bi_stride] : b;
      const int64_t capacity = a.paged ? (int64_t)a.pages_per_seq * a.P : a.P;
      if (row < 0 || row >= a.rows || pos < 0 || pos >= capacity) continue;
      int64_t block = row, offset = pos;
      if (a.paged) {
        const int64_t pg = a.pshift >= 0 ? (pos >> a.pshift) : pos / a.P;
        block = a.table[row * a.bt0 + pg * a.bt1];
        offset = pos - pg * a.P;
      }
      if (block < 0 || block >= a.blocks) continue;
      out_tok = s.dst + (block * s.ds0 + offset * s.ds1) * dst_elt;
    }
    const uint8_t* in_tok = s.x + (b * s.xs0 + j * s.xs1) * (int64_t)sizeof(T);
    for (int u = threadIdx.x; u < units; u += blockDim.x) {
      const int h = s.vshift >= 0 ? (u >> s.vshift) : u / s.V;
      const int c0 = (u - h * s.V) * 8;
      uint8_t* out = out_tok + h * s.ds2 * dst_elt;
      const uint8_t* in = in_tok + h * s.xs2 * (int64_t)sizeof(T);
      const float scale = s.fp8 && s.scale ? s.scale[h * s.scale_stride] : 1.0f;
      const bool rotated = s.rotate && c0 < 2 * a.half;
      if (!rotated) {
        if (!s.fp8) {
          *reinterpret_cast<uint4*>(out + (int64_t)c0 * sizeof(T)) =
              __ldg(reinterpret_cast<const uint4*>(in + (int64_t)c0 * sizeof(T)));
        } else {
          float f[8];
          unpack8<T>(__ldg(reinterpret_cast<const uint4*>(in + (int64_t)c0 * sizeof(T))), f);
          put8<T>(s, out, c0, f, scale);
        }
        continue;
      }
      if (a.interleaved) {
        // Pairs (c0 + 2k, c0 + 2k + 1) use angle index c0/2 + k.
        float x[8], o[8];
        unpack8<T>(__ldg(reinterpret_cast<const uint4*>(in + (int64_t)c0 * sizeof(T))), x);
        const float4 cv = __ldg(reinterpret_cast<const float4*>(a.cos + pos * a.cs0 + c0 / 2));
        const float4 sv = __ldg(reinterpret_cast<const float4*>(a.sin + pos * a.ss0 + c0 / 2));
        const float cc[4] = {cv.x, cv.y, cv.z, cv.w}, ss[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          o[2 * k] = __fadd_rn(__fmul_rn(x[2 * k], cc[k]), -__fmul_rn(x[2 * k + 1], ss[k]));
          o[2 * k + 1] = __fadd_rn(__fmul_rn(x[2 * k + 1], cc[k]), __fmul_rn(x[2 * k], ss[k]));
        }
        put8<T>(s, out, c0, o, scale);
      } else {
        if (c0 >= a.half) continue;  // the partner vector at c0 - half writes this one
        float x1[8], x2[8], o1[8], o2[8];
        unpack8<T>(__ldg(reinterpret_cast<const uint4*>(in + (int64_t)c0 * sizeof(T))), x1);
        unpack8<T>(__ldg(reinterpret_cast<const uint4*>(in + (int64_t)(c0 + a.half) * sizeof(T))), x2);
        const float4* cp = reinterpret_cast<const float4*>(a.cos + pos * a.cs0 + c0);
        const float4* sp = reinterpret_cast<const float4*>(a.sin + pos * a.ss0 + c0);
        const float4 ca = __ldg(cp), cb = __ldg(cp + 1), sa = __ldg(sp), sb = __ldg(sp + 1);
        const float cc[8] = {ca.x, ca.y, ca.z, ca.w, cb.x, cb.y, cb.z, cb.w};
        const float ss[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          o1[k] = __fadd_rn(__fmul_rn(x1[k], cc[k]), -__fmul_rn(x2[k], ss[k]));
          o2[k] = __fadd_rn(__fmul_rn(x2[k], cc[k]), __fmul_rn(x1[k], ss[k]));
        }
        put8<T>(s, out, c0, o1, scale);
        put8<T>(s, out, c0 + a.half, o2, scale);
      }
    }
  }
}

// Warp-per-token-row variant of rope_append_vec_kernel (same arithmetic, same
// results bit for bit). A warp owns one (token, head group) of one side at a
// time; lane L takes one column group c = L % U of a head (U = column groups
// per head: a rotated split-half pair (c, c + half), or one 16-byte vector) for
// MAXU heads of the group, 32 / U apart, so its cos/sin columns are loaded
// once per item. The input vectors do not depend on the request's length or
// page table and are loaded first; the length of the warp's next item is
// prefetched while the current one is written. Rows wider than 32 * MAXU
// column groups (16 query heads of 128 dims) take several warps, which keeps
// the kernel at 80 registers (3 CTAs per SM).
template <typename T, int MAXU, bool FP8>
__global__ void __launch_bounds__(256) rope_append_warp_kernel(VecArgs a) {
  const int which = blockIdx.y;
  const VecSide& s = a.side[which];
  if (s.x == nullptr) return;
  const int lane = threadIdx.x & 31;
  const bool split = s.rotate && !a.interleaved;
  const int r2 = split ? a.half / 8 : 0;  // rotated pairs per head
  const int uph = s.V - r2;               // column groups per head (divides 32)
  const int c = lane % uph, hstep = 32 / uph;
  // A token row is split into head groups of 32 * MAXU / uph heads; a warp
  // work item is one (token, head group).
  const int group_heads = hstep * MAXU;
  const int groups = (s.H + group_heads - 1) / group_heads;
  const int64_t items = a.tokens * groups;
  const bool pair = split && c < r2;
  const int c0 = split && !pair ? (r2 + c) * 8 : c * 8;
  const bool rot = s.rotate && (split ? pair : c0 < 2 * a.half);
  const bool fp8 = FP8 && s.fp8;  // FP8 = some side writes an FP8 cache
  const int64_t dst_elt = which != 2 && fp8 ? 1 : (int64_t)sizeof(T);
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  auto split_tok = [&](int64_t t, int64_t& b, int& j) {
    b = t <= 0x7fffffff ? (int64_t)((uint32_t)t / (uint32_t)a.S) : t / a.S;
    j = (int)(t - b * a.S);
  };
  int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  int64_t b = 0;
  int j = 0, hbase = 0;
  int64_t len = 0;
  auto split_item = [&](int64_t w, int64_t& bb, int& jj, int& hb) {
    const int64_t t = groups == 1 ? w : w / groups;
    hb = (int)(w - t * groups) * group_heads + lane / uph;
    split_tok(t, bb, jj);
  };
  if (item < items) {
    split_item(item, b, j, hbase);
    len = a.lengths[b * a.len_stride];
  }
  for (; item < items; item += warps) {
    const uint8_t* in_tok = s.x + (b * s.xs0 + j * s.xs1) * (int64_t)sizeof(T);
    uint4 xa[MAXU], xb[MAXU];
#pragma unroll
    for (int k = 0; k < MAXU; ++k) {
      const int h = hbase + k * hstep;
      if (h < s.H) {
        const uint8_t* in = in_tok + h * s.xs2 * (int64_t)sizeof(T);
        xa[k] = __ldg(reinterpret_cast<const uint4*>(in + (int64_t)c0 * sizeof(T)));
        if (pair) xb[k] = __ldg(reinterpret_cast<const uint4*>(in + (int64_t)(c0 + a.half) * sizeof(T)));
      }
    }
    // Row geometry of this token; the next item's length is loaded meanwhile.
    int64_t nb = 0, nlen = 0;
    int nj = 0, nhbase = 0;
    if (item + warps < items) {
      split_item(item + warps, nb, nj, nhbase);
      nlen = a.lengths[nb * a.len_stride];
    }
    int64_t pos;
    uint8_t* out_tok = nullptr;
    if (which == 2) {
      pos = len + (a.advance_q ? j : 0);
      out_tok = s.dst + (b * s.ds0 + j * s.ds1) * dst_elt;
    } else {
      pos = len + j;
      const int64_t row = a.remap ? (int64_t)a.batch_idx[b * a.bi_stride] : b;
      const int64_t capacity = a.paged ? (int64_t)a.pages_per_seq * a.P : a.P;
      if (row >= 0 && row < a.rows && pos >= 0 && pos < capacity) {
        int64_t block = row, offset = pos;
        if (a.paged) {
          const int64_t pg = a.pshift >= 0 ? (pos >> a.pshift) : pos / a.P;
          block = a.table[row * a.bt0 + pg * a.bt1];
          offset = pos - pg * a.P;
        }
        if (block >= 0 && block < a.blocks) out_tok = s.dst + (block * s.ds0 + offset * s.ds1) * dst_elt;
      }
    }
    if (out_tok != nullptr) {
      float cc[8], ss[8];
      if (rot) {
        if (split) {
          const float4* cp = reinterpret_cast<const float4*>(a.cos + pos * a.cs0 + c0);
          const float4* sp = reinterpret_cast<const float4*>(a.sin + pos * a.ss0 + c0);
          const float4 ca = __ldg(cp), cb = __ldg(cp + 1), sa = __ldg(sp), sb = __ldg(sp + 1);
          cc[0] = ca.x; cc[1] = ca.y; cc[2] = ca.z; cc[3] = ca.w; cc[4] = cb.x; cc[5] = cb.y; cc[6] = cb.z; cc[7] = cb.w;
          ss[0] = sa.x; ss[1] = sa.y; ss[2] = sa.z; ss[3] = sa.w; ss[4] = sb.x; ss[5] = sb.y; ss[6] = sb.z; ss[7] = sb.w;
        } else {
          const float4 cv = __ldg(reinterpret_cast<const float4*>(a.cos + pos * a.cs0 + c0 / 2));
          const float4 sv = __ldg(reinterpret_cast<const float4*>(a.sin + pos * a.ss0 + c0 / 2));
          cc[0] = cv.x; cc[1] = cv.y; cc[2] = cv.z; cc[3] = cv.w;
          ss[0] = sv.x; ss[1] = sv.y; ss[2] = sv.z; ss[3] = sv.w;
        }
      }
#pragma unroll
      for (int k = 0; k < MAXU; ++k) {
        const int h = hbase + k * hstep;
        if (h >= s.H) continue;
        uint8_t* out = out_tok + h * s.ds2 * dst_elt;
        const float scale = fp8 && s.scale ? s.scale[h * s.scale_stride] : 1.0f;
        if (!rot) {
          if (!fp8) {
            *reinterpret_cast<uint4*>(out + (int64_t)c0 * sizeof(T)) = xa[k];
          } else {
            float f[8];
            unpack8<T>(xa[k], f);
            put8<T>(s, out, c0, f, scale);
          }
        } else if (split) {
          float x1[8], x2[8], o1[8], o2[8];
          unpack8<T>(xa[k], x1);
          unpack8<T>(xb[k], x2);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            o1[i] = __fadd_rn(__fmul_rn(x1[i], cc[i]), -__fmul_rn(x2[i], ss[i]));
            o2[i] = __fadd_rn(__fmul_rn(x2[i], cc[i]), __fmul_rn(x1[i], ss[i]));
          }
          put8<T>(s, out, c0, o1, scale);
          put8<T>(s, out, c0 + a.half, o2, scale);
        } else {
          float x[8], o[8];
          unpack8<T>(xa[k], x);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            o[2 * i] = __fadd_rn(__fmul_rn(x[2 * i], cc[i]), -__fmul_rn(x[2 * i + 1], ss[i]));
            o[2 * i + 1] = __fadd_rn(__fmul_rn(x[2 * i + 1], cc[i]), __fmul_rn(x[2 * i], ss[i]));
          }
          put8<T>(s, out, c0, o, scale);
        }
      }
    }
    b = nb;
    j = nj;
    hbase = nhbase;
    len = nlen;
  }
}

// Whether the warp kernel applies to this side: its column groups per head
// must divide 32 (rows wider than 64 column groups are split over warps).
bool warp_fits(const VecSide& s, const VecArgs& a) {
  if (!s.x) return true;
  const int r2 = s.rotate && !a.interleaved ? a.half / 8 : 0;
  const int uph = s.V - r2;
  return uph > 0 && 32 % uph == 0;
}

inline bool aligned(const void* p, int bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }

inline int log2_exact(int64_t v) {
  if (v <= 0 || (v & (v - 1))) return -1;
  int k = 0;
  while ((int64_t(1) << k) < v) ++k;
  return k;
}

// Launch the vectorized kernel when every operand qualifies; returns 1 when it
// did not apply (the caller runs the scalar kernel), else FA_OK / an error.
// `r` may be null (plain append, nothing rotated).
int launch_rope_append_vec(const AppendArgs& a, const RopeArgs* r, int64_t batch, cudaStream_t stream) {
  int dtype = -1;
  VecArgs v{};
  bool any = false;
  for (int i = 0; i < 2; ++i) {
    const AppendSide& s = a.side[i];
    if (!s.x) continue;
    if (s.xdtype != FA_BF16 && s.xdtype != FA_F16) return 1;
    if (dtype >= 0 && s.xdtype != dtype) return 1;
    dtype = s.xdtype;
    if (s.D % 8 || s.xs3 != 1 || s.cs3 != 1) return 1;
    if (s.xs0 % 8 || s.xs1 % 8 || s.xs2 % 8 || !aligned(s.x, 16)) return 1;
    if (s.cs0 % 8 || s.cs1 % 8 || s.cs2 % 8 || !aligned(s.cache, s.fp8 ? 8 : 16)) return 1;
    if (v.S && v.S != s.S) return 1;
    v.S = s.S;
    VecSide& o = v.side[i];
    o.x = reinterpret_cast<const uint8_t*>(s.x); o.dst = reinterpret_cast<uint8_t*>(s.cache);
    o.xs0 = s.xs0; o.xs1 = s.xs1; o.xs2 = s.xs2; o.ds0 = s.cs0; o.ds1 = s.cs1; o.ds2 = s.cs2;
    o.scale = s.scale; o.scale_stride = s.scale_stride;
    o.H = s.H; o.V = s.D / 8; o.fp8 = s.fp8; o.rotate = (r != nullptr && i == 0);
    any = true;
  }
  int sides = 2;
  if (r) {
    if (r->cdtype != FA_F32 || r->cs1 != 1 || r->ss1 != 1 || r->cs0 % 4 || r->ss0 % 4) return 1;
    if (!aligned(r->cos, 16) || !aligned(r->sin, 16)) return 1;
    if (r->interleaved ? (r->half % 4) : (r->half % 8)) return 1;
    v.cos = reinterpret_cast<const float*>(r->cos); v.sin = reinterpret_cast<const float*>(r->sin);
    v.cs0 = r->cs0; v.ss0 = r->ss0;
    v.half = r->half; v.interleaved = r->interleaved; v.advance_q = r->advance_q;
    if (r->q) {
      if (r->qdtype != dtype || r->QD % 8 || r->qs3 != 1 || r->qo3 != 1) return 1;
      if (r->qs0 % 8 || r->qs1 % 8 || r->qs2 % 8 || r->qo0 % 8 || r->qo1 % 8 || r->qo2 % 8) return 1;
      if (!aligned(r->q, 16) || !aligned(r->q_out, 16) || (v.S && r->QS != v.S)) return 1;
      VecSide& o = v.side[2];
      o.x = reinterpret_cast<const uint8_t*>(r->q); o.dst = reinterpret_cast<uint8_t*>(r->q_out);
      o.xs0 = r->qs0; o.xs1 = r->qs1; o.xs2 = r->qs2; o.ds0 = r->qo0; o.ds1 = r->qo1; o.ds2 = r->qo2;
      o.H = r->QH; o.V = r->QD / 8; o.rotate = 1;
      v.S = r->QS;
      sides = 3;
      any = true;
    }
  }
  if (!any || dtype < 0) return 1;
  v.lengths = a.lengths; v.len_stride = a.len_stride;
  v.batch_idx = a.batch_idx; v.bi_stride = a.bi_stride;
  v.table = a.table; v.bt0 = a.bt0; v.bt1 = a.bt1;
  v.paged = a.paged; v.pages_per_seq = a.pages_per_seq; v.P = a.P; v.remap = a.remap;
  v.blocks = a.blocks; v.rows = a.rows; v.tokens = batch * v.S;
  v.pshift = log2_exact(a.P);
  bool work = false;
  for (int i = 0; i < 3; ++i)
    if (v.side[i].x) {
      v.side[i].vshift = log2_exact(v.side[i].V);
      work = work || (int64_t)v.side[i].H * v.side[i].V > 0;
    }
  if (v.tokens == 0 || !work) return FA_OK;
  bool fits = true;
  for (int i = 0; i < 3; ++i) fits = fits && warp_fits(v.side[i], v);
  if (fits) {
    const bool fp8 = (v.side[0].x && v.side[0].fp8) || (v.side[1].x && v.side[1].fp8);
    const bool bf = dtype == FA_BF16;
    // Two heads per lane at most: wider rows take several warps per token.
    auto kernel = bf ? (fp8 ? rope_append_warp_kernel<__nv_bfloat16, 2, true> : rope_append_warp_kernel<__nv_bfloat16, 2, false>)
                     : (fp8 ? rope_append_warp_kernel<__half, 2, true> : rope_append_warp_kernel<__half, 2, false>);
    // One warp per token row (8 per CTA); the grid holds exactly the CTAs that
    // are resident at once (all sides together), each looping over tokens.
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 256, 0) != cudaSuccess || per_sm < 1)
      per_sm = 1;
    int64_t cap = (int64_t)sm_count() * per_sm / sides;
    if (cap < 1) cap = 1;
    const int64_t want = (v.tokens * 2 + 7) / 8;
    const dim3 grid((unsigned)(want < cap ? want : cap), sides);
    kernel<<<grid, 256, 0, stream>>>(v);
    note_launch();
    FAB_LAUNCH_CHECK("vectorized append launch");
    return FA_OK;
  }
  const int64_t cap = (int64_t)sm_count() * 16;
  const dim3 grid((unsigned)(v.tokens < cap ? v.tokens : cap), sides);
  if (dtype == FA_BF16) rope_append_vec_kernel<__nv_bfloat16><<<grid, 128, 0, stream>>>(v);
  else rope_append_vec_kernel<__half><<<grid, 128, 0, stream>>>(v);
  note_launch();
  FAB_LAUNCH_CHECK("vectorized append launch");
  return FA_OK;
}

int prepare_append_side(const fa_tensor* x, const fa_tensor* cache, const fa_tensor* scale,
                        int64_t batch, AppendSide* s) {
  s->x = nullptr;
  if (!present(x)) return FA_OK;
  FAB_CHECK_ARG(present(cache), "cache is required for each provided K/V input");
  FAB_CHECK_ARG(x->ndim == 4 && cache->ndim == 4, "K/V must be [B,S,H,D] and caches 4-D");
  FAB_CHECK_ARG(x->shape[0] == batch, "K/V batch must match lengths");
  FAB_CHECK_ARG(cache->shape[2] == x->shape[2] && cache->shape[3] == x->shape[3],
                "cache must have shape [rows, capacity, heads, dim]");
  FAB_CHECK_ARG(is_float(x->dtype), "input dtype must be float16, bfloat16 or float32");
  const bool fp8 = cache->dtype == FA_E4M3;
  FAB_CHECK_ARG(fp8 || cache->dtype == x->dtype, "cache dtype must match input or be float8_e4m3fn");
  s->x = x->ptr; s->cache = cache->ptr;
  for (int i = 0; i < 4; ++i) { (&s->xs0)[i] = x->stride[i]; (&s->cs0)[i] = cache->stride[i]; }
  s->S = (int32_t)x->shape[1]; s->H = (int32_t)x->shape[2]; s->D = (int32_t)x->shape[3];
  s->xdtype = x->dtype; s->fp8 = fp8;
  s->scale = nullptr; s->scale_stride = 0;
  if (fp8 && present(scale)) {
    int64_t n = 1;
    for (int i = 0; i < scale->ndim; ++i) n *= scale->shape[i];
    FAB_CHECK_ARG(scale->dtype == FA_F32 && (n == 1 || n == s->H),
                  "scale must be scalar or have one value per KV head");
    s->scale = reinterpret_cast<const float*>(scale->ptr);
    s->scale_stride = n == 1 ? 0 : scale->stride[scale->ndim - 1];
  }
  return FA_OK;
}

}  // namespace
}  // namespace fab

using namespace fab;

extern "C" int fa_store_kvcache(const fa_tensor* key, const fa_tensor* value,
                                const fa_tensor* k_cache, const fa_tensor* v_cache,
                                const fa_tensor* slot_mapping,
                                const fa_tensor* k_scale, const fa_tensor* v_scale,
                                void* stream) {
  FAB_CHECK_ARG(present(slot_mapping) && slot_mapping->ndim == 1 &&
                    (slot_mapping->dtype == FA_I32 || slot_mapping->dtype == FA_I64),
                "slot_mapping must be int32/int64 with one slot per token");
  const int64_t tokens = slot_mapping->shape[0];
  StoreArgs a{};
  a.slots = slot_mapping->ptr;
  a.slot_dtype = slot_mapping->dtype;
  a.slot_stride = slot_mapping->stride[0];
  int dt[2] = {0, 0};
  bool fp8[2] = {false, false}, vec[2] = {false, false};
  int rc = prepare_side(key, k_cache, k_scale, tokens, &a.side[0], &dt[0], &fp8[0], &vec[0]);
  if (rc) return rc;
  rc = prepare_side(value, v_cache, v_scale, tokens, &a.side[1], &dt[1], &fp8[1], &vec[1]);
  if (rc) return rc;
  if (tokens == 0) return FA_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool have0 = a.side[0].x != nullptr, have1 = a.side[1].x != nullptr;
  if (have0 && have1 && dt[0] == dt[1] && fp8[0] == fp8[1] && vec[0] == vec[1]) {
    if ((int64_t)a.side[0].H * a.side[0].D == 0 && (int64_t)a.side[1].H * a.side[1].D == 0) return FA_OK;
    return dispatch_store(a, dt[0], fp8[0], vec[0], 2, st);
  }
  for (int i = 0; i < 2; ++i) {
    if (a.side[i].x == nullptr || (int64_t)a.side[i].H * a.side[i].D == 0) continue;
    StoreArgs one = a;
    one.side[0] = a.side[i];
    rc = dispatch_store(one, dt[i], fp8[i], vec[i], 1, st);
    if (rc) return rc;
  }
  return FA_OK;
}

extern "C" int fa_append_kvcache(const fa_tensor* key, const fa_tensor* value,
                                 const fa_tensor* k_cache, const fa_tensor* v_cache,
                                 const fa_tensor* lengths, const fa_tensor* cache_batch_idx,
                                 const fa_tensor* block_table,
                                 const fa_tensor* k_scale, const fa_tensor* v_scale,
                                 void* stream) {
  FAB_CHECK_ARG(present(lengths) && lengths->dtype == FA_I32 && lengths->ndim == 1,
                "lengths must be int32 [B]");
  const int64_t batch = lengths->shape[0];
  AppendArgs a{};
  int rc = prepare_append_side(key, k_cache, k_scale, batch, &a.side[0]);
  if (rc) return rc;
  rc = prepare_append_side(value, v_cache, v_scale, batch, &a.side[1]);
  if (rc) return rc;
  const fa_tensor* ref_cache = present(k_cache) ? k_cache : v_cache;
  FAB_CHECK_ARG(present(ref_cache), "a cache is required");
  a.lengths = reinterpret_cast<const int32_t*>(lengths->ptr);
  a.len_stride = lengths->stride[0];
  a.paged = present(block_table);
  a.remap = !a.paged && present(cache_batch_idx);
  if (a.remap) {
    FAB_CHECK_ARG(cache_batch_idx->dtype == FA_I32 && cache_batch_idx->ndim == 1 &&
                      cache_batch_idx->shape[0] == batch, "cache_batch_idx must be int32 [B]");
    a.batch_idx = reinterpret_cast<const int32_t*>(cache_batch_idx->ptr);
    a.bi_stride = cache_batch_idx->stride[0];
  }
  if (a.paged) {
    FAB_CHECK_ARG(block_table->dtype == FA_I32 && block_table->ndim == 2,
                  "block_table must have shape [cache_batch, blocks_per_sequence]");
    a.table = reinterpret_cast<const int32_t*>(block_table->ptr);
    a.bt0 = block_table->stride[0];
    a.bt1 = block_table->stride[1];
    a.pages_per_seq = (int32_t)block_table->shape[1];
    a.rows = block_table->shape[0];
  } else {
    a.rows = ref_cache->shape[0];
  }
  a.P = (int32_t)ref_cache->shape[1];
  a.blocks = ref_cache->shape[0];
  int64_t units = 0;
  for (int i = 0; i < 2; ++i)
    if (a.side[i].x) {
      const int64_t n = batch * a.side[i].S * (int64_t)a.side[i].H * a.side[i].D;
      units = n > units ? n : units;
    }
  if (units == 0) return FA_OK;
  const int vrc = launch_rope_append_vec(a, nullptr, batch, reinterpret_cast<cudaStream_t>(stream));
  if (vrc != 1) return vrc;
  // Each side iterates over its own element count; the shorter one exits early.
  a.units = units;
  AppendArgs per[2] = {a, a};
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  for (int i = 0; i < 2; ++i) {
    if (!a.side[i].x) continue;
    per[i].side[0] = a.side[i];
    per[i].units = batch * a.side[i].S * (int64_t)a.side[i].H * a.side[i].D;
    if (per[i].units == 0) continue;
    append_kernel<<<dim3(grid_for(per[i].units), 1), 256, 0, st>>>(per[i]);
    note_launch();
    FAB_LAUNCH_CHECK("append_kvcache launch");
  }
  return FA_OK;
}

extern "C" int fa_rotary_append_kvcache(const fa_tensor* q, const fa_tensor* q_out,
                                        const fa_tensor* key, const fa_tensor* value,
                                        const fa_tensor* k_cache, const fa_tensor* v_cache,
                                        const fa_tensor* lengths, const fa_tensor* cache_batch_idx,
                                        const fa_tensor* block_table,
                                        const fa_tensor* k_scale, const fa_tensor* v_scale,
                                        const fa_tensor* cos, const fa_tensor* sin,
                                        int32_t interleaved, int32_t advance_q, void* stream) {
  FAB_CHECK_ARG(present(lengths) && lengths->dtype == FA_I32 && lengths->ndim == 1,
                "lengths must be int32 [B]");
  const int64_t batch = lengths->shape[0];
  FAB_CHECK_ARG(present(key) && present(value), "rotary append needs new k and v");
  AppendArgs a{};
  int rc = prepare_append_side(key, k_cache, k_scale, batch, &a.side[0]);
  if (rc) return rc;
  rc = prepare_append_side(value, v_cache, v_scale, batch, &a.side[1]);
  if (rc) return rc;
  FAB_CHECK_ARG(present(cos) && present(sin) && cos->ndim == 2 && sin->ndim == 2 && is_float(cos->dtype) &&
                    sin->dtype == cos->dtype && cos->shape[0] == sin->shape[0] && cos->shape[1] == sin->shape[1],
                "rotary cosine/sine must be float [positions, rotary_dim/2] of one dtype");
  FAB_CHECK_ARG(cos->shape[1] * 2 <= key->shape[3], "rotary dimension exceeds head dimension");
  a.lengths = reinterpret_cast<const int32_t*>(lengths->ptr);
  a.len_stride = lengths->stride[0];
  a.paged = present(block_table);
  a.remap = !a.paged && present(cache_batch_idx);
  if (a.remap) {
    FAB_CHECK_ARG(cache_batch_idx->dtype == FA_I32 && cache_batch_idx->ndim == 1 &&
                      cache_batch_idx->shape[0] == batch, "cache_batch_idx must be int32 [B]");
    a.batch_idx = reinterpret_cast<const int32_t*>(cache_batch_idx->ptr);
    a.bi_stride = cache_batch_idx->stride[0];
  }
  if (a.paged) {
    FAB_CHECK_ARG(block_table->dtype == FA_I32 && block_table->ndim == 2,
                  "block_table must have shape [cache_batch, blocks_per_sequence]");
    a.table = reinterpret_cast<const int32_t*>(block_table->ptr);
    a.bt0 = block_table->stride[0];
    a.bt1 = block_table->stride[1];
    a.pages_per_seq = (int32_t)block_table->shape[1];
    a.rows = block_table->shape[0];
  } else {
    a.rows = k_cache->shape[0];
  }
  a.P = (int32_t)k_cache->shape[1];
  a.blocks = k_cache->shape[0];
  RopeArgs r{};
  r.cos = cos->ptr; r.sin = sin->ptr; r.cdtype = cos->dtype;
  r.cs0 = cos->stride[0]; r.cs1 = cos->stride[1]; r.ss0 = sin->stride[0]; r.ss1 = sin->stride[1];
  r.half = (int32_t)cos->shape[1];
  r.interleaved = interleaved; r.advance_q = advance_q;
  r.batch = batch;
  int64_t units = 0;
  for (int i = 0; i < 2; ++i) {
    const int64_t n = batch * a.side[i].S * (int64_t)a.side[i].H * a.side[i].D;
    units = n > units ? n : units;
  }
  int sides = 2;
  if (present(q)) {
    FAB_CHECK_ARG(present(q_out) && q->ndim == 4 && q_out->ndim == 4 && q->shape[0] == batch &&
                      q->dtype == q_out->dtype && is_float(q->dtype),
                  "q and q_out must be float [B,S,H,D] of one dtype");
    for (int i = 0; i < 4; ++i) FAB_CHECK_ARG(q->shape[i] == q_out->shape[i], "q_out must match q");
    FAB_CHECK_ARG(cos->shape[1] * 2 <= q->shape[3], "rotary dimension exceeds head dimension");
    r.q = q->ptr; r.q_out = q_out->ptr; r.qdtype = q->dtype;
    r.QS = (int32_t)q->shape[1]; r.QH = (int32_t)q->shape[2]; r.QD = (int32_t)q->shape[3];
    for (int i = 0; i < 4; ++i) { (&r.qs0)[i] = q->stride[i]; (&r.qo0)[i] = q_out->stride[i]; }
    r.q_units = batch * r.QS * (int64_t)r.QH * r.QD;
    units = r.q_units > units ? r.q_units : units;
    sides = 3;
  }
  if (units == 0) return FA_OK;
  const int vrc = launch_rope_append_vec(a, &r, batch, reinterpret_cast<cudaStream_t>(stream));
  if (vrc != 1) return vrc;
  rotary_append_kernel<<<dim3(grid_for(units), sides), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a, r);
  note_launch();
  FAB_LAUNCH_CHECK("rotary append launch");
  return FA_OK;
}

extern "C" int fa_rotary(const fa_tensor* x, const fa_tensor* out, const fa_tensor* cos,
                         const fa_tensor* sin, const fa_tensor* lengths, int32_t interleaved,
                         int32_t advance, void* stream) {
  FAB_CHECK_ARG(present(x) && present(out) && x->ndim == 4 && out->ndim == 4,
                "Q/K must have shape [batch, tokens, heads, dim]");
  for (int i = 0; i < 4; ++i) FAB_CHECK_ARG(x->shape[i] == out->shape[i], "out must match x");
  FAB_CHECK_ARG(x->dtype == out->dtype && is_float(x->dtype), "x/out must share a float dtype");
  FAB_CHECK_ARG(present(cos) && present(sin) && cos->ndim == 2 && sin->ndim == 2 &&
                    cos->dtype == FA_F32 && sin->dtype == FA_F32 &&
                    cos->shape[0] == sin->shape[0] && cos->shape[1] == sin->shape[1],
                "rotary cosine/sine must be float32 [positions, rotary_dim/2]");
  FAB_CHECK_ARG(cos->shape[1] * 2 <= x->shape[3], "rotary dimension exceeds head dimension");
  FAB_CHECK_ARG(present(lengths) && lengths->dtype == FA_I32 && lengths->ndim == 1 &&
                    lengths->shape[0] == x->shape[0], "lengths must be int32 [B]");
  RotaryArgs a{};
  a.x = x->ptr; a.out = out->ptr;
  for (int i = 0; i < 4; ++i) { (&a.xs0)[i] = x->stride[i]; (&a.os0)[i] = out->stride[i]; }
  a.cos = reinterpret_cast<const float*>(cos->ptr);
  a.sin = reinterpret_cast<const float*>(sin->ptr);
  a.cs0 = cos->stride[0]; a.cs1 = cos->stride[1]; a.ss0 = sin->stride[0]; a.ss1 = sin->stride[1];
  a.lengths = reinterpret_cast<const int32_t*>(lengths->ptr);
  a.len_stride = lengths->stride[0];
  a.S = (int32_t)x->shape[1]; a.H = (int32_t)x->shape[2]; a.D = (int32_t)x->shape[3];
  a.half = (int32_t)cos->shape[1];
  a.interleaved = interleaved; a.advance = advance; a.dtype = x->dtype;
  a.units = x->shape[0] * x->shape[1] * x->shape[2] * x->shape[3];
  if (a.units == 0) return FA_OK;
  rotary_kernel<<<grid_for(a.units), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  note_launch();
  FAB_LAUNCH_CHECK("rotary launch");
  return FA_OK;
}
