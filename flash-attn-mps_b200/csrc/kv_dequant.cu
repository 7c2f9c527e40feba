// Exact E4M3 -> 16-bit K/V copy in front of the tensor-core prefill.
//
// Prefill over an FP8 E4M3 K/V cache (vLLM's FP8 KV cache with chunked
// prefill) runs the tcgen05 prefill on 16-bit operands: every E4M3 value is
// exactly representable in f16 and in bf16 (4-bit exponent, 3-bit mantissa),
// so the K/V rows a call reads are decoded once -- by the hardware
// cvt.rn.f16x2.e4m3x2, then widened and repacked for bf16 queries -- into a
// contiguous [rows, Hkv, D] buffer in the caller's workspace. Packed K/V keep
// their row numbering (the prefill's cu_seqlens_k / seqused_k still apply);
// paged K/V are gathered per request into rows b * max_k + t, with row starts
// and lengths clipped to max_k written beside them. The k/v descales stay
// where the reference applies them (scores and output: attention.metal:84-86),
// inside the prefill kernel. NaN codes (0x7F/0xFF) decode to NaN, like the
// reference's read_decode (attention_decode.metal:9-16).
#include "kernels.cuh"
#include "ptx.cuh"

#ifndef FAB_FP8_PREFILL_MAX_COPY
// Largest 16-bit K+V copy (bytes) the route allocates in the workspace; larger
// calls (long paged contexts x many requests) keep reading the FP8 bytes on
// the mma.sync kernel instead of asking the caller for gigabytes per call.
#define FAB_FP8_PREFILL_MAX_COPY (4LL << 30)
#endif

namespace fab {
namespace {

struct DequantArgs {
  const uint8_t* src[2];               // K, V (E4M3 bytes)
  int64_t s0[2], s1[2], s2[2];         // byte strides: paged (page, token, head), packed (-, row, head)
  uint8_t* dst[2];                     // 16-bit [rows, HK, D], contiguous
  const int32_t* cu_k; int64_t ck0;    // optional
  const int32_t* used; int64_t u0;     // optional
  const int32_t* table; int64_t bt0, bt1;
  int32_t* cu_out; int32_t* used_out;  // paged: b * max_k and min(len_b, max_k)
  int64_t rows, k_pages;
  int32_t HK, D, vpr, paged, page, pshift, bt_cols, max_k, B, bf16;
};

__device__ __forceinline__ int seq_len(const DequantArgs& a, int64_t b) {
  return a.used ? a.used[b * a.u0] : a.cu_k[(b + 1) * a.ck0] - a.cu_k[b * a.ck0];
}

// 16 E4M3 bytes -> 16 exact 16-bit values (two 16-byte vectors).
__device__ __forceinline__ void decode16(const uint4& in, bool bf16, uint4& lo, uint4& hi) {
  const uint32_t w[4] = {in.x, in.y, in.z, in.w};
  uint32_t h[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) e4m3x4_to_f16x2x2(w[i], h[2 * i], h[2 * i + 1]);
  if (bf16) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h[i]));
      const __nv_bfloat162 b = __floats2bfloat162_rn(f.x, f.y);  // exact: E4M3 values fit bf16
      h[i] = *reinterpret_cast<const uint32_t*>(&b);
    }
  }
  lo = make_uint4(h[0], h[1], h[2], h[3]);
  hi = make_uint4(h[4], h[5], h[6], h[7]);
}

__global__ void __launch_bounds__(256) kv_dequant_kernel(DequantArgs a) {
  const int side = blockIdx.y;
  const uint8_t* src = a.src[side];
  uint8_t* dst = a.dst[side];
  const int per_head = a.D / 16;
  const int64_t total = a.rows * a.vpr;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += step) {
    const int64_t r = e / a.vpr;
    const int c = (int)(e - r * a.vpr);
    const int h = c / per_head, d = (c - h * per_head) * 16;
    int64_t off = -1;
    if (a.paged) {
      const int64_t b = r / a.max_k;
      const int t = (int)(r - b * a.max_k);
      // Rows past the sequence are left unwritten: the prefill masks their
      // scores and zeroes their V rows before they meet a probability.
      if (t >= min(seq_len(a, b), a.max_k)) continue;
      const int pg = a.pshift >= 0 ? t >> a.pshift : t / a.page;
      const int64_t blk = pg < a.bt_cols ? (int64_t)a.table[b * a.bt0 + (int64_t)pg * a.bt1] : -1;
      // A page outside the cache reads as zeros (the TMA gathers' fill value).
      if (blk >= 0 && blk < a.k_pages)
        off = blk * a.s0[side] + (int64_t)(t - pg * a.page) * a.s1[side] + h * a.s2[side] + d;
    } else {
      off = r * a.s1[side] + h * a.s2[side] + d;
    }
    uint4 lo = make_uint4(0, 0, 0, 0), hi = lo;
    if (off >= 0) decode16(__ldg(reinterpret_cast<const uint4*>(src + off)), a.bf16, lo, hi);
    uint4* out = reinterpret_cast<uint4*>(dst + ((r * a.HK + h) * a.D + d) * 2);
    out[0] = lo;
    out[1] = hi;
  }
  if (a.paged && side == 0 && blockIdx.x == 0) {
    for (int b = threadIdx.x; b <= a.B; b += blockDim.x) {
      a.cu_out[b] = b * a.max_k;
      if (b < a.B) a.used_out[b] = min(seq_len(a, b), a.max_k);
    }
  }
}

int log2_or_minus1(int v) {
  if (v <= 0 || (v & (v - 1))) return -1;
  int k = 0;
  while ((1 << k) < v) ++k;
  return k;
}

}  // namespace

int64_t fp8_prefill_rows(const AttnParams& p) {
  return p.paged ? (int64_t)p.B * p.max_k : p.k_rows;
}

bool fp8_prefill_view(const AttnParams& p, AttnParams* view) {
  if (p.kt != FA_E4M3 || p.vt != FA_E4M3 || !(p.qt == FA_BF16 || p.qt == FA_F16)) return false;
  if (p.DQ != p.DV || p.DQ % 16 || p.DQ < 16 || p.DQ > 128) return false;
  if (p.ks3 != 1 || p.vs3 != 1 || p.max_k <= 0 || p.HK <= 0) return false;
  if (((uintptr_t)p.k & 15u) || ((uintptr_t)p.v & 15u)) return false;
  const int64_t st[6] = {p.paged ? p.ks0 : 16, p.ks1, p.ks2, p.paged ? p.vs0 : 16, p.vs1, p.vs2};
  for (int64_t s : st)
    if (s <= 0 || s % 16) return false;
  if (p.paged && (p.page <= 0 || p.k_pages <= 0 || p.bt_cols <= 0)) return false;
  const int64_t rows = fp8_prefill_rows(p);
  if (rows <= 0 || rows >= (1 << 30)) return false;
  if (2 * rows * p.HK * p.DQ * 2 > (int64_t)FAB_FP8_PREFILL_MAX_COPY) return false;
  AttnParams v = p;
  v.kt = v.vt = p.qt;
  v.ks0 = v.vs0 = 0;
  v.ks1 = v.vs1 = (int64_t)p.HK * p.DQ;
  v.ks2 = v.vs2 = p.DQ;
  v.ks3 = v.vs3 = 1;
  v.paged = 0;
  v.page = 0;
  v.k_rows = rows;
  v.k_pages = 0;
  v.table = nullptr;
  v.bt_cols = 0;
  // Placeholders until the workspace is carved (only alignment is checked).
  v.k = v.v = reinterpret_cast<const void*>(uintptr_t(256));
  if (!prefill_sm100_supported(v)) return false;
  *view = v;
  return true;
}

int launch_kv_dequant(const AttnParams& p, void* k_out, void* v_out, int32_t* cu_out, int32_t* used_out,
                      cudaStream_t stream) {
  DequantArgs a{};
  a.src[0] = reinterpret_cast<const uint8_t*>(p.k);
  a.src[1] = reinterpret_cast<const uint8_t*>(p.v);
  a.s0[0] = p.ks0; a.s1[0] = p.ks1; a.s2[0] = p.ks2;
  a.s0[1] = p.vs0; a.s1[1] = p.vs1; a.s2[1] = p.vs2;
  a.dst[0] = reinterpret_cast<uint8_t*>(k_out);
  a.dst[1] = reinterpret_cast<uint8_t*>(v_out);
  a.cu_k = p.cu_k; a.ck0 = p.ck0;
  a.used = p.used; a.u0 = p.u0;
  a.table = p.table; a.bt0 = p.bt0; a.bt1 = p.bt1;
  a.cu_out = cu_out; a.used_out = used_out;
  a.rows = fp8_prefill_rows(p);
  a.k_pages = p.k_pages;
  a.HK = p.HK; a.D = p.DQ; a.vpr = p.HK * p.DQ / 16;
  a.paged = p.paged; a.page = p.page; a.pshift = log2_or_minus1(p.page);
  a.bt_cols = (int32_t)p.bt_cols; a.max_k = p.max_k; a.B = p.B;
  a.bf16 = p.qt == FA_BF16;
  if (a.paged && (cu_out == nullptr || used_out == nullptr))
    return fail(FA_ERR_INVALID, "FP8 prefill needs its row-start and length buffers");
  const int64_t vectors = a.rows * a.vpr;
  int64_t blocks = (vectors + 255) / 256;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  kv_dequant_kernel<<<dim3((unsigned)blocks, 2), 256, 0, stream>>>(a);
  note_launch();
  FAB_LAUNCH_CHECK("FP8 K/V dequant launch");
  return FA_OK;
}

}  // namespace fab
