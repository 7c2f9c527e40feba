// Tensor-core attention (mma.sync m16n8k16, fp32 accumulation) for the
// f16/bf16 cases that neither the tcgen05 prefill nor the paged-decode kernel
// takes: FP8 E4M3 K/V in prefill, head dims 96 and 256, DiffKV 192->128, ALiBi,
// mask kinds 1/2, leftpad, explicit split counts, q_len = 1 with those
// features. fp32 inputs keep the SIMT generic kernel (fp32 exactness).
//
// One CTA = 64 query rows (4 warps x 16) of one (request, query head, split).
// K/V tiles of 64 keys are gathered (packed rows or block_table pages, leftpad
// applied) with 16-byte cp.async into a 2-stage shared ring, rows padded by
// 16 bytes so that ldmatrix is conflict-free; keys past the sequence are
// zero-filled. FP8 tiles are converted exactly to the query's 16-bit type in
// shared memory (E4M3 values are representable in f16 and bf16). S = Q K^T on
// tensor cores; every score gets the reference's features in its order (scale,
// softcap, ALiBi, allowed_key: causal / windows / masks) and the online softmax
// in the log2 domain; P stays in registers as the A operand of O += P V
// (V fragments through ldmatrix.trans). Sinks seed split 0; descales fold
// into the scale (q, k) and the output (v). Semantics follow
// flash_attn_mps/kernels/attention.metal:29-51 (allowed_key, attention_score)
// and 60-181 (tile bounds per split, LSE).
#include <type_traits>

#include "features.cuh"
#include "kernels.cuh"
#include "ptx.cuh"

namespace fab {
namespace {

constexpr int kBM = 64;  // query rows per CTA
constexpr int kBN = 64;  // keys per tile
constexpr int kThreads = 128;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

template <typename T> __device__ __forceinline__ T from_float(float x);
template <> __device__ __forceinline__ __half from_float<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// Eight E4M3 bytes -> eight exact 16-bit values of type T.
template <typename T>
__device__ __forceinline__ uint4 e4m3x8_to(uint2 raw) {
  uint32_t h[4];
  e4m3x4_to_f16x2x2(raw.x, h[0], h[1]);
  e4m3x4_to_f16x2x2(raw.y, h[2], h[3]);
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h[i]));
      h[i] = pack2<__nv_bfloat16>(f.x, f.y);
    }
  }
  return make_uint4(h[0], h[1], h[2], h[3]);
}

template <bool KV8, int DQ, int DV>
struct Layout {
  static constexpr int kQStride = DQ + 8;  // elements (16-byte row padding)
  static constexpr int kKStride = DQ + 8;
  static constexpr int kVStride = DV + 8;
  static constexpr int kQBytes = kBM * kQStride * 2;
  static constexpr int kKBytes = kBN * kKStride * 2;
  static constexpr int kVBytes = kBN * kVStride * 2;
  static constexpr int kRawKStride = DQ + 16;  // bytes, FP8 staging rows
  static constexpr int kRawVStride = DV + 16;
  static constexpr int kRawKBytes = KV8 ? kBN * kRawKStride : kKBytes;
  static constexpr int kRawVBytes = KV8 ? kBN * kRawVStride : kVBytes;
  static constexpr int kStageBytes = kRawKBytes + kRawVBytes;
  static constexpr int kConvBytes = KV8 ? kKBytes + kVBytes : 0;
  static constexpr int kSmem = kQBytes + 2 * kStageBytes + kConvBytes;
};

// PREC (fp32 outputs): P = hi + lo in two 16-bit halves, two PV MMAs, so the
// probabilities keep ~16 (bf16) / ~22 (f16) bits as an fp32 reference expects.
// SIMPLE: no ALiBi, softcap or mask descriptor (causal, windows, lengths
// only): scores are scaled in one multiply and masked only in warp tiles that
// straddle a causal / window / length edge.
template <typename T, bool KV8, int DQ, int DV, bool PREC, bool SIMPLE>
__global__ void __launch_bounds__(kThreads) mma_attention_kernel(const AttnParams p) {
  using L = Layout<KV8, DQ, DV>;
  constexpr bool kQRegs = DQ <= 128;  // Q fragments kept in registers
  constexpr int esz = KV8 ? 1 : 2;
  extern __shared__ __align__(128) uint8_t smem[];
  T* qs = reinterpret_cast<T*>(smem);
  uint8_t* stage0 = smem + L::kQBytes;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, qd = lane & 3;
  const int b = blockIdx.z / p.splits, split = blockIdx.z % p.splits;
  const int h = blockIdx.y, kh = h / (p.HQ / p.HK);
  const int q_begin = p.cu_q[b * p.cq0];
  const int q_len = p.cu_q[(b + 1) * p.cq0] - q_begin;
  const int q_block = blockIdx.x * kBM;
  if (q_block >= q_len) return;
  const int k_cu_begin = p.cu_k ? p.cu_k[b * p.ck0] : 0;
  const int k_begin = p.paged ? 0 : k_cu_begin;
  const int k_len = p.used ? p.used[b * p.u0] : p.cu_k[(b + 1) * p.ck0] - k_cu_begin;
  const int left = p.leftpad ? p.leftpad[b * p.lp0] : 0;
  const bool causal = p.dynamic ? p.causal_b[b * p.ca0] != 0 : p.causal != 0;
  const float scale = p.scale * (p.qd ? p.qd[b * p.qd0 + kh * p.qd1] : 1.f) *
                      (p.kd ? p.kd[b * p.kd0 + kh * p.kd1] : 1.f);
  const float vscale = p.vd ? p.vd[b * p.vd0 + kh * p.vd1] : 1.f;
  const float slope = p.alibi ? p.alibi[b * p.a0 + h * p.a1] : 0.f;
  const float sink = (p.sinks && split == 0 && p.cp_r == 0) ? load_float(p.sinks, p.sink_t, h * p.si0) : -INFINITY;
  const int k_tot = kv_total(p, b, k_len);  // global KV length (context parallelism)

  // Tile bounds of this split (attention.metal:108-118, 64-key tiles).
  const int tile_count = (k_len + kBN - 1) / kBN;
  int first = (int)((int64_t)tile_count * split / p.splits);
  int last = (int)((int64_t)tile_count * (split + 1) / p.splits);
  const int row_end = min(q_block + kBM, q_len);
  if (p.cp_n <= 1) {  // tile skipping in local positions (positions are strided under context parallelism)
    if (causal && p.mask == 0) last = min(last, max(0, (row_end + k_len - q_len + kBN - 1) / kBN));
    if (p.mask == 0 && p.win_l >= 0) first = max(first, max(0, q_block + k_len - q_len - p.win_l) / kBN);
    if (p.mask == 0 && p.win_r >= 0) last = min(last, max(0, (row_end + k_len - q_len + p.win_r + kBN - 1) / kBN));
  }

  auto load_tile = [&](int kb, int st) {
    uint8_t* kdst = stage0 + st * L::kStageBytes;
    uint8_t* vdst = kdst + L::kRawKBytes;
    constexpr int kChK = DQ * esz / 16, kChV = DV * esz / 16;
    constexpr int kRowK = KV8 ? L::kRawKStride : L::kKStride * 2;
    constexpr int kRowV = KV8 ? L::kRawVStride : L::kVStride * 2;
    for (int z = tid; z < kBN * kChK; z += kThreads) {
      const int r = z / kChK, c = z - r * kChK, t = kb * kBN + r;
      const bool ok = t < k_len;
      const int64_t off = ok ? kv_offset(p, b, (int64_t)k_begin + left + t, kh, false) : 0;
      cp_async_16(smem_u32(kdst + r * kRowK + c * 16), reinterpret_cast<const uint8_t*>(p.k) + off * esz + c * 16,
                  ok ? 16 : 0);
    }
    for (int z = tid; z < kBN * kChV; z += kThreads) {
      const int r = z / kChV, c = z - r * kChV, t = kb * kBN + r;
      const bool ok = t < k_len;
      const int64_t off = ok ? kv_offset(p, b, (int64_t)k_begin + left + t, kh, true) : 0;
      cp_async_16(smem_u32(vdst + r * kRowV + c * 16), reinterpret_cast<const uint8_t*>(p.v) + off * esz + c * 16,
                  ok ? 16 : 0);
    }
  };

  if (first < last) load_tile(first, 0);
  cp_async_commit();

  // Q tile -> shared memory (rows past the sequence are zero).
  for (int z = tid; z < kBM * DQ; z += kThreads) {
    const int r = z / DQ, d = z - r * DQ;
    const float x = q_block + r < q_len
                        ? load_float(p.q, p.qt,
                                     (int64_t)(q_begin + q_block + r) * p.qs0 + (int64_t)h * p.qs1 + (int64_t)d * p.qs2)
                        : 0.f;
    qs[r * L::kQStride + d] = from_float<T>(x);
  }
  __syncthreads();
  auto q_frag = [&](int kk, uint32_t (&a)[4]) {
    const int r = warp * 16 + (lane & 15), c = kk * 16 + (lane >> 4) * 8;
    ldsm_x4(smem_u32(qs + r * L::kQStride + c), a[0], a[1], a[2], a[3]);
  };
  uint32_t qf[kQRegs ? DQ / 16 : 1][4];
  if constexpr (kQRegs) {
#pragma unroll
    for (int kk = 0; kk < DQ / 16; ++kk) q_frag(kk, qf[kk]);
  }

  float o[DV / 8][4];
#pragma unroll
  for (int n = 0; n < DV / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  const float sink_l2 = sink * kLog2e;
  float m[2] = {sink_l2, sink_l2};
  float l[2];
  l[0] = l[1] = (isfinite(sink) && qd == 0) ? 1.f : 0.f;  // the sink counts once per row

  for (int kb = first; kb < last; ++kb) {
    const int st = (kb - first) & 1;
    if (kb + 1 < last) load_tile(kb + 1, st ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const T* ks;
    const T* vs;
    if constexpr (KV8) {
      // Exact E4M3 -> T conversion of this stage into the single converted tile.
      const uint8_t* kraw = stage0 + st * L::kStageBytes;
      const uint8_t* vraw = kraw + L::kRawKBytes;
      T* kc = reinterpret_cast<T*>(stage0 + 2 * L::kStageBytes);
      T* vc = kc + kBN * L::kKStride;
      for (int z = tid; z < kBN * DQ / 8; z += kThreads) {
        const int r = z / (DQ / 8), c = z - r * (DQ / 8);
        *reinterpret_cast<uint4*>(kc + r * L::kKStride + c * 8) =
            e4m3x8_to<T>(*reinterpret_cast<const uint2*>(kraw + r * L::kRawKStride + c * 8));
      }
      for (int z = tid; z < kBN * DV / 8; z += kThreads) {
        const int r = z / (DV / 8), c = z - r * (DV / 8);
        *reinterpret_cast<uint4*>(vc + r * L::kVStride + c * 8) =
            e4m3x8_to<T>(*reinterpret_cast<const uint2*>(vraw + r * L::kRawVStride + c * 8));
      }
      __syncthreads();
      ks = kc;
      vs = vc;
    } else {
      ks = reinterpret_cast<const T*>(stage0 + st * L::kStageBytes);
      vs = reinterpret_cast<const T*>(stage0 + st * L::kStageBytes + L::kRawKBytes);
    }

    // S = Q K^T for this warp's 16 rows x 64 keys.
    float s[kBN / 8][4];
#pragma unroll
    for (int n = 0; n < kBN / 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < DQ / 16; ++kk) {
      uint32_t a[4];
      if constexpr (kQRegs) {
        a[0] = qf[kk][0]; a[1] = qf[kk][1]; a[2] = qf[kk][2]; a[3] = qf[kk][3];
      } else {
        q_frag(kk, a);
      }
#pragma unroll
      for (int np = 0; np < kBN / 16; ++np) {
        uint32_t b0, b1, b2, b3;
        const int r = np * 16 + (lane & 7) + ((lane >> 4) << 3), c = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(smem_u32(ks + r * L::kKStride + c), b0, b1, b2, b3);
        mma16816<T>(s[2 * np], a, b0, b1);
        mma16816<T>(s[2 * np + 1], a, b2, b3);
      }
    }

    // Scores with the reference's features, then the online softmax (log2).
    float mx[2] = {-INFINITY, -INFINITY};
    if constexpr (SIMPLE) {
      // Visible keys of the warp's first and last row; the tile needs no
      // per-element test when every (row, key) pair is visible.
      const int q_lo = q_block + warp * 16, q_hi = min(q_lo + 15, q_len - 1);
      const int off = k_len - q_len, key0 = kb * kBN, key1 = key0 + kBN - 1;
      bool full = q_hi >= q_lo && key1 < k_len;
      if (causal) full = full && key1 <= q_lo + off;
      if (p.win_r >= 0) full = full && key1 <= q_lo + off + p.win_r;
      if (p.win_l >= 0) full = full && key0 >= q_hi + off - p.win_l;
      const float sl2 = scale * kLog2e;
#pragma unroll
      for (int n = 0; n < kBN / 8; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int row = e >> 1;
          float x = s[n][e] * sl2;
          if (!full) {
            const int q = q_block + warp * 16 + g + 8 * row;
            const int t = key0 + n * 8 + 2 * qd + (e & 1);
            const int diff = q + off - t;
            const bool keep = q < q_len && t < k_len && (!causal || diff >= 0) &&
                              (p.win_l < 0 || diff <= p.win_l) && (p.win_r < 0 || -diff <= p.win_r);
            x = keep ? x : -INFINITY;
          }
          s[n][e] = x;
          mx[row] = fmaxf(mx[row], x);
        }
      }
    } else {
#pragma unroll
      for (int n = 0; n < kBN / 8; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int row = e >> 1;
          const int q = q_block + warp * 16 + g + 8 * row;
          const int t = kb * kBN + n * 8 + 2 * qd + (e & 1), tg = key_pos(p, t);
          const int q_abs = q + k_tot - q_len;
          float x = s[n][e] * scale;
          if (p.softcap > 0.f) x = p.softcap * tanhf(x / p.softcap);
          x -= slope * fabsf((float)(q_abs - tg));
          const bool keep = q < q_len && t < k_len && allowed_key(p, b, tg, q_abs, (int64_t)q_begin + q, causal);
          x = keep ? x * kLog2e : -INFINITY;
          s[n][e] = x;
          mx[row] = fmaxf(mx[row], x);
        }
      }
    }
    float factor[2], nsafe[2];
#pragma unroll
    for (int row = 0; row < 2; ++row) {
      mx[row] = fmaxf(mx[row], __shfl_xor_sync(0xffffffffu, mx[row], 1));
      mx[row] = fmaxf(mx[row], __shfl_xor_sync(0xffffffffu, mx[row], 2));
      const float mn = fmaxf(m[row], mx[row]);
      nsafe[row] = mn == -INFINITY ? 0.f : mn;
      factor[row] = ex2f(m[row] - nsafe[row]);  // 0 when m was -inf
      m[row] = mn;
      l[row] *= factor[row];
    }
#pragma unroll
    for (int n = 0; n < DV / 8; ++n) {
      o[n][0] *= factor[0]; o[n][1] *= factor[0];
      o[n][2] *= factor[1]; o[n][3] *= factor[1];
    }
#pragma unroll
    for (int n = 0; n < kBN / 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float pe = ex2f(s[n][e] - nsafe[e >> 1]);
        s[n][e] = pe;
        l[e >> 1] += pe;
      }
    }

    // O += P V: P (C layout of S) is the A operand, 16 keys per MMA.
#pragma unroll
    for (int kk = 0; kk < kBN / 16; ++kk) {
      uint32_t a[4], alo[4];
      a[0] = pack2<T>(s[2 * kk][0], s[2 * kk][1]);
      a[1] = pack2<T>(s[2 * kk][2], s[2 * kk][3]);
      a[2] = pack2<T>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      a[3] = pack2<T>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
      if constexpr (PREC) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 hi = unpack2<T>(a[i]);
          const float lo0 = s[2 * kk + (i >> 1)][(i & 1) * 2] - hi.x;
          const float lo1 = s[2 * kk + (i >> 1)][(i & 1) * 2 + 1] - hi.y;
          alo[i] = pack2<T>(lo0, lo1);
        }
      }
#pragma unroll
      for (int np = 0; np < DV / 16; ++np) {
        uint32_t b0, b1, b2, b3;
        const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, c = np * 16 + (lane >> 4) * 8;
        ldsm_x4_t(smem_u32(vs + r * L::kVStride + c), b0, b1, b2, b3);
        mma16816<T>(o[2 * np], a, b0, b1);
        mma16816<T>(o[2 * np + 1], a, b2, b3);
        if constexpr (PREC) {
          mma16816<T>(o[2 * np], alo, b0, b1);
          mma16816<T>(o[2 * np + 1], alo, b2, b3);
        }
      }
    }
    __syncthreads();  // every warp is done with this stage before it is refilled
  }
  cp_async_wait<0>();

  // Epilogue: row sums over the quad, normalisation, LSE (natural log).
#pragma unroll
  for (int row = 0; row < 2; ++row) {
    l[row] += __shfl_xor_sync(0xffffffffu, l[row], 1);
    l[row] += __shfl_xor_sync(0xffffffffu, l[row], 2);
  }
#pragma unroll
  for (int row = 0; row < 2; ++row) {
    const int q = q_block + warp * 16 + g + 8 * row;
    if (q >= q_len) continue;
    const int64_t t = (int64_t)q_begin + q;
    const float norm = l[row] > 0.f ? vscale / l[row] : 0.f;
    const float lse = l[row] > 0.f ? (m[row] + log2f(l[row])) * kLn2 : -INFINITY;
    if (p.splits == 1) {
#pragma unroll
      for (int n = 0; n < DV / 8; ++n) {
        const int d = n * 8 + 2 * qd;
        store_float(p.out, p.ot, t * p.os0 + (int64_t)h * p.os1 + (int64_t)d * p.os2, o[n][2 * row] * norm);
        store_float(p.out, p.ot, t * p.os0 + (int64_t)h * p.os1 + (int64_t)(d + 1) * p.os2, o[n][2 * row + 1] * norm);
      }
      if (qd == 0) p.lse[(int64_t)h * p.ls0 + t * p.ls1] = lse;
    } else {
      float* dst = p.part + (((int64_t)split * p.T + t) * p.HQ + h) * DV;
#pragma unroll
      for (int n = 0; n < DV / 8; ++n) {
        const int d = n * 8 + 2 * qd;
        *reinterpret_cast<float2*>(dst + d) = make_float2(o[n][2 * row] * norm, o[n][2 * row + 1] * norm);
      }
      if (qd == 0) p.part_lse[((int64_t)split * p.HQ + h) * p.T + t] = lse;
    }
  }
}

template <typename T, bool KV8, int DQ, int DV>
int launch_shape(const AttnParams& p, cudaStream_t stream) {
  constexpr int smem = Layout<KV8, DQ, DV>::kSmem;
  const bool simple = p.alibi == nullptr && p.softcap <= 0.f && p.mask == 0 && p.cp_n <= 1;
  auto kernel = p.ot == FA_F32 ? mma_attention_kernel<T, KV8, DQ, DV, true, false>
                : simple       ? mma_attention_kernel<T, KV8, DQ, DV, false, true>
                               : mma_attention_kernel<T, KV8, DQ, DV, false, false>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return fail(FA_ERR_CUDA, "mma attention smem attribute: %s", cudaGetErrorString(e));
  dim3 grid((unsigned)((p.max_q + kBM - 1) / kBM), (unsigned)p.HQ, (unsigned)((int64_t)p.B * p.splits));
  kernel<<<grid, kThreads, smem, stream>>>(p);
  note_launch();
  FAB_LAUNCH_CHECK("mma attention launch");
  return FA_OK;
}

template <typename T, bool KV8>
int launch_dims(const AttnParams& p, cudaStream_t stream) {
  if (p.DQ == 64 && p.DV == 64) return launch_shape<T, KV8, 64, 64>(p, stream);
  if (p.DQ == 96 && p.DV == 96) return launch_shape<T, KV8, 96, 96>(p, stream);
  if (p.DQ == 128 && p.DV == 128) return launch_shape<T, KV8, 128, 128>(p, stream);
  if (p.DQ == 192 && p.DV == 128) return launch_shape<T, KV8, 192, 128>(p, stream);
  if (p.DQ == 256 && p.DV == 256) return launch_shape<T, KV8, 256, 256>(p, stream);
  return fail(FA_ERR_UNSUPPORTED, "mma attention: head dims %d/%d", p.DQ, p.DV);
}

bool dims_ok(int dq, int dv) {
  return (dq == dv && (dq == 64 || dq == 96 || dq == 128 || dq == 256)) || (dq == 192 && dv == 128);
}

bool al16(const void* ptr) { return ((uintptr_t)ptr & 15u) == 0; }

}  // namespace

int mma_attention_supported(const AttnParams& p) {
  if (p.qt != FA_F16 && p.qt != FA_BF16) return 0;
  const bool kv8 = p.kt == FA_E4M3 && p.vt == FA_E4M3;
  if (!kv8 && (p.kt != p.qt || p.vt != p.qt)) return 0;
  if (!dims_ok(p.DQ, p.DV)) return 0;
  if (p.ks3 != 1 || p.vs3 != 1) return 0;
  if (!al16(p.k) || !al16(p.v)) return 0;
  const int64_t elt = kv8 ? 1 : 2;
  const int64_t st[6] = {p.ks0, p.ks1, p.ks2, p.vs0, p.vs1, p.vs2};
  for (int i = 0; i < 6; ++i) {
    if (!p.paged && (i == 0 || i == 3)) continue;
    if ((st[i] * elt) % 16 != 0) return 0;
  }
  if (p.HQ > 65535 || (int64_t)p.B * p.splits > 65535) return 0;
  return 1;
}

int launch_mma_attention(const AttnParams& p, cudaStream_t stream) {
  const bool kv8 = p.kt == FA_E4M3;
  if (p.qt == FA_BF16)
    return kv8 ? launch_dims<__nv_bfloat16, true>(p, stream) : launch_dims<__nv_bfloat16, false>(p, stream);
  return kv8 ? launch_dims<__half, true>(p, stream) : launch_dims<__half, false>(p, stream);
}

}  // namespace fab
