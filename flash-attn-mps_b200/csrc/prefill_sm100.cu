// Varlen / dense prefill on 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// One CTA computes one 128-row query tile of one (request, query head):
//   warp 0      TMA producer: Q once, then K/V tiles of 128 keys into a
//               2-stage ring (128-byte swizzled boxes of 64 head dims).
//   warp 1      TMEM owner and MMA issuer: S = Q K^T and O += P V as
//               tcgen05.mma kind::f16 (M=128, N=128, K=16 per instruction),
//               fp32 accumulators S and O in TMEM (256 columns).
//   warps 2..5  softmax: each thread owns one query row (its TMEM lane),
//               loads its S row with tcgen05.ld, applies scale and the
//               lower-right causal / length masks, runs the online softmax
//               in the log2 domain, rescales its O row in TMEM when the row
//               max grows, and writes P (bf16/f16) into a 128-byte swizzled
//               shared tile that the next MMA reads as its A operand.
// The MMA warp issues S(j+1) as soon as the softmax warps have read S(j), so
// the QK^T of the next tile overlaps the exponentials of the current one.
// Every mbarrier wait is bounded; on a timeout the kernel records a flag,
// drains its own TMA loads and MMAs, frees TMEM and returns.
//
// Semantics (lower-right causal, natural-log LSE, zero output and -inf LSE
// for rows with no visible key) follow the reference's fast kernel
// flash_attn_mps/kernels/attention_fast.metal:94-597 and its eligibility
// predicate flash_attn_mps/_attention.py:231-240.
#include <cudaTypedefs.h>

#include <mutex>

#include "kernels.cuh"
#include "sm100.cuh"

namespace fab {
namespace {

using namespace sm100;

constexpr int BM = 128;          // query rows per tile
constexpr int BN = 128;          // keys per tile
constexpr int HD = 128;          // head dim
constexpr int NS = 2;            // K/V pipeline stages
constexpr int kRegion = 128 * 128;            // one 128-row x 64-element box (bytes)
constexpr int kTileBytes = 2 * kRegion;       // 128 x 128 bf16
constexpr int kThreads = 192;
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + kTileBytes;
constexpr int OFF_V = OFF_K + NS * kTileBytes;
constexpr int OFF_P = OFF_V + NS * kTileBytes;
constexpr int OFF_BAR = OFF_P + kTileBytes;
constexpr int kSmemBytes = OFF_BAR + 256 + 1024;
constexpr uint32_t kTmemCols = 256;
constexpr float kLn2 = 0.6931471805599453f;

enum { B_Q = 0, B_KVF = 1, B_KVE = B_KVF + NS, B_SF = B_KVE + NS, B_SE, B_PF, B_OD, B_FIN, B_COUNT };

__device__ int g_prefill_timeout;

struct PrefillParams {
  void* out; int64_t os0, os1;
  float* lse; int64_t ls0, ls1;
  const int32_t* cu_q; int64_t cq0;
  const int32_t* cu_k; int64_t ck0;
  const int32_t* used; int64_t u0;
  int32_t HQ, HK, n_qtiles, causal;
  float scale_log2;
};

__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity) {
  bool ok = mbar_wait(bar, parity, &g_prefill_timeout);
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

template <bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_sm100_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                         const __grid_constant__ CUtensorMap tv, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z, h = blockIdx.y;
  const int qt = p.n_qtiles - 1 - (int)blockIdx.x;  // longest causal tiles first
  const int q_begin = p.cu_q[b * p.cq0];
  const int q_len = p.cu_q[(b + 1) * p.cq0] - q_begin;
  if (qt * BM >= q_len) return;
  const int k_begin = p.cu_k ? p.cu_k[b * p.ck0] : 0;
  const int k_len = p.used ? p.used[b * p.u0] : p.cu_k[(b + 1) * p.ck0] - k_begin;
  const int kh = h / (p.HQ / p.HK);
  int n_tiles = (k_len + BN - 1) / BN;
  if (p.causal) {
    const int last_abs = min(qt * BM + BM, q_len) - 1 + k_len - q_len;
    n_tiles = last_abs < 0 ? 0 : min(n_tiles, last_abs / BN + 1);
  }
  auto bar = [&](int i) { return base + OFF_BAR + 8u * (uint32_t)i; };
  const uint32_t holder = base + OFF_BAR + 8u * B_COUNT;
  volatile uint32_t* holder_ptr = reinterpret_cast<volatile uint32_t*>(gbase + OFF_BAR + 8 * B_COUNT);

  if (threadIdx.x == 0) {
    mbar_init(bar(B_Q), 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(bar(B_KVF + s), 1);
      mbar_init(bar(B_KVE + s), 1);
    }
    mbar_init(bar(B_SF), 1);
    mbar_init(bar(B_SE), 128);
    mbar_init(bar(B_PF), 128);
    mbar_init(bar(B_OD), 1);
    mbar_init(bar(B_FIN), 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(holder, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *holder_ptr;
  const uint32_t tS = tmem, tO = tmem + 128;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    int issued = 0;
    if (n_tiles > 0) {
      if (lane == 0) {
        tma_prefetch_desc(&tq);
        tma_prefetch_desc(&tk);
        tma_prefetch_desc(&tv);
        mbar_expect_tx(bar(B_Q), kTileBytes);
        const int row = q_begin + qt * BM;
        tma_load_3d(base + OFF_Q, &tq, bar(B_Q), 0, h, row);
        tma_load_3d(base + OFF_Q + kRegion, &tq, bar(B_Q), 64, h, row);
      }
      for (int j = 0; j < n_tiles; ++j) {
        const int s = j % NS;
        if (j >= NS && !warp_wait(bar(B_KVE + s), ((j / NS) - 1) & 1)) break;
        if (lane == 0) {
          mbar_expect_tx(bar(B_KVF + s), 2 * kTileBytes);
          const int row = k_begin + j * BN;
          const uint32_t kd = base + OFF_K + s * kTileBytes, vd = base + OFF_V + s * kTileBytes;
          tma_load_3d(kd, &tk, bar(B_KVF + s), 0, kh, row);
          tma_load_3d(kd + kRegion, &tk, bar(B_KVF + s), 64, kh, row);
          tma_load_3d(vd, &tv, bar(B_KVF + s), 0, kh, row);
          tma_load_3d(vd + kRegion, &tv, bar(B_KVF + s), 64, kh, row);
        }
        issued = j + 1;
      }
      // Drain: the last loads of each stage must have landed before exit.
      warp_wait(bar(B_Q), 0);
      for (int j = max(0, issued - NS); j < issued; ++j) warp_wait(bar(B_KVF + j % NS), (j / NS) & 1);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (n_tiles > 0) {
      const uint32_t idesc_qk = f16_idesc(BM, BN, BF16 ? 1 : 0, 0);
      const uint32_t idesc_pv = f16_idesc(BM, HD, BF16 ? 1 : 0, 1);
      auto issue_pv = [&](int jj) -> bool {
        const int sp = jj % NS;
        if (!warp_wait(bar(B_PF), jj & 1)) return false;
        tc_fence_after();
        if (lane == 0) {
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const uint64_t a = sw128_desc(base + OFF_P + (kk >> 2) * kRegion + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = sw128_desc(base + OFF_V + sp * kTileBytes + kk * 2048, kRegion, 1024);
            mma_f16_ss(tO, a, bd, idesc_pv, (jj > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(bar(B_OD));
          mma_commit(bar(B_KVE + sp));
        }
        __syncwarp();
        return true;
      };
      bool ok = warp_wait(bar(B_Q), 0);
      for (int j = 0; ok && j < n_tiles; ++j) {
        const int s = j % NS;
        ok = warp_wait(bar(B_KVF + s), (j / NS) & 1);
        if (ok && j > 0) ok = warp_wait(bar(B_SE), (j - 1) & 1);
        if (!ok) break;
        tc_fence_after();
        if (lane == 0) {
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint64_t a = sw128_desc(base + OFF_Q + (kk >> 2) * kRegion + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = sw128_desc(base + OFF_K + s * kTileBytes + (kk >> 2) * kRegion + (kk & 3) * 32, 16, 1024);
            mma_f16_ss(tS, a, bd, idesc_qk, kk > 0 ? 1u : 0u);
          }
          mma_commit(bar(B_SF));
        }
        __syncwarp();
        if (j > 0) ok = issue_pv(j - 1);
      }
      if (ok) issue_pv(n_tiles - 1);
      // All MMAs of this CTA must be complete before TMEM is released.
      if (lane == 0) mma_commit(bar(B_FIN));
      __syncwarp();
      warp_wait(bar(B_FIN), 0);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int sub = warp & 3;
    const int row = sub * 32 + lane;
    const uint32_t lane_off = (uint32_t)(sub * 32) << 16;
    const int q_row = qt * BM + row;
    const int q_abs = q_row + k_len - q_len;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    uint8_t* prow0 = gbase + OFF_P + row * 128;
    for (int j = 0; j < n_tiles; ++j) {
      if (!(ok = warp_wait(bar(B_SF), j & 1))) break;
      tc_fence_after();
      float s[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tS + lane_off + c * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c * 32 + i] = __uint_as_float(r[i]);
      }
      tc_fence_before();
      mbar_arrive(bar(B_SE));
      const int key0 = j * BN;
      const bool need_mask = key0 + BN > k_len || (p.causal && key0 + BN - 1 > q_abs);
      const int limit = p.causal ? min(k_len - 1, q_abs) : k_len - 1;  // last visible key
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < BN; ++i) {
        float x = s[i] * p.scale_log2;
        if (need_mask && key0 + i > limit) x = -INFINITY;
        s[i] = x;
        mx = fmaxf(mx, x);
      }
      const float m_new = fmaxf(m_run, mx);
      const float m_safe = m_new == -INFINITY ? 0.f : m_new;
      const float factor = exp2f(m_run - m_safe);
      if (j > 0) {
        if (!(ok = warp_wait(bar(B_OD), (j - 1) & 1))) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, factor != 1.f)) {
#pragma unroll
          for (int c = 0; c < HD / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(tO + lane_off + c * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * factor);
            tmem_st32(tO + lane_off + c * 32, r);
          }
          tmem_wait_st();
        }
      }
      l_run *= factor;
      m_run = m_new;
      float lsum = 0.f;
#pragma unroll
      for (int chunk = 0; chunk < BN / 8; ++chunk) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float p0 = exp2f(s[chunk * 8 + 2 * i] - m_safe);
          const float p1 = exp2f(s[chunk * 8 + 2 * i + 1] - m_safe);
          lsum += p0 + p1;
          w[i] = pack_p<BF16>(p0, p1);
        }
        const int region = chunk >> 3, cc = chunk & 7;
        *reinterpret_cast<uint4*>(prow0 + region * kRegion + ((cc ^ (row & 7)) << 4)) =
            make_uint4(w[0], w[1], w[2], w[3]);
      }
      l_run += lsum;
      if (key0 + BN > k_len) {
        // Keys past the sequence in the last tile: zero their V rows so that a
        // non-finite neighbour value can never meet a zero probability.
        const int s = j % NS;
        if (!(ok = warp_wait(bar(B_KVF + s), (j / NS) & 1))) break;
        if (key0 + row >= k_len) {
          uint8_t* vrow = gbase + OFF_V + s * kTileBytes + row * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            *reinterpret_cast<uint4*>(vrow + c * 16) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4*>(vrow + kRegion + c * 16) = make_uint4(0, 0, 0, 0);
          }
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(bar(B_PF));
    }
    if (ok && n_tiles > 0) {
      ok = warp_wait(bar(B_OD), (n_tiles - 1) & 1);
      tc_fence_after();
    }
    // ------------------------------------------------------------ epilogue
    const bool row_ok = q_row < q_len;
    const int64_t t = (int64_t)q_begin + q_row;
    const bool have = ok && n_tiles > 0 && l_run > 0.f;
    const float inv = have ? 1.f / l_run : 0.f;
    uint8_t* orow = reinterpret_cast<uint8_t*>(p.out) + (t * p.os0 + (int64_t)h * p.os1) * 2;
#pragma unroll
    for (int c = 0; c < HD / 32; ++c) {
      uint32_t r[32];
      if (ok && n_tiles > 0) {
        tmem_ld32(tO + lane_off + c * 32, r);
        tmem_wait_ld();
      }
      if (row_ok) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float a = have ? __uint_as_float(r[v * 8 + 2 * i]) * inv : 0.f;
            const float bb = have ? __uint_as_float(r[v * 8 + 2 * i + 1]) * inv : 0.f;
            w[i] = pack_p<BF16>(a, bb);
          }
          *reinterpret_cast<uint4*>(orow + (c * 32 + v * 8) * 2) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
    if (row_ok) p.lse[(int64_t)h * p.ls0 + t * p.ls1] = have ? (m_run + log2f(l_run)) * kLn2 : -INFINITY;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------- host helpers
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

// [rows, heads, 128] tensor with unit inner stride -> 3-D map, box {64, 1, 128}.
int make_map(CUtensorMap* map, const void* ptr, int dtype, int64_t rows, int64_t heads, int64_t s_row,
             int64_t s_head) {
  auto fn = encode_fn();
  if (!fn) return fail(FA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)HD, (cuuint64_t)heads, (cuuint64_t)rows};
  cuuint64_t strides[2] = {(cuuint64_t)(s_head * 2), (cuuint64_t)(s_row * 2)};
  cuuint32_t box[3] = {64, 1, (cuuint32_t)BM};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dtype == FA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return FA_OK;
}

bool al16(const void* ptr) { return ((uintptr_t)ptr & 15u) == 0; }

}  // namespace

int prefill_sm100_supported(const AttnParams& p) {
  if (!(p.qt == FA_BF16 || p.qt == FA_F16) || p.kt != p.qt || p.vt != p.qt || p.ot != p.qt) return 0;
  if (p.DQ != HD || p.DV != HD || p.paged) return 0;
  if (p.win_l >= 0 || p.win_r >= 0 || p.alibi || p.sinks || p.qd || p.kd || p.vd || p.mask || p.leftpad ||
      p.dynamic || p.softcap > 0.f)
    return 0;
  if (p.qs2 != 1 || p.ks3 != 1 || p.vs3 != 1 || p.os2 != 1) return 0;
  if (!al16(p.q) || !al16(p.k) || !al16(p.v) || !al16(p.out)) return 0;
  const int64_t s[8] = {p.qs0, p.qs1, p.ks1, p.ks2, p.vs1, p.vs2, p.os0, p.os1};
  for (int64_t v : s)
    if (v <= 0 || (v * 2) % 16 != 0) return 0;
  if (p.T >= (1 << 30) || p.k_rows <= 0 || p.k_rows >= (1 << 30)) return 0;
  if (!encode_fn()) return 0;
  return 1;
}

int launch_prefill_sm100(const AttnParams& p, cudaStream_t stream) {
  if (p.k_rows <= 0) return fail(FA_ERR_INVALID, "prefill needs packed K/V rows");
  CUtensorMap mq, mk, mv;
  int rc = make_map(&mq, p.q, p.qt, p.T, p.HQ, p.qs0, p.qs1);
  if (rc) return rc;
  rc = make_map(&mk, p.k, p.kt, p.k_rows, p.HK, p.ks1, p.ks2);
  if (rc) return rc;
  rc = make_map(&mv, p.v, p.vt, p.k_rows, p.HK, p.vs1, p.vs2);
  if (rc) return rc;
  PrefillParams pp{};
  pp.out = p.out; pp.os0 = p.os0; pp.os1 = p.os1;
  pp.lse = p.lse; pp.ls0 = p.ls0; pp.ls1 = p.ls1;
  pp.cu_q = p.cu_q; pp.cq0 = p.cq0;
  pp.cu_k = p.cu_k; pp.ck0 = p.ck0;
  pp.used = p.used; pp.u0 = p.u0;
  pp.HQ = p.HQ; pp.HK = p.HK;
  pp.n_qtiles = (p.max_q + BM - 1) / BM;
  pp.causal = p.causal;
  pp.scale_log2 = p.scale * 1.4426950408889634f;
  auto kernel = p.qt == FA_BF16 ? prefill_sm100_kernel<true> : prefill_sm100_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return fail(FA_ERR_CUDA, "prefill smem attribute: %s", cudaGetErrorString(e));
  dim3 grid((unsigned)pp.n_qtiles, (unsigned)p.HQ, (unsigned)p.B);
  kernel<<<grid, kThreads, kSmemBytes, stream>>>(mq, mk, mv, pp);
  FAB_LAUNCH_CHECK("prefill launch");
  return FA_OK;
}

}  // namespace fab
