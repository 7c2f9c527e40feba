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

constexpr int BM = 128;          // query rows per tile (two tiles per CTA)
constexpr int BN = 128;          // keys per tile
constexpr int HD = 128;          // head dim
constexpr int NSLOT = 3;         // K/V ring slots (each holds one K or one V tile)
constexpr int kRegion = 128 * 128;            // one 128-row x 64-element box (bytes)
constexpr int kTileBytes = 2 * kRegion;       // 128 x 128 bf16
constexpr int kThreads = 320;                 // 2 softmax warpgroups + TMA warp + MMA warp
constexpr int OFF_QA = 0;
constexpr int OFF_QB = OFF_QA + kTileBytes;
constexpr int OFF_PA = OFF_QB + kTileBytes;
constexpr int OFF_PB = OFF_PA + kTileBytes;
constexpr int OFF_RING = OFF_PB + kTileBytes;
constexpr int OFF_BAR = OFF_RING + NSLOT * kTileBytes;
constexpr int kSmemBytes = OFF_BAR + 256 + 1024;
constexpr uint32_t kTmemCols = 512;           // S_A, S_B, O_A, O_B (128 fp32 columns each)
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;     // log2 units: P stays <= 2^8 between rescales

enum {
  B_Q = 0, B_FULL = 1, B_EMPTY = B_FULL + NSLOT, B_SFA = B_EMPTY + NSLOT, B_SFB, B_PFA, B_PFB, B_ODA, B_ODB,
  B_FIN, B_COUNT
};

__device__ int g_prefill_timeout;

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
  int32_t HQ, HK, n_pairs, causal, win_l, win_r;
  float scale, softcap;
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

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
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

template <bool BF16, bool SOFTCAP>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_sm100_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                         const __grid_constant__ CUtensorMap tv, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z, h = blockIdx.y;
  const int pair = p.n_pairs - 1 - (int)blockIdx.x;  // longest causal tiles first
  const int q_begin = p.cu_q[b * p.cq0];
  const int q_len = p.cu_q[(b + 1) * p.cq0] - q_begin;
  const int row_a = pair * 2 * BM, row_b = row_a + BM;
  if (row_a >= q_len) return;
  const int k_begin = p.cu_k ? p.cu_k[b * p.ck0] : 0;
  const int k_len = p.used ? p.used[b * p.u0] : p.cu_k[(b + 1) * p.ck0] - k_begin;
  const int kh = h / (p.HQ / p.HK);
  const bool causal = p.causal_b ? p.causal_b[b * p.ca0] != 0 : p.causal != 0;
  int a0, a1, b0, b1;
  tile_range(row_a, q_len, k_len, causal, p.win_l, p.win_r, &a0, &a1);
  tile_range(row_b, q_len, k_len, causal, p.win_l, p.win_r, &b0, &b1);
  const int n_a = a1 - a0, n_b = b1 - b0;
  // KV tiles [j_first, j_last) cover both query tiles; item i = 2*(j - j_first) (+1 for V).
  const int j_first = n_a > 0 ? (n_b > 0 ? min(a0, b0) : a0) : b0;
  const int j_last = max(n_a > 0 ? a1 : 0, n_b > 0 ? b1 : 0);
  const int n_all = (n_a > 0 || n_b > 0) ? j_last - j_first : 0;
  auto bar = [&](int i) { return base + OFF_BAR + 8u * (uint32_t)i; };
  const uint32_t holder = base + OFF_BAR + 8u * B_COUNT;
  volatile uint32_t* holder_ptr = reinterpret_cast<volatile uint32_t*>(gbase + OFF_BAR + 8 * B_COUNT);

  if (threadIdx.x == 0) {
    mbar_init(bar(B_Q), 1);
    for (int s = 0; s < NSLOT; ++s) {
      mbar_init(bar(B_FULL + s), 1);
      mbar_init(bar(B_EMPTY + s), 1);
    }
    mbar_init(bar(B_SFA), 1);
    mbar_init(bar(B_SFB), 1);
    mbar_init(bar(B_PFA), 128);
    mbar_init(bar(B_PFB), 128);
    mbar_init(bar(B_ODA), 1);
    mbar_init(bar(B_ODB), 1);
    mbar_init(bar(B_FIN), 1);
    mbar_fence_init();
  }
  if (warp == 9) {
    tmem_alloc(holder, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *holder_ptr;

  if (warp == 8) {
    // ---------------------------------------------------------------- TMA
    if (n_all > 0) {
      const int items = 2 * n_all;  // K(0), V(0), K(1), V(1), ...
      int issued = 0;
      if (lane == 0) {
        tma_prefetch_desc(&tq);
        tma_prefetch_desc(&tk);
        tma_prefetch_desc(&tv);
        mbar_expect_tx(bar(B_Q), 2 * kTileBytes);
        tma_load_3d(base + OFF_QA, &tq, bar(B_Q), 0, h, q_begin + row_a);
        tma_load_3d(base + OFF_QA + kRegion, &tq, bar(B_Q), 64, h, q_begin + row_a);
        tma_load_3d(base + OFF_QB, &tq, bar(B_Q), 0, h, q_begin + row_b);
        tma_load_3d(base + OFF_QB + kRegion, &tq, bar(B_Q), 64, h, q_begin + row_b);
      }
      for (int i = 0; i < items; ++i) {
        const int slot = i % NSLOT;
        if (i >= NSLOT && !warp_wait(bar(B_EMPTY + slot), ((i / NSLOT) - 1) & 1)) break;
        if (lane == 0) {
          const CUtensorMap* map = (i & 1) ? &tv : &tk;
          const int row = k_begin + (j_first + (i >> 1)) * BN;
          const uint32_t dst = base + OFF_RING + slot * kTileBytes;
          mbar_expect_tx(bar(B_FULL + slot), kTileBytes);
          tma_load_3d(dst, map, bar(B_FULL + slot), 0, kh, row);
          tma_load_3d(dst + kRegion, map, bar(B_FULL + slot), 64, kh, row);
        }
        issued = i + 1;
      }
      // Drain: every issued load must have landed before the CTA exits.
      warp_wait(bar(B_Q), 0);
      for (int i = max(0, issued - NSLOT); i < issued; ++i) warp_wait(bar(B_FULL + i % NSLOT), (i / NSLOT) & 1);
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------------- MMA
    if (n_all > 0) {
      const uint32_t idesc_qk = f16_idesc(BM, BN, BF16 ? 1 : 0, 0);
      const uint32_t idesc_pv = f16_idesc(BM, HD, BF16 ? 1 : 0, 1);
      const uint32_t tSA = tmem, tSB = tmem + 128, tOA = tmem + 256, tOB = tmem + 384;
      auto slot_addr = [&](int item) { return base + OFF_RING + (item % NSLOT) * kTileBytes; };
      auto wait_item = [&](int item) { return warp_wait(bar(B_FULL + item % NSLOT), (item / NSLOT) & 1); };
      auto qk = [&](uint32_t q_off, uint32_t kaddr, uint32_t d, int sfbar) {
        if (lane == 0) {
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint64_t a = sw128_desc(base + q_off + (kk >> 2) * kRegion + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = sw128_desc(kaddr + (kk >> 2) * kRegion + (kk & 3) * 32, 16, 1024);
            mma_f16_ss(d, a, bd, idesc_qk, kk > 0 ? 1u : 0u);
          }
          mma_commit(bar(sfbar));
        }
        __syncwarp();
      };
      auto pv = [&](uint32_t p_off, uint32_t vaddr, uint32_t d, bool acc) {
        if (lane == 0) {
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const uint64_t a = sw128_desc(base + p_off + (kk >> 2) * kRegion + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = sw128_desc(vaddr + kk * 2048, kRegion, 1024);
            mma_f16_ss(d, a, bd, idesc_pv, (acc || kk > 0) ? 1u : 0u);
          }
        }
        __syncwarp();
      };
      auto commit = [&](int barid) {
        if (lane == 0) mma_commit(bar(barid));
        __syncwarp();
      };
      auto act_a = [&](int j) { return j >= a0 && j < a1; };
      auto act_b = [&](int j) { return j >= b0 && j < b1; };
      bool ok = warp_wait(bar(B_Q), 0) && wait_item(0);
      if (ok) {
        tc_fence_after();
        if (act_a(j_first)) qk(OFF_QA, slot_addr(0), tSA, B_SFA);
        if (act_b(j_first)) qk(OFF_QB, slot_addr(0), tSB, B_SFB);
        commit(B_EMPTY + 0);
      }
      for (int t = 0; ok && t < n_all; ++t) {
        const int j = j_first + t;
        const int iv = 2 * t + 1, ik = 2 * t + 2;
        if (!(ok = wait_item(iv))) break;
        if (act_a(j)) {
          if (!(ok = warp_wait(bar(B_PFA), (j - a0) & 1))) break;
          tc_fence_after();
          pv(OFF_PA, slot_addr(iv), tOA, j > a0);
          if (j == a1 - 1) commit(B_ODA);
        }
        const bool next = t + 1 < n_all;
        if (next && !(ok = wait_item(ik))) break;
        tc_fence_after();
        if (next && act_a(j + 1)) qk(OFF_QA, slot_addr(ik), tSA, B_SFA);
        if (act_b(j)) {
          if (!(ok = warp_wait(bar(B_PFB), (j - b0) & 1))) break;
          tc_fence_after();
          pv(OFF_PB, slot_addr(iv), tOB, j > b0);
          if (j == b1 - 1) commit(B_ODB);
        }
        commit(B_EMPTY + iv % NSLOT);
        if (next && act_b(j + 1)) qk(OFF_QB, slot_addr(ik), tSB, B_SFB);
        if (next) commit(B_EMPTY + ik % NSLOT);
      }
      // All MMAs of this CTA must be complete before TMEM is released.
      commit(B_FIN);
      warp_wait(bar(B_FIN), 0);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const bool is_b = warp >= 4;
    const int sub = warp & 3;
    const int row = sub * 32 + lane;
    const uint32_t lane_off = (uint32_t)(sub * 32) << 16;
    const uint32_t tS = tmem + (is_b ? 128 : 0) + lane_off;
    const uint32_t tO = tmem + (is_b ? 384 : 256) + lane_off;
    const int x0 = is_b ? b0 : a0, n_x = is_b ? n_b : n_a;
    const int q_row = (is_b ? row_b : row_a) + row;
    const int q_abs = q_row + k_len - q_len;
    const KeyRange vis = key_range(q_abs, k_len, causal, p.win_l, p.win_r);
    const int sf = is_b ? B_SFB : B_SFA, pf = is_b ? B_PFB : B_PFA, od = is_b ? B_ODB : B_ODA;
    uint8_t* prow = gbase + (is_b ? OFF_PB : OFF_PA) + row * 128;
    const float qk_scale = p.scale * (p.qd ? p.qd[b * p.qd0 + kh * p.qd1] : 1.f) *
                           (p.kd ? p.kd[b * p.kd0 + kh * p.kd1] : 1.f);
    const float vscale = p.vd ? p.vd[b * p.vd0 + kh * p.vd1] : 1.f;
    const float sl2 = qk_scale * 1.4426950408889634f;       // raw score -> log2 units
    const float cap_l2 = p.softcap * 1.4426950408889634f;    // softcap: cap*log2e*tanh(s*scale/cap)
    const float cap_in = SOFTCAP ? qk_scale / p.softcap : 0.f;
    // Running max in log2 units; a sink acts as one extra logit with zero value.
    float m_run = -INFINITY, l_run = 0.f;
    if (p.sinks) {
      m_run = load_float(p.sinks, p.sink_t, h * p.si0) * 1.4426950408889634f;
      l_run = 1.f;
    }
    bool ok = true;
    for (int jj = 0; jj < n_x; ++jj) {
      const int j = x0 + jj;
      if (!(ok = warp_wait(bar(sf), jj & 1))) break;
      tc_fence_after();
      const int key0 = j * BN;
      const int c_lo = vis.lo - key0, c_hi = vis.hi - key0;  // visible columns of this tile
      const bool need_mask = c_lo > 0 || c_hi < BN - 1;
      // Pass 1: row max, 64 columns (two TMEM loads in flight) at a time, as 8
      // independent chains (fp max is exact in any order).
      float mx8[8];
#pragma unroll
      for (int k8 = 0; k8 < 8; ++k8) mx8[k8] = -INFINITY;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t r[64];
        tmem_ld32_at<0>(tS + hh * 64, r);
        tmem_ld32_at<32>(tS + hh * 64 + 32, r);
        tmem_wait_ld();
        if (need_mask) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (hh * 64 + i < c_lo || hh * 64 + i > c_hi) r[i] = __float_as_uint(-INFINITY);
        }
#pragma unroll
        for (int i = 0; i < 64; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], __uint_as_float(r[i]));
      }
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      // scale > 0 and tanh is increasing: the max commutes with both.
      const float m_tile = SOFTCAP ? (mx == -INFINITY ? -INFINITY : cap_l2 * tanhf(mx * cap_in)) : mx * sl2;
      float factor = 1.f;
      if (m_tile > m_run + kRescaleThreshold || (m_run == -INFINITY && m_tile != -INFINITY)) {
        factor = m_run == -INFINITY ? 0.f : ex2(m_run - m_tile);
        m_run = m_tile;
      }
      if (jj > 0 && __any_sync(0xffffffffu, factor != 1.f)) {
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
          tmem_st32(tO + c * 32, o);
        }
        tmem_wait_st();
      }
      l_run *= factor;
      const float msub = m_run == -INFINITY ? 0.f : m_run;
      // Pass 2: P = 2^(s*scale_log2 - m), masked columns -> 0, written to the
      // swizzled P tile; the row sum runs as 8 independent chains.
      float ls8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t r[64];
        tmem_ld32_at<0>(tS + hh * 64, r);
        tmem_ld32_at<32>(tS + hh * 64 + 32, r);
        tmem_wait_ld();
        if (need_mask) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (hh * 64 + i < c_lo || hh * 64 + i > c_hi) r[i] = __float_as_uint(-INFINITY);
        }
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float p0, p1;
            if constexpr (SOFTCAP) {
              const float s0 = __uint_as_float(r[c8 * 8 + 2 * i]), s1 = __uint_as_float(r[c8 * 8 + 2 * i + 1]);
              p0 = s0 == -INFINITY ? 0.f : ex2(fmaf(cap_l2, tanhf(s0 * cap_in), -msub));
              p1 = s1 == -INFINITY ? 0.f : ex2(fmaf(cap_l2, tanhf(s1 * cap_in), -msub));
            } else {
              p0 = ex2(fmaf(__uint_as_float(r[c8 * 8 + 2 * i]), sl2, -msub));
              p1 = ex2(fmaf(__uint_as_float(r[c8 * 8 + 2 * i + 1]), sl2, -msub));
            }
            ls8[2 * i] += p0;
            ls8[2 * i + 1] += p1;
            w[i] = pack_p<BF16>(p0, p1);
          }
          const int chunk = hh * 8 + c8, region = chunk >> 3, cc = chunk & 7;
          *reinterpret_cast<uint4*>(prow + region * kRegion + ((cc ^ (row & 7)) << 4)) =
              make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      const float lsum = ((ls8[0] + ls8[1]) + (ls8[2] + ls8[3])) + ((ls8[4] + ls8[5]) + (ls8[6] + ls8[7]));
      l_run += lsum;
      if (key0 + BN > k_len) {
        // Keys past the sequence in the last tile: zero their V rows so that a
        // non-finite neighbour value can never meet a zero probability.
        const int item = 2 * (j - j_first) + 1;
        if (!(ok = warp_wait(bar(B_FULL + item % NSLOT), (item / NSLOT) & 1))) break;
        // Each warpgroup that consumes this tile zeroes the rows itself before
        // releasing its P (identical zero stores, no cross-group barrier).
        if (key0 + row >= k_len) {
          uint8_t* vrow = gbase + OFF_RING + (item % NSLOT) * kTileBytes + row * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            *reinterpret_cast<uint4*>(vrow + c * 16) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4*>(vrow + kRegion + c * 16) = make_uint4(0, 0, 0, 0);
          }
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(bar(pf));
    }
    if (ok && n_x > 0) {
      ok = warp_wait(bar(od), 0);
      tc_fence_after();
    }
    // ------------------------------------------------------------ epilogue
    const bool row_ok = q_row < q_len;
    const int64_t t = (int64_t)q_begin + q_row;
    const bool have = ok && n_x > 0 && l_run > 0.f;
    const float inv = have ? vscale / l_run : 0.f;
    uint8_t* orow = reinterpret_cast<uint8_t*>(p.out) + (t * p.os0 + (int64_t)h * p.os1) * 2;
#pragma unroll
    for (int c = 0; c < HD / 32; ++c) {
      uint32_t r[32];
      if (ok && n_x > 0) {
        tmem_ld32(tO + c * 32, r);
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
    if (row_ok) p.lse[(int64_t)h * p.ls0 + t * p.ls1] = ok && l_run > 0.f ? (m_run + log2f(l_run)) * kLn2 : -INFINITY;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
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
  if (p.alibi || p.mask || p.leftpad) return 0;
  if (p.sinks && !(p.sink_t == FA_F32 || p.sink_t == FA_F16 || p.sink_t == FA_BF16)) return 0;
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
  pp.n_pairs = (p.max_q + 2 * BM - 1) / (2 * BM);
  pp.causal = p.causal;
  pp.causal_b = p.dynamic ? p.causal_b : nullptr; pp.ca0 = p.ca0;
  pp.sinks = p.sinks; pp.sink_t = p.sink_t; pp.si0 = p.si0;
  pp.qd = p.qd; pp.qd0 = p.qd0; pp.qd1 = p.qd1;
  pp.kd = p.kd; pp.kd0 = p.kd0; pp.kd1 = p.kd1;
  pp.vd = p.vd; pp.vd0 = p.vd0; pp.vd1 = p.vd1;
  pp.win_l = p.win_l; pp.win_r = p.win_r;
  pp.scale = p.scale;
  pp.softcap = p.softcap;
  const bool cap = p.softcap > 0.f;
  auto kernel = p.qt == FA_BF16 ? (cap ? prefill_sm100_kernel<true, true> : prefill_sm100_kernel<true, false>)
                                : (cap ? prefill_sm100_kernel<false, true> : prefill_sm100_kernel<false, false>);
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return fail(FA_ERR_CUDA, "prefill smem attribute: %s", cudaGetErrorString(e));
  dim3 grid((unsigned)pp.n_pairs, (unsigned)p.HQ, (unsigned)p.B);
  kernel<<<grid, kThreads, kSmemBytes, stream>>>(mq, mk, mv, pp);
  FAB_LAUNCH_CHECK("prefill launch");
  return FA_OK;
}

}  // namespace fab
