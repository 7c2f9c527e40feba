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
#include <algorithm>
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
constexpr int kSmemBytes = OFF_BAR + 512 + 1024;
constexpr int NWORK = 4;  // work-id ring slots
constexpr uint32_t kTmemCols = 512;           // S_A, S_B, O_A, O_B (128 fp32 columns each)
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;     // log2 units: P stays <= 2^8 between rescales

enum {
  B_Q = 0, B_QE, B_FULL, B_EMPTY = B_FULL + NSLOT, B_SFA = B_EMPTY + NSLOT, B_SFB, B_PFA, B_PFB, B_ODA, B_ODB,
  B_FIN, B_WFULL, B_WEMPTY = B_WFULL + NWORK, B_COUNT = B_WEMPTY + NWORK
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
  int* counter;                           // work counter, zero at launch
  int32_t B, HQ, HK, n_pairs, causal, win_l, win_r;
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
__device__ __forceinline__ float rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}
// tanh from the identity tanh(y) = 1 - 2 / (e^(2y) + 1): one ex2, one rcp, one
// FFMA. Absolute error ~1e-6 over the whole range (saturates cleanly to +-1),
// which a softcap multiplies by the cap.
__device__ __forceinline__ float tanh_id(float y) {
  return fmaf(-2.f, rcp(1.f + ex2(y * 2.8853900817779268f)), 1.f);
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

// One work item: a pair of 128-row query tiles of one (request, query head).
// Items are ordered by pair index descending (the costliest causal tiles
// first), then head, then request.
struct Item {
  bool valid;
  int b, h, kh, q_begin, q_len, k_begin, k_len, row_a, row_b;
  bool causal;
  int a0, a1, b0, b1, j_first, n_all;
};

__device__ __forceinline__ Item make_item(const PrefillParams& p, int w) {
  Item it;
  const int per = p.HQ * p.B;
  const int pair = p.n_pairs - 1 - w / per;
  const int rem = w - (w / per) * per;
  it.h = rem % p.HQ;
  it.b = rem / p.HQ;
  it.q_begin = p.cu_q[it.b * p.cq0];
  it.q_len = p.cu_q[(it.b + 1) * p.cq0] - it.q_begin;
  it.row_a = pair * 2 * BM;
  it.row_b = it.row_a + BM;
  it.valid = it.row_a < it.q_len;
  it.n_all = 0;
  it.a0 = it.a1 = it.b0 = it.b1 = it.j_first = 0;
  if (!it.valid) return it;
  it.k_begin = p.cu_k ? p.cu_k[it.b * p.ck0] : 0;
  it.k_len = p.used ? p.used[it.b * p.u0] : p.cu_k[(it.b + 1) * p.ck0] - it.k_begin;
  it.kh = it.h / (p.HQ / p.HK);
  it.causal = p.causal_b ? p.causal_b[it.b * p.ca0] != 0 : p.causal != 0;
  tile_range(it.row_a, it.q_len, it.k_len, it.causal, p.win_l, p.win_r, &it.a0, &it.a1);
  tile_range(it.row_b, it.q_len, it.k_len, it.causal, p.win_l, p.win_r, &it.b0, &it.b1);
  const bool ha = it.a1 > it.a0, hb = it.b1 > it.b0;
  if (!ha && !hb) return it;
  it.j_first = ha ? (hb ? min(it.a0, it.b0) : it.a0) : it.b0;
  const int j_last = max(ha ? it.a1 : 0, hb ? it.b1 : 0);
  it.n_all = j_last - it.j_first;
  return it;
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
  const int n_work = p.n_pairs * p.HQ * p.B;
  auto bar = [&](int i) { return base + OFF_BAR + 8u * (uint32_t)i; };
  const uint32_t holder = base + OFF_BAR + 8u * B_COUNT;
  volatile uint32_t* holder_ptr = reinterpret_cast<volatile uint32_t*>(gbase + OFF_BAR + 8 * B_COUNT);
  volatile int* wring = reinterpret_cast<volatile int*>(gbase + OFF_BAR + 8 * B_COUNT + 16);
  // Work ids flow from the TMA warp (which claims them with an atomic counter,
  // heaviest first) to the MMA warp and the 8 softmax warps through a ring.
  auto next_work = [&](uint32_t& cnt) -> int {
    const uint32_t slot = cnt % NWORK;
    if (!warp_wait(base + OFF_BAR + 8u * (B_WFULL + slot), (cnt / NWORK) & 1)) return -2;
    const int w = wring[slot];
    __syncwarp();
    if (lane == 0) mbar_arrive(base + OFF_BAR + 8u * (B_WEMPTY + slot));
    ++cnt;
    return w;
  };

  if (threadIdx.x == 0) {
    mbar_init(bar(B_Q), 1);
    mbar_init(bar(B_QE), 1);
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
    for (int s = 0; s < NWORK; ++s) {
      mbar_init(bar(B_WFULL + s), 1);
      mbar_init(bar(B_WEMPTY + s), 9);  // MMA warp + 8 softmax warps
    }
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
    uint32_t items = 0, qloads = 0;
    bool ok = true;
    if (lane == 0) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
    }
    uint32_t fwd = 0;
    while (ok) {
      int w = 0;
      if (lane == 0) w = atomicAdd(p.counter, 1);
      w = __shfl_sync(0xffffffffu, w, 0);
      const bool end = w >= n_work;
      const Item it = make_item(p, end ? 0 : w);
      if (!end && !it.valid) continue;
      {
        const uint32_t slot = fwd % NWORK;
        if (fwd >= NWORK && !(ok = warp_wait(bar(B_WEMPTY + slot), ((fwd / NWORK) - 1) & 1))) break;
        if (lane == 0) {
          wring[slot] = end ? -1 : w;
          mbar_arrive(bar(B_WFULL + slot));
        }
        __syncwarp();
        ++fwd;
      }
      if (end) break;
      if (it.n_all == 0) continue;
      // The previous item's last QK^T must be done before its Q tiles are replaced.
      if (qloads > 0 && !(ok = warp_wait(bar(B_QE), (qloads - 1) & 1))) break;
      if (lane == 0) {
        mbar_expect_tx(bar(B_Q), 2 * kTileBytes);
        tma_load_3d(base + OFF_QA, &tq, bar(B_Q), 0, it.h, it.q_begin + it.row_a);
        tma_load_3d(base + OFF_QA + kRegion, &tq, bar(B_Q), 64, it.h, it.q_begin + it.row_a);
        tma_load_3d(base + OFF_QB, &tq, bar(B_Q), 0, it.h, it.q_begin + it.row_b);
        tma_load_3d(base + OFF_QB + kRegion, &tq, bar(B_Q), 64, it.h, it.q_begin + it.row_b);
      }
      ++qloads;
      for (int i = 0; i < 2 * it.n_all; ++i) {  // K(j), V(j), K(j+1), ...
        const uint32_t slot = items % NSLOT;
        if (items >= NSLOT && !(ok = warp_wait(bar(B_EMPTY + slot), ((items / NSLOT) - 1) & 1))) break;
        if (lane == 0) {
          const CUtensorMap* map = (i & 1) ? &tv : &tk;
          const int row = it.k_begin + (it.j_first + (i >> 1)) * BN;
          const uint32_t dst = base + OFF_RING + slot * kTileBytes;
          mbar_expect_tx(bar(B_FULL + slot), kTileBytes);
          tma_load_3d(dst, map, bar(B_FULL + slot), 0, it.kh, row);
          tma_load_3d(dst + kRegion, map, bar(B_FULL + slot), 64, it.kh, row);
        }
        ++items;
      }
    }
    // Drain: every issued load must have landed before the CTA exits.
    if (qloads > 0) warp_wait(bar(B_Q), (qloads - 1) & 1);
    for (uint32_t i = items > NSLOT ? items - NSLOT : 0; i < items; ++i)
      warp_wait(bar(B_FULL + i % NSLOT), (i / NSLOT) & 1);
  } else if (warp == 9) {
    // ---------------------------------------------------------------- MMA
    const uint32_t idesc_qk = f16_idesc(BM, BN, BF16 ? 1 : 0, 0);
    const uint32_t idesc_pv = f16_idesc(BM, HD, BF16 ? 1 : 0, 1);
    const uint32_t tSA = tmem, tSB = tmem + 128, tOA = tmem + 256, tOB = tmem + 384;
    auto slot_addr = [&](uint32_t item) { return base + OFF_RING + (item % NSLOT) * kTileBytes; };
    auto wait_item = [&](uint32_t item) { return warp_wait(bar(B_FULL + item % NSLOT), (item / NSLOT) & 1); };
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
    uint32_t items = 0, qloads = 0, pa = 0, pb = 0, wcnt = 0;
    bool ok = true;
    while (ok) {
      const int w = next_work(wcnt);
      if (w < 0) break;
      const Item it = make_item(p, w);
      if (it.n_all == 0) continue;
      auto act_a = [&](int j) { return j >= it.a0 && j < it.a1; };
      auto act_b = [&](int j) { return j >= it.b0 && j < it.b1; };
      if (!(ok = warp_wait(bar(B_Q), qloads & 1) && wait_item(items))) break;
      ++qloads;
      tc_fence_after();
      if (act_a(it.j_first)) qk(OFF_QA, slot_addr(items), tSA, B_SFA);
      if (act_b(it.j_first)) qk(OFF_QB, slot_addr(items), tSB, B_SFB);
      commit(B_EMPTY + items % NSLOT);
      if (it.n_all == 1) commit(B_QE);
      for (int t = 0; ok && t < it.n_all; ++t) {
        const int j = it.j_first + t;
        const uint32_t iv = items + 2 * t + 1, ik = items + 2 * t + 2;
        if (!(ok = wait_item(iv))) break;
        if (act_a(j)) {
          if (!(ok = warp_wait(bar(B_PFA), pa & 1))) break;
          ++pa;
          tc_fence_after();
          pv(OFF_PA, slot_addr(iv), tOA, j > it.a0);
          if (j == it.a1 - 1) commit(B_ODA);
        }
        const bool next = t + 1 < it.n_all;
        if (next && !(ok = wait_item(ik))) break;
        tc_fence_after();
        if (next && act_a(j + 1)) qk(OFF_QA, slot_addr(ik), tSA, B_SFA);
        if (act_b(j)) {
          if (!(ok = warp_wait(bar(B_PFB), pb & 1))) break;
          ++pb;
          tc_fence_after();
          pv(OFF_PB, slot_addr(iv), tOB, j > it.b0);
          if (j == it.b1 - 1) commit(B_ODB);
        }
        commit(B_EMPTY + iv % NSLOT);
        if (next && act_b(j + 1)) qk(OFF_QB, slot_addr(ik), tSB, B_SFB);
        if (next) commit(B_EMPTY + ik % NSLOT);
        if (t + 2 == it.n_all) commit(B_QE);  // the item's last QK^T has been issued
      }
      items += 2 * it.n_all;
    }
    // All MMAs of this CTA must be complete before TMEM is released.
    commit(B_FIN);
    warp_wait(bar(B_FIN), 0);
  } else {
    // ------------------------------------------------------------ softmax
    const bool is_b = warp >= 4;
    const int sub = warp & 3;
    const int row = sub * 32 + lane;
    const uint32_t lane_off = (uint32_t)(sub * 32) << 16;
    const uint32_t tS = tmem + (is_b ? 128 : 0) + lane_off;
    const uint32_t tO = tmem + (is_b ? 384 : 256) + lane_off;
    const int sf = is_b ? B_SFB : B_SFA, pf = is_b ? B_PFB : B_PFA, od = is_b ? B_ODB : B_ODA;
    uint8_t* prow = gbase + (is_b ? OFF_PB : OFF_PA) + row * 128;
    uint32_t s_cnt = 0, o_cnt = 0, items = 0, wcnt = 0;
    bool ok = true;
    while (ok) {
      const int w = next_work(wcnt);
      if (w < 0) break;
      const Item it = make_item(p, w);
      const int x0 = is_b ? it.b0 : it.a0, n_x = (is_b ? it.b1 : it.a1) - x0;
      const int q_row = (is_b ? it.row_b : it.row_a) + row;
      const int q_abs = q_row + it.k_len - it.q_len;
      const KeyRange vis = key_range(q_abs, it.k_len, it.causal, p.win_l, p.win_r);
      const int b = it.b, h = it.h, kh = it.kh;
      const float qk_scale = p.scale * (p.qd ? p.qd[b * p.qd0 + kh * p.qd1] : 1.f) *
                             (p.kd ? p.kd[b * p.kd0 + kh * p.kd1] : 1.f);
      const float vscale = p.vd ? p.vd[b * p.vd0 + kh * p.vd1] : 1.f;
      const float sl2 = qk_scale * 1.4426950408889634f;     // raw score -> log2 units
      const float cap_l2 = p.softcap * 1.4426950408889634f;  // softcap: cap*log2e*tanh(s*scale/cap)
      const float cap_in = SOFTCAP ? qk_scale / p.softcap : 0.f;
      // Running max in log2 units; a sink acts as one extra logit with zero value.
      float m_run = -INFINITY, l_run = 0.f;
      if (p.sinks) {
        m_run = load_float(p.sinks, p.sink_t, h * p.si0) * 1.4426950408889634f;
        l_run = 1.f;
      }
      for (int jj = 0; jj < n_x; ++jj) {
        const int j = x0 + jj;
        if (!(ok = warp_wait(bar(sf), s_cnt & 1))) break;
        ++s_cnt;
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
        const float m_tile = SOFTCAP ? (mx == -INFINITY ? -INFINITY : cap_l2 * tanh_id(mx * cap_in)) : mx * sl2;
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
            uint32_t wv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              float p0, p1;
              const float s0 = __uint_as_float(r[c8 * 8 + 2 * i]), s1 = __uint_as_float(r[c8 * 8 + 2 * i + 1]);
              if constexpr (SOFTCAP) {
                p0 = s0 == -INFINITY ? 0.f : ex2(fmaf(cap_l2, tanh_id(s0 * cap_in), -msub));
                p1 = s1 == -INFINITY ? 0.f : ex2(fmaf(cap_l2, tanh_id(s1 * cap_in), -msub));
              } else {
                p0 = ex2(fmaf(s0, sl2, -msub));
                p1 = ex2(fmaf(s1, sl2, -msub));
              }
              ls8[2 * i] += p0;
              ls8[2 * i + 1] += p1;
              wv[i] = pack_p<BF16>(p0, p1);
            }
            const int chunk = hh * 8 + c8, region = chunk >> 3, cc = chunk & 7;
            *reinterpret_cast<uint4*>(prow + region * kRegion + ((cc ^ (row & 7)) << 4)) =
                make_uint4(wv[0], wv[1], wv[2], wv[3]);
          }
        }
        const float lsum = ((ls8[0] + ls8[1]) + (ls8[2] + ls8[3])) + ((ls8[4] + ls8[5]) + (ls8[6] + ls8[7]));
        l_run += lsum;
        if (key0 + BN > it.k_len) {
          // Keys past the sequence in the last tile: zero their V rows so that a
          // non-finite neighbour value can never meet a zero probability. Each
          // warpgroup consuming the tile zeroes them itself (identical stores).
          const uint32_t item = items + 2 * (j - it.j_first) + 1;
          if (!(ok = warp_wait(bar(B_FULL + item % NSLOT), (item / NSLOT) & 1))) break;
          if (key0 + row >= it.k_len) {
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
      items += 2 * it.n_all;
      if (!ok) break;
      if (n_x > 0) {
        if (!(ok = warp_wait(bar(od), o_cnt & 1))) break;
        ++o_cnt;
        tc_fence_after();
      }
      // ---------------------------------------------------------- epilogue
      const bool row_ok = q_row < it.q_len;
      const int64_t t = (int64_t)it.q_begin + q_row;
      const bool have = n_x > 0 && l_run > 0.f;
      const float inv = have ? vscale / l_run : 0.f;
      uint8_t* orow = reinterpret_cast<uint8_t*>(p.out) + (t * p.os0 + (int64_t)h * p.os1) * 2;
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t r[32];
        if (n_x > 0) {
          tmem_ld32(tO + c * 32, r);
          tmem_wait_ld();
        }
        if (row_ok) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint32_t wv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float a = have ? __uint_as_float(r[v * 8 + 2 * i]) * inv : 0.f;
              const float bb = have ? __uint_as_float(r[v * 8 + 2 * i + 1]) * inv : 0.f;
              wv[i] = pack_p<BF16>(a, bb);
            }
            *reinterpret_cast<uint4*>(orow + (c * 32 + v * 8) * 2) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
          }
        }
      }
      if (row_ok) p.lse[(int64_t)h * p.ls0 + t * p.ls1] = l_run > 0.f ? (m_run + log2f(l_run)) * kLn2 : -INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------- host helpers
// [rows, heads, 128] tensor with unit inner stride -> 3-D map, box {64, 1, 128}.
int make_map(CUtensorMap* map, const void* ptr, int dtype, int64_t rows, int64_t heads, int64_t s_row,
             int64_t s_head) {
  const uint64_t dims[3] = {(uint64_t)HD, (uint64_t)heads, (uint64_t)rows};
  const uint64_t strides[2] = {(uint64_t)(s_head * 2), (uint64_t)(s_row * 2)};
  const uint32_t box[3] = {64, 1, (uint32_t)BM};
  return encode_tensor_map(map, dtype, 3, ptr, dims, strides, box, true);
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
  if ((int64_t)((p.max_q + 2 * BM - 1) / (2 * BM)) * p.HQ * p.B >= (1LL << 31)) return 0;
  if (!tensor_map_available()) return 0;
  return 1;
}

int prefill_timeout_flag(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_prefill_timeout, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_prefill_timeout, &zero, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
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
  pp.B = p.B; pp.HQ = p.HQ; pp.HK = p.HK;
  pp.counter = reinterpret_cast<int*>(p.scratch);
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
  const int64_t n_work = (int64_t)pp.n_pairs * p.HQ * p.B;
  const int grid = (int)std::min<int64_t>(n_work, (int64_t)sm_count());
  if (pp.counter == nullptr) return fail(FA_ERR_INVALID, "prefill needs its workspace counter");
  e = cudaMemsetAsync(pp.counter, 0, sizeof(int), stream);
  if (e != cudaSuccess) return fail(FA_ERR_CUDA, "prefill counter reset: %s", cudaGetErrorString(e));
  kernel<<<grid, kThreads, kSmemBytes, stream>>>(mq, mk, mv, pp);
  FAB_LAUNCH_CHECK("prefill launch");
  return FA_OK;
}

}  // namespace fab
