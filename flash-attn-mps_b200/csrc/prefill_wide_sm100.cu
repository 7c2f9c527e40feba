// Varlen / dense prefill for wide head dims on tcgen05 (QK head dim 129..256,
// V head dim up to 256; the reference's fast path covers head dim 256,
// flash_attn_mps/_attention.py:149-158, and its generic kernels any
// dq != dv up to 512).
//
// One persistent CTA per SM claims work items -- one 128-row query block of
// one (request, query head), heaviest causal blocks first -- from an atomic
// counter. With a 256-wide output tile the tensor memory holds one query
// tile: S (128 fp32 columns), P (64 columns of 16-bit pairs, separate from S)
// and O (up to 256 fp32 columns). Per CTA:
//   warp 4      TMA: claims and publishes the items, loads Q once per item
//               and K(j) tiles (128 keys x DQK, 64-dim 128-byte swizzled
//               boxes) into a single K buffer;
//   warp 6      TMA: V(j) tiles (128 keys x DV) into a single V buffer;
//   warp 5      TMEM owner and MMA issuer (kind::f16, M=128, K=16):
//               S = Q K^T (N=128, both operands from shared memory) and
//               O += P V (N = DV, P from tensor memory, V from shared memory);
//   warps 0..3  softmax: one query row per thread, as in the two-tile kernel.
// Because P does not overwrite S, the MMA warp issues QK^T of key tile j+1 as
// soon as the softmax has loaded S(j) into registers, and PV(j) when P(j) is
// in tensor memory: QK^T(j+1) and PV(j) alternate on the tensor pipe while
// the softmax works, and PV(j) has N = DV (at DV = 256 a tcgen05.mma with A
// in tensor memory runs at ~94 % of the pipe's peak, against ~65 % at N=128).
// The next item's first QK^T is issued before the current item's last PV.
// Output rows are written from registers. Every mbarrier wait is bounded; a
// timeout sets g_prefill_wide_timeout, drains the CTA's own loads and MMAs,
// frees TMEM and returns.
//
// Semantics (lower-right causal, natural-log LSE, zero output and -inf LSE for
// rows with no visible key, softcap before masking, sinks, q/k/v descales,
// windows, dynamic causal) are those of the two-tile kernel.
#include <algorithm>
#include <type_traits>

#include "kernels.cuh"
#include "prefill_common.cuh"
#include "sm100.cuh"

namespace fab {
namespace {

using namespace sm100;
using namespace pf;

constexpr int kWThreads = 256;          // softmax warpgroup + (K TMA, MMA, V TMA, idle)
constexpr uint32_t kWTmemCols = 512;    // S [0, 128), P [128, 192), O [256, 256 + DV)
constexpr uint32_t kColP = 128, kColO = 256;

template <int DQK, int DV>
struct WideLayout {
  static constexpr int RQ = DQK / 64, RV = DV / 64;    // 64-element swizzle regions per row
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + RQ * kRegion;
  static constexpr int OFF_V = OFF_K + RQ * kKVRegion;
  static constexpr int OFF_BAR = OFF_V + RV * kKVRegion;
  // Barriers, TMEM holder, work-id ring and item ring, then alignment slack.
  static constexpr int kSmem = OFF_BAR + 1024 + 1024;
  static_assert(kSmem <= 227 * 1024, "shared memory");
};

// W_Q: Q landed; W_QE: the item's last QK^T done (Q may be replaced);
// W_KF/W_KE, W_VF/W_VE: K / V buffer full / empty; W_SF: S ready;
// W_SC: S loaded by the softmax (one arrival per warp); W_PF: P in TMEM (one
// arrival per warp); W_PVD: a PV finished (P may be replaced, O read);
// W_OD: the item's last PV finished.
enum {
  W_Q = 0, W_QE, W_KF, W_KE, W_VF, W_VE, W_SF, W_SC, W_PF, W_PVD, W_OD, W_FIN, W_WFULL,
  W_WEMPTY = W_WFULL + NWORK, W_COUNT = W_WEMPTY + NWORK
};

__device__ int g_prefill_wide_timeout;

__device__ __forceinline__ bool wwait(uint32_t bar, uint32_t parity) {
  return warp_wait_flag(bar, parity, &g_prefill_wide_timeout);
}

// One 128-row query block of one (request, query head). Items come in groups
// of group_reqs requests (whose K/V stay in L2 together); within a group by
// block index descending (the costliest causal blocks first), then head, then
// request. Tile B of the record is unused.
__device__ __forceinline__ Item make_wide_item(const PrefillParams& p, int w) {
  Item it;
  const int per_group = p.n_pairs * p.HQ * p.group_reqs;
  const int g = w / per_group;
  const int local = w - g * per_group;
  const int b0 = g * p.group_reqs;
  const int per = p.HQ * min(p.group_reqs, p.B - b0);
  const int blk = p.n_pairs - 1 - local / per;
  const int rem = local - (local / per) * per;
  it.h = rem % p.HQ;
  it.h_b = it.h;
  it.b = b0 + rem / p.HQ;
  it.q_begin = p.cu_q[it.b * p.cq0];
  it.q_len = p.cu_q[(it.b + 1) * p.cq0] - it.q_begin;
  it.row_a = blk * BM;
  it.row_b = it.row_a;
  it.valid = it.row_a < it.q_len;
  it.n_all = 0;
  it.a0 = it.a1 = it.b0 = it.b1 = it.j_first = 0;
  it.k_begin = it.k_len = it.kh = it.causal = 0;
  it.qk_scale = it.vscale = 1.f;
  if (!it.valid) return it;
  it.k_begin = p.cu_k ? p.cu_k[it.b * p.ck0] : 0;
  it.k_len = p.used ? p.used[it.b * p.u0] : p.cu_k[(it.b + 1) * p.ck0] - it.k_begin;
  it.kh = it.h / (p.HQ / p.HK);
  it.causal = p.causal_b ? p.causal_b[it.b * p.ca0] != 0 : p.causal != 0;
  it.qk_scale = p.scale * (p.qd ? p.qd[it.b * p.qd0 + it.kh * p.qd1] : 1.f) *
                (p.kd ? p.kd[it.b * p.kd0 + it.kh * p.kd1] : 1.f);
  it.vscale = p.vd ? p.vd[it.b * p.vd0 + it.kh * p.vd1] : 1.f;
  tile_range(it.row_a, it.q_len, it.k_len, it.causal, p.win_l, p.win_r, &it.a0, &it.a1);
  it.j_first = it.a0;
  it.n_all = it.a1 - it.a0;
  return it;
}

// One BN-key tile of R 64-column regions into dst. Packed K/V: one 3-D box per
// region. Paged K/V: the keys arrive as page boxes (box_rows tokens x 64 head
// dims each, spread over the warp's lanes) through block_table; pages past the
// sequence or the table use page -1, which TMA fills with zeros. Called by the
// whole warp; lane 0 arms the barrier first.
template <int R>
__device__ __forceinline__ void load_kv_tile(const PrefillParams& p, const Item& it, const CUtensorMap* map,
                                             uint32_t dst, uint32_t full_bar, int key0, int lane) {
  if (p.table == nullptr) {
    if (lane == 0) {
      mbar_expect_tx(full_bar, R * kKVRegion);
#pragma unroll
      for (int r = 0; r < R; ++r) tma_load_3d(dst + r * kKVRegion, map, full_bar, r * 64, it.kh, it.k_begin + key0);
    }
    __syncwarp();
    return;
  }
  const int nb = BN / p.box_rows;
  if (lane == 0) mbar_expect_tx(full_bar, R * kKVRegion);
  __syncwarp();
  for (int bx = lane; bx < R * nb; bx += 32) {
    const int r = bx / nb, c = bx - r * nb;
    const int pos = key0 + c * p.box_rows;
    const int pg = pos >> p.page_shift;
    int blk = -1;
    if (pos < it.k_len && pg < p.bt_cols) blk = __ldg(p.table + (int64_t)it.b * p.bt0 + (int64_t)pg * p.bt1);
    tma_load_4d(dst + r * kKVRegion + c * p.box_rows * 128, map, full_bar, r * 64, it.kh,
                pos & ((1 << p.page_shift) - 1), blk);
  }
  __syncwarp();
}

// DQK / DV: padded QK and V head dims (multiples of 64); the tensor maps
// carry the true dims, so padded columns load as zeros and are never stored.
template <bool BF16, bool SOFTCAP, int DQK, int DV>
__global__ void __launch_bounds__(kWThreads, 1)
    prefill_wide_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv, const PrefillParams p) {
  using L = WideLayout<DQK, DV>;
  constexpr int RQ = L::RQ, RV = L::RV;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_work = p.n_pairs * p.HQ * p.B;
  auto bar = [&](int i) { return base + L::OFF_BAR + 8u * (uint32_t)i; };
  const uint32_t holder = base + L::OFF_BAR + 8u * W_COUNT;
  volatile uint32_t* holder_ptr = reinterpret_cast<volatile uint32_t*>(gbase + L::OFF_BAR + 8 * W_COUNT);
  volatile int* wring = reinterpret_cast<volatile int*>(gbase + L::OFF_BAR + 8 * W_COUNT + 16);
  volatile int* iring =  // [NWORK][20], 16-byte aligned
      reinterpret_cast<volatile int*>(gbase + ((L::OFF_BAR + 8 * W_COUNT + 32 + 15) & ~15));
  // Work ids flow from warp 4 (which claims them, heaviest first) to the MMA
  // warp, the V loader and the 4 softmax warps through a ring.
  auto next_work = [&](uint32_t& cnt, Item& it) -> int {
    const uint32_t slot = cnt % NWORK;
    if (!wwait(bar(W_WFULL + slot), (cnt / NWORK) & 1)) return -2;
    const int w = wring[slot];
    item_load(iring + slot * kItemWords, it);
    __syncwarp();
    if (lane == 0) mbar_arrive(bar(W_WEMPTY + slot));
    ++cnt;
    return w;
  };

  if (threadIdx.x == 0) {
    for (int b : {W_Q, W_QE, W_KF, W_KE, W_VF, W_VE, W_SF, W_PVD, W_OD, W_FIN}) mbar_init(bar(b), 1);
    mbar_init(bar(W_SC), 4);  // one arrival per softmax warp
    mbar_init(bar(W_PF), 4);
    for (int s = 0; s < NWORK; ++s) {
      mbar_init(bar(W_WFULL + s), 1);
      mbar_init(bar(W_WEMPTY + s), 6);  // MMA warp + V loader + 4 softmax warps
    }
    mbar_fence_init();
  }
  if (warp == 5) {
    tmem_alloc(holder, kWTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *holder_ptr;

  if (warp == 4) {
    // -------------------------------------------------------- Q and K loads
    uint32_t kloads = 0, qloads = 0, fwd = 0;
    bool ok = true;
    if (lane == 0) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
    }
    while (ok) {
      int w = 0;
      if (lane == 0) w = atomicAdd(p.counter, 1);
      w = __shfl_sync(0xffffffffu, w, 0);
      const bool end = w >= n_work;
      const Item it = make_wide_item(p, end ? 0 : w);
      if (!end && !it.valid) continue;
      {
        const uint32_t slot = fwd % NWORK;
        if (fwd >= NWORK && !(ok = wwait(bar(W_WEMPTY + slot), ((fwd / NWORK) - 1) & 1))) break;
        if (lane == 0) {
          wring[slot] = end ? -1 : w;
          item_store(iring + slot * kItemWords, it);
          mbar_arrive(bar(W_WFULL + slot));
        }
        __syncwarp();
        ++fwd;
      }
      if (end) break;
      if (it.n_all == 0) continue;
      // The previous item's last QK^T must be done before its Q is replaced.
      if (qloads > 0 && !(ok = wwait(bar(W_QE), (qloads - 1) & 1))) break;
      if (lane == 0) {
        mbar_expect_tx(bar(W_Q), RQ * kRegion);
#pragma unroll
        for (int r = 0; r < RQ; ++r)
          tma_load_3d(base + L::OFF_Q + r * kRegion, &tq, bar(W_Q), r * 64, it.h, it.q_begin + it.row_a);
      }
      __syncwarp();
      ++qloads;
      for (int t = 0; t < it.n_all; ++t) {
        if (kloads > 0 && !(ok = wwait(bar(W_KE), (kloads - 1) & 1))) break;
        load_kv_tile<RQ>(p, it, &tk, base + L::OFF_K, bar(W_KF), (it.j_first + t) * BN, lane);
        ++kloads;
      }
    }
    // Drain: every issued load must have landed before the CTA exits.
    if (qloads > 0) wwait(bar(W_Q), (qloads - 1) & 1);
    if (kloads > 0) wwait(bar(W_KF), (kloads - 1) & 1);
  } else if (warp == 6) {
    // ---------------------------------------------------------------- V loads
    uint32_t vloads = 0, wcnt = 0;
    bool ok = true;
    if (lane == 0) tma_prefetch_desc(&tv);
    while (ok) {
      Item it;
      const int w = next_work(wcnt, it);
      if (w < 0) break;
      for (int t = 0; t < it.n_all; ++t) {
        if (vloads > 0 && !(ok = wwait(bar(W_VE), (vloads - 1) & 1))) break;
        load_kv_tile<RV>(p, it, &tv, base + L::OFF_V, bar(W_VF), (it.j_first + t) * BN, lane);
        ++vloads;
      }
    }
    if (vloads > 0) wwait(bar(W_VF), (vloads - 1) & 1);
  } else if (warp == 5) {
    // ---------------------------------------------------------------- MMA
    const uint32_t idesc_qk = f16_idesc(BM, BN, BF16 ? 1 : 0, 0);
    const uint32_t idesc_pv = f16_idesc(BM, DV, BF16 ? 1 : 0, 1);
    uint32_t wcnt = 0, qc = 0, kc = 0, vc = 0, nqk = 0, npv = 0;
    bool ok = true;
    auto commit = [&](int b) {
      if (lane == 0) mma_commit(bar(b));
      __syncwarp();
    };
    // QK^T of the next key tile into S, once the softmax has loaded the
    // previous S and the K tile has landed (false on timeout).
    auto issue_qk = [&]() {
      if (nqk > 0 && !wwait(bar(W_SC), (nqk - 1) & 1)) return false;
      if (!wwait(bar(W_KF), kc & 1)) return false;
      ++kc;
      tc_fence_after();
      if (lane == 0) {
#pragma unroll
        for (int kk = 0; kk < DQK / 16; ++kk) {
          const uint64_t a = sw128_desc(base + L::OFF_Q + (kk >> 2) * kRegion + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sw128_desc(base + L::OFF_K + (kk >> 2) * kKVRegion + (kk & 3) * 32, 16, 1024);
          mma_f16_ss(tmem, a, bd, idesc_qk, kk > 0 ? 1u : 0u);
        }
        mma_commit(bar(W_SF));
        mma_commit(bar(W_KE));
      }
      __syncwarp();
      ++nqk;
      return true;
    };
    // PV of the current P once it is in tensor memory and V has landed.
    auto issue_pv = [&](bool acc) {
      if (!wwait(bar(W_VF), vc & 1)) return false;
      ++vc;
      if (!wwait(bar(W_PF), npv & 1)) return false;
      tc_fence_after();
      if (lane == 0) {
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t bd = sw128_desc(base + L::OFF_V + kk * 2048, kKVRegion, 1024);
          mma_f16_ts(tmem + kColO, tmem + kColP + kk * 8, bd, idesc_pv, (acc || kk > 0) ? 1u : 0u);
        }
        mma_commit(bar(W_PVD));
        mma_commit(bar(W_VE));
      }
      __syncwarp();
      ++npv;
      return true;
    };
    // Next item with key tiles: 1, 0 at the end of the work, -1 on a timeout.
    auto fetch = [&](Item& it) {
      while (true) {
        const int w = next_work(wcnt, it);
        if (w == -2) return -1;
        if (w < 0) return 0;
        if (it.n_all > 0) return 1;
      }
    };
    // Q of an item landed, then QK^T of its first key tile.
    auto first_qk = [&](const Item& it) {
      if (!wwait(bar(W_Q), qc & 1)) return false;
      ++qc;
      if (!issue_qk()) return false;
      if (it.n_all == 1) commit(W_QE);
      return true;
    };
    Item cur;
    int have = fetch(cur);
    if (have == 1) ok = first_qk(cur);
    while (ok && have == 1) {
      Item nxt;
      int have_next = 0;
      for (int t = 0; ok && t < cur.n_all; ++t) {
        if (t + 1 < cur.n_all) {
          // Scores of key tile j+1 while the softmax works on j.
          if (!(ok = issue_qk())) break;
          if (t + 2 == cur.n_all) commit(W_QE);  // the item's last QK^T has been issued
        } else {
          // Last key tile: the next item's first scores before the last PV.
          have_next = fetch(nxt);
          if (have_next < 0) {
            ok = false;
            break;
          }
          if (have_next == 1 && !(ok = first_qk(nxt))) break;
        }
        if (!(ok = issue_pv(t > 0))) break;
        if (t + 1 == cur.n_all) commit(W_OD);
      }
      cur = nxt;
      have = have_next;
    }
    // All MMAs of this CTA must be complete before TMEM is released.
    commit(W_FIN);
    wwait(bar(W_FIN), 0);
  } else if (warp < 4) {
    // ------------------------------------------------------------ softmax
    const int row = warp * 32 + lane;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const uint32_t tS = tmem + lane_off, tP = tmem + kColP + lane_off, tO = tmem + kColO + lane_off;
    // s_cnt: score tiles consumed = P tiles published = V tiles used.
    uint32_t s_cnt = 0, o_cnt = 0, wcnt = 0;
    bool ok = true;
    while (ok) {
      Item it;
      const int w = next_work(wcnt, it);
      if (w < 0) break;
      const int x0 = it.j_first, n_x = it.n_all;
      const int q_row = it.row_a + row;
      const int q_abs = q_row + it.k_len - it.q_len;
      const KeyRange vis = key_range(q_abs, it.k_len, it.causal, p.win_l, p.win_r);
      const int h = it.h;
      const float qk_scale = it.qk_scale, vscale = it.vscale;
      const float sl2 = qk_scale * 1.4426950408889634f;     // raw score -> log2 units
      const float cap_l2 = p.softcap * 1.4426950408889634f;  // softcap: cap*log2e*tanh(s*scale/cap)
      const float cap_in = SOFTCAP ? qk_scale / p.softcap : 0.f;
      // Scores up to this magnitude take the softcap's FMA-pipe polynomial.
      const float cap_lim = SOFTCAP ? softcap_poly_limit(cap_in) : -1.f;
      // Running max in log2 units; a sink acts as one extra logit with zero value.
      float m_run = p.sinks ? load_float(p.sinks, p.sink_t, h * p.si0) * 1.4426950408889634f : -INFINITY;
      float l_run = p.sinks ? 1.f : 0.f;
      for (int jj = 0; jj < n_x; ++jj) {
        const int j = x0 + jj;
        if (!(ok = wwait(bar(W_SF), s_cnt & 1))) break;
        tc_fence_after();
        const int key0 = j * BN;
        const int c_lo = vis.lo - key0, c_hi = vis.hi - key0;  // visible columns of this tile
        const bool need_mask = c_lo > 0 || c_hi < BN - 1;
        uint32_t r[BN];
        tmem_ld32_at<0>(tS, r);
        tmem_ld32_at<32>(tS + 32, r);
        tmem_ld32_at<64>(tS + 64, r);
        tmem_ld32_at<96>(tS + 96, r);
        tmem_wait_ld();
        // S is in registers: the MMA warp may compute the next scores into it.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(W_SC));
        // Softcap route for this tile, uniform over the warp: the polynomial
        // tanh when every raw score of the warp's 32 rows (masked columns
        // included) has |s * scale / cap| <= 3/4, else the identity route.
        bool cap_poly = false;
        if constexpr (SOFTCAP) cap_poly = __all_sync(0xffffffffu, row_absmax(r) <= cap_lim);
        if (need_mask) {
#pragma unroll
          for (int i = 0; i < BN; ++i)
            if (i < c_lo || i > c_hi) r[i] = __float_as_uint(-INFINITY);
        }
        // Row max as 8 independent 3-input max chains (exact in any order).
        float mx8[8];
#pragma unroll
        for (int k8 = 0; k8 < 8; ++k8) mx8[k8] = -INFINITY;
#pragma unroll
        for (int i = 0; i < BN; i += 2)
          mx8[(i >> 1) & 7] = max3(mx8[(i >> 1) & 7], __uint_as_float(r[i]), __uint_as_float(r[i + 1]));
        const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                               fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
        // scale > 0 and tanh is increasing: the max commutes with both.
        const float m_tile = SOFTCAP ? (mx == -INFINITY ? -INFINITY : cap_l2 * tanh_id(mx * cap_in)) : mx * sl2;
        float factor = 1.f;
        if (m_tile > m_run + kRescaleThreshold || (m_run == -INFINITY && m_tile != -INFINITY)) {
          factor = m_run == -INFINITY ? 0.f : ex2(m_run - m_tile);
          m_run = m_tile;
        }
        l_run *= factor;
        const float msub = m_run == -INFINITY ? 0.f : m_run;
        // P = 2^(s*scale_log2 - m) as 16-bit pairs in registers; the row sum as
        // 8 independent chains (4 packed pairs).
        uint64_t ls2[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) ls2[i] = f2pack(0.f, 0.f);
        const uint64_t nmsub2 = f2pack(-msub, -msub);
        uint32_t pk[BN / 2];
        // kMode 0: plain scores; 1: softcap by the polynomial tanh; 2: softcap
        // by the identity (one route per warp and tile, see cap_poly).
        auto exp_stage = [&](auto mode) {
          constexpr int kMode = decltype(mode)::value;
          const uint64_t sl2x2 = f2pack(sl2, sl2);
          const uint64_t tanh_k2 = f2pack(cap_in * 2.8853900817779268f, cap_in * 2.8853900817779268f);
          const uint64_t one2 = f2pack(1.f, 1.f), neg_two2 = f2pack(-2.f, -2.f), cap_l2x2 = f2pack(cap_l2, cap_l2);
#pragma unroll
          for (int i = 0; i < BN / 2; ++i) {
            float p0, p1;
            const float s0 = __uint_as_float(r[2 * i]), s1 = __uint_as_float(r[2 * i + 1]);
            if constexpr (kMode == 1) {
              // cap*log2e*tanh(s*scale/cap) - m by the polynomial, one MUFU ex2.
              const TanhPoly tpoly(sl2, cap_in);
              float l0, l1;
              f2unpack(tpoly.fma(f2pack(s0, s1), nmsub2), l0, l1);
              p0 = ex2(l0);  // a masked score gives l = -inf exactly: p = 0
              p1 = ex2(l1);
            } else if constexpr (kMode == 2) {
              // cap*log2e*tanh(s*scale/cap) - m with tanh(y) = 1 - 2/(e^(2y)+1).
              const Exp2Poly<false> tanh_poly;  // degree 4: tanh error ~3e-6
              float u0, u1;
              f2unpack(fmul2(f2pack(s0, s1), tanh_k2), u0, u1);
              float e0, e1;
              tanh_poly.in_range(f2pack(fminf(fmaxf(u0, -64.f), 64.f), fminf(fmaxf(u1, -64.f), 64.f)), e0, e1);
              float d0, d1;
              f2unpack(fadd2(f2pack(e0, e1), one2), d0, d1);
              const uint64_t t2 = ffma2(f2pack(rcp(d0), rcp(d1)), neg_two2, one2);
              float l0, l1;
              f2unpack(ffma2(t2, cap_l2x2, nmsub2), l0, l1);
              p0 = s0 == -INFINITY ? 0.f : ex2(l0);
              p1 = s1 == -INFINITY ? 0.f : ex2(l1);
            } else {
              float x0, x1;
              f2unpack(ffma2(f2pack(s0, s1), sl2x2, nmsub2), x0, x1);
              p0 = ex2(x0);
              p1 = ex2(x1);
            }
            ls2[i & 3] = fadd2(ls2[i & 3], f2pack(p0, p1));
            pk[i] = pack_p<BF16>(p0, p1);
          }
        };
        if constexpr (SOFTCAP) {
          if (cap_poly) exp_stage(std::integral_constant<int, 1>());
          else exp_stage(std::integral_constant<int, 2>());
        } else {
          exp_stage(std::integral_constant<int, 0>());
        }
        // The previous PV must have read its P and added into O before P is
        // replaced and O rescaled.
        if (s_cnt > 0) {
          if (!(ok = wwait(bar(W_PVD), (s_cnt - 1) & 1))) break;
          tc_fence_after();
        }
        ++s_cnt;
        // Lazy O rescale.
        if (jj > 0 && __any_sync(0xffffffffu, factor != 1.f)) {
#pragma unroll
          for (int c = 0; c < DV / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(tO + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
            tmem_st32(tO + c * 32, o);
          }
        }
        tmem_st32_at<0>(tP, pk);
        tmem_st32_at<32>(tP + 32, pk);
        tmem_wait_st();
        float ls8[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) f2unpack(ls2[i], ls8[2 * i], ls8[2 * i + 1]);
        l_run += ((ls8[0] + ls8[1]) + (ls8[2] + ls8[3])) + ((ls8[4] + ls8[5]) + (ls8[6] + ls8[7]));
        if (key0 + BN > it.k_len) {
          // Keys past the sequence in the last tile: zero their V rows so that
          // a non-finite neighbour value never meets a zero probability.
          if (!(ok = wwait(bar(W_VF), (s_cnt - 1) & 1))) break;
          if (key0 + row >= it.k_len) {
            uint8_t* vrow = gbase + L::OFF_V + row * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
#pragma unroll
              for (int rv = 0; rv < RV; ++rv)
                *reinterpret_cast<uint4*>(vrow + rv * kKVRegion + c * 16) = make_uint4(0, 0, 0, 0);
            }
          }
          fence_proxy_async_smem();  // generic stores -> the MMA's async-proxy reads
        }
        // P of every lane is in tensor memory; one lane publishes the warp's rows.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(W_PF));
      }
      if (!ok) break;
      if (n_x > 0) {
        if (!(ok = wwait(bar(W_OD), o_cnt & 1))) break;
        ++o_cnt;
        tc_fence_after();
      }
      // ---------------------------------------------------------- epilogue
      // O / l in bf16/f16, each thread writing its own row (32 columns at a
      // time from tensor memory).
      const bool row_ok = q_row < it.q_len;
      const int64_t t = (int64_t)it.q_begin + q_row;
      const bool have = n_x > 0 && l_run > 0.f;
      const float inv = have ? vscale / l_run : 0.f;
      uint8_t* orow = reinterpret_cast<uint8_t*>(p.out) + (t * p.os0 + (int64_t)h * p.os1) * 2;
#pragma unroll
      for (int c = 0; c < DV / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + c * 32, o);
        tmem_wait_ld();
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint32_t wv[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float a = have ? __uint_as_float(o[v * 8 + 2 * i]) * inv : 0.f;
            const float bb = have ? __uint_as_float(o[v * 8 + 2 * i + 1]) * inv : 0.f;
            wv[i] = pack_p<BF16>(a, bb);
          }
          if (row_ok && c * 32 + v * 8 < p.dim)
            *reinterpret_cast<uint4*>(orow + (c * 32 + v * 8) * 2) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
        }
      }
      if (row_ok) p.lse[(int64_t)h * p.ls0 + t * p.ls1] = l_run > 0.f ? (m_run + log2f(l_run)) * kLn2 : -INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, kWTmemCols);
  }
}

template <int DQK, int DV>
void* pick_wide(bool bf16, bool cap) {
  if (bf16)
    return cap ? reinterpret_cast<void*>(prefill_wide_kernel<true, true, DQK, DV>)
               : reinterpret_cast<void*>(prefill_wide_kernel<true, false, DQK, DV>);
  return cap ? reinterpret_cast<void*>(prefill_wide_kernel<false, true, DQK, DV>)
             : reinterpret_cast<void*>(prefill_wide_kernel<false, false, DQK, DV>);
}

}  // namespace

// QK head dims 129..256 and V head dims up to 256, multiples of 8 (16-byte
// rows), packed or paged K/V, no ALiBi; the other conditions (page sizes,
// strides, alignment) are those of the two-tile kernel (checked by the caller).
bool prefill_wide_dims(const AttnParams& p) {
  return p.DQ > 128 && p.DQ <= 256 && p.DV >= 8 && p.DV <= 256 && p.DQ % 8 == 0 && p.DV % 8 == 0;
}

int prefill_wide_supported(const AttnParams& p) {
  if (!prefill_wide_dims(p)) return 0;
  if (p.alibi) return 0;
  return 1;
}

int prefill_wide_timeout_flag(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_prefill_wide_timeout, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_prefill_wide_timeout, &zero, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

int launch_prefill_wide(const AttnParams& p, const PrefillParams& pp_in, cudaStream_t stream) {
  CUtensorMap mq, mk, mv;
  int rc = make_map(&mq, p.q, p.qt, p.DQ, p.T, p.HQ, p.qs0, p.qs1);
  if (rc) return rc;
  if (p.paged) {
    rc = make_page_map(&mk, p.k, p.kt, p.DQ, p.HK, p.page, p.k_pages, p.ks0, p.ks1, p.ks2, pp_in.box_rows);
    if (rc) return rc;
    rc = make_page_map(&mv, p.v, p.vt, p.DV, p.HK, p.page, p.k_pages, p.vs0, p.vs1, p.vs2, pp_in.box_rows);
  } else {
    rc = make_map(&mk, p.k, p.kt, p.DQ, p.k_rows, p.HK, p.ks1, p.ks2, BN);
    if (rc) return rc;
    rc = make_map(&mv, p.v, p.vt, p.DV, p.k_rows, p.HK, p.vs1, p.vs2, BN);
  }
  if (rc) return rc;
  PrefillParams pp = pp_in;
  pp.n_pairs = (p.max_q + BM - 1) / BM;
  pp.head_pairs = 0;
  pp.dim = p.DV;
  const bool bf16 = p.qt == FA_BF16, cap = p.softcap > 0.f;
  void* kernel;
  int smem;
  if (p.DQ <= 192) {
    if (p.DV <= 128) { kernel = pick_wide<192, 128>(bf16, cap); smem = WideLayout<192, 128>::kSmem; }
    else { kernel = pick_wide<192, 256>(bf16, cap); smem = WideLayout<192, 256>::kSmem; }
  } else {
    if (p.DV <= 128) { kernel = pick_wide<256, 128>(bf16, cap); smem = WideLayout<256, 128>::kSmem; }
    else { kernel = pick_wide<256, 256>(bf16, cap); smem = WideLayout<256, 256>::kSmem; }
  }
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return fail(FA_ERR_CUDA, "wide prefill smem attribute: %s", cudaGetErrorString(e));
  const int64_t n_work = (int64_t)pp.n_pairs * p.HQ * p.B;
  const int grid = (int)std::min<int64_t>(n_work, (int64_t)sm_count());
  if (pp.counter == nullptr) return fail(FA_ERR_INVALID, "prefill needs its workspace counter");
  e = cudaMemsetAsync(pp.counter, 0, sizeof(int), stream);
  if (e != cudaSuccess) return fail(FA_ERR_CUDA, "prefill counter reset: %s", cudaGetErrorString(e));
  void* args[] = {&mq, &mk, &mv, &pp};
  e = cudaLaunchKernel(kernel, dim3(grid), dim3(kWThreads), args, smem, stream);
  note_launch();
  if (e != cudaSuccess) return fail(FA_ERR_CUDA, "wide prefill launch: %s", cudaGetErrorString(e));
  return FA_OK;
}

}  // namespace fab
