// Varlen / dense prefill on 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Persistent CTAs (one per SM) claim work items -- a pair of 128-row query
// tiles (A, B) of one (request, query head) -- from an atomic counter,
// heaviest causal pairs first. Per CTA:
//   warp 8      TMA producer: Q_A/Q_B once per item, then K(j), V(j), ... as
//               128-key tiles into an NSLOT-deep ring of 128-byte swizzled
//               boxes (64 head dims each).
//   warp 9      TMEM owner and MMA issuer: S = Q K^T from shared memory and
//               O += P V with P read from tensor memory, as tcgen05.mma
//               kind::f16 (M=128, N=128, K=16 per instruction); fp32 S_A,
//               S_B, O_A, O_B in TMEM (4 x 128 columns).
//   warps 0..3  softmax of tile A, warps 4..7 softmax of tile B: each thread
//               owns one query row (its TMEM lane), loads its S row with
//               tcgen05.ld, applies scale, softcap and the lower-right
//               causal / window / length masks, runs the online softmax in
//               the log2 domain (lazy rescale of its O row in TMEM when the
//               max grows by more than 2^8), and stores P as packed 16-bit
//               pairs over the first 64 columns of its own S row
//               (tcgen05.st). P never touches shared memory, so the tensor
//               cores' shared-memory operand traffic is Q, K and V only.
// The MMA warp issues PV(j) of tile A, then QK(j+1) of tile A (which reuses
// S_A's columns after PV(j) has read P; one thread's tcgen05 MMAs execute in
// issue order), then the same for tile B, so either warpgroup's exponentials
// overlap the other tile's MMAs.
// Every mbarrier wait is bounded; on a timeout the kernel records a flag,
// drains its own TMA loads and MMAs, frees TMEM and returns.
//
// Semantics (lower-right causal, natural-log LSE, zero output and -inf LSE
// for rows with no visible key) follow the reference's fast kernel
// flash_attn_mps/kernels/attention_fast.metal:94-597 and its eligibility
// predicate flash_attn_mps/_attention.py:149-158.
#include <algorithm>
#include <type_traits>
#include <mutex>

#include "kernels.cuh"
#include "prefill_common.cuh"
#include "sm100.cuh"

namespace fab {
namespace {

using namespace sm100;
using namespace pf;

// One S/P buffer per query tile (its 128 TMEM columns hold one 128-key score
// tile). A 64-key variant with two S buffers per tile (QK^T of key tile j+2
// while the softmax works on j) was measured and removed: a tcgen05.mma of
// M=128, K=16 costs ~100 cycles at N=64 as at N=128, so the 64-key schedule
// ran at 648 against 1160 TFLOP/s non-causal.
constexpr int SBUF = 1;
#ifndef FAB_PREFILL_NSLOT
#define FAB_PREFILL_NSLOT 0
#endif
// K/V ring slots (each holds one K or one V tile), 96 KB in all. With SBUF = 2
// the MMA warp needs K(j+2) before it releases V(j): at least 4 slots.
constexpr int NSLOT = FAB_PREFILL_NSLOT > 0 ? FAB_PREFILL_NSLOT : 3 * SBUF;
static_assert(SBUF == 1 || NSLOT >= 4, "ring too shallow for the QK look-ahead");
constexpr int kTileBytes = 2 * kRegion;       // 128 x 128 bf16 Q tile
constexpr int kKVTileBytes = 2 * kKVRegion;   // BN x 128 bf16 K or V tile
constexpr int kThreads = 384;                 // 2 softmax warpgroups + (TMA, MMA, 2 idle) warpgroup
// Registers: the CTA launches with kLaunchRegs per thread (checked on the host
// before every launch); the producer warpgroup gives registers back and the
// softmax warpgroups take them, so that each softmax thread holds its whole
// 128-column S row. 8 warps x 208 + 4 warps x 88 = 12 warps x 168.
constexpr int kLaunchRegs = 168;

#ifndef FAB_PF_SM_REGS
#define FAB_PF_SM_REGS 208
#endif
#ifndef FAB_PF_PR_REGS
#define FAB_PF_PR_REGS 88
#endif
constexpr int kSoftmaxRegs = FAB_PF_SM_REGS;
constexpr int kProducerRegs = FAB_PF_PR_REGS;
static_assert(8 * kSoftmaxRegs + 4 * kProducerRegs <= (kThreads / 32) * kLaunchRegs, "register split");
static_assert(kLaunchRegs * kThreads <= 65536, "launch registers");
constexpr int OFF_QA = 0;
constexpr int OFF_QB = OFF_QA + kTileBytes;
constexpr int OFF_RING = OFF_QB + kTileBytes;
constexpr int OFF_STAGE = OFF_RING + NSLOT * kKVTileBytes;  // 8 softmax warps x [2][32 rows][128 B]
constexpr int kStageWarpBytes = 2 * 32 * 128;
constexpr int OFF_BAR = OFF_STAGE + 8 * kStageWarpBytes;
// Barriers, TMEM holder, work-id ring and item ring, then alignment slack.
constexpr int kSmemBytes = OFF_BAR + 1024 + 1024;
constexpr uint32_t kTmemCols = 512;           // S_A, S_B, O_A, O_B (128 fp32 columns each; S as SBUF tiles)
#ifndef FAB_PREFILL_POLY_PAIRS
#define FAB_PREFILL_POLY_PAIRS 0
#endif
// Of every 8 exponential pairs, how many run on the FMA pipe (Exp2Poly)
// instead of MUFU ex2. Measured on B200 with the single-pass softmax: 0 is
// fastest (2 and 4 pairs cost 3% and 8%: the softmax is issue-, not
// MUFU-bound), so the default keeps every exponential on MUFU.
constexpr int kPolyPairs = FAB_PREFILL_POLY_PAIRS;

// Per query tile t (0 = A, 1 = B) and S buffer b: B_SF + t*SBUF + b (scores
// ready), B_PF + t*SBUF + b (P ready, 128 arrivals); B_PVD + t (a PV finished).
enum {
  B_Q = 0, B_QE, B_FULL, B_EMPTY = B_FULL + NSLOT, B_SF = B_EMPTY + NSLOT, B_PF = B_SF + 2 * SBUF,
  B_PVD = B_PF + 2 * SBUF, B_ODA = B_PVD + 2, B_ODB, B_FIN, B_WFULL, B_WEMPTY = B_WFULL + NWORK,
  B_COUNT = B_WEMPTY + NWORK
};

__device__ int g_prefill_timeout;

__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity) {  // flag: g_prefill_timeout
  bool ok = mbar_wait(bar, parity, &g_prefill_timeout);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ Item make_item(const PrefillParams& p, int w) {
  Item it;
  const int hsteps = p.HQ >> p.head_pairs;  // query heads, or head pairs
  // Work order: groups of group_reqs requests, whose K/V stay in L2 while the
  // CTAs work through them; within a group row blocks heaviest first, then
  // head (pair), then request.
  const int per_group = p.n_pairs * hsteps * p.group_reqs;
  const int g = w / per_group;
  const int local = w - g * per_group;
  const int b0 = g * p.group_reqs;
  const int per = hsteps * min(p.group_reqs, p.B - b0);
  const int pair = p.n_pairs - 1 - local / per;
  const int rem = local - (local / per) * per;
  it.h = (rem % hsteps) << p.head_pairs;
  it.h_b = it.h + p.head_pairs;
  it.b = b0 + rem / hsteps;
  it.q_begin = p.cu_q[it.b * p.cq0];
  it.q_len = p.cu_q[(it.b + 1) * p.cq0] - it.q_begin;
  it.row_a = pair * (p.head_pairs ? BM : 2 * BM);
  it.row_b = it.row_a + (p.head_pairs ? 0 : BM);
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
  tile_range(it.row_b, it.q_len, it.k_len, it.causal, p.win_l, p.win_r, &it.b0, &it.b1);
  const bool ha = it.a1 > it.a0, hb = it.b1 > it.b0;
  if (!ha && !hb) return it;
  it.j_first = ha ? (hb ? min(it.a0, it.b0) : it.a0) : it.b0;
  const int j_last = max(ha ? it.a1 : 0, hb ? it.b1 : 0);
  it.n_all = j_last - it.j_first;
  return it;
}

// HDIM: head dim (64 or 128) = number of 64-element swizzle regions x 64.
// ALIBI: scores minus slope * |q_abs - key|; with SOFTCAP as well, the
// softcapped score minus the bias (the softcap then runs before the row max).
template <bool BF16, bool SOFTCAP, int HDIM, bool ALIBI>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_sm100_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                         const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap to,
                         const PrefillParams p) {
  static_assert(HDIM == 64 || HDIM == 128, "head dim");
  // Softcap in the exponential stage (its max commutes with tanh); with ALiBi
  // the capped and biased scores are formed before the row max instead.
  constexpr bool CAP_IN_EXP = SOFTCAP && !ALIBI;
  constexpr int kHalves = HDIM / 64;             // 64-element regions per row
  constexpr int kLoadBytes = kHalves * kRegion;      // bytes of one Q tile actually loaded
  constexpr int kKVLoadBytes = kHalves * kKVRegion;  // bytes of one K/V tile actually loaded
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_work = p.n_pairs * (p.HQ >> p.head_pairs) * p.B;
  auto bar = [&](int i) { return base + OFF_BAR + 8u * (uint32_t)i; };
  const uint32_t holder = base + OFF_BAR + 8u * B_COUNT;
  volatile uint32_t* holder_ptr = reinterpret_cast<volatile uint32_t*>(gbase + OFF_BAR + 8 * B_COUNT);
  volatile int* wring = reinterpret_cast<volatile int*>(gbase + OFF_BAR + 8 * B_COUNT + 16);
  volatile int* iring =  // [NWORK][20], 16-byte aligned
      reinterpret_cast<volatile int*>(gbase + ((OFF_BAR + 8 * B_COUNT + 32 + 15) & ~15));
  // Work ids flow from the TMA warp (which claims them with an atomic counter,
  // heaviest first) to the MMA warp and the 8 softmax warps through a ring.
  auto next_work = [&](uint32_t& cnt, Item& it) -> int {
    const uint32_t slot = cnt % NWORK;
    if (!warp_wait(base + OFF_BAR + 8u * (B_WFULL + slot), (cnt / NWORK) & 1)) return -2;
    const int w = wring[slot];
    item_load(iring + slot * kItemWords, it);
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
    for (int b = 0; b < 2 * SBUF; ++b) {
      mbar_init(bar(B_SF + b), 1);
      mbar_init(bar(B_PF + b), 128);
    }
    mbar_init(bar(B_PVD), 1);
    mbar_init(bar(B_PVD + 1), 1);
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

  if (warp >= 8) {
  // Producer warpgroup: TMA warp, MMA warp and two idle warps.
  reg_dealloc<kProducerRegs>();
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
          item_store(iring + slot * kItemWords, it);
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
        mbar_expect_tx(bar(B_Q), 2 * kLoadBytes);
#pragma unroll
        for (int hf = 0; hf < kHalves; ++hf) {
          tma_load_3d(base + OFF_QA + hf * kRegion, &tq, bar(B_Q), hf * 64, it.h, it.q_begin + it.row_a);
          tma_load_3d(base + OFF_QB + hf * kRegion, &tq, bar(B_Q), hf * 64, it.h_b, it.q_begin + it.row_b);
        }
      }
      ++qloads;
      for (int i = 0; i < 2 * it.n_all; ++i) {  // K(j), V(j), K(j+1), ...
        const uint32_t slot = items % NSLOT;
        if (items >= NSLOT && !(ok = warp_wait(bar(B_EMPTY + slot), ((items / NSLOT) - 1) & 1))) break;
        const CUtensorMap* map = (i & 1) ? &tv : &tk;
        const uint32_t dst = base + OFF_RING + slot * kKVTileBytes;
        if (p.table == nullptr) {
          if (lane == 0) {
            const int row = it.k_begin + (it.j_first + (i >> 1)) * BN;
            mbar_expect_tx(bar(B_FULL + slot), kKVLoadBytes);
#pragma unroll
            for (int hf = 0; hf < kHalves; ++hf)
              tma_load_3d(dst + hf * kKVRegion, map, bar(B_FULL + slot), hf * 64, it.kh, row);
          }
        } else {
          // Paged K/V: the tile's BN keys arrive as page boxes (box_rows
          // tokens x 64 head dims each, one lane per box) through
          // block_table; pages past the sequence or the table use page -1,
          // which TMA fills with zeros.
          const int nb = BN / p.box_rows;
          const int key0 = (it.j_first + (i >> 1)) * BN;
          if (lane == 0) mbar_expect_tx(bar(B_FULL + slot), kKVLoadBytes);
          __syncwarp();
          if (lane < kHalves * nb) {
            const int half = lane / nb, c = lane - half * nb;
            const int pos = key0 + c * p.box_rows;
            const int pg = pos >> p.page_shift;
            int blk = -1;
            if (pos < it.k_len && pg < p.bt_cols) blk = __ldg(p.table + (int64_t)it.b * p.bt0 + (int64_t)pg * p.bt1);
            tma_load_4d(dst + half * kKVRegion + c * p.box_rows * 128, map, bar(B_FULL + slot), half * 64, it.kh,
                        pos & ((1 << p.page_shift) - 1), blk);
          }
          __syncwarp();
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
    const uint32_t idesc_pv = f16_idesc(BM, HDIM, BF16 ? 1 : 0, 1);
    auto slot_addr = [&](uint32_t item) { return base + OFF_RING + (item % NSLOT) * kKVTileBytes; };
    auto wait_item = [&](uint32_t item) { return warp_wait(bar(B_FULL + item % NSLOT), (item / NSLOT) & 1); };
    // S tile number n of query tile t lives in TMEM columns t*128 + (n % SBUF)*BN.
    auto s_tmem = [&](int t, uint32_t n) { return tmem + (uint32_t)(t * 128) + (n % SBUF) * (uint32_t)BN; };
    auto qk = [&](uint32_t q_off, uint32_t kaddr, uint32_t d, int sfbar) {
      if (lane == 0) {
#pragma unroll
        for (int kk = 0; kk < HDIM / 16; ++kk) {
          const uint64_t a = sw128_desc(base + q_off + (kk >> 2) * kRegion + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sw128_desc(kaddr + (kk >> 2) * kKVRegion + (kk & 3) * 32, 16, 1024);
          mma_f16_ss(d, a, bd, idesc_qk, kk > 0 ? 1u : 0u);
        }
        mma_commit(bar(sfbar));
      }
      __syncwarp();
    };
    // P (M=128 rows x K=BN keys) is the A operand in TMEM: 16 keys = 8 columns.
    auto pv = [&](uint32_t p_tmem, uint32_t vaddr, uint32_t d, bool acc) {
      if (lane == 0) {
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t bd = sw128_desc(vaddr + kk * 2048, kKVRegion, 1024);
          mma_f16_ts(d, p_tmem + kk * 8, bd, idesc_pv, (acc || kk > 0) ? 1u : 0u);
        }
      }
      __syncwarp();
    };
    auto commit = [&](int barid) {
      if (lane == 0) mma_commit(bar(barid));
      __syncwarp();
    };
    // Per query tile t: nq[t] QK^T and np[t] PV issued so far (S buffer and
    // barrier phase of each follow from these counts on both sides).
    uint32_t items = 0, qloads = 0, wcnt = 0;
    uint32_t nqa = 0, nqb = 0, npa = 0, npb = 0;
    bool ok = true;
    auto issue_qk = [&](int t, uint32_t& nq, uint32_t kaddr) {
      qk(t ? OFF_QB : OFF_QA, kaddr, s_tmem(t, nq), B_SF + t * SBUF + (int)(nq % SBUF));
      ++nq;
    };
    // PV of query tile t once its softmax has published P; false on timeout.
    auto issue_pv = [&](int t, uint32_t& np, uint32_t vaddr, bool acc) {
      const uint32_t n = np;
      if (!warp_wait(bar(B_PF + t * SBUF + (int)(n % SBUF)), (n / SBUF) & 1)) return false;
      tc_fence_after();
      pv(s_tmem(t, n), vaddr, tmem + 256 + (uint32_t)(t * 128), acc);
      ++np;
      if constexpr (SBUF > 1) commit(B_PVD + t);
      return true;
    };
    while (ok) {
      Item it;
      const int w = next_work(wcnt, it);
      if (w < 0) break;
      if (it.n_all == 0) continue;
      auto act_a = [&](int j) { return j >= it.a0 && j < it.a1; };
      auto act_b = [&](int j) { return j >= it.b0 && j < it.b1; };
      if (!(ok = warp_wait(bar(B_Q), qloads & 1))) break;
      ++qloads;
      // QK^T of the first SBUF key tiles, then per tile j: PV(j) of A, QK^T(j+SBUF)
      // of A, PV(j) of B, QK^T(j+SBUF) of B, so a tile's scores for j+1..j+SBUF
      // are computed while its softmax works on j.
      const int pre = it.n_all < SBUF ? it.n_all : SBUF;
      for (int t = 0; t < pre; ++t) {
        const uint32_t ik = items + 2 * t;
        if (!(ok = wait_item(ik))) break;
        tc_fence_after();
        if (act_a(it.j_first + t)) issue_qk(0, nqa, slot_addr(ik));
        if (act_b(it.j_first + t)) issue_qk(1, nqb, slot_addr(ik));
        commit(B_EMPTY + ik % NSLOT);
      }
      if (!ok) break;
      if (it.n_all <= SBUF) commit(B_QE);
      for (int t = 0; ok && t < it.n_all; ++t) {
        const int j = it.j_first + t;
        const uint32_t iv = items + 2 * t + 1, ik = items + 2 * (t + SBUF);
        const bool next = t + SBUF < it.n_all;
        if (!(ok = wait_item(iv))) break;
        if (act_a(j)) {
          if (!(ok = issue_pv(0, npa, slot_addr(iv), j > it.a0))) break;
          if (j == it.a1 - 1) commit(B_ODA);
        }
        if (next && !(ok = wait_item(ik))) break;
        tc_fence_after();
        if (next && act_a(j + SBUF)) issue_qk(0, nqa, slot_addr(ik));
        if (act_b(j)) {
          if (!(ok = issue_pv(1, npb, slot_addr(iv), j > it.b0))) break;
          if (j == it.b1 - 1) commit(B_ODB);
        }
        commit(B_EMPTY + iv % NSLOT);
        if (next && act_b(j + SBUF)) issue_qk(1, nqb, slot_addr(ik));
        if (next) commit(B_EMPTY + ik % NSLOT);
        if (t + SBUF + 1 == it.n_all) commit(B_QE);  // the item's last QK^T has been issued
      }
      items += 2 * it.n_all;
    }
    // All MMAs of this CTA must be complete before TMEM is released.
    commit(B_FIN);
    warp_wait(bar(B_FIN), 0);
  }
  } else {
    // ------------------------------------------------------------ softmax
    reg_alloc<kSoftmaxRegs>();
    const bool is_b = warp >= 4;
    const int sub = warp & 3;
    const int row = sub * 32 + lane;
    const uint32_t lane_off = (uint32_t)(sub * 32) << 16;
    const int tq = is_b ? 1 : 0;
    const uint32_t tS0 = tmem + (uint32_t)(tq * 128) + lane_off;
    const uint32_t tO = tmem + (is_b ? 384 : 256) + lane_off;
    const int od = is_b ? B_ODB : B_ODA;
    // s_cnt: score tiles consumed (= P tiles published) by this warpgroup; tile
    // n uses S buffer n % SBUF and phase n / SBUF of that buffer's barriers.
    uint32_t s_cnt = 0, o_cnt = 0, items = 0, wcnt = 0;
    bool ok = true;
    while (ok) {
      Item it;
      const int w = next_work(wcnt, it);
      if (w < 0) break;
      const int x0 = is_b ? it.b0 : it.a0, n_x = (is_b ? it.b1 : it.a1) - x0;
      const int q_row = (is_b ? it.row_b : it.row_a) + row;
      const int q_abs = q_row + it.k_len - it.q_len;
      const KeyRange vis = key_range(q_abs, it.k_len, it.causal, p.win_l, p.win_r);
      const int h = is_b ? it.h_b : it.h;
      const float qk_scale = it.qk_scale, vscale = it.vscale;
      const float sl2 = qk_scale * 1.4426950408889634f;     // raw score -> log2 units
      // ALiBi slope in log2 units; with ALiBi the scores are biased (and thus
      // already in log2 units) before the row max, so the exp stage scales by 1.
      const float slope_l2 = ALIBI ? p.alibi[it.b * p.al0 + (int64_t)h * p.al1] * 1.4426950408889634f : 0.f;
      const float sl2e = ALIBI ? 1.f : sl2;
      const float cap_l2 = p.softcap * 1.4426950408889634f;  // softcap: cap*log2e*tanh(s*scale/cap)
      const float cap_in = SOFTCAP ? qk_scale / p.softcap : 0.f;
      // Scores up to this magnitude take the softcap's FMA-pipe polynomial.
      const float cap_lim = SOFTCAP ? softcap_poly_limit(cap_in) : -1.f;
      // Running max in log2 units; a sink acts as one extra logit with zero value.
      float m_run = p.sinks ? load_float(p.sinks, p.sink_t, h * p.si0) * 1.4426950408889634f : -INFINITY;
      float l_run = p.sinks ? 1.f : 0.f;
      for (int jj = 0; jj < n_x; ++jj) {
        const int j = x0 + jj;
        const int sbuf = (int)(s_cnt % SBUF);
        if (!(ok = warp_wait(bar(B_SF + tq * SBUF + sbuf), (s_cnt / SBUF) & 1))) break;
        ++s_cnt;
        tc_fence_after();
        const uint32_t tS = tS0 + (uint32_t)(sbuf * BN);
        const int key0 = j * BN;
        const int c_lo = vis.lo - key0, c_hi = vis.hi - key0;  // visible columns of this tile
        const bool need_mask = c_lo > 0 || c_hi < BN - 1;
        // The whole S row of the tile in registers: BN/32 TMEM loads, one wait.
        uint32_t r[BN];
        tmem_ld32_at<0>(tS, r);
        tmem_ld32_at<32>(tS + 32, r);
        if constexpr (BN == 128) {
          tmem_ld32_at<64>(tS + 64, r);
          tmem_ld32_at<96>(tS + 96, r);
        }
        tmem_wait_ld();
        // Softcap route for this tile, uniform over the warp: the polynomial
        // tanh when every raw score of the warp's 32 rows (masked columns
        // included) has |s * scale / cap| <= 3/4, else the identity route.
        bool cap_poly = false;
        if constexpr (SOFTCAP) cap_poly = __all_sync(0xffffffffu, row_absmax(r) <= cap_lim);
        if (!(ALIBI && SOFTCAP) && need_mask) {
#pragma unroll
          for (int i = 0; i < BN; ++i)
            if (i < c_lo || i > c_hi) r[i] = __float_as_uint(-INFINITY);
        }
        if constexpr (ALIBI && SOFTCAP) {
          // v = cap*log2e*tanh(s*scale/cap) - slope*log2e*|q_abs - key| (the
          // reference's capped score minus the ALiBi bias, in log2 units):
          // in one pass with the polynomial tanh, or with
          // tanh(y) = 1 - 2/(e^(2y)+1) as in the softcap-only stage below, in
          // two in-place passes over the row; then the mask.
          const float base = (float)(q_abs - key0);
          const uint64_t nslope2 = f2pack(-slope_l2, -slope_l2);
          if (cap_poly) {
            const TanhPoly tpoly(sl2, cap_in);
#pragma unroll
            for (int i = 0; i < BN; i += 2) {
              const uint64_t dist2 = f2pack(fabsf(base - (float)i), fabsf(base - (float)(i + 1)));
              float v0, v1;
              f2unpack(tpoly.fma(f2pack(__uint_as_float(r[i]), __uint_as_float(r[i + 1])), fmul2(dist2, nslope2)),
                       v0, v1);
              r[i] = __float_as_uint(v0);
              r[i + 1] = __float_as_uint(v1);
            }
          } else {
            const uint64_t tanh_k2 = f2pack(cap_in * 2.8853900817779268f, cap_in * 2.8853900817779268f);
            {
              const Exp2Poly<false> tanh_poly;
#pragma unroll
              for (int i = 0; i < BN; i += 2) {
                float u0, u1, e0, e1;
                f2unpack(fmul2(f2pack(__uint_as_float(r[i]), __uint_as_float(r[i + 1])), tanh_k2), u0, u1);
                tanh_poly.in_range(f2pack(fminf(fmaxf(u0, -64.f), 64.f), fminf(fmaxf(u1, -64.f), 64.f)), e0, e1);
                r[i] = __float_as_uint(e0);
                r[i + 1] = __float_as_uint(e1);
              }
            }
            const uint64_t cap_l2x2 = f2pack(cap_l2, cap_l2);
            const uint64_t one2 = f2pack(1.f, 1.f), neg_two2 = f2pack(-2.f, -2.f);
#pragma unroll
            for (int i = 0; i < BN; i += 2) {
              float d0, d1, v0, v1;
              f2unpack(fadd2(f2pack(__uint_as_float(r[i]), __uint_as_float(r[i + 1])), one2), d0, d1);
              const uint64_t t2 = ffma2(f2pack(rcp(d0), rcp(d1)), neg_two2, one2);
              const uint64_t dist2 = f2pack(fabsf(base - (float)i), fabsf(base - (float)(i + 1)));
              f2unpack(ffma2(t2, cap_l2x2, fmul2(dist2, nslope2)), v0, v1);
              r[i] = __float_as_uint(v0);
              r[i + 1] = __float_as_uint(v1);
            }
          }
          if (need_mask) {
#pragma unroll
            for (int i = 0; i < BN; ++i)
              if (i < c_lo || i > c_hi) r[i] = __float_as_uint(-INFINITY);
          }
        } else if constexpr (ALIBI) {
          // v = s*scale*log2e - slope*log2e*|q_abs - key| (the reference's
          // score minus the ALiBi bias, in log2 units); masked scores stay -inf.
          const float base = (float)(q_abs - key0);
          const uint64_t sl2x2a = f2pack(sl2, sl2), nslope2 = f2pack(-slope_l2, -slope_l2);
#pragma unroll
          for (int i = 0; i < BN; i += 2) {
            const uint64_t d2 = f2pack(fabsf(base - (float)i), fabsf(base - (float)(i + 1)));
            const uint64_t t2 = fmul2(f2pack(__uint_as_float(r[i]), __uint_as_float(r[i + 1])), sl2x2a);
            float v0, v1;
            f2unpack(ffma2(d2, nslope2, t2), v0, v1);
            r[i] = __float_as_uint(v0);
            r[i + 1] = __float_as_uint(v1);
          }
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
        const float m_tile = CAP_IN_EXP ? (mx == -INFINITY ? -INFINITY : cap_l2 * tanh_id(mx * cap_in)) : mx * sl2e;
        float factor = 1.f;
        if (m_tile > m_run + kRescaleThreshold || (m_run == -INFINITY && m_tile != -INFINITY)) {
          factor = m_run == -INFINITY ? 0.f : ex2(m_run - m_tile);
          m_run = m_tile;
        }
        l_run *= factor;
        const float msub = m_run == -INFINITY ? 0.f : m_run;
        // P = 2^(s*scale_log2 - m), masked columns -> 0, packed as 16-bit pairs
        // into TMEM columns [0, BN/2) of this row's S tile, 8 columns per store;
        // the row sum runs as 8 independent chains (4 packed pairs).
        uint64_t ls2[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) ls2[i] = f2pack(0.f, 0.f);
        const uint64_t nmsub2 = f2pack(-msub, -msub);
        // kMode 0: scores already scaled or biased; 1: softcap by the
        // polynomial tanh; 2: softcap by the identity. The softcap tile takes
        // one route for the whole warp (cap_poly), so the two loops never mix.
        auto exp_stage = [&](auto mode) {
          constexpr int kMode = decltype(mode)::value;
          const uint64_t sl2x2 = f2pack(sl2e, sl2e);
          // identity route: e^(2y) = 2^(s * cap_in * 2 log2e)
          const uint64_t tanh_k2 = f2pack(cap_in * 2.8853900817779268f, cap_in * 2.8853900817779268f);
          const uint64_t one2 = f2pack(1.f, 1.f), neg_two2 = f2pack(-2.f, -2.f), cap_l2x2 = f2pack(cap_l2, cap_l2);
#pragma unroll
          for (int c8 = 0; c8 < BN / 16; ++c8) {
            uint32_t pk[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              float p0, p1;
              const float s0 = __uint_as_float(r[c8 * 16 + 2 * i]), s1 = __uint_as_float(r[c8 * 16 + 2 * i + 1]);
              if constexpr (kMode == 1) {
                // cap*log2e*tanh(s*scale/cap) - m = s * R(s^2) - m on the FMA
                // pipe, one MUFU ex2.
                const TanhPoly tpoly(sl2, cap_in);
                float l0, l1;
                f2unpack(tpoly.fma(f2pack(s0, s1), nmsub2), l0, l1);
                p0 = ex2(l0);  // a masked score gives l = -inf exactly: p = 0
                p1 = ex2(l1);
              } else if constexpr (kMode == 2) {
                // cap*log2e*tanh(s*scale/cap) - m with tanh(y) = 1 - 2/(e^(2y)+1):
                // e^(2y) on the FMA pipe (degree-4 polynomial, argument clamped
                // to +-64 where tanh is +-1 in fp32), one MUFU rcp, one MUFU ex2.
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
                const uint64_t x2 = ffma2(f2pack(s0, s1), sl2x2, nmsub2);
                if (i >= 8 - kPolyPairs) {
                  const Exp2Poly<BF16> poly;  // degree 3 for bf16 P, 4 for f16 P
                  poly(x2, p0, p1);  // FMA pipe
                } else {
                  float x0, x1;
                  f2unpack(x2, x0, x1);
                  p0 = ex2(x0);  // MUFU
                  p1 = ex2(x1);
                }
              }
              ls2[i & 3] = fadd2(ls2[i & 3], f2pack(p0, p1));
              pk[i] = pack_p<BF16>(p0, p1);
            }
            tmem_st8_at<0>(tS + c8 * 8, pk);
          }
        };
        if constexpr (CAP_IN_EXP) {
          if (cap_poly) exp_stage(std::integral_constant<int, 1>());
          else exp_stage(std::integral_constant<int, 2>());
        } else {
          exp_stage(std::integral_constant<int, 0>());
        }
        // Lazy O rescale (after the exponentials, while S no longer occupies
        // registers). PV(j) is issued only after this row's P-ready arrival.
        // With one S buffer, PV(j-1) completed before S(j) was signalled; with
        // SBUF buffers S(j) only follows PV(j-SBUF), so wait for PV(j-1) (the
        // s_cnt-1'th PV of this tile, at most one phase behind) first.
        if (jj > 0 && __any_sync(0xffffffffu, factor != 1.f)) {
          if constexpr (SBUF > 1) {
            if (!(ok = warp_wait(bar(B_PVD + tq), (s_cnt - 2) & 1))) break;
            tc_fence_after();
          }
#pragma unroll
          for (int c = 0; c < HDIM / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(tO + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
            tmem_st32(tO + c * 32, o);
          }
        }
        tmem_wait_st();
        float ls8[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) f2unpack(ls2[i], ls8[2 * i], ls8[2 * i + 1]);
        const float lsum = ((ls8[0] + ls8[1]) + (ls8[2] + ls8[3])) + ((ls8[4] + ls8[5]) + (ls8[6] + ls8[7]));
        l_run += lsum;
        if (key0 + BN > it.k_len) {
          // Keys past the sequence in the last tile: zero their V rows so that a
          // non-finite neighbour value can never meet a zero probability. Each
          // warpgroup consuming the tile zeroes them itself (identical stores).
          const uint32_t item = items + 2 * (j - it.j_first) + 1;
          if (!(ok = warp_wait(bar(B_FULL + item % NSLOT), (item / NSLOT) & 1))) break;
          if (row < BN && key0 + row >= it.k_len) {
            uint8_t* vrow = gbase + OFF_RING + (item % NSLOT) * kKVTileBytes + row * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
#pragma unroll
              for (int hf = 0; hf < kHalves; ++hf)
                *reinterpret_cast<uint4*>(vrow + hf * kKVRegion + c * 16) = make_uint4(0, 0, 0, 0);
            }
          }
          fence_proxy_async_smem();  // generic stores -> the MMA's async-proxy reads
        }
        tc_fence_before();
        mbar_arrive(bar(B_PF + tq * SBUF + sbuf));
      }
      items += 2 * it.n_all;
      if (!ok) break;
      if (n_x > 0) {
        if (!(ok = warp_wait(bar(od), o_cnt & 1))) break;
        ++o_cnt;
        tc_fence_after();
      }
      // ---------------------------------------------------------- epilogue
      // O / l in bf16/f16. A warp whose 32 rows all lie inside the sequence
      // stages them in its own 128-byte-swizzled shared buffer and writes them
      // with two asynchronous TMA tile stores (coalesced); a warp at the end
      // of a sequence stores its valid rows directly.
      const bool row_ok = q_row < it.q_len;
      const int64_t t = (int64_t)it.q_begin + q_row;
      const bool have = n_x > 0 && l_run > 0.f;
      const float inv = have ? vscale / l_run : 0.f;
      const int wrow0 = (is_b ? it.row_b : it.row_a) + sub * 32;
      const bool staged = wrow0 + 32 <= it.q_len;  // warp-uniform
      uint8_t* stg = gbase + OFF_STAGE + warp * kStageWarpBytes;
      uint8_t* orow = reinterpret_cast<uint8_t*>(p.out) + (t * p.os0 + (int64_t)h * p.os1) * 2;
      if (staged) {
        if (lane == 0) bulk_wait_read();  // this warp's previous stores have read the buffer
        __syncwarp();
      }
      // The whole O row in registers with one TMEM round trip (also when this
      // tile saw no key: the values are then unused, see `have`).
      uint32_t r[HDIM];
      {
        tmem_ld32_at<0>(tO, r);
        tmem_ld32_at<32>(tO + 32, r);
        if constexpr (HDIM == 128) {
          tmem_ld32_at<64>(tO + 64, r);
          tmem_ld32_at<96>(tO + 96, r);
        }
        tmem_wait_ld();
      }
#pragma unroll
      for (int c = 0; c < HDIM / 32; ++c) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint32_t wv[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float a = have ? __uint_as_float(r[c * 32 + v * 8 + 2 * i]) * inv : 0.f;
            const float bb = have ? __uint_as_float(r[c * 32 + v * 8 + 2 * i + 1]) * inv : 0.f;
            wv[i] = pack_p<BF16>(a, bb);
          }
          const uint4 val = make_uint4(wv[0], wv[1], wv[2], wv[3]);
          if (staged) {
            const int chunk = (c & 1) * 4 + v;
            *reinterpret_cast<uint4*>(stg + (c >> 1) * 4096 + lane * 128 + ((chunk ^ (lane & 7)) << 4)) = val;
          } else if (row_ok && c * 32 + v * 8 < p.dim) {
            *reinterpret_cast<uint4*>(orow + (c * 32 + v * 8) * 2) = val;
          }
        }
      }
      if (staged) {
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          const uint32_t sa = smem_addr(stg);
#pragma unroll
          for (int hf = 0; hf < kHalves; ++hf) tma_store_3d(&to, sa + hf * 4096, hf * 64, h, it.q_begin + wrow0);
          bulk_commit();
        }
      }
      if (row_ok) p.lse[(int64_t)h * p.ls0 + t * p.ls1] = l_run > 0.f ? (m_run + log2f(l_run)) * kLn2 : -INFINITY;
    }
    if (lane == 0) bulk_wait_all();  // staged output stores complete before the CTA exits
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}


}  // namespace

int prefill_sm100_supported(const AttnParams& p) {
  if (!(p.qt == FA_BF16 || p.qt == FA_F16) || p.kt != p.qt || p.vt != p.qt || p.ot != p.qt) return 0;
  // Head dims up to 128 in multiples of 8 (16-byte rows): the 64- or 128-wide
  // instantiation runs them, the tensor maps' true extent zero-fills the
  // padded columns on loads (adding nothing to Q K^T; V's give O columns that
  // are never stored) and clips them on the tile stores.
  // Head dims above 128 (QK up to 256, V up to 256): the one-tile kernel of
  // prefill_wide_sm100.cu, packed or paged K/V without ALiBi.
  const bool wide = prefill_wide_dims(p);
  if (wide && !prefill_wide_supported(p)) return 0;
  if (!wide && (p.DQ != p.DV || p.DQ < 8 || p.DQ > 128 || p.DQ % 8)) return 0;
  if (p.paged) {
    // Paged K/V: power-of-two pages of >= 8 tokens (whole 1024-byte swizzle
    // atoms per box), a page stride TMA can address.
    if (p.page < 8 || (p.page & (p.page - 1)) || p.k_pages <= 0 || p.k_pages >= (1LL << 31)) return 0;
    if (p.bt_cols <= 0 || p.bt_cols >= (1LL << 31)) return 0;
    const int64_t ps[2] = {p.ks0, p.vs0};
    for (int64_t v : ps)
      if (v <= 0 || (v * 2) % 16 != 0) return 0;
  }
  if (p.mask || p.leftpad || p.cp_n > 1) return 0;
  if (p.sinks && !(p.sink_t == FA_F32 || p.sink_t == FA_F16 || p.sink_t == FA_BF16)) return 0;
  if (p.qs2 != 1 || p.ks3 != 1 || p.vs3 != 1 || p.os2 != 1) return 0;
  if (!al16(p.q) || !al16(p.k) || !al16(p.v) || !al16(p.out)) return 0;
  const int64_t s[8] = {p.qs0, p.qs1, p.ks1, p.ks2, p.vs1, p.vs2, p.os0, p.os1};
  for (int64_t v : s)
    if (v <= 0 || (v * 2) % 16 != 0) return 0;
  if (p.T >= (1 << 30)) return 0;
  if (!p.paged && (p.k_rows <= 0 || p.k_rows >= (1 << 30))) return 0;
  if ((int64_t)((p.max_q + BM - 1) / BM) * p.HQ * p.B >= (1LL << 31)) return 0;
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
  const int w = prefill_wide_timeout_flag(clear);
  if (w < 0) return -1;
  return v | w;
}

int launch_prefill_sm100(const AttnParams& p, cudaStream_t stream) {
  if (p.T <= 0) return fail(FA_ERR_INVALID, "prefill needs query rows");
  if (!p.paged && p.k_rows <= 0) return fail(FA_ERR_INVALID, "prefill needs packed K/V rows");
  int page_shift = 0, box_rows = 0;
  if (p.paged) {
    while ((1 << page_shift) < p.page) ++page_shift;
    box_rows = p.page < BN ? p.page : BN;  // whole pages, at most one key tile per box
  }
  PrefillParams pp{};
  pp.out = p.out; pp.os0 = p.os0; pp.os1 = p.os1;
  pp.lse = p.lse; pp.ls0 = p.ls0; pp.ls1 = p.ls1;
  pp.cu_q = p.cu_q; pp.cq0 = p.cq0;
  pp.cu_k = p.cu_k; pp.ck0 = p.ck0;
  pp.used = p.used; pp.u0 = p.u0;
  pp.B = p.B; pp.HQ = p.HQ; pp.HK = p.HK;
  pp.counter = reinterpret_cast<int*>(p.scratch);
  if (p.paged) {
    pp.table = p.table; pp.bt0 = p.bt0; pp.bt1 = p.bt1;
    pp.bt_cols = (int32_t)p.bt_cols; pp.page_shift = page_shift; pp.box_rows = box_rows;
  }
  // Pair query heads h, h+1 (same KV head) when the heads per KV head are even.
  pp.head_pairs = (p.HQ / p.HK) % 2 == 0 ? 1 : 0;
  pp.n_pairs = pp.head_pairs ? (p.max_q + BM - 1) / BM : (p.max_q + 2 * BM - 1) / (2 * BM);
  pp.group_reqs = prefill_group_reqs(p);
  pp.causal = p.causal;
  pp.causal_b = p.dynamic ? p.causal_b : nullptr; pp.ca0 = p.ca0;
  pp.sinks = p.sinks; pp.sink_t = p.sink_t; pp.si0 = p.si0;
  pp.qd = p.qd; pp.qd0 = p.qd0; pp.qd1 = p.qd1;
  pp.kd = p.kd; pp.kd0 = p.kd0; pp.kd1 = p.kd1;
  pp.vd = p.vd; pp.vd0 = p.vd0; pp.vd1 = p.vd1;
  pp.win_l = p.win_l; pp.win_r = p.win_r;
  pp.scale = p.scale;
  pp.softcap = p.softcap;
  pp.alibi = p.alibi; pp.al0 = p.a0; pp.al1 = p.a1;
  pp.dim = p.DV;
  if (prefill_wide_dims(p)) return launch_prefill_wide(p, pp, stream);
  CUtensorMap mq, mk, mv;
  int rc = make_map(&mq, p.q, p.qt, p.DQ, p.T, p.HQ, p.qs0, p.qs1);
  if (rc) return rc;
  if (p.paged) {
    rc = make_page_map(&mk, p.k, p.kt, p.DQ, p.HK, p.page, p.k_pages, p.ks0, p.ks1, p.ks2, box_rows);
    if (rc) return rc;
    rc = make_page_map(&mv, p.v, p.vt, p.DV, p.HK, p.page, p.k_pages, p.vs0, p.vs1, p.vs2, box_rows);
    if (rc) return rc;
  } else {
    rc = make_map(&mk, p.k, p.kt, p.DQ, p.k_rows, p.HK, p.ks1, p.ks2, BN);
    if (rc) return rc;
    rc = make_map(&mv, p.v, p.vt, p.DV, p.k_rows, p.HK, p.vs1, p.vs2, BN);
    if (rc) return rc;
  }
  CUtensorMap mo;  // output tile stores: 32 rows x 64 head dims per box
  rc = make_map(&mo, p.out, p.ot, p.DV, p.T, p.HQ, p.os0, p.os1, 32);
  if (rc) return rc;
  const bool cap = p.softcap > 0.f, alibi = p.alibi != nullptr;
  auto pick = [&](auto hd) {
    constexpr int H = decltype(hd)::value;
    if (p.qt == FA_BF16)
      return cap ? (alibi ? prefill_sm100_kernel<true, true, H, true> : prefill_sm100_kernel<true, true, H, false>)
                 : alibi ? prefill_sm100_kernel<true, false, H, true> : prefill_sm100_kernel<true, false, H, false>;
    return cap ? (alibi ? prefill_sm100_kernel<false, true, H, true> : prefill_sm100_kernel<false, true, H, false>)
               : alibi ? prefill_sm100_kernel<false, false, H, true> : prefill_sm100_kernel<false, false, H, false>;
  };
  auto kernel = p.DQ <= 64 ? pick(std::integral_constant<int, 64>{}) : pick(std::integral_constant<int, 128>{});
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return fail(FA_ERR_CUDA, "prefill smem attribute: %s", cudaGetErrorString(e));
  // The warpgroups' setmaxnreg split assumes exactly kLaunchRegs registers per
  // thread at launch; a build that allocated another count must not run.
  cudaFuncAttributes fa;
  e = cudaFuncGetAttributes(&fa, kernel);
  if (e != cudaSuccess) return fail(FA_ERR_CUDA, "prefill attributes: %s", cudaGetErrorString(e));
  if (fa.numRegs != kLaunchRegs)
    return fail(FA_ERR_CUDA, "prefill kernel built with %d registers per thread, expected %d", fa.numRegs,
                kLaunchRegs);
  const int64_t n_work = (int64_t)pp.n_pairs * (p.HQ >> pp.head_pairs) * p.B;
  const int grid = (int)std::min<int64_t>(n_work, (int64_t)sm_count());
  if (pp.counter == nullptr) return fail(FA_ERR_INVALID, "prefill needs its workspace counter");
  e = cudaMemsetAsync(pp.counter, 0, sizeof(int), stream);
  if (e != cudaSuccess) return fail(FA_ERR_CUDA, "prefill counter reset: %s", cudaGetErrorString(e));
  kernel<<<grid, kThreads, kSmemBytes, stream>>>(mq, mk, mv, mo, pp);
  note_launch();
  FAB_LAUNCH_CHECK("prefill launch");
  return FA_OK;
}

}  // namespace fab
