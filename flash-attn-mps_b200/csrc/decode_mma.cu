// Paged / packed single-query decode on tensor cores (HBM-bound).
//
// Work unit: one CTA = (request b, KV head kh, block of <=16 query heads of the
// group, KV split). The query heads of a GQA group are the N columns of the
// MMAs, so every K/V page is read from HBM exactly once per group:
//   S^T[tokens x heads] = K[tokens x D] * Q^T[D x heads]        (A = K tile)
//   O^T[D x heads]     += V^T[D x tokens] * P^T[tokens x heads]  (A = V^T tile)
// on mma.sync m16n8k16 with fp32 accumulation. Tokens as the M dimension keep
// the padding of small groups (4 heads in an n8 tile) off the big operands.
//   * K/V token rows are gathered through block_table with 16-byte cp.async
//     (zero-fill outside the visible range, so NaN-poisoned tails never reach
//     the MMAs) into an NST-stage ring of XOR-swizzled shared-memory tiles.
//   * Each warp owns 16 tokens of a stage; the online softmax runs per head
//     column in the log2 domain; P^T reaches the B operand of the PV MMA via
//     movmatrix.trans, with no shared-memory round trip.
//   * FP8 E4M3 K/V are converted in registers by the exact hardware
//     cvt.rn.f16x2.e4m3x2; ldmatrix on byte tiles fixes a per-thread
//     permutation of the QK reduction dimension (undone in the Q fragments)
//     and of the output dimension (undone in the epilogue).
//   * The warps' states are merged through shared memory; with one split the
//     CTA writes the final output and LSE, otherwise an fp32 partial that the
//     N-way merge kernel combines.
// Semantics follow the reference decode_partitions
// (flash_attn_mps/kernels/attention_decode.metal:18-149; split span and window
// begin at 40-47, sink seeding at 54-56, softcap at 94, descales at 41-44,
// FP8 decode at 9-16) and its dispatcher (flash_attn_mps/_decode.py:40-99).
#include "kernels.cuh"
#include "ptx.cuh"
#include "sm100.cuh"

namespace fab {
namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// Set by a TMA-pipeline wait that gave up (a bounded mbarrier wait); the host
// reads it through decode_timeout_flag().
__device__ int g_decode_timeout;

template <bool FP8, int D, int W, int NH>
struct Geometry {
  static constexpr int kTile = 16 * W;                 // tokens per stage
  static constexpr int kRowBytes = D * (FP8 ? 1 : 2);
  static constexpr int kChunks = kRowBytes / 16;
  static constexpr int kStageBytes = 2 * kTile * kRowBytes;
  static constexpr int kN8 = NH / 8;                   // head tiles
  static constexpr int kDT = D / 16;                   // 16-row output tiles per head tile
  static constexpr int kHalves = kRowBytes / 128;      // 128-byte column blocks of a row
  static_assert(kChunks >= 8 && kChunks % 8 == 0, "rows must span whole 128-byte swizzle atoms");
  // Byte offset of 16-byte chunk c of token row r inside a K or V stage tile:
  // [column block][row][128 B], chunks XOR-swizzled by (r & 7) -- the layout
  // TMA's 128-byte swizzle writes into a 1024-byte-aligned tile.
  static __device__ __forceinline__ uint32_t off(int r, int c) {
    return (uint32_t)((((c >> 3) * kTile + r) << 7) + (((c & 7) ^ (r & 7)) << 4));
  }
};

// Head-dimension index of row (g or g+8) of output tile j.
template <bool FP8>
__device__ __forceinline__ int out_dim(int j, int row) {
  if constexpr (!FP8) {
    return j * 16 + row;
  } else {
    // tile 2m: dims 32m + 2r (+16 for rows 8..15); tile 2m+1: the odd dims.
    const int r = row & 7;
    return (j >> 1) * 32 + 2 * r + (row >> 3) * 16 + (j & 1);
  }
}

template <typename MT, bool FP8, int D, int W, int NH, int NST, bool PREC, bool QFOLD, bool TMA, int MINB>
__global__ void __launch_bounds__((W + (TMA ? 1 : 0)) * 32, MINB)
    decode_mma_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                      const AttnParams p, const int span, const int hblocks, const int page_shift,
                      const int box_tok) {
  using G = Geometry<FP8, D, W, NH>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);  // 1024-aligned tiles
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, qd = lane & 3;
  const int split = blockIdx.x;
  const int kh = blockIdx.y / hblocks, hb = blockIdx.y - kh * hblocks;
  const int b = blockIdx.z;
  const int token = p.cu_q[b * p.cq0];
  if (p.cu_q[(b + 1) * p.cq0] == token) return;
  const int group = p.HQ / p.HK;
  const int h0 = kh * group + hb * NH;
  const int nh = min(NH, group - hb * NH);
  const int k_cu_begin = p.cu_k ? p.cu_k[b * p.ck0] : 0;
  const int len = p.used ? p.used[b * p.u0] : p.cu_k[(b + 1) * p.ck0] - k_cu_begin;
  int left = p.leftpad ? p.leftpad[b * p.lp0] : 0;
  if (!p.paged) left += k_cu_begin;
  // Left window in local positions; under context parallelism local key j is
  // global j * cp_n + cp_r and the query is the last of cp_tot[b] tokens.
  int visible_begin = p.win_l >= 0 ? max(0, len - p.win_l - 1) : 0;
  if (p.cp_n > 1 && p.win_l >= 0) {
    const int first_global = p.cp_tot[b * p.ct0] - 1 - p.win_l;  // smallest visible global position
    visible_begin = max(0, (first_global - p.cp_r + p.cp_n - 1) / p.cp_n);
  }
  const int begin = visible_begin + split * span;
  const int end = min(len, begin + span);
  const float qdesc = p.qd ? p.qd[b * p.qd0 + kh * p.qd1] : 1.f;
  const float kdesc = p.kd ? p.kd[b * p.kd0 + kh * p.kd1] : 1.f;
  const float vscale = p.vd ? p.vd[b * p.vd0 + kh * p.vd1] : 1.f;
  const float scale = p.scale * qdesc * kdesc;
  const float dot_scale = QFOLD ? 1.f : scale;  // applied to fp32 dots
  const bool capped = p.softcap > 0.f;

  // ---- Q^T fragments (B operand: k = head dim, n = query head) -------------
  uint32_t qb[G::kN8][D / 16][2];
#pragma unroll
  for (int n8 = 0; n8 < G::kN8; ++n8) {
    const int hrow = n8 * 8 + g;
    const bool ok = hrow < nh;
    const int64_t base = (int64_t)token * p.qs0 + (int64_t)(h0 + hrow) * p.qs1;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int khalf = 0; khalf < 2; ++khalf) {
        const int d = FP8 ? kk * 16 + 4 * qd + 2 * khalf : kk * 16 + 8 * khalf + 2 * qd;
        // Head dims below D (the instantiation) read as zero past the true dim.
        float x0 = ok && d < p.DQ ? load_float(p.q, p.qt, base + d * p.qs2) : 0.f;
        float x1 = ok && d + 1 < p.DQ ? load_float(p.q, p.qt, base + (d + 1) * p.qs2) : 0.f;
        if (QFOLD) { x0 *= scale; x1 *= scale; }
        qb[n8][kk][khalf] = pack2<MT>(x0, x1);
      }
    }
  }

  // Per thread: head columns 2*qd, 2*qd+1 of each head tile.
  float o[G::kN8][G::kDT][4];
#pragma unroll
  for (int n8 = 0; n8 < G::kN8; ++n8)
#pragma unroll
    for (int j = 0; j < G::kDT; ++j) o[n8][j][0] = o[n8][j][1] = o[n8][j][2] = o[n8][j][3] = 0.f;
  float m[G::kN8][2], l[G::kN8][2];
#pragma unroll
  for (int n8 = 0; n8 < G::kN8; ++n8) {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      m[n8][c] = -INFINITY;
      l[n8][c] = 0.f;
      const int hcol = n8 * 8 + 2 * qd + c;
      if (p.sinks && split == 0 && p.cp_r == 0 && warp == 0 && hcol < nh) {
        m[n8][c] = load_float(p.sinks, p.sink_t, (h0 + hcol) * p.si0) * kLog2e;
        l[n8][c] = g == 0 ? 1.f : 0.f;  // counted once across the column's lanes
      }
    }
  }

  // ---- K/V gather -----------------------------------------------------------
  // Tile it covers logical cache positions [L0 + it*kTile, +kTile); the TMA
  // path aligns L0 down to the tile size so whole pages arrive as boxes.
  const int L0 = TMA ? ((begin + left) / G::kTile) * G::kTile : begin + left;
  const int n_tiles = end > begin ? (end + left - L0 + G::kTile - 1) / G::kTile : 0;
  const uint32_t bar_base = smem_u32(smem) + NST * G::kStageBytes;
  auto full_bar = [&](int s_) { return bar_base + 8u * (uint32_t)s_; };
  auto empty_bar = [&](int s_) { return bar_base + 8u * (uint32_t)(NST + s_); };
  if constexpr (TMA) {
    if (tid == 0) {
      for (int s_ = 0; s_ < NST; ++s_) {
        sm100::mbar_init(full_bar(s_), 1);
        sm100::mbar_init(empty_bar(s_), W);
      }
      sm100::mbar_fence_init();
    }
    __syncthreads();
  }
  const int elt = FP8 ? 1 : 2;
  const uint8_t* kglob = reinterpret_cast<const uint8_t*>(p.k) + (int64_t)kh * p.ks2 * elt;
  const uint8_t* vglob = reinterpret_cast<const uint8_t*>(p.v) + (int64_t)kh * p.vs2 * elt;
  const int32_t* trow = p.paged ? p.table + (int64_t)b * p.bt0 : nullptr;
  auto load_stage = [&](int stage, int tile_start) {
    uint8_t* ks = smem + stage * G::kStageBytes;
    uint8_t* vs = ks + G::kTile * G::kRowBytes;
    constexpr int kRowsPerPass = W * 32 / G::kChunks;
    const int c = tid % G::kChunks;
#pragma unroll
    for (int r = tid / G::kChunks; r < G::kTile; r += kRowsPerPass) {
      const int t = tile_start + r;
      const bool ok = t < end;
      int64_t koff = 0, voff = 0;
      if (ok) {
        const int logical = t + left;
        if (p.paged) {
          const int pg = page_shift >= 0 ? logical >> page_shift : logical / p.page;
          const int in = logical - pg * p.page;
          const int64_t blk = __ldg(trow + (int64_t)pg * p.bt1);
          koff = blk * p.ks0 + (int64_t)in * p.ks1;
          voff = blk * p.vs0 + (int64_t)in * p.vs1;
        } else {
          koff = (int64_t)logical * p.ks1;
          voff = (int64_t)logical * p.vs1;
        }
      }
      const uint32_t o = G::off(r, c);
      const bool col = c * 16 < p.DQ * elt;  // 16-byte chunks past the true head dim are zero-filled
      cp_async_16(smem_u32(ks) + o, kglob + koff * elt + c * 16, ok && col ? 16 : 0);
      cp_async_16(smem_u32(vs) + o, vglob + voff * elt + c * 16, ok && col ? 16 : 0);
    }
  };

  if constexpr (TMA) {
    if (warp == W) {
      // ---------------------------------------------------- TMA producer warp
      // One box = box_tok consecutive tokens of one page (128 bytes of each row
      // per box); boxes of pages past the sequence use page -1, which TMA
      // treats as out of bounds and fills with zeros. The block-table entries
      // of tile it+1 are fetched right after tile it is issued, so their
      // latency overlaps the wait for a free slot.
      constexpr int kBoxesMax = 2 * G::kHalves * (G::kTile / 8);
      constexpr int kPerLane = (kBoxesMax + 31) / 32;
      const int nbox = G::kTile / box_tok;
      const int total = 2 * G::kHalves * nbox;
      auto lookup = [&](int it, int (&blk)[kPerLane]) {
        const int lb = L0 + it * G::kTile;
#pragma unroll
        for (int j = 0; j < kPerLane; ++j) {
          const int i = lane + 32 * j;
          const int bx = i % nbox;
          const int logical = lb + bx * box_tok;
          const int pg = logical >> page_shift;
          int v = -1;
          if (i < total && logical - left < len && pg < p.bt_cols) v = __ldg(trow + (int64_t)pg * p.bt1);
          blk[j] = v;
        }
      };
      if (lane == 0) {
        sm100::tma_prefetch_desc(&tmk);
        sm100::tma_prefetch_desc(&tmv);
      }
      int next[kPerLane];
      if (n_tiles > 0) lookup(0, next);
      int issued = 0;
      for (int it = 0; it < n_tiles; ++it) {
        int cur[kPerLane];
#pragma unroll
        for (int j = 0; j < kPerLane; ++j) cur[j] = next[j];
        const int st = it % NST;
        if (it >= NST) {
          const bool ok = sm100::mbar_wait(empty_bar(st), ((it / NST) - 1) & 1, &g_decode_timeout);
          if (!__all_sync(0xffffffffu, ok)) break;
        }
        if (lane == 0) sm100::mbar_expect_tx(full_bar(st), G::kStageBytes);
        __syncwarp();
        const int lb = L0 + it * G::kTile;
        const uint32_t sbase = smem_u32(smem) + st * G::kStageBytes;
#pragma unroll
        for (int j = 0; j < kPerLane; ++j) {
          const int i = lane + 32 * j;
          if (i < total) {
            const int tensor = i / (G::kHalves * nbox);
            const int rem = i - tensor * G::kHalves * nbox;
            const int half = rem / nbox, bx = rem - half * nbox;
            const int logical = lb + bx * box_tok;
            const uint32_t dst =
                sbase + tensor * (G::kTile * G::kRowBytes) + (uint32_t)((half * G::kTile + bx * box_tok) << 7);
            sm100::tma_load_4d(dst, tensor ? &tmv : &tmk, full_bar(st), half * (128 / elt), kh,
                               logical & (p.page - 1), cur[j]);
          }
        }
        __syncwarp();
        issued = it + 1;
        if (it + 1 < n_tiles) lookup(it + 1, next);
      }
      // Every issued load must land before the CTA leaves.
      for (int it = max(0, issued - NST); it < issued; ++it)
        sm100::mbar_wait(full_bar(it % NST), (it / NST) & 1, &g_decode_timeout);
    }
  } else {
#pragma unroll
    for (int s_ = 0; s_ < NST - 1; ++s_) {
      if (s_ < n_tiles) load_stage(s_, L0 - left + s_ * G::kTile);
      cp_async_commit();
    }
  }

  for (int it = 0; it < n_tiles && (!TMA || warp < W); ++it) {
    if constexpr (!TMA) {
      cp_async_wait<NST - 2>();
      __syncthreads();
      const int nxt = it + NST - 1;
      if (nxt < n_tiles) load_stage(nxt % NST, L0 - left + nxt * G::kTile);
      cp_async_commit();
    } else {
      const bool ok = sm100::mbar_wait(full_bar(it % NST), (it / NST) & 1, &g_decode_timeout);
      if (!__all_sync(0xffffffffu, ok)) break;
    }
    const int t0 = L0 - left + it * G::kTile + warp * 16;
    const bool any = t0 + 16 > begin && t0 < end;
    const uint32_t kbase = smem_u32(smem + (it % NST) * G::kStageBytes);
    const uint32_t vbase = kbase + G::kTile * G::kRowBytes;
    const int wt0 = warp * 16;
    if (TMA && any && !(t0 >= begin && t0 + 16 <= end)) {
      // Rows of this warp outside [begin, end) came from whole-page boxes:
      // zero their V rows so a NaN-poisoned slot never meets a zero weight.
      const int rr = lane & 15, part = lane >> 4;
      if (t0 + rr < begin || t0 + rr >= end) {
#pragma unroll
        for (int hf = 0; hf < G::kHalves; ++hf)
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4)
            *reinterpret_cast<uint4*>(smem + (it % NST) * G::kStageBytes + G::kTile * G::kRowBytes +
                                      ((hf * G::kTile + wt0 + rr) << 7) + part * 64 + q4 * 16) = make_uint4(0, 0, 0, 0);
        // Order these generic stores before the next TMA write of the slot.
        sm100::fence_proxy_async_smem();
      }
      __syncwarp();
    }
    if (any) {
    // S^T = K Q^T over this warp's 16 tokens, as two independent MMA chains.
    float s[G::kN8][4], s2[G::kN8][4];
#pragma unroll
    for (int n8 = 0; n8 < G::kN8; ++n8)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[n8][e] = s2[n8][e] = 0.f;
    {
      const int mi = lane >> 3;
      const int tok = wt0 + (mi & 1) * 8 + (lane & 7);
      if constexpr (!FP8) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int ch = kk * 2 + (mi >> 1);
          uint32_t a[4];
          ldsm_x4(kbase + G::off(tok, ch), a[0], a[1], a[2], a[3]);
#pragma unroll
          for (int n8 = 0; n8 < G::kN8; ++n8) {
            if (kk & 1) mma16816<MT>(s2[n8], a, qb[n8][kk][0], qb[n8][kk][1]);
            else mma16816<MT>(s[n8], a, qb[n8][kk][0], qb[n8][kk][1]);
          }
        }
      } else {
#pragma unroll
        for (int kc = 0; kc < D / 32; ++kc) {
          const int ch = 2 * kc + (mi >> 1);
          uint32_t r0, r1, r2, r3;
          ldsm_x4(kbase + G::off(tok, ch), r0, r1, r2, r3);
          uint32_t a0[4], a1[4];
          e4m3x4_to_f16x2x2(r0, a0[0], a0[2]);
          e4m3x4_to_f16x2x2(r1, a0[1], a0[3]);
          e4m3x4_to_f16x2x2(r2, a1[0], a1[2]);
          e4m3x4_to_f16x2x2(r3, a1[1], a1[3]);
#pragma unroll
          for (int n8 = 0; n8 < G::kN8; ++n8) {
            mma16816<MT>(s[n8], a0, qb[n8][2 * kc][0], qb[n8][2 * kc][1]);
            mma16816<MT>(s2[n8], a1, qb[n8][2 * kc + 1][0], qb[n8][2 * kc + 1][1]);
          }
        }
      }
    }
#pragma unroll
    for (int n8 = 0; n8 < G::kN8; ++n8)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[n8][e] += s2[n8][e];

    // Online softmax per head column (log2 domain). Element e of tile n8:
    // token (e < 2 ? g : g + 8), head column 2*qd + (e & 1).
    const bool full = t0 >= begin && t0 + 16 <= end;
    const bool tok_lo = t0 + g >= begin && t0 + g < end, tok_hi = t0 + g + 8 >= begin && t0 + g + 8 < end;
    bool changed = false;
    uint32_t pb[G::kN8][2], pl[G::kN8][2];
#pragma unroll
    for (int n8 = 0; n8 < G::kN8; ++n8) {
      float mx[2];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x = s[n8][e];
        if (capped) x = p.softcap * tanhf(x * dot_scale / p.softcap) * kLog2e;
        else x *= dot_scale * kLog2e;
        if (!full) x = (e < 2 ? tok_lo : tok_hi) ? x : -INFINITY;
        s[n8][e] = x;
      }
      mx[0] = fmaxf(s[n8][0], s[n8][2]);
      mx[1] = fmaxf(s[n8][1], s[n8][3]);
      float nsafe[2];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        mx[c] = fmaxf(mx[c], __shfl_xor_sync(0xffffffffu, mx[c], 4));
        mx[c] = fmaxf(mx[c], __shfl_xor_sync(0xffffffffu, mx[c], 8));
        mx[c] = fmaxf(mx[c], __shfl_xor_sync(0xffffffffu, mx[c], 16));
        const float n = fmaxf(m[n8][c], mx[c]);
        // ex2(-inf) = 0, so one guard per column keeps fully masked columns NaN-free.
        nsafe[c] = n == -INFINITY ? 0.f : n;
        const float f = fast_exp2(m[n8][c] - nsafe[c]);
        changed |= f != 1.f;
        mx[c] = f;  // reuse as the rescale factor
        m[n8][c] = n;
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) s[n8][e] = fast_exp2(s[n8][e] - nsafe[e & 1]);
      l[n8][0] = l[n8][0] * mx[0] + s[n8][0] + s[n8][2];
      l[n8][1] = l[n8][1] * mx[1] + s[n8][1] + s[n8][3];
      if (__any_sync(0xffffffffu, changed)) {
#pragma unroll
        for (int j = 0; j < G::kDT; ++j) {
          o[n8][j][0] *= mx[0]; o[n8][j][1] *= mx[1];
          o[n8][j][2] *= mx[0]; o[n8][j][3] *= mx[1];
        }
      }
      // P^T as the B operand: transpose the (token, head) 8x8 blocks.
      const uint32_t lo = pack2<MT>(s[n8][0], s[n8][1]);
      const uint32_t hi = pack2<MT>(s[n8][2], s[n8][3]);
      pb[n8][0] = movmatrix_t(lo);
      pb[n8][1] = movmatrix_t(hi);
      if constexpr (PREC) {
        // P = hi + lo keeps ~22 bits of each probability for fp32 outputs.
        const float2 h0f = unpack2<MT>(lo), h1f = unpack2<MT>(hi);
        pl[n8][0] = movmatrix_t(pack2<MT>(s[n8][0] - h0f.x, s[n8][1] - h0f.y));
        pl[n8][1] = movmatrix_t(pack2<MT>(s[n8][2] - h1f.x, s[n8][3] - h1f.y));
      }
    }

    // O^T += V^T P^T
    {
      const int mi = lane >> 3;
      const int tok = wt0 + (mi >> 1) * 8 + (lane & 7);
      if constexpr (!FP8) {
#pragma unroll
        for (int j = 0; j < G::kDT; ++j) {
          const int ch = j * 2 + (mi & 1);
          uint32_t a[4];
          ldsm_x4_t(vbase + G::off(tok, ch), a[0], a[1], a[2], a[3]);
#pragma unroll
          for (int n8 = 0; n8 < G::kN8; ++n8) {
            mma16816<MT>(o[n8][j], a, pb[n8][0], pb[n8][1]);
            if constexpr (PREC) mma16816<MT>(o[n8][j], a, pl[n8][0], pl[n8][1]);
          }
        }
      } else {
#pragma unroll
        for (int jg = 0; jg < D / 32; ++jg) {
          const int ch = jg * 2 + (mi & 1);
          uint32_t r[4];
          ldsm_x4_t(vbase + G::off(tok, ch), r[0], r[1], r[2], r[3]);
          // Bytes (0,2) are one output dim over two tokens, (1,3) the next dim.
          uint32_t ae[4], ao[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) e4m3x4_to_f16x2x2(__byte_perm(r[i], 0, 0x3120), ae[i], ao[i]);
#pragma unroll
          for (int n8 = 0; n8 < G::kN8; ++n8) {
            mma16816<MT>(o[n8][2 * jg], ae, pb[n8][0], pb[n8][1]);
            mma16816<MT>(o[n8][2 * jg + 1], ao, pb[n8][0], pb[n8][1]);
            if constexpr (PREC) {
              mma16816<MT>(o[n8][2 * jg], ae, pl[n8][0], pl[n8][1]);
              mma16816<MT>(o[n8][2 * jg + 1], ao, pl[n8][0], pl[n8][1]);
            }
          }
        }
      }
    }
    }  // any
    if constexpr (TMA) {
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(empty_bar(it % NST));
    }
  }
  if constexpr (!TMA) cp_async_wait<0>();
  __syncthreads();

  // ---- merge the warps' states through shared memory -------------------------
  float* cm = reinterpret_cast<float*>(smem);   // [W][NH]
  float* cl = cm + W * NH;                      // [W][NH]
  float* co = cl + W * NH;                      // [W][NH][D]
#pragma unroll
  for (int n8 = 0; n8 < G::kN8 && warp < W; ++n8) {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float x = l[n8][c];
      x += __shfl_xor_sync(0xffffffffu, x, 4);
      x += __shfl_xor_sync(0xffffffffu, x, 8);
      x += __shfl_xor_sync(0xffffffffu, x, 16);
      const int hcol = n8 * 8 + 2 * qd + c;
      if (g == 0) {
        cm[warp * NH + hcol] = m[n8][c];
        cl[warp * NH + hcol] = x;
      }
#pragma unroll
      for (int j = 0; j < G::kDT; ++j) {
        co[(warp * NH + hcol) * D + out_dim<FP8>(j, g)] = o[n8][j][c];
        co[(warp * NH + hcol) * D + out_dim<FP8>(j, g + 8)] = o[n8][j][2 + c];
      }
    }
  }
  __syncthreads();
  constexpr int kThreadsPerHead = W * 32 / NH;
  constexpr int kPer = D / kThreadsPerHead;
  const int hcol = tid / kThreadsPerHead;
  if (hcol >= nh) return;
  float mstar = -INFINITY;
#pragma unroll
  for (int w = 0; w < W; ++w) mstar = fmaxf(mstar, cm[w * NH + hcol]);
  float wgt[W], lstar = 0.f;
#pragma unroll
  for (int w = 0; w < W; ++w) {
    const float mw = cm[w * NH + hcol];
    wgt[w] = mw == -INFINITY ? 0.f : fast_exp2(mw - mstar);
    lstar += wgt[w] * cl[w * NH + hcol];
  }
  const float norm = lstar > 0.f ? vscale / lstar : 0.f;
  const float lse = lstar > 0.f ? (mstar + log2f(lstar)) * kLn2 : -INFINITY;
  const int h = h0 + hcol;
  const int dbase = (tid % kThreadsPerHead) * kPer;
  if (p.part == nullptr) {
#pragma unroll 4
    for (int i = 0; i < kPer; ++i) {
      const int d = dbase + i;
      if (d >= p.DV) break;
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < W; ++w) v += wgt[w] * co[(w * NH + hcol) * D + d];
      store_float(p.out, p.ot, (int64_t)token * p.os0 + (int64_t)h * p.os1 + (int64_t)d * p.os2, v * norm);
    }
    if (tid % kThreadsPerHead == 0) p.lse[(int64_t)h * p.ls0 + (int64_t)token * p.ls1] = lse;
  } else {
    float* dst = p.part + (((int64_t)split * p.T + token) * p.HQ + h) * p.DV;
#pragma unroll 4
    for (int i = 0; i < kPer; ++i) {
      const int d = dbase + i;
      if (d >= p.DV) break;
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < W; ++w) v += wgt[w] * co[(w * NH + hcol) * D + d];
      dst[d] = v * norm;
    }
    if (tid % kThreadsPerHead == 0) p.part_lse[((int64_t)split * p.HQ + h) * p.T + token] = lse;
  }
}

// Stage ring + its 2*NST mbarriers (the warp merge reuses the ring), plus
// slack to align the ring to 1024 bytes for the 128-byte TMA swizzle.
template <bool FP8, int D, int W, int NH>
constexpr int smem_bytes(int nst) {
  using G = Geometry<FP8, D, W, NH>;
  const int pipe = nst * G::kStageBytes;
  const int merge = (2 * W * NH + W * NH * D) * 4;
  return (pipe > merge ? pipe : merge) + 16 * nst + 1024;
}

int page_shift_of(const AttnParams& p) {
  if (!p.paged || p.page <= 0 || (p.page & (p.page - 1))) return -1;
  int s = 0;
  while ((1 << s) < p.page) ++s;
  return s;
}

// CTA shape: consumer warps per CTA (16 tokens each per stage), pipeline
// stages and the occupancy bound, per K/V storage type. Measured on B200 with
// the TMA gather: FP8 4 warps x 3 stages x 4 CTAs/SM (48 KB ring each) beat
// 8 x 3 x 2 by 2-3% on 64 x 131072-token contexts. 16-bit K/V: 2 warps x 3
// stages x 4 CTAs/SM (48 KB ring) beat 4 x 3 x 2 (96 KB) by 17% at 64 x 1152
// tokens, 7% at 64 x 4096 and 1% on config 3 (256 x U[512, 32768]): with more,
// smaller CTAs per SM one CTA's prologue and pipeline fill overlap the others'
// streaming; 4 x 2 x 3, 2 x 2 x 5, 2 x 4 x 3 and 1 x 4 x 8 measured slower.
#ifndef FAB_DECODE_FP8_W
#define FAB_DECODE_FP8_W 4
#endif
#ifndef FAB_DECODE_FP8_NST
#define FAB_DECODE_FP8_NST 3
#endif
#ifndef FAB_DECODE_FP8_MINB
#define FAB_DECODE_FP8_MINB 4
#endif
#ifndef FAB_DECODE_16_W
#define FAB_DECODE_16_W 2
#endif
#ifndef FAB_DECODE_16_NST
#define FAB_DECODE_16_NST 3
#endif
#ifndef FAB_DECODE_16_MINB
#define FAB_DECODE_16_MINB 4
#endif
#ifndef FAB_DECODE_FP8_MIN_SPLITS
#define FAB_DECODE_FP8_MIN_SPLITS 4
#endif
#ifndef FAB_DECODE_16_MIN_SPLITS
#define FAB_DECODE_16_MIN_SPLITS 4
#endif
#ifndef FAB_DECODE_16_SLOT_FILL  // target CTAs per resident slot x 10 (16-bit, grid below the slots)
#define FAB_DECODE_16_SLOT_FILL 8
#endif
#ifndef FAB_DECODE_16_MIN_SPLITS_SMALL
#define FAB_DECODE_16_MIN_SPLITS_SMALL 1
#endif
#ifndef FAB_DECODE_TMA
#define FAB_DECODE_TMA 1
#endif

// TMA page gathers: paged K/V whose pages are whole 1024-byte swizzle atoms
// (page >= 8 tokens, power of two) and whose strides suit a tensor map. Odd
// page sizes and packed K/V keep the per-row cp.async gather.
bool use_tma(const AttnParams& p, int page_shift) {
  if (!FAB_DECODE_TMA || !p.paged || page_shift < 3 || !tensor_map_available()) return false;
  const int64_t elt = p.kt == FA_E4M3 ? 1 : 2;
  const int64_t lim = (int64_t)1 << 40;
  for (int64_t st : {p.ks0, p.ks1, p.ks2, p.vs0, p.vs1, p.vs2})
    if (st <= 0 || (st * elt) % 16 != 0 || st * elt >= lim) return false;
  return p.k_pages > 0 && p.k_pages < ((int64_t)1 << 31);
}

// 4-D map over one K or V cache: (head dim, kv head, token in page, page).
int make_page_map(CUtensorMap* map, const void* base, int dtype, const AttnParams& p, bool is_v, int box_tok) {
  const int64_t elt = dtype == FA_E4M3 ? 1 : 2;
  const int D = is_v ? p.DV : p.DQ;
  const uint64_t dims[4] = {(uint64_t)D, (uint64_t)p.HK, (uint64_t)p.page, (uint64_t)p.k_pages};
  const uint64_t strides[3] = {(uint64_t)((is_v ? p.vs2 : p.ks2) * elt), (uint64_t)((is_v ? p.vs1 : p.ks1) * elt),
                               (uint64_t)((is_v ? p.vs0 : p.ks0) * elt)};
  const uint32_t box[4] = {(uint32_t)(128 / elt), 1u, (uint32_t)box_tok, 1u};
  return encode_tensor_map(map, dtype, 4, base, dims, strides, box, true);
}

template <typename MT, bool FP8, int D, int NH, bool PREC, bool QFOLD>
int launch_cfg(const AttnParams& p, int splits, int span, cudaStream_t stream) {
  constexpr int W = FP8 ? FAB_DECODE_FP8_W : FAB_DECODE_16_W;
  constexpr int NST = FP8 ? FAB_DECODE_FP8_NST : FAB_DECODE_16_NST;
  // 256-wide rows: a 3-stage ring of 32 KB stages leaves room for 2 CTAs per
  // SM (FP8 with 16 heads per CTA: one, its accumulators need the registers).
  constexpr int MINB = (FP8 && NH == 16) ? 1 : D > 128 ? 2 : (FP8 ? FAB_DECODE_FP8_MINB : FAB_DECODE_16_MINB);
  constexpr int smem = smem_bytes<FP8, D, W, NH>(NST);
  const int shift = page_shift_of(p);
  const bool tma = use_tma(p, shift);
  auto kernel = tma ? decode_mma_kernel<MT, FP8, D, W, NH, NST, PREC, QFOLD, true, MINB>
                    : decode_mma_kernel<MT, FP8, D, W, NH, NST, PREC, QFOLD, false, MINB>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return fail(FA_ERR_CUDA, "decode smem attribute: %s", cudaGetErrorString(e));
  const int group = p.HQ / p.HK;
  const int hblocks = (group + NH - 1) / NH;
  constexpr int kTile = Geometry<FP8, D, W, NH>::kTile;
  const int box_tok = tma ? min(p.page, kTile) : 0;
  CUtensorMap tmk, tmv;
  memset(&tmk, 0, sizeof(tmk));
  memset(&tmv, 0, sizeof(tmv));
  if (tma) {
    const int kd = FP8 ? FA_E4M3 : p.kt;
    int rc = make_page_map(&tmk, p.k, kd, p, false, box_tok);
    if (rc == FA_OK) rc = make_page_map(&tmv, p.v, kd, p, true, box_tok);
    if (rc != FA_OK) return rc;
  }
  dim3 grid((unsigned)splits, (unsigned)(p.HK * hblocks), (unsigned)p.B);
  kernel<<<grid, (W + (tma ? 1 : 0)) * 32, smem, stream>>>(tmk, tmv, p, span, hblocks, shift, box_tok);
  note_launch();
  FAB_LAUNCH_CHECK("decode launch");
  return FA_OK;
}

template <typename MT, bool FP8, int D>
int launch_heads(const AttnParams& p, int splits, int span, bool prec, bool qfold, cudaStream_t st) {
  const bool wide = p.HQ / p.HK > 8;
  if (qfold) {
    // bf16 queries over FP8 K/V: scale folded into f16 query fragments; an
    // fp32 output (e.g. a multi-GPU partial) also keeps P to ~22 bits.
    if (prec)
      return wide ? launch_cfg<MT, FP8, D, 16, true, true>(p, splits, span, st)
                  : launch_cfg<MT, FP8, D, 8, true, true>(p, splits, span, st);
    return wide ? launch_cfg<MT, FP8, D, 16, false, true>(p, splits, span, st)
                : launch_cfg<MT, FP8, D, 8, false, true>(p, splits, span, st);
  }
  if (prec) {
    return wide ? launch_cfg<MT, FP8, D, 16, true, false>(p, splits, span, st)
                : launch_cfg<MT, FP8, D, 8, true, false>(p, splits, span, st);
  }
  return wide ? launch_cfg<MT, FP8, D, 16, false, false>(p, splits, span, st)
              : launch_cfg<MT, FP8, D, 8, false, false>(p, splits, span, st);
}

bool aligned16(const void* ptr) { return ((uintptr_t)ptr & 15u) == 0; }

int tile_tokens(const AttnParams& p) { return p.kt == FA_E4M3 ? 16 * FAB_DECODE_FP8_W : 16 * FAB_DECODE_16_W; }

}  // namespace

int decode_mma_supported(const AttnParams& p) {
  const bool q16 = p.qt == FA_F16 || p.qt == FA_BF16;
  if (!q16 || p.kt != p.vt) return 0;
  const bool fp8 = p.kt == FA_E4M3;
  if (!fp8 && p.kt != p.qt) return 0;
  if (p.DQ != p.DV) return 0;
  // Head dims up to 128 (multiples of 8, of 16 for FP8 rows) run on the 64-
  // (16-bit) or 128-wide instantiation, head dims 129..256 on the 256-wide
  // one: the tail of Q reads as zero, K/V chunks past the true dim are
  // zero-filled (TMA out-of-bounds fill or cp.async zero fill) and only
  // true-dim outputs are written.
  if (p.DQ < 8 || p.DQ > 256 || p.DQ % (fp8 ? 16 : 8)) return 0;
  if (p.alibi || p.mask != 0) return 0;
  if (p.ks3 != 1 || p.vs3 != 1) return 0;
  const int elt = fp8 ? 1 : 2;
  if (!aligned16(p.k) || !aligned16(p.v)) return 0;
  const int64_t ks[3] = {p.ks0, p.ks1, p.ks2}, vs[3] = {p.vs0, p.vs1, p.vs2};
  for (int i = p.paged ? 0 : 1; i < 3; ++i)
    if ((ks[i] * elt) % 16 != 0 || (vs[i] * elt) % 16 != 0) return 0;
  if (p.B > 65535 || p.HK * ((p.HQ / p.HK + 15) / 16) > 65535) return 0;
  return 1;
}

int decode_default_splits(const AttnParams& p, int* span) {
  const int eff = p.win_l >= 0 ? min(p.max_k, p.win_l + 1) : p.max_k;
  const int group = p.HQ / p.HK;
  const int64_t units = (int64_t)p.B * p.HK * ((group + 15) / 16);
  const int by_len = max(1, (eff + 255) / 256);
  int splits;
  if (p.kt == FA_E4M3) {
    // Few long splits amortise each CTA's prologue and pipeline fill (measured:
    // 4 splits beat 8..32 on uniform 131072-token contexts); more splits only
    // when the grid would not fill the SMs.
    const int want = (int)((8LL * sm_count() + units - 1) / units);
    splits = max(want, FAB_DECODE_FP8_MIN_SPLITS);
  } else {
    // When one split per (request, KV head) already fills the resident CTA
    // slots, 4 splits keep a ragged batch from ending on its longest request
    // (config 3: 6.84 TB/s; 2 splits 6.64); otherwise enough splits for ~0.8
    // CTAs per slot, all resident at once without a second partial wave (64
    // requests x 1152 / 2048 / 4096 / 16384 tokens: 1 split 5.62 / 6.10 /
    // 6.43 / 6.99 TB/s against 4.32 / 5.18 / 6.03 / 6.80 with 2).
    const int64_t slots = (int64_t)sm_count() * FAB_DECODE_16_MINB;
    const int want = (int)((FAB_DECODE_16_SLOT_FILL * slots + 10 * units - 1) / (10 * units));
    splits = max(want, units >= slots ? FAB_DECODE_16_MIN_SPLITS : FAB_DECODE_16_MIN_SPLITS_SMALL);
  }
  splits = max(1, min(splits, by_len));
  *span = (eff + splits - 1) / splits;
  return splits;
}

int decode_timeout_flag(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_decode_timeout, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_decode_timeout, &zero, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

int launch_decode_mma(const AttnParams& p, int splits, int span, cudaStream_t stream) {
  const int tile = tile_tokens(p);
  span = (span + tile - 1) / tile * tile;
  const bool fp8 = p.kt == FA_E4M3;
  const bool prec = p.ot == FA_F32;
  if (fp8) {
    const bool qfold = p.qt == FA_BF16;
    return p.DQ <= 128 ? launch_heads<__half, true, 128>(p, splits, span, prec, qfold, stream)
                       : launch_heads<__half, true, 256>(p, splits, span, prec, qfold, stream);
  }
  if (p.qt == FA_BF16) {
    return p.DQ <= 64    ? launch_heads<__nv_bfloat16, false, 64>(p, splits, span, prec, false, stream)
           : p.DQ <= 128 ? launch_heads<__nv_bfloat16, false, 128>(p, splits, span, prec, false, stream)
                         : launch_heads<__nv_bfloat16, false, 256>(p, splits, span, prec, false, stream);
  }
  return p.DQ <= 64    ? launch_heads<__half, false, 64>(p, splits, span, prec, false, stream)
         : p.DQ <= 128 ? launch_heads<__half, false, 128>(p, splits, span, prec, false, stream)
                       : launch_heads<__half, false, 256>(p, splits, span, prec, false, stream);
}

}  // namespace fab
