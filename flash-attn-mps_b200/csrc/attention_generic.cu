// Generic attention kernel: every feature, every storage dtype (f16, bf16,
// f32, FP8 E4M3), head dims 1..512 and DiffKV, packed or paged K/V, split-KV.
//
// It is the semantic backbone of the library (the fast kernels cover the
// common shapes): one CTA owns ROWS query rows of one (request, head, split),
// stages BK-key tiles of K and V in shared memory as fp32, and each warp runs
// an fp32 online softmax over its rows (natural exp, precise expf/logf/tanhf).
// Semantics follow the reference's attention_tiled / attention_vector
// (flash_attn_mps/kernels/attention.metal:29-51 allowed_key/attention_score,
// 60-181 tile bounds and LSE, 185-248 per-row loop). Keys outside the visible
// range are zero-filled in shared memory, so NaN-poisoned cache tails never
// reach the arithmetic.
#include "features.cuh"
#include "kernels.cuh"

namespace fab {
namespace {

constexpr int kRowsPerWarp = 2;
constexpr int kWarps = 8;
constexpr int kRows = kRowsPerWarp * kWarps;
constexpr int kBK = 32;

template <int NC>  // NC = number of 32-wide value-dimension chunks per lane
__global__ void __launch_bounds__(kWarps * 32) generic_attention_kernel(AttnParams p) {
  extern __shared__ float smem[];
  const int DQ = p.DQ, DV = p.DV, LK = DQ + 1;
  float* qs = smem;                    // [kRows][DQ]
  float* ks = qs + kRows * DQ;         // [kBK][DQ+1]
  float* vs = ks + kBK * LK;           // [kBK][DV]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.z / p.splits, split = blockIdx.z % p.splits;
  const int h = blockIdx.y, kh = h / (p.HQ / p.HK);
  const int q_begin = p.cu_q[b * p.cq0];
  const int q_len = p.cu_q[(b + 1) * p.cq0] - q_begin;
  const int q_block = blockIdx.x * kRows;
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

  for (int z = tid; z < kRows * DQ; z += kWarps * 32) {
    const int r = z / DQ, d = z - r * DQ;
    qs[z] = q_block + r < q_len
                ? load_float(p.q, p.qt, (int64_t)(q_begin + q_block + r) * p.qs0 + h * p.qs1 + d * p.qs2)
                : 0.f;
  }

  // Tile bounds of this split (attention.metal:108-118).
  const int tile_count = (k_len + kBK - 1) / kBK;
  int first = (int)((int64_t)tile_count * split / p.splits);
  int last = (int)((int64_t)tile_count * (split + 1) / p.splits);
  const int row_end = min(q_block + kRows, q_len);
  if (p.cp_n <= 1) {  // tile skipping in local positions (positions are strided under context parallelism)
    if (causal && p.mask == 0) last = min(last, max(0, (row_end + k_len - q_len + kBK - 1) / kBK));
    if (p.mask == 0 && p.win_l >= 0) first = max(first, max(0, q_block + k_len - q_len - p.win_l) / kBK);
    if (p.mask == 0 && p.win_r >= 0)
      last = min(last, max(0, (row_end + k_len - q_len + p.win_r + kBK - 1) / kBK));
  }

  float m[kRowsPerWarp], l[kRowsPerWarp], acc[kRowsPerWarp][NC];
#pragma unroll
  for (int rr = 0; rr < kRowsPerWarp; ++rr) {
    m[rr] = sink;
    l[rr] = isfinite(sink) ? 1.f : 0.f;
#pragma unroll
    for (int i = 0; i < NC; ++i) acc[rr][i] = 0.f;
  }

  for (int kb = first; kb < last; ++kb) {
    __syncthreads();
    for (int z = tid; z < kBK * DQ; z += kWarps * 32) {
      const int j = z / DQ, d = z - j * DQ, t = kb * kBK + j;
      float x = 0.f;
      if (t < k_len) x = load_float(p.k, p.kt, kv_offset(p, b, (int64_t)k_begin + left + t, kh, false) + d * p.ks3);
      ks[j * LK + d] = x;
    }
    for (int z = tid; z < kBK * DV; z += kWarps * 32) {
      const int j = z / DV, d = z - j * DV, t = kb * kBK + j;
      float x = 0.f;
      if (t < k_len) x = load_float(p.v, p.vt, kv_offset(p, b, (int64_t)k_begin + left + t, kh, true) + d * p.vs3);
      vs[z] = x;
    }
    __syncthreads();
#pragma unroll
    for (int rr = 0; rr < kRowsPerWarp; ++rr) {
      const int r = warp * kRowsPerWarp + rr;
      if (q_block + r >= q_len) continue;
      const int q_abs = q_block + r + k_tot - q_len;
      const int t = kb * kBK + lane, tg = key_pos(p, t);
      float dot = 0.f;
      const float* qrow = qs + r * DQ;
      const float* krow = ks + lane * LK;
      for (int d = 0; d < DQ; ++d) dot = fmaf(qrow[d], krow[d], dot);
      float s = dot * scale;
      if (p.softcap > 0.f) s = p.softcap * tanhf(s / p.softcap);
      s -= slope * fabsf((float)(q_abs - tg));
      const bool keep = t < k_len && allowed_key(p, b, tg, q_abs, (int64_t)q_begin + q_block + r, causal);
      s = keep ? s : -INFINITY;
      const float m_new = fmaxf(m[rr], warp_max(s));
      const float pr = (m_new == -INFINITY || s == -INFINITY) ? 0.f : expf(s - m_new);
      const float factor = m[rr] == -INFINITY ? 0.f : expf(m[rr] - m_new);
      l[rr] = l[rr] * factor + warp_sum(pr);
#pragma unroll
      for (int i = 0; i < NC; ++i) acc[rr][i] *= factor;
      for (int j = 0; j < kBK; ++j) {
        const float pj = __shfl_sync(0xffffffffu, pr, j);
        if (pj == 0.f) continue;
        const float* vrow = vs + j * DV;
#pragma unroll
        for (int i = 0; i < NC; ++i) {
          const int d = lane + 32 * i;
          if (d < DV) acc[rr][i] = fmaf(pj, vrow[d], acc[rr][i]);
        }
      }
      m[rr] = m_new;
    }
  }

#pragma unroll
  for (int rr = 0; rr < kRowsPerWarp; ++rr) {
    const int r = warp * kRowsPerWarp + rr;
    if (q_block + r >= q_len) continue;
    const int64_t t = q_begin + q_block + r;
    const float norm = l[rr] > 0.f ? vscale / l[rr] : 0.f;
    const float lse = l[rr] > 0.f ? m[rr] + logf(l[rr]) : -INFINITY;
    if (p.splits == 1) {
#pragma unroll
      for (int i = 0; i < NC; ++i) {
        const int d = lane + 32 * i;
        if (d < DV) store_float(p.out, p.ot, t * p.os0 + h * p.os1 + d * p.os2, acc[rr][i] * norm);
      }
      if (lane == 0) p.lse[h * p.ls0 + t * p.ls1] = lse;
    } else {
      float* dst = p.part + (((int64_t)split * p.T + t) * p.HQ + h) * DV;
#pragma unroll
      for (int i = 0; i < NC; ++i) {
        const int d = lane + 32 * i;
        if (d < DV) dst[d] = acc[rr][i] * norm;
      }
      if (lane == 0) p.part_lse[((int64_t)split * p.HQ + h) * p.T + t] = lse;
    }
  }
}

template <int NC>
int launch_nc(const AttnParams& p, cudaStream_t stream) {
  const size_t smem = sizeof(float) * ((size_t)kRows * p.DQ + (size_t)kBK * (p.DQ + 1) + (size_t)kBK * p.DV);
  auto kernel = generic_attention_kernel<NC>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(FA_ERR_CUDA, "generic attention smem attribute: %s", cudaGetErrorString(e));
  }
  dim3 grid((unsigned)((p.max_q + kRows - 1) / kRows), (unsigned)p.HQ, (unsigned)((int64_t)p.B * p.splits));
  kernel<<<grid, kWarps * 32, smem, stream>>>(p);
  note_launch();
  FAB_LAUNCH_CHECK("generic attention launch");
  return FA_OK;
}

}  // namespace

int launch_generic_attention(const AttnParams& p, cudaStream_t stream) {
  if ((int64_t)p.B * p.splits > 65535 * 1024LL) return fail(FA_ERR_UNSUPPORTED, "batch*splits too large");
  const int nc = (p.DV + 31) / 32;
  if (nc <= 1) return launch_nc<1>(p, stream);
  if (nc <= 2) return launch_nc<2>(p, stream);
  if (nc <= 4) return launch_nc<4>(p, stream);
  if (nc <= 8) return launch_nc<8>(p, stream);
  return launch_nc<16>(p, stream);
}

}  // namespace fab
