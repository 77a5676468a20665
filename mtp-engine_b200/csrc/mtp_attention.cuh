// mtp_attention.cuh -- single-query (decode) attention on CUDA cores.
//
// One 128-thread block per query row.  It serves the reference's two
// single-query operators exactly as they are defined -- fused_tree_attention
// (contiguous K/V with a float mask shared by all heads,
// mtp_kernels.py:560-613 / 859-872) and fused_paged_attention (per-token page
// table, mtp_kernels.py:495-554 / 832-856) -- and is the general-shape path of
// the paged tree attention (context pages + tree nodes under the ancestor
// mask, with GQA).  Each warp streams every 4th key with 16-bit/32-bit loads
// spread over the head dimension, keeps an online softmax (running max, sum,
// fp32 accumulator), and the four warps are merged at the end.  A row whose
// keys are all masked yields NaN, like the reference's eager softmax.
#pragma once

#include "mtp_common.cuh"

namespace mtp {

enum AttnKind : int { ATTN_CONTIG = 0, ATTN_PAGED = 1, ATTN_TREE_PAGED = 2 };

struct AttnArgs {
  int kind;
  int dtype;
  const void* q;
  void* out;
  int64_t B, T, Hq, Hkv, D;  // queries: B x T x Hq (T = 1 for the single-query ops)
  float scale;
  // ATTN_CONTIG: k/v [B,H,L,D], mask [L] (nullable)
  const void* k;
  const void* v;
  const float* mask;
  int64_t L;
  // ATTN_PAGED / ATTN_TREE_PAGED: pages [P,B,Hkv,page_size,D], table [B, table_stride]
  const void* k_pages;
  const void* v_pages;
  const int32_t* page_table;
  int64_t table_stride, num_pages, page_size, ctx_len;
  // ATTN_TREE_PAGED: tree K/V [B,Hkv,T,D], tree_mask [T,T]
  const void* tree_k;
  const void* tree_v;
  const float* tree_mask;
  // kv_custom != 0: K/V in kv_dtype (e.g. E4M3), each multiplied by
  // kscale[kv head] / vscale[kv head] (null = 1) -- fused_causal_attention_fp8,
  // mtp_kernels.py:1105-1133 (eager 817-830).  0: K/V in dtype, unscaled.
  int kv_custom;
  int kv_dtype;
  const float* kscale;
  const float* vscale;
};

constexpr int kAttnMaxDPerLane = 8;  // head_dim <= 256

__global__ void __launch_bounds__(128) decode_attention_kernel(AttnArgs a) {
  __shared__ float sm_m[4], sm_l[4];
  __shared__ float sm_acc[4][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // query row -> (b, n, h); q/out are [B, T, Hq, D]
  const int64_t qrow = blockIdx.x;
  const int64_t h = qrow % a.Hq;
  const int64_t n = (qrow / a.Hq) % a.T;
  const int64_t b = qrow / (a.Hq * a.T);
  const int64_t hk = h / (a.Hq / a.Hkv);
  const int64_t D = a.D;
  const int nd = (int)((D + 31) / 32);
  const int kvdt = a.kv_custom ? a.kv_dtype : a.dtype;
  const float ks = (a.kv_custom && a.kscale) ? a.kscale[hk] : 1.0f;
  const float vs = (a.kv_custom && a.vscale) ? a.vscale[hk] : 1.0f;

  float qv[kAttnMaxDPerLane], acc[kAttnMaxDPerLane];
#pragma unroll
  for (int i = 0; i < kAttnMaxDPerLane; ++i) {
    const int64_t d = lane + 32 * i;
    qv[i] = (i < nd && d < D) ? load_f32(a.q, a.dtype, qrow * D + d) : 0.f;
    acc[i] = 0.f;
  }
  float m = -INFINITY, l = 0.f;

  int64_t nkeys;
  if (a.kind == ATTN_CONTIG) nkeys = a.L;
  else if (a.kind == ATTN_PAGED) nkeys = a.L;
  else nkeys = a.ctx_len + a.T;

  for (int64_t j = warp; j < nkeys; j += 4) {
    const void* kp;
    const void* vp;
    int64_t off;
    if (a.kind == ATTN_CONTIG) {
      if (a.mask && !(a.mask[j] > 0.5f)) continue;
      off = ((b * a.Hkv + hk) * a.L + j) * D;
      kp = a.k;
      vp = a.v;
    } else if (a.kind == ATTN_PAGED || j < a.ctx_len) {
      const int64_t page = resolve_page(a.page_table[b * a.table_stride + j], a.num_pages);
      if (page < 0) {
        if (lane == 0) record_error(MTP_ERR_DEVICE);
        continue;
      }
      off = (((int64_t)page * a.B + b) * a.Hkv + hk) * a.page_size * D + (j % a.page_size) * D;
      kp = a.k_pages;
      vp = a.v_pages;
    } else {
      const int64_t t = j - a.ctx_len;
      if (!(a.tree_mask[n * a.T + t] > 0.5f)) continue;
      off = ((b * a.Hkv + hk) * a.T + t) * D;
      kp = a.tree_k;
      vp = a.tree_v;
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kAttnMaxDPerLane; ++i) {
      const int64_t d = lane + 32 * i;
      if (i < nd && d < D) s = fmaf(qv[i], load_f32(kp, kvdt, off + d) * ks, s);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    s *= a.scale;
    const float m_new = fmaxf(m, s);
    const float corr = expf(m - m_new);
    const float p = expf(s - m_new);
    l = l * corr + p;
#pragma unroll
    for (int i = 0; i < kAttnMaxDPerLane; ++i) {
      const int64_t d = lane + 32 * i;
      if (i < nd && d < D) acc[i] = acc[i] * corr + p * (load_f32(vp, kvdt, off + d) * vs);
    }
    m = m_new;
  }
  if (lane == 0) {
    sm_m[warp] = m;
    sm_l[warp] = l;
  }
#pragma unroll
  for (int i = 0; i < kAttnMaxDPerLane; ++i) {
    const int64_t d = lane + 32 * i;
    if (i < nd && d < D) sm_acc[warp][d] = acc[i];
  }
  __syncthreads();
  const float M = fmaxf(fmaxf(sm_m[0], sm_m[1]), fmaxf(sm_m[2], sm_m[3]));
  float w[4], L = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    w[i] = sm_m[i] == -INFINITY ? 0.f : expf(sm_m[i] - M);
    L += sm_l[i] * w[i];
  }
  for (int64_t d = threadIdx.x; d < D; d += blockDim.x) {
    float o = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) o += sm_acc[i][d] * w[i];
    store_f32(a.out, a.dtype, qrow * D + d, o / L);
  }
}

}  // namespace mtp
