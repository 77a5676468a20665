// mtp_sqattn.cuh -- single-query attention for 16-bit K/V, head size a
// multiple of 8 up to 256: the reference's fused_tree_attention (contiguous
// K/V, one float mask shared by every (b, h), mtp_kernels.py:1165-1191,
// eager 859-872) and fused_paged_attention (per-token page table,
// mtp_kernels.py:1136-1162, eager 832-856), built to keep HBM busy.
//
// One 256-thread CTA per query row (b, h).  A key's D elements are CPK =
// D/8 chunks of 16 bytes; a warp covers KPW = 32/CPK keys at once.
//   1. kept keys: with a mask, compacted in key order with ballots; a paged
//      row resolves each key's page once here (ids checked against the pool);
//   2. scores: every lane loads its 16-byte chunk of U = 4 keys before any
//      arithmetic (4 loads in flight per lane), dot product with its chunk of
//      q (in registers), segmented shuffle sum over the key's CPK lanes;
//   3. softmax statistics over the scores in shared memory;
//   4. P V: thread t owns chunk t % CPK of D and every (256/CPK)-th key,
//      again 4 keys' loads in flight; the partial rows are summed in shared
//      memory and divided by the softmax sum.
// A row with no kept key is NaN (the reference's softmax of all -inf).
#pragma once

#include "mtp_rowattn.cuh"

namespace mtp {
namespace sq {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxD = 256;
constexpr int kUnroll = 4;

struct Args {
  const void* q;
  void* out;
  int64_t B, H, D;
  float scale;
  // contiguous K/V [B, H, L, D] and mask [L] (nullable), or paged pools
  // [P, B, H, page_size, D] with page_table [B, table_stride]
  const void* k;
  const void* v;
  const float* mask;
  const int32_t* page_table;
  int64_t table_stride, num_pages, page_size;
  int64_t L;
  int paged;
};

// Dynamic shared memory: scores [L] fp32, key offsets [L] int64 (element
// offset of each kept key's row), partial O [256/CPK][D] fp32.
inline size_t smem_bytes(int64_t L, int64_t D) {
  const int64_t cpk = D / 8, groups = kThreads / cpk;
  return (size_t)L * 4 + (size_t)L * 8 + (size_t)groups * D * 4 + 16;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) sq_attention_kernel(Args a) {
  extern __shared__ float4 smem4[];
  const int D = (int)a.D, L = (int)a.L;
  const int CPK = D / 8, KPW = 32 / CPK, GROUPS = kThreads / CPK;
  float* sp = reinterpret_cast<float*>(smem4);
  int64_t* soff = reinterpret_cast<int64_t*>(reinterpret_cast<uint8_t*>(smem4) + (((size_t)L * 4 + 15) & ~size_t(15)));
  float* spo = reinterpret_cast<float*>(soff + L);
  __shared__ float red[kWarps];
  __shared__ int red_i[kWarps];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = blockIdx.x;
  const int64_t b = row / a.H, h = row % a.H;
  const T* kbase = static_cast<const T*>(a.k);
  const T* vbase = static_cast<const T*>(a.v);

  // 1. kept keys and their element offsets
  int nkeep = 0;
  for (int base = 0; base < L; base += kThreads) {
    const int j = base + threadIdx.x;
    bool keep = j < L && (a.paged || a.mask == nullptr || a.mask[j] > 0.5f);
    int64_t off = 0;
    if (keep) {
      if (a.paged) {
        const int64_t page = resolve_page(a.page_table[b * a.table_stride + j], a.num_pages);
        if (page < 0) {
          record_error(MTP_ERR_DEVICE);
          keep = false;
        } else {
          off = ((((int64_t)page * a.B + b) * a.H + h) * a.page_size + j % a.page_size) * a.D;
        }
      } else {
        off = ((b * a.H + h) * (int64_t)L + j) * a.D;
      }
    }
    const unsigned bal = __ballot_sync(0xffffffffu, keep);
    if (lane == 0) red_i[warp] = __popc(bal);
    __syncthreads();
    int before = nkeep, total = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      before += (w < warp) ? red_i[w] : 0;
      total += red_i[w];
    }
    if (keep) soff[before + __popc(bal & ((1u << lane) - 1u))] = off;
    nkeep += total;
    __syncthreads();
  }

  // 2. scores: lane -> (key slot lane / CPK, chunk lane % CPK)
  const int chunk = lane % CPK, kslot = lane / CPK;
  float qv[8];
  rowattn::load_vec<T, 8>(static_cast<const T*>(a.q) + row * a.D + chunk * 8, qv);
  const int keys_per_step = kWarps * KPW;  // keys the CTA covers per unroll slot
  for (int i0 = 0; i0 < nkeep; i0 += keys_per_step * kUnroll) {
    float f[kUnroll][8];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int i = i0 + u * keys_per_step + warp * KPW + kslot;
      if (kslot < KPW && i < nkeep) rowattn::load_vec<T, 8>(kbase + soff[i] + chunk * 8, f[u]);
      else
#pragma unroll
        for (int e = 0; e < 8; ++e) f[u][e] = 0.f;
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) s = fmaf(qv[e], f[u][e], s);
      for (int o = CPK >> 1; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      const int i = i0 + u * keys_per_step + warp * KPW + kslot;
      if (chunk == 0 && kslot < KPW && i < nkeep) sp[i] = s * a.scale;
    }
  }
  __syncthreads();

  // 3. softmax statistics
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < nkeep; i += kThreads) mx = fmaxf(mx, sp[i]);
  mx = rowattn::block_max(mx, red);
  float sum = 0.f;
  for (int i = threadIdx.x; i < nkeep; i += kThreads) {
    const float p = expf(sp[i] - mx);
    sp[i] = p;
    sum += p;
  }
  sum = rowattn::block_sum(sum, red);  // its barriers also publish sp

  // 4. P V: thread -> (key group t / CPK, chunk t % CPK)
  const int pchunk = threadIdx.x % CPK, grp = threadIdx.x / CPK;
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  for (int i0 = grp; i0 < nkeep; i0 += GROUPS * kUnroll) {
    float f[kUnroll][8];
    float p[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int i = i0 + u * GROUPS;
      p[u] = 0.f;
      if (i < nkeep) {
        rowattn::load_vec<T, 8>(vbase + soff[i] + pchunk * 8, f[u]);
        p[u] = sp[i];
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) f[u][e] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = fmaf(p[u], f[u][e], acc[e]);
  }
  if (grp < GROUPS) {
#pragma unroll
    for (int e = 0; e < 8; ++e) spo[grp * D + pchunk * 8 + e] = acc[e];
  }
  __syncthreads();
  const float inv = nkeep > 0 ? 1.0f / sum : __int_as_float(0x7fc00000);  // no kept key: NaN
  T* orow = static_cast<T*>(a.out) + row * a.D;
  for (int d = threadIdx.x; d < D; d += kThreads) {
    float o = 0.f;
    for (int g = 0; g < GROUPS; ++g) o += spo[g * D + d];
    orow[d] = rowattn::from_f32<T>(o * inv);
  }
}

}  // namespace sq
}  // namespace mtp
