// mtp_attention_tc2.cuh -- second tensor-core paged tree attention kernel:
// 64-key chunks with the score tile double-buffered per query tile in TMEM,
// so the MMA for chunk c+2 runs while the softmax works on chunk c+1.
//
// Same unit and roles as tree_attention_tc_kernel (mtp_attention_tc.cuh):
// one CTA per (sequence, KV head), the unit's query rows held as two 128-row
// tiles, TMA producer (warp 0), page-table reader (warp 10), MMA issuer
// (warp 1), softmax warps 2-5 (tile 0) and 6-9 (tile 1).  What changes:
//   TMEM   tile t: S_t[0] (64 cols) | S_t[1] (64 cols) | O_t (128 cols) at t*256
//   S_t(c)   = Q_t K(c)^T, M128 N64 K128, into S_t[c % 2]
//   P_t(c)   bf16 pairs over the first 32 columns of S_t[c % 2]
//   O_t     += P_t(c) V(c), M128 N128 K64 (A from TMEM, V MN-major)
//   order    S(0) S(1) | PV_t(c), then S_t(c+2) into the buffer PV_t(c) just
//            read (tcgen05 MMAs of one thread execute in issue order)
// A softmax thread waits only for its own S_t(c); it waits for the previous
// PV only when the lazy rescale of O is needed.  K and V chunks are 16 KB, in
// a 9-deep ring.  Page sizes 8..64.
//
// This kernel runs only when the environment sets MTP_ATTN_KERNEL=2.
#pragma once

#include "mtp_attention_tc.cuh"

namespace mtp {
namespace attn2 {

using attn::Params;
using attn::ex2;
using attn::fmax3;
using attn::ffma2;
using attn::add2;
using attn::pack_bf16;

constexpr int kThreads = 352;
constexpr int kD = 128;
constexpr int kChunk = 64;                       // keys per chunk
constexpr int kQHalf = 128 * 128;                // Q tile: 128 rows x 128 bytes per D-half
constexpr int kQTile = 2 * kQHalf;
constexpr int kHalf = kChunk * 128;              // K/V chunk: 64 rows x 128 bytes per D-half
constexpr int kItem = 2 * kHalf;                 // one K or V chunk, 16 KB
constexpr int kNumBuf = 9;
constexpr int kIdRing = 16;
constexpr int kMaxPages = 8;                     // page_size >= 8
constexpr int kBarBytes = 640;                   // 64 mbarriers + TMEM slot + abort flag
constexpr int kSmemBytes = 2 * kQTile + kNumBuf * kItem + kIdRing * kMaxPages * 4 + kBarBytes + 1024;
constexpr float kRescaleThreshold = 8.0f;
// mbarriers: q_full, buf_full/empty [kNumBuf], s_full [4], p_full [4], pv_done [2],
// o_done [2], ids_full/empty [kIdRing], drain; then the TMEM slot and the abort flag
static_assert((1 + 2 * kNumBuf + 4 + 4 + 2 + 2 + 2 * kIdRing + 1) * 8 + 8 <= kBarBytes, "barrier area");
static_assert(kQTile % 1024 == 0 && kItem % 1024 == 0 && (kIdRing * kMaxPages * 4) % 8 == 0, "buffer alignment");
static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");

template <int AB_FMT>
__global__ void __launch_bounds__(kThreads, 1)
    tree_attention_tc2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                              const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmTK,
                              const __grid_constant__ CUtensorMap tmTV, Params p) {
  constexpr uint32_t IDESC_S = make_idesc(AB_FMT, 128, kChunk);        // Q (K-major) x K (K-major)
  constexpr uint32_t IDESC_PV = make_idesc(AB_FMT, 128, kD, 0u, 1u);  // P (TMEM) x V (MN-major)

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sBuf = sQ + 2 * kQTile;
  int* sIds = reinterpret_cast<int*>(sBuf + kNumBuf * kItem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sIds + kIdRing * kMaxPages);
  uint64_t* q_full = bars;
  uint64_t* buf_full = q_full + 1;             // [kNumBuf]
  uint64_t* buf_empty = buf_full + kNumBuf;    // [kNumBuf]
  uint64_t* s_full = buf_empty + kNumBuf;      // [tile][buffer]
  uint64_t* p_full = s_full + 4;               // [tile][buffer]
  uint64_t* pv_done = p_full + 4;              // [tile], one phase per PV
  uint64_t* o_done = pv_done + 2;              // [tile], completes once: after the last PV
  uint64_t* ids_full = o_done + 2;             // [kIdRing]
  uint64_t* ids_empty = ids_full + kIdRing;    // [kIdRing]
  uint64_t* drain = ids_empty + kIdRing;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int unit = blockIdx.x / p.splits, split = blockIdx.x % p.splits;
  const int b = unit / p.Hkv, kvh = unit % p.Hkv;
  const int c0 = split * p.chunks_per_split;
  const int c1 = min(p.n_chunks, c0 + p.chunks_per_split);
  const int n_iter = c1 - c0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kNumBuf; ++i) {
      mbar_init(&buf_full[i], 1);
      mbar_init(&buf_empty[i], 1);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);  // one arrival per softmax warp
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&pv_done[t], 1);
      mbar_init(&o_done[t], 1);
    }
    for (int i = 0; i < kIdRing; ++i) {
      mbar_init(&ids_full[i], 1);
      mbar_init(&ids_empty[i], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (n_iter > 0 && warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    const int ppc = kChunk / p.ps;
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmTK);
      tma_prefetch_desc(&tmTV);
      mbar_expect_tx(q_full, p.n_tiles * kQTile);
      for (int t = 0; t < p.n_tiles; ++t)
        for (int h = 0; h < 2; ++h)
          tma_load_4d(sQ + t * kQTile + h * kQHalf, &tmQ, h * 64, kvh * p.G, t * p.t_per_tile, b, q_full);
    }
    int item = 0;
    bool ok = true;
    for (int c = c0; c < c1 && ok; ++c) {
      const bool is_ctx = c < p.n_ctx_chunks;
      const int slot = (c - c0) % kIdRing;
      int pg = 0;
      if (is_ctx) {
        bool got = true;
        if (lane == 0) got = mbar_wait(&ids_full[slot], ((c - c0) / kIdRing) & 1, abort_flag);
        if (!__shfl_sync(0xffffffffu, got, 0)) break;
        if (lane < ppc) pg = sIds[slot * kMaxPages + lane];
        __syncwarp();
        if (lane == 0) mbar_arrive(&ids_empty[slot]);
      }
      for (int kv = 0; kv < 2; ++kv, ++item) {
        const int buf = item % kNumBuf;
        bool got = true;
        if (lane == 0) {
          got = mbar_wait(&buf_empty[buf], ((item / kNumBuf) & 1) ^ 1u, abort_flag);
          if (got) mbar_expect_tx(&buf_full[buf], kItem);
        }
        if (!__shfl_sync(0xffffffffu, got, 0)) {
          ok = false;
          break;
        }
        __syncwarp();
        uint8_t* dst = sBuf + buf * kItem;
        if (is_ctx) {
          if (lane < ppc) {
            const CUtensorMap* map = kv ? &tmV : &tmK;
            const int row = ((pg * p.B + b) * p.Hkv + kvh) * p.ps;
            for (int h = 0; h < 2; ++h)
              tma_load_2d(dst + h * kHalf + lane * p.ps * 128, map, h * 64, row, &buf_full[buf]);
          }
        } else if (lane == 0) {
          const CUtensorMap* map = kv ? &tmTV : &tmTK;
          const int tc = c - p.n_ctx_chunks;
          for (int h = 0; h < 2; ++h)
            tma_load_3d(dst + h * kHalf, map, h * 64, tc * kChunk, b * p.Hkv + kvh, &buf_full[buf]);
        }
      }
    }
  } else if (n_iter > 0 && warp == 10) {
    // ---------------------------------------------------------------- page-table reader
    const int ppc = kChunk / p.ps;
    const int32_t* table = p.page_table + (int64_t)b * p.table_stride;
    const int c_end = min(c1, p.n_ctx_chunks);
    for (int c = c0; c < c_end; ++c) {
      const int slot = (c - c0) % kIdRing;
      bool got = true;
      if (lane == 0) got = mbar_wait(&ids_empty[slot], (((c - c0) / kIdRing) & 1) ^ 1u, abort_flag);
      if (!__shfl_sync(0xffffffffu, got, 0)) break;
      int pg = -1;  // slot past the context: reload a valid page, its keys are masked
      if (lane < ppc) {
        const int tok = c * kChunk + lane * p.ps;
        if (tok < p.ctx_len) {
          pg = table[tok];
          const int n = min(p.ps, p.ctx_len - tok);
          bool bad = pg < 0 || pg >= p.num_pages;
          if (p.table_vec && n == p.ps) {
            const int4* v = reinterpret_cast<const int4*>(table + tok);
            for (int s = 0; s < p.ps / 4; ++s) {
              const int4 e = __ldg(v + s);
              bad |= (e.x != pg) | (e.y != pg) | (e.z != pg) | (e.w != pg);
            }
          } else {
            for (int s = 1; s < n; ++s) bad |= (table[tok + s] != pg);
          }
          if (bad) {
            record_error(MTP_ERR_DEVICE);
            if (pg < 0 || pg >= p.num_pages) pg = 0;
          }
        }
      }
      const int first = __shfl_sync(0xffffffffu, pg, 0);
      if (lane < ppc) sIds[slot * kMaxPages + lane] = pg < 0 ? first : pg;
      __syncwarp();
      if (lane == 0) mbar_arrive(&ids_full[slot]);
    }
  } else if (n_iter > 0 && warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      bool ok = mbar_wait(q_full, 0, abort_flag);
      auto wait_item = [&](int it) -> bool {
        return mbar_wait(&buf_full[it % kNumBuf], (it / kNumBuf) & 1, abort_flag);
      };
      auto issue_s = [&](int t, int sb, int buf) {
        const uint32_t d = tmem_base + (uint32_t)(t * 256 + sb * 64);
        const uint32_t qa = smem_u32(sQ + t * kQTile), ka = smem_u32(sBuf + buf * kItem);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          umma_f16(d, sw128_kmajor_desc(qa + (k >> 2) * kQHalf + (k & 3) * 32),
                   sw128_kmajor_desc(ka + (k >> 2) * kHalf + (k & 3) * 32), IDESC_S, k > 0);
      };
      auto issue_pv = [&](int t, int sb, int buf, bool acc) {
        const uint32_t d = tmem_base + (uint32_t)(t * 256 + 128);
        const uint32_t pa = tmem_base + (uint32_t)(t * 256 + sb * 64);
        const uint32_t va = smem_u32(sBuf + buf * kItem);
#pragma unroll
        for (int k = 0; k < 4; ++k)  // 16 keys per MMA: 8 TMEM columns of P, 16 rows of V
          umma_f16_ts(d, pa + k * 8, sw128_mnmajor_desc(va + k * 16 * 128, kHalf), IDESC_PV,
                      (acc || k > 0) ? 1u : 0u);
      };
      // scores of the first two chunks into both buffers of every tile
      for (int j = 0; j < 2 && j < n_iter && ok; ++j) {
        if (!(ok = wait_item(2 * j))) break;
        tc_fence_after();
        for (int t = 0; t < p.n_tiles; ++t) {
          issue_s(t, j, (2 * j) % kNumBuf);
          umma_commit(&s_full[2 * t + j]);
        }
        umma_commit(&buf_empty[(2 * j) % kNumBuf]);
      }
      for (int i = 0; i < n_iter && ok; ++i) {
        const int sb = i & 1;
        const int vitem = 2 * i + 1, knext = 2 * i + 4;  // V of chunk i, K of chunk i+2
        for (int t = 0; t < p.n_tiles && ok; ++t) {
          if (!(ok = mbar_wait(&p_full[2 * t + sb], (i >> 1) & 1, abort_flag))) break;
          tc_fence_after();
          if (t == 0) {
            if (!(ok = wait_item(vitem))) break;
            tc_fence_after();
          }
          issue_pv(t, sb, vitem % kNumBuf, i > 0);
          umma_commit(&pv_done[t]);
          if (i == n_iter - 1) umma_commit(&o_done[t]);
          if (t == p.n_tiles - 1) umma_commit(&buf_empty[vitem % kNumBuf]);
          if (i + 2 < n_iter) {
            if (t == 0) {
              if (!(ok = wait_item(knext))) break;
              tc_fence_after();
            }
            issue_s(t, sb, knext % kNumBuf);  // reuses S_t[sb]: PV_t(i) above read it first
            umma_commit(&s_full[2 * t + sb]);
            if (t == p.n_tiles - 1) umma_commit(&buf_empty[knext % kNumBuf]);
          }
        }
      }
      umma_commit(drain);
      mbar_wait(drain, 0, abort_flag, /*honour_abort=*/false);
    }
  } else if (n_iter > 0 && warp >= 2 && warp < 10 && (warp - 2) / 4 < p.n_tiles) {
    // ---------------------------------------------------------------- softmax
    const int t = (warp - 2) / 4;
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const int t_node = t * p.t_per_tile + r / p.G;
    const int g = r % p.G;
    const bool row_ok = t_node < p.T;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const uint32_t o_addr = tmem_base + lane_off + (uint32_t)(t * 256 + 128);
    const float* mrow = p.tree_mask + (int64_t)(row_ok ? t_node : 0) * p.T;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int i = 0; i < n_iter; ++i) {
      const int c = c0 + i;
      const int sb = i & 1;
      const uint32_t s_addr = tmem_base + lane_off + (uint32_t)(t * 256 + sb * 64);
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[2 * t + sb], (i >> 1) & 1, abort_flag))) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t s[64];
      tmem_ld32(s_addr, *reinterpret_cast<uint32_t(*)[32]>(&s[0]));
      tmem_ld32(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&s[32]));
      tmem_wait_ld();
      uint32_t mw[2];  // keep-bits of the 64 keys
      if (c < p.n_ctx_chunks) {
        const int valid = p.ctx_len - c * kChunk;
#pragma unroll
        for (int w = 0; w < 2; ++w) {
          const int v = valid - 32 * w;
          mw[w] = v >= 32 ? 0xffffffffu : (v <= 0 ? 0u : ((1u << v) - 1u));
        }
      } else {
        const int m0 = (c - p.n_ctx_chunks) * kChunk;
#pragma unroll 1
        for (int w = 0; w < 2; ++w) {
          uint32_t bits = 0;
#pragma unroll 8
          for (int k = 0; k < 32; ++k) {
            const int m = m0 + 32 * w + k;
            if (row_ok && m < p.T && __ldg(mrow + m) > 0.5f) bits |= 1u << k;
          }
          mw[w] = bits;
        }
      }
      if ((mw[0] & mw[1]) != 0xffffffffu) {
#pragma unroll
        for (int j = 0; j < 64; ++j)
          if (!((mw[j >> 5] >> (j & 31)) & 1u)) s[j] = 0xff800000u;  // -inf
      }
      // row max on raw scores (positive scale folded into the exponent)
      float m4[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) m4[k] = fmaxf(__uint_as_float(s[k]), __uint_as_float(s[k + 4]));
#pragma unroll
      for (int j = 8; j < 64; j += 8)
#pragma unroll
        for (int k = 0; k < 4; ++k) m4[k] = fmax3(m4[k], __uint_as_float(s[j + k]), __uint_as_float(s[j + 4 + k]));
      const float mx = p.scale_log2 * fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      const float m_new = fmaxf(m_run, mx);
      if (i == 0) {
        m_run = m_new;
      } else {
        const bool need = m_new > m_run + kRescaleThreshold;
        if (__any_sync(0xffffffffu, need)) {
          // O must hold every PV so far before it is rescaled
          if (!__all_sync(0xffffffffu, mbar_wait(&pv_done[t], (i - 1) & 1, abort_flag))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const float alpha = need ? ex2(m_run - m_new) : 1.0f;
#pragma unroll 1
          for (int j = 0; j < 8; ++j) {
            uint32_t o[16];
            tmem_ld16(o_addr + j * 16, o);
            tmem_wait_ld();
#pragma unroll
            for (int k = 0; k < 16; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
            tmem_st16(o_addr + j * 16, o);
          }
          tmem_wait_st();
          if (need) {
            l_run *= alpha;
            m_run = m_new;
          }
        }
      }
      const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
      const float mul = p.scale_log2;
      float ls0 = 0.f, ls1 = 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) {  // packed in place: s[j] is free once s[2j], s[2j+1] are read
        float x0, x1;
        ffma2(x0, x1, __uint_as_float(s[2 * j]), __uint_as_float(s[2 * j + 1]), mul, mul, -m_use, -m_use);
        const float e0 = ex2(x0), e1 = ex2(x1);
        add2(ls0, ls1, e0, e1);
        s[j] = pack_bf16(e0, e1, AB_FMT == 1 ? MTP_DTYPE_BF16 : MTP_DTYPE_F16);
      }
      l_run += ls0 + ls1;
      tmem_st32(s_addr, *reinterpret_cast<uint32_t(*)[32]>(&s[0]));
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[2 * t + sb]);
    }
    // pv_done may be two phases behind here (the softmax waits on it only to
    // rescale), so a parity wait on it could pass early: o_done completes once.
    if (ok && __all_sync(0xffffffffu, mbar_wait(&o_done[t], 0, abort_flag))) {
      tc_fence_after();
      const int row_in_unit = t * 128 + r;
      if (p.splits == 1) {
        const float inv = 1.0f / l_run;
        uint8_t* orow = static_cast<uint8_t*>(p.out) +
                        ((((int64_t)b * p.T + t_node) * p.Hq + (int64_t)kvh * p.G + g) * kD) * 2;
#pragma unroll 1
        for (int j = 0; j < 4; ++j) {
          uint32_t o[32];
          tmem_ld32(o_addr + j * 32, o);
          tmem_wait_ld();
          if (row_ok) {
            uint32_t w[16];
#pragma unroll
            for (int k = 0; k < 16; ++k)
              w[k] = pack_bf16(__uint_as_float(o[2 * k]) * inv, __uint_as_float(o[2 * k + 1]) * inv, p.out_dtype);
            uint4* dst = reinterpret_cast<uint4*>(orow + j * 64);
#pragma unroll
            for (int k = 0; k < 4; ++k) dst[k] = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
          }
        }
      } else {
        const int64_t slot = ((int64_t)unit * p.splits + split) * 256 + row_in_unit;
        float* po = p.part_o + slot * kD;
#pragma unroll 1
        for (int j = 0; j < 4; ++j) {
          uint32_t o[32];
          tmem_ld32(o_addr + j * 32, o);
          tmem_wait_ld();
          float4* dst = reinterpret_cast<float4*>(po + j * 32);
#pragma unroll
          for (int k = 0; k < 8; ++k)
            dst[k] = make_float4(__uint_as_float(o[4 * k]), __uint_as_float(o[4 * k + 1]),
                                 __uint_as_float(o[4 * k + 2]), __uint_as_float(o[4 * k + 3]));
        }
        p.part_ml[slot * 2] = m_run;
        p.part_ml[slot * 2 + 1] = l_run;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace attn2
}  // namespace mtp
