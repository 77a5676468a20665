// mtp_attention_tc.cuh -- paged tree attention with grouped-query heads on
// the sm_100a tensor cores (tcgen05 + TMEM), the composite of the reference's
// fused_paged_attention (page-table gather, mtp_kernels.py:495-554) and
// fused_tree_attention (masked keys, mtp_kernels.py:560-613).
//
// Work unit = one (sequence b, KV head). Its query rows are every tree node t
// times the G = Hq/Hkv query heads that share the KV head: up to 256 rows,
// held as two 128-row tiles (row r = t_local*G + g) for the whole kernel, so
// each K/V byte is read from HBM once per unit and feeds 256 query rows.
//
// 384 threads, one CTA per SM, roles grouped by warpgroup:
//   warps 0-3   softmax for query tile 0, warps 4-7 for tile 1 (warpgroups
//               0 and 1, 184 registers per thread after set-up): one query
//               row per thread; tcgen05.ld of the scores, mask (context
//               length, or the tree ancestor mask), running max in the log2
//               domain with lazy rescaling (O in TMEM is rescaled only when
//               the max grows by more than 2^8), exp2, P packed to bf16
//               pairs and stored back into TMEM with tcgen05.st.
//   warp 8      TMA producer: Q once (4-D map over [B,T,Hq,D]); then per
//               128-key chunk the K and V slabs -- context chunks gather
//               128/page_size pages of the PagedKVCache pool
//               [P,B,Hkv,page_size,D] (each (page,b,h) slab is contiguous),
//               the tree chunk reads [B,Hkv,T,D] -- into a 5-deep ring of
//               32 KB buffers, 128-byte swizzled; one lane per page slab.
//   warp 9      TMEM allocator + tcgen05.mma issuer:
//               S_t = Q_t K^T (M128 N128 K128) and O_t += P_t V
//               (M128 N128 K128, P read from TMEM, V MN-major from shared
//               memory), accumulators in TMEM (S0, S1, O0, O1 = 4 x 128
//               columns; P_t overwrites the first 64 columns of S_t), ordered
//               S0 S1 | PV0 S0' PV1 S1' | ... so one tile's softmax overlaps
//               the other tile's MMAs.
//   warp 10     page-table reader: stages the page ids of up to 16 chunks
//               ahead of the TMA producer (shared-memory ring) and marks
//               chunks whose table is not page-granular, which the producer
//               then gathers token by token (16-byte loads into the ring).
//   warp 11     idle (completes warpgroup 2, 136 registers per thread with
//               warps 8-10).
// Long contexts with few units are split over CTAs (flash-decoding); the
// partial (O, max, sum) triples are merged by attn_merge_kernel.
// Every wait is bounded (mbar_wait).  No clusters; every TMA load fills its own CTA.
#pragma once

#include "mtp_common.cuh"

namespace mtp {
namespace attn {

// Roles grouped by warpgroup so registers can move between them: softmax
// tiles 0 / 1 = warpgroups 0 / 1 (warps 0-3, 4-7), producer 8, MMA 9, page
// table 10, warp 11 idle.  After set-up warpgroup 2 drops to kRegsAux
// registers per thread and warpgroups 0-1 rise to kRegsSoftmax; per SM
// sub-partition (one warp of each warpgroup) 2 * 184 + 136 = 3 * 168, the
// registers the launch reserves (checked on the host before every launch).
// 136 keeps the producer's per-token gather (64 asynchronous copies per
// lane in flight) as fast as with 168; at 120 or fewer it ran 30-45 %
// slower on fully per-token tables, while the softmax gains little above
// 184 (224: 3 % more on page-granular tables).
constexpr int kThreads = 384;
constexpr int kWarpProducer = 8, kWarpMma = 9, kWarpTable = 10, kWarpSoftmax0 = 0;
constexpr int kLaunchRegs = 168, kRegsSoftmax = 184, kRegsAux = 136;
static_assert(2 * kRegsSoftmax + kRegsAux == 3 * kLaunchRegs, "register split must equal the launch's reservation");
constexpr int kD = 128;
constexpr int kChunk = 128;                      // keys per chunk
constexpr int kHalfBytes = 128 * 128;            // 128 rows x 128 bytes (64 bf16 of D)
constexpr int kTileBytes = 2 * kHalfBytes;       // 128 rows x D=128 bf16
constexpr int kNumBuf = 5;                       // K/V ring depth (32 KB each)
constexpr int kIdRing = 16;                      // page-id ring: chunks the table warp may run ahead
constexpr int kMaxPagesPerChunk = 16;            // page_size >= 8
constexpr int kSmemBytes = 2 * kTileBytes /*Q*/ + kNumBuf * kTileBytes /*K,V*/ +
                           kIdRing * kMaxPagesPerChunk * 4 /*page ids*/ + 512 /*barriers*/ + 1024;
constexpr float kRescaleThreshold = 8.0f;        // log2 units: rescale O only when the max grows by > 2^8
// mbarriers: q_full, buf_full/empty [kNumBuf], s_full [2], p_full [4], pv_done [2],
// ids_full/empty [kIdRing], drain; then the TMEM slot and the abort flag
static_assert((1 + 2 * kNumBuf + 2 + 4 + 2 + 2 * kIdRing + 1) * 8 + 8 <= 512, "barrier area");
static_assert(kTileBytes % 1024 == 0 && (kIdRing * kMaxPagesPerChunk * 4) % 8 == 0, "buffer alignment");
static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");

// Optional cycle stamps of CTA 0 (build with -DMTP_ATTN_TRACE): slot
// (kind, tile, iteration) -> clock64.  Compiled out otherwise.  Kinds:
// softmax 0 scores ready, 1 scores loaded, 8 row max done, 2 previous PV
// seen done, 9 first half of P handed over, 3 both halves handed over;
// MMA warp 10 first half of P seen, 4 second half seen, 11 PV committed,
// 5 next S issued; producer 6 K buffer acquired, 7 V buffer acquired.
// The same builds also stamp every CTA's phases (CTA_STAMP slot k of CTA
// blockIdx.x; slot 0 is the entry %globaltimer, the others clock64):
// 1 entry, 2 Q and first K landed (MMA warp), 3 first scores seen, 4 last
// context chunk's P stored, 5 last chunk's P stored, 6 output written, 7 exit
// (softmax tile 0, row 0, for 3-6).
#ifdef MTP_ATTN_TRACE
static __device__ unsigned long long g_attn_trace[12 * 2 * 64];
static __device__ unsigned long long g_attn_cta[1024 * 8];
#define ATTN_TRACE_IF(cond, k, tile, it)                                         \
  do {                                                                           \
    if (blockIdx.x == 0 && (cond) && (it) < 64)                                  \
      g_attn_trace[(((k) * 2 + (tile)) * 64 + (it))] = clock64();                \
  } while (0)
#define CTA_STAMP(cond, k)                                                       \
  do {                                                                           \
    if ((cond) && blockIdx.x < 1024) g_attn_cta[blockIdx.x * 8 + (k)] = clock64(); \
  } while (0)
#else
#define ATTN_TRACE_IF(cond, k, tile, it) \
  do {                                   \
  } while (0)
#define CTA_STAMP(cond, k) \
  do {                     \
  } while (0)
#endif
#define ATTN_TRACE(k, tile, it) ATTN_TRACE_IF(r == 0, k, tile, it)

struct Params {
  const int32_t* page_table;
  int64_t table_stride;
  const uint8_t* k_pool;   // [P, B, Hkv, page_size, D] pools, for the per-token gather
  const uint8_t* v_pool;
  const float* tree_mask;  // [T, T]
  void* out;               // [B, T, Hq, D]
  float* part_o;           // [units, splits, 256, D]   (splits > 1)
  float* part_ml;          // [units, splits, 256, 2]   (max, sum)
  int B, T, Hq, Hkv, G, ps, num_pages, ctx_len;
  int n_ctx_chunks, n_chunks, splits, chunks_per_split, n_tiles, t_per_tile;
  int out_dtype;
  int table_vec;     // page-table rows 16-byte aligned: check pages with int4 loads
  float scale_log2;  // softmax scale * log2(e)
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// (d0, d1) = (a0, a1) * (b0, b1) + (c0, c1) as one packed f32x2 FMA
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0,
                                      float c1) {
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}

// (s0, s1) += (a0, a1) as one packed f32x2 add
__device__ __forceinline__ void add2(float& s0, float& s1, float a0, float a1) {
  asm("{\n\t.reg .b64 ra, rs;\n\t"
      "mov.b64 rs, {%0, %1};\n\tmov.b64 ra, {%2, %3};\n\t"
      "add.rn.f32x2 rs, rs, ra;\n\tmov.b64 {%0, %1}, rs;\n\t}"
      : "+f"(s0), "+f"(s1)
      : "f"(a0), "f"(a1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi, int dtype) {
  if (dtype == MTP_DTYPE_BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// P for keys 64h .. 64h + 63 of a score row: 2^(s*mul - m) packed as 16-bit
// pairs into s[32h .. 32h + 31] (s[j] is free once s[2j], s[2j+1] are read),
// with the running sums in (ls0, ls1).
template <int AB_FMT>
__device__ __forceinline__ void exp_pack_half(uint32_t (&s)[128], int h, float mul, float m_use, float& ls0,
                                              float& ls1) {
#pragma unroll
  for (int j = 32 * h; j < 32 * h + 32; ++j) {
    float x0, x1;
    ffma2(x0, x1, __uint_as_float(s[2 * j]), __uint_as_float(s[2 * j + 1]), mul, mul, -m_use, -m_use);
    const float e0 = ex2(x0), e1 = ex2(x1);
    add2(ls0, ls1, e0, e1);
    s[j] = pack_bf16(e0, e1, AB_FMT == 1 ? MTP_DTYPE_BF16 : MTP_DTYPE_F16);
  }
}

// Per-token gather of a context chunk (tables that are not page-granular).
// rows[i] (lane l) = pool row -- ((page * B + b) * Hkv + h) * page_size + slot,
// 256 bytes of K or V -- of token tok0 + l + 32 i, or -1 past the context or
// for a page id outside [-P, P) (recorded as MTP_ERR_DEVICE, where the
// reference raises); such rows are zero-filled, so masked keys stay finite.
__device__ __forceinline__ void token_rows(const Params& p, int b, int kvh, int tok0, int lane, int (&rows)[4]) {
  const int32_t* table = p.page_table + (int64_t)b * p.table_stride;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int tok = tok0 + lane + 32 * i;
    rows[i] = -1;
    if (tok < p.ctx_len) {
      const int64_t pg = resolve_page(__ldg(table + tok), p.num_pages);
      if (pg >= 0)
        rows[i] = (int)(((pg * p.B + b) * p.Hkv + kvh) * p.ps + tok % p.ps);
      else
        record_error(MTP_ERR_DEVICE);
    }
  }
}

// 16-byte asynchronous copy global -> shared (L2 only); bytes past
// src_bytes (0 or 16) are zero-filled, so src is not read when it is 0.
__device__ __forceinline__ void cp_async16(uint32_t smem_dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_dst), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Starts the fill of one 32 KB K or V buffer (128 keys x D = 128, two 16 KB
// halves of 64 dims, rows 128 bytes, 128-byte swizzle: 16-byte piece j of
// row r sits at piece j ^ (r & 7)) from the pool rows of token_rows: lane l
// copies piece l & 15 of tokens 2k + (l >> 4), all 64 of its copies in
// flight at once; rows of -1 are zero-filled.  The caller waits for them
// (cp_async_wait_all) before handing the buffer to the tensor cores.
__device__ __forceinline__ void fill_tokens(uint8_t* dst, const uint8_t* pool, const int (&rows)[4], int lane) {
  const int j = lane & 15, half = j >> 3, jj = j & 7;
  const uint32_t base = smem_u32(dst) + half * kHalfBytes;
#pragma unroll
  for (int q = 0; q < 4; ++q) {  // tokens 32 q .. 32 q + 31, whose rows lane (i & 31) holds in rows[q]
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const int i = 32 * q + 2 * u + (lane >> 4);
      const int row = __shfl_sync(0xffffffffu, rows[q], i & 31);
      const uint8_t* src = row >= 0 ? pool + (int64_t)row * (kD * 2) + j * 16 : pool;
      cp_async16(base + i * 128 + ((jj ^ (i & 7)) << 4), src, row >= 0 ? 16u : 0u);
    }
  }
}

// Keep-bits of tree keys m0 .. m0 + 31 for the query row of tree node
// t_node (bit k set: tree_mask[t_node, m0 + k] > 0.5); 0 past T or for a
// padding row.
__device__ __forceinline__ uint32_t tree_mask_bits(const Params& p, bool row_ok, int t_node, int m0) {
  uint32_t bits = 0;
  if (row_ok && m0 < p.T) {
    const float* mrow = p.tree_mask + (int64_t)t_node * p.T + m0;
    const int n = min(32, p.T - m0);
#pragma unroll 8
    for (int k = 0; k < 32; ++k)
      if (k < n && __ldg(mrow + k) > 0.5f) bits |= 1u << k;
  }
  return bits;
}

// AB_FMT: 1 = bf16, 0 = f16 (q/k/v dtype)
template <int AB_FMT>
__global__ void __launch_bounds__(kThreads, 1)
    tree_attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                             const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmTK,
                             const __grid_constant__ CUtensorMap tmTV, Params p) {
  constexpr uint32_t IDESC_S = make_idesc(AB_FMT, 128, kChunk);          // Q (K-major) x K (K-major)
  constexpr uint32_t IDESC_PV = make_idesc(AB_FMT, 128, kD, 0u, 1u);    // P (K-major) x V (MN-major)

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                  // 2 tiles x 32 KB
  uint8_t* sBuf = sQ + 2 * kTileBytes;                 // kNumBuf x 32 KB
  int* sIds = reinterpret_cast<int*>(sBuf + kNumBuf * kTileBytes);  // [kIdRing][kMaxPagesPerChunk]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sIds + kIdRing * kMaxPagesPerChunk);
  uint64_t* q_full = bars;
  uint64_t* buf_full = bars + 1;
  uint64_t* buf_empty = buf_full + kNumBuf;
  uint64_t* s_full = buf_empty + kNumBuf;  // [2]
  uint64_t* p_full = s_full + 2;           // [2 tiles][2 halves of 64 keys]
  uint64_t* pv_done = p_full + 4;          // [2]
  uint64_t* ids_full = pv_done + 2;        // [kIdRing]
  uint64_t* ids_empty = ids_full + kIdRing;  // [kIdRing]
  uint64_t* drain = ids_empty + kIdRing;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int unit = blockIdx.x / p.splits, split = blockIdx.x % p.splits;
  const int b = unit / p.Hkv, kvh = unit % p.Hkv;
  const int c0 = split * p.chunks_per_split;
  const int c1 = min(p.n_chunks, c0 + p.chunks_per_split);
  const int n_iter = c1 - c0;
#ifdef MTP_ATTN_TRACE
  if (threadIdx.x == 0 && blockIdx.x < 1024) g_attn_cta[blockIdx.x * 8] = globaltimer_ns();
#endif
  CTA_STAMP(threadIdx.x == 0, 1);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kNumBuf; ++i) {
      mbar_init(&buf_full[i], 1);
      mbar_init(&buf_empty[i], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[2 * t], 4);  // one arrival per softmax warp
      mbar_init(&p_full[2 * t + 1], 4);
      mbar_init(&pv_done[t], 1);
    }
    for (int i = 0; i < kIdRing; ++i) {
      mbar_init(&ids_full[i], 1);
      mbar_init(&ids_empty[i], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kWarpMma) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp >= 8) {  // warpgroup 2: producer, MMA, page table, idle
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsAux));
  if (n_iter > 0 && warp == kWarpProducer) {
    // ---------------------------------------------------------------- TMA producer (whole warp)
    // lane i < pages_per_chunk issues the loads of page slot i of a context
    // chunk; page ids come checked from the table warp through sIds.
    const int ppc = kChunk / p.ps;
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmTK);
      tma_prefetch_desc(&tmTV);
      mbar_expect_tx(q_full, p.n_tiles * kTileBytes);
      for (int t = 0; t < p.n_tiles; ++t)
        for (int h = 0; h < 2; ++h)
          tma_load_4d(sQ + t * kTileBytes + h * kHalfBytes, &tmQ, h * 64, kvh * p.G, t * p.t_per_tile, b, q_full);
    }
    int item = 0;
    bool ok = true;
    for (int c = c0; c < c1 && ok; ++c) {
      const bool is_ctx = c < p.n_ctx_chunks;
      const int slot = (c - c0) % kIdRing;
      int pg = 0;
      bool per_token = false;  // this chunk's table is not page-granular: gather token by token
      int rows[4];             // per-token mode: pool row of token lane + 32 i (-1: zero-fill)
      if (is_ctx) {
        bool got = true;
        if (lane == 0) got = mbar_wait(&ids_full[slot], ((c - c0) / kIdRing) & 1, abort_flag);
        if (!__shfl_sync(0xffffffffu, got, 0)) break;
        if (lane < ppc) pg = sIds[slot * kMaxPagesPerChunk + lane];
        per_token = sIds[slot * kMaxPagesPerChunk] < 0;
        __syncwarp();
        if (lane == 0) mbar_arrive(&ids_empty[slot]);
        if (per_token) token_rows(p, b, kvh, c * kChunk, lane, rows);
      }
      for (int kv = 0; kv < 2; ++kv, ++item) {
        const int buf = item % kNumBuf;
        bool got = true;
        if (lane == 0) {
          got = mbar_wait(&buf_empty[buf], ((item / kNumBuf) & 1) ^ 1u, abort_flag);
          if (got && !per_token) mbar_expect_tx(&buf_full[buf], kTileBytes);
        }
        if (!__shfl_sync(0xffffffffu, got, 0)) {
          ok = false;
          break;
        }
        ATTN_TRACE_IF(lane == 0, 6 + kv, 0, c - c0);
        __syncwarp();
        uint8_t* dst = sBuf + buf * kTileBytes;
        if (per_token) {
          // K's copies stay in flight while V's are issued; then each lane
          // waits for its own, fences them for the tensor cores (async
          // proxy), and both buffers are handed over
          fill_tokens(dst, kv ? p.v_pool : p.k_pool, rows, lane);
          if (kv == 1) {
            cp_async_wait_all();
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              mbar_arrive(&buf_full[(item - 1) % kNumBuf]);
              mbar_arrive(&buf_full[buf]);
            }
          }
        } else if (is_ctx) {
          if (lane < ppc) {
            const CUtensorMap* map = kv ? &tmV : &tmK;
            const int row = ((pg * p.B + b) * p.Hkv + kvh) * p.ps;
            for (int h = 0; h < 2; ++h)
              tma_load_2d(dst + h * kHalfBytes + lane * p.ps * 128, map, h * 64, row, &buf_full[buf]);
          }
        } else if (lane == 0) {
          const CUtensorMap* map = kv ? &tmTV : &tmTK;
          const int tc = c - p.n_ctx_chunks;
          for (int h = 0; h < 2; ++h)
            tma_load_3d(dst + h * kHalfBytes, map, h * 64, tc * kChunk, b * p.Hkv + kvh, &buf_full[buf]);
        }
      }
    }
    cp_async_wait_all();  // after an abort too: none of this warp's copies may still be landing at exit
  } else if (n_iter > 0 && warp == kWarpTable) {
    // ---------------------------------------------------------------- page-table warp
    // Reads the page ids of up to kIdRing context chunks ahead of the TMA
    // producer and decides how each chunk is gathered.  The reference
    // gathers per token (mtp_kernels.py:520-531, eager 839-848): key t of
    // sequence b is slot t % page_size of page table[b, t].  Lane i <
    // pages_per_chunk takes page slot i; when every token of every slot maps
    // to its slot's page (resolved like torch indexing, resolve_page), the
    // chunk is page-granular and the producer loads whole page slabs with
    // TMA.  Otherwise -- tables that PagedKVCache.reserve built with
    // n_tokens not a multiple of page_size, or that swap_logical_pages
    // rearranged (mtp_engine.py:567-593) -- the chunk is marked per-token
    // (page id -1 in slot 0) and the producer gathers it token by token.
    const int ppc = kChunk / p.ps;
    const int32_t* table = p.page_table + (int64_t)b * p.table_stride;
    const int c_end = min(c1, p.n_ctx_chunks);
    for (int c = c0; c < c_end; ++c) {
      const int slot = (c - c0) % kIdRing;
      bool got = true;
      if (lane == 0) got = mbar_wait(&ids_empty[slot], (((c - c0) / kIdRing) & 1) ^ 1u, abort_flag);
      if (!__shfl_sync(0xffffffffu, got, 0)) break;
      int pg = -1;  // slot past the context: reload a valid page, its keys are masked
      bool gran = true;
      if (lane < ppc) {
        const int tok = c * kChunk + lane * p.ps;
        if (tok < p.ctx_len) {
          const int64_t r0 = resolve_page(__ldg(table + tok), p.num_pages);
          const int n = min(p.ps, p.ctx_len - tok);
          gran = r0 >= 0;
          if (p.table_vec && n == p.ps) {
            const int4* v = reinterpret_cast<const int4*>(table + tok);
            for (int s = 0; s < p.ps / 4; ++s) {
              const int4 e = __ldg(v + s);
              gran &= (resolve_page(e.x, p.num_pages) == r0) & (resolve_page(e.y, p.num_pages) == r0) &
                      (resolve_page(e.z, p.num_pages) == r0) & (resolve_page(e.w, p.num_pages) == r0);
            }
          } else {
            for (int s = 1; s < n; ++s) gran &= resolve_page(__ldg(table + tok + s), p.num_pages) == r0;
          }
          pg = (int)r0;
        }
      }
      const bool chunk_gran = __all_sync(0xffffffffu, gran);
      const int first = __shfl_sync(0xffffffffu, pg, 0);  // slot 0 of a context chunk is always in the context
      if (lane < ppc) sIds[slot * kMaxPagesPerChunk + lane] = !chunk_gran ? -1 : (pg < 0 ? first : pg);
      __syncwarp();
      if (lane == 0) mbar_arrive(&ids_full[slot]);
    }
  } else if (n_iter > 0 && warp == kWarpMma) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      bool ok = mbar_wait(q_full, 0, abort_flag);
      auto wait_item = [&](int item) -> bool {
        return mbar_wait(&buf_full[item % kNumBuf], (item / kNumBuf) & 1, abort_flag);
      };
      auto issue_s = [&](int t, int buf) {
        const uint32_t d = tmem_base + (uint32_t)(t * 128);
        const uint32_t qa = smem_u32(sQ + t * kTileBytes), ka = smem_u32(sBuf + buf * kTileBytes);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (k >> 2) * kHalfBytes + (k & 3) * 32;
          umma_f16(d, sw128_kmajor_desc(qa + off), sw128_kmajor_desc(ka + off), IDESC_S, k > 0);
        }
      };
      // O_t += P_t V for keys [64*half, 64*half + 64) of the chunk
      auto issue_pv = [&](int t, int buf, int half, bool acc) {
        const uint32_t d = tmem_base + (uint32_t)(256 + t * 128);
        const uint32_t pa = tmem_base + (uint32_t)(t * 128);  // P (bf16 pairs) over S_t's first 64 columns
        const uint32_t va = smem_u32(sBuf + buf * kTileBytes);
#pragma unroll
        for (int k = 4 * half; k < 4 * half + 4; ++k)  // 16 keys per MMA: 8 TMEM columns of P, 16 rows of V
          umma_f16_ts(d, pa + k * 8, sw128_mnmajor_desc(va + k * 16 * 128, kHalfBytes), IDESC_PV,
                      (acc || k > 0) ? 1u : 0u);
      };
      if (ok && (ok = wait_item(0))) {
        CTA_STAMP(true, 2);
        tc_fence_after();
        for (int t = 0; t < p.n_tiles; ++t) {
          issue_s(t, 0);
          umma_commit(&s_full[t]);
        }
        umma_commit(&buf_empty[0]);
      }
      for (int i = 0; i < n_iter && ok; ++i) {
        const int kitem = 2 * i, vitem = 2 * i + 1, knext = 2 * i + 2;
        for (int t = 0; t < p.n_tiles && ok; ++t) {
          if (!(ok = mbar_wait(&p_full[2 * t], i & 1, abort_flag))) break;
          tc_fence_after();
          if (t == 0) {
            if (!(ok = wait_item(vitem))) break;
            tc_fence_after();
          }
          ATTN_TRACE_IF(true, 10, t, i);
          issue_pv(t, vitem % kNumBuf, 0, i > 0);  // first 64 keys while the softmax finishes the rest
          if (!(ok = mbar_wait(&p_full[2 * t + 1], i & 1, abort_flag))) break;
          tc_fence_after();
          ATTN_TRACE_IF(true, 4, t, i);
          issue_pv(t, vitem % kNumBuf, 1, true);
          umma_commit(&pv_done[t]);
          ATTN_TRACE_IF(true, 11, t, i);
          if (t == p.n_tiles - 1) umma_commit(&buf_empty[vitem % kNumBuf]);
          if (i + 1 < n_iter) {
            if (t == 0) {
              if (!(ok = wait_item(knext))) break;
              tc_fence_after();
            }
            issue_s(t, knext % kNumBuf);
            umma_commit(&s_full[t]);
            ATTN_TRACE_IF(true, 5, t, i);
            if (t == p.n_tiles - 1) umma_commit(&buf_empty[knext % kNumBuf]);
          }
        }
        (void)kitem;
      }
      umma_commit(drain);
      mbar_wait(drain, 0, abort_flag, /*honour_abort=*/false);
    }
  }
  } else {  // warpgroups 0-1: softmax of query tiles 0 and 1
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
  if (n_iter > 0 && (warp - kWarpSoftmax0) / 4 < p.n_tiles) {
    // ---------------------------------------------------------------- softmax
    const int t = (warp - kWarpSoftmax0) / 4;
    const int q = warp & 3;
    const int r = q * 32 + lane;  // row within the tile == TMEM lane
    const int t_node = t * p.t_per_tile + r / p.G;
    const int g = r % p.G;
    const bool row_ok = t_node < p.T;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const uint32_t s_addr = tmem_base + lane_off + (uint32_t)(t * 128);
    const uint32_t o_addr = tmem_base + lane_off + (uint32_t)(256 + t * 128);
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    // Keep-bits of this row over the first 128 tree keys, read from the
    // float mask before the first scores arrive: the loads overlap the
    // pipeline fill, and the tree chunk's softmax makes no global loads
    // (a second tree chunk, T > 128, reads its bits when it comes).
    uint32_t tbits[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) tbits[w] = tree_mask_bits(p, row_ok, t_node, 32 * w);
    for (int i = 0; i < n_iter; ++i) {
      const int c = c0 + i;
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[t], i & 1, abort_flag))) {
        ok = false;
        break;
      }
      tc_fence_after();
      ATTN_TRACE(0, t, i);
      CTA_STAMP(t == 0 && r == 0 && i == 0, 3);
      // keep-bits of the 128 keys of this chunk (bit k of word w: key 32w + k)
      uint32_t mw[4];
      if (c < p.n_ctx_chunks) {
        const int valid = p.ctx_len - c * kChunk;  // keys [0, valid) are context tokens
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const int v = valid - 32 * w;
          mw[w] = v >= 32 ? 0xffffffffu : (v <= 0 ? 0u : ((1u << v) - 1u));
        }
      } else {
        const int m0 = (c - p.n_ctx_chunks) * kChunk;
        if (m0 == 0) {
#pragma unroll
          for (int w = 0; w < 4; ++w) mw[w] = tbits[w];
        } else {
#pragma unroll 1
          for (int w = 0; w < 4; ++w) mw[w] = tree_mask_bits(p, row_ok, t_node, m0 + 32 * w);
        }
      }
      const bool no_masked = (mw[0] & mw[1] & mw[2] & mw[3]) == 0xffffffffu;
      // the whole 128-column score row in one TMEM round trip
      uint32_t s[128];
#pragma unroll
      for (int j = 0; j < 4; ++j) tmem_ld32(s_addr + j * 32, *reinterpret_cast<uint32_t(*)[32]>(&s[32 * j]));
      tmem_wait_ld();
      ATTN_TRACE(1, t, i);
      // Row max on the raw scores: the scale is positive (checked on the
      // host), so max(s)*scale == max(s*scale) and the scale is folded into
      // the exponent below.  Masked keys become -inf.  Eight independent
      // partial maxima keep the dependency chains short.
      if (!no_masked) {
#pragma unroll
        for (int j = 0; j < 128; ++j)
          if (!((mw[j >> 5] >> (j & 31)) & 1u)) s[j] = 0xff800000u;  // -inf
      }
      float m8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) m8[k] = fmaxf(__uint_as_float(s[k]), __uint_as_float(s[k + 8]));
#pragma unroll
      for (int j = 16; j < 128; j += 16)  // 3-input max: 8 chains, two new scores per step
#pragma unroll
        for (int k = 0; k < 8; ++k) m8[k] = fmax3(m8[k], __uint_as_float(s[j + k]), __uint_as_float(s[j + 8 + k]));
      const float mx = p.scale_log2 * fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]),
                                            fmaxf(m8[6], m8[7]));
      const float mul = p.scale_log2;
      const float m_new = fmaxf(m_run, mx);
      ATTN_TRACE(8, t, i);
      if (i > 0) {
        // P and O may be touched only after the previous PV completed
        if (!__all_sync(0xffffffffu, mbar_wait(&pv_done[t], (i - 1) & 1, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        ATTN_TRACE(2, t, i);
        const bool need = m_new > m_run + kRescaleThreshold;
        if (__any_sync(0xffffffffu, need)) {
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
      } else {
        m_run = m_new;
      }
      const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
      // P = 2^(s*scale - m) as bf16 pairs, packed in place (s[j] is free once
      // s[2j], s[2j+1] are read), written over S_t's first 64 columns in two
      // halves so the MMA warp starts the first half of PV early.
      float ls0 = 0.f, ls1 = 0.f;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        exp_pack_half<AB_FMT>(s, h, mul, m_use, ls0, ls1);
        tmem_st32(s_addr + 32 * h, *reinterpret_cast<uint32_t(*)[32]>(&s[32 * h]));
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[2 * t + h]);
        ATTN_TRACE_IF(r == 0 && h == 0, 9, t, i);
      }
      l_run += ls0 + ls1;
      ATTN_TRACE(3, t, i);
      CTA_STAMP(t == 0 && r == 0 && c == p.n_ctx_chunks - 1, 4);
      CTA_STAMP(t == 0 && r == 0 && i == n_iter - 1, 5);
    }
    if (ok && __all_sync(0xffffffffu, mbar_wait(&pv_done[t], (n_iter - 1) & 1, abort_flag))) {
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
      CTA_STAMP(t == 0 && r == 0, 6);
    }
  }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
  CTA_STAMP(threadIdx.x == 0, 7);
}

// Merge split partials: out = sum_s w_s O_s / sum_s w_s l_s, w_s = 2^(m_s - max m).
// One warp per (unit, query row); each lane owns 4 of the 128 head dims.
__global__ void __launch_bounds__(256) attn_merge_kernel(Params p) {
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t units = (int64_t)p.B * p.Hkv;
  const int rows = p.n_tiles * 128;
  if (wid >= units * rows) return;
  const int unit = (int)(wid / rows), row = (int)(wid % rows);
  const int t = row / 128, r = row % 128;
  const int t_node = t * p.t_per_tile + r / p.G, g = r % p.G;
  if (t_node >= p.T) return;
  const int b = unit / p.Hkv, kvh = unit % p.Hkv;
  float M = -INFINITY;
  for (int s = 0; s < p.splits; ++s) M = fmaxf(M, p.part_ml[(((int64_t)unit * p.splits + s) * 256 + row) * 2]);
  float acc[4] = {0.f, 0.f, 0.f, 0.f}, L = 0.f;
  for (int s = 0; s < p.splits; ++s) {
    const int64_t slot = ((int64_t)unit * p.splits + s) * 256 + row;
    const float ms = p.part_ml[slot * 2];
    const float w = (ms == -INFINITY) ? 0.f : ex2(ms - M);
    L += w * p.part_ml[slot * 2 + 1];
    const float4 v = reinterpret_cast<const float4*>(p.part_o + slot * kD)[lane];
    acc[0] += w * v.x;
    acc[1] += w * v.y;
    acc[2] += w * v.z;
    acc[3] += w * v.w;
  }
  const float inv = 1.0f / L;
  uint8_t* orow = static_cast<uint8_t*>(p.out) + ((((int64_t)b * p.T + t_node) * p.Hq + (int64_t)kvh * p.G + g) * kD) * 2;
  uint2 w2 = make_uint2(pack_bf16(acc[0] * inv, acc[1] * inv, p.out_dtype), pack_bf16(acc[2] * inv, acc[3] * inv, p.out_dtype));
  reinterpret_cast<uint2*>(orow)[lane] = w2;
}

}  // namespace attn
}  // namespace mtp
