// mtp_gemm_sk.cuh -- stream-K schedule for the tcgen05 GEMM of
// mtp_gemm_tc.cuh (same roles, same operand staging, same epilogues).
//
// A persistent data-parallel launch gives each CTA whole 128 x BN tiles; when
// the tile count is not a multiple of the SM count the last round runs part
// empty (1503 verify tiles on 148 SMs: 10.16 rounds of work in 11).  Here
// every CTA first takes `dp_rounds` whole tiles as before, then an equal
// share `q` of the remaining tiles' K blocks, counted over (tile, K block)
// in tile order -- so a tile can be cut between consecutive CTAs.
//
// A CTA that computed only part of a tile stores its fp32 partial
// accumulator into its own slot of the workspace, then takes a ticket on the
// tile's counter; the part that arrives last sums all parts in K order
// (part 0 + part 1 + ...; its own part straight from TMEM), so the sum does not
// depend on which CTA finishes first, and runs the ordinary epilogue on the
// sums.  No CTA ever waits for another.
//
// Workspace: counters [num_tiles - dp_tiles] int64 at rest = INT64_MIN (each
// ticket adds 1; the last part puts the counter back), and 2 slots per CTA
// (head part, tail part) of 128 x BN floats, laid out per slot as
// [BN/4 column quads][128 rows] float4 so a warp's stores are contiguous.
// With clean_slots the last part also writes the rest pattern (INT64_MIN
// words) over every slot it summed, so a verify workspace -- whose keys must
// be at rest whenever a call starts, wherever they fall -- is all at rest
// again after the call.
#pragma once

#include "mtp_gemm_tc.cuh"

namespace mtp {
namespace sk {

struct Sched {
  int num_m;           // 128-row tiles along M (tiles are numbered M-fastest)
  int num_tiles;
  int num_kb;          // 128-byte K blocks per tile
  int dp_rounds;       // whole tiles per CTA before the stream-K phase
  int dp_tiles;        // dp_rounds * grid
  int q;               // K blocks per CTA in the stream-K phase (>= 1)
  long long sk_total;  // (num_tiles - dp_tiles) * num_kb
};

struct Work {
  int tile;       // tile index (M-fastest)
  int kb0, kb1;   // this item's K blocks [kb0, kb1)
  int split;      // another CTA computes the rest of this tile
  int x;          // stream-K tile index, tile - dp_tiles (split items)
  int part;       // this CTA's part of the tile, counted in K order
  int parts;      // number of parts of the tile
  int slot;       // slot of this part: 2 * cta + (0 first item | 1 later item)
};

// Slot and owner of part p of stream-K tile x: part p is computed by CTA
// first + p, which holds it in slot 0 when its range starts inside the tile
// (it is that CTA's first item) and in slot 1 otherwise (its last item).
__host__ __device__ inline int part_slot(const Sched& s, int x, int p) {
  const long long lx = (long long)x * s.num_kb;
  const int cta = (int)(lx / s.q) + p;
  return 2 * cta + (((long long)cta * s.q >= lx) ? 0 : 1);
}

__host__ __device__ inline int tile_parts(const Sched& s, int x) {
  const long long lx = (long long)x * s.num_kb;
  return (int)((lx + s.num_kb - 1) / s.q - lx / s.q) + 1;
}

// The work items of CTA c of a grid of `grid` CTAs, in order.  Host and
// device run the same code (the host to size and check schedules).
struct Iter {
  int c, grid, j;
  long long lin, end;
  __host__ __device__ void init(const Sched& s, int c_, int grid_) {
    c = c_;
    grid = grid_;
    j = 0;
    lin = (long long)c * s.q;
    end = lin + s.q < s.sk_total ? lin + s.q : s.sk_total;
  }
  __host__ __device__ bool next(const Sched& s, Work& w) {
    // whole tiles (a data-parallel-only plan may leave the last round ragged)
    if (j < s.dp_rounds && c + j * grid < s.num_tiles) {
      w.tile = c + j * grid;
      w.kb0 = 0;
      w.kb1 = s.num_kb;
      w.split = 0;
      w.x = w.part = w.slot = 0;
      w.parts = 1;
      ++j;
      return true;
    }
    j = s.dp_rounds;
    if (lin >= end) return false;
    const long long x = lin / s.num_kb;
    const long long tile_end = (x + 1) * s.num_kb;
    const long long e = end < tile_end ? end : tile_end;
    w.tile = s.dp_tiles + (int)x;
    w.kb0 = (int)(lin - x * s.num_kb);
    w.kb1 = w.kb0 + (int)(e - lin);
    w.split = (w.kb0 > 0 || w.kb1 < s.num_kb) ? 1 : 0;
    w.x = (int)x;
    w.parts = w.split ? tile_parts(s, (int)x) : 1;
    w.part = w.split ? c - (int)(x * s.num_kb / s.q) : 0;
    w.slot = 2 * c + (lin == (long long)c * s.q ? 0 : 1);
    lin = e;
    return true;
  }
};

using tc::Cfg;
using tc::epi_bar_sync;
using tc::kBM;
using tc::kKBlockBytes;
using tc::kThreads;

constexpr unsigned long long kCounterRest = 0x8000000000000000ull;

// Named barrier 1 over the four epilogue warps with an AND of `v`: the warps
// leave the work loop together, so the barriers of the split path below are
// always reached by all 128 threads.
__device__ __forceinline__ bool epi_bar_and(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.and.pred p, 1, 128, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v)
      : "memory");
  return r != 0;
}

template <int BN, bool FP8, int AB_FMT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_sk_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N,
                   Sched sched, unsigned long long* counters, float* slots, int clean_slots, GemmEpilogue ep) {
  using C = Cfg<BN>;
  constexpr int KB_ELEMS = FP8 ? 128 : 64;
  constexpr int UMMA_K_BYTES = 32;
  constexpr int K_STEPS = kKBlockBytes / UMMA_K_BYTES;
  constexpr uint32_t IDESC = make_idesc(FP8 ? 0u : (uint32_t)AB_FMT, kBM, BN);
  constexpr int SLOT_F4 = kBM * BN / 4;  // float4 per slot

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + C::STAGES;
  uint64_t* tfull = bars + 2 * C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);
  volatile int* part_last = reinterpret_cast<volatile int*>(tmem_slot + 3);
  volatile int* peers_ok = reinterpret_cast<volatile int*>(tmem_slot + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    *last_flag = 0;
    *part_last = 0;
    *peers_ok = 1;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  Iter it;
  it.init(sched, blockIdx.x, gridDim.x);
  Work w;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      while (ok && it.next(sched, w)) {
        const int mb = w.tile % sched.num_m, nb = w.tile / sched.num_m;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[stage], C::STAGE_BYTES);
          tma_load_2d(sA + stage * C::A_BYTES, &tmA, kb * KB_ELEMS, mb * kBM, &full[stage]);
          tma_load_2d(sB + stage * C::B_BYTES, &tmB, kb * KB_ELEMS, nb * BN, &full[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int local = 0;
      while (ok && it.next(sched, w)) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < K_STEPS; ++k) {
            const uint64_t ad = sw128_kmajor_desc(a_addr + k * UMMA_K_BYTES);
            const uint64_t bd = sw128_kmajor_desc(b_addr + k * UMMA_K_BYTES);
            const uint32_t accumulate = (kb > w.kb0 || k != 0) ? 1u : 0u;
            if constexpr (FP8) umma_f8(d_tmem, ad, bd, IDESC, accumulate);
            else umma_f16(d_tmem, ad, bd, IDESC, accumulate);
          }
          umma_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        ++local;
      }
      umma_commit(drain);
      mbar_wait(drain, 0, abort_flag, /*honour_abort=*/false);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int row_in_tile = q * 32 + lane;
    // fused exchange: this call's epoch and key parity (the previous call's
    // last CTA wrote the epoch before this launch began)
    unsigned long long* my_buf = ep.peers ? reinterpret_cast<unsigned long long*>(ep.peers[ep.rank]) : nullptr;
    const unsigned long long epoch =
        ep.peers ? __ldcg(reinterpret_cast<const unsigned long long*>(
                       reinterpret_cast<const uint8_t*>(my_buf) + peer_epoch_offset(ep.peer_rows, ep.world))) + 1ull
                 : 0ull;
    const int par = (int)(epoch & 1ull);
    int local = 0;
    while (it.next(sched, w)) {
      const int mb = w.tile % sched.num_m, nb = w.tile / sched.num_m;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      ++local;
      const bool got = mbar_wait(&tfull[acc], acc_phase, abort_flag);
      if (!epi_bar_and(got)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + (uint32_t)(acc * BN) + ((uint32_t)(q * 32) << 16);

      bool sum_parts = false;
      if (w.split) {
        // 1. this part -> its slot (every row: rows past M hold zeros)
        float4* mine = reinterpret_cast<float4*>(slots) + (size_t)w.slot * SLOT_F4 + row_in_tile;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tbase + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            __stcg(mine + (c * 8 + j) * kBM, make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                                          __uint_as_float(r[4 * j + 2]),
                                                          __uint_as_float(r[4 * j + 3])));
        }
        // 2. ticket on the tile's counter; the last part to arrive sums them
        __threadfence();
        epi_bar_sync();
        if (threadIdx.x == 64) {
          const unsigned long long old = atomicAdd(&counters[w.x], 1ull);
          const bool last = (old - kCounterRest) == (unsigned long long)(w.parts - 1);
          if (last) counters[w.x] = kCounterRest;  // every part has arrived: back at rest
          *part_last = last ? 1 : 0;
        }
        epi_bar_sync();
        if (!*part_last) {
          tc_fence_before();
          mbar_arrive(&tempty[acc]);
          continue;
        }
        __threadfence();
        sum_parts = true;
      }

      // accumulator values of 32 columns: this CTA's TMEM, or the K-ordered
      // sum of every part's slot with this part taken from TMEM
      auto chunk_values = [&](int c, float (&v)[32]) {
        uint32_t r[32];
        tmem_ld32(tbase + c * 32, r);
        tmem_wait_ld();
        if (!sum_parts) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          return;
        }
        for (int p = 0; p < w.parts; ++p) {
          float t[32];
          if (p == w.part) {
#pragma unroll
            for (int j = 0; j < 32; ++j) t[j] = __uint_as_float(r[j]);
          } else {
            const float4* src = reinterpret_cast<const float4*>(slots) +
                                (size_t)part_slot(sched, w.x, p) * SLOT_F4 + row_in_tile;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 f = __ldcg(src + (c * 8 + j) * kBM);
              t[4 * j] = f.x;
              t[4 * j + 1] = f.y;
              t[4 * j + 2] = f.z;
              t[4 * j + 3] = f.w;
            }
          }
          if (p == 0) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = t[j];
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] += t[j];
          }
        }
      };

      const int row = mb * kBM + row_in_tile;
      const bool row_ok = row < M;
      if (ep.mode == EPI_STORE) {
        const float rs = (ep.row_scale && row_ok) ? ep.row_scale[row] : 1.0f;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          chunk_values(c, v);  // every warp loads: tcgen05.ld is warp-wide
          const int n0 = nb * BN + c * 32;
          if (row_ok && n0 < N) tc::epi_store32(ep, v, row, n0, N, rs);
        }
      } else {
        int32_t best = INT32_MIN;
        int best_n = nb * BN;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          chunk_values(c, v);
          tc::epi_argmax32(ep, v, nb * BN + c * 32, N, best, best_n);
        }
        if (row_ok) {
          const long long key = make_key(best, (uint32_t)(ep.col_offset + best_n));
          if (ep.peers) {
            // the all-reduce(max) of the keys, tile by tile, over NVLink
            for (int p = 0; p < ep.world; ++p) {
              long long* kp = reinterpret_cast<long long*>(ep.peers[p]) + (int64_t)par * ep.peer_rows + row;
              if (p == ep.rank) atomicMax(kp, key);
              else atomicMax_system(kp, key);
            }
          } else {
            atomicMax(&ep.keys[row], key);
          }
        }
      }
      if (sum_parts && clean_slots) {
        const float rest = __uint_as_float(0u), rest_hi = __uint_as_float(0x80000000u);  // INT64_MIN words
        for (int p = 0; p < w.parts; ++p) {
          float4* dst = reinterpret_cast<float4*>(slots) + (size_t)part_slot(sched, w.x, p) * SLOT_F4 + row_in_tile;
#pragma unroll 4
          for (int i = 0; i < BN / 4; ++i) __stcg(dst + i * kBM, make_float4(rest, rest_hi, rest, rest_hi));
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
    if (ep.mode == EPI_ARGMAX && ep.finalize != FIN_NONE) {
      // last CTA to finish decodes the keys (threadFenceReduction pattern);
      // keys sent to peers must be visible system-wide before the ticket
      if (ep.peers) __threadfence_system();
      else __threadfence();
      epi_bar_sync();
      if (threadIdx.x == 64) {
        const unsigned int ticket = atomicAdd(ep.counter, 1u);
        *last_flag = (ticket == gridDim.x - 1) ? 1 : 0;
      }
      epi_bar_sync();
      if (*last_flag && !*abort_flag) {
        if (ep.finalize == FIN_CHAIN_PEERS) {
          // every CTA of this rank has sent its keys: tell every rank, wait
          // (bounded) until every rank has told this one, then decode the
          // global keys of this parity (verify_finalize puts them back to rest)
          __threadfence_system();
          if (threadIdx.x == 64)
            for (int p = 0; p < ep.world; ++p)
              st_release_sys_u64(reinterpret_cast<unsigned long long*>(reinterpret_cast<uint8_t*>(ep.peers[p]) +
                                                                        peer_flags_offset(ep.peer_rows)) +
                                     (int64_t)par * ep.world + ep.rank,
                                 epoch);
          const int tq = threadIdx.x - 64;
          if (tq < ep.world) {
            const unsigned long long* f =
                reinterpret_cast<const unsigned long long*>(reinterpret_cast<const uint8_t*>(my_buf) +
                                                            peer_flags_offset(ep.peer_rows)) +
                (int64_t)par * ep.world + tq;
            const uint64_t t0 = globaltimer_ns();
            while (ld_acquire_sys_u64(f) < epoch) {
              if (globaltimer_ns() - t0 > kWaitLimitNs) {
                record_error(MTP_ERR_TIMEOUT);
                *peers_ok = 0;
                break;
              }
            }
          }
          epi_bar_sync();
          GemmEpilogue f = ep;
          f.keys = reinterpret_cast<long long*>(my_buf) + (int64_t)par * ep.peer_rows;
          f.finalize = FIN_CHAIN;
          if (*peers_ok) {
            verify_finalize(f, tq, 128);
          } else {
            for (int64_t r = tq; r < ep.peer_rows; r += 128) f.keys[r] = KEY_EMPTY;
          }
          epi_bar_sync();
          if (threadIdx.x == 64) {
            *reinterpret_cast<unsigned long long*>(reinterpret_cast<uint8_t*>(my_buf) +
                                                   peer_epoch_offset(ep.peer_rows, ep.world)) = epoch;
            *ep.counter = 0u;
          }
        } else {
          __threadfence();
          verify_finalize(ep, threadIdx.x - 64, 128);
          if (threadIdx.x == 64) *ep.counter = 0u;
        }
      } else if (*last_flag) {
        // this CTA gave up on a wait: put this rank's keys and ticket back at
        // rest (the exchange buffers of a peer call are rebuilt on every rank)
        __threadfence();
        if (ep.finalize != FIN_CHAIN_PEERS) verify_keys_rest(ep, threadIdx.x - 64, 128);
        if (threadIdx.x == 64) *ep.counter = 0u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace sk
}  // namespace mtp
