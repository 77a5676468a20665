// mtp_gemm_vt.cuh -- vocabulary-tiled, CTA-pair tcgen05 GEMM for the verify argmax.
//
// The verify multiplies a few hundred candidate rows (hidden states, B*S of
// them) by the whole lm_head [V, K] and keeps, per candidate, only the
// argmax over the vocabulary (fused_multi_verify_kernel,
// mtp_fused_verify.py:89-156; _eager_fused_multi_verify 184-195).  Here the
// weight is the MMA's A operand: a cluster of two CTAs on neighbouring SMs
// computes a 256-row vocabulary tile with tcgen05.mma.cta_group::2 (M = 256,
// 128 TMEM lanes per CTA) against every candidate (up to 4 groups of 128
// TMEM columns), so each weight byte is read from HBM by exactly one CTA and
// the candidates (a few MB) stream from L2.
//
// What bounds a tcgen05 GEMM here is the tensor cores' operand reads from
// shared memory (about 128 bytes per SM per cycle): an M = 128 x N = 256
// MMA reads 16 + 32 bytes of A and B per 128 MAC-cycles (96 B/clk, a 75 %
// ceiling, which the one-CTA kernels reach).  In a pair MMA each SM reads its
// own A rows and only its half of B, so M = 256 x N = 256 needs 64 B/clk.
// Two adjacent 128-column TMEM groups are therefore written by one N = 256
// MMA whenever the tile has them: its B is candidate group ga from the
// leader's shared memory and ga + 1 from the peer's; a group left over is an
// N = 128 MMA whose B is rows 0-63 of the group from the leader and 64-127
// from the peer.
//
// The leader CTA (rank 0) issues the MMAs; both CTAs' TMA loads complete on
// the leader's barriers; the MMA commits arrive on both CTAs' barriers
// (commit multicast).  No TMA load uses cluster multicast and every load
// reads global memory into its own CTA, so the kernel is safe in multi-GPU
// jobs.
//
// Block of 352 threads, one CTA per SM, persistent over vocabulary tiles:
//   warp 0      TMA producer of the weight ring (WST stages of 16 KB);
//   warp 1      TMEM allocator (all 512 columns) + MMA issuer (leader only);
//   warp 2      TMA producer of the candidate ring (XST stages of G x 8 KB);
//   warps 3-10  epilogue, two teams of four warps (one per TMEM lane
//               quadrant).  Team e drains the groups whose sequence number
//               is e mod 2: it copies a group's 128 x 128 accumulators to
//               registers, frees the group at once, then takes the column
//               maximum over its 128 vocabulary rows (warp max + ballot for
//               the lowest row among ties) into a per-CTA key array in
//               shared memory.  Each CTA adds its keys to the global ones
//               once, at the end; the last CTA decodes them (verify_finalize).
// TMEM is a ring of 4 groups of 128 columns; a tile takes the next G of
// them, so the next tile starts as soon as the previous tile's first groups
// are drained, while the rest of its epilogue runs beside the mainloop.
#pragma once

#include "mtp_gemm_tc.cuh"
#include "mtp_pair.cuh"

namespace mtp {
namespace vt {

using namespace pair;

constexpr int kRows = 128;                       // vocabulary rows per CTA = TMEM lanes
constexpr int kTileRows = 2 * kRows;             // vocabulary rows per pair tile
constexpr int kGroupCols = 128;                  // candidates per group = TMEM columns
constexpr int kGroups = 4;                       // TMEM ring: 4 x 128 = 512 columns
constexpr int kThreads = 352;                    // 11 warps
constexpr int kEpiThreads = 256;                 // warps 3-10
constexpr int kWBytes = kRows * 128;             // weight block: 128 rows x 128 bytes of K
constexpr int kHalfRows = kGroupCols / 2;        // candidate rows per TMA box
constexpr int kHalfBytes = kHalfRows * 128;      // 8 KB
constexpr int kMaxCands = kGroups * kGroupCols;  // 512

template <int G, int WST, int XST>
struct Cfg {
  static constexpr int X_BYTES = G * kHalfBytes;  // this CTA's share of every group
  static constexpr int KEYS_BYTES = G * kGroupCols * 8;
  static constexpr int BAR_BYTES = 512;
  static constexpr int SMEM_BYTES = WST * kWBytes + XST * X_BYTES + KEYS_BYTES + BAR_BYTES + 1024;
  static_assert(G >= 1 && G <= kGroups, "candidate groups");
  static_assert(WST >= 2 && XST >= 2, "double-buffered rings at least");
  // wfull/wempty, xfull/xempty, gfull/gempty, drain; then the TMEM slot and two flags
  static_assert((2 * WST + 2 * XST + 2 * kGroups + 1) * 8 + 3 * 4 <= BAR_BYTES, "barrier area");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory per CTA");
};

// The MMAs of one K step of a tile whose first group has sequence number
// seq: up to two, each either a pair of candidate groups (N = 256, group g
// and g + 1 in adjacent TMEM groups) or a single group (N = 128).  They are
// also the order of the parts of a candidate stage in shared memory (16 KB
// for a pair, 8 KB for a single).
struct Plan {
  int n;
  int group[2];
  bool pair[2];
};
__host__ __device__ __forceinline__ Plan tile_plan(int G, int seq) {
  Plan p{};
  if (G == 1) {
    p.n = 1; p.group[0] = 0; p.pair[0] = false;
  } else if (G == 2) {  // seq is even: TMEM groups (0,1) or (2,3)
    p.n = 1; p.group[0] = 0; p.pair[0] = true;
  } else if (G == 3) {  // the tile's TMEM groups seq..seq+2 (mod 4) wrap at most once
    p.n = 2;
    if ((seq & 3) == 3) {  // groups 3,0,1: single 3, pair (0,1)
      p.group[0] = 0; p.pair[0] = false; p.group[1] = 1; p.pair[1] = true;
    } else {               // pair (s, s+1), single s+2
      p.group[0] = 0; p.pair[0] = true; p.group[1] = 2; p.pair[1] = false;
    }
  } else {  // G == 4, seq a multiple of 4: pairs (0,1), (2,3)
    p.n = 2; p.group[0] = 0; p.pair[0] = true; p.group[1] = 2; p.pair[1] = true;
  }
  return p;
}

__device__ __forceinline__ void epi_bar_sync() { asm volatile("bar.sync 2, 256;" ::: "memory"); }

// ab_fmt: 0 = f16, 1 = bf16 (kind::f16).  tmW: weight [N, K], boxes of 128
// rows; tmX: candidates [M, K], M <= G * 128, boxes of 64 rows; both
// K-major, 128 bytes of K per box, 128-byte swizzle (rows past the end read
// as zeros).  Launched in clusters of 2 CTAs along x.
template <int G, int WST, int XST, int AB_FMT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_vt_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, int M,
                   int N, int num_kb, GemmEpilogue ep) {
  using C = Cfg<G, WST, XST>;
  constexpr int K_STEPS = 4;  // 128 bytes of K per block, 16 elements (32 bytes) per MMA
  constexpr uint32_t IDESC_PAIR = make_idesc((uint32_t)AB_FMT, kTileRows, 2 * kGroupCols);
  constexpr uint32_t IDESC_ONE = make_idesc((uint32_t)AB_FMT, kTileRows, kGroupCols);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem;
  uint8_t* sX = smem + WST * kWBytes;
  long long* skeys = reinterpret_cast<long long*>(sX + XST * C::X_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(skeys) + C::KEYS_BYTES);
  uint64_t* wfull = bars;
  uint64_t* wempty = wfull + WST;
  uint64_t* xfull = wempty + WST;
  uint64_t* xempty = xfull + XST;
  uint64_t* gfull = xempty + XST;
  uint64_t* gempty = gfull + kGroups;
  uint64_t* drain = gempty + kGroups;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int unit = (int)(blockIdx.x >> 1);  // cluster index
  const int units = (int)(gridDim.x >> 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < WST; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], 1);
    }
    for (int s = 0; s < XST; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 1);
    }
    for (int g = 0; g < kGroups; ++g) {
      mbar_init(&gfull[g], 1);
      mbar_init(&gempty[g], 8);  // lane 0 of each of the owning team's four warps, in both CTAs
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    *last_flag = 0;
    fence_barrier_init();
  }
  for (int i = threadIdx.x; i < G * kGroupCols; i += kThreads) skeys[i] = KEY_EMPTY;
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 1) {
    tmem_alloc2(tmem_slot, 512);
    tmem_relinquish2();
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers exist before either CTA's loads or commits reach them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_tiles = (N + kTileRows - 1) / kTileRows;

  if (warp == 0 || warp == 2) {
    // ------------------------------------------------------------ producers
    // warp 0: this CTA's 128 weight rows of the tile; warp 2: its share of
    // the candidates, in the parts of the tile's plan.  Only the leader
    // expects the bytes (both CTAs' loads complete on the leader's barrier).
    if (lane == 0) {
      const bool wprod = warp == 0;
      const int nst = wprod ? WST : XST;
      uint64_t* fullb = wprod ? wfull : xfull;
      uint64_t* emptyb = wprod ? wempty : xempty;
      const uint32_t stage_bytes = wprod ? (uint32_t)kWBytes : (uint32_t)C::X_BYTES;
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      int seq = 0;
      for (int t = unit; t < num_tiles && ok; t += units, seq += G) {
        const Plan plan = tile_plan(G, seq);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&emptyb[s], ph ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t bar = cluster_addr(&fullb[s], 0);
          if (leader) mbar_expect_tx(&fullb[s], 2 * stage_bytes);
          if (wprod) {
            tma_load_2d_pair(sW + s * kWBytes, &tmW, kb * 64, t * kTileRows + (int)rank * kRows, bar);
          } else {
            uint8_t* dst = sX + s * C::X_BYTES;
            for (int i = 0; i < plan.n; ++i) {
              const int g = plan.group[i];
              if (plan.pair[i]) {  // this CTA holds all of group g + rank
                const int row = (g + (int)rank) * kGroupCols;
                tma_load_2d_pair(dst, &tmX, kb * 64, row, bar);
                tma_load_2d_pair(dst + kHalfBytes, &tmX, kb * 64, row + kHalfRows, bar);
                dst += 2 * kHalfBytes;
              } else {  // this CTA holds half `rank` of group g
                tma_load_2d_pair(dst, &tmX, kb * 64, g * kGroupCols + (int)rank * kHalfRows, bar);
                dst += kHalfBytes;
              }
            }
          }
          if (++s == nst) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (lane == 0 && leader) {
      int ws = 0, xs = 0;
      uint32_t wph = 0, xph = 0;
      bool ok = true;
      int seq = 0;  // TMEM group sequence number of this tile's first group
      for (int t = unit; t < num_tiles && ok; t += units, seq += G) {
        // group sequence s lives in TMEM group s & 3, its (s >> 2)-th use
        for (int g = 0; g < G && ok; ++g) {
          const int s = seq + g;
          ok = mbar_wait_cluster(&gempty[s & 3], ((s >> 2) & 1) ^ 1u, abort_flag);
        }
        if (!ok) break;
        tc_fence_after();
        const Plan plan = tile_plan(G, seq);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&wfull[ws], wph, abort_flag) || !mbar_wait(&xfull[xs], xph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t w_addr = smem_u32(sW + ws * kWBytes);
          const uint32_t x_addr = smem_u32(sX + xs * C::X_BYTES);
#pragma unroll
          for (int k = 0; k < K_STEPS; ++k) {
            const uint64_t ad = sw128_kmajor_desc(w_addr + k * 32);
            uint32_t off = 0;
            for (int i = 0; i < plan.n; ++i) {
              const uint32_t d_tmem = tmem_base + (uint32_t)(((seq + plan.group[i]) & 3) * kGroupCols);
              const uint64_t bd = sw128_kmajor_desc(x_addr + off + k * 32);
              umma2_f16(d_tmem, ad, bd, plan.pair[i] ? IDESC_PAIR : IDESC_ONE, (kb | k) != 0);
              off += plan.pair[i] ? 2 * kHalfBytes : kHalfBytes;
            }
          }
          // both stages are free (in both CTAs) once these MMAs have read them
          umma2_commit_both(&wempty[ws]);
          umma2_commit_both(&xempty[xs]);
          if (++ws == WST) {
            ws = 0;
            wph ^= 1u;
          }
          if (++xs == XST) {
            xs = 0;
            xph ^= 1u;
          }
        }
        if (!ok) break;
        for (int g = 0; g < G; ++g) umma2_commit_both(&gfull[(seq + g) & 3]);  // tile complete -> epilogues
      }
      // every MMA issued by this thread has finished before TMEM is released
      umma2_commit_own(drain);
      mbar_wait(drain, 0, abort_flag, /*honour_abort=*/false);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int team = (warp - 3) >> 2;
    const int q = warp & 3;  // TMEM lane quadrant accessible to this warp
    int seq = 0;
    bool stop = false;
    for (int t = unit; t < num_tiles && !stop; t += units, seq += G) {
      const int v = t * kTileRows + (int)rank * kRows + q * 32 + lane;  // this lane's vocabulary row
      const bool v_ok = v < N;
      const float bias = (ep.bias && v_ok) ? load_f32(ep.bias, ep.bias_dtype, v) : 0.0f;
      for (int g = 0; g < G; ++g) {
        const int s = seq + g;
        if ((s & 1) != team) continue;
        const bool got = mbar_wait(&gfull[s & 3], (s >> 2) & 1, abort_flag);
        if (!__all_sync(0xffffffffu, got)) {
          stop = true;
          break;
        }
        tc_fence_after();
        uint32_t r[4][32];
        const uint32_t tb = tmem_base + (uint32_t)((s & 3) * kGroupCols) + ((uint32_t)(q * 32) << 16);
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tb + c * 32, r[c]);
        tmem_wait_ld();
        // the loaded registers are read only after the wait (an empty asm
        // per register orders their uses behind it)
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int j = 0; j < 32; ++j) asm volatile("" : "+r"(r[c][j]));
        tc_fence_before();
        __syncwarp();
        // the group is in registers: free it (the leader's barrier counts both CTAs)
        if (lane == 0) {
          if (leader) mbar_arrive(&gempty[s & 3]);
          else mbar_arrive_remote(cluster_addr(&gempty[s & 3], 0));
        }
        if (!__any_sync(0xffffffffu, v_ok)) continue;  // the whole quadrant is past the vocabulary
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          // lane j ends with column c*32 + j: the maximum over this
          // quadrant's 32 rows and the lowest row that reaches it
          int32_t col_best = INT32_MIN;
          int col_lane = 0;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int32_t o = v_ok ? ordered_i32(__uint_as_float(r[c][j]) + bias) : INT32_MIN;
            const int32_t mx = __reduce_max_sync(0xffffffffu, o);
            const unsigned hit = __ballot_sync(0xffffffffu, o == mx);
            if (lane == j) {
              col_best = mx;
              col_lane = __ffs(hit) - 1;
            }
          }
          const int m = g * kGroupCols + c * 32 + lane;
          if (m < M)
            atomicMax(&skeys[m], make_key(col_best, (uint32_t)(ep.col_offset + (int64_t)t * kTileRows +
                                                               (int)rank * kRows + q * 32 + col_lane)));
        }
      }
    }
    // this CTA's keys into the global ones, then the last CTA decodes
    epi_bar_sync();
    const int et = threadIdx.x - 96;
    for (int i = et; i < M && i < G * kGroupCols; i += kEpiThreads)
      if (skeys[i] != KEY_EMPTY) atomicMax(&ep.keys[i], skeys[i]);
    if (ep.finalize != FIN_NONE) {
      __threadfence();
      epi_bar_sync();
      if (et == 0) {
        const unsigned int ticket = atomicAdd(ep.counter, 1u);
        *last_flag = (ticket == gridDim.x - 1) ? 1 : 0;
      }
      epi_bar_sync();
      if (*last_flag) {
        // every other CTA has taken its ticket: decode, or after a timeout
        // only put the keys back at rest; either way the ticket resets
        __threadfence();
        if (!*abort_flag) verify_finalize(ep, et, kEpiThreads);
        else verify_keys_rest(ep, et, kEpiThreads);
        if (et == 0) *ep.counter = 0u;
      }
    }
  }

  // neither CTA of the pair releases TMEM (or exits, taking its shared
  // memory with it) while the leader's MMAs may still use the other's
  __syncwarp();
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc2(tmem_base, 512);
  }
}

}  // namespace vt
}  // namespace mtp
