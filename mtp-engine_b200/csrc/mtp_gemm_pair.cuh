// mtp_gemm_pair.cuh -- CTA-pair tcgen05 GEMM with the store epilogue.
//
// C[M,N] = A[M,K] * B[N,K]^T (both K-major, the activations and the weight
// as the reference stores them) for the RMSNorm-linear operators: it
// replaces the tl.dot mainloops of fused_rmsnorm_linear_kernel
// (mtp_kernels.py:152-229) and fused_rmsnorm_linear_fp8_kernel (304-367),
// with the same epilogue as gemm_tc_kernel (row scale = rstd or sx*rstd,
// column scale, bias, output scale, cast).
//
// A cluster of two CTAs computes a 256 x BN tile with
// tcgen05.mma.cta_group::2: each CTA loads its own 128 rows of A and half of
// the tile's BN weight rows, and keeps its 128 x BN accumulator in its own
// TMEM (double-buffered, so a tile's epilogue overlaps the next mainloop).
// Per 16-element K step an SM's tensor core then reads 4 KB of A and
// BN/2 x 32 bytes of B from shared memory for 128 x BN x 16 MACs -- 64
// B/clk at BN = 256 against 96 for a one-CTA 128 x 256 tile, whose operand
// reads from shared memory cap it at about 75 % of the tensor rate.
//
// Block of 192 threads, one CTA per SM, persistent over pair tiles
// (numbered M-fastest, so the pairs that share a weight tile run together):
//   warp 0      TMA producer (this CTA's A rows and weight half; both CTAs'
//               loads complete on the leader's full barrier);
//   warp 1      TMEM allocator + MMA issuer (leader only), commits arrive
//               on both CTAs' barriers;
//   warps 2-5   epilogue of this CTA's 128 rows (one row per thread).
// No TMA load uses cluster multicast and every load reads global memory
// into its own CTA, so the kernel is safe in multi-GPU jobs.
#pragma once

#include "mtp_gemm_tc.cuh"
#include "mtp_pair.cuh"

namespace mtp {
namespace pg {

using namespace pair;

constexpr int kRows = 128;       // A rows per CTA = TMEM lanes
constexpr int kTileM = 2 * kRows;
constexpr int kThreads = 192;

template <int BN>
struct Cfg {
  static constexpr int A_BYTES = kRows * 128;  // 128 rows x 128 bytes of K
  static constexpr int B_ROWS = BN / 2;        // weight rows held by one CTA
  static constexpr int B_BYTES = B_ROWS * 128;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (216 * 1024 / STAGE_BYTES) < 8 ? (216 * 1024 / STAGE_BYTES) : 8;
  static constexpr int TMEM_COLS = (2 * BN <= 256) ? 256 : 512;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + BAR_BYTES + 1024;
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "tile width: 32-column epilogue chunks, pair MMA N");
  static_assert(B_BYTES % 1024 == 0, "swizzle atoms stay 1024-byte aligned");
  static_assert(STAGES >= 2, "at least a double-buffered ring");
  // full/empty per stage, tfull/tempty x2, drain; then the TMEM slot and the abort flag
  static_assert((2 * STAGES + 5) * 8 + 2 * 4 <= BAR_BYTES, "barrier area");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory per CTA");
};

// ab_fmt: 0 = f16, 1 = bf16 (kind::f16); FP8: E4M3 x E4M3 (kind::f8f6f4).
// tmA: A [M, K] in boxes of 128 rows; tmB: B [N, K] in boxes of BN/2 rows;
// 128 bytes of K per box, 128-byte swizzle (rows past the end read as
// zeros).  ep.mode must be EPI_STORE.  Launched in clusters of 2 CTAs.
template <int BN, bool FP8, int AB_FMT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M,
                     int N, int num_kb, GemmEpilogue ep) {
  using C = Cfg<BN>;
  constexpr int KB_ELEMS = FP8 ? 128 : 64;  // elements per 128-byte K block
  constexpr int K_STEPS = 4;                // 32 bytes of K per MMA
  constexpr uint32_t IDESC = make_idesc(FP8 ? 0u : (uint32_t)AB_FMT, kTileM, BN);

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

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int unit = (int)(blockIdx.x >> 1);  // cluster index
  const int units = (int)(gridDim.x >> 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);  // lane 0 of the four epilogue warps, in both CTAs
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc2(tmem_slot, C::TMEM_COLS);
    tmem_relinquish2();
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers exist before either CTA's loads or commits reach them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_m = (M + kTileM - 1) / kTileM;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = unit; t < num_tiles && ok; t += units) {
        const int mb = t % num_m, nb = t / num_m;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t bar = cluster_addr(&full[stage], 0);
          if (leader) mbar_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
          tma_load_2d_pair(sA + stage * C::A_BYTES, &tmA, kb * KB_ELEMS, mb * kTileM + (int)rank * kRows, bar);
          tma_load_2d_pair(sB + stage * C::B_BYTES, &tmB, kb * KB_ELEMS, nb * BN + (int)rank * C::B_ROWS, bar);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int local = 0;
      for (int t = unit; t < num_tiles && ok; t += units, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_cluster(&tempty[acc], acc_phase ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < K_STEPS; ++k) {
            const uint64_t ad = sw128_kmajor_desc(a_addr + k * 32);
            const uint64_t bd = sw128_kmajor_desc(b_addr + k * 32);
            if constexpr (FP8) umma2_f8(d_tmem, ad, bd, IDESC, (kb | k) != 0);
            else umma2_f16(d_tmem, ad, bd, IDESC, (kb | k) != 0);
          }
          umma2_commit_both(&empty[stage]);  // the stage is free in both CTAs once these MMAs read it
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma2_commit_both(&tfull[acc]);  // accumulators complete -> both epilogues
      }
      // every MMA issued by this thread has finished before TMEM is released
      umma2_commit_own(drain);
      mbar_wait(drain, 0, abort_flag, /*honour_abort=*/false);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quadrant accessible to this warp
    int local = 0;
    for (int t = unit; t < num_tiles; t += units, ++local) {
      const int mb = t % num_m, nb = t / num_m;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      const bool got = mbar_wait(&tfull[acc], acc_phase, abort_flag);
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      const int row = mb * kTileM + (int)rank * kRows + q * 32 + lane;
      const bool row_ok = row < M;
      const float rs = (ep.row_scale && row_ok) ? ep.row_scale[row] : 1.0f;
      const uint32_t tbase = tmem_base + (uint32_t)(acc * BN) + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        float v[32];
        tc::tmem_ld32_f(tbase + c * 32, v);  // every warp loads: tcgen05.ld is warp-wide
        const int n0 = nb * BN + c * 32;
        if (row_ok && n0 < N) tc::epi_store32(ep, v, row, n0, N, rs);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {  // the accumulator is read (tcgen05 wait and fence above)
        if (leader) mbar_arrive(&tempty[acc]);
        else mbar_arrive_remote(cluster_addr(&tempty[acc], 0));
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
    tmem_dealloc2(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace pg
}  // namespace mtp
