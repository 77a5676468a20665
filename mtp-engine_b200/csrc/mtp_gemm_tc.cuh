// mtp_gemm_tc.cuh -- persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
// C[M,N] = A[M,K] * B[N,K]^T with both operands K-major in HBM (activations
// x / hidden and the weight W / lm_head exactly as the reference stores
// them).  It replaces the fp32 tl.dot mainloops of
// fused_rmsnorm_linear_kernel (mtp_kernels.py:152-229),
// fused_rmsnorm_linear_fp8_kernel (304-367) and the per-position GEMV of
// fused_multi_verify_kernel (mtp_fused_verify.py:89-156).
//
// Block of 192 threads, one CTA per SM, persistent over 128 x BN tiles:
//   warp 0      TMA producer: 128-byte-swizzled A and B K-blocks into a
//               STAGES-deep shared-memory ring (full/empty mbarriers);
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer, fp32
//               accumulator double-buffered in TMEM (2 x BN columns) so the
//               epilogue of tile i overlaps the mainloop of tile i+1;
//   warps 2-5   epilogue: tcgen05.ld of one accumulator row per thread,
//               then either the RMSNorm-linear store (row/col scales, bias,
//               scale, cast) or the verify argmax (bias, running row max,
//               one atomicMax of a packed (value, index) key per row and
//               tile -- no logits ever reach HBM).
// Tiles are numbered M-fastest so the CTAs that share a weight tile run at
// the same time and the weight is read from HBM about once.
// No clusters; every TMA load fills its own CTA, so the same kernel serves multi-GPU jobs.
#pragma once

#include "mtp_verify.cuh"

namespace mtp {
namespace tc {

constexpr int kBM = 128;
constexpr int kThreads = 192;
constexpr int kKBlockBytes = 128;  // one 128-byte swizzle row of K per stage

template <int BN>
struct Cfg {
  static constexpr int TILE_M = kBM;
  static constexpr int A_BYTES = kBM * kKBlockBytes;
  static constexpr int B_BYTES = BN * kKBlockBytes;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (220 * 1024 / STAGE_BYTES) < 8 ? (220 * 1024 / STAGE_BYTES) : 8;
  static constexpr int ACC_COLS = BN;  // one tile's accumulators
  static constexpr int ACC_BUFS = 2;   // double-buffered: tile i's epilogue overlaps tile i+1's mainloop
  static constexpr int TMEM_COLS = (ACC_BUFS * ACC_COLS <= 256) ? 256 : 512;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + BAR_BYTES + 1024;
  // UMMA with M = 128: N a multiple of 16 in [16, 256]
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "tile width");
  // SW128 operand atoms are 8 rows x 128 bytes; every stage base stays 1024-byte aligned
  static_assert(A_BYTES % 1024 == 0 && B_BYTES % 1024 == 0, "stage alignment");
  static_assert(STAGES >= 2, "at least a double-buffered ring");
  // full/empty per stage, tfull/tempty x2, drain; then the TMEM slot and four flags (stream-K uses all)
  static_assert((2 * STAGES + 5) * 8 + 5 * 4 <= BAR_BYTES, "barrier area");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory per CTA");
  static_assert(ACC_BUFS * ACC_COLS <= TMEM_COLS && TMEM_COLS <= 512, "accumulators in TMEM");
};

// Tile t (taken by a CTA as t = blockIdx.x + j * gridDim.x) -> row tile mb
// and column tile nb, M-fastest so the CTAs that share a weight tile run at
// the same time.  Host and device run the same code (the host to check the
// order).
__host__ __device__ __forceinline__ void tile_coords(int t, int num_m, int& mb, int& nb) {
  nb = t / num_m;
  mb = t % num_m;
}

__device__ __forceinline__ void epi_bar_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Store epilogue for 32 accumulator values of one row (row < M), columns
// n0..n0+31 (n0 < N): y = (acc * rs * col_scale[n] + bias[n]) * scale in y's
// dtype, as 16-byte stores when the 32 columns are all inside N and aligned.
__device__ __forceinline__ void epi_store32(const GemmEpilogue& ep, const float (&acc)[32], int64_t row, int n0,
                                            int N, float rs) {
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int n = n0 + j;
    float x = acc[j] * rs;
    if (n < N) {
      if (ep.col_scale) x *= ep.col_scale[n];
      if (ep.bias) x += load_f32(ep.bias, ep.bias_dtype, n);
    }
    v[j] = x * ep.scale;
  }
  const int64_t off = row * ep.ldy + n0;
  if (ep.y_vec_ok && n0 + 32 <= N && ep.y_dtype != MTP_DTYPE_F32) {
    uint32_t packed[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (ep.y_dtype == MTP_DTYPE_BF16) {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
        packed[j] = *reinterpret_cast<uint32_t*>(&h);
      } else {
        __half2 h = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
        packed[j] = *reinterpret_cast<uint32_t*>(&h);
      }
    }
    uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(ep.y) + off);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      dst[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
  } else {
    for (int j = 0; j < 32 && n0 + j < N; ++j) store_f32(ep.y, ep.y_dtype, off + j, v[j]);
  }
}

// Argmax epilogue over 32 accumulator values, columns n0..n0+31: logit =
// acc + bias[n]; only a strictly greater logit replaces (best, best_n), so
// the first (lowest) index wins a tie.
__device__ __forceinline__ void epi_argmax32(const GemmEpilogue& ep, const float (&acc)[32], int n0, int N,
                                             int32_t& best, int& best_n) {
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int n = n0 + j;
    if (n < N) {
      float x = acc[j];
      if (ep.bias) x += load_f32(ep.bias, ep.bias_dtype, n);
      const int32_t o = ordered_i32(x);
      if (o > best) {
        best = o;
        best_n = n;
      }
    }
  }
}

// 32 fp32 accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32_f(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  tmem_ld32(taddr, r);
  tmem_wait_ld();
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

// ab_fmt: 0 = f16, 1 = bf16 (kind::f16); FP8: E4M3 x E4M3 (kind::f8f6f4)
template <int BN, bool FP8, int AB_FMT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M,
                   int N, int num_kb, GemmEpilogue ep) {
  using C = Cfg<BN>;
  constexpr int KB_ELEMS = FP8 ? 128 : 64;       // elements per 128-byte K block
  constexpr int UMMA_K_BYTES = 32;               // K per tcgen05.mma: 16 x 16-bit or 32 x 8-bit
  constexpr int K_STEPS = kKBlockBytes / UMMA_K_BYTES;
  constexpr uint32_t IDESC = make_idesc(FP8 ? 0u : (uint32_t)AB_FMT, kBM, BN);

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

  const int num_m = (M + kBM - 1) / kBM;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, num_m, mb, nb);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[stage], C::A_BYTES + C::B_BYTES);
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
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * C::ACC_COLS);
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
            const uint64_t ad = sw128_kmajor_desc(a_addr + k * UMMA_K_BYTES);
            const uint64_t bd = sw128_kmajor_desc(b_addr + k * UMMA_K_BYTES);
            if constexpr (FP8) umma_f8(d_tmem, ad, bd, IDESC, (kb | k) != 0);
            else umma_f16(d_tmem, ad, bd, IDESC, (kb | k) != 0);
          }
          umma_commit(&empty[stage]);  // frees this stage once its MMAs have read it
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);  // accumulator complete -> epilogue
      }
      // every MMA issued by this thread has finished before TMEM is released
      umma_commit(drain);
      mbar_wait(drain, 0, abort_flag, /*honour_abort=*/false);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quadrant accessible to this warp
    const int row_in_tile = q * 32 + lane;
    int local = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++local) {
      int mb, nb;
      tile_coords(t, num_m, mb, nb);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      const bool got = mbar_wait(&tfull[acc], acc_phase, abort_flag);
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      {
        const int row = mb * kBM + row_in_tile;
        const bool row_ok = row < M;
        const uint32_t tbase = tmem_base + (uint32_t)(acc * C::ACC_COLS) + ((uint32_t)(q * 32) << 16);
        if (ep.mode == EPI_STORE) {
          const float rs = (ep.row_scale && row_ok) ? ep.row_scale[row] : 1.0f;
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            float v[32];
            tmem_ld32_f(tbase + c * 32, v);  // every warp loads: tcgen05.ld is warp-wide
            const int n0 = nb * BN + c * 32;
            if (row_ok && n0 < N) epi_store32(ep, v, row, n0, N, rs);
          }
        } else {
          int32_t best = INT32_MIN;
          int best_n = nb * BN;
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            float v[32];
            tmem_ld32_f(tbase + c * 32, v);
            epi_argmax32(ep, v, nb * BN + c * 32, N, best, best_n);
          }
          if (row_ok) atomicMax(&ep.keys[row], make_key(best, (uint32_t)(ep.col_offset + best_n)));
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
    if (ep.mode == EPI_ARGMAX && ep.finalize != FIN_NONE) {
      // last CTA to finish decodes the keys (threadFenceReduction pattern)
      __threadfence();
      epi_bar_sync();
      if (threadIdx.x == 64) {
        const unsigned int ticket = atomicAdd(ep.counter, 1u);
        *last_flag = (ticket == gridDim.x - 1) ? 1 : 0;
      }
      epi_bar_sync();
      if (*last_flag) {
        // every other CTA has taken its ticket: decode, or after a timeout
        // only put the keys back at rest; either way the ticket resets, so
        // the workspace is at rest when the launch ends
        __threadfence();
        if (!*abort_flag) verify_finalize(ep, threadIdx.x - 64, 128);
        else verify_keys_rest(ep, threadIdx.x - 64, 128);
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

}  // namespace tc
}  // namespace mtp
