// mtp_int4.cuh -- y = x @ dequant(W)^T for group-quantised INT4 weights:
// fused_int4_matmul (mtp_kernels.py:1194-1219; Triton kernel 433-489; eager
// _eager_int4_matmul 875-878 over dequantize_int4 754-767).
//
// W is packed two 4-bit codes per byte along K (element 2j in the low nibble
// of byte j, 2j+1 in the high nibble), decoded as (code - 8) * scales[n, k /
// group] -- the decoding of both reference paths (lines 761-762, 475-476).
// The weight is read once at half a byte per element; the product is exact
// fp32 FMA on CUDA cores, matching the reference's fp32 dot
// (allow_tf32=False, line 485).  64 x 64 output tile per 256-thread block;
// each thread decodes whole bytes (two K elements) of the weight tile.
#pragma once

#include "mtp_common.cuh"

namespace mtp {
namespace w4 {

constexpr int kTile = 64;
constexpr int kBK = 32;  // K elements per step: 16 bytes of each weight row

__global__ void __launch_bounds__(256)
    int4_matmul_kernel(const void* x, int x_dt, const uint8_t* __restrict__ packed, const float* __restrict__ scales,
                       int group, void* y, int y_dt, int M, int N, int K) {
  __shared__ float As[kBK][kTile + 4];
  __shared__ float Bs[kBK][kTile + 4];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * kTile, n0 = blockIdx.x * kTile;
  const int64_t row_bytes = K / 2;
  const int64_t groups = (K + group - 1) / group;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  for (int k0 = 0; k0 < K; k0 += kBK) {
    // activations: 64 rows x 32 K, 8 per thread
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int idx = tid + 256 * i, r = idx >> 5, kk = idx & 31, k = k0 + kk, m = m0 + r;
      As[kk][r] = (m < M && k < K) ? load_f32(x, x_dt, (int64_t)m * K + k) : 0.f;
    }
    // weights: 64 rows x 16 bytes, 4 bytes (8 K elements) per thread
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = tid + 256 * i, r = idx >> 4, jb = idx & 15, n = n0 + r;
      const int k = k0 + 2 * jb;
      float lo = 0.f, hi = 0.f;
      if (n < N && k < K) {
        const int byte = packed[(int64_t)n * row_bytes + k / 2];
        const float* srow = scales + (int64_t)n * groups;
        lo = (float)((byte & 0x0F) - 8) * srow[k / group];
        if (k + 1 < K) hi = (float)(((byte >> 4) & 0x0F) - 8) * srow[(k + 1) / group];
      }
      Bs[2 * jb][r] = lo;
      Bs[2 * jb + 1][r] = hi;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kBK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty + 16 * i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx + 16 * j;
      if (n < N) store_f32(y, y_dt, (int64_t)m * N + n, acc[i][j]);
    }
  }
}

// Decode-sized M (<= 8 rows): the packed weight is streamed at HBM speed.
// 8 warps per block, gemv_rows_per_warp(MR) weight rows per warp (fewer as
// MR grows, to keep the rows x MR accumulators in registers); each lane owns
// 32 consecutive K codes (one 16-byte load per row and 1024-element chunk).  x is staged
// per chunk in shared memory transposed within 32-element groups, padded to 33
// words per group, so both the staging stores (consecutive K) and the reads
// (lane l, code j) fall in distinct banks.  Per-lane partial sums, then a
// warp reduction.  Needs K % 32 == 0 and a 16-byte-aligned packed array.
__host__ __device__ constexpr int gemv_rows_per_warp(int mr) { return mr <= 2 ? 8 : (mr == 4 ? 4 : 2); }
__host__ __device__ constexpr int gemv_block_rows(int mr) { return 8 * gemv_rows_per_warp(mr); }
constexpr int kGemvKC = 1024;
constexpr int kGemvPitch = 33;  // words per 32-code group in the staged x

template <int MR>
__global__ void __launch_bounds__(256)
    int4_gemv_kernel(const void* x, int x_dt, const uint8_t* __restrict__ packed, const float* __restrict__ scales,
                     int group, void* y, int y_dt, int M, int N, int K) {
  constexpr int kGemvRowsPerWarp = gemv_rows_per_warp(MR);
  __shared__ float xs[MR][32 * kGemvPitch];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * gemv_block_rows(MR) + warp * kGemvRowsPerWarp;
  const int64_t row_bytes = K / 2;
  const int64_t groups = (K + group - 1) / group;
  const bool one_scale = group % 32 == 0;  // a lane's 32 codes share one scale
  float acc[kGemvRowsPerWarp][MR];
#pragma unroll
  for (int r = 0; r < kGemvRowsPerWarp; ++r)
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[r][m] = 0.f;

  for (int kc = 0; kc < K; kc += kGemvKC) {
    __syncthreads();
    for (int i = threadIdx.x; i < MR * kGemvKC; i += 256) {
      const int m = i / kGemvKC, kl = i % kGemvKC, k = kc + kl;
      xs[m][(kl & 31) * kGemvPitch + (kl >> 5)] = (m < M && k < K) ? load_f32(x, x_dt, (int64_t)m * K + k) : 0.f;
    }
    __syncthreads();
    const int kb = kc + lane * 32;  // this lane's codes kb .. kb + 31
    if (kb >= K) continue;
    // every row's 32 codes first (rows past N: code 8 everywhere, weight 0)
    uint32_t wd[kGemvRowsPerWarp][4];
    float s0[kGemvRowsPerWarp];
    const float* srow[kGemvRowsPerWarp];
#pragma unroll
    for (int r = 0; r < kGemvRowsPerWarp; ++r) {
      const int n = n0 + r < N ? n0 + r : N - 1;
      srow[r] = scales + (int64_t)n * groups;
      uint4 u = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);
      if (n0 + r < N) u = __ldg(reinterpret_cast<const uint4*>(packed + (int64_t)n * row_bytes + kb / 2));
      wd[r][0] = u.x;
      wd[r][1] = u.y;
      wd[r][2] = u.z;
      wd[r][3] = u.w;
      s0[r] = one_scale ? srow[r][kb / group] : 0.f;
    }
    // then each x value once, against every row
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      float xv[MR];
#pragma unroll
      for (int m = 0; m < MR; ++m) xv[m] = xs[m][j * kGemvPitch + lane];
#pragma unroll
      for (int r = 0; r < kGemvRowsPerWarp; ++r) {
        const int code = (int)((wd[r][j >> 3] >> (4 * (j & 7))) & 0xFu);
        const float w = (float)(code - 8) * (one_scale ? s0[r] : srow[r][(kb + j) / group]);
#pragma unroll
        for (int m = 0; m < MR; ++m) acc[r][m] = fmaf(xv[m], w, acc[r][m]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kGemvRowsPerWarp; ++r) {
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      float v = acc[r][m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      const int n = n0 + r;
      if (lane == 0 && m < M && n < N) store_f32(y, y_dt, (int64_t)m * N + n, v);
    }
  }
}

}  // namespace w4
}  // namespace mtp
