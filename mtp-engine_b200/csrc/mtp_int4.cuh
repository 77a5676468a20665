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

}  // namespace w4
}  // namespace mtp
