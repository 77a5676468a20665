// mtp_gemm_simt.cuh -- fp32 CUDA-core GEMM with the same epilogues as the
// tensor-core kernel.  It runs the dtype combinations the tensor cores cannot
// take bit-faithfully (anything involving fp32 -- the reference computes in
// IEEE fp32, mtp_kernels.py:782-787 and mtp_fused_verify.py:179-181, and
// tf32 would not match), and shapes whose rows are not 16-byte aligned for
// TMA.  64x64 output tile per 256-thread block, 4x4 outputs per thread.
#pragma once

#include "mtp_verify.cuh"

namespace mtp {
namespace simt {

constexpr int kTile = 64;
constexpr int kBK = 16;

__global__ void __launch_bounds__(256)
    gemm_simt_kernel(const void* A, int a_dt, const void* B, int b_dt, int M, int N, int K, GemmEpilogue ep) {
  __shared__ float As[kBK][kTile + 4];
  __shared__ float Bs[kBK][kTile + 4];
  __shared__ int last;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * kTile, n0 = blockIdx.x * kTile;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  for (int k0 = 0; k0 < K; k0 += kBK) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = tid + 256 * i, r = idx >> 4, kk = idx & 15, k = k0 + kk;
      const int m = m0 + r, n = n0 + r;
      As[kk][r] = (m < M && k < K) ? load_f32(A, a_dt, (int64_t)m * K + k) : 0.f;
      Bs[kk][r] = (n < N && k < K) ? load_f32(B, b_dt, (int64_t)n * K + k) : 0.f;
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

  if (ep.mode == EPI_STORE) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m = m0 + ty + 16 * i;
      if (m >= M) continue;
      const float rs = ep.row_scale ? ep.row_scale[m] : 1.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = n0 + tx + 16 * j;
        if (n >= N) continue;
        float x = acc[i][j] * rs;
        if (ep.col_scale) x *= ep.col_scale[n];
        if (ep.bias) x += load_f32(ep.bias, ep.bias_dtype, n);
        store_f32(ep.y, ep.y_dtype, (int64_t)m * ep.ldy + n, x * ep.scale);
      }
    }
    return;
  }

  // EPI_ARGMAX
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty + 16 * i;
    long long key = KEY_EMPTY;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx + 16 * j;
      if (n < N) {
        float x = acc[i][j];
        if (ep.bias) x += load_f32(ep.bias, ep.bias_dtype, n);
        const long long k = make_key(ordered_i32(x), (uint32_t)(ep.col_offset + n));
        key = k > key ? k : key;
      }
    }
    // the 16 threads of a row are 16 consecutive lanes
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) {
      const long long o = __shfl_xor_sync(0xffffffffu, key, off);
      key = o > key ? o : key;
    }
    if (tx == 0 && m < M && key != KEY_EMPTY) atomicMax(&ep.keys[m], key);
  }
  if (ep.finalize == FIN_NONE) return;
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned int ticket = atomicAdd(ep.counter, 1u);
    last = (ticket == gridDim.x * gridDim.y - 1) ? 1 : 0;
  }
  __syncthreads();
  if (last) {
    __threadfence();
    verify_finalize(ep, tid, 256);
    if (tid == 0) *ep.counter = 0u;
  }
}

}  // namespace simt
}  // namespace mtp
