// mtp_rownorm.cuh -- per-row pre-pass of the RMSNorm-linear GEMMs.
//
// The RMSNorm statistic is a per-row scalar, so it commutes with the K-sum:
//   (x * rstd) @ W^T == rstd * (x @ W^T).
// The GEMM therefore consumes x unmodified and applies rstd (times the FP8
// activation scale) as a per-row factor in its epilogue; this pre-pass reads
// each row once and produces that factor (mtp_kernels.py:179-191 computes the
// same mean of squares in its first pass over x).  Modes:
//   ROW_RSTD     row_out = rstd(x)
//   ROW_GAMMA    row_out = rstd(x); xo = x * gamma (16-bit, the GEMM operand)
//   ROW_QUANT    per-token E4M3: sx = amax/448 (1 for a zero row),
//                xo = e4m3(clamp(x / sx)), row_out = sx * rstd(xo * sx)
//   ROW_PREQUANT x already E4M3 with scale x_scale[m]:
//                row_out = x_scale[m] * rstd(x * x_scale[m])
#pragma once

#include "mtp_common.cuh"

namespace mtp {

enum RowMode : int { ROW_RSTD = 0, ROW_GAMMA = 1, ROW_QUANT = 2, ROW_PREQUANT = 3 };

// Block-wide reduction; `identity` fills the lanes beyond the warp count.
template <typename Op>
__device__ __forceinline__ float block_reduce(float v, Op op, float identity, float* red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, off));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < (int)(blockDim.x >> 5) ? red[lane] : identity;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, off));
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

struct AddOp {
  __device__ float operator()(float a, float b) const { return a + b; }
};
struct MaxOp {
  __device__ float operator()(float a, float b) const { return fmaxf(a, b); }
};

__global__ void __launch_bounds__(256)
    rownorm_kernel(const void* x, int x_dt, const void* gamma, int g_dt, const float* x_scale, int K, float eps,
                   int mode, float* row_out, void* xo, int xo_dt) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int64_t base = row * (int64_t)K;
  float ss = 0.f;
  if (mode == ROW_RSTD || mode == ROW_GAMMA) {
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
      const float v = load_f32(x, x_dt, base + k);
      ss = fmaf(v, v, ss);
      if (mode == ROW_GAMMA) store_f32(xo, xo_dt, base + k, v * load_f32(gamma, g_dt, k));
    }
    ss = block_reduce(ss, AddOp(), 0.0f, red);
    if (threadIdx.x == 0) row_out[row] = 1.0f / sqrtf(ss / (float)K + eps);
    return;
  }
  float sx;
  if (mode == ROW_QUANT) {
    float amax = 0.f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) amax = fmaxf(amax, fabsf(load_f32(x, x_dt, base + k)));
    amax = block_reduce(amax, MaxOp(), 0.0f, red);
    sx = amax > 0.f ? amax / 448.0f : 1.0f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
      const float v = fminf(fmaxf(load_f32(x, x_dt, base + k) / sx, -448.0f), 448.0f);
      const __nv_fp8_storage_t qb = __nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
      static_cast<__nv_fp8_storage_t*>(xo)[base + k] = qb;
      __nv_fp8_e4m3 q;
      q.__x = qb;
      const float d = static_cast<float>(q) * sx;
      ss = fmaf(d, d, ss);
    }
  } else {  // ROW_PREQUANT
    sx = x_scale[row];
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
      const float d = load_f32(x, MTP_DTYPE_E4M3, base + k) * sx;
      ss = fmaf(d, d, ss);
    }
  }
  ss = block_reduce(ss, AddOp(), 0.0f, red);
  if (threadIdx.x == 0) row_out[row] = sx * (1.0f / sqrtf(ss / (float)K + eps));
}

}  // namespace mtp
