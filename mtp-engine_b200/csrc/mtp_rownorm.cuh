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

// ---------------------------------------------------------------------------
// Vectorised variant (16-byte loads / stores) for rows whose length is a
// multiple of 8 and whose pointers are 16-byte aligned; same modes and the
// same arithmetic (ROW_PREQUANT stays on the scalar kernel).
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]);
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x, v[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x, v[2 * i + 1] = f.y;
  }
}

template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&v)[8]);
template <>
__device__ __forceinline__ void store8<float>(float* p, const float (&v)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
template <>
__device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}
template <>
__device__ __forceinline__ void store8<__half>(__half* p, const float (&v)[8]) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

template <typename T>
__global__ void __launch_bounds__(256)
    rownorm_vec_kernel(const T* x, const float* gamma, int K, float eps, int mode, float* row_out, void* xo) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * (int64_t)K;
  const int n8 = K / 8;
  float ss = 0.f;
  if (mode == ROW_RSTD || mode == ROW_GAMMA) {
    for (int i = threadIdx.x; i < n8; i += blockDim.x) {
      float v[8];
      load8<T>(xr + 8 * i, v);
#pragma unroll
      for (int k = 0; k < 8; ++k) ss = fmaf(v[k], v[k], ss);
      if (mode == ROW_GAMMA) {
        float g[8];
        load8<float>(gamma + 8 * i, g);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] *= g[k];
        store8<T>(static_cast<T*>(xo) + row * (int64_t)K + 8 * i, v);
      }
    }
    ss = block_reduce(ss, AddOp(), 0.0f, red);
    if (threadIdx.x == 0) row_out[row] = 1.0f / sqrtf(ss / (float)K + eps);
    return;
  }
  // ROW_QUANT
  float amax = 0.f;
  for (int i = threadIdx.x; i < n8; i += blockDim.x) {
    float v[8];
    load8<T>(xr + 8 * i, v);
#pragma unroll
    for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(v[k]));
  }
  amax = block_reduce(amax, MaxOp(), 0.0f, red);
  const float sx = amax > 0.f ? amax / 448.0f : 1.0f;
  uint8_t* qr = static_cast<uint8_t*>(xo) + row * (int64_t)K;
  for (int i = threadIdx.x; i < n8; i += blockDim.x) {
    float v[8];
    load8<T>(xr + 8 * i, v);
    uint32_t w[2] = {0u, 0u};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float c = fminf(fmaxf(v[k] / sx, -448.0f), 448.0f);
      const __nv_fp8_storage_t qb = __nv_cvt_float_to_fp8(c, __NV_SATFINITE, __NV_E4M3);
      w[k >> 2] |= (uint32_t)qb << (8 * (k & 3));
      __nv_fp8_e4m3 q;
      q.__x = qb;
      const float d = static_cast<float>(q) * sx;
      ss = fmaf(d, d, ss);
    }
    *reinterpret_cast<uint2*>(qr + 8 * i) = make_uint2(w[0], w[1]);
  }
  ss = block_reduce(ss, AddOp(), 0.0f, red);
  if (threadIdx.x == 0) row_out[row] = sx * (1.0f / sqrtf(ss / (float)K + eps));
}

}  // namespace mtp
