// mtp_rowattn.cuh -- single-query attention over a contiguous key block for
// any head size up to 8192, followed by the RMSNorm of its output: the
// attention and normalisation half of fused_tree_attn_rmsnorm_linear
// (mtp_kernels.py:1222-1250, eager _eager_tree_attn_rmsnorm_linear 881-905,
// whose callers pass the whole hidden state as one head, mtp_engine.py:812,
// 1492).  The projection half is the GEMM (store epilogue with wscale as the
// column scale and the bias).
//
// One 256-thread CTA per query row (b, h); HBM-bound: each row reads its
// L x D keys and values once.
//   1. q -> shared memory (fp32), laid out lane-interleaved so that a warp
//      reading "its" VEC elements of 32 consecutive chunks hits 32 banks;
//   2. the kept keys (mask[j] > 0.5; the mask is shared by every row) are
//      compacted in key order with warp ballots;
//   3. scores: one warp per kept key, 16-byte loads across the head
//      dimension, warp-shuffle sum;
//   4. softmax statistics over the kept scores (block reductions);
//   5. P V: each thread owns fixed VEC-element chunks of the head dimension
//      and accumulates over the kept keys (a warp's loads are contiguous);
//   6. out = o * rsqrt(mean(o^2) + eps) * gamma, written in the GEMM's operand
//      dtype.
// A row with no kept key is NaN (the reference's softmax of all -inf).
#pragma once

#include <type_traits>

#include "mtp_common.cuh"

namespace mtp {
namespace rowattn {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxD = 8192;
constexpr int kAccPerThread = kMaxD / kThreads;  // 32 fp32 accumulators

template <typename T>
__device__ __forceinline__ float to_f32(T x) {
  if constexpr (std::is_same<T, float>::value) return x;
  else if constexpr (std::is_same<T, __nv_bfloat16>::value) return __bfloat162float(x);
  else return __half2float(x);
}

template <typename T>
__device__ __forceinline__ T from_f32(float x) {
  if constexpr (std::is_same<T, float>::value) return x;
  else if constexpr (std::is_same<T, __nv_bfloat16>::value) return __float2bfloat16_rn(x);
  else return __float2half_rn(x);
}

// VEC consecutive elements as fp32: VEC = 1 (scalar), 4 (fp32 as float4) or
// 8 (16-bit as one 16-byte load).
template <typename T, int VEC>
__device__ __forceinline__ void load_vec(const T* p, float (&f)[VEC]) {
  if constexpr (VEC == 1) {
    f[0] = to_f32(*p);
  } else if constexpr (std::is_same<T, float>::value) {
    static_assert(VEC == 4, "fp32 vectors are float4");
    const float4 u = __ldg(reinterpret_cast<const float4*>(p));
    f[0] = u.x;
    f[1] = u.y;
    f[2] = u.z;
    f[3] = u.w;
  } else {
    static_assert(VEC == 8, "16-bit vectors are 8 elements");
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        f[2 * i] = __uint_as_float(w[i] << 16);
        f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      } else {
        const float2 h = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        f[2 * i] = h.x;
        f[2 * i + 1] = h.y;
      }
    }
  }
}

template <typename TO, int VEC>
__device__ __forceinline__ void store_vec(TO* p, const float (&f)[VEC]) {
  if constexpr (VEC == 1) {
    p[0] = from_f32<TO>(f[0]);
  } else if constexpr (std::is_same<TO, float>::value) {
#pragma unroll
    for (int i = 0; i < VEC; i += 4)
      *reinterpret_cast<float4*>(p + i) = make_float4(f[i], f[i + 1], f[i + 2], f[i + 3]);
  } else {
    static_assert(VEC == 8, "16-bit vectors are 8 elements");
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (std::is_same<TO, __nv_bfloat16>::value) {
        __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
        w[i] = *reinterpret_cast<uint32_t*>(&h);
      } else {
        __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
        w[i] = *reinterpret_cast<uint32_t*>(&h);
      }
    }
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// shared-memory index of element e of chunk c in the lane-interleaved q copy
template <int VEC>
__device__ __forceinline__ int qidx(int c, int e) {
  return ((c >> 5) * VEC + e) * 32 + (c & 31);
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) t += red[w];
  return t;
}

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = -INFINITY;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) t = fmaxf(t, red[w]);
  return t;
}

// Floats of the lane-interleaved q copy: whole groups of 32 chunks.
__host__ __device__ inline int q_floats(int D, int vec) { return ((D / vec + 31) / 32) * 32 * vec; }

// Dynamic shared memory: q (lane-interleaved), p [L] fp32, ids [L].
inline size_t smem_bytes(int64_t L, int64_t D, int vec) { return ((size_t)q_floats((int)D, vec) + 2 * L) * 4; }

template <typename T, typename TO, int VEC>
__global__ void __launch_bounds__(kThreads) row_attn_norm_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                                 const T* __restrict__ v,
                                                                 const float* __restrict__ mask,
                                                                 const float* __restrict__ gamma,
                                                                 TO* __restrict__ out, int L, int D, float scale,
                                                                 float eps) {
  constexpr int CH = kAccPerThread / VEC;  // chunks a thread owns in P V
  extern __shared__ float4 smem4[];
  float* sq = reinterpret_cast<float*>(smem4);
  float* sp = sq + q_floats(D, VEC);
  int* sid = reinterpret_cast<int*>(sp + L);
  __shared__ float red[kWarps];
  __shared__ int red_i[kWarps];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = blockIdx.x;
  const int nc = D / VEC;
  const T* qr = q + row * (int64_t)D;
  const T* kr = k + row * (int64_t)L * D;
  const T* vr = v + row * (int64_t)L * D;

  // 1. q
  for (int c = threadIdx.x; c < nc; c += kThreads) {
    float f[VEC];
    load_vec<T, VEC>(qr + (int64_t)c * VEC, f);
#pragma unroll
    for (int e = 0; e < VEC; ++e) sq[qidx<VEC>(c, e)] = f[e];
  }
  // 2. kept keys, in key order
  int nkeep = 0;
  for (int base = 0; base < L; base += kThreads) {
    const int j = base + threadIdx.x;
    const bool keep = j < L && (mask == nullptr || mask[j] > 0.5f);
    const unsigned bal = __ballot_sync(0xffffffffu, keep);
    if (lane == 0) red_i[warp] = __popc(bal);
    __syncthreads();
    int before = nkeep, total = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      before += (w < warp) ? red_i[w] : 0;
      total += red_i[w];
    }
    if (keep) sid[before + __popc(bal & ((1u << lane) - 1u))] = j;
    nkeep += total;
    __syncthreads();
  }
  // 3. scores of the kept keys
  for (int i = warp; i < nkeep; i += kWarps) {
    const T* kj = kr + (int64_t)sid[i] * D;
    float acc = 0.f;
#pragma unroll 4
    for (int c = lane; c < nc; c += 32) {
      float f[VEC];
      load_vec<T, VEC>(kj + (int64_t)c * VEC, f);
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc = fmaf(sq[qidx<VEC>(c, e)], f[e], acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) sp[i] = acc * scale;
  }
  __syncthreads();
  // 4. softmax statistics
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < nkeep; i += kThreads) mx = fmaxf(mx, sp[i]);
  mx = block_max(mx, red);
  float sum = 0.f;
  for (int i = threadIdx.x; i < nkeep; i += kThreads) {
    const float p = expf(sp[i] - mx);
    sp[i] = p;
    sum += p;
  }
  sum = block_sum(sum, red);  // its barriers also publish sp
  // 5. P V
  float acc[kAccPerThread];
#pragma unroll
  for (int i = 0; i < kAccPerThread; ++i) acc[i] = 0.f;
#pragma unroll 2
  for (int i = 0; i < nkeep; ++i) {
    const float p = sp[i];
    const T* vj = vr + (int64_t)sid[i] * D;
#pragma unroll
    for (int u = 0; u < CH; ++u) {
      const int c = threadIdx.x + u * kThreads;
      if (c < nc) {
        float f[VEC];
        load_vec<T, VEC>(vj + (int64_t)c * VEC, f);
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[u * VEC + e] = fmaf(p, f[e], acc[u * VEC + e]);
      }
    }
  }
  // 6. normalise, RMSNorm, gamma
  const float inv = nkeep > 0 ? 1.0f / sum : __int_as_float(0x7fc00000);  // no kept key: NaN
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < CH; ++u) {
    const int c = threadIdx.x + u * kThreads;
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float o = acc[u * VEC + e] * inv;
      acc[u * VEC + e] = o;
      if (c < nc) ss = fmaf(o, o, ss);
    }
  }
  ss = block_sum(ss, red);
  const float rstd = 1.0f / sqrtf(ss / (float)D + eps);
  TO* orow = out + row * (int64_t)D;
#pragma unroll
  for (int u = 0; u < CH; ++u) {
    const int c = threadIdx.x + u * kThreads;
    if (c < nc) {
      float f[VEC];
#pragma unroll
      for (int e = 0; e < VEC; ++e) f[e] = acc[u * VEC + e] * rstd * (gamma ? gamma[c * VEC + e] : 1.0f);
      store_vec<TO, VEC>(orow + (int64_t)c * VEC, f);
    }
  }
}

}  // namespace rowattn
}  // namespace mtp
