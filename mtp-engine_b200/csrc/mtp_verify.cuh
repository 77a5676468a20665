// mtp_verify.cuh -- GEMM epilogue parameters shared by the tensor-core and
// CUDA-core GEMMs, and the acceptance scan that turns argmax keys into the
// outputs of fused_verify / fused_multi_verify (mtp_fused_verify.py:43-156;
// eager semantics mtp_fused_verify.py:159-196).
#pragma once

#include "mtp_common.cuh"

namespace mtp {

enum EpiMode : int { EPI_STORE = 0, EPI_ARGMAX = 1 };
enum FinMode : int { FIN_NONE = 0, FIN_CHAIN = 1, FIN_SINGLE = 2 };

struct GemmEpilogue {
  int mode;  // EpiMode
  // EPI_STORE: y[m,n] = (acc * row_scale[m] * col_scale[n] + bias[n]) * scale
  const float* row_scale;  // [M] or null
  const float* col_scale;  // [N] or null
  const void* bias;        // [N] or null
  int bias_dtype;
  float scale;
  void* y;
  int y_dtype;
  int y_vec_ok;  // 16-byte vector stores allowed (alignment checked on the host)
  int64_t ldy;
  // EPI_ARGMAX: keys[m] = max(keys[m], key(acc + bias[n], col_offset + n))
  long long* keys;
  int64_t col_offset;
  // fused finalisation by the last CTA to finish (FinMode)
  int finalize;
  unsigned int* counter;
  const int32_t* draft;
  int8_t* accept;
  int32_t* accepted_n;
  int32_t* tokens;  // FIN_CHAIN: corrected[B]; FIN_SINGLE: top[M]
  int64_t B, S;     // FIN_CHAIN: rows = B*S; FIN_SINGLE: rows = B, S = 1
};

// Decode keys into the verify outputs and put the keys back to KEY_EMPTY.
// FIN_CHAIN follows the prefix-gated loop of _eager_fused_multi_verify
// (mtp_fused_verify.py:184-195): accept[b,d] = 1 while every draft so far
// matched top[b,d+1]; entries after the first reject stay 0; accepted_n is
// the accepted prefix length; corrected is the anchor top[b,0].
// FIN_SINGLE follows _eager_fused_verify (mtp_fused_verify.py:159-166).
__device__ inline void verify_finalize(const GemmEpilogue& ep, int tid, int nthreads) {
  if (ep.finalize == FIN_CHAIN) {
    const int64_t S = ep.S, D = S - 1;
    for (int64_t b = tid; b < ep.B; b += nthreads) {
      long long* kr = ep.keys + b * S;
      const int32_t t0 = key_index(__ldcg(kr));
      int32_t n = 0;
      bool ok = true;
      for (int64_t d = 0; d < D; ++d) {
        const int32_t t = key_index(__ldcg(kr + d + 1));
        const bool acc = ok && (t == ep.draft[b * D + d]);
        ep.accept[b * D + d] = acc ? 1 : 0;
        if (acc) n = (int32_t)(d + 1);
        else ok = false;
      }
      ep.accepted_n[b] = n;
      ep.tokens[b] = t0;
      for (int64_t s = 0; s < S; ++s) kr[s] = KEY_EMPTY;
    }
  } else if (ep.finalize == FIN_SINGLE) {
    for (int64_t m = tid; m < ep.B; m += nthreads) {
      const int32_t t = key_index(__ldcg(ep.keys + m));
      ep.tokens[m] = t;
      ep.accept[m] = (t == ep.draft[m]) ? 1 : 0;
      ep.keys[m] = KEY_EMPTY;
    }
  }
}

__global__ void verify_finalize_kernel(GemmEpilogue ep) {
  verify_finalize(ep, blockIdx.x * blockDim.x + threadIdx.x, gridDim.x * blockDim.x);
}

__global__ void keys_fill_kernel(long long* keys, int64_t n, unsigned int* counter) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) keys[i] = KEY_EMPTY;
  if (i == 0 && counter) *counter = 0u;
}

}  // namespace mtp
