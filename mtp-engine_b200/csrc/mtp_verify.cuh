// mtp_verify.cuh -- GEMM epilogue parameters shared by the tensor-core and
// CUDA-core GEMMs, and the acceptance scan that turns argmax keys into the
// outputs of fused_verify / fused_multi_verify (mtp_fused_verify.py:43-156;
// eager semantics mtp_fused_verify.py:159-196).
#pragma once

#include "mtp_common.cuh"

namespace mtp {

enum EpiMode : int { EPI_STORE = 0, EPI_ARGMAX = 1 };
enum FinMode : int { FIN_NONE = 0, FIN_CHAIN = 1, FIN_SINGLE = 2, FIN_CHAIN_PEERS = 3 };

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
  // Vocab-parallel verify with the reduction fused into the GEMM
  // (FIN_CHAIN_PEERS, stream-K kernel only): every rank owns a buffer
  //   keys [2 parities][peer_rows] int64 | flags [2][world] uint64 | epoch uint64
  // mapped into every rank; peers[r] is rank r's buffer.  Keys go to the
  // parity (epoch + 1) & 1 of every rank's buffer; null peers: keys[] only.
  const unsigned long long* peers;
  int rank, world;
  int64_t peer_rows;
};

// Offsets inside a fused-exchange buffer (see GemmEpilogue::peers).
__host__ __device__ inline int64_t peer_flags_offset(int64_t rows) { return 2 * rows * 8; }
__host__ __device__ inline int64_t peer_epoch_offset(int64_t rows, int world) {
  return 2 * rows * 8 + 2 * (int64_t)world * 8;
}

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

// The keys of a verify whose CTAs gave up on a bounded wait, put back at
// rest without decoding: that call's outputs are undefined (the error word
// holds MTP_ERR_TIMEOUT), the next call on the workspace runs normally.
__device__ inline void verify_keys_rest(const GemmEpilogue& ep, int tid, int nthreads) {
  const int64_t n = ep.finalize == FIN_CHAIN ? ep.B * ep.S : ep.B;
  for (int64_t i = tid; i < n; i += nthreads) ep.keys[i] = KEY_EMPTY;
}

__global__ void verify_finalize_kernel(GemmEpilogue ep) {
  verify_finalize(ep, blockIdx.x * blockDim.x + threadIdx.x, gridDim.x * blockDim.x);
}

// ---------------------------------------------------------------------------
// Vocab-parallel key exchange over peer memory (the NCCL all-reduce's job, in
// one kernel, followed by the acceptance scan).  Every rank owns a buffer of
//   keys  [2 parities][world][rows] int64, then flags [2 parities][world] uint64
// mapped into every peer (symmetric memory); peers[r] is rank r's buffer.
// Call e (a per-rank device counter, identical on all ranks because every
// rank makes the same calls) uses parity e & 1: this rank stores its local
// keys into slot [rank] of every peer's buffer with plain stores over NVLink,
// fences at system scope, releases flag [rank] = e in every peer, waits until
// its own flags of all ranks reach e (bounded: 2 s, then MTP_ERR_TIMEOUT),
// and decodes the max over ranks.  A rank can only reach call e+2 after every
// rank has started call e+1, i.e. after every rank finished reading call e,
// so two parities suffice.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(256)
    verify_exchange_chain_kernel(long long* local_keys, const unsigned long long* peers, int rank, int world,
                                 unsigned long long* epoch_counter, GemmEpilogue ep) {
  __shared__ unsigned long long s_epoch;
  __shared__ int s_ok;
  const int64_t rows = ep.B * ep.S;
  if (threadIdx.x == 0) {
    s_epoch = ++(*epoch_counter);
    s_ok = 1;
  }
  __syncthreads();
  const unsigned long long e = s_epoch;
  const int par = (int)(e & 1ull);
  auto keys_of = [&](unsigned long long base, int slot) {
    return reinterpret_cast<long long*>(base) + ((int64_t)par * world + slot) * rows;
  };
  auto flags_of = [&](unsigned long long base) {
    return reinterpret_cast<unsigned long long*>(reinterpret_cast<long long*>(base) + 2 * (int64_t)world * rows) +
           (int64_t)par * world;
  };
  // 1. push this rank's keys into every peer (its own buffer included)
  for (int p = 0; p < world; ++p) {
    long long* dst = keys_of(peers[p], rank);
    for (int64_t r = threadIdx.x; r < rows; r += blockDim.x) dst[r] = local_keys[r];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0)
    for (int p = 0; p < world; ++p) st_release_sys_u64(flags_of(peers[p]) + rank, e);
  // 2. wait for every rank's keys in this rank's buffer
  if (threadIdx.x < world) {
    const unsigned long long* f = flags_of(peers[rank]) + threadIdx.x;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys_u64(f) < e) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        record_error(MTP_ERR_TIMEOUT);
        s_ok = 0;
        break;
      }
    }
  }
  __syncthreads();
  // 3. max over ranks, then the acceptance scan into the outputs.  Peers wrote
  // these slots over NVLink into this GPU's L2: read them from L2 (__ldcg).
  const long long* mine = keys_of(peers[rank], 0);
  for (int64_t r = threadIdx.x; r < rows; r += blockDim.x) {
    long long k = __ldcg(mine + r);
    for (int p = 1; p < world; ++p) {
      const long long o = __ldcg(mine + (int64_t)p * rows + r);
      k = o > k ? o : k;
    }
    local_keys[r] = k;  // reduced key; verify_finalize reads then resets it
  }
  __threadfence_block();
  __syncthreads();
  if (s_ok) {
    GemmEpilogue f = ep;
    f.keys = local_keys;
    verify_finalize(f, threadIdx.x, blockDim.x);
  } else {
    for (int64_t r = threadIdx.x; r < rows; r += blockDim.x) local_keys[r] = KEY_EMPTY;
  }
}

// The host step that follows fused_multi_verify in generate_fused and
// generate_optimized (mtp_engine.py:1244-1258, 1326-1337), on the device:
// n = min over the batch of accepted_n (one shared rollback index per step);
// the step's tokens are draft[:, :n] followed by corrected when some draft
// was rejected (n < D), else all D drafts; info = {n, width}.  One block.
__global__ void __launch_bounds__(256)
    verify_step_kernel(const int32_t* draft, const int32_t* accepted_n, const int32_t* corrected, int64_t B,
                       int64_t D, int32_t* step_tokens, int64_t ld, int32_t* info) {
  __shared__ int red[8];
  int m = INT32_MAX;
  for (int64_t b = threadIdx.x; b < B; b += blockDim.x) m = min(m, accepted_n[b]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = min(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  int n = red[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) n = min(n, red[w]);
  n = max(0, min(n, (int)D));
  const int64_t width = n == D ? D : (int64_t)n + 1;
  // every column of [0, min(ld, D + 1)) is written: tokens up to width, then
  // -1 (no token), so a replayed step leaves the same bytes as an eager one
  const int64_t cols = ld < D + 1 ? ld : D + 1;
  for (int64_t i = threadIdx.x; i < B * cols; i += blockDim.x) {
    const int64_t b = i / cols, j = i - b * cols;
    step_tokens[b * ld + j] = j >= width ? -1 : (j < n ? draft[b * D + j] : corrected[b]);
  }
  if (threadIdx.x == 0) {
    info[0] = n;
    info[1] = (int32_t)width;
  }
}

__global__ void keys_fill_kernel(long long* keys, int64_t n, unsigned int* counter) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) keys[i] = KEY_EMPTY;
  if (i == 0 && counter) *counter = 0u;
}

}  // namespace mtp
