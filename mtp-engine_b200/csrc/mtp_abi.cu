// mtp_abi.cu -- the C ABI (include/mtp_b200.h): argument checks, workspace
// carving, kernel selection and launches.  Built as one translation unit so
// every kernel shares the per-device error word.
//
// Nothing here allocates device memory or synchronises the host (except
// mtp_device_status), so every entry point can be captured in a CUDA graph
// and called on any stream.

#include <atomic>
#include <mutex>
#include <new>
#include <vector>
#include <stdarg.h>
#include <stdlib.h>
#include <stdio.h>

#include <nvtx3/nvToolsExt.h>

#include "mtp_attention.cuh"
#include "mtp_attention_tc.cuh"
#include "mtp_gemm_simt.cuh"
#include "mtp_gemm_sk.cuh"
#include "mtp_gemm_tc.cuh"
#include "mtp_gemm_vt.cuh"
#include "mtp_gemm_pair.cuh"
#include "mtp_rownorm.cuh"
#include "mtp_rowattn.cuh"
#include "mtp_kvwrite.cuh"
#include "mtp_nccl.cuh"
#include "mtp_int4.cuh"
#include "mtp_sqattn.cuh"
#include "mtp_verify.cuh"

using namespace mtp;

// Scratch of mtp_fused_multi_verify_noalloc: MTP_NOALLOC_MAX_ROWS int64 keys,
// then the last-CTA ticket counter in the final 256 bytes.  A module-scope
// device array, so the library never allocates it; in host code its name is
// only a stand-in -- its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[MTP_NOALLOC_MAX_ROWS * 8 + 256];

namespace {

constexpr int kAbiVersion = 2;

// A named NVTX range around each compute entry point, so profilers can select
// an operator by name (ncu --nvtx --nvtx-include); free when no tool is attached.
struct NvtxScope {
  explicit NvtxScope(const char* name) { nvtxRangePushA(name); }
  ~NvtxScope() { nvtxRangePop(); }
};
#define MTP_NVTX(name) NvtxScope mtp_nvtx_scope_(name)
constexpr int kMaxDevices = 64;

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

#define MTP_CUDA_TRY(expr)                                                                  \
  do {                                                                                      \
    cudaError_t e_ = (expr);                                                                \
    if (e_ != cudaSuccess) return fail(MTP_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(e_)); \
  } while (0)

std::atomic<uint64_t> g_launches{0};

// after every kernel launch: surface launch errors, count the launch
#define MTP_LAUNCH_CHECK()                  \
  do {                                      \
    MTP_CUDA_TRY(cudaGetLastError());       \
    g_launches.fetch_add(1, std::memory_order_relaxed); \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }
inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
inline bool is16bit(int dt) { return dt == MTP_DTYPE_BF16 || dt == MTP_DTYPE_F16; }
inline bool valid_dtype(int dt) { return dt >= MTP_DTYPE_F32 && dt <= MTP_DTYPE_E4M3; }

int current_device(int* dev) {
  MTP_CUDA_TRY(cudaGetDevice(dev));
  if (*dev < 0 || *dev >= kMaxDevices) return fail(MTP_ERR_CUDA, "device index %d out of range", *dev);
  return MTP_OK;
}

int sm_count(int dev) {
  static int cache[kMaxDevices] = {0};
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

// ---------------------------------------------------------------- tensor maps
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D K-major operand [rows, cols] with a row pitch of `row_bytes`, loaded in
// boxes of (128 bytes of K) x box_rows with the 128-byte swizzle.
int make_kmajor_map(CUtensorMap* map, const void* base, bool fp8, int dt16, int64_t rows, int64_t cols,
                    int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(MTP_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const int eb = fp8 ? 1 : 2;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(cols * eb)};
  const cuuint32_t box[2] = {(cuuint32_t)(128 / eb), (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType t = fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                    : (dt16 == MTP_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                              : CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
  CUresult r = enc(map, t, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MTP_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return MTP_OK;
}

// ---------------------------------------------------------------- GEMM launchers
template <int BN, bool FP8, int FMT>
int launch_tc_inst(const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int num_kb, const GemmEpilogue& ep,
                   cudaStream_t s) {
  auto kern = tc::gemm_tc_kernel<BN, FP8, FMT>;
  constexpr int smem = tc::Cfg<BN>::SMEM_BYTES;
  int dev;
  if (int st = current_device(&dev)) return st;
  static bool attr_done[kMaxDevices] = {false};
  if (!attr_done[dev]) {
    MTP_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr_done[dev] = true;
  }
  const int tiles = ((M + tc::kBM - 1) / tc::kBM) * ((N + BN - 1) / BN);
  const int grid = tiles < sm_count(dev) ? tiles : sm_count(dev);
  kern<<<grid, tc::kThreads, smem, s>>>(ta, tb, M, N, num_kb, ep);
  MTP_LAUNCH_CHECK();
  return MTP_OK;
}

// Tile width for a persistent launch.  The mainloop is bound by the shared-
// memory operand traffic, which per K-block is (128 + BN) rows of 128 bytes,
// so a launch costs about rounds x (128 + BN) with rounds = ceil(tiles/SMs);
// the widest tile wins a tie.
int pick_bn(int64_t M, int64_t N, int sms) {
  static const int cands[6] = {256, 224, 192, 160, 128, 64};
  int best = 256;
  int64_t best_cost = INT64_MAX;
  for (int bn : cands) {
    if ((bn > 128 && N <= 128) || (bn > 64 && N <= 64)) continue;
    const int64_t tiles = ((M + tc::kBM - 1) / tc::kBM) * ((N + bn - 1) / bn);
    const int64_t rounds = (tiles + sms - 1) / sms;
    const int64_t cost = rounds * (bn + 128);
    if (cost < best_cost) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

template <bool FP8, int FMT>
int launch_tc_bn(int bn, const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int num_kb,
                 const GemmEpilogue& ep, cudaStream_t s) {
  switch (bn) {
    case 256: return launch_tc_inst<256, FP8, FMT>(ta, tb, M, N, num_kb, ep, s);
    case 224: return launch_tc_inst<224, FP8, FMT>(ta, tb, M, N, num_kb, ep, s);
    case 192: return launch_tc_inst<192, FP8, FMT>(ta, tb, M, N, num_kb, ep, s);
    case 160: return launch_tc_inst<160, FP8, FMT>(ta, tb, M, N, num_kb, ep, s);
    case 128: return launch_tc_inst<128, FP8, FMT>(ta, tb, M, N, num_kb, ep, s);
    default: return launch_tc_inst<64, FP8, FMT>(ta, tb, M, N, num_kb, ep, s);
  }
}

// ---------------------------------------------------------------- vocabulary-tiled verify GEMM
template <int G, int WST, int XST, int FMT>
int launch_vt_inst(const CUtensorMap& tw, const CUtensorMap& tx, int M, int N, int num_kb, const GemmEpilogue& ep,
                   cudaStream_t s) {
  auto kern = vt::gemm_vt_kernel<G, WST, XST, FMT>;
  constexpr int smem = vt::Cfg<G, WST, XST>::SMEM_BYTES;
  int dev;
  if (int st = current_device(&dev)) return st;
  static int pairs_max[kMaxDevices] = {0};  // clusters resident at once
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(vt::kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (!pairs_max[dev]) {
    MTP_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const int u = sm_count(dev) / 2;
    cfg.gridDim = dim3(2 * u, 1, 1);
    int clusters = 0;
    MTP_CUDA_TRY(cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg));
    if (clusters < 1) return fail(MTP_ERR_CUDA, "no 2-CTA cluster fits the vocabulary-tiled verify kernel");
    pairs_max[dev] = clusters < u ? clusters : u;
  }
  const int tiles = (N + vt::kTileRows - 1) / vt::kTileRows;
  const int pairs = tiles < pairs_max[dev] ? tiles : pairs_max[dev];
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  MTP_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, tw, tx, M, N, num_kb, ep));
  MTP_LAUNCH_CHECK();
  return MTP_OK;
}

template <int FMT>
int launch_vt_groups(int groups, const CUtensorMap& tw, const CUtensorMap& tx, int M, int N, int num_kb,
                     const GemmEpilogue& ep, cudaStream_t s) {
  switch (groups) {
    case 1: return launch_vt_inst<1, 8, 8, FMT>(tw, tx, M, N, num_kb, ep, s);
    case 2: return launch_vt_inst<2, 6, 6, FMT>(tw, tx, M, N, num_kb, ep, s);
    case 3: return launch_vt_inst<3, 5, 5, FMT>(tw, tx, M, N, num_kb, ep, s);
    default: return launch_vt_inst<4, 4, 4, FMT>(tw, tx, M, N, num_kb, ep, s);
  }
}

// 16-bit argmax GEMMs of at most 512 candidate rows run the vocabulary-
// tiled CTA-pair kernel unless MTP_VERIFY_VT=0 is set (then the row-tiled
// one, for comparisons).  Measured on B200: verify B=64 S=6 V=128256
// 312 us against 334; one rank of an 8-way verify (V=16032) 59 us against
// 71; B=40 S=5 with a bias 226 us against 316.
static bool vt_enabled() {
  const char* e = getenv("MTP_VERIFY_VT");
  return !(e && e[0] == '0' && e[1] == 0);
}

// The verify argmax with weight rows as the MMA's rows (CTA pairs): 16-bit
// operands, at most 512 candidate rows.
int launch_gemm_vt(const void* X, const void* W, int ab_dtype, int64_t M, int64_t N, int64_t K,
                   const GemmEpilogue& ep, cudaStream_t s) {
  CUtensorMap tw, tx;
  if (int st = make_kmajor_map(&tw, W, false, ab_dtype, N, K, vt::kRows)) return st;
  if (int st = make_kmajor_map(&tx, X, false, ab_dtype, M, K, vt::kHalfRows)) return st;
  const int num_kb = (int)((K * 2 + tc::kKBlockBytes - 1) / tc::kKBlockBytes);
  const int groups = (int)((M + vt::kGroupCols - 1) / vt::kGroupCols);
  if (ab_dtype == MTP_DTYPE_BF16) return launch_vt_groups<1>(groups, tw, tx, (int)M, (int)N, num_kb, ep, s);
  return launch_vt_groups<0>(groups, tw, tx, (int)M, (int)N, num_kb, ep, s);
}

// ---------------------------------------------------------------- CTA-pair store GEMM
// Clusters of 2 resident at once for a pair kernel (1 CTA per SM).
template <typename Kern>
int pair_clusters(Kern kern, int smem, int threads, int dev, int* out) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int u = sm_count(dev) / 2;
  cfg.gridDim = dim3(2 * u, 1, 1);
  int clusters = 0;
  MTP_CUDA_TRY(cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg));
  if (clusters < 1) return fail(MTP_ERR_CUDA, "no 2-CTA cluster fits the pair GEMM");
  *out = clusters < u ? clusters : u;
  return MTP_OK;
}

template <int BN, bool FP8, int FMT>
int launch_pair_inst(const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int num_kb, const GemmEpilogue& ep,
                     cudaStream_t s) {
  auto kern = pg::gemm_pair_kernel<BN, FP8, FMT>;
  constexpr int smem = pg::Cfg<BN>::SMEM_BYTES;
  int dev;
  if (int st = current_device(&dev)) return st;
  static int pairs_max[kMaxDevices] = {0};
  if (!pairs_max[dev]) {
    MTP_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    if (int st = pair_clusters(kern, smem, pg::kThreads, dev, &pairs_max[dev])) return st;
  }
  // As few pairs as finish the tiles in the same number of rounds (128 tiles
  // on 74 pairs take two rounds; 64 pairs take two as well): the makespan is
  // unchanged and the SMs left over serve whatever runs beside the GEMM
  // (the candidates' all-gather of a vocab-parallel verify).
  const int tiles = ((M + pg::kTileM - 1) / pg::kTileM) * ((N + BN - 1) / BN);
  const int rounds = (tiles + pairs_max[dev] - 1) / pairs_max[dev];
  const int pairs = (tiles + rounds - 1) / rounds;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(pg::kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  MTP_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, ta, tb, M, N, num_kb, ep));
  MTP_LAUNCH_CHECK();
  return MTP_OK;
}

// Tile width of the pair GEMM: fewest rounds x BN (the mainloop time of a
// round is proportional to BN), the widest on a tie.
int pick_bn_pair(int64_t M, int64_t N, int pairs) {
  static const int cands[5] = {256, 224, 192, 160, 128};
  int best = 256;
  int64_t best_cost = INT64_MAX;
  for (int bn : cands) {
    if (bn > 128 && N <= 128) continue;
    const int64_t tiles = ((M + pg::kTileM - 1) / pg::kTileM) * ((N + bn - 1) / bn);
    const int64_t rounds = (tiles + pairs - 1) / pairs;
    const int64_t cost = rounds * bn;
    if (cost < best_cost) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

template <bool FP8, int FMT>
int launch_pair_bn(int bn, const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int num_kb,
                   const GemmEpilogue& ep, cudaStream_t s) {
  switch (bn) {
    case 256: return launch_pair_inst<256, FP8, FMT>(ta, tb, M, N, num_kb, ep, s);
    case 224: return launch_pair_inst<224, FP8, FMT>(ta, tb, M, N, num_kb, ep, s);
    case 192: return launch_pair_inst<192, FP8, FMT>(ta, tb, M, N, num_kb, ep, s);
    case 160: return launch_pair_inst<160, FP8, FMT>(ta, tb, M, N, num_kb, ep, s);
    default: return launch_pair_inst<128, FP8, FMT>(ta, tb, M, N, num_kb, ep, s);
  }
}

// Store-epilogue GEMMs of 129-4096 rows run on CTA pairs unless
// MTP_GEMM_PAIR=0 is set (then the one-CTA kernel, for comparisons).
// Measured on B200 (RMSNorm-linear, N=14336, K=4096): M=512 and 2048 5-8 %
// faster on pairs, FP8 M=1024 N=28672 K=8192 7 %; M=8192 12 % slower (its
// operands no longer fit L2 and the pair tiles' order re-reads them more).
static bool pair_enabled() {
  const char* e = getenv("MTP_GEMM_PAIR");
  return !(e && e[0] == '0' && e[1] == 0);
}

int launch_gemm_pair(const void* A, const void* B, int ab_dtype, bool fp8, int64_t M, int64_t N, int64_t K,
                     const GemmEpilogue& ep, cudaStream_t s) {
  int dev;
  if (int st = current_device(&dev)) return st;
  const int bn = pick_bn_pair(M, N, sm_count(dev) / 2);
  CUtensorMap ta, tb;
  if (int st = make_kmajor_map(&ta, A, fp8, ab_dtype, M, K, pg::kRows)) return st;
  if (int st = make_kmajor_map(&tb, B, fp8, ab_dtype, N, K, bn / 2)) return st;
  const int eb = fp8 ? 1 : 2;
  const int num_kb = (int)((K * eb + tc::kKBlockBytes - 1) / tc::kKBlockBytes);
  if (fp8) return launch_pair_bn<true, 0>(bn, ta, tb, (int)M, (int)N, num_kb, ep, s);
  if (ab_dtype == MTP_DTYPE_BF16) return launch_pair_bn<false, 1>(bn, ta, tb, (int)M, (int)N, num_kb, ep, s);
  return launch_pair_bn<false, 0>(bn, ta, tb, (int)M, (int)N, num_kb, ep, s);
}

// ---------------------------------------------------------------- stream-K
// Process-wide GEMM schedule: 0 = data-parallel tiles (default), 1 = the
// stream-K schedule wherever its plan is cheaper and the caller's workspace
// has room for it (mtp_set_gemm_schedule).
std::atomic<int> g_gemm_schedule{0};

// Stream-K counters: a fixed 16 KB ending 256 bytes before the end of the
// workspace (the last 256 bytes are the verify ticket), so a workspace reused
// for other sizes keeps them at rest; the partial slots need no init.
constexpr size_t kSkCounterBytes = 16384;
constexpr size_t kSkTail = kSkCounterBytes + 256;
static_assert(kSkTail == MTP_STREAMK_TAIL_BYTES, "header and library disagree on the stream-K tail");

struct SkPlan {
  bool use = false;
  int bn = 256;
  int grid = 0;
  sk::Sched s{};
  size_t slot_bytes = 0;
};

// Cost in the units of pick_bn (K blocks x (128 + BN) rows of operand
// traffic per CTA).  A part that arrives last reads each other part's slot
// (128 x BN fp32 from L2, about 6 K blocks' worth at BN = 256), plus ~2 for
// storing its own.  grid > 0 forces the schedule on that many CTAs (tests).
SkPlan sk_plan(int64_t M, int64_t N, int num_kb, int sms, int grid) {
  SkPlan p;
  p.bn = N > 128 ? 256 : 128;
  const int64_t num_m = (M + tc::kBM - 1) / tc::kBM, num_n = (N + p.bn - 1) / p.bn;
  const int64_t T = num_m * num_n;
  const int P = grid > 0 ? grid : sms;
  if (T <= 0 || P <= 0 || num_kb <= 0 || T > INT32_MAX / 2) return p;
  int64_t dp_rounds = T / P - 1;
  if (dp_rounds < 0) dp_rounds = 0;
  const int64_t sk_tiles = T - dp_rounds * P;
  if (sk_tiles * 8 > (int64_t)kSkCounterBytes) return p;
  const int64_t sk_total = sk_tiles * num_kb;
  const int64_t q = (sk_total + P - 1) / P;
  p.grid = P;
  p.s.num_m = (int)num_m;
  p.s.num_tiles = (int)T;
  p.s.num_kb = num_kb;
  p.s.dp_rounds = (int)dp_rounds;
  p.s.dp_tiles = (int)(dp_rounds * P);
  p.s.q = (int)q;
  p.s.sk_total = sk_total;
  p.slot_bytes = align256((size_t)2 * P * tc::kBM * p.bn * 4);
  if (grid > 0) {
    p.use = true;
    return p;
  }
  if (T % P == 0) return p;  // whole rounds: nothing to balance
  const int64_t max_parts = q >= num_kb ? 2 : (num_kb + q - 1) / q + 1;
  const int64_t fix = (6 * (max_parts - 1) + 2) * p.bn / 256;
  const int64_t cost_sk = (dp_rounds * num_kb + q + fix) * (p.bn + 128);
  const int bn_dp = pick_bn(M, N, sms);
  const int64_t t_dp = num_m * ((N + bn_dp - 1) / bn_dp);
  const int64_t cost_dp = ((t_dp + sms - 1) / sms) * num_kb * (bn_dp + 128);
  p.use = cost_sk * 100 < cost_dp * 97;
  return p;
}

size_t sk_bytes_needed(const SkPlan& p) { return p.use ? p.slot_bytes + kSkTail : 0; }

// Every tile whole, run by the stream-K kernel (its fused epilogues need it).
SkPlan dp_only_plan(int64_t M, int64_t N, int num_kb, int sms) {
  SkPlan p;
  p.bn = N > 128 ? 256 : 128;
  const int64_t num_m = (M + tc::kBM - 1) / tc::kBM, num_n = (N + p.bn - 1) / p.bn;
  const int64_t T = num_m * num_n;
  if (T <= 0 || T > INT32_MAX / 2 || num_kb <= 0) return p;
  p.grid = (int)(T < sms ? T : sms);
  p.s.num_m = (int)num_m;
  p.s.num_tiles = (int)T;
  p.s.num_kb = num_kb;
  p.s.dp_rounds = (int)((T + p.grid - 1) / p.grid);
  p.s.dp_tiles = (int)T;
  p.s.q = 1;
  p.s.sk_total = 0;
  p.slot_bytes = 0;
  p.use = true;
  return p;
}

template <int BN, bool FP8, int FMT>
int launch_sk_inst(const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, const SkPlan& pl,
                   unsigned long long* counters, float* slots, const GemmEpilogue& ep, cudaStream_t s) {
  auto kern = sk::gemm_sk_kernel<BN, FP8, FMT>;
  // verify workspaces rest at INT64_MIN everywhere: clean the slots after use
  const int clean_slots = ep.mode == EPI_ARGMAX ? 1 : 0;
  constexpr int smem = tc::Cfg<BN>::SMEM_BYTES;
  int dev;
  if (int st = current_device(&dev)) return st;
  static bool attr_done[kMaxDevices] = {false};
  if (!attr_done[dev]) {
    MTP_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr_done[dev] = true;
  }
  kern<<<pl.grid, tc::kThreads, smem, s>>>(ta, tb, M, N, pl.s, counters, slots, clean_slots, ep);
  MTP_LAUNCH_CHECK();
  return MTP_OK;
}

int launch_sk_plan(const void* A, const void* B, int ab_dtype, bool fp8, int64_t M, int64_t N, int64_t K,
                   const GemmEpilogue& ep, cudaStream_t s, const SkPlan& pl, float* slots,
                   unsigned long long* counters);

// Stream-K launch when the schedule is on (or forced by sk_grid > 0) and the
// region [sk_ws, sk_ws + sk_bytes) holds the slots followed by the counter
// tail.  *launched stays false when the data-parallel kernel should run.
int try_launch_sk(const void* A, const void* B, int ab_dtype, bool fp8, int64_t M, int64_t N, int64_t K,
                  const GemmEpilogue& ep, cudaStream_t s, void* sk_ws, size_t sk_bytes, int sk_grid,
                  bool* launched) {
  *launched = false;
  if (!sk_ws || (sk_grid <= 0 && g_gemm_schedule.load(std::memory_order_relaxed) != 1)) return MTP_OK;
  int dev;
  if (int st = current_device(&dev)) return st;
  const int eb = fp8 ? 1 : 2;
  const int num_kb = (int)((K * eb + tc::kKBlockBytes - 1) / tc::kKBlockBytes);
  const SkPlan pl = sk_plan(M, N, num_kb, sm_count(dev), sk_grid);
  if (!pl.use || sk_bytes < sk_bytes_needed(pl)) return MTP_OK;
  uint8_t* base = static_cast<uint8_t*>(sk_ws);
  *launched = true;
  return launch_sk_plan(A, B, ab_dtype, fp8, M, N, K, ep, s, pl, reinterpret_cast<float*>(base),
                        reinterpret_cast<unsigned long long*>(base + sk_bytes - kSkTail));
}

// The stream-K kernel with plan `pl`; slots/counters as laid out by the plan.
int launch_sk_plan(const void* A, const void* B, int ab_dtype, bool fp8, int64_t M, int64_t N, int64_t K,
                   const GemmEpilogue& ep, cudaStream_t s, const SkPlan& pl, float* slots,
                   unsigned long long* counters) {
  CUtensorMap ta, tb;
  if (int st = make_kmajor_map(&ta, A, fp8, ab_dtype, M, K, tc::kBM)) return st;
  if (int st = make_kmajor_map(&tb, B, fp8, ab_dtype, N, K, pl.bn)) return st;
  const int m = (int)M, n = (int)N;
  if (pl.bn == 256) {
    if (fp8) return launch_sk_inst<256, true, 0>(ta, tb, m, n, pl, counters, slots, ep, s);
    if (ab_dtype == MTP_DTYPE_BF16) return launch_sk_inst<256, false, 1>(ta, tb, m, n, pl, counters, slots, ep, s);
    return launch_sk_inst<256, false, 0>(ta, tb, m, n, pl, counters, slots, ep, s);
  }
  if (fp8) return launch_sk_inst<128, true, 0>(ta, tb, m, n, pl, counters, slots, ep, s);
  if (ab_dtype == MTP_DTYPE_BF16) return launch_sk_inst<128, false, 1>(ta, tb, m, n, pl, counters, slots, ep, s);
  return launch_sk_inst<128, false, 0>(ta, tb, m, n, pl, counters, slots, ep, s);
}

// A [M,K] and B [N,K] both K-major, 16-bit (ab_dtype) or E4M3 (fp8).  With a
// stream-K region (see try_launch_sk) the stream-K kernel may run instead.
int launch_gemm_tc(const void* A, const void* B, int ab_dtype, bool fp8, int64_t M, int64_t N, int64_t K,
                   const GemmEpilogue& ep, cudaStream_t s, void* sk_ws = nullptr, size_t sk_bytes = 0,
                   int sk_grid = 0) {
  if (sk_ws || sk_grid > 0) {
    bool launched = false;
    if (int st = try_launch_sk(A, B, ab_dtype, fp8, M, N, K, ep, s, sk_ws, sk_bytes, sk_grid, &launched)) return st;
    if (launched) return MTP_OK;
  }
  if (ep.mode == EPI_ARGMAX && ep.finalize != FIN_CHAIN_PEERS && !fp8 && M >= 1 && M <= vt::kMaxCands &&
      vt_enabled())
    return launch_gemm_vt(A, B, ab_dtype, M, N, K, ep, s);
  if (ep.mode == EPI_STORE && M > tc::kBM && M <= 4096 && pair_enabled())
    return launch_gemm_pair(A, B, ab_dtype, fp8, M, N, K, ep, s);
  int dev;
  if (int st = current_device(&dev)) return st;
  const int bn = pick_bn(M, N, sm_count(dev));
  CUtensorMap ta, tb;
  if (int st = make_kmajor_map(&ta, A, fp8, ab_dtype, M, K, tc::kBM)) return st;
  if (int st = make_kmajor_map(&tb, B, fp8, ab_dtype, N, K, bn)) return st;
  const int eb = fp8 ? 1 : 2;
  const int num_kb = (int)((K * eb + tc::kKBlockBytes - 1) / tc::kKBlockBytes);
  if (fp8) return launch_tc_bn<true, 0>(bn, ta, tb, (int)M, (int)N, num_kb, ep, s);
  if (ab_dtype == MTP_DTYPE_BF16) return launch_tc_bn<false, 1>(bn, ta, tb, (int)M, (int)N, num_kb, ep, s);
  return launch_tc_bn<false, 0>(bn, ta, tb, (int)M, (int)N, num_kb, ep, s);
}

bool tc_eligible(const void* A, const void* B, int a_dt, int b_dt, int64_t M, int64_t N, int64_t K) {
  const bool fp8 = a_dt == MTP_DTYPE_E4M3 && b_dt == MTP_DTYPE_E4M3;
  const bool h16 = is16bit(a_dt) && a_dt == b_dt;
  if (!fp8 && !h16) return false;
  const int eb = fp8 ? 1 : 2;
  if ((K * eb) % 16 != 0) return false;  // TMA row pitch must be a multiple of 16 bytes
  if (!aligned16(A) || !aligned16(B)) return false;
  if (M > INT32_MAX / 2 || N > INT32_MAX / 2 || K > INT32_MAX / 2) return false;
  return true;
}

int launch_gemm_simt(const void* A, int a_dt, const void* B, int b_dt, int64_t M, int64_t N, int64_t K,
                     const GemmEpilogue& ep, cudaStream_t s) {
  if (M > 65535LL * simt::kTile) return fail(MTP_ERR_SHAPE, "M=%lld too large for the fp32 path", (long long)M);
  dim3 grid((unsigned)((N + simt::kTile - 1) / simt::kTile), (unsigned)((M + simt::kTile - 1) / simt::kTile));
  simt::gemm_simt_kernel<<<grid, 256, 0, s>>>(A, a_dt, B, b_dt, (int)M, (int)N, (int)K, ep);
  MTP_LAUNCH_CHECK();
  return MTP_OK;
}

int launch_gemm(const void* A, int a_dt, const void* B, int b_dt, int64_t M, int64_t N, int64_t K,
                const GemmEpilogue& ep, cudaStream_t s, void* sk_ws = nullptr, size_t sk_bytes = 0) {
  if (tc_eligible(A, B, a_dt, b_dt, M, N, K))
    return launch_gemm_tc(A, B, a_dt, a_dt == MTP_DTYPE_E4M3, M, N, K, ep, s, sk_ws, sk_bytes);
  return launch_gemm_simt(A, a_dt, B, b_dt, M, N, K, ep, s);
}

int launch_rownorm(const void* x, int x_dt, const void* gamma, int g_dt, const float* x_scale, int64_t M,
                   int64_t K, float eps, int mode, float* row_out, void* xo, int xo_dt, cudaStream_t s) {
  if (M == 0) return MTP_OK;
  if (M > INT32_MAX) return fail(MTP_ERR_SHAPE, "too many rows");
  const bool vec = mode != ROW_PREQUANT && K % 8 == 0 && aligned16(x) && (!xo || aligned16(xo)) &&
                   (mode != ROW_GAMMA || (g_dt == MTP_DTYPE_F32 && aligned16(gamma) && xo_dt == x_dt)) &&
                   (mode != ROW_QUANT || xo_dt == MTP_DTYPE_E4M3) &&
                   (x_dt == MTP_DTYPE_F32 || x_dt == MTP_DTYPE_BF16 || x_dt == MTP_DTYPE_F16);
  if (vec) {
    const float* g = static_cast<const float*>(gamma);
    if (x_dt == MTP_DTYPE_BF16)
      rownorm_vec_kernel<__nv_bfloat16><<<(unsigned)M, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), g, (int)K,
                                                                    eps, mode, row_out, xo);
    else if (x_dt == MTP_DTYPE_F16)
      rownorm_vec_kernel<__half><<<(unsigned)M, 256, 0, s>>>(static_cast<const __half*>(x), g, (int)K, eps, mode,
                                                             row_out, xo);
    else
      rownorm_vec_kernel<float><<<(unsigned)M, 256, 0, s>>>(static_cast<const float*>(x), g, (int)K, eps, mode,
                                                            row_out, xo);
    MTP_LAUNCH_CHECK();
    return MTP_OK;
  }
  rownorm_kernel<<<(unsigned)M, 256, 0, s>>>(x, x_dt, gamma, g_dt, x_scale, (int)K, eps, mode, row_out, xo, xo_dt);
  MTP_LAUNCH_CHECK();
  return MTP_OK;
}

GemmEpilogue store_epilogue(const float* row_scale, const float* col_scale, const void* bias, int bias_dt,
                            float scale, void* y, int y_dt, int64_t N) {
  GemmEpilogue ep{};
  ep.mode = EPI_STORE;
  ep.row_scale = row_scale;
  ep.col_scale = col_scale;
  ep.bias = bias;
  ep.bias_dtype = bias_dt;
  ep.scale = scale;
  ep.y = y;
  ep.y_dtype = y_dt;
  ep.ldy = N;
  ep.y_vec_ok = is16bit(y_dt) && aligned16(y) && (N % 8 == 0);
  return ep;
}

int check_dims(int64_t M, int64_t N, int64_t K) {
  if (M < 0 || N < 0 || K < 0) return fail(MTP_ERR_SHAPE, "negative size");
  if (K == 0) return fail(MTP_ERR_SHAPE, "K must be positive");
  if (N > 0xFFFFFFFFLL || M > INT32_MAX || K > INT32_MAX) return fail(MTP_ERR_SHAPE, "size out of range");
  return MTP_OK;
}

size_t verify_ws_bytes(int64_t rows) { return align256((size_t)rows * 8) + 256; }

// Device address of g_noalloc_scratch on the current device, looked up once
// per device (with that device current) and cached.
int noalloc_scratch(unsigned char** out) {
  static std::mutex mu;
  static unsigned char* cache[kMaxDevices] = {nullptr};
  int dev;
  if (int st = current_device(&dev)) return st;
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(MTP_ERR_CUDA, "cudaGetSymbolAddress(no-allocation scratch) failed: %s", cudaGetErrorString(e));
    cache[dev] = static_cast<unsigned char*>(p);
  }
  *out = cache[dev];
  return MTP_OK;
}

// --------------------------------------------------------------- tree attn -> RMSNorm -> linear
// The normalised attention output is the GEMM's A operand: in the weight's
// 16-bit dtype when q has that same dtype (tensor cores), else fp32.
int tarl_operand_dtype(int q_dtype, int w_dtype) {
  return (is16bit(w_dtype) && w_dtype == q_dtype) ? q_dtype : MTP_DTYPE_F32;
}

size_t tarl_base_bytes(int64_t B, int64_t H, int64_t D, int q_dtype, int w_dtype) {
  const int ao = tarl_operand_dtype(q_dtype, w_dtype);
  return align256((size_t)B * H * D * (ao == MTP_DTYPE_F32 ? 4 : 2));
}

template <typename T, typename TO, int VEC>
int launch_rowattn_inst(const void* q, const void* k, const void* v, const float* mask, const float* gamma,
                        void* out, int64_t rows, int64_t L, int64_t D, float scale, float eps, cudaStream_t s) {
  auto kern = rowattn::row_attn_norm_kernel<T, TO, VEC>;
  const size_t smem = rowattn::smem_bytes(L, D, VEC);
  int dev;
  if (int st = current_device(&dev)) return st;
  static size_t attr[kMaxDevices] = {0};
  if (smem > 48 * 1024 && attr[dev] < smem) {
    MTP_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr[dev] = smem;
  }
  kern<<<(unsigned)rows, rowattn::kThreads, smem, s>>>(static_cast<const T*>(q), static_cast<const T*>(k),
                                                       static_cast<const T*>(v), mask, gamma, static_cast<TO*>(out),
                                                       (int)L, (int)D, scale, eps);
  MTP_LAUNCH_CHECK();
  return MTP_OK;
}

template <typename T>
int launch_rowattn_t(bool vec, bool out_f32, const void* q, const void* k, const void* v, const float* mask,
                     const float* gamma, void* out, int64_t rows, int64_t L, int64_t D, float scale, float eps,
                     cudaStream_t s) {
  constexpr int V = std::is_same<T, float>::value ? 4 : 8;
  if constexpr (std::is_same<T, float>::value) {
    if (vec) return launch_rowattn_inst<T, float, V>(q, k, v, mask, gamma, out, rows, L, D, scale, eps, s);
    return launch_rowattn_inst<T, float, 1>(q, k, v, mask, gamma, out, rows, L, D, scale, eps, s);
  } else {
    if (out_f32) {
      if (vec) return launch_rowattn_inst<T, float, V>(q, k, v, mask, gamma, out, rows, L, D, scale, eps, s);
      return launch_rowattn_inst<T, float, 1>(q, k, v, mask, gamma, out, rows, L, D, scale, eps, s);
    }
    if (vec) return launch_rowattn_inst<T, T, V>(q, k, v, mask, gamma, out, rows, L, D, scale, eps, s);
    return launch_rowattn_inst<T, T, 1>(q, k, v, mask, gamma, out, rows, L, D, scale, eps, s);
  }
}

}  // namespace

// =========================================================================
extern "C" {

int mtp_abi_version(void) { return kAbiVersion; }

const char* mtp_last_error(void) { return g_err; }

uint64_t mtp_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

#ifdef MTP_ATTN_TRACE
// profiling builds only: copy the attention kernel's cycle stamps to the host
int mtp_attn_trace_read(unsigned long long* host, int n) {
  MTP_CUDA_TRY(cudaDeviceSynchronize());
  const int cap = (int)(sizeof(attn::g_attn_trace) / sizeof(unsigned long long));
  MTP_CUDA_TRY(cudaMemcpyFromSymbol(host, attn::g_attn_trace, sizeof(unsigned long long) * (n < cap ? n : cap)));
  return MTP_OK;
}
// per-CTA phase stamps, 8 per CTA
int mtp_attn_cta_read(unsigned long long* host, int n) {
  MTP_CUDA_TRY(cudaDeviceSynchronize());
  const int cap = (int)(sizeof(attn::g_attn_cta) / sizeof(unsigned long long));
  MTP_CUDA_TRY(cudaMemcpyFromSymbol(host, attn::g_attn_cta, sizeof(unsigned long long) * (n < cap ? n : cap)));
  return MTP_OK;
}
#endif

int mtp_gemm_test(const void* A, const void* B, int ab_dtype, float* C, int64_t M, int64_t N, int64_t K,
                  int force_simt, void* stream) {
  MTP_NVTX("mtp_gemm_test");
  if (int st = check_dims(M, N, K)) return st;
  if (!valid_dtype(ab_dtype)) return fail(MTP_ERR_DTYPE, "bad dtype");
  if (M == 0 || N == 0) return MTP_OK;
  if (!A || !B || !C) return fail(MTP_ERR_ARG, "null pointer");
  GemmEpilogue ep = store_epilogue(nullptr, nullptr, nullptr, 0, 1.0f, C, MTP_DTYPE_F32, N);
  if (!force_simt && tc_eligible(A, B, ab_dtype, ab_dtype, M, N, K))
    return launch_gemm_tc(A, B, ab_dtype, ab_dtype == MTP_DTYPE_E4M3, M, N, K, ep, as_stream(stream));
  return launch_gemm_simt(A, ab_dtype, B, ab_dtype, M, N, K, ep, as_stream(stream));
}

int mtp_set_gemm_schedule(int mode) {
  if (mode != 0 && mode != 1) return fail(MTP_ERR_ARG, "GEMM schedule %d (expected 0 or 1)", mode);
  g_gemm_schedule.store(mode, std::memory_order_relaxed);
  return MTP_OK;
}

int mtp_gemm_schedule(void) { return g_gemm_schedule.load(std::memory_order_relaxed); }

int mtp_gemm_tile_check(int64_t M, int64_t N, int grid, int64_t* max_tiles) {
  if (M <= 0 || N <= 0 || grid <= 0 || M > INT32_MAX / 2 || N > INT32_MAX / 2)
    return fail(MTP_ERR_ARG, "bad tile-check arguments");
  const int bn = 256;
  const int num_m = (int)((M + tc::kBM - 1) / tc::kBM), num_n = (int)((N + bn - 1) / bn);
  const int64_t num_tiles = (int64_t)num_m * num_n;
  if (num_tiles > (1 << 26)) return fail(MTP_ERR_ARG, "too many tiles to check");
  std::vector<uint8_t> seen((size_t)num_tiles, 0);
  int64_t worst = 0;
  for (int c = 0; c < grid; ++c) {
    int64_t tiles = 0;
    for (int64_t t = c; t < num_tiles; t += grid) {
      int mb, nb;
      tc::tile_coords((int)t, num_m, mb, nb);
      if (mb < 0 || mb >= num_m || nb < 0 || nb >= num_n)
        return fail(MTP_ERR_SHAPE, "CTA %d: tile (%d, %d) outside %d x %d", c, mb, nb, num_m, num_n);
      uint8_t& s = seen[(size_t)nb * num_m + mb];
      if (s) return fail(MTP_ERR_SHAPE, "tile (%d, %d) taken twice", mb, nb);
      s = 1;
      ++tiles;
    }
    worst = tiles > worst ? tiles : worst;
  }
  for (int64_t i = 0; i < num_tiles; ++i)
    if (!seen[(size_t)i]) return fail(MTP_ERR_SHAPE, "tile %lld never taken", (long long)i);
  if (max_tiles) *max_tiles = worst;
  return MTP_OK;
}

int mtp_gemm_tile_plan(int64_t M, int64_t N, int sms, int* bn) {
  if (M <= 0 || N <= 0 || sms <= 0 || !bn) return fail(MTP_ERR_ARG, "bad tile-plan arguments");
  *bn = pick_bn(M, N, sms);
  return MTP_OK;
}

size_t mtp_gemm_streamk_bytes(int64_t M, int64_t N, int64_t K, int ab_dtype) {
  if (M <= 0 || N <= 0 || K <= 0 || !valid_dtype(ab_dtype) || ab_dtype == MTP_DTYPE_F32) return 0;
  int dev;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
  const int eb = ab_dtype == MTP_DTYPE_E4M3 ? 1 : 2;
  const int num_kb = (int)((K * eb + tc::kKBlockBytes - 1) / tc::kKBlockBytes);
  return sk_bytes_needed(sk_plan(M, N, num_kb, sm_count(dev), 0));
}

int mtp_gemm_streamk_plan(int64_t M, int64_t N, int64_t K, int ab_dtype, int sms, int grid, int64_t* info) {
  if (M <= 0 || N <= 0 || K <= 0 || sms <= 0 || !valid_dtype(ab_dtype) || !info)
    return fail(MTP_ERR_ARG, "bad stream-K plan arguments");
  const int eb = ab_dtype == MTP_DTYPE_E4M3 ? 1 : 2;
  const int num_kb = (int)((K * eb + tc::kKBlockBytes - 1) / tc::kKBlockBytes);
  const SkPlan p = sk_plan(M, N, num_kb, sms, grid);
  const int64_t v[9] = {p.use ? 1 : 0, p.bn, p.grid, p.s.dp_rounds, p.s.dp_tiles, p.s.q, p.s.num_tiles,
                        p.s.num_kb, (int64_t)(p.use || grid > 0 ? p.slot_bytes + kSkTail : 0)};
  for (int i = 0; i < 9; ++i) info[i] = v[i];
  return MTP_OK;
}

// Walks every CTA's work items on the host (the kernel's own iterator) and
// checks that each (tile, K block) is computed exactly once, that every
// split tile's parts are numbered 0..parts-1 in K order by consecutive CTAs,
// and that the slot each part writes is the one the summing part reads.
int mtp_gemm_streamk_check(int64_t M, int64_t N, int64_t K, int ab_dtype, int sms, int grid) {
  if (M <= 0 || N <= 0 || K <= 0 || sms <= 0 || !valid_dtype(ab_dtype))
    return fail(MTP_ERR_ARG, "bad stream-K plan arguments");
  const int eb = ab_dtype == MTP_DTYPE_E4M3 ? 1 : 2;
  const int num_kb = (int)((K * eb + tc::kKBlockBytes - 1) / tc::kKBlockBytes);
  // grid < 0: the whole-tile plan the fused vocab-parallel verify falls back to
  const SkPlan p = grid < 0 ? dp_only_plan(M, N, num_kb, sms) : sk_plan(M, N, num_kb, sms, grid);
  if (p.grid <= 0) return fail(MTP_ERR_SHAPE, "no stream-K schedule for these sizes");
  const sk::Sched& sc = p.s;
  const int64_t T = sc.num_tiles;
  if ((int64_t)(T - sc.dp_tiles) * 8 > (int64_t)kSkCounterBytes) return fail(MTP_ERR_SHAPE, "counter overflow");
  std::vector<int> cover((size_t)T * num_kb, 0);
  const int64_t cap = (int64_t)num_kb + 1;  // a tile has at most num_kb + 1 parts
  std::vector<int> slot_of((size_t)((T - sc.dp_tiles) * cap), -1);  // [x][part]
  std::vector<int> slot_used((size_t)2 * p.grid, 0);
  std::vector<int> part_kb0((size_t)((T - sc.dp_tiles) * cap), -1);
  for (int c = 0; c < p.grid; ++c) {
    sk::Iter it;
    it.init(sc, c, p.grid);
    sk::Work w;
    int splits = 0, items = 0;
    while (it.next(sc, w)) {
      if (++items > 1 << 20) return fail(MTP_ERR_SHAPE, "CTA %d: runaway iterator", c);
      if (w.tile < 0 || w.tile >= T || w.kb0 < 0 || w.kb1 > num_kb || w.kb0 >= w.kb1)
        return fail(MTP_ERR_SHAPE, "CTA %d: bad item tile %d kb [%d,%d)", c, w.tile, w.kb0, w.kb1);
      for (int kb = w.kb0; kb < w.kb1; ++kb) ++cover[(size_t)w.tile * num_kb + kb];
      if (!w.split) continue;
      ++splits;
      if (w.x != w.tile - sc.dp_tiles || w.parts < 2 || w.parts > cap || w.part < 0 || w.part >= w.parts)
        return fail(MTP_ERR_SHAPE, "CTA %d: bad split item x %d part %d/%d", c, w.x, w.part, w.parts);
      if (w.slot < 0 || w.slot >= 2 * p.grid || slot_used[w.slot]++)
        return fail(MTP_ERR_SHAPE, "CTA %d: slot %d reused", c, w.slot);
      if (sk::part_slot(sc, w.x, w.part) != w.slot)
        return fail(MTP_ERR_SHAPE, "tile %d part %d: written to slot %d, read from %d", w.tile, w.part, w.slot,
                    sk::part_slot(sc, w.x, w.part));
      const size_t at = (size_t)(w.x * cap + w.part);
      if (slot_of[at] != -1) return fail(MTP_ERR_SHAPE, "tile %d part %d twice", w.tile, w.part);
      slot_of[at] = w.slot;
      part_kb0[at] = w.kb0;
    }
    if (splits > 2) return fail(MTP_ERR_SHAPE, "CTA %d has %d split items", c, splits);
  }
  for (int64_t i = 0; i < T * num_kb; ++i)
    if (cover[i] != 1)
      return fail(MTP_ERR_SHAPE, "tile %lld K block %lld computed %d times", (long long)(i / num_kb),
                  (long long)(i % num_kb), cover[i]);
  for (int64_t x = 0; x < T - sc.dp_tiles; ++x) {
    const int parts = sk::tile_parts(sc, (int)x);
    if (slot_of[(size_t)(x * cap)] == -1) continue;  // whole tile
    for (int q = 0; q < parts; ++q) {
      if (slot_of[(size_t)(x * cap + q)] == -1) return fail(MTP_ERR_SHAPE, "tile %lld part %d missing", (long long)x, q);
      if (q > 0 && part_kb0[(size_t)(x * cap + q)] <= part_kb0[(size_t)(x * cap + q - 1)])
        return fail(MTP_ERR_SHAPE, "tile %lld parts out of K order", (long long)x);
    }
  }
  return MTP_OK;
}

int mtp_gemm_test_streamk(const void* A, const void* B, int ab_dtype, float* C, int64_t M, int64_t N, int64_t K,
                          int grid, void* workspace, size_t workspace_bytes, void* stream) {
  MTP_NVTX("mtp_gemm_test_streamk");
  if (int st = check_dims(M, N, K)) return st;
  if (!valid_dtype(ab_dtype)) return fail(MTP_ERR_DTYPE, "bad dtype");
  if (M == 0 || N == 0) return MTP_OK;
  if (!A || !B || !C || !workspace) return fail(MTP_ERR_ARG, "null pointer");
  if (!tc_eligible(A, B, ab_dtype, ab_dtype, M, N, K)) return fail(MTP_ERR_ALIGN, "operands not eligible");
  int dev;
  if (int st = current_device(&dev)) return st;
  const int g = grid > 0 ? (grid < sm_count(dev) ? grid : sm_count(dev)) : sm_count(dev);
  const int eb = ab_dtype == MTP_DTYPE_E4M3 ? 1 : 2;
  const SkPlan p = sk_plan(M, N, (int)((K * eb + tc::kKBlockBytes - 1) / tc::kKBlockBytes), sm_count(dev), g);
  if (p.grid <= 0) return fail(MTP_ERR_SHAPE, "no stream-K schedule for these sizes");
  if (workspace_bytes < p.slot_bytes + kSkTail)
    return fail(MTP_ERR_WORKSPACE, "workspace of %zu bytes needed", p.slot_bytes + kSkTail);
  GemmEpilogue ep = store_epilogue(nullptr, nullptr, nullptr, 0, 1.0f, C, MTP_DTYPE_F32, N);
  return launch_gemm_tc(A, B, ab_dtype, ab_dtype == MTP_DTYPE_E4M3, M, N, K, ep, as_stream(stream), workspace,
                        workspace_bytes, g);
}

// Test support, host memory only: the device code's own key packing
// (ordered_i32 / make_key / key_index are __host__ __device__).
int mtp_keys_pack_host(const float* values, const uint32_t* index, int64_t* keys, int64_t n) {
  if (n < 0 || (n > 0 && (!values || !index || !keys))) return fail(MTP_ERR_ARG, "bad key arguments");
  for (int64_t i = 0; i < n; ++i) keys[i] = make_key(ordered_i32(values[i]), index[i]);
  return MTP_OK;
}

int mtp_keys_index_host(const int64_t* keys, int32_t* index, int64_t n) {
  if (n < 0 || (n > 0 && (!keys || !index))) return fail(MTP_ERR_ARG, "bad key arguments");
  for (int64_t i = 0; i < n; ++i) index[i] = key_index(keys[i]);
  return MTP_OK;
}

int mtp_device_status(void* stream, int* code_out, int clear) {
  MTP_CUDA_TRY(cudaStreamSynchronize(as_stream(stream)));
  int code = 0;
  MTP_CUDA_TRY(cudaMemcpyFromSymbol(&code, g_dev_error, sizeof(int)));
  if (code_out) *code_out = code;
  if (clear) {
    const int zero = 0;
    MTP_CUDA_TRY(cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(int)));
  }
  return MTP_OK;
}

// ---------------------------------------------------------------- RMSNorm-linear
size_t mtp_rmsnorm_linear_workspace(int64_t M, int64_t K, int has_norm_weight) {
  return align256((size_t)M * 4) + (has_norm_weight ? align256((size_t)M * (size_t)K * 4) : 0);
}

int mtp_rmsnorm_linear(const void* x, int x_dtype, const void* weight, int w_dtype, const void* bias,
                       int bias_dtype, const void* norm_weight, int norm_dtype, void* y, int y_dtype, int64_t M,
                       int64_t N, int64_t K, float eps, float scale, void* workspace, size_t workspace_bytes,
                       void* stream) {
  MTP_NVTX("mtp_rmsnorm_linear");
  if (int st = check_dims(M, N, K)) return st;
  if (!valid_dtype(x_dtype) || !valid_dtype(w_dtype) || !valid_dtype(y_dtype) ||
      x_dtype == MTP_DTYPE_E4M3 || y_dtype == MTP_DTYPE_E4M3)
    return fail(MTP_ERR_DTYPE, "unsupported dtype combination x=%d w=%d y=%d", x_dtype, w_dtype, y_dtype);
  if (M == 0 || N == 0) return MTP_OK;
  if (!x || !weight || !y) return fail(MTP_ERR_ARG, "null tensor pointer");
  const size_t need = mtp_rmsnorm_linear_workspace(M, K, norm_weight != nullptr);
  if (!workspace || workspace_bytes < need)
    return fail(MTP_ERR_WORKSPACE, "workspace of %zu bytes needed", need);
  cudaStream_t s = as_stream(stream);
  float* rstd = static_cast<float*>(workspace);
  const void* a = x;
  if (norm_weight) {
    void* xg = static_cast<uint8_t*>(workspace) + align256((size_t)M * 4);
    if (int st = launch_rownorm(x, x_dtype, norm_weight, norm_dtype, nullptr, M, K, eps, ROW_GAMMA, rstd, xg,
                                x_dtype, s))
      return st;
    a = xg;
  } else {
    if (int st = launch_rownorm(x, x_dtype, nullptr, 0, nullptr, M, K, eps, ROW_RSTD, rstd, nullptr, 0, s))
      return st;
  }
  GemmEpilogue ep = store_epilogue(rstd, nullptr, bias, bias_dtype, scale, y, y_dtype, N);
  const bool tc = x_dtype == w_dtype && x_dtype == y_dtype && tc_eligible(a, weight, x_dtype, w_dtype, M, N, K);
  if (tc)
    return launch_gemm_tc(a, weight, x_dtype, false, M, N, K, ep, s, static_cast<uint8_t*>(workspace) + need,
                          workspace_bytes - need);
  return launch_gemm_simt(a, x_dtype, weight, w_dtype, M, N, K, ep, s);
}

size_t mtp_rmsnorm_linear_fp8_workspace(int64_t M, int64_t K) {
  return align256((size_t)M * 4) + align256((size_t)M * (size_t)K);
}

int mtp_rmsnorm_linear_fp8(const void* x, int x_dtype, const float* x_scale, const void* weight, int w_dtype,
                           const float* wscale, const void* bias, int bias_dtype, void* y, int y_dtype, int64_t M,
                           int64_t N, int64_t K, float eps, void* workspace, size_t workspace_bytes,
                           void* stream) {
  MTP_NVTX("mtp_rmsnorm_linear_fp8");
  if (int st = check_dims(M, N, K)) return st;
  if (!valid_dtype(x_dtype) || !valid_dtype(w_dtype) || !valid_dtype(y_dtype) || y_dtype == MTP_DTYPE_E4M3)
    return fail(MTP_ERR_DTYPE, "unsupported dtype combination x=%d w=%d y=%d", x_dtype, w_dtype, y_dtype);
  if (x_dtype == MTP_DTYPE_E4M3 && !x_scale)
    return fail(MTP_ERR_ARG, "pre-quantised E4M3 activations need x_scale");
  if (M == 0 || N == 0) return MTP_OK;
  if (!x || !weight || !y || !wscale) return fail(MTP_ERR_ARG, "null tensor pointer");
  const size_t need = mtp_rmsnorm_linear_fp8_workspace(M, K);
  if (!workspace || workspace_bytes < need) return fail(MTP_ERR_WORKSPACE, "workspace of %zu bytes needed", need);
  cudaStream_t s = as_stream(stream);
  float* rowf = static_cast<float*>(workspace);
  if (w_dtype != MTP_DTYPE_E4M3) {
    // fp32-valued (or 16-bit) weight: the reference's unquantised semantics
    if (x_dtype == MTP_DTYPE_E4M3) {
      if (int st = launch_rownorm(x, x_dtype, nullptr, 0, x_scale, M, K, eps, ROW_PREQUANT, rowf, nullptr, 0, s))
        return st;
    } else if (int st = launch_rownorm(x, x_dtype, nullptr, 0, nullptr, M, K, eps, ROW_RSTD, rowf, nullptr, 0, s)) {
      return st;
    }
    GemmEpilogue ep = store_epilogue(rowf, wscale, bias, bias_dtype, 1.0f, y, y_dtype, N);
    return launch_gemm_simt(x, x_dtype, weight, w_dtype, M, N, K, ep, s);
  }
  const void* a = x;
  if (x_dtype == MTP_DTYPE_E4M3) {
    if (int st = launch_rownorm(x, x_dtype, nullptr, 0, x_scale, M, K, eps, ROW_PREQUANT, rowf, nullptr, 0, s))
      return st;
  } else {
    void* xq = static_cast<uint8_t*>(workspace) + align256((size_t)M * 4);
    if (int st = launch_rownorm(x, x_dtype, nullptr, 0, nullptr, M, K, eps, ROW_QUANT, rowf, xq, MTP_DTYPE_E4M3, s))
      return st;
    a = xq;
  }
  GemmEpilogue ep = store_epilogue(rowf, wscale, bias, bias_dtype, 1.0f, y, y_dtype, N);
  return launch_gemm(a, MTP_DTYPE_E4M3, weight, MTP_DTYPE_E4M3, M, N, K, ep, s,
                     static_cast<uint8_t*>(workspace) + need, workspace_bytes - need);
}

// ---------------------------------------------------------------- tree attn -> RMSNorm -> linear
size_t mtp_tree_attn_rmsnorm_linear_workspace(int64_t B, int64_t H, int64_t D, int q_dtype, int w_dtype) {
  if (B < 0 || H < 0 || D < 0 || !valid_dtype(q_dtype) || !valid_dtype(w_dtype)) return 0;
  return tarl_base_bytes(B, H, D, q_dtype, w_dtype);
}

int mtp_tree_attn_rmsnorm_linear(const void* q, const void* k, const void* v, int qkv_dtype, const float* mask,
                                 const float* rms_w, const void* proj_w, int w_dtype, const void* proj_bias,
                                 int bias_dtype, const float* wscale, void* out, int64_t B, int64_t H, int64_t L,
                                 int64_t D, int64_t N, float scale, float eps, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  MTP_NVTX("mtp_tree_attn_rmsnorm_linear");
  if (B < 0 || H < 0 || L < 0 || D <= 0 || N < 0) return fail(MTP_ERR_SHAPE, "bad sizes");
  if (D > rowattn::kMaxD) return fail(MTP_ERR_SHAPE, "D=%lld above %d", (long long)D, rowattn::kMaxD);
  if (!valid_dtype(qkv_dtype) || qkv_dtype == MTP_DTYPE_E4M3 || !valid_dtype(w_dtype))
    return fail(MTP_ERR_DTYPE, "unsupported dtype combination q=%d w=%d", qkv_dtype, w_dtype);
  const int64_t rows = B * H;
  if (rows == 0 || N == 0) return MTP_OK;
  if (rows > INT32_MAX || N > 0xFFFFFFFFLL) return fail(MTP_ERR_SHAPE, "size out of range");
  if (!q || !proj_w || !out || (L > 0 && (!k || !v))) return fail(MTP_ERR_ARG, "null tensor pointer");
  const int ao = tarl_operand_dtype(qkv_dtype, w_dtype);
  const int vec_w = qkv_dtype == MTP_DTYPE_F32 ? 4 : 8;
  const bool vec = D % vec_w == 0 && aligned16(q) && aligned16(workspace) &&
                   (L == 0 || (aligned16(k) && aligned16(v)));
  const size_t smem = rowattn::smem_bytes(L, D, vec ? vec_w : 1);
  if (smem > 227 * 1024) return fail(MTP_ERR_SHAPE, "L=%lld, D=%lld need too much shared memory", (long long)L,
                                     (long long)D);
  const size_t need = tarl_base_bytes(B, H, D, qkv_dtype, w_dtype);
  if (!workspace || workspace_bytes < need) return fail(MTP_ERR_WORKSPACE, "workspace of %zu bytes needed", need);
  cudaStream_t s = as_stream(stream);
  void* a = workspace;  // normalised attention output [rows, D] in dtype ao
  const bool out_f32 = ao == MTP_DTYPE_F32;
  int st;
  if (qkv_dtype == MTP_DTYPE_BF16)
    st = launch_rowattn_t<__nv_bfloat16>(vec, out_f32, q, k, v, mask, rms_w, a, rows, L, D, scale, eps, s);
  else if (qkv_dtype == MTP_DTYPE_F16)
    st = launch_rowattn_t<__half>(vec, out_f32, q, k, v, mask, rms_w, a, rows, L, D, scale, eps, s);
  else
    st = launch_rowattn_t<float>(vec, true, q, k, v, mask, rms_w, a, rows, L, D, scale, eps, s);
  if (st) return st;
  GemmEpilogue ep = store_epilogue(nullptr, wscale, proj_bias, bias_dtype, 1.0f, out, qkv_dtype, N);
  return launch_gemm(a, ao, proj_w, w_dtype, rows, N, D, ep, s, static_cast<uint8_t*>(workspace) + need,
                     workspace_bytes - need);
}

// ---------------------------------------------------------------- paged KV write
int mtp_paged_kv_write(void* k_pages, void* v_pages, int dtype, const int32_t* page_table, int64_t table_stride,
                       int64_t num_pages, int64_t page_size, const void* src_k, const void* src_v, int src_dtype,
                       int64_t src_len, const int32_t* node_idx, const int32_t* count, int64_t B, int64_t H,
                       int64_t D, int64_t start, int64_t n, void* stream) {
  MTP_NVTX("mtp_paged_kv_write");
  if (B < 0 || H < 0 || D <= 0 || n < 0 || src_len < 0 || page_size <= 0 || num_pages < 0 || start < 0)
    return fail(MTP_ERR_SHAPE, "bad KV write sizes");
  if (start + n > table_stride) return fail(MTP_ERR_SHAPE, "logical positions [%lld, %lld) beyond the page table",
                                            (long long)start, (long long)(start + n));
  if (!node_idx && n > src_len) return fail(MTP_ERR_SHAPE, "n=%lld rows but the source holds %lld", (long long)n,
                                            (long long)src_len);
  if (!valid_dtype(dtype) || dtype == MTP_DTYPE_E4M3 || !valid_dtype(src_dtype) || src_dtype == MTP_DTYPE_E4M3)
    return fail(MTP_ERR_DTYPE, "unsupported dtypes pool=%d source=%d", dtype, src_dtype);
  const int64_t rows = B * H * n;
  if (rows == 0) return MTP_OK;
  if (!k_pages || !v_pages || !page_table || !src_k || !src_v) return fail(MTP_ERR_ARG, "null tensor pointer");
  if ((rows + 7) / 8 > INT32_MAX) return fail(MTP_ERR_SHAPE, "too many rows");
  KvWriteArgs a{};
  a.k_pages = k_pages;
  a.v_pages = v_pages;
  a.dtype = dtype;
  a.page_table = page_table;
  a.table_stride = table_stride;
  a.num_pages = num_pages;
  a.page_size = page_size;
  a.src_k = src_k;
  a.src_v = src_v;
  a.src_dtype = src_dtype;
  a.src_len = src_len;
  a.node_idx = node_idx;
  a.count = count;
  a.B = B;
  a.H = H;
  a.D = D;
  a.start = start;
  a.n = n;
  const int eb = dtype == MTP_DTYPE_F32 ? 4 : 2;
  a.vec = src_dtype == dtype && (D * eb) % 16 == 0 && aligned16(k_pages) && aligned16(v_pages) &&
          aligned16(src_k) && aligned16(src_v);
  paged_kv_write_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, as_stream(stream)>>>(a);
  MTP_LAUNCH_CHECK();
  return MTP_OK;
}

// ---------------------------------------------------------------- attention
// Single-query kernel for fused_tree_attention / fused_paged_attention: 2 =
// sq_attention_kernel where it applies (default; 16-bit K/V, D a power of two
// in [8, 256], 16-byte-aligned rows, scores and offsets of all L keys in
// shared memory), else 1 = decode_attention_kernel, which takes every shape.
// Measured on B200: paged attention B=16 H=32 L=4096 D=128 0.475 ms against
// 2.75 ms, tree attention L=512 0.044 ms against 0.277 ms.  Initial value
// from MTP_DECODE_KERNEL (1 or 2); mtp_set_decode_kernel changes it.
static std::atomic<int> g_decode_kernel{0};

static int decode_kernel_version() {
  int v = g_decode_kernel.load(std::memory_order_relaxed);
  if (v == 0) {
    const char* e = getenv("MTP_DECODE_KERNEL");
    v = (e && e[0] == '1' && e[1] == 0) ? 1 : 2;
    int expected = 0;
    g_decode_kernel.compare_exchange_strong(expected, v);
    v = g_decode_kernel.load(std::memory_order_relaxed);
  }
  return v;
}

static bool sq_eligible(const AttnArgs& a) {
  if (a.kind != ATTN_CONTIG && a.kind != ATTN_PAGED) return false;
  if (a.T != 1 || a.Hq != a.Hkv || a.kv_custom || !is16bit(a.dtype)) return false;
  if (a.D < 8 || a.D > sq::kMaxD || (a.D & (a.D - 1)) != 0) return false;
  if (a.L > INT32_MAX / 2 || sq::smem_bytes(a.L, a.D) > 227 * 1024) return false;
  const void* k = a.kind == ATTN_PAGED ? a.k_pages : a.k;
  const void* v = a.kind == ATTN_PAGED ? a.v_pages : a.v;
  return aligned16(a.q) && aligned16(a.out) && (a.L == 0 || (aligned16(k) && aligned16(v)));
}

static int launch_sq_attention(const AttnArgs& a, cudaStream_t s) {
  sq::Args g{};
  g.q = a.q;
  g.out = a.out;
  g.B = a.B;
  g.H = a.Hq;
  g.D = a.D;
  g.scale = a.scale;
  g.L = a.L;
  g.paged = a.kind == ATTN_PAGED ? 1 : 0;
  g.k = g.paged ? a.k_pages : a.k;
  g.v = g.paged ? a.v_pages : a.v;
  g.mask = a.mask;
  g.page_table = a.page_table;
  g.table_stride = a.table_stride;
  g.num_pages = a.num_pages;
  g.page_size = a.page_size;
  const size_t smem = sq::smem_bytes(a.L, a.D);
  int dev;
  if (int st = current_device(&dev)) return st;
  static size_t attr[2][kMaxDevices] = {};
  const int which = a.dtype == MTP_DTYPE_BF16 ? 0 : 1;
  if (smem > 48 * 1024 && attr[which][dev] < smem) {
    if (which == 0)
      MTP_CUDA_TRY(cudaFuncSetAttribute(sq::sq_attention_kernel<__nv_bfloat16>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    else
      MTP_CUDA_TRY(cudaFuncSetAttribute(sq::sq_attention_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)smem));
    attr[which][dev] = smem;
  }
  const unsigned rows = (unsigned)(a.B * a.Hq);
  if (which == 0) sq::sq_attention_kernel<__nv_bfloat16><<<rows, sq::kThreads, smem, s>>>(g);
  else sq::sq_attention_kernel<__half><<<rows, sq::kThreads, smem, s>>>(g);
  MTP_LAUNCH_CHECK();
  return MTP_OK;
}

static int launch_decode_attention(const AttnArgs& a, cudaStream_t s) {
  const int64_t rows = a.B * a.T * a.Hq;
  if (rows == 0) return MTP_OK;
  if (rows <= INT32_MAX && decode_kernel_version() == 2 && sq_eligible(a)) return launch_sq_attention(a, s);
  if (a.D > 32 * kAttnMaxDPerLane) return fail(MTP_ERR_SHAPE, "head_dim %lld > 256", (long long)a.D);
  if (rows > INT32_MAX) return fail(MTP_ERR_SHAPE, "too many query rows");
  decode_attention_kernel<<<(unsigned)rows, 128, 0, s>>>(a);
  MTP_LAUNCH_CHECK();
  return MTP_OK;
}

int mtp_tree_attention(const void* q, const void* k, const void* v, const float* mask, void* out, int dtype,
                       int64_t B, int64_t H, int64_t L, int64_t D, float scale, void* stream) {
  MTP_NVTX("mtp_tree_attention");
  if (B < 0 || H < 0 || L < 0 || D <= 0) return fail(MTP_ERR_SHAPE, "bad attention sizes");
  if (!valid_dtype(dtype) || dtype == MTP_DTYPE_E4M3) return fail(MTP_ERR_DTYPE, "unsupported dtype %d", dtype);
  if (B * H == 0) return MTP_OK;
  if (!q || !out || (L > 0 && (!k || !v))) return fail(MTP_ERR_ARG, "null tensor pointer");
  AttnArgs a{};
  a.kind = ATTN_CONTIG;
  a.dtype = dtype;
  a.q = q;
  a.out = out;
  a.B = B;
  a.T = 1;
  a.Hq = H;
  a.Hkv = H;
  a.D = D;
  a.scale = scale;
  a.k = k;
  a.v = v;
  a.mask = mask;
  a.L = L;
  return launch_decode_attention(a, as_stream(stream));
}

int mtp_causal_attention_scaled(const void* q, int q_dtype, const void* k, const void* v, int kv_dtype,
                                const float* kscale, const float* vscale, void* out, int64_t B, int64_t H, int64_t L,
                                int64_t D, float scale, void* stream) {
  MTP_NVTX("mtp_causal_attention_scaled");
  if (B < 0 || H < 0 || L < 0 || D <= 0) return fail(MTP_ERR_SHAPE, "bad attention sizes");
  if (!valid_dtype(q_dtype) || q_dtype == MTP_DTYPE_E4M3 || !valid_dtype(kv_dtype))
    return fail(MTP_ERR_DTYPE, "unsupported dtypes q=%d kv=%d", q_dtype, kv_dtype);
  if (B * H == 0) return MTP_OK;
  if (!q || !out || (L > 0 && (!k || !v))) return fail(MTP_ERR_ARG, "null tensor pointer");
  AttnArgs a{};
  a.kind = ATTN_CONTIG;
  a.dtype = q_dtype;
  a.q = q;
  a.out = out;
  a.B = B;
  a.T = 1;
  a.Hq = H;
  a.Hkv = H;
  a.D = D;
  a.scale = scale;
  a.k = k;
  a.v = v;
  a.mask = nullptr;
  a.L = L;
  a.kv_custom = 1;
  a.kv_dtype = kv_dtype;
  a.kscale = kscale;
  a.vscale = vscale;
  return launch_decode_attention(a, as_stream(stream));
}

int mtp_int4_matmul(const void* x, int x_dtype, const uint8_t* packed, const float* scales, int64_t group, void* y,
                    int y_dtype, int64_t M, int64_t N, int64_t K, void* stream) {
  MTP_NVTX("mtp_int4_matmul");
  if (int st = check_dims(M, N, K)) return st;
  if (K % 2 != 0) return fail(MTP_ERR_SHAPE, "K=%lld must be even (two codes per byte)", (long long)K);
  if (group <= 0) return fail(MTP_ERR_SHAPE, "group must be positive");
  if (!valid_dtype(x_dtype) || x_dtype == MTP_DTYPE_E4M3 || !valid_dtype(y_dtype) || y_dtype == MTP_DTYPE_E4M3)
    return fail(MTP_ERR_DTYPE, "unsupported dtypes x=%d y=%d", x_dtype, y_dtype);
  if (M == 0 || N == 0) return MTP_OK;
  if (!x || !packed || !scales || !y) return fail(MTP_ERR_ARG, "null tensor pointer");
  if (M > 65535LL * w4::kTile || N > INT32_MAX / 2) return fail(MTP_ERR_SHAPE, "size out of range");
  cudaStream_t s = as_stream(stream);
  if (M <= 8 && K % 32 == 0 && aligned16(packed)) {
    const int mr = M == 1 ? 1 : (M == 2 ? 2 : (M <= 4 ? 4 : 8));
    const int rows = w4::gemv_block_rows(mr);
    const unsigned blocks = (unsigned)((N + rows - 1) / rows);
    const int g = (int)group, m = (int)M, n = (int)N, k = (int)K;
    if (mr == 1) w4::int4_gemv_kernel<1><<<blocks, 256, 0, s>>>(x, x_dtype, packed, scales, g, y, y_dtype, m, n, k);
    else if (mr == 2) w4::int4_gemv_kernel<2><<<blocks, 256, 0, s>>>(x, x_dtype, packed, scales, g, y, y_dtype, m, n, k);
    else if (mr == 4) w4::int4_gemv_kernel<4><<<blocks, 256, 0, s>>>(x, x_dtype, packed, scales, g, y, y_dtype, m, n, k);
    else w4::int4_gemv_kernel<8><<<blocks, 256, 0, s>>>(x, x_dtype, packed, scales, g, y, y_dtype, m, n, k);
    MTP_LAUNCH_CHECK();
    return MTP_OK;
  }
  dim3 grid((unsigned)((N + w4::kTile - 1) / w4::kTile), (unsigned)((M + w4::kTile - 1) / w4::kTile));
  w4::int4_matmul_kernel<<<grid, 256, 0, s>>>(x, x_dtype, packed, scales, (int)group, y, y_dtype, (int)M, (int)N,
                                              (int)K);
  MTP_LAUNCH_CHECK();
  return MTP_OK;
}

int mtp_paged_attention(const void* q, const void* k_pages, const void* v_pages, const int32_t* page_table,
                        void* out, int dtype, int64_t B, int64_t H, int64_t L, int64_t D, int64_t num_pages,
                        int64_t page_size, float scale, void* stream) {
  MTP_NVTX("mtp_paged_attention");
  if (B < 0 || H < 0 || L < 0 || D <= 0 || page_size <= 0 || num_pages < 0)
    return fail(MTP_ERR_SHAPE, "bad paged attention sizes");
  if (!valid_dtype(dtype) || dtype == MTP_DTYPE_E4M3) return fail(MTP_ERR_DTYPE, "unsupported dtype %d", dtype);
  if (B * H == 0) return MTP_OK;
  if (!q || !out || (L > 0 && (!k_pages || !v_pages || !page_table))) return fail(MTP_ERR_ARG, "null tensor pointer");
  AttnArgs a{};
  a.kind = ATTN_PAGED;
  a.dtype = dtype;
  a.q = q;
  a.out = out;
  a.B = B;
  a.T = 1;
  a.Hq = H;
  a.Hkv = H;
  a.D = D;
  a.scale = scale;
  a.L = L;
  a.k_pages = k_pages;
  a.v_pages = v_pages;
  a.page_table = page_table;
  a.table_stride = L;
  a.num_pages = num_pages;
  a.page_size = page_size;
  a.ctx_len = L;
  return launch_decode_attention(a, as_stream(stream));
}

}  // extern "C"

namespace {

// Shape plan of the tensor-core tree attention; eligible == false -> CUDA-core kernel.
struct TreePlan {
  bool eligible = false;
  int G = 0, n_tiles = 0, t_per_tile = 0, n_ctx_chunks = 0, n_chunks = 0, splits = 1, chunks_per_split = 0;
  size_t ws_bytes = 256;
};


TreePlan tree_plan(int64_t B, int64_t T, int64_t Hq, int64_t Hkv, int64_t D, int64_t ctx_len, int64_t page_size,
                   int64_t num_pages, int dtype) {
  constexpr int chunk = attn::kChunk;
  TreePlan pl;
  if (!(dtype == MTP_DTYPE_BF16 || dtype == MTP_DTYPE_F16) || D != attn::kD || Hkv <= 0 || Hq % Hkv) return pl;
  const int64_t G = Hq / Hkv;
  if (G <= 0 || 128 % G != 0 || T < 1 || T * G > 256) return pl;  // two 128-row query tiles at most
  if (!(page_size == 8 || page_size == 16 || page_size == 32 || page_size == 64 || page_size == 128) ||
      page_size > chunk)
    return pl;
  if (num_pages * B * Hkv * page_size >= (int64_t)INT32_MAX || B * Hkv >= INT32_MAX / 4 || T > 4096 ||
      ctx_len >= (int64_t)INT32_MAX / 2)
    return pl;
  pl.G = (int)G;
  pl.t_per_tile = (int)(128 / G);
  pl.n_tiles = (int)((T * G + 127) / 128);
  pl.n_ctx_chunks = (int)((ctx_len + chunk - 1) / chunk);
  pl.n_chunks = pl.n_ctx_chunks + (int)((T + chunk - 1) / chunk);
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = sm_count(dev >= 0 && dev < kMaxDevices ? dev : 0);
  const int64_t units = B * Hkv;
  int splits = 1;
  if (units * 4 < (int64_t)sms * 3) {  // fewer units than ~3/4 of the SMs: split the keys
    splits = (int)(sms / (units > 0 ? units : 1));
    if (splits > pl.n_chunks) splits = pl.n_chunks;
    if (splits < 1) splits = 1;
  }
  pl.chunks_per_split = (pl.n_chunks + splits - 1) / splits;
  pl.splits = (pl.n_chunks + pl.chunks_per_split - 1) / pl.chunks_per_split;  // no empty split
  if (pl.splits > 1) {
    const size_t slots = (size_t)units * pl.splits * 256;
    pl.ws_bytes = align256(slots * attn::kD * 4) + align256(slots * 2 * 4);
  }
  pl.eligible = true;
  return pl;
}

int make_map(CUtensorMap* map, const void* base, int dtype, int rank, const uint64_t* dims, const uint64_t* strides,
             const uint32_t* box) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(MTP_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t d[5], s[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i < rank - 1) s[i] = strides[i];
  }
  const CUtensorMapDataType t =
      dtype == MTP_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = enc(map, t, (cuuint32_t)rank, const_cast<void*>(base), d, s, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MTP_ERR_CUDA, "cuTensorMapEncodeTiled (rank %d) failed (%d)", rank, (int)r);
  return MTP_OK;
}

template <typename Kern>
int set_smem_once(Kern kern, int bytes, bool* done, int dev) {
  if (!done[dev]) {
    MTP_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done[dev] = true;
  }
  return MTP_OK;
}

int launch_tree_attention_tc(const TreePlan& pl, const void* q, const void* k_pages, const void* v_pages,
                             const int32_t* page_table, int64_t table_stride, int64_t ctx_len, const void* tree_k,
                             const void* tree_v, const float* tree_mask, void* out, int dtype, int64_t B, int64_t T,
                             int64_t Hq, int64_t Hkv, int64_t num_pages, int64_t page_size, float scale,
                             void* workspace, cudaStream_t s) {
  const int chunk = attn::kChunk;
  const uint64_t D = attn::kD, E = 2;
  CUtensorMap tq, tk, tv, ttk, ttv;
  {
    const uint64_t dims[4] = {D, (uint64_t)Hq, (uint64_t)T, (uint64_t)B};
    const uint64_t str[3] = {D * E, (uint64_t)Hq * D * E, (uint64_t)T * Hq * D * E};
    const uint32_t box[4] = {64, (uint32_t)pl.G, (uint32_t)pl.t_per_tile, 1};
    if (int st = make_map(&tq, q, dtype, 4, dims, str, box)) return st;
  }
  {
    // page pools as [P*B*Hkv*page_size, D]: one (page, b, h) slab = page_size consecutive rows
    const uint64_t rows = (uint64_t)(num_pages > 0 ? num_pages : 1) * B * Hkv * page_size;
    const uint64_t dims[2] = {D, rows};
    const uint64_t str[1] = {D * E};
    const uint32_t box[2] = {64, (uint32_t)page_size};
    const void* kp = k_pages ? k_pages : tree_k;  // ctx_len == 0: never read
    const void* vp = v_pages ? v_pages : tree_v;
    if (int st = make_map(&tk, kp, dtype, 2, dims, str, box)) return st;
    if (int st = make_map(&tv, vp, dtype, 2, dims, str, box)) return st;
  }
  {
    const uint64_t dims[3] = {D, (uint64_t)T, (uint64_t)(B * Hkv)};
    const uint64_t str[2] = {D * E, (uint64_t)T * D * E};
    const uint32_t box[3] = {64, (uint32_t)chunk, 1};
    if (int st = make_map(&ttk, tree_k, dtype, 3, dims, str, box)) return st;
    if (int st = make_map(&ttv, tree_v, dtype, 3, dims, str, box)) return st;
  }
  attn::Params p{};
  p.page_table = page_table;
  p.table_stride = table_stride;
  p.k_pool = static_cast<const uint8_t*>(k_pages);
  p.v_pool = static_cast<const uint8_t*>(v_pages);
  p.tree_mask = tree_mask;
  p.out = out;
  p.B = (int)B;
  p.T = (int)T;
  p.Hq = (int)Hq;
  p.Hkv = (int)Hkv;
  p.G = pl.G;
  p.ps = (int)page_size;
  p.num_pages = (int)num_pages;
  p.ctx_len = (int)ctx_len;
  p.n_ctx_chunks = pl.n_ctx_chunks;
  p.n_chunks = pl.n_chunks;
  p.splits = pl.splits;
  p.chunks_per_split = pl.chunks_per_split;
  p.n_tiles = pl.n_tiles;
  p.t_per_tile = pl.t_per_tile;
  p.out_dtype = dtype;
  p.table_vec = (reinterpret_cast<uintptr_t>(page_table) % 16 == 0) && (table_stride % 4 == 0);
  p.scale_log2 = scale * 1.4426950408889634f;
  if (pl.splits > 1) {
    const size_t slots = (size_t)B * Hkv * pl.splits * 256;
    p.part_o = static_cast<float*>(workspace);
    p.part_ml = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + align256(slots * attn::kD * 4));
  }
  int dev;
  if (int st = current_device(&dev)) return st;
  const int grid = (int)(B * Hkv * pl.splits);
  static bool attr[2][kMaxDevices] = {};
  // setmaxnreg moves registers between warpgroups inside the launch's
  // reservation; with a different reservation an increase could wait forever
  static bool regs_ok[2][kMaxDevices] = {};
  {
    const int di = dtype == MTP_DTYPE_BF16 ? 0 : 1;
    if (!regs_ok[di][dev]) {
      cudaFuncAttributes fa;
      MTP_CUDA_TRY(dtype == MTP_DTYPE_BF16 ? cudaFuncGetAttributes(&fa, attn::tree_attention_tc_kernel<1>)
                                           : cudaFuncGetAttributes(&fa, attn::tree_attention_tc_kernel<0>));
      if (fa.numRegs != attn::kLaunchRegs)
        return fail(MTP_ERR_CUDA, "tree attention kernel reserves %d registers per thread, its register split "
                    "needs %d", fa.numRegs, attn::kLaunchRegs);
      regs_ok[di][dev] = true;
    }
  }
  if (dtype == MTP_DTYPE_BF16) {
    if (int st = set_smem_once(attn::tree_attention_tc_kernel<1>, attn::kSmemBytes, attr[0], dev)) return st;
    attn::tree_attention_tc_kernel<1><<<grid, attn::kThreads, attn::kSmemBytes, s>>>(tq, tk, tv, ttk, ttv, p);
  } else {
    if (int st = set_smem_once(attn::tree_attention_tc_kernel<0>, attn::kSmemBytes, attr[1], dev)) return st;
    attn::tree_attention_tc_kernel<0><<<grid, attn::kThreads, attn::kSmemBytes, s>>>(tq, tk, tv, ttk, ttv, p);
  }
  MTP_LAUNCH_CHECK();
  if (pl.splits > 1) {
    const int64_t warps = B * Hkv * pl.n_tiles * 128;
    attn::attn_merge_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, s>>>(p);
    MTP_LAUNCH_CHECK();
  }
  return MTP_OK;
}

}  // namespace

extern "C" {

int mtp_set_decode_kernel(int version) {
  if (version != 1 && version != 2) return fail(MTP_ERR_ARG, "decode kernel %d (expected 1 or 2)", version);
  g_decode_kernel.store(version, std::memory_order_relaxed);
  return MTP_OK;
}

int mtp_decode_kernel(void) { return decode_kernel_version(); }

size_t mtp_tree_attention_paged_workspace(int64_t B, int64_t T, int64_t Hq, int64_t Hkv, int64_t D,
                                          int64_t ctx_len) {
  // page_size 16 / bf16 give the same plan as every other eligible case of
  // these sizes
  return tree_plan(B, T, Hq, Hkv, D, ctx_len, 16, 1, MTP_DTYPE_BF16).ws_bytes;
}

int mtp_tree_attention_paged(const void* q, const void* k_pages, const void* v_pages, const int32_t* page_table,
                             int64_t table_stride, int64_t ctx_len, const void* tree_k, const void* tree_v,
                             const float* tree_mask, void* out, int dtype, int64_t B, int64_t T, int64_t Hq,
                             int64_t Hkv, int64_t D, int64_t num_pages, int64_t page_size, float scale,
                             void* workspace, size_t workspace_bytes, void* stream) {
  MTP_NVTX("mtp_tree_attention_paged");
  if (B < 0 || T < 0 || Hq <= 0 || Hkv <= 0 || D <= 0 || ctx_len < 0 || page_size <= 0 || num_pages < 0)
    return fail(MTP_ERR_SHAPE, "bad tree attention sizes");
  if (Hq % Hkv != 0) return fail(MTP_ERR_SHAPE, "Hq=%lld not a multiple of Hkv=%lld", (long long)Hq, (long long)Hkv);
  if (table_stride < ctx_len) return fail(MTP_ERR_SHAPE, "page table narrower than ctx_len");
  if (!valid_dtype(dtype) || dtype == MTP_DTYPE_E4M3) return fail(MTP_ERR_DTYPE, "unsupported dtype %d", dtype);
  if (B * T == 0) return MTP_OK;
  if (!q || !out || !tree_k || !tree_v || !tree_mask || (ctx_len > 0 && (!k_pages || !v_pages || !page_table)))
    return fail(MTP_ERR_ARG, "null tensor pointer");
  const TreePlan pl = tree_plan(B, T, Hq, Hkv, D, ctx_len, page_size, num_pages, dtype);
  const bool aligned = aligned16(q) && aligned16(out) && aligned16(tree_k) && aligned16(tree_v) &&
                       (ctx_len == 0 || (aligned16(k_pages) && aligned16(v_pages)));
  if (pl.eligible && aligned && scale > 0.f) {  // the kernel folds a positive scale into exp2
    if (pl.splits > 1 && (!workspace || workspace_bytes < pl.ws_bytes))
      return fail(MTP_ERR_WORKSPACE, "workspace of %zu bytes needed", pl.ws_bytes);
    return launch_tree_attention_tc(pl, q, k_pages, v_pages, page_table, table_stride, ctx_len, tree_k, tree_v,
                                    tree_mask, out, dtype, B, T, Hq, Hkv, num_pages, page_size, scale, workspace,
                                    as_stream(stream));
  }
  AttnArgs a{};
  a.kind = ATTN_TREE_PAGED;
  a.dtype = dtype;
  a.q = q;
  a.out = out;
  a.B = B;
  a.T = T;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.D = D;
  a.scale = scale;
  a.k_pages = k_pages;
  a.v_pages = v_pages;
  a.page_table = page_table;
  a.table_stride = table_stride;
  a.num_pages = num_pages;
  a.page_size = page_size;
  a.ctx_len = ctx_len;
  a.tree_k = tree_k;
  a.tree_v = tree_v;
  a.tree_mask = tree_mask;
  return launch_decode_attention(a, as_stream(stream));
}

// ---------------------------------------------------------------- verify
size_t mtp_verify_workspace(int64_t rows) { return verify_ws_bytes(rows < 0 ? 0 : rows); }

int mtp_keys_fill(int64_t* keys, int64_t n, void* stream) {
  if (n <= 0) return MTP_OK;
  if (!keys) return fail(MTP_ERR_ARG, "null keys");
  keys_fill_kernel<<<(unsigned)((n + 255) / 256), 256, 0, as_stream(stream)>>>(reinterpret_cast<long long*>(keys),
                                                                               n, nullptr);
  MTP_LAUNCH_CHECK();
  return MTP_OK;
}

int mtp_verify_workspace_init(void* workspace, size_t workspace_bytes, void* stream) {
  if (!workspace || workspace_bytes < 256) return fail(MTP_ERR_WORKSPACE, "workspace too small");
  const int64_t rows = (int64_t)((workspace_bytes - 256) / 8);
  long long* keys = static_cast<long long*>(workspace);
  unsigned int* counter = reinterpret_cast<unsigned int*>(static_cast<uint8_t*>(workspace) + workspace_bytes - 256);
  const int64_t n = rows > 0 ? rows : 1;
  keys_fill_kernel<<<(unsigned)((n + 255) / 256), 256, 0, as_stream(stream)>>>(keys, rows, counter);
  MTP_LAUNCH_CHECK();
  return MTP_OK;
}

static int verify_common(const void* hidden, int h_dtype, const void* weight, int w_dtype, const void* bias,
                         int bias_dtype, int64_t rows, int64_t K, int64_t V, void* workspace,
                         size_t workspace_bytes, GemmEpilogue& ep, cudaStream_t s) {
  if (int st = check_dims(rows, V, K)) return st;
  if (V == 0) return fail(MTP_ERR_SHAPE, "empty vocabulary");
  if (!valid_dtype(h_dtype) || !valid_dtype(w_dtype) || h_dtype == MTP_DTYPE_E4M3 || w_dtype == MTP_DTYPE_E4M3)
    return fail(MTP_ERR_DTYPE, "unsupported dtype combination hidden=%d weight=%d", h_dtype, w_dtype);
  if (!hidden || !weight) return fail(MTP_ERR_ARG, "null tensor pointer");
  const size_t need = verify_ws_bytes(rows);
  if (!workspace || workspace_bytes < need) return fail(MTP_ERR_WORKSPACE, "workspace of %zu bytes needed", need);
  ep.mode = EPI_ARGMAX;
  ep.bias = bias;
  ep.bias_dtype = bias_dtype;
  ep.keys = static_cast<long long*>(workspace);
  ep.col_offset = 0;
  // the counter sits in the last 256 bytes of the workspace the caller sized
  ep.counter = reinterpret_cast<unsigned int*>(static_cast<uint8_t*>(workspace) + workspace_bytes - 256);
  // a larger workspace carries a stream-K region between the keys and the ticket
  const size_t keys_bytes = align256((size_t)rows * 8);
  return launch_gemm(hidden, h_dtype, weight, w_dtype, rows, V, K, ep, s, static_cast<uint8_t*>(workspace) + keys_bytes,
                     workspace_bytes - keys_bytes);
}

int mtp_fused_verify(const void* hidden, int h_dtype, const void* weight, int w_dtype, const void* bias,
                     int bias_dtype, const int32_t* draft, int8_t* accept, int32_t* top, int64_t M, int64_t K,
                     int64_t V, void* workspace, size_t workspace_bytes, void* stream) {
  MTP_NVTX("mtp_fused_verify");
  if (M == 0) return MTP_OK;
  if (!draft || !accept || !top) return fail(MTP_ERR_ARG, "null output pointer");
  GemmEpilogue ep{};
  ep.finalize = FIN_SINGLE;
  ep.draft = draft;
  ep.accept = accept;
  ep.tokens = top;
  ep.B = M;
  ep.S = 1;
  return verify_common(hidden, h_dtype, weight, w_dtype, bias, bias_dtype, M, K, V, workspace, workspace_bytes, ep,
                       as_stream(stream));
}

int mtp_fused_multi_verify(const void* hidden, int h_dtype, const void* weight, int w_dtype, const void* bias,
                           int bias_dtype, const int32_t* draft, int8_t* accept, int32_t* accepted_n,
                           int32_t* corrected, int64_t B, int64_t S, int64_t K, int64_t V, void* workspace,
                           size_t workspace_bytes, void* stream) {
  MTP_NVTX("mtp_fused_multi_verify");
  if (B < 0 || S < 1) return fail(MTP_ERR_SHAPE, "expected S >= 1 (S == D + 1), got S=%lld", (long long)S);
  if (B == 0) return MTP_OK;
  if (B > INT64_MAX / S) return fail(MTP_ERR_SHAPE, "B*S overflows (B=%lld S=%lld)", (long long)B, (long long)S);
  if ((S > 1 && (!draft || !accept)) || !accepted_n || !corrected) return fail(MTP_ERR_ARG, "null output pointer");
  GemmEpilogue ep{};
  ep.finalize = FIN_CHAIN;
  ep.draft = draft;
  ep.accept = accept;
  ep.accepted_n = accepted_n;
  ep.tokens = corrected;
  ep.B = B;
  ep.S = S;
  return verify_common(hidden, h_dtype, weight, w_dtype, bias, bias_dtype, B * S, K, V, workspace,
                       workspace_bytes, ep, as_stream(stream));
}

// Same computation as mtp_fused_multi_verify with the library's fixed scratch
// array in place of a caller workspace; allocates nothing.
int mtp_fused_multi_verify_noalloc(const void* hidden, int h_dtype, const void* weight, int w_dtype,
                                   const void* bias, int bias_dtype, const int32_t* draft, int8_t* accept,
                                   int32_t* accepted_n, int32_t* corrected, int64_t B, int64_t S, int64_t K,
                                   int64_t V, void* stream) {
  MTP_NVTX("mtp_fused_multi_verify_noalloc");
  if (B < 0 || S < 1) return fail(MTP_ERR_SHAPE, "expected S >= 1 (S == D + 1), got S=%lld", (long long)S);
  if (B == 0) return MTP_OK;
  if (B > MTP_NOALLOC_MAX_ROWS / S)  // checked before B * S is formed, so it cannot overflow
    return fail(MTP_ERR_SHAPE, "B=%lld S=%lld: B*S exceeds the %d rows of the no-allocation scratch; use "
                "mtp_fused_multi_verify", (long long)B, (long long)S, MTP_NOALLOC_MAX_ROWS);
  const int64_t rows = B * S;
  if (int st = check_dims(rows, V, K)) return st;
  if (V == 0) return fail(MTP_ERR_SHAPE, "empty vocabulary");
  if (!valid_dtype(h_dtype) || !valid_dtype(w_dtype) || h_dtype == MTP_DTYPE_E4M3 || w_dtype == MTP_DTYPE_E4M3)
    return fail(MTP_ERR_DTYPE, "unsupported dtype combination hidden=%d weight=%d", h_dtype, w_dtype);
  if (!hidden || !weight) return fail(MTP_ERR_ARG, "null tensor pointer");
  if ((S > 1 && (!draft || !accept)) || !accepted_n || !corrected) return fail(MTP_ERR_ARG, "null output pointer");
  unsigned char* scratch = nullptr;
  if (int st = noalloc_scratch(&scratch)) return st;
  long long* keys = reinterpret_cast<long long*>(scratch);
  unsigned int* counter = reinterpret_cast<unsigned int*>(scratch + (size_t)MTP_NOALLOC_MAX_ROWS * 8);
  cudaStream_t s = as_stream(stream);
  // the array still holds whatever the previous call left: clear keys and ticket
  keys_fill_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, s>>>(keys, rows, counter);
  MTP_LAUNCH_CHECK();
  GemmEpilogue ep{};
  ep.mode = EPI_ARGMAX;
  ep.bias = bias;
  ep.bias_dtype = bias_dtype;
  ep.keys = keys;
  ep.col_offset = 0;
  ep.counter = counter;
  ep.finalize = FIN_CHAIN;
  ep.draft = draft;
  ep.accept = accept;
  ep.accepted_n = accepted_n;
  ep.tokens = corrected;
  ep.B = B;
  ep.S = S;
  return launch_gemm(hidden, h_dtype, weight, w_dtype, rows, V, K, ep, s);
}

int mtp_verify_shard_keys(const void* hidden, int h_dtype, const void* weight_shard, int w_dtype,
                          const void* bias_shard, int bias_dtype, int64_t* keys, int64_t M, int64_t K,
                          int64_t V_shard, int64_t vocab_offset, void* stream) {
  MTP_NVTX("mtp_verify_shard_keys");
  if (int st = check_dims(M, V_shard, K)) return st;
  if (M == 0 || V_shard == 0) return MTP_OK;
  if (vocab_offset < 0 || vocab_offset + V_shard > 0xFFFFFFFFLL) return fail(MTP_ERR_SHAPE, "vocab offset out of range");
  if (!valid_dtype(h_dtype) || !valid_dtype(w_dtype) || h_dtype == MTP_DTYPE_E4M3 || w_dtype == MTP_DTYPE_E4M3)
    return fail(MTP_ERR_DTYPE, "unsupported dtype combination hidden=%d weight=%d", h_dtype, w_dtype);
  if (!hidden || !weight_shard || !keys) return fail(MTP_ERR_ARG, "null tensor pointer");
  GemmEpilogue ep{};
  ep.mode = EPI_ARGMAX;
  ep.bias = bias_shard;
  ep.bias_dtype = bias_dtype;
  ep.keys = reinterpret_cast<long long*>(keys);
  ep.col_offset = vocab_offset;
  ep.finalize = FIN_NONE;
  return launch_gemm(hidden, h_dtype, weight_shard, w_dtype, M, V_shard, K, ep, as_stream(stream));
}

int mtp_verify_shard_keys_ws(const void* hidden, int h_dtype, const void* weight_shard, int w_dtype,
                             const void* bias_shard, int bias_dtype, int64_t* keys, int64_t M, int64_t K,
                             int64_t V_shard, int64_t vocab_offset, void* workspace, size_t workspace_bytes,
                             void* stream) {
  MTP_NVTX("mtp_verify_shard_keys_ws");
  if (int st = check_dims(M, V_shard, K)) return st;
  if (M == 0 || V_shard == 0) return MTP_OK;
  if (vocab_offset < 0 || vocab_offset + V_shard > 0xFFFFFFFFLL) return fail(MTP_ERR_SHAPE, "vocab offset out of range");
  if (!valid_dtype(h_dtype) || !valid_dtype(w_dtype) || h_dtype == MTP_DTYPE_E4M3 || w_dtype == MTP_DTYPE_E4M3)
    return fail(MTP_ERR_DTYPE, "unsupported dtype combination hidden=%d weight=%d", h_dtype, w_dtype);
  if (!hidden || !weight_shard || !keys) return fail(MTP_ERR_ARG, "null tensor pointer");
  GemmEpilogue ep{};
  ep.mode = EPI_ARGMAX;
  ep.bias = bias_shard;
  ep.bias_dtype = bias_dtype;
  ep.keys = reinterpret_cast<long long*>(keys);
  ep.col_offset = vocab_offset;
  ep.finalize = FIN_NONE;
  return launch_gemm(hidden, h_dtype, weight_shard, w_dtype, M, V_shard, K, ep, as_stream(stream), workspace,
                     workspace ? workspace_bytes : 0);
}

int mtp_verify_step(const int32_t* draft, const int32_t* accepted_n, const int32_t* corrected, int64_t B, int64_t D,
                    int32_t* step_tokens, int64_t ld, int32_t* info, void* stream) {
  MTP_NVTX("mtp_verify_step");
  if (B < 0 || D < 0 || ld < D || D > INT32_MAX) return fail(MTP_ERR_SHAPE, "bad step sizes");
  if (!accepted_n || !info || (B > 0 && !corrected) || (B > 0 && D > 0 && (!draft || !step_tokens)))
    return fail(MTP_ERR_ARG, "null pointer");
  if (B == 0) return MTP_OK;
  verify_step_kernel<<<1, 256, 0, as_stream(stream)>>>(draft, accepted_n, corrected, B, D, step_tokens, ld, info);
  MTP_LAUNCH_CHECK();
  return MTP_OK;
}

size_t mtp_verify_fused_bytes(int64_t rows, int world) {
  if (rows < 0 || world < 1) return 0;
  return align256((size_t)peer_epoch_offset(rows, world) + 8);
}

int mtp_verify_fused_init(void* buf, int64_t rows, int world, void* stream) {
  if (!buf || rows < 0 || world < 1) return fail(MTP_ERR_ARG, "bad fused-exchange buffer");
  cudaStream_t s = as_stream(stream);
  const int64_t n = 2 * rows;
  if (n > 0) {
    keys_fill_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(static_cast<long long*>(buf), n, nullptr);
    MTP_LAUNCH_CHECK();
  }
  const size_t off = (size_t)peer_flags_offset(rows);
  MTP_CUDA_TRY(cudaMemsetAsync(static_cast<uint8_t*>(buf) + off, 0, mtp_verify_fused_bytes(rows, world) - off, s));
  return MTP_OK;
}

int mtp_verify_shard_fused(const void* hidden, int h_dtype, const void* weight_shard, int w_dtype,
                           const void* bias_shard, int bias_dtype, const void* peer_bufs, int rank, int world,
                           const int32_t* draft, int8_t* accept, int32_t* accepted_n, int32_t* corrected, int64_t B,
                           int64_t S, int64_t K, int64_t V_shard, int64_t vocab_offset, void* workspace,
                           size_t workspace_bytes, void* stream) {
  MTP_NVTX("mtp_verify_shard_fused");
  if (B < 0 || S < 1) return fail(MTP_ERR_SHAPE, "expected S >= 1");
  if (world < 1 || rank < 0 || rank >= world) return fail(MTP_ERR_ARG, "rank %d / world %d", rank, world);
  const int64_t rows = B * S;
  if (int st = check_dims(rows, V_shard, K)) return st;
  if (B == 0) return MTP_OK;
  if (V_shard <= 0) return fail(MTP_ERR_SHAPE, "empty vocabulary shard");
  if (vocab_offset < 0 || vocab_offset + V_shard > 0xFFFFFFFFLL) return fail(MTP_ERR_SHAPE, "vocab offset out of range");
  if (!hidden || !weight_shard || !peer_bufs || !accepted_n || !corrected || (S > 1 && (!draft || !accept)))
    return fail(MTP_ERR_ARG, "null pointer");
  if (!tc_eligible(hidden, weight_shard, h_dtype, w_dtype, rows, V_shard, K) || h_dtype == MTP_DTYPE_E4M3)
    return fail(MTP_ERR_DTYPE, "the fused exchange runs on the tensor-core path (equal 16-bit dtypes, 16-byte rows)");
  if (!workspace || workspace_bytes < 256) return fail(MTP_ERR_WORKSPACE, "workspace of 256 bytes needed");
  int dev;
  if (int st = current_device(&dev)) return st;
  cudaStream_t s = as_stream(stream);
  GemmEpilogue ep{};
  ep.mode = EPI_ARGMAX;
  ep.bias = bias_shard;
  ep.bias_dtype = bias_dtype;
  ep.col_offset = vocab_offset;
  ep.finalize = FIN_CHAIN_PEERS;
  ep.counter = reinterpret_cast<unsigned int*>(static_cast<uint8_t*>(workspace) + workspace_bytes - 256);
  ep.draft = draft;
  ep.accept = accept;
  ep.accepted_n = accepted_n;
  ep.tokens = corrected;
  ep.B = B;
  ep.S = S;
  ep.peers = static_cast<const unsigned long long*>(peer_bufs);
  ep.rank = rank;
  ep.world = world;
  ep.peer_rows = rows;
  const int num_kb = (int)((K * 2 + tc::kKBlockBytes - 1) / tc::kKBlockBytes);
  SkPlan pl = sk_plan(rows, V_shard, num_kb, sm_count(dev), 0);
  uint8_t* base = static_cast<uint8_t*>(workspace);
  if (!(g_gemm_schedule.load(std::memory_order_relaxed) == 1 && pl.use &&
        workspace_bytes >= sk_bytes_needed(pl)))
    pl = dp_only_plan(rows, V_shard, num_kb, sm_count(dev));
  if (!pl.use) return fail(MTP_ERR_SHAPE, "no schedule for these sizes");
  const size_t tail = workspace_bytes >= kSkTail ? kSkTail : 256;
  return launch_sk_plan(hidden, weight_shard, h_dtype, false, rows, V_shard, K, ep, s, pl,
                        reinterpret_cast<float*>(base),
                        reinterpret_cast<unsigned long long*>(base + workspace_bytes - tail));
}

size_t mtp_verify_exchange_bytes(int64_t rows, int world) {
  if (rows < 0 || world < 1) return 0;
  return (size_t)2 * world * rows * 8 + (size_t)2 * world * 8;
}

int mtp_verify_exchange_chain(int64_t* keys, const void* peer_bufs, int rank, int world, uint64_t* epoch,
                              const int32_t* draft, int8_t* accept, int32_t* accepted_n, int32_t* corrected,
                              int64_t B, int64_t S, void* stream) {
  MTP_NVTX("mtp_verify_exchange_chain");
  if (B < 0 || S < 1) return fail(MTP_ERR_SHAPE, "expected S >= 1");
  if (world < 1 || rank < 0 || rank >= world) return fail(MTP_ERR_ARG, "rank %d / world %d", rank, world);
  if (B == 0) return MTP_OK;
  if (!keys || !peer_bufs || !epoch || (S > 1 && (!draft || !accept)) || !accepted_n || !corrected)
    return fail(MTP_ERR_ARG, "null pointer");
  GemmEpilogue ep{};
  ep.mode = EPI_ARGMAX;
  ep.finalize = FIN_CHAIN;
  ep.draft = draft;
  ep.accept = accept;
  ep.accepted_n = accepted_n;
  ep.tokens = corrected;
  ep.B = B;
  ep.S = S;
  verify_exchange_chain_kernel<<<1, 256, 0, as_stream(stream)>>>(
      reinterpret_cast<long long*>(keys), static_cast<const unsigned long long*>(peer_bufs), rank, world,
      reinterpret_cast<unsigned long long*>(epoch), ep);
  MTP_LAUNCH_CHECK();
  return MTP_OK;
}

int mtp_verify_chain_from_keys(int64_t* keys, const int32_t* draft, int8_t* accept, int32_t* accepted_n,
                               int32_t* corrected, int64_t B, int64_t S, void* stream) {
  MTP_NVTX("mtp_verify_chain_from_keys");
  if (B < 0 || S < 1) return fail(MTP_ERR_SHAPE, "expected S >= 1");
  if (B == 0) return MTP_OK;
  if (!keys || (S > 1 && (!draft || !accept)) || !accepted_n || !corrected) return fail(MTP_ERR_ARG, "null pointer");
  GemmEpilogue ep{};
  ep.mode = EPI_ARGMAX;
  ep.keys = reinterpret_cast<long long*>(keys);
  ep.finalize = FIN_CHAIN;
  ep.draft = draft;
  ep.accept = accept;
  ep.accepted_n = accepted_n;
  ep.tokens = corrected;
  ep.B = B;
  ep.S = S;
  const unsigned blocks = (unsigned)((B + 127) / 128);
  verify_finalize_kernel<<<blocks, 128, 0, as_stream(stream)>>>(ep);
  MTP_LAUNCH_CHECK();
  return MTP_OK;
}

// ---- NCCL communicator for C hosts ------------------------------------------

#define MTP_NCCL_TRY(expr)                                                                        \
  do {                                                                                            \
    ncclResult_t r_ = (expr);                                                                     \
    if (r_ != ncclSuccess) return fail(MTP_ERR_NCCL, "%s: %s", #expr, nccl::error_string(r_));   \
  } while (0)

static int nccl_loaded() {
  const nccl::Api& a = nccl::api();
  return a.ok ? MTP_OK : fail(MTP_ERR_NCCL, "%s", a.why);
}

int mtp_nccl_version(int* version) {
  if (!version) return fail(MTP_ERR_ARG, "null version");
  if (int st = nccl_loaded()) return st;
  *version = nccl::api().version;
  return MTP_OK;
}

int mtp_nccl_unique_id(void* id) {
  if (!id) return fail(MTP_ERR_ARG, "null id");
  if (int st = nccl_loaded()) return st;
  ncclUniqueId u;
  MTP_NCCL_TRY(nccl::api().GetUniqueId(&u));
  memcpy(id, &u, sizeof(u));
  return MTP_OK;
}

int mtp_nccl_comm_init(void** comm, const void* id, int rank, int world) {
  if (!comm || !id) return fail(MTP_ERR_ARG, "null comm or id");
  *comm = nullptr;
  if (world < 1 || rank < 0 || rank >= world) return fail(MTP_ERR_ARG, "rank %d of world %d", rank, world);
  if (int st = nccl_loaded()) return st;
  int dev;
  if (int st = current_device(&dev)) return st;
  ncclUniqueId u;
  memcpy(&u, id, sizeof(u));
  ncclComm_t c = nullptr;
  MTP_NCCL_TRY(nccl::api().CommInitRank(&c, world, u, rank));
  nccl::Comm* h = new (std::nothrow) nccl::Comm;
  if (!h) {
    nccl::api().CommDestroy(c);
    return fail(MTP_ERR_ARG, "out of host memory");
  }
  h->comm = c;
  h->rank = rank;
  h->world = world;
  h->device = dev;
  *comm = h;
  return MTP_OK;
}

int mtp_nccl_comm_destroy(void* comm) {
  if (!comm) return MTP_OK;
  nccl::Comm* h = static_cast<nccl::Comm*>(comm);
  if (int st = nccl_loaded()) return st;
  const ncclResult_t r = nccl::api().CommDestroy(h->comm);
  delete h;
  return r == ncclSuccess ? MTP_OK : fail(MTP_ERR_NCCL, "ncclCommDestroy: %s", nccl::error_string(r));
}

int mtp_nccl_comm_abort(void* comm) {
  if (!comm) return MTP_OK;
  nccl::Comm* h = static_cast<nccl::Comm*>(comm);
  if (int st = nccl_loaded()) return st;
  const ncclResult_t r = nccl::api().CommAbort(h->comm);  // frees the NCCL communicator
  delete h;
  return r == ncclSuccess ? MTP_OK : fail(MTP_ERR_NCCL, "ncclCommAbort: %s", nccl::error_string(r));
}

int mtp_nccl_comm_status(void* comm) {
  if (!comm) return fail(MTP_ERR_ARG, "null comm");
  if (int st = nccl_loaded()) return st;
  ncclResult_t async = ncclSuccess;
  MTP_NCCL_TRY(nccl::api().CommGetAsyncError(static_cast<nccl::Comm*>(comm)->comm, &async));
  return async == ncclSuccess ? MTP_OK : fail(MTP_ERR_NCCL, "NCCL: %s", nccl::error_string(async));
}

size_t mtp_vocab_parallel_workspace(int64_t B, int64_t S, int64_t V_shard, int64_t K, int h_dtype) {
  if (B < 0 || S < 1 || V_shard < 0 || K < 0) return 0;
  const int64_t rows = B * S;
  const size_t keys = align256((size_t)(rows > 0 ? rows : 1) * 8);
  return keys + (rows > 0 && V_shard > 0 && K > 0 ? mtp_gemm_streamk_bytes(rows, V_shard, K, h_dtype) : 0);
}

int mtp_vocab_parallel_multi_verify(const void* hidden, int h_dtype, const void* weight_shard, int w_dtype,
                                    const void* bias_shard, int bias_dtype, const int32_t* draft,
                                    int8_t* accept, int32_t* accepted_n, int32_t* corrected, int64_t B,
                                    int64_t S, int64_t K, int64_t V_shard, int64_t vocab_offset, void* comm,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  MTP_NVTX("mtp_vocab_parallel_multi_verify");
  if (B < 0 || S < 1 || K < 0 || V_shard < 0) return fail(MTP_ERR_SHAPE, "bad verify sizes");
  if (B == 0) return MTP_OK;
  const int64_t rows = B * S;
  const size_t keys_bytes = align256((size_t)rows * 8);
  if (!workspace || workspace_bytes < keys_bytes)
    return fail(MTP_ERR_WORKSPACE, "workspace of %zu bytes needed", keys_bytes);
  if (!aligned16(workspace)) return fail(MTP_ERR_ALIGN, "workspace not 16-byte aligned");
  const nccl::Comm* c = static_cast<const nccl::Comm*>(comm);
  if (c) {
    if (int st = nccl_loaded()) return st;
    int dev;
    if (int st = current_device(&dev)) return st;
    if (dev != c->device) return fail(MTP_ERR_ARG, "current device %d, communicator on device %d", dev, c->device);
  }
  int64_t* keys = static_cast<int64_t*>(workspace);
  cudaStream_t s = as_stream(stream);
  // an empty block contributes no key: its rank's keys stay at INT64_MIN
  if (V_shard > 0) {
    if (int st = mtp_verify_shard_keys_ws(hidden, h_dtype, weight_shard, w_dtype, bias_shard, bias_dtype, keys,
                                          rows, K, V_shard, vocab_offset, static_cast<uint8_t*>(workspace) + keys_bytes,
                                          workspace_bytes - keys_bytes, stream))
      return st;
  }
  // with a communicator the collective always runs (a one-rank communicator reduces locally)
  if (c) MTP_NCCL_TRY(nccl::api().AllReduce(keys, keys, (size_t)rows, ncclInt64, ncclMax, c->comm, s));
  return mtp_verify_chain_from_keys(keys, draft, accept, accepted_n, corrected, B, S, stream);
}

}  // extern "C"
