/*
 * mtp_b200.h -- C ABI of the B200-native (sm_100a) tree-verification hot path.
 *
 * Every entry point replaces one operator of Dahacker444/mtp-engine's Python
 * API (the citation beside each declaration is the reference function it
 * replaces, file:line within that project).  Conventions:
 *
 *   - plain device pointers, element counts and dtype codes; no torch types;
 *   - every tensor is dense and row-major (the reference's wrappers call
 *     .contiguous() before launching, e.g. mtp_kernels.py:945-946);
 *   - outputs and workspaces are allocated by the caller (the reference
 *     allocates outputs with torch.empty, mtp_kernels.py:960); the library
 *     never calls cudaMalloc, so calls are safe inside CUDA-graph capture;
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default);
 *     nothing synchronises the host except mtp_device_status();
 *   - the return value is an MTP_* status; mtp_last_error() gives a
 *     thread-local message for the last non-zero status.
 *
 * Page ids index the pool the way the reference's torch indexing does: an id
 * in [-num_pages, num_pages) is valid and a negative one counts from the end
 * (the -1 that PagedKVCache leaves in unreserved columns reads page
 * num_pages - 1, mtp_engine.py:550-552, 582-586; mtp_kernels.py:839-848).
 *
 * Device-side checks (page ids outside [-num_pages, num_pages),
 * bounded waits that ran out) are recorded in a per-device error word that
 * mtp_device_status() reads.
 */
#ifndef MTP_B200_H
#define MTP_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes */
#define MTP_DTYPE_F32 0
#define MTP_DTYPE_BF16 1
#define MTP_DTYPE_F16 2
#define MTP_DTYPE_E4M3 3 /* float8_e4m3fn */

/* status codes */
#define MTP_OK 0
#define MTP_ERR_SHAPE 1       /* inconsistent or unsupported sizes */
#define MTP_ERR_DTYPE 2       /* dtype combination not supported */
#define MTP_ERR_ALIGN 3       /* pointer alignment violated */
#define MTP_ERR_CUDA 4        /* a CUDA runtime call failed */
#define MTP_ERR_TIMEOUT 5     /* a bounded device wait ran out */
#define MTP_ERR_WORKSPACE 6   /* workspace missing or too small */
#define MTP_ERR_DEVICE 7      /* a device-side check failed */
#define MTP_ERR_ARG 8         /* null pointer or bad scalar argument */
#define MTP_ERR_NCCL 9        /* NCCL missing, or an NCCL call failed */

/* ABI version of this header (bumped on any signature change). */
int mtp_abi_version(void);

/* Thread-local description of the last failing call on this thread (the
 * reference raises AssertionError from its wrappers instead, e.g.
 * mtp_kernels.py:949; the Python layer here raises from this text). */
const char* mtp_last_error(void);

/* Synchronises `stream`, then reports the current device's error word
 * (0 = clean, else an MTP_ERR_* code recorded by a kernel) in *code_out.
 * clear != 0 resets the word.  Returns MTP_OK or MTP_ERR_CUDA.
 *
 * After MTP_ERR_TIMEOUT (a bounded wait ran out; the call's outputs are
 * undefined):
 *   - single-device verify calls (mtp_fused_verify, mtp_fused_multi_verify,
 *     mtp_verify_shard_keys*, mtp_fused_multi_verify_noalloc) still leave
 *     their keys and ticket at rest, so the next call on the same workspace
 *     runs normally; a workspace with GEMM schedule 1 (stream-K) room must
 *     be filled again with mtp_keys_fill;
 *   - the peer-memory exchanges (mtp_verify_exchange_chain,
 *     mtp_verify_shard_fused) must be rebuilt on EVERY rank, not only on the
 *     one that saw the timeout: synchronise all ranks, zero the exchange
 *     buffers and epoch counters (mtp_verify_fused_init for the fused
 *     form), then resume -- a rank that gave up is one call out of step
 *     with its peers. */
int mtp_device_status(void* stream, int* code_out, int clear);

/* ------------------------------------------------------------------------- */
/* GEMM schedule (no counterpart in the reference, whose Triton kernels use  */
/* one program per output tile)                                              */
/* ------------------------------------------------------------------------- */

/* Process-wide schedule of the tensor-core GEMM inside mtp_rmsnorm_linear,
 * mtp_rmsnorm_linear_fp8, mtp_fused_verify and mtp_fused_multi_verify:
 * 0 (default) = whole output tiles per CTA; 1 = stream-K, where the tiles
 * of the last, part-empty round are cut along K between CTAs and their fp32
 * partials summed in K order by the part that finishes last (deterministic,
 * not bit-identical to schedule 0).  Schedule 1 applies only to calls whose
 * workspace has room for it (mtp_gemm_streamk_bytes) and where it is
 * estimated to be faster; other calls run schedule 0.  Returns MTP_ERR_ARG
 * for other modes.
 *
 * Under schedule 0 the verify calls with 16-bit operands and at most 512
 * logit rows (B*S) run the vocabulary-tiled kernel: pairs of CTAs (thread-
 * block clusters of 2) each take 256 vocabulary rows against every logit
 * row, so the weight streams from HBM exactly once; the environment
 * variable MTP_VERIFY_VT=0 selects the row-tiled kernel instead.  Both give
 * identical outputs. */
int mtp_set_gemm_schedule(int mode);
int mtp_gemm_schedule(void);

/* Test support, host only: the tile width *bn of the tensor-core GEMM of
 * C[M,N] on `sms` SMs (tiles are 128 rows x *bn columns). */
int mtp_gemm_tile_plan(int64_t M, int64_t N, int sms, int* bn);

/* Test support, host only: walks the tensor-core GEMM's tile order (128 x
 * 256 tiles, M fastest) for every CTA of a `grid`-CTA launch and checks that
 * each tile is taken exactly once.  *max_tiles (may be NULL) receives the
 * most tiles any one CTA takes.  MTP_OK or MTP_ERR_SHAPE (message in
 * mtp_last_error). */
int mtp_gemm_tile_check(int64_t M, int64_t N, int grid, int64_t* max_tiles);

/* Process-wide choice of the single-query kernel behind mtp_tree_attention
 * and mtp_paged_attention: 2 (default) = 16-byte loads with several keys in
 * flight per lane and P V split over key groups, for 16-bit K/V with a
 * power-of-two head size up to 256 (other shapes run kernel 1); 1 = one
 * warp per key with scalar loads, every shape.  MTP_DECODE_KERNEL=1 sets the
 * initial value.  Returns MTP_ERR_ARG for other values. */
int mtp_set_decode_kernel(int version);
int mtp_decode_kernel(void);

/* Extra workspace bytes that let a GEMM of C[M,N] = A[M,K] B[N,K]^T
 * (ab_dtype: 16-bit or E4M3) run stream-K on the current device; 0 when it
 * would not.  Add it to the operator's own workspace size.  The stream-K
 * counters sit in the 16 KB that end 256 bytes before the end of the
 * workspace and rest at INT64_MIN: fill a new workspace once with
 * mtp_keys_fill over all of it (mtp_verify_workspace_init does this for
 * verify workspaces); every call leaves them at rest.  After a call fails
 * with MTP_ERR_TIMEOUT, fill the workspace again. */
size_t mtp_gemm_streamk_bytes(int64_t M, int64_t N, int64_t K, int ab_dtype);

/* The counters and the final 256 bytes: a workspace that is reused for
 * calls of other sizes under schedule 1 keeps at least this many bytes after
 * the operator's own part, so no call writes over the counters. */
#define MTP_STREAMK_TAIL_BYTES 16640

/* Test support: the stream-K plan for `sms` SMs (grid > 0 forces the
 * schedule on that many CTAs).  info[9] = {used, BN, grid, dp_rounds,
 * dp_tiles, q (K blocks per CTA in the stream-K phase), tiles, K blocks per
 * tile, workspace bytes}. */
int mtp_gemm_streamk_plan(int64_t M, int64_t N, int64_t K, int ab_dtype, int sms, int grid, int64_t* info);

/* Test support, host only: walks the kernel's work iterator for every CTA of
 * that plan and checks that each (tile, K block) is computed once and that
 * split tiles' parts and slots agree.  grid < 0 checks the whole-tile plan
 * of the same kernel instead.  MTP_OK or MTP_ERR_SHAPE (message in
 * mtp_last_error). */
int mtp_gemm_streamk_check(int64_t M, int64_t N, int64_t K, int ab_dtype, int sms, int grid);

/* Test support: C[M,N] (fp32) = A[M,K] @ B[N,K]^T through the stream-K
 * kernel on `grid` CTAs (<= 0: one per SM), whatever the schedule setting.
 * workspace: info[8] bytes of mtp_gemm_streamk_plan, filled once with
 * INT64_MIN. */
int mtp_gemm_test_streamk(const void* A, const void* B, int ab_dtype, float* C, int64_t M, int64_t N, int64_t K,
                          int grid, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------- */
/* RMSNorm -> linear                                                          */
/* ------------------------------------------------------------------------- */

/* Bytes of workspace mtp_rmsnorm_linear needs for these sizes. */
size_t mtp_rmsnorm_linear_workspace(int64_t M, int64_t K, int has_norm_weight);

/* y[M,N] = ((rmsnorm(x) * norm_weight) @ W^T + bias) * scale.
 * Replaces fused_rmsnorm_linear, mtp_kernels.py:936-977 (eager reference
 * _eager_rmsnorm_linear, mtp_kernels.py:778-787).  norm_weight (the RMSNorm
 * gamma, [K]) may be NULL, which is the reference's signature; bias may be
 * NULL.  x/W/y dtypes: bf16 or f16 with x, W and y all equal runs on the
 * tcgen05 tensor cores (fp32 accumulation); any mix involving f32 runs the
 * fp32 CUDA-core kernel (IEEE fp32 throughout, like the reference). */
int mtp_rmsnorm_linear(const void* x, int x_dtype, const void* weight, int w_dtype,
                       const void* bias, int bias_dtype, const void* norm_weight, int norm_dtype,
                       void* y, int y_dtype, int64_t M, int64_t N, int64_t K, float eps,
                       float scale, void* workspace, size_t workspace_bytes, void* stream);

/* Bytes of workspace mtp_rmsnorm_linear_fp8 needs for these sizes
 * (caller-provided scratch; the reference allocates inside the call). */
size_t mtp_rmsnorm_linear_fp8_workspace(int64_t M, int64_t K);

/* y[M,N] = rmsnorm(x) @ (W * wscale[:,None])^T + bias.
 * Replaces fused_rmsnorm_linear_fp8, mtp_kernels.py:1014-1044 (eager
 * reference _eager_rmsnorm_linear_fp8, mtp_kernels.py:804-814).  wscale is
 * the fp32 per-output-channel scale, typically a slice of the flat buffer
 * of pack_scales (mtp_kernels.py:1336-1353), i.e. flat + offsets[idx].
 * With an E4M3 weight the activations are quantised per token
 * (sx = amax_row / 448) and the product runs on the tensor cores
 * (kind::f8f6f4); rstd is computed from the dequantised activations, so the
 * result equals the reference evaluated on those dequantised activations.
 * x may also be passed pre-quantised (x_dtype = E4M3, x_scale = sx[M]).
 * A non-E4M3 weight (the reference's own fp32-valued self-check weight,
 * mtp_engine.py:1792-1800) runs unquantised in fp32. */
int mtp_rmsnorm_linear_fp8(const void* x, int x_dtype, const float* x_scale,
                           const void* weight, int w_dtype, const float* wscale,
                           const void* bias, int bias_dtype, void* y, int y_dtype,
                           int64_t M, int64_t N, int64_t K, float eps,
                           void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------- */
/* attention                                                                  */
/* ------------------------------------------------------------------------- */

/* out[B,H,D] = softmax(q k^T * scale, keys with mask[j] <= 0.5 dropped) v.
 * Replaces fused_tree_attention, mtp_kernels.py:1165-1191 (eager
 * _eager_tree_attention, 859-872).  k, v: [B,H,L,D]; mask: [L] float32
 * shared by every (b,h).  dtype applies to q, k, v and out. */
int mtp_tree_attention(const void* q, const void* k, const void* v, const float* mask, void* out,
                       int dtype, int64_t B, int64_t H, int64_t L, int64_t D, float scale,
                       void* stream);

/* Single-query attention per (b, h) over L contiguous keys, no mask, with K
 * and V in kv_dtype (any, e.g. E4M3) scaled per head: k * kscale[h],
 * v * vscale[h] (NULL = 1).  Replaces fused_causal_attention_fp8,
 * mtp_kernels.py:1105-1133 (eager _eager_causal_attention_fp8, 817-830),
 * and with kv_dtype = q_dtype and NULL scales fused_causal_attention,
 * 980-1006 (eager 790-802).  q/out [B,H,D] in q_dtype, k/v [B,H,L,D],
 * D <= 256. */
int mtp_causal_attention_scaled(const void* q, int q_dtype, const void* k, const void* v, int kv_dtype,
                                const float* kscale, const float* vscale, void* out, int64_t B, int64_t H, int64_t L,
                                int64_t D, float scale, void* stream);

/* y[M,N] = x[M,K] @ dequant(packed, scales)^T with 4-bit weights packed two
 * per byte along K (low nibble first) and decoded as (code - 8) *
 * scales[n, k / group].  Replaces fused_int4_matmul, mtp_kernels.py:1194-1219
 * (eager _eager_int4_matmul 875-878 over dequantize_int4 754-767).  packed
 * [N, K/2] uint8, scales [N, ceil(K/group)] f32, K even; fp32 products and
 * sums (the reference's fp32 dot). */
int mtp_int4_matmul(const void* x, int x_dtype, const uint8_t* packed, const float* scales, int64_t group, void* y,
                    int y_dtype, int64_t M, int64_t N, int64_t K, void* stream);

/* Single-query attention over a page pool with a per-token page table.
 * Replaces fused_paged_attention, mtp_kernels.py:1136-1162 (eager
 * _eager_paged_attention, 832-856).  k_pages/v_pages:
 * [num_pages, B, H, page_size, D] (PagedKVCache layout, mtp_engine.py:542-549);
 * page_table: [B, L] int32, token t of sequence b at
 * pages[page_table[b,t], b, h, t % page_size] (per token; any table). */
int mtp_paged_attention(const void* q, const void* k_pages, const void* v_pages,
                        const int32_t* page_table, void* out, int dtype, int64_t B, int64_t H,
                        int64_t L, int64_t D, int64_t num_pages, int64_t page_size, float scale,
                        void* stream);

/* Bytes of workspace mtp_tree_attention_paged needs (caller-provided
 * scratch for split keys; no counterpart in the reference). */
size_t mtp_tree_attention_paged_workspace(int64_t B, int64_t T, int64_t Hq, int64_t Hkv,
                                          int64_t D, int64_t ctx_len);

/* Paged tree attention with GQA (the composite of fused_paged_attention and
 * fused_tree_attention, mtp_kernels.py:1136-1191; it has no single
 * counterpart in the reference).  For tree node n and query head h
 * (kv head h / (Hq/Hkv)) the keys are the ctx_len context tokens of
 * sequence b (paged, as in mtp_paged_attention; page_table row stride
 * `table_stride` >= ctx_len) followed by the tree nodes m with
 * tree_mask[n,m] > 0.5 (SpeculativeDraftTree.tree_mask,
 * mtp_engine.py:671-680).  q/out: [B,T,Hq,D]; tree_k/tree_v: [B,Hkv,T,D];
 * tree_mask: [T,T] float32.  Any per-token page table is taken: 128-key
 * chunks whose tokens fill whole pages are loaded page by page, others
 * (tables that PagedKVCache.reserve built from token counts that are not
 * multiples of page_size, or that swap_logical_pages rearranged,
 * mtp_engine.py:567-593) token by token. */
int mtp_tree_attention_paged(const void* q, const void* k_pages, const void* v_pages,
                             const int32_t* page_table, int64_t table_stride, int64_t ctx_len,
                             const void* tree_k, const void* tree_v, const float* tree_mask,
                             void* out, int dtype, int64_t B, int64_t T, int64_t Hq, int64_t Hkv,
                             int64_t D, int64_t num_pages, int64_t page_size, float scale,
                             void* workspace, size_t workspace_bytes, void* stream);

/* Bytes of workspace mtp_tree_attn_rmsnorm_linear needs (the normalised
 * attention output, [B*H, D] in the GEMM operand dtype).  Under GEMM
 * schedule 1 add mtp_gemm_streamk_bytes(B*H, N, D, operand dtype), where the
 * operand dtype is q's when proj_w has q's 16-bit dtype, else f32. */
size_t mtp_tree_attn_rmsnorm_linear_workspace(int64_t B, int64_t H, int64_t D, int q_dtype, int w_dtype);

/* out[b,h,:] = rmsnorm(attn[b,h,:]) * rms_w @ (proj_w * wscale[:,None])^T + proj_bias,
 * attn = single-query tree attention of q[b,h] over k/v[b,h,0:L] under the
 * shared mask[L] (key j kept iff mask[j] > 0.5).  Replaces
 * fused_tree_attn_rmsnorm_linear, mtp_kernels.py:1222-1250 (which runs the
 * eager _eager_tree_attn_rmsnorm_linear, 881-905).  q [B,H,D], k/v
 * [B,H,L,D] (qkv_dtype), mask [L] f32 (NULL keeps every key), rms_w [D] f32
 * or NULL (ones), proj_w [N,D] (any dtype), proj_bias [N] or NULL, wscale
 * [N] f32 or NULL, out [B,H,N] in qkv_dtype.  D <= 8192.  The attention and
 * RMSNorm run on CUDA cores (HBM-bound); the projection is the GEMM of
 * mtp_rmsnorm_linear (tensor cores when proj_w and q share a 16-bit dtype).
 * A row with every key masked is NaN, as in the reference. */
int mtp_tree_attn_rmsnorm_linear(const void* q, const void* k, const void* v, int qkv_dtype, const float* mask,
                                 const float* rms_w, const void* proj_w, int w_dtype, const void* proj_bias,
                                 int bias_dtype, const float* wscale, void* out, int64_t B, int64_t H, int64_t L,
                                 int64_t D, int64_t N, float scale, float eps, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* Batched PagedKVCache write (replaces the per-token
 * PagedKVCache.write_inplace, mtp_engine.py:582-586, which reads every page
 * id to the host).  For b < B, h < H, t < n (and t < count[b] when count is
 * given): logical = start + t, page = page_table[b, logical],
 * k_pages[page, b, h, logical % page_size, :] = src_k[b, h, node, :] with
 * node = node_idx[b, t] (e.g. the accepted path of a draft tree; NULL: t);
 * v likewise.  Pools [num_pages, B, H, page_size, D] in dtype; sources
 * [B, H, src_len, D] in src_dtype (converted like .to(dtype)); page_table
 * [B, table_stride] int32.  Rows whose page id is outside [-num_pages,
 * num_pages) or whose node index is out of range are skipped and recorded
 * (MTP_ERR_DEVICE via mtp_device_status). */
int mtp_paged_kv_write(void* k_pages, void* v_pages, int dtype, const int32_t* page_table, int64_t table_stride,
                       int64_t num_pages, int64_t page_size, const void* src_k, const void* src_v, int src_dtype,
                       int64_t src_len, const int32_t* node_idx, const int32_t* count, int64_t B, int64_t H,
                       int64_t D, int64_t start, int64_t n, void* stream);

/* ------------------------------------------------------------------------- */
/* verification (lm_head GEMM -> argmax -> acceptance)                        */
/* ------------------------------------------------------------------------- */

/* Bytes of verify workspace for `rows` (= B*S or M) logit rows. */
size_t mtp_verify_workspace(int64_t rows);

/* Puts a verify workspace into its resting state.  Needed once after
 * allocation; every verify call leaves the workspace in that state again. */
int mtp_verify_workspace_init(void* workspace, size_t workspace_bytes, void* stream);

/* top[m] = argmax_v(hidden[m] . W[v] + bias[v]); accept[m] = top[m] == draft[m].
 * Replaces fused_verify, mtp_fused_verify.py:199-234 (eager
 * _eager_fused_verify, 159-166).  accept: int8 [M], top: int32 [M],
 * draft: int32 [M].  No logits are written to memory. */
int mtp_fused_verify(const void* hidden, int h_dtype, const void* weight, int w_dtype,
                     const void* bias, int bias_dtype, const int32_t* draft, int8_t* accept,
                     int32_t* top, int64_t M, int64_t K, int64_t V, void* workspace,
                     size_t workspace_bytes, void* stream);

/* Chain verification.  Replaces fused_multi_verify,
 * mtp_fused_verify.py:237-290 (eager _eager_fused_multi_verify, 169-196).
 * hidden: [B,S,K]; weight: [V,K]; draft: int32 [B,S-1]; accept: int8 [B,S-1]
 * (prefix-gated: 1 only while every earlier draft matched);
 * accepted_n: int32 [B]; corrected: int32 [B] (argmax at position 0). */
int mtp_fused_multi_verify(const void* hidden, int h_dtype, const void* weight, int w_dtype,
                           const void* bias, int bias_dtype, const int32_t* draft, int8_t* accept,
                           int32_t* accepted_n, int32_t* corrected, int64_t B, int64_t S,
                           int64_t K, int64_t V, void* workspace, size_t workspace_bytes,
                           void* stream);

/* Vocab-parallel verify, step 1 (per rank): fold this rank's vocabulary
 * block [vocab_offset, vocab_offset + V_shard) into keys[M] (int64, in place,
 * keys must start at INT64_MIN or hold earlier partial maxima).
 * key = (signed-ordered fp32 logit << 32) | (0xFFFFFFFF - global index), so
 * max over keys = argmax with ties to the lowest index.  Step 2 is an
 * all-reduce(MAX) of keys over the ranks (int64).  This pair replaces the
 * gathered logits of RowParallelLinear, mtp_parallel.py:84-118. */
int mtp_verify_shard_keys(const void* hidden, int h_dtype, const void* weight_shard, int w_dtype,
                          const void* bias_shard, int bias_dtype, int64_t* keys, int64_t M,
                          int64_t K, int64_t V_shard, int64_t vocab_offset, void* stream);

/* mtp_verify_shard_keys with a stream-K region: under GEMM schedule 1 the
 * shard's GEMM may run stream-K using [workspace, workspace +
 * workspace_bytes), which holds mtp_gemm_streamk_bytes(M, V_shard, K,
 * h_dtype) bytes filled once with INT64_MIN (every call leaves it so).
 * workspace may be NULL (then identical to mtp_verify_shard_keys). */
int mtp_verify_shard_keys_ws(const void* hidden, int h_dtype, const void* weight_shard, int w_dtype,
                             const void* bias_shard, int bias_dtype, int64_t* keys, int64_t M, int64_t K,
                             int64_t V_shard, int64_t vocab_offset, void* workspace, size_t workspace_bytes,
                             void* stream);

/* Vocab-parallel verify, step 3: decode reduced keys [B*S] into the outputs
 * of mtp_fused_multi_verify and reset keys to INT64_MIN. */
int mtp_verify_chain_from_keys(int64_t* keys, const int32_t* draft, int8_t* accept,
                               int32_t* accepted_n, int32_t* corrected, int64_t B, int64_t S,
                               void* stream);

/* ---- NCCL communicator for C hosts -------------------------------------
 * The reference's vocab-parallel exchange is a torch process group
 * (ParallelPrimitives, mtp_parallel.py:12-66; RowParallelLinear's gather,
 * mtp_parallel.py:114-118).  A host without torch.distributed creates one
 * NCCL communicator per rank with these calls and passes it to
 * mtp_vocab_parallel_multi_verify.  NCCL is opened at run time
 * (libnccl.so.2, or the file named by the MTP_NCCL_LIBRARY environment
 * variable; a copy the process already loaded is reused); when it cannot be
 * opened these calls return MTP_ERR_NCCL and the rest of the library is
 * unaffected. */
#define MTP_NCCL_ID_BYTES 128

/* NCCL's version code (e.g. 22809 for 2.28.9) in *version. */
int mtp_nccl_version(int* version);

/* ncclGetUniqueId: rank 0 makes the id and the host sends its
 * MTP_NCCL_ID_BYTES bytes to every rank. */
int mtp_nccl_unique_id(void* id);

/* ncclCommInitRank on the current CUDA device (mtp_nccl_init of the
 * boundary): collective, returns once all `world` ranks have joined.
 * *comm receives an opaque handle. */
int mtp_nccl_comm_init(void** comm, const void* id, int rank, int world);

/* ncclCommDestroy (comm may be NULL). */
int mtp_nccl_comm_destroy(void* comm);

/* ncclCommAbort: ends a communicator whose collective cannot finish (a
 * rank died) without waiting for it, e.g. from a host thread that watches a
 * stream the collective holds.  The handle is freed, as by destroy; no
 * other call may be using it. */
int mtp_nccl_comm_abort(void* comm);

/* ncclCommGetAsyncError: MTP_OK, or MTP_ERR_NCCL with NCCL's error text. */
int mtp_nccl_comm_status(void* comm);

/* Workspace of mtp_vocab_parallel_multi_verify: the keys [B*S] int64 (a
 * multiple of 256 bytes) followed by mtp_gemm_streamk_bytes(B*S, V_shard,
 * K, h_dtype) bytes for the shard GEMM's stream-K schedule.  Fill it once
 * with mtp_keys_fill over all of it; every successful call leaves it so. */
size_t mtp_vocab_parallel_workspace(int64_t B, int64_t S, int64_t V_shard, int64_t K, int h_dtype);

/* One rank's vocab-parallel fused_multi_verify in one call: this rank's
 * block [vocab_offset, vocab_offset + V_shard) of the lm_head folded into
 * argmax keys (mtp_verify_shard_keys_ws), the keys all-reduced with MAX
 * over `comm` (ncclInt64, in place; every call with a communicator runs it,
 * a one-rank communicator included; comm NULL = a single-rank run with no
 * collective), then decoded into accept [B, S-1] int8, accepted_n [B]
 * and corrected [B] int32 -- identical on every rank and equal to
 * mtp_fused_multi_verify over the whole lm_head (mtp_fused_verify.py:
 * 237-290 with the weight split as torch.chunk splits it,
 * mtp_parallel.py:62-66).  The current device must be the communicator's.
 * After MTP_ERR_NCCL or MTP_ERR_TIMEOUT the keys may be mid-reduction: fill
 * the workspace again before the next call. */
int mtp_vocab_parallel_multi_verify(const void* hidden, int h_dtype, const void* weight_shard, int w_dtype,
                                    const void* bias_shard, int bias_dtype, const int32_t* draft,
                                    int8_t* accept, int32_t* accepted_n, int32_t* corrected, int64_t B,
                                    int64_t S, int64_t K, int64_t V_shard, int64_t vocab_offset, void* comm,
                                    void* workspace, size_t workspace_bytes, void* stream);

/* Largest B*S that mtp_fused_multi_verify_noalloc accepts. */
#define MTP_NOALLOC_MAX_ROWS 8192

/* Chain verification that allocates nothing and takes no workspace.
 * It has no counterpart in the reference.  It exists for callers that
 * cannot hand the library scratch memory: a host whose device memory is
 * already claimed up front by another allocator (for example a serving
 * process that reserved the free HBM for its KV cache), or a plain C/FFI
 * host that owns only its input and output buffers and must not call
 * cudaMalloc (which can synchronise the device) in the middle of a step.
 * Same inputs, outputs and results as mtp_fused_multi_verify.  Its keys and
 * ticket live in one fixed array of MTP_NOALLOC_MAX_ROWS * 8 + 256 bytes
 * inside the library, which every GPU that loads the library keeps until
 * the process exits; B*S above MTP_NOALLOC_MAX_ROWS is rejected with
 * MTP_ERR_SHAPE.  The first call on a device looks up that array's device
 * address (make that first call before any stream capture).  Each call
 * clears the array first; all calls on a device share it, so calls whose
 * kernels overlap on the GPU (different streams, no ordering) race.  It
 * runs the data-parallel GEMM schedule whatever mtp_set_gemm_schedule chose
 * (the fixed array has no room for stream-K partials). */
int mtp_fused_multi_verify_noalloc(const void* hidden, int h_dtype, const void* weight, int w_dtype,
                                   const void* bias, int bias_dtype, const int32_t* draft, int8_t* accept,
                                   int32_t* accepted_n, int32_t* corrected, int64_t B, int64_t S, int64_t K,
                                   int64_t V, void* stream);

/* Vocab-parallel verify, steps 2+3 fused, over peer memory instead of a
 * collective library (replaces the all-reduce that would gather
 * RowParallelLinear's shards, mtp_parallel.py:114-118).  Each rank owns a
 * buffer of mtp_verify_exchange_bytes(B*S, world) bytes mapped into every
 * rank (symmetric memory, zero-filled once); peer_bufs is a device array of
 * the world buffer addresses, indexed by rank.  One kernel pushes this rank's
 * keys[B*S] (from mtp_verify_shard_keys) into every peer over NVLink,
 * publishes a per-call flag, waits (bounded) for every rank's keys, takes
 * the max and writes the outputs of mtp_fused_multi_verify; keys are reset
 * to INT64_MIN.  epoch is a device uint64 that starts at 0 on every rank;
 * all ranks must make the same sequence of calls. */
size_t mtp_verify_exchange_bytes(int64_t rows, int world);
int mtp_verify_exchange_chain(int64_t* keys, const void* peer_bufs, int rank, int world, uint64_t* epoch,
                              const int32_t* draft, int8_t* accept, int32_t* accepted_n, int32_t* corrected,
                              int64_t B, int64_t S, void* stream);

/* Vocab-parallel verify as ONE kernel per rank, the all-reduce fused into the
 * shard GEMM (replaces mtp_verify_shard_keys + the all-reduce + the scan,
 * i.e. RowParallelLinear's gather, mtp_parallel.py:114-118).  Each rank owns
 * a buffer of mtp_verify_fused_bytes(B*S, world) bytes mapped into every rank
 * (keys [2][B*S] int64, flags [2][world], a call counter), put at rest once
 * with mtp_verify_fused_init; peer_bufs is a device array of the world
 * buffer addresses.  Every tile's (logit, index) key goes to every rank's
 * keys by atomic max over NVLink as the tile finishes; the last CTA of the
 * rank's GEMM then publishes a per-call flag to every rank, waits (bounded,
 * MTP_ERR_TIMEOUT) for every rank's flag, and writes the outputs of
 * mtp_fused_multi_verify from the global keys, which it puts back to rest.
 * hidden/weight_shard: equal 16-bit dtypes with 16-byte rows (tensor
 * cores).  workspace: a verify workspace (mtp_verify_workspace(0) bytes, plus
 * mtp_gemm_streamk_bytes under GEMM schedule 1), put at rest once.  All
 * ranks must make the same sequence of calls with the same B*S.  After a call
 * reports MTP_ERR_TIMEOUT (a rank did not arrive), keys may still be landing:
 * synchronise every rank, then run mtp_verify_fused_init on every buffer
 * again before the next call. */
size_t mtp_verify_fused_bytes(int64_t rows, int world);
int mtp_verify_fused_init(void* buf, int64_t rows, int world, void* stream);
int mtp_verify_shard_fused(const void* hidden, int h_dtype, const void* weight_shard, int w_dtype,
                           const void* bias_shard, int bias_dtype, const void* peer_bufs, int rank, int world,
                           const int32_t* draft, int8_t* accept, int32_t* accepted_n, int32_t* corrected, int64_t B,
                           int64_t S, int64_t K, int64_t V_shard, int64_t vocab_offset, void* workspace,
                           size_t workspace_bytes, void* stream);

/* The host step after fused_multi_verify in generate_fused /
 * generate_optimized (mtp_engine.py:1244-1258, 1326-1337), on the device so
 * the loop needs no .item(): n = min_b accepted_n[b] (one rollback index per
 * step); step_tokens[b, 0:width] = draft[b, 0:n] ++ corrected[b] when n < D
 * (width n + 1), else draft[b, 0:D] (width D); columns width .. D of each
 * row (those below ld) are set to -1, "no token".  info[0] = n, info[1] = width.
 * draft [B,D], accepted_n/corrected [B] int32 (outputs of
 * mtp_fused_multi_verify), step_tokens [B, ld] int32 with ld >= D + 1
 * recommended (ld >= D accepted), info [2] int32.  One small launch. */
int mtp_verify_step(const int32_t* draft, const int32_t* accepted_n, const int32_t* corrected, int64_t B, int64_t D,
                    int32_t* step_tokens, int64_t ld, int32_t* info, void* stream);

/* Fills keys[n] with INT64_MIN (workspace plumbing; no counterpart in the
 * reference, whose temporaries are allocated inside each call). */
int mtp_keys_fill(int64_t* keys, int64_t n, void* stream);

/* Number of kernels this library has launched in this process (all
 * devices).  Benchmarks read it around a timed region. */
uint64_t mtp_launch_count(void);

/* Test support, host memory only: the argmax key packing the kernels use
 * (key = order-preserving int32 of the fp32 value << 32 | 0xFFFFFFFF - index;
 * max over keys = largest value, lowest index among equals) and its decode. */
int mtp_keys_pack_host(const float* values, const uint32_t* index, int64_t* keys, int64_t n);
int mtp_keys_index_host(const int64_t* keys, int32_t* index, int64_t n);

/* Test support (no counterpart in the reference): C[M,N] (fp32) = A[M,K] @ B[N,K]^T
 * through the GEMM mainloop the operators use -- the tcgen05 kernel when
 * force_simt == 0 and the operands qualify (bf16/f16/E4M3, 16-byte rows),
 * else the fp32 CUDA-core kernel. */
int mtp_gemm_test(const void* A, const void* B, int ab_dtype, float* C, int64_t M, int64_t N, int64_t K,
                  int force_simt, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MTP_B200_H */
