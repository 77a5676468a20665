/* A plain C99 host of the library: compiles against include/mtp_b200.h
 * alone, links libmtp_b200.so, and calls the entry points that need no
 * GPU (argument checks, plans, schedule checks).  Built and run by
 * tests/test_abi.py; prints "ok" and exits 0 when every check holds. */
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "mtp_b200.h"

#define CHECK(cond)                                                   \
  do {                                                                \
    if (!(cond)) {                                                    \
      fprintf(stderr, "check failed at line %d: %s (%s)\n", __LINE__, \
              #cond, mtp_last_error());                               \
      return 1;                                                       \
    }                                                                 \
  } while (0)

int main(void) {
  CHECK(mtp_abi_version() >= 1);

  /* schedule and kernel switches */
  CHECK(mtp_set_gemm_schedule(2) == MTP_ERR_ARG);
  CHECK(strlen(mtp_last_error()) > 0);
  int bn = 0;
  CHECK(mtp_gemm_tile_plan(384, 128256, 148, &bn) == MTP_OK && bn == 256);

  /* host walks of the kernels' own schedules */
  int64_t tiles = 0;
  CHECK(mtp_gemm_tile_check(384, 128256, 148, &tiles) == MTP_OK && tiles == 11);
  CHECK(mtp_gemm_streamk_check(384, 128256, 4096, MTP_DTYPE_BF16, 148, 0) == MTP_OK);
  int64_t info[9];
  CHECK(mtp_gemm_streamk_plan(384, 128256, 4096, MTP_DTYPE_BF16, 148, 0, info) == MTP_OK && info[0] == 1);

  /* argument checks answer before anything is launched */
  CHECK(mtp_fused_multi_verify(NULL, MTP_DTYPE_BF16, NULL, MTP_DTYPE_BF16, NULL, 0, NULL, NULL, NULL, NULL,
                               2, 0, 64, 100, NULL, 0, NULL) != MTP_OK);
  CHECK(mtp_vocab_parallel_multi_verify(NULL, MTP_DTYPE_BF16, NULL, MTP_DTYPE_BF16, NULL, 0, NULL, NULL, NULL,
                                        NULL, 2, 6, 64, 100, 0, NULL, NULL, 0, NULL) == MTP_ERR_WORKSPACE);
  CHECK(mtp_vocab_parallel_workspace(64, 6, 16032, 4096, MTP_DTYPE_BF16) >= 3072);

  /* key packing: a larger logit wins; equal logits -> the lower index */
  float v[3] = {1.5f, 2.0f, 2.0f};
  uint32_t idx[3] = {7, 9, 3};
  int64_t keys[3];
  CHECK(mtp_keys_pack_host(v, idx, keys, 3) == MTP_OK);
  CHECK(keys[1] > keys[0] && keys[2] > keys[1]);
  int32_t back[3];
  CHECK(mtp_keys_index_host(keys, back, 3) == MTP_OK && back[0] == 7 && back[1] == 9 && back[2] == 3);

  /* the NCCL entries answer without a GPU: a version, or MTP_ERR_NCCL */
  int ver = 0;
  int st = mtp_nccl_version(&ver);
  CHECK(st == MTP_OK || st == MTP_ERR_NCCL);
  void* comm = NULL;
  char id[MTP_NCCL_ID_BYTES] = {0};
  CHECK(mtp_nccl_comm_init(&comm, id, 3, 2) == MTP_ERR_ARG && comm == NULL);

  printf("ok\n");
  return 0;
}
