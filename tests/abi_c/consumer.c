/* A plain C host of the library: includes the boundary header, links the shared
 * library, and calls the entry points that need no GPU (version, the host-only
 * GEMM plan, argument checks).  Built and run by tests/test_abi_c.py. */
#include <stdio.h>
#include <string.h>

#include "ltxfp8.h"

static int fails = 0;
#define CHECK(cond)                                               \
  do {                                                            \
    if (!(cond)) {                                                \
      fprintf(stderr, "check failed: %s (line %d)\n", #cond, __LINE__); \
      ++fails;                                                    \
    }                                                             \
  } while (0)

int main(void) {
  CHECK((ltxfp8_version() >> 16) == 1);

  ltxfp8_gemm_plan_info info;
  /* 8-GPU FFN down shard: full waves unsplit, the last two M-tile rows split 4 ways */
  CHECK(ltxfp8_gemm_plan_for_sms(6144, 4096, 16384, 148, &info) == LTXFP8_OK);
  CHECK(info.split_row0 == 5888 && info.splits == 4 && info.launches == 3);
  CHECK(info.workspace_bytes == 32ull * 4 * 128 * 256 * 4);
  CHECK(info.workspace_bytes <= LTXFP8_STATIC_SCRATCH_BYTES);
  /* a full-wave shape needs nothing */
  CHECK(ltxfp8_gemm_plan_for_sms(24576, 16384, 4096, 148, &info) == LTXFP8_OK);
  CHECK(info.splits == 1 && info.launches == 1 && info.workspace_bytes == 0 && info.split_row0 == 24576);

  /* errors: a negative code and a message, nothing touched */
  CHECK(ltxfp8_gemm_plan_for_sms(128, 100, 256, 148, &info) == LTXFP8_ERR_UNSUPPORTED_SHAPE);
  CHECK(strstr(ltxfp8_last_error(), "gemm_plan") != NULL);
  CHECK(ltxfp8_gemm(NULL, NULL, 128, NULL, NULL, NULL, NULL, 128, 256, 256, NULL, NULL) ==
        LTXFP8_ERR_INVALID_ARGUMENT);

  if (fails == 0) printf("abi_c ok\n");
  return fails == 0 ? 0 : 1;
}
