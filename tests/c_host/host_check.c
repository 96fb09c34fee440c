/*
 * Plain-C host of libspx: what a cgo / FFI binding of the drop-in boundary
 * sees.  Compiled with a C compiler against include/spx.h only (no C++,
 * no CUDA headers), linked against libspx.so, and run by tests/test_host.py.
 * Checks, without launching device work: the registry mirrors the
 * reference's kernel names and push-constant counts, options round-trip,
 * the GEMM plan query answers, argument errors come back as status codes
 * with a message, and compute calls report SPX_ERR_NO_DEVICE when there is
 * no CUDA device (on a GPU host one relu dispatch runs instead).
 * Prints "ok" and exits 0, or prints the failed check and exits 1.
 */
#include <stdio.h>
#include <string.h>

#include "spx.h"

#define CHECK(c)                                                      \
  do {                                                                \
    if (!(c)) {                                                       \
      printf("FAILED %s:%d: %s (%s)\n", __FILE__, __LINE__, #c,       \
             spx_last_error() ? spx_last_error() : "");               \
      return 1;                                                       \
    }                                                                 \
  } while (0)

int main(void) {
  /* registry: names as the reference's kernels.rs, push counts per entry */
  int n = spx_kernel_count(), found_conv = 0, found_relu = 0;
  CHECK(n > 20);
  for (int i = 0; i < n; ++i) {
    const char* name = spx_kernel_name(i);
    CHECK(name != NULL && spx_kernel_push_count(name) >= 0);
    if (strcmp(name, "conv2d") == 0) found_conv = 1;
    if (strcmp(name, "relu") == 0) found_relu = 1;
  }
  CHECK(found_conv && found_relu);
  CHECK(spx_kernel_name(n) == NULL);
  CHECK(spx_kernel_push_count("warp_drive") == -1);

  /* options */
  CHECK(spx_get_option("gemm_path") == 0);
  CHECK(spx_set_option("gemm_path", 1) == SPX_OK && spx_get_option("gemm_path") == 1);
  CHECK(spx_set_option("gemm_path", 0) == SPX_OK);
  CHECK(spx_set_option("gemm_path", 7) == SPX_ERR_INVALID_ARGUMENT);
  CHECK(spx_last_error() != NULL && strlen(spx_last_error()) > 0);

  /* GEMM plan (host only): expand 16 -> 96 at 112x112, batch 256 */
  int32_t plan[17];
  CHECK(spx_gemm_tc_plan(3211264, 96, 16, 1, 0, 1, plan, 17) == SPX_OK);
  CHECK(plan[0] == 96 && plan[2] == 1 && plan[4] >= 2);
  CHECK(spx_gemm_tc_plan(0, 96, 16, 1, 0, 1, plan, 17) == SPX_ERR_INVALID_ARGUMENT);

  /* the drop-in dispatch: relu over 8 floats */
  float in[8] = {-2.f, -1.f, 0.f, 1.f, 2.f, -0.5f, 0.5f, 3.f}, out[8] = {0};
  int32_t push[1] = {8};
  CHECK(spx_kernel_push_count("relu") == 1);
  spx_kernel_output_info info;
  int rc = spx_run_kernel("relu.spv", in, 8, NULL, 0, out, 8, push, 1, 0, &info);
  if (spx_device_count() == 0) {
    CHECK(rc == SPX_ERR_NO_DEVICE);
  } else {
    CHECK(rc == SPX_OK);
    for (int i = 0; i < 8; ++i) CHECK(out[i] == (in[i] > 0.f ? in[i] : 0.f));
    CHECK(info.vendor_id == 0x10de);
  }
  /* unknown kernel and wrong push count are status codes, not crashes */
  CHECK(spx_run_kernel("warp_drive.spv", in, 8, NULL, 0, out, 8, push, 1, 0, NULL) != SPX_OK);
  CHECK(spx_op_unary(NULL, 0, NULL, NULL, 0, 0.0f) == SPX_ERR_INVALID_ARGUMENT);
  printf("ok\n");
  return 0;
}
