/*
 * A plain C99 host of the library, as a cgo / JNI / FFI binding would be: it includes only
 * include/mi_paged.h and include/mi_layers.h, links libmi_paged.so and calls the host-side paths
 * (version, workspace planning, argument rejection, zero-sized work) that need no GPU.
 * Each check prints one "ok <name>" line or "FAIL <name>: ..." and the exit status counts failures.
 * Test infrastructure: compiled and run by tests/test_c_consumer.py.
 */
#include <stdio.h>
#include <string.h>

#include "mi_layers.h"
#include "mi_paged.h"

static int failures = 0;

static void check(int cond, const char* name, const char* detail) {
  if (cond) {
    printf("ok %s\n", name);
  } else {
    printf("FAIL %s: %s\n", name, detail);
    ++failures;
  }
}

int main(void) {
  const int64_t zero_strides[3] = {0, 0, 0};
  int rc;
  size_t ws_small, ws_big, ws_f32;

  check(mi_version() >= 100, "version", "mi_version() below 1.0.0");
  check(mi_last_error() != NULL, "last_error", "mi_last_error() returned NULL");

  /* Null pools with work to do: rejected on the host, before any CUDA call. */
  rc = mi_kv_scatter(NULL, NULL, zero_strides, zero_strides, 4, 1, NULL, NULL, NULL, 4, NULL, NULL, 8, 16, 2, 32,
                     MI_F32, NULL);
  check(rc == MI_ERR_INVALID && strstr(mi_last_error(), "null pointer") != NULL, "scatter_null_pointer",
        mi_last_error());

  /* An element type outside MI_F32 / MI_BF16 / MI_F16. */
  rc = mi_kv_scatter(NULL, NULL, zero_strides, zero_strides, 4, 1, NULL, NULL, NULL, 4, NULL, NULL, 8, 16, 2, 32, 9,
                     NULL);
  check(rc == MI_ERR_INVALID && strstr(mi_last_error(), "dtype") != NULL, "scatter_bad_dtype", mi_last_error());

  /* Zero tokens: a no-op that never touches the device. */
  rc = mi_kv_scatter(NULL, NULL, zero_strides, zero_strides, 0, 1, NULL, NULL, NULL, 0, NULL, NULL, 8, 16, 2, 32,
                     MI_BF16, NULL);
  check(rc == MI_OK, "scatter_zero_tokens", mi_last_error());

  /* Query heads that are not a multiple of the KV heads. */
  rc = mi_paged_decode(NULL, zero_strides, NULL, NULL, NULL, NULL, NULL, NULL, 8, 16, 3, 32, NULL, 1, 1, NULL, 2, 4,
                       1.0f, NULL, 0, NULL, 0, MI_F32, NULL);
  check(rc == MI_ERR_INVALID && strstr(mi_last_error(), "multiple") != NULL, "decode_head_ratio", mi_last_error());

  /* Workspace planning is host-only: split-K partials for 16-bit types, none for the fp32 path. */
  ws_small = mi_paged_decode_workspace_size(256, 16, 8, 128, 256, 16, MI_BF16);
  ws_big = mi_paged_decode_workspace_size(512, 32, 8, 128, 2048, 16, MI_BF16);
  ws_f32 = mi_paged_decode_workspace_size(256, 16, 8, 128, 256, 16, MI_F32);
  check(ws_small > 0 && ws_small % 256 == 0, "decode_workspace_aligned", "size 0 or not a multiple of 256");
  check(ws_big > ws_small, "decode_workspace_grows", "a larger batch and context did not need more");
  check(ws_f32 == 0, "decode_workspace_f32", "the fp32 path asked for workspace");

  return failures;
}
