/* A C host of libint4kv_b200.so: compiled against include/int4kv_b200.h with a
 * plain C compiler and linked to the library, as a C / cgo / FFI binding of
 * the reference's launchers would be. It calls only the host-side argument
 * checks (no device memory, no launch), so it runs without a GPU. Exit 0 when
 * every call answers as the header documents. */
#include <stdio.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#include "int4kv_b200.h"

static int failures = 0;

static void expect(const char* what, cudaError_t got, cudaError_t want) {
  if (got != want) {
    fprintf(stderr, "FAIL %s: got %d, want %d\n", what, (int)got, (int)want);
    ++failures;
  }
}

int main(void) {
  const cudaError_t bad = cudaErrorInvalidValue;
  size_t bytes = 0;
  /* the reference launchers' own checks (csrc/flash_decode_int4.cu:228-284) */
  expect("cu_quantize_int4 rows=0", cu_quantize_int4(NULL, 0, 4, NULL, NULL, NULL, NULL), bad);
  expect("cu_flash_decode_int4 head_dim=257",
         cu_flash_decode_int4(NULL, NULL, NULL, NULL, NULL, NULL, 1, 1, 257, 1, 1, NULL, NULL), bad);
  expect("cu_flash_decode_int4 batch=0",
         cu_flash_decode_int4(NULL, NULL, NULL, NULL, NULL, NULL, 0, 1, 64, 1, 1, NULL, NULL), bad);
  /* the paged path */
  expect("quantize_grouped head_dim % 4",
         int4kv_quantize_grouped(NULL, 8, 2, 6, 128, NULL, NULL, NULL, NULL), bad);
  expect("paged_decode_workspace_size head_dim 96",
         int4kv_paged_decode_workspace_size(1, 2, 2, 96, &bytes), bad);
  expect("paged_decode_workspace_size_ex bad value kind",
         int4kv_paged_decode_workspace_size_ex(1, 2, 2, 128, 7, &bytes), bad);
  expect("paged_decode kv heads not dividing q heads",
         int4kv_paged_decode(NULL, NULL, NULL, NULL, NULL, NULL, 1, 3, 2, 128, 16, 128, 4, 4,
                             NULL, NULL, 0, NULL, NULL), bad);
  expect("cache_append_rope head_dim % 8 with a table",
         int4kv_cache_append_rope((const float*)16, NULL, (const int32_t*)16, (const int32_t*)16,
                                  (float*)16, 1, 1, 2, 12, 128, 16, (const int32_t*)16, 4, 4,
                                  (uint8_t*)16, NULL, INT4KV_VALUES_F32, (float*)16,
                                  (const float*)16, (const float*)16, 8, NULL, NULL, 0, NULL,
                                  NULL), bad);
  expect("rope overlapping in/out",
         int4kv_rope((const float*)4096, (const int32_t*)4096, 4, 2, 64, (const float*)4096,
                     (const float*)4096, 8, (float*)(4096 + 256), NULL, NULL), bad);
  expect("exchange_bytes 9 ranks", int4kv_exchange_bytes(9, 8, 128, &bytes), bad);
  expect("exchange_bytes ok", int4kv_exchange_bytes(INT4KV_EXCHANGE_MAX_RANKS, 32, 128, &bytes),
         cudaSuccess);
  if (bytes == 0) { fprintf(stderr, "FAIL exchange_bytes returned 0\n"); ++failures; }
  expect("merge_partials head_dim 96", int4kv_merge_partials((const void*)16, 2, 4, 96, (float*)16, NULL), bad);
  expect("block_decode null query",
         int4kv_block_decode(NULL, NULL, NULL, NULL, NULL, INT4KV_VALUES_F16, NULL, NULL, 1, 1, 1,
                             1, 128, 16, NULL, NULL, 0, NULL), bad);
  if (INT4KV_PARTIAL_RECORD_BYTES(128) != 16 + 4 * 128) {
    fprintf(stderr, "FAIL record size\n");
    ++failures;
  }
  {
    const char* info = int4kv_build_info();
    if (!info || !strstr(info, "sm_100a")) { fprintf(stderr, "FAIL build info\n"); ++failures; }
  }
  if (failures == 0) printf("c abi ok\n");
  return failures ? 1 : 0;
}
