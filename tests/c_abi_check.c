/*
 * A plain C99 caller of libl3g's C ABI, compiled the way a cgo preamble is
 * (C, not C++, with the header alone) and run on a host with no GPU.  It
 * exercises the host-only entry points and the error contract a Go shim
 * relies on: an int status per call, the message of the calling thread's
 * last failure from l3g_last_error(), the reference's wording for GGUF
 * errors (internal/gguf/gguf.go:73, internal/llama/model.go:210), and no
 * silent CPU fallback for anything that needs a device.
 *
 * Usage: c_abi_check <dir for scratch files>.  Prints "ok" and exits 0.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "l3g.h"

static int failures = 0;

#define CHECK(cond)                                                   \
  do {                                                                \
    if (!(cond)) {                                                    \
      fprintf(stderr, "%s:%d: check failed: %s (last error: %s)\n",   \
              __FILE__, __LINE__, #cond, l3g_last_error());           \
      ++failures;                                                     \
    }                                                                 \
  } while (0)

static int contains(const char *s, const char *sub) {
  return s != NULL && strstr(s, sub) != NULL;
}

static void write_file(const char *path, const void *bytes, size_t n) {
  FILE *f = fopen(path, "wb");
  if (!f) {
    fprintf(stderr, "cannot write %s\n", path);
    exit(2);
  }
  fwrite(bytes, 1, n, f);
  fclose(f);
}

int main(int argc, char **argv) {
  char path[4096];
  l3g_options opt;
  l3g_model *m = NULL;
  l3g_hparams hp;
  l3g_shard sh;
  int32_t n = -1;
  uint64_t bytes = 0;
  int rc;

  if (argc != 2) {
    fprintf(stderr, "usage: %s <scratch dir>\n", argv[0]);
    return 2;
  }

  CHECK(l3g_version() == L3G_VERSION);

  /* defaults: one GPU, the current device, the reference's f32 cache */
  memset(&opt, 0x5a, sizeof opt);
  l3g_options_default(&opt);
  CHECK(opt.world_size == 1 && opt.rank == 0 && opt.device == -1);
  CHECK(opt.kv_dtype == L3G_KV_F32);

  /* no device here: the device query fails loudly */
  CHECK(l3g_device_count(&n) != L3G_OK);
  CHECK(strlen(l3g_last_error()) > 0);

  /* tensor-parallel shard of the 8B shape, host-only */
  memset(&hp, 0, sizeof hp);
  hp.vocab_size = 128256;
  hp.n_layers = 32;
  hp.n_emb = 4096;
  hp.n_heads = 32;
  hp.n_heads_kv = 8;
  hp.n_ff = 14336;
  hp.rope_dim = 128;
  hp.ctx_len = 8192;
  hp.rms_eps = 1e-5f;
  hp.rope_base = 500000.0f;
  rc = l3g_shard_plan(&hp, 8, 3, &sh);
  CHECK(rc == L3G_OK);
  CHECK(sh.q_rows == 4 * 128 && sh.q_row0 == 3 * 4 * 128);
  CHECK(sh.kv_rows == 128 && sh.kv_row0 == 3 * 128);
  CHECK(sh.o_col0 == sh.q_row0 && sh.o_cols == sh.q_rows);
  CHECK(sh.ff_rows == 14336 / 8 && sh.ff_row0 == 3 * (14336 / 8));
  CHECK(sh.down_col0 == sh.ff_row0 && sh.down_cols == sh.ff_rows);
  CHECK(sh.vocab_rows > 0 && sh.vocab_row0 == 3 * sh.vocab_stride);
  /* a split that cuts a kv head is refused with a message */
  rc = l3g_shard_plan(&hp, 16, 0, &sh);
  CHECK(rc == L3G_E_INVALID && strlen(l3g_last_error()) > 0);
  CHECK(l3g_shard_plan(NULL, 1, 0, &sh) == L3G_E_INVALID);

  /* sizes of the batched product's buffers, host-only */
  CHECK(l3g_gemm_matrix_bytes(256, 4096, &bytes) == L3G_OK && bytes > 256u * 4096u);
  CHECK(l3g_gemm_act_bytes(64, 4096, &bytes) == L3G_OK && bytes >= 64u * 4096u);
  CHECK(l3g_gemm_matrix_bytes(256, 100, &bytes) == L3G_E_INVALID); /* cols % 32 */

  /* GGUF errors before any device work, in the reference's wording */
  snprintf(path, sizeof path, "%s/not_gguf.bin", argv[1]);
  {
    unsigned char junk[68];
    memset(junk, 0, sizeof junk);
    memcpy(junk, "NOPE", 4);
    write_file(path, junk, sizeof junk);
  }
  rc = l3g_model_load_gguf(path, &opt, &m);
  CHECK(rc == L3G_E_FORMAT && m == NULL);
  CHECK(contains(l3g_last_error(), "not a gguf file"));
  snprintf(path, sizeof path, "%s/does_not_exist.gguf", argv[1]);
  rc = l3g_model_load_gguf(path, &opt, &m);
  CHECK(rc != L3G_OK && m == NULL);
  CHECK(contains(l3g_last_error(), "open"));

  /* a null handle is an error, never a crash */
  CHECK(l3g_model_load(NULL, NULL, 0, &opt, &m) == L3G_E_INVALID);
  CHECK(l3g_forward(NULL, NULL, NULL, 0, NULL) == L3G_E_INVALID);
  CHECK(l3g_state_new(NULL, 16, NULL) == L3G_E_INVALID);
  {
    l3g_kvpool *pool = NULL;
    l3g_state *ps = NULL;
    int32_t n = 0;
    uint64_t pb = 0;
    CHECK(l3g_kvpool_new(NULL, 4, &pool) == L3G_E_INVALID && pool == NULL);
    CHECK(l3g_kvpool_page_bytes(NULL, &pb) == L3G_E_INVALID);
    CHECK(l3g_kvpool_free_pages(NULL, &n) == L3G_E_INVALID);
    CHECK(l3g_state_new_in_pool(NULL, NULL, 16, &ps) == L3G_E_INVALID);
    CHECK(l3g_state_pages(NULL, &n) == L3G_E_INVALID);
    CHECK(L3G_KV_PAGE == 256);
    l3g_kvpool_free(NULL);
  }
  CHECK(l3g_workspace_set_topk_fast_exp(NULL, 1) == L3G_E_INVALID);
  l3g_model_free(NULL);
  l3g_state_free(NULL);
  l3g_workspace_free(NULL);

  if (failures) {
    fprintf(stderr, "%d check(s) failed\n", failures);
    return 1;
  }
  printf("ok\n");
  return 0;
}
