/* The C ABI from a plain C99 host program: the header compiles as C, the
 * library links, and the host-only entry points (no device work) behave as
 * the reference's tests for them say.  tests/test_abi_c.py compiles and runs
 * it; it needs no GPU. */
#include <stdio.h>
#include <string.h>

#include "klearu_gpu.h"

static int failures = 0;
#define CHECK(cond)                                               \
  do {                                                            \
    if (!(cond)) {                                                \
      fprintf(stderr, "%s:%d: check failed: %s\n", __FILE__, __LINE__, #cond); \
      ++failures;                                                 \
    }                                                             \
  } while (0)

int main(void) {
  CHECK(kl_abi_version() == KLEARU_GPU_ABI_VERSION);
  CHECK(kl_dist_unique_id_size() > 0);

  /* NULL handles are argument errors, never crashes */
  CHECK(kl_ctx_destroy(NULL) == KL_EINVAL);
  CHECK(kl_net_destroy(NULL) == KL_EINVAL);
  CHECK(kl_net_sync(NULL) == KL_EINVAL);
  CHECK(kl_net_comm_abort(NULL) == KL_EINVAL);
  CHECK(kl_dataset_destroy(NULL) == KL_EINVAL);
  CHECK(kl_batch_iter_destroy(NULL) == KL_EINVAL);

  /* LibSvmDataset, 1-based indices detected (libsvm.rs:235-249) */
  {
    const char* text = "0 1:1.0 3:2.0\n1 2:5.0\n";
    kl_dataset_t ds = NULL;
    int64_t n = -1, dim = -1, nl = -1, nnz = -1, nlab = -1;
    const int64_t *rp = NULL, *lp = NULL;
    const uint32_t *idx = NULL, *lab = NULL;
    const float* val = NULL;
    CHECK(kl_libsvm_parse(text, strlen(text), 4, 2, 1, &ds) == KL_OK);
    CHECK(kl_dataset_info(ds, &n, &dim, &nl, &nnz, &nlab) == KL_OK);
    CHECK(n == 2 && dim == 4 && nl == 2 && nnz == 3 && nlab == 2);
    CHECK(kl_dataset_csr(ds, &rp, &idx, &val, &lp, &lab) == KL_OK);
    CHECK(rp[0] == 0 && rp[1] == 2 && rp[2] == 3);
    CHECK(idx[0] == 0 && idx[1] == 2 && idx[2] == 1);
    CHECK(val[0] == 1.0f && val[1] == 2.0f && val[2] == 5.0f);
    CHECK(lp[1] == 1 && lab[0] == 0 && lab[1] == 1);
    CHECK(kl_dataset_destroy(ds) == KL_OK);
  }

  /* a malformed label is an error with the reference's message (libsvm.rs:291-298) */
  {
    const char* bad = "abc 0:1.0\n";
    kl_dataset_t ds = NULL;
    CHECK(kl_libsvm_parse(bad, strlen(bad), 10, 5, 1, &ds) == KL_EINVAL);
    CHECK(ds == NULL);
    CHECK(strstr(kl_last_error(NULL), "invalid label") != NULL);
  }

  /* BatchIterator: 10 examples in batches of 3 -> 3, 3, 3, 1, then the end
   * (dataset.rs:170-189); every example once */
  {
    char text[256] = "";
    int seen[10] = {0};
    int sizes[8], nb = 0, i;
    kl_dataset_t ds = NULL;
    kl_batch_iter_t it = NULL;
    for (i = 0; i < 10; ++i) {
      char line[32];
      snprintf(line, sizeof line, "%d 0:1.0\n", i);
      strcat(text, line);
    }
    CHECK(kl_libsvm_parse(text, strlen(text), 4, 10, 1, &ds) == KL_OK);
    CHECK(kl_batch_iter_create(ds, 3, 42, 1, &it) == KL_OK);
    for (;;) {
      kl_batch b;
      int s;
      memset(&b, 0, sizeof b);
      if (kl_batch_iter_next(it, &b) != KL_OK || b.batch == 0 || nb == 8) break;
      sizes[nb++] = b.batch;
      CHECK(b.nlabels == b.batch && b.nnz == b.batch);
      for (s = 0; s < b.batch; ++s) {
        const uint32_t id = b.labels[b.label_ptr[s]];
        CHECK(id < 10);
        if (id < 10) ++seen[id];
      }
    }
    CHECK(nb == 4 && sizes[0] == 3 && sizes[1] == 3 && sizes[2] == 3 && sizes[3] == 1);
    for (i = 0; i < 10; ++i) CHECK(seen[i] == 1);
    CHECK(kl_batch_iter_destroy(it) == KL_OK);
    CHECK(kl_dataset_destroy(ds) == KL_OK);
  }

  if (failures) return 1;
  printf("ok\n");
  return 0;
}
