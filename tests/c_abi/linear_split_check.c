/* A C host of the offloaded linear, with no Python or torch in the process:
 * the binding a non-Python caller of the reference's gemv_horizontal path
 * (src/torch_runtime.cu:223-246) would write against include/dak_b200.h.
 *
 * y[ntok, N] = x[ntok, K] . W^T with W's first HOST_COLS output features in
 * pinned host memory (cudaHostAlloc, read by the GPU over the host link) and
 * the rest in device memory, both in the transposed [K, cols] layout; checked
 * against a double-precision product on the CPU.  Exit status 0 on success.
 *
 * Build: gcc -I include tests/c_abi/linear_split_check.c -I<cuda>/include
 *        -L directaccesskernel_b200 -ldak_b200 -L<cuda>/lib64 -lcudart -lm */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime.h>

#include "dak_b200.h"

enum { N = 384, K = 520, HOST_COLS = 128, DEV_COLS = N - HOST_COLS };

static unsigned long long lcg_state = 12345;
static float uniform(void) { /* in [-1, 1) */
  lcg_state = lcg_state * 6364136223846793005ull + 1442695040888963407ull;
  return (float)((lcg_state >> 40) & 0xFFFFFF) / 8388608.0f - 1.0f;
}

#define CHECK_CUDA(call)                                                         \
  do {                                                                           \
    cudaError_t e_ = (call);                                                     \
    if (e_ != cudaSuccess) {                                                     \
      fprintf(stderr, "%s: %s\n", #call, cudaGetErrorString(e_));                \
      return 2;                                                                  \
    }                                                                            \
  } while (0)

static int run(int ntok) {
  _Float16 *w = malloc(sizeof(_Float16) * N * K), *x = malloc(sizeof(_Float16) * ntok * K);
  _Float16 *y = malloc(sizeof(_Float16) * ntok * N);
  _Float16 *wd_t = malloc(sizeof(_Float16) * K * DEV_COLS);
  for (int i = 0; i < N * K; ++i) w[i] = (_Float16)(0.05f * uniform());
  for (int i = 0; i < ntok * K; ++i) x[i] = (_Float16)uniform();

  _Float16 *wh_t = NULL; /* [K, HOST_COLS] pinned */
  CHECK_CUDA(cudaHostAlloc((void **)&wh_t, sizeof(_Float16) * K * HOST_COLS, cudaHostAllocDefault));
  for (int k = 0; k < K; ++k) {
    for (int c = 0; c < HOST_COLS; ++c) wh_t[k * HOST_COLS + c] = w[c * K + k];
    for (int c = 0; c < DEV_COLS; ++c) wd_t[k * DEV_COLS + c] = w[(HOST_COLS + c) * K + k];
  }
  void *d_w = NULL, *d_x = NULL, *d_y = NULL;
  CHECK_CUDA(cudaMalloc(&d_w, sizeof(_Float16) * K * DEV_COLS));
  CHECK_CUDA(cudaMalloc(&d_x, sizeof(_Float16) * ntok * K));
  CHECK_CUDA(cudaMalloc(&d_y, sizeof(_Float16) * ntok * N));
  CHECK_CUDA(cudaMemcpy(d_w, wd_t, sizeof(_Float16) * K * DEV_COLS, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(d_x, x, sizeof(_Float16) * ntok * K, cudaMemcpyHostToDevice));

  dak_linear_args a;
  memset(&a, 0, sizeof(a));
  a.w_host = wh_t;
  a.host_cols = HOST_COLS;
  a.ld_host = HOST_COLS;
  a.host_col_offset = 0;
  a.w_dev = d_w;
  a.dev_cols = DEV_COLS;
  a.ld_dev = DEV_COLS;
  a.dev_col_offset = HOST_COLS;
  a.x = d_x;
  a.ldx = K;
  a.y = d_y;
  a.ldy = N;
  a.ntok = ntok;
  a.K = K;
  a.dtype = DAK_DTYPE_F16;
  a.path = DAK_PATH_AUTO;
  int st = dak_linear_split(&a, NULL);
  if (st != DAK_OK) {
    fprintf(stderr, "dak_linear_split: %s (%s)\n", dak_strerror(st), dak_last_error_message());
    return 1;
  }
  int dev_status = -1;
  st = dak_device_status(1, &dev_status);
  if (st != DAK_OK || dev_status != 0) {
    fprintf(stderr, "device status %d (%s)\n", dev_status, dak_last_error_message());
    return 1;
  }
  CHECK_CUDA(cudaMemcpy(y, d_y, sizeof(_Float16) * ntok * N, cudaMemcpyDeviceToHost));

  double max_err = 0.0, max_ref = 0.0;
  for (int t = 0; t < ntok; ++t)
    for (int n = 0; n < N; ++n) {
      double ref = 0.0;
      for (int k = 0; k < K; ++k) ref += (double)x[t * K + k] * (double)w[n * K + k];
      max_err = fmax(max_err, fabs((double)y[t * N + n] - ref));
      max_ref = fmax(max_ref, fabs(ref));
    }
  const double rel = max_err / max_ref;
  printf("ntok %d: max |y - y_ref| / max |y_ref| = %.3g\n", ntok, rel);
  cudaFree(d_w);
  cudaFree(d_x);
  cudaFree(d_y);
  cudaFreeHost(wh_t);
  free(w);
  free(x);
  free(y);
  free(wd_t);
  return rel <= 1e-2 ? 0 : 1;
}

int main(void) {
  const int counts[] = {1, 2, 8, 48};  /* both kernels: CUDA core and tcgen05 */
  for (unsigned i = 0; i < sizeof(counts) / sizeof(counts[0]); ++i) {
    const int rc = run(counts[i]);
    if (rc) return rc;
  }
  printf("ok\n");
  return 0;
}
