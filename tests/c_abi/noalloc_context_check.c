/* dak_attn_decode_noalloc from a C host that manages its own CUDA contexts
 * through the driver API, with no Python, torch or CUDA runtime of its own in
 * the process.  Such a host is the typical caller of the allocation-free entry
 * point: it binds only the C ABI and may switch contexts on one device.
 *
 * The library's fixed scratch array has one address per context (each context
 * loads its own copy of the library's module), so the entry point must look
 * the address up again whenever a different context is current.  This program
 * runs the same decode through dak_attn_decode (scratch from cuMemAlloc) and
 * dak_attn_decode_noalloc, and compares the two outputs, in this order:
 *   the primary context; a second context created with cuCtxCreate; the
 *   primary again; the second again; the primary after the second is
 *   destroyed; and the primary context after cuDevicePrimaryCtxReset (what
 *   cudaDeviceReset does), which gives it a new identity.
 * Exit status 0 and a last line "ok" on success.
 *
 * Build: gcc -I include -I<cuda>/include tests/c_abi/noalloc_context_check.c
 *        -L directaccesskernel_b200 -ldak_b200 -L<cuda>/lib64/stubs -lcuda -lm */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda.h>

#include "dak_b200.h"

enum { B = 4, HQ = 8, HKV = 2, S = 1000, D = 128, SPLIT = 64 };
#define NSPLIT ((S + SPLIT - 1) / SPLIT)

static unsigned long long lcg_state;
static float uniform(void) { /* in [-1, 1) */
  lcg_state = lcg_state * 6364136223846793005ull + 1442695040888963407ull;
  return (float)((lcg_state >> 40) & 0xFFFFFF) / 8388608.0f - 1.0f;
}

#define CHECK_CU(call)                                                           \
  do {                                                                           \
    CUresult r_ = (call);                                                        \
    if (r_ != CUDA_SUCCESS) {                                                    \
      const char *s_ = NULL;                                                     \
      cuGetErrorString(r_, &s_);                                                 \
      fprintf(stderr, "%s: %s\n", #call, s_ ? s_ : "?");                         \
      return 2;                                                                  \
    }                                                                            \
  } while (0)

#define CHECK_DAK(call)                                                          \
  do {                                                                           \
    int s_ = (call);                                                             \
    if (s_ != DAK_OK) {                                                          \
      fprintf(stderr, "%s: %d %s\n", #call, s_, dak_last_error_message());       \
      return 3;                                                                  \
    }                                                                            \
  } while (0)

/* One decode in the current context: both entry points, outputs compared. */
static int run_case(const char *where, unsigned seed) {
  const size_t nq = (size_t)B * HQ * D, nkv = (size_t)B * HKV * S * D;
  _Float16 *hq = malloc(nq * 2), *hk = malloc(nkv * 2), *hv = malloc(nkv * 2);
  _Float16 *o_ref = malloc(nq * 2), *o_got = malloc(nq * 2);
  lcg_state = 1000003ull * seed + 7;
  const float qs = 1.0f / sqrtf((float)D);
  for (size_t i = 0; i < nq; ++i) hq[i] = (_Float16)(uniform() * qs * 3.0f);
  for (size_t i = 0; i < nkv; ++i) hk[i] = (_Float16)(uniform() * 1.7f);
  for (size_t i = 0; i < nkv; ++i) hv[i] = (_Float16)(uniform() * 1.7f);

  CUdeviceptr dq, dk, dv, dref, dgot, po, pml;
  CHECK_CU(cuMemAlloc(&dq, nq * 2));
  CHECK_CU(cuMemAlloc(&dk, nkv * 2));
  CHECK_CU(cuMemAlloc(&dv, nkv * 2));
  CHECK_CU(cuMemAlloc(&dref, nq * 2));
  CHECK_CU(cuMemAlloc(&dgot, nq * 2));
  CHECK_CU(cuMemAlloc(&po, (size_t)B * HQ * NSPLIT * D * 4));
  CHECK_CU(cuMemAlloc(&pml, (size_t)B * HQ * NSPLIT * 2 * 4));
  CHECK_CU(cuMemcpyHtoD(dq, hq, nq * 2));
  CHECK_CU(cuMemcpyHtoD(dk, hk, nkv * 2));
  CHECK_CU(cuMemcpyHtoD(dv, hv, nkv * 2));
  CHECK_CU(cuMemsetD8(dgot, 0xFF, nq * 2)); /* NaN until written */

  dak_attn_decode_args a;
  memset(&a, 0, sizeof(a));
  a.query = (const void *)dq;
  a.q_stride_b = HQ * D;
  a.q_stride_h = D;
  a.key = (const void *)dk;
  a.value = (const void *)dv;
  a.kv_stride_b = (int64_t)HKV * S * D;
  a.kv_stride_h = (int64_t)S * D;
  a.out = (void *)dref;
  a.o_stride_b = HQ * D;
  a.o_stride_h = D;
  a.partial_o = (float *)po;
  a.partial_ml = (float *)pml;
  a.batch = B;
  a.host_size = 0;
  a.num_q_heads = HQ;
  a.num_kv_heads = HKV;
  a.head_dim = D;
  a.seq_len = S;
  a.split_size = SPLIT;
  a.scaling = 1.0f / sqrtf((float)D);
  a.dtype = DAK_DTYPE_F16;
  CHECK_DAK(dak_attn_decode(&a, NULL));
  dak_attn_decode_args b = a;
  b.out = (void *)dgot;
  b.partial_o = NULL;
  b.partial_ml = NULL;
  CHECK_DAK(dak_attn_decode_noalloc(&b, NULL));
  CHECK_CU(cuCtxSynchronize());
  int status = -1;
  CHECK_DAK(dak_device_status(1, &status));
  CHECK_CU(cuMemcpyDtoH(o_ref, dref, nq * 2));
  CHECK_CU(cuMemcpyDtoH(o_got, dgot, nq * 2));

  double num = 0.0, den = 0.0;
  int nan = 0;
  for (size_t i = 0; i < nq; ++i) {
    const double r = (double)o_ref[i], g = (double)o_got[i];
    if (g != g || r != r) nan = 1;
    if (fabs(g - r) > num) num = fabs(g - r);
    if (fabs(r) > den) den = fabs(r);
  }
  const double err = den > 0 ? num / den : 1.0;
  printf("%s: rel err %.3g, device status %d\n", where, err, status);
  cuMemFree(dq);
  cuMemFree(dk);
  cuMemFree(dv);
  cuMemFree(dref);
  cuMemFree(dgot);
  cuMemFree(po);
  cuMemFree(pml);
  free(hq);
  free(hk);
  free(hv);
  free(o_ref);
  free(o_got);
  /* The attention parity tolerance used by the other GPU tests. */
  return (nan || status != 0 || den == 0.0 || err > 2e-3) ? 1 : 0;
}

int main(void) {
  CUdevice dev;
  CUcontext primary, other;
  CHECK_CU(cuInit(0));
  CHECK_CU(cuDeviceGet(&dev, 0));
  CHECK_CU(cuDevicePrimaryCtxRetain(&primary, dev));
  CHECK_CU(cuCtxSetCurrent(primary));
  int rc = run_case("primary", 0);
  if (!rc) {
    CHECK_CU(cuCtxCreate(&other, 0, dev)); /* current from here on */
    rc = run_case("second context", 1);
  }
  if (!rc) {
    CHECK_CU(cuCtxSetCurrent(primary));
    rc = run_case("primary again", 2);
  }
  if (!rc) {
    CHECK_CU(cuCtxSetCurrent(other));
    rc = run_case("second context again", 3);
  }
  if (!rc) {
    CHECK_CU(cuCtxDestroy(other));
    CHECK_CU(cuCtxSetCurrent(primary));
    rc = run_case("primary after the second is destroyed", 4);
  }
  if (!rc) {
    CHECK_CU(cuDevicePrimaryCtxRelease(dev));
    CHECK_CU(cuDevicePrimaryCtxReset(dev));
    CHECK_CU(cuDevicePrimaryCtxRetain(&primary, dev));
    CHECK_CU(cuCtxSetCurrent(primary));
    rc = run_case("primary after reset", 5);
  }
  cuDevicePrimaryCtxRelease(dev);
  if (rc) return rc;
  printf("ok\n");
  return 0;
}
