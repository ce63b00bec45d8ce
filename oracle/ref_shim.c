/* ref_shim.c - TEST INFRASTRUCTURE, not part of the product.
 *
 * Runs the reference's own libtinycublas host layer (cuda-shim/libtinycublas/cublas.c, compiled
 * unchanged from its place in the reference tree) and its own kernels (cuda-shim/libtinycublas/
 * gemm.cu, compiled from source here for sm_100a) on a datacenter GPU. The reference drives the GPU
 * through its userspace driver libtinynv (cuda-shim/include/tinynv.h) and its runtime shim
 * libtinycudart; this file implements the 17 functions cublas.c imports from those two on top of
 * NVIDIA's CUDA driver API, which is loaded with dlopen so the library builds without a GPU.
 *
 * Only what cublas.c calls is here:
 *   tinynv_{module_load, get_kernel, launch, malloc, free, memset, memcpy_dtoh, stream_sync, last_error}
 *   tinycudart_{device, default_stream, trace, count_launch, time_launch, now_ns, capturing_nv,
 *               capture_launch}
 * Launches use CU_LAUNCH_PARAM_BUFFER_POINTER with the reference's packed parameter blobs, exactly as
 * its own standalone benches launch them (bf16-20260921/bench_gemm_contract.cu:151-154).
 */
#include <dlfcn.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include "tinynv.h"

typedef int CUresult_;
typedef int CUdevice_;
typedef void *CUcontext_;
typedef void *CUmodule_;
typedef void *CUfunction_;
typedef void *CUstream_;
typedef unsigned long long CUdeviceptr_;

static struct {
  int loaded;
  CUresult_ (*cuInit)(unsigned);
  CUresult_ (*cuCtxGetCurrent)(CUcontext_ *);
  CUresult_ (*cuCtxSetCurrent)(CUcontext_);
  CUresult_ (*cuDeviceGet)(CUdevice_ *, int);
  CUresult_ (*cuDevicePrimaryCtxRetain)(CUcontext_ *, CUdevice_);
  CUresult_ (*cuModuleLoadData)(CUmodule_ *, const void *);
  CUresult_ (*cuModuleGetFunction)(CUfunction_ *, CUmodule_, const char *);
  CUresult_ (*cuLaunchKernel)(CUfunction_, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned,
                              CUstream_, void **, void **);
  CUresult_ (*cuMemAlloc)(CUdeviceptr_ *, size_t);
  CUresult_ (*cuMemFree)(CUdeviceptr_);
  CUresult_ (*cuMemsetD8Async)(CUdeviceptr_, unsigned char, size_t, CUstream_);
  CUresult_ (*cuMemcpyDtoHAsync)(void *, CUdeviceptr_, size_t, CUstream_);
  CUresult_ (*cuStreamSynchronize)(CUstream_);
} D;

static __thread char g_err[256] = "no error";

static tinynv_status_t fail(const char *what, int rc) {
  snprintf(g_err, sizeof g_err, "%s failed (CUresult %d)", what, rc);
  return TINYNV_ERR_DRIVER;
}

#define SYM(name)                                                            \
  do {                                                                       \
    *(void **)&D.name = dlsym(h, #name "_v2");                               \
    if (!D.name) *(void **)&D.name = dlsym(h, #name);                        \
    if (!D.name) {                                                           \
      snprintf(g_err, sizeof g_err, "libcuda.so.1 lacks %s", #name);         \
      return -1;                                                             \
    }                                                                        \
  } while (0)

/* resolve the driver API and make sure the calling thread has the primary context current */
static int ensure(void) {
  if (!D.loaded) {
    void *h = dlopen("libcuda.so.1", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      snprintf(g_err, sizeof g_err, "dlopen libcuda.so.1: %s", dlerror());
      return -1;
    }
    SYM(cuInit);
    SYM(cuCtxGetCurrent);
    SYM(cuCtxSetCurrent);
    SYM(cuDeviceGet);
    SYM(cuDevicePrimaryCtxRetain);
    SYM(cuModuleLoadData);
    SYM(cuModuleGetFunction);
    SYM(cuLaunchKernel);
    SYM(cuMemAlloc);
    SYM(cuMemFree);
    SYM(cuMemsetD8Async);
    SYM(cuMemcpyDtoHAsync);
    SYM(cuStreamSynchronize);
    if (D.cuInit(0) != 0) {
      snprintf(g_err, sizeof g_err, "cuInit failed");
      return -1;
    }
    D.loaded = 1;
  }
  CUcontext_ cur = NULL;
  if (D.cuCtxGetCurrent(&cur) == 0 && cur) return 0;
  CUdevice_ dev;
  CUcontext_ ctx;
  if (D.cuDeviceGet(&dev, 0) || D.cuDevicePrimaryCtxRetain(&ctx, dev) || D.cuCtxSetCurrent(ctx)) {
    snprintf(g_err, sizeof g_err, "no primary context");
    return -1;
  }
  return 0;
}

const char *tinynv_last_error(void) { return g_err; }

tinynv_status_t tinynv_module_load(tinynv_device_t d, const void *cubin, size_t len, tinynv_module_t *out) {
  (void)d;
  (void)len;
  if (ensure()) return TINYNV_ERR_NODEV;
  CUmodule_ m = NULL;
  int rc = D.cuModuleLoadData(&m, cubin);
  if (rc) return fail("cuModuleLoadData", rc);
  *out = (tinynv_module_t)m;
  return TINYNV_OK;
}

tinynv_status_t tinynv_get_kernel(tinynv_module_t m, const char *name, tinynv_kernel_t *out) {
  if (ensure()) return TINYNV_ERR_NODEV;
  CUfunction_ f = NULL;
  int rc = D.cuModuleGetFunction(&f, (CUmodule_)m, name);
  if (rc) return fail("cuModuleGetFunction", rc);
  *out = (tinynv_kernel_t)f;
  return TINYNV_OK;
}

tinynv_status_t tinynv_launch(tinynv_stream_t s, tinynv_kernel_t k, unsigned gx, unsigned gy, unsigned gz, unsigned bx,
                              unsigned by, unsigned bz, unsigned dyn_smem, const void *params, size_t params_len) {
  if (ensure()) return TINYNV_ERR_NODEV;
  size_t len = params_len;
  void *extra[] = {(void *)1 /* CU_LAUNCH_PARAM_BUFFER_POINTER */, (void *)params,
                   (void *)2 /* CU_LAUNCH_PARAM_BUFFER_SIZE */, &len, (void *)0 /* CU_LAUNCH_PARAM_END */};
  int rc = D.cuLaunchKernel((CUfunction_)k, gx, gy, gz, bx, by, bz, dyn_smem, (CUstream_)s, NULL, extra);
  if (rc) return fail("cuLaunchKernel", rc);
  return TINYNV_OK;
}

tinynv_status_t tinynv_malloc(tinynv_device_t d, size_t n, tinynv_devptr_t *out) {
  (void)d;
  if (ensure()) return TINYNV_ERR_NODEV;
  CUdeviceptr_ p = 0;
  int rc = D.cuMemAlloc(&p, n);
  if (rc) return fail("cuMemAlloc", rc);
  *out = (tinynv_devptr_t)p;
  return TINYNV_OK;
}

tinynv_status_t tinynv_free(tinynv_device_t d, tinynv_devptr_t p) {
  (void)d;
  if (ensure()) return TINYNV_ERR_NODEV;
  int rc = D.cuMemFree((CUdeviceptr_)p);
  return rc ? fail("cuMemFree", rc) : TINYNV_OK;
}

tinynv_status_t tinynv_memset(tinynv_stream_t s, tinynv_devptr_t dst, int value, size_t n) {
  if (ensure()) return TINYNV_ERR_NODEV;
  int rc = D.cuMemsetD8Async((CUdeviceptr_)dst, (unsigned char)value, n, (CUstream_)s);
  return rc ? fail("cuMemsetD8Async", rc) : TINYNV_OK;
}

tinynv_status_t tinynv_memcpy_dtoh(tinynv_stream_t s, void *dst, tinynv_devptr_t src, size_t n) {
  if (ensure()) return TINYNV_ERR_NODEV;
  int rc = D.cuMemcpyDtoHAsync(dst, (CUdeviceptr_)src, n, (CUstream_)s);
  return rc ? fail("cuMemcpyDtoHAsync", rc) : TINYNV_OK;
}

tinynv_status_t tinynv_stream_sync(tinynv_stream_t s) {
  if (ensure()) return TINYNV_ERR_NODEV;
  int rc = D.cuStreamSynchronize((CUstream_)s);
  return rc ? fail("cuStreamSynchronize", rc) : TINYNV_OK;
}

/* ---- the libtinycudart hooks cublas.c uses ---- */
tinynv_device_t tinycudart_device(void) { return (tinynv_device_t)(uintptr_t)1; }
tinynv_stream_t tinycudart_default_stream(void) { return (tinynv_stream_t)0; /* the legacy default stream */ }
int tinycudart_trace(void) {
  static int v = -1;
  if (v < 0) {
    const char *e = getenv("TINYCUDART_TRACE");
    v = e && *e && *e != '0';
  }
  return v;
}
void tinycudart_count_launch(const char *name) { (void)name; }
void tinycudart_time_launch(const char *name, double ns) {
  (void)name;
  (void)ns;
}
double tinycudart_now_ns(void) {
  struct timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return ts.tv_sec * 1e9 + ts.tv_nsec;
}
/* a real CUDA stream records launches into a capture by itself, so the shim never diverts them */
int tinycudart_capturing_nv(tinynv_stream_t s) {
  (void)s;
  return 0;
}
int tinycudart_capture_launch(tinynv_kernel_t k, const char *name, unsigned gx, unsigned gy, unsigned gz, unsigned bx,
                              unsigned by, unsigned bz, unsigned smem, const void *params, size_t plen) {
  (void)name;
  return tinynv_launch((tinynv_stream_t)0, k, gx, gy, gz, bx, by, bz, smem, params, plen) == TINYNV_OK ? 0 : -1;
}

/* which reference this library was built from: set by build_ref.sh */
#ifndef REF_PROVENANCE
#define REF_PROVENANCE "unknown"
#endif
const char *tinycublas_ref_provenance(void) { return REF_PROVENANCE; }
