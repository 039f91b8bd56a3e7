// Library-wide C-ABI entry points: version, error reporting, the device error word.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include "qp_api_internal.h"
#include "qp_common.cuh"

namespace qp {
__device__ int g_device_error = 0;
}

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(QP_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return QP_OK;
}

int device_sm_count() {
  static int counts[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (counts[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    counts[dev] = n;
  }
  return counts[dev];
}

extern "C" int qp_version(void) { return 100; }

extern "C" const char* qp_last_error(void) { return g_last_error; }

// Reads and clears the device error word of the current device (synchronous). *code = 0 when no kernel gave up a
// bounded wait since the last call.
extern "C" int qp_device_error(int* code) {
  if (!code) return set_error(QP_ERR_INVALID, "qp_device_error: null pointer");
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(code, qp::g_device_error, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(qp::g_device_error, &zero, sizeof(int));
  if (e != cudaSuccess) return set_error(QP_ERR_CUDA, "qp_device_error: %s", cudaGetErrorString(e));
  return QP_OK;
}
