// Host-side error reporting shared by the C-ABI entry points.
#pragma once
#include <cuda_runtime.h>

// Return codes of every qp_* entry point (0 = success). Mirrored in include/quantpack_b200.h.
enum {
  QP_OK = 0,
  QP_ERR_INVALID = 1,      // bad argument (null pointer, negative size, ...)
  QP_ERR_UNSUPPORTED = 2,  // a shape or dtype this build does not serve
  QP_ERR_LAYOUT = 3,       // cache layout / alignment the kernel cannot read
  QP_ERR_WORKSPACE = 4,    // workspace too small
  QP_ERR_CUDA = 5,         // a CUDA runtime error
};

// Records a formatted message for qp_last_error() (thread-local) and returns `code`.
int set_error(int code, const char* fmt, ...);
// Checks cudaGetLastError() after a launch; returns QP_OK or QP_ERR_CUDA with the message recorded.
int check_launch(const char* what);
// Number of SMs of the current device (cached per device).
int device_sm_count();
