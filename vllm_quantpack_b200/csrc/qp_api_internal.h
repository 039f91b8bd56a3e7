// Host-side error reporting shared by the C-ABI entry points.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

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

// Chunk prefill of one sequence through the split-KV decode kernel (qp_decode.cu), used by qp_prefill at head 512:
// the arguments and outputs of qp_prefill (out_mode 0 or 1), with its own workspace size.
int64_t decode_chunk_workspace_bytes(int qlen, int n, int num_q_heads, int num_kv_heads, int head_size);
int decode_chunk_prefill(int fmt, int dtype, const void* q, int64_t q_stride_token, int64_t q_stride_head, void* out,
                         int64_t out_stride_token, int64_t out_stride_head, int qlen, int n, const int32_t* block_row,
                         const void* cache, int block_size, int64_t block_stride, int64_t head_stride,
                         int64_t slot_stride, int64_t k_off, int64_t ks_off, int64_t v_off, int64_t vs_off,
                         int num_q_heads, int num_kv_heads, int head_size, float softmax_scale,
                         const uint32_t* rht_sign_bits, int q_rotated, int tokens_after_keys, int out_mode,
                         float* lse_out, void* workspace, int64_t workspace_bytes, void* stream);
