// K0 / K0': cache write of int4_per_token_head and k8v4_per_token_head, with the randomized Hadamard transform
// fused in front of the quantizer; and the standalone RHT (`single_rht`).
//
// One warp per (token, KV head): the warp holds the head's hs values (lane L: elements [E L, E L + E)), rotates them
// in fp32, rounds them to the model dtype (as `single_rht(x.float()).to(x.dtype)`,
// vllm_quantpack/attention/k8v4_kv.py:71-72), then quantizes with warp reductions for min / max / absmax and writes
// the packed codes and scale words into the cell. The quantizer performs the fp32 operations of the reference's
// source (vllm_quantpack/attention/k8v4_ops.py:30-63) the way Triton compiles them for the GPU: every `/` is PTX
// div.full.f32 (Triton's plain fp32 division; its IEEE-rounded one is the separate tl.math.div_rn), and
// v * (1 / scale) + zp is one FMA (Triton fuses by default). Codes and scale words are then bit-exact with the
// reference's store as it runs on the B200 (measured); against the same source evaluated in IEEE fp32 (Triton's
// interpreter, the CPU oracle) they differ only next to rounding ties, by one code step or a couple of ulp.
#include "qp_api_internal.h"
#include "qp_common.cuh"

namespace qp {

// The division the reference's compiled store performs: Triton lowers a plain fp32 `/` to PTX div.full.f32 (its
// IEEE-rounded division is the separate tl.math.div_rn), so the same instruction gives the same codes and scales.
__device__ __forceinline__ float div_full(float a, float b) {
  float r;
  asm("div.full.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

struct StoreParams {
  const void* key;
  const void* value;
  int64_t num_tokens;
  int num_kv_heads;
  int64_t k_st, k_sh, v_st, v_sh;  // element strides
  const int64_t* slot_mapping;
  uint8_t* cache;
  int block_size;
  int64_t block_stride, head_stride, slot_stride;  // bytes
  int k_off, ks_off, v_off, vs_off;                 // bytes inside the cell
  const uint32_t* sign_bits;
  int rotate;  // 0: key / value are already in the RHT domain (the `_store_k8v4` kernel contract)
};

template <int E, int DT>
__device__ __forceinline__ void load_rotate_round(const void* base, int64_t off, const uint32_t* sign_bits, int lane,
                                                  int rotate, float (&x)[E]) {
  using EL = Elem<DT>;
  const typename EL::T* p = reinterpret_cast<const typename EL::T*>(base) + off + lane * E;
#pragma unroll
  for (int i = 0; i < E; ++i) x[i] = EL::to_f(p[i]);
  if (!rotate) return;
  apply_signs<E>(x, sign_bits, lane);
  warp_wht<E>(x, lane);
#pragma unroll
  for (int i = 0; i < E; ++i) x[i] = EL::to_f(EL::from_f(x[i]));  // round to the model dtype
}

// int4 quantizer of one warp-held row (k8v4_ops.py:44-63). Writes E/2 packed bytes per lane and the scale word.
template <int E>
__device__ __forceinline__ void quant_store_int4(const float (&x)[E], uint8_t* cell, int codes_off, int word_off,
                                                 int lane) {
  float mn = x[0], mx = x[0];
#pragma unroll
  for (int i = 1; i < E; ++i) {
    mn = fminf(mn, x[i]);
    mx = fmaxf(mx, x[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  const float scale = fmaxf(div_full(__fsub_rn(mx, mn), 15.0f), 1e-6f);
  const float zp = fminf(fmaxf(round_half_away(div_full(-mn, scale)), 0.0f), 15.0f);
  const float inv = div_full(1.0f, scale);
  uint32_t packed[E / 8 > 0 ? E / 8 : 1] = {};
#pragma unroll
  for (int i = 0; i < E; ++i) {
    float q = round_half_away(__fmaf_rn(x[i], inv, zp));
    q = fminf(fmaxf(q, 0.0f), 15.0f);
    packed[i / 8] |= (static_cast<uint32_t>(q) & 0xFu) << (4 * (i % 8));
  }
  // E/2 bytes per lane, 4-byte aligned (codes_off and the cell are multiples of 4)
  if constexpr (E >= 8) {
    uint32_t* dst = reinterpret_cast<uint32_t*>(cell + codes_off + lane * (E / 2));
#pragma unroll
    for (int w = 0; w < E / 8; ++w) dst[w] = packed[w];
  } else {
    uint16_t* dst = reinterpret_cast<uint16_t*>(cell + codes_off + lane * (E / 2));
    *dst = static_cast<uint16_t>(packed[0]);
  }
  if (lane == 0) {
    const uint32_t word = (__float_as_uint(scale) & 0xFFFFFFF0u) | (static_cast<uint32_t>(zp) & 0xFu);
    *reinterpret_cast<uint32_t*>(cell + word_off) = word;
  }
}

// int8 key quantizer of k8v4 (k8v4_ops.py:33-42).
template <int E>
__device__ __forceinline__ void quant_store_int8(const float (&x)[E], uint8_t* cell, int codes_off, int word_off,
                                                 int lane) {
  float am = 0.f;
#pragma unroll
  for (int i = 0; i < E; ++i) am = fmaxf(am, fabsf(x[i]));
  am = warp_max(am);
  const float scale = fmaxf(div_full(am, 127.0f), 1e-6f);
  uint32_t words[E / 4] = {};
#pragma unroll
  for (int i = 0; i < E; ++i) {
    float q = round_half_away(div_full(x[i], scale));
    q = fminf(fmaxf(q, -127.0f), 127.0f);
    words[i / 4] |= (static_cast<uint32_t>(static_cast<int>(q)) & 0xFFu) << (8 * (i % 4));
  }
  uint32_t* dst = reinterpret_cast<uint32_t*>(cell + codes_off + lane * E);
#pragma unroll
  for (int w = 0; w < E / 4; ++w) dst[w] = words[w];
  if (lane == 0) *reinterpret_cast<float*>(cell + word_off) = scale;
}

template <int FMT, int DT, int E>
__global__ void __launch_bounds__(256) store_kernel(const StoreParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (item >= p.num_tokens * p.num_kv_heads) return;
  const int64_t tok = item / p.num_kv_heads;
  const int head = static_cast<int>(item % p.num_kv_heads);
  const int64_t slot = p.slot_mapping[tok];
  if (slot < 0) return;  // padding token (k8v4_ops.py:23-24)
  const int64_t blk = slot / p.block_size;
  const int64_t s = slot % p.block_size;
  uint8_t* cell = p.cache + blk * p.block_stride + head * p.head_stride + s * p.slot_stride;

  float x[E];
  load_rotate_round<E, DT>(p.key, tok * p.k_st + head * p.k_sh, p.sign_bits, lane, p.rotate, x);
  if constexpr (FMT == FMT_INT4)
    quant_store_int4<E>(x, cell, p.k_off, p.ks_off, lane);
  else
    quant_store_int8<E>(x, cell, p.k_off, p.ks_off, lane);
  load_rotate_round<E, DT>(p.value, tok * p.v_st + head * p.v_sh, p.sign_bits, lane, p.rotate, x);
  quant_store_int4<E>(x, cell, p.v_off, p.vs_off, lane);
}

template <int E>
__global__ void __launch_bounds__(256) rht_kernel(const float* x, float* y, int64_t rows, const uint32_t* sign_bits,
                                                  int inverse) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  float v[E];
  const float* src = x + row * (32 * E) + lane * E;
#pragma unroll
  for (int i = 0; i < E; ++i) v[i] = src[i];
  if (!inverse) apply_signs<E>(v, sign_bits, lane);
  warp_wht<E>(v, lane);
  if (inverse) apply_signs<E>(v, sign_bits, lane);
  float* dst = y + row * (32 * E) + lane * E;
#pragma unroll
  for (int i = 0; i < E; ++i) dst[i] = v[i];
}

template <int FMT, int DT>
static int launch_store_dt(const StoreParams& p, int head_size, cudaStream_t st) {
  const int64_t items = p.num_tokens * p.num_kv_heads;
  const dim3 grid(static_cast<unsigned>((items + 7) / 8)), block(256);
  switch (head_size) {
    case 128: store_kernel<FMT, DT, 4><<<grid, block, 0, st>>>(p); break;
    case 256: store_kernel<FMT, DT, 8><<<grid, block, 0, st>>>(p); break;
    case 512: store_kernel<FMT, DT, 16><<<grid, block, 0, st>>>(p); break;
    default: return set_error(QP_ERR_UNSUPPORTED, "store: head size %d not in {128, 256, 512}", head_size);
  }
  return check_launch("store");
}

}  // namespace qp

using namespace qp;

static int store_entry(int fmt, const void* key, const void* value, int dtype, int64_t num_tokens, int num_kv_heads,
                       int head_size, int64_t key_stride_token, int64_t key_stride_head, int64_t value_stride_token,
                       int64_t value_stride_head, const int64_t* slot_mapping, void* cache, int block_size,
                       int64_t block_stride, int64_t head_stride, int64_t slot_stride, int64_t k_off, int64_t ks_off,
                       int64_t v_off, int64_t vs_off, const uint32_t* rht_sign_bits, int rotate, void* stream) {
  if (dtype != DT_BF16 && dtype != DT_F16) return set_error(QP_ERR_UNSUPPORTED, "store: dtype %d", dtype);
  if (num_tokens < 0 || num_kv_heads <= 0 || block_size <= 0)
    return set_error(QP_ERR_INVALID, "store: bad sizes (tokens %lld, kv heads %d, block %d)", (long long)num_tokens,
                     num_kv_heads, block_size);
  if (num_tokens == 0) return QP_OK;
  if (!key || !value || !slot_mapping || !cache || (rotate && !rht_sign_bits))
    return set_error(QP_ERR_INVALID, "store: null pointer");
  if ((k_off | ks_off | v_off | vs_off | slot_stride | head_stride | block_stride) & 3)
    return set_error(QP_ERR_LAYOUT, "store: cell fields and strides must be 4-byte aligned");
  if (reinterpret_cast<uintptr_t>(cache) & 3) return set_error(QP_ERR_LAYOUT, "store: cache not 4-byte aligned");
  StoreParams p{key,          value,       num_tokens,   num_kv_heads, key_stride_token, key_stride_head,
                value_stride_token, value_stride_head, slot_mapping, static_cast<uint8_t*>(cache), block_size,
                block_stride, head_stride, slot_stride, (int)k_off, (int)ks_off, (int)v_off, (int)vs_off,
                rht_sign_bits, rotate};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (fmt == FMT_INT4)
    return dtype == DT_BF16 ? launch_store_dt<FMT_INT4, DT_BF16>(p, head_size, st)
                            : launch_store_dt<FMT_INT4, DT_F16>(p, head_size, st);
  return dtype == DT_BF16 ? launch_store_dt<FMT_K8V4, DT_BF16>(p, head_size, st)
                          : launch_store_dt<FMT_K8V4, DT_F16>(p, head_size, st);
}

extern "C" int qp_reshape_and_cache_int4(const void* key, const void* value, int dtype, int64_t num_tokens,
                                         int num_kv_heads, int head_size, int64_t key_stride_token,
                                         int64_t key_stride_head, int64_t value_stride_token,
                                         int64_t value_stride_head, const int64_t* slot_mapping, void* cache,
                                         int block_size, int64_t block_stride, int64_t head_stride,
                                         int64_t slot_stride, int64_t k_off, int64_t ks_off, int64_t v_off,
                                         int64_t vs_off, const uint32_t* rht_sign_bits, int rotate, void* stream) {
  return store_entry(FMT_INT4, key, value, dtype, num_tokens, num_kv_heads, head_size, key_stride_token,
                     key_stride_head, value_stride_token, value_stride_head, slot_mapping, cache, block_size,
                     block_stride, head_stride, slot_stride, k_off, ks_off, v_off, vs_off, rht_sign_bits, rotate,
                     stream);
}

extern "C" int qp_reshape_and_cache_k8v4(const void* key, const void* value, int dtype, int64_t num_tokens,
                                         int num_kv_heads, int head_size, int64_t key_stride_token,
                                         int64_t key_stride_head, int64_t value_stride_token,
                                         int64_t value_stride_head, const int64_t* slot_mapping, void* cache,
                                         int block_size, int64_t block_stride, int64_t head_stride,
                                         int64_t slot_stride, int64_t k_off, int64_t ks_off, int64_t v_off,
                                         int64_t vs_off, const uint32_t* rht_sign_bits, int rotate, void* stream) {
  return store_entry(FMT_K8V4, key, value, dtype, num_tokens, num_kv_heads, head_size, key_stride_token,
                     key_stride_head, value_stride_token, value_stride_head, slot_mapping, cache, block_size,
                     block_stride, head_stride, slot_stride, k_off, ks_off, v_off, vs_off, rht_sign_bits, rotate,
                     stream);
}

extern "C" int qp_single_rht(const float* x, float* y, int64_t rows, int head_size, int inverse,
                             const uint32_t* rht_sign_bits, void* stream) {
  if (rows < 0) return set_error(QP_ERR_INVALID, "single_rht: rows %lld", (long long)rows);
  if (rows == 0) return QP_OK;
  if (!x || !y || !rht_sign_bits) return set_error(QP_ERR_INVALID, "single_rht: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid(static_cast<unsigned>((rows + 7) / 8)), block(256);
  switch (head_size) {
    case 128: rht_kernel<4><<<grid, block, 0, st>>>(x, y, rows, rht_sign_bits, inverse); break;
    case 256: rht_kernel<8><<<grid, block, 0, st>>>(x, y, rows, rht_sign_bits, inverse); break;
    case 512: rht_kernel<16><<<grid, block, 0, st>>>(x, y, rows, rht_sign_bits, inverse); break;
    default: return set_error(QP_ERR_UNSUPPORTED, "single_rht: head size %d not in {128, 256, 512}", head_size);
  }
  return check_launch("single_rht");
}
