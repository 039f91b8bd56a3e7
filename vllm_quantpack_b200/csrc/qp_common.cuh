// Shared device helpers for the quantized KV-cache kernels (sm_100a only).
//
// Cache cell of one (block, KV head, slot), bytes:
//   int4 : [K hs/2 nibbles | K scale f32 | V hs/2 nibbles | V scale f32]   (hs + 8 bytes; 264 at hs 256)
//   k8v4 : [K hs int8      | K scale f32 | V hs/2 nibbles | V scale f32]   (1.5 hs + 8 bytes; 392 at hs 256)
// Low nibble = even channel. An int4 scale word carries the 4-bit zero point in its low mantissa bits.
// (vllm_quantpack/attention/k8v4_kv.py:10-11, 41-65; tests/test_int4_kv.py:95-103.)
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ != 1000)
#error "quantpack_b200 kernels are written for sm_100a only"
#endif

namespace qp {

enum { FMT_INT4 = 0, FMT_K8V4 = 1 };
enum { DT_BF16 = 0, DT_F16 = 1 };

// Error codes written by kernels into the device error word (qp_device_error()).
enum { DEV_ERR_NONE = 0, DEV_ERR_WAIT_TIMEOUT = 1 };

// Device-side error word: the first kernel that gives up a bounded wait records its code here.
extern __device__ int g_device_error;

// ------------------------------------------------------------------------------------------------ conversions

template <int DT>
struct Elem;
template <>
struct Elem<DT_BF16> {
  using T = __nv_bfloat16;
  static __device__ __forceinline__ float to_f(T x) { return __bfloat162float(x); }
  static __device__ __forceinline__ T from_f(float x) { return __float2bfloat16_rn(x); }
};
template <>
struct Elem<DT_F16> {
  using T = __half;
  static __device__ __forceinline__ float to_f(T x) { return __half2float(x); }
  static __device__ __forceinline__ T from_f(float x) { return __float2half_rn(x); }
};

// Round half away from zero exactly as k8v4_ops.py:5-8: fp32 add of +-0.5 (round to nearest), then truncation.
__device__ __forceinline__ float round_half_away(float x) {
  return x >= 0.f ? (float)__float2int_rz(__fadd_rn(x, 0.5f)) : (float)__float2int_rz(__fsub_rn(x, 0.5f));
}

// ------------------------------------------------------------------------------------------------ PTX wrappers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: a waiting thread sleeps until the phase completes or the hint runs out, instead
// of spinning and taking issue slots from the warps doing the work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait for phase `parity` of `bar`, at most `limit_ns` nanoseconds. On timeout records DEV_ERR_WAIT_TIMEOUT and
// returns false: the caller stops its work and returns (never traps, never spins forever).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait_sleep(bar, parity)) {
    if (global_timer_ns() - t0 > limit_ns) {
      atomicCAS(&g_device_error, DEV_ERR_NONE, DEV_ERR_WAIT_TIMEOUT);
      return false;
    }
  }
  return true;
}

// Same bound as mbar_wait_bounded, but polling without the suspend hint: for warp-specialised pipelines where every
// hand-off sits on the critical path and the wake-up latency of a suspended waiter costs more than its issue slots.
__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity, uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > limit_ns) {
      atomicCAS(&g_device_error, DEV_ERR_NONE, DEV_ERR_WAIT_TIMEOUT);
      return false;
    }
  }
  return true;
}

// 1-D bulk copy (TMA engine, no tensor map, no multicast) global -> this CTA's shared memory, completing on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x2(uint32_t& r0, uint32_t& r1, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                                  uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x2_trans(uint32_t& r0, uint32_t& r1, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}

// D = A * B + D, fp16 operands, fp32 accumulators (m16n8k16, row.col).
__device__ __forceinline__ void mma_f16_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// (x & and_mask) | or_mask in one lop3 (truth table 0xEA).
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t x, uint32_t and_mask, uint32_t or_mask) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(x), "r"(and_mask), "r"(or_mask));
  return r;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// both halves of an f16x2 set to x (round to nearest)
__device__ __forceinline__ uint32_t h2_bits(float x) {
  const __half2 h = __floats2half2_rn(x, x);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

// 2^x in one MUFU instruction (ex2.approx; callers keep x <= a small bound, very negative x flush to 0)
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Named barrier over `threads` threads that also ORs `pred` across them (all of them get the result).
__device__ __forceinline__ bool named_bar_or(int id, int threads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(threads)
      : "memory");
  return r != 0;
}

// 2^e exactly, e in [-149, 127] (subnormal results below 2^-126), by building the float's bits
__device__ __forceinline__ float exp2_int(int e) {
  return e >= -126 ? __uint_as_float(static_cast<uint32_t>(e + 127) << 23) : __uint_as_float(1u << (e + 149));
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ------------------------------------------------------------------------------------------------ RHT
//
// The randomized Hadamard transform of this build: y = H (d * x), H the unnormalised Sylvester Hadamard matrix,
// evaluated by fp32 butterflies of stride 1, 2, 4, ..., n/2 in that order; inverse x' = d * (H y). Sign bit i of
// `sign_bits` set means d_i = -1. The butterfly order is fixed so that every result is reproducible bit for bit.
//
// Warp version for n = 32 * E: lane L holds elements [E L, E L + E). Strides < E run inside the lane, strides >= E
// across lanes (xor of lane bits). For a pair (a at the lower index, b at the upper) the lower lane keeps a + b,
// the upper lane a - b.
template <int E>
__device__ __forceinline__ void warp_wht(float (&x)[E], int lane) {
#pragma unroll
  for (int h = 1; h < E; h <<= 1) {
#pragma unroll
    for (int i = 0; i < E; ++i) {
      if ((i & h) == 0) {
        const float a = x[i], b = x[i + h];
        x[i] = __fadd_rn(a, b);
        x[i + h] = __fsub_rn(a, b);
      }
    }
  }
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    const bool upper = (lane & m) != 0;
#pragma unroll
    for (int i = 0; i < E; ++i) {
      const float o = __shfl_xor_sync(0xffffffffu, x[i], m);
      x[i] = upper ? __fsub_rn(o, x[i]) : __fadd_rn(x[i], o);
    }
  }
}

template <int E>
__device__ __forceinline__ void apply_signs(float (&x)[E], const uint32_t* sign_bits, int lane) {
#pragma unroll
  for (int i = 0; i < E; ++i) {
    const int c = lane * E + i;
    if ((sign_bits[c >> 5] >> (c & 31)) & 1u) x[i] = -x[i];
  }
}

}  // namespace qp
