// tcgen05 / TMEM / UMMA descriptor wrappers shared by the decode and prefill kernels (inline PTX, sm_100a).
#pragma once
#include <stdint.h>

#include "qp_common.cuh"

namespace qp {

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// true in one lane of the (converged, full) warp: the lane that issues a tcgen05.mma / commit for the whole warp
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b32 r;\n\t"
      "elect.sync r|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// D[tmem] (+)= A[smem desc] * B[smem desc], fp16 operands, fp32 accumulate
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]: A (M rows = TMEM lanes, K along columns, two fp16 per 32-bit column)
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on `bar` once every tcgen05 op this thread issued so far has completed
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 64 columns of fp32 from TMEM (this warp's lane quarter)
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,"
      "%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,"
      "%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]),
        "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]),
        "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]),
        "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]),
        "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,"
      "%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
// v = (32 columns at ta) + (32 columns at tb): both loads in flight before the one wait (the wait names every
// destination register, so no use of them can be scheduled above it)
__device__ __forceinline__ void tmem_ld32_sum2(uint32_t ta, uint32_t tb, float (&v)[32]) {
  uint32_t r[32], u[32];
#define QP_LD32(R, ADDR)                                                                                             \
  asm volatile(                                                                                                      \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "                                                                      \
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,"  \
      "%29,%30,%31}, [%32];"                                                                                         \
      : "=r"(R[0]), "=r"(R[1]), "=r"(R[2]), "=r"(R[3]), "=r"(R[4]), "=r"(R[5]), "=r"(R[6]), "=r"(R[7]), "=r"(R[8]), \
        "=r"(R[9]), "=r"(R[10]), "=r"(R[11]), "=r"(R[12]), "=r"(R[13]), "=r"(R[14]), "=r"(R[15]), "=r"(R[16]),      \
        "=r"(R[17]), "=r"(R[18]), "=r"(R[19]), "=r"(R[20]), "=r"(R[21]), "=r"(R[22]), "=r"(R[23]), "=r"(R[24]),     \
        "=r"(R[25]), "=r"(R[26]), "=r"(R[27]), "=r"(R[28]), "=r"(R[29]), "=r"(R[30]), "=r"(R[31])                   \
      : "r"(ADDR))
  QP_LD32(r, ta);
  QP_LD32(u, tb);
#undef QP_LD32
#define QP_W8(R, o) "+r"(R[o]), "+r"(R[o + 1]), "+r"(R[o + 2]), "+r"(R[o + 3]), "+r"(R[o + 4]), "+r"(R[o + 5]), \
                    "+r"(R[o + 6]), "+r"(R[o + 7])
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : QP_W8(r, 0), QP_W8(r, 8), QP_W8(r, 16), QP_W8(r, 24), QP_W8(u, 0), QP_W8(u, 8), QP_W8(u, 16),
                 QP_W8(u, 24)
               :
               : "memory");
#undef QP_W8
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) + __uint_as_float(u[i]);
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,"
      "%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,"
      "%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

// Loads of 32 lanes x 8 / 16 columns into registers, and a wait that names those registers as read-write operands:
// without them in the wait's operand list, the compiler may schedule a use of a destination register above the
// wait, reading it before the load has landed.
#define QP_TLD8(R, o, ADDR)                                                                                       \
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"                           \
               : "=r"(R[o]), "=r"(R[o + 1]), "=r"(R[o + 2]), "=r"(R[o + 3]), "=r"(R[o + 4]), "=r"(R[o + 5]),      \
                 "=r"(R[o + 6]), "=r"(R[o + 7])                                                                   \
               : "r"(ADDR))
#define QP_TLD16(R, o, ADDR)                                                                                      \
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "  \
               "[%16];"                                                                                           \
               : "=r"(R[o]), "=r"(R[o + 1]), "=r"(R[o + 2]), "=r"(R[o + 3]), "=r"(R[o + 4]), "=r"(R[o + 5]),      \
                 "=r"(R[o + 6]), "=r"(R[o + 7]), "=r"(R[o + 8]), "=r"(R[o + 9]), "=r"(R[o + 10]), "=r"(R[o + 11]), \
                 "=r"(R[o + 12]), "=r"(R[o + 13]), "=r"(R[o + 14]), "=r"(R[o + 15])                               \
               : "r"(ADDR))
#define QP_TLD4(R, o, ADDR)                                                                                       \
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"                                       \
               : "=r"(R[o]), "=r"(R[o + 1]), "=r"(R[o + 2]), "=r"(R[o + 3])                                       \
               : "r"(ADDR))
#define QP_TW4(R, o) "+r"(R[o]), "+r"(R[o + 1]), "+r"(R[o + 2]), "+r"(R[o + 3])
#define QP_TW8(R, o) "+r"(R[o]), "+r"(R[o + 1]), "+r"(R[o + 2]), "+r"(R[o + 3]), "+r"(R[o + 4]), "+r"(R[o + 5]), \
                     "+r"(R[o + 6]), "+r"(R[o + 7])
// N (4, 8, 12, 16, 24 or 32) columns of fp32 from TMEM (this warp's lane quarter), waited for
template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, float (&v)[N]) {
  static_assert(N == 4 || N == 8 || N == 12 || N == 16 || N == 24 || N == 32, "4, 8, 12, 16, 24 or 32 columns");
  uint32_t r[32];
  if constexpr (N >= 16) QP_TLD16(r, 0, taddr);
  if constexpr (N == 8 || N == 12) QP_TLD8(r, 0, taddr);
  if constexpr (N == 4) QP_TLD4(r, 0, taddr);
  if constexpr (N == 12) QP_TLD4(r, 8, taddr + 8);
  if constexpr (N == 24) QP_TLD8(r, 16, taddr + 16);
  if constexpr (N == 32) QP_TLD16(r, 16, taddr + 16);
  if constexpr (N == 4) asm volatile("tcgen05.wait::ld.sync.aligned;" : QP_TW4(r, 0) : : "memory");
  if constexpr (N == 12) asm volatile("tcgen05.wait::ld.sync.aligned;" : QP_TW8(r, 0), QP_TW4(r, 8) : : "memory");
  if constexpr (N == 8) asm volatile("tcgen05.wait::ld.sync.aligned;" : QP_TW8(r, 0) : : "memory");
  if constexpr (N == 16) asm volatile("tcgen05.wait::ld.sync.aligned;" : QP_TW8(r, 0), QP_TW8(r, 8) : : "memory");
  if constexpr (N == 24)
    asm volatile("tcgen05.wait::ld.sync.aligned;" : QP_TW8(r, 0), QP_TW8(r, 8), QP_TW8(r, 16) : : "memory");
  if constexpr (N == 32)
    asm volatile("tcgen05.wait::ld.sync.aligned;" : QP_TW8(r, 0), QP_TW8(r, 8), QP_TW8(r, 16), QP_TW8(r, 24) : :
                 "memory");
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = __uint_as_float(r[i]);
}
#undef QP_TW8
#undef QP_TW4
#undef QP_TLD16
#undef QP_TLD8
#undef QP_TLD4
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
}
// N (4, 8, 12, 16, 24 or 32) columns of fp32 into TMEM (this warp's lane quarter); the caller waits (wait::st)
template <int N>
__device__ __forceinline__ void tmem_st_cols(uint32_t taddr, const float (&v)[N]) {
  static_assert(N % 4 == 0 && N <= 32, "a multiple of 4 columns, at most 32");
#pragma unroll
  for (int c = 0; c < N; c += 4)
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr + c),
                 "r"(__float_as_uint(v[c])), "r"(__float_as_uint(v[c + 1])), "r"(__float_as_uint(v[c + 2])),
                 "r"(__float_as_uint(v[c + 3]))
                 : "memory");
}
// 16 lanes x 256 bits, two repetitions along the columns: thread i writes v[4r], v[4r + 1] to lane i / 4, columns
// 8 r + 2 (i % 4) + {0, 1}, and v[4r + 2], v[4r + 3] to lane 8 + i / 4, the same columns (r = 0, 1); lanes counted
// from the lane in taddr (0 or 16 inside the warp's quarter)
__device__ __forceinline__ void tmem_st_16x256b_x2(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.16x256b.x2.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}
// one repetition of the above (r = 0 only: 8 columns)
__device__ __forceinline__ void tmem_st_16x256b_x1(uint32_t taddr, const uint32_t (&v)[4]) {
  asm volatile("tcgen05.st.sync.aligned.16x256b.x1.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr), "r"(v[0]), "r"(v[1]),
               "r"(v[2]), "r"(v[3])
               : "memory");
}

__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

// 128B-swizzled canonical UMMA shared-memory descriptor (sm_100 version 1). K-major: SBO = 8-row group stride;
// MN-major: LBO = 64-element block stride along M/N, SBO = 8-row group stride along K.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}
// Canonical UMMA shared-memory descriptor without swizzle (sm_100 version 1, layout type 0): core matrices of 8 rows
// x 16 bytes stored as 128 contiguous bytes. K-major: LBO = byte stride between core matrices along K, SBO = along
// M/N. MN-major (a core matrix holds 8 M/N elements of each of 8 K indices): SBO = byte stride between core matrices
// along M/N, LBO = along K.
__device__ __forceinline__ uint64_t interleave_desc(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// instruction descriptor: fp32 accumulate, fp16 A and B, A K-major, B K- or MN-major, M x N
__host__ __device__ constexpr uint32_t f16_idesc(int m, int n, bool b_mn_major) {
  return (1u << 4) | (0u << 7) | (0u << 10) | (0u << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// byte offset of 16-byte chunk `chunk` (0..7) of row `row` inside a 128B-swizzled tile of 8-row groups
__device__ __forceinline__ uint32_t sw128_off(int row, int chunk) {
  return (row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4);
}


}  // namespace qp
