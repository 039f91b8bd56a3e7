// K3: long-chunk prefill over the int4 / k8v4 paged cache on the 5th-generation tensor cores (tcgen05 + TMEM),
// dequantising each key / value tile in shared memory: no scratch unpack of the cache.
//
// Reference behaviour (what this computes): vllm_quantpack/attention/int4_prefill.py:203-232 `prefill_sequence`
// (attention of a chunk of qlen queries, the last qlen positions of a context of n tokens, over the whole cached
// context, causal inside the chunk, RHT domain, scale softmax_scale / head), which the reference runs as 16k-token
// bf16 unpacks + FlashAttention 2 + an fp32 log-sum-exp fold, and the 2D Triton path (int4_kv.py:113-119).
//
// B200 design (one persistent CTA of 10 warps per SM):
//   warp 0      producer: 1-D bulk copies of the raw 264 / 392-byte cells of a 64-key tile (whole 16-key runs) into a
//               ring of raw stages;
//   warp 1      MMA issuer (one thread): S = Q K^T (M 128 rows, N 64 keys, K 256; Q read from TMEM) into TMEM, then
//               O += P V (M 128, N 256 channels, K 64 keys) into TMEM, each finished with tcgen05.commit onto
//               mbarriers;
//   warps 2-5   dequant into double-buffered key and value operand tiles (the conversion of tile j + 1 overlaps the
//               MMAs of tile j): raw cells -> fp16 operands in shared memory, 128B-swizzled canonical UMMA layouts. One lop3
//               turns two nibbles into fp16, one f16x2 subtract makes the exact (u - zp) (int8 codes for k8v4 keys),
//               one f16x2 multiply applies the token's scale over a power of two (the tile's largest key scale; the
//               piece's running largest value scale), so the softmax never touches per-key scales. The channel order
//               inside every 8 channels is [0 4 1 5 2 6 3 7] (what one lop3 pair yields), the same for Q and K (a dot
//               product does not see the order) and undone on O in the epilogue;
//   warps 6-9   softmax: one thread per TMEM lane (= query row); at the start of each piece it stores its row of the
//               prepared Q tile into TMEM (columns 128-255). Scores in log2 units = S x (softmax_scale / head x
//               log2 e x 2^-row exponent x 2^key-tile exponent); the running maximum is lazy and per thread (P may
//               reach 2^8 before O is rescaled in TMEM, which is rare); P in fp16 is stored back into TMEM over the
//               S buffer it came from, as the A operand of the PV MMA (no shared-memory round trip). The epilogue
//               reads O from TMEM and writes fp32 partials + base-2 lse.
// Rows of an M-tile are (query token, query head of the KV head's group) pairs, head fastest: the 6 heads of a group
// share every dequantised key / value tile. The (M-tile, key-tile) space is split evenly over the CTAs (stream-K):
// an M-tile may be finished by two CTAs, whose partials the merge kernel folds (with the inverse RHT).
#include <math.h>

#include <algorithm>

#include "qp_api_internal.h"
#include "qp_common.cuh"

namespace qp {

constexpr int PF_HS = 256;
constexpr int PF_BM = 128;  // query rows per M-tile (TMEM lanes)
constexpr int PF_BN = 64;   // keys per tile
constexpr int PF_THREADS = 448;  // 14 warps: producer, MMA, 4 dequant, 8 softmax
constexpr float PF_SLACK = 8.f;
constexpr float PF_LOG2E = 1.4426950408889634f;

template <int FMT>
struct PfCfg {
  static constexpr int CELL = FMT == FMT_INT4 ? PF_HS + 8 : PF_HS * 3 / 2 + 8;
  static constexpr int KB = FMT == FMT_INT4 ? PF_HS / 2 : PF_HS;  // key bytes in a cell
  static constexpr int RS = FMT == FMT_INT4 ? 4 : 3;               // raw stages
  static constexpr int RAW_BYTES = PF_BN * CELL;
  // shared memory map (operand tiles 1024-byte aligned for the 128B swizzle); Q, S, P and O live in TMEM
  static constexpr int OFF_K = 0;                       // 2 buffers x 4 K-blocks x 64 keys x 128 B = 64 KB
  static constexpr int OFF_V = OFF_K + 65536;           // 2 buffers x 4 N-blocks x 8 key groups x 1024 B = 64 KB
  static constexpr int OFF_RAW = OFF_V + 65536;         // RS x RAW_BYTES
  static constexpr int OFF_SC = OFF_RAW + RS * RAW_BYTES;  // [2 buffers][key factor 2^F, value exponent E] (16 B)
  static constexpr int OFF_XCH = OFF_SC + 2 * 16;          // [k / v][2 buffers][2 warps] tile maxima exchange
  static constexpr int OFF_HX = OFF_XCH + 2 * 2 * 2 * 4;  // softmax pairs: [2 buffers][2 halves][128] row maxima,
                                                         // then [2 halves][128] row sums
  static constexpr int OFF_BAR = OFF_HX + (2 * 2 * 128 + 2 * 128) * 4;
  static constexpr int NBAR = 40;
  static constexpr int OFF_TMEM = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_TMEM + 16;
};

// barrier slots
enum {
  B_RAW_FULL = 0,    // [RS <= 4]
  B_RAW_EMPTY = 4,   // [RS <= 4]
  B_Q_FULL = 8,      // the piece's Q rows are in TMEM (4 softmax warps)
  B_K_FULL = 10,     // [2] key operand buffers
  B_K_FREE = 12,     // [2]
  B_V_FULL = 14,     // [2] value operand buffers
  B_V_FREE = 16,     // [2]
  B_S_FULL = 18,     // [2]
  B_P_FULL = 22,     // [2] P of the tile stored in TMEM over its S buffer (the softmax is done with that S)
  B_SC_FULL = 26,    // [2]
  B_SC_FREE = 28,    // [2]
  B_O_DONE = 30,
  B_O_FREE = 31,
  B_FINAL = 32,      // the MMA thread's last commit: every tcgen05.mma done before TMEM is released
};

struct PrefillParams {
  const uint8_t* cache;
  int block_size;
  int64_t block_stride, head_stride;
  const int32_t* block_row;  // block table row of the sequence
  int n;                     // context length (the chunk's keys included)
  int qlen;
  int vis_base;              // last key query token 0 sees: n - qlen + tokens after the keys (may exceed n - 1)
  int nq, nkv, group;
  int mt_per_kv;             // M-tiles per KV head
  const uint8_t* qprep;      // [nkv][mt_per_kv][65536 B] operand-layout Q tiles
  const float* qscale;       // [nkv][mt_per_kv][128]
  float* part_o;             // [qlen][nq][parts][256]
  float* part_lse;           // [qlen][nq][parts]
  int parts;
  int64_t total_tiles;       // (M-tile, key-tile) pairs over all KV heads
};

// ---------------------------------------------------------------------------------------------------- PTX wrappers
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
// instruction descriptor: fp32 accumulate, fp16 A and B, A K-major, B K- or MN-major, M x N
__host__ __device__ constexpr uint32_t f16_idesc(int m, int n, bool b_mn_major) {
  return (1u << 4) | (0u << 7) | (0u << 10) | (0u << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// byte offset of 16-byte chunk `chunk` (0..7) of row `row` inside a 128B-swizzled tile of 8-row groups
__device__ __forceinline__ uint32_t sw128_off(int row, int chunk) {
  return (row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4);
}

// position of channel c inside its group of 8 in the operand order [0 4 1 5 2 6 3 7]
__device__ __forceinline__ int perm8_pos(int c) { return 2 * (c & 3) + ((c >> 2) & 1); }

// ---------------------------------------------------------------------------------------------------- schedule
// Key tiles the rows of M-tile m (of any KV head) attend to: keys 0 .. min(n - 1, vis_base + i_hi).
__device__ __forceinline__ int mtile_key_tiles(const PrefillParams& p, int m) {
  const int rows = p.qlen * p.group;
  const int r_hi = min(rows - 1, m * PF_BM + PF_BM - 1);
  const int keys = min(p.n, p.vis_base + r_hi / p.group + 1);
  return (keys + PF_BN - 1) / PF_BN;
}

// Walk of the tiles of this CTA: [g_begin, g_end) of the flattened (KV head, M-tile, key tile) space.
struct Walk {
  int kvh, m, kt, kt_end;  // current M-tile and key tile
  int piece;               // index of this CTA's piece of the M-tile
  bool first_of_piece, last_of_piece, new_mtile;
};

struct Sched {
  const PrefillParams* p;
  int64_t g, g_end;  // current / end global tile index
  int kvh, m;        // current M-tile
  int64_t m_start;   // global index of the M-tile's first tile
  int m_tiles;       // key tiles of the current M-tile
  int first_kt;      // first key tile of this CTA inside the current M-tile
  int cta, ctas;

  __device__ void init(const PrefillParams& prm, int cta_, int ctas_) {
    p = &prm;
    cta = cta_;
    ctas = ctas_;
    g = prm.total_tiles * cta / ctas;
    g_end = prm.total_tiles * (cta + 1) / ctas;
    kvh = 0;
    m = 0;
    m_start = 0;
    m_tiles = mtile_key_tiles(prm, 0);
    // advance to the M-tile holding g (M-tiles of each KV head in order)
    while (m_start + m_tiles <= g) {
      m_start += m_tiles;
      if (++m == prm.mt_per_kv) {
        m = 0;
        ++kvh;
      }
      m_tiles = mtile_key_tiles(prm, m);
    }
    first_kt = static_cast<int>(g - m_start);
  }
  __device__ bool done() const { return g >= g_end; }
  // piece index of this CTA inside the current M-tile: CTAs whose range starts inside it before this one
  __device__ int piece() const {
    const int64_t start = m_start + first_kt;
    // the CTA covering m_start: largest c with total * c / ctas <= m_start
    int c0 = static_cast<int>((m_start * ctas) / p->total_tiles);
    while (c0 + 1 < ctas && p->total_tiles * (c0 + 1) / ctas <= m_start) ++c0;
    while (c0 > 0 && p->total_tiles * c0 / ctas > m_start) --c0;
    (void)start;
    return cta - c0;
  }
  __device__ Walk current() const {
    Walk w;
    w.kvh = kvh;
    w.m = m;
    w.kt = static_cast<int>(g - m_start);
    w.kt_end = m_tiles;
    w.piece = piece();
    w.first_of_piece = w.kt == first_kt;
    w.last_of_piece = (w.kt + 1 == m_tiles) || (g + 1 == g_end);
    w.new_mtile = w.first_of_piece;
    return w;
  }
  __device__ void next() {
    ++g;
    if (g < g_end && g - m_start >= m_tiles) {
      m_start += m_tiles;
      if (++m == p->mt_per_kv) {
        m = 0;
        ++kvh;
      }
      m_tiles = mtile_key_tiles(*p, m);
      first_kt = 0;
    }
  }
};

// ---------------------------------------------------------------------------------------------------- Q prep
// One warp per (M-tile row): rotate (unless already rotated), scale to fp16 by a per-row power of two, write the row
// (512 bytes, the channel order of the key operand) into its M-tile, ready to be stored as the A operand in TMEM
// (lane = row, two fp16 per column); record the row's score scale; padding rows become zeros. Also sets every lse
// partial to -inf (absent pieces).
template <int FMT, int DT>
__global__ void __launch_bounds__(256) prefill_qprep_kernel(const void* q, int64_t q_st, int64_t q_sh, int qlen,
                                                            int nq, int nkv, int group, int mt_per_kv,
                                                            const uint32_t* sign_bits, int q_rotated, float qk_scale,
                                                            uint8_t* qprep, float* qscale, float* part_lse,
                                                            int64_t lse_count) {
  const int lane = threadIdx.x & 31;
  const int64_t row_id = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x; i < lse_count;
       i += static_cast<int64_t>(gridDim.x) * 256)
    part_lse[i] = -INFINITY;
  const int64_t total_rows = static_cast<int64_t>(nkv) * mt_per_kv * PF_BM;
  if (row_id >= total_rows) return;
  const int kvh = static_cast<int>(row_id / (static_cast<int64_t>(mt_per_kv) * PF_BM));
  const int mr = static_cast<int>(row_id % (static_cast<int64_t>(mt_per_kv) * PF_BM));  // row inside the KV head
  const int m = mr / PF_BM, r = mr % PF_BM;
  uint8_t* tile = qprep + (static_cast<int64_t>(kvh) * mt_per_kv + m) * 65536;
  float* qs = qscale + (static_cast<int64_t>(kvh) * mt_per_kv + m) * PF_BM;
  float x[8];
  int ex = 0;
  if (mr < qlen * group) {
    using EL = Elem<DT>;
    const int tok = mr / group, qh = kvh * group + mr % group;
    const typename EL::T* src = reinterpret_cast<const typename EL::T*>(q) + tok * q_st + qh * q_sh + lane * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = EL::to_f(src[i]);
    if (!q_rotated) {
      apply_signs<8>(x, sign_bits, lane);
      warp_wht<8>(x, lane);
    }
    float am = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(x[i]));
    am = warp_max(am);
    if (am > 0.f) {
      frexpf(am, &ex);
      ex = 14 - ex;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = 0.f;
  }
  // lane holds channels 8 lane .. 8 lane + 7 = one operand chunk (K-block lane / 8, chunk lane % 8)
  __half h[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int pos = FMT == FMT_INT4 ? perm8_pos(i) : i;
    h[pos] = __float2half_rn(ldexpf(x[i], ex));
  }
  uint4 v;
  v.x = *reinterpret_cast<uint32_t*>(&h[0]);
  v.y = *reinterpret_cast<uint32_t*>(&h[2]);
  v.z = *reinterpret_cast<uint32_t*>(&h[4]);
  v.w = *reinterpret_cast<uint32_t*>(&h[6]);
  *reinterpret_cast<uint4*>(tile + r * (PF_HS * 2) + lane * 16) = v;
  if (lane == 0) qs[r] = mr < qlen * group ? ldexpf(qk_scale, -ex) : 0.f;
}

// ---------------------------------------------------------------------------------------------------- main kernel
template <int FMT>
__global__ void __launch_bounds__(PF_THREADS, 1) prefill_kernel(const PrefillParams p) {
  using C = PfCfg<FMT>;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_TMEM);
  float* sc = reinterpret_cast<float*>(smem + C::OFF_SC);  // [buf][ks 64 | vs 64]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < C::RS; ++s) {
      mbar_init(&bars[B_RAW_FULL + s], 1);
      mbar_init(&bars[B_RAW_EMPTY + s], 4);
    }
    mbar_init(&bars[B_Q_FULL], 8);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars[B_K_FULL + b], 2);
      mbar_init(&bars[B_K_FREE + b], 1);
      mbar_init(&bars[B_V_FULL + b], 2);
      mbar_init(&bars[B_V_FREE + b], 1);
      mbar_init(&bars[B_S_FULL + b], 1);
      mbar_init(&bars[B_P_FULL + b], 8);
      mbar_init(&bars[B_SC_FULL + b], 4);
      mbar_init(&bars[B_SC_FREE + b], 8);
    }
    mbar_init(&bars[B_O_DONE], 1);
    mbar_init(&bars[B_O_FREE], 8);
    mbar_init(&bars[B_FINAL], 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // S buffers: columns [0, 64), [64, 128); P of a tile (fp16 pairs) is stored over the first 32 columns of its S
  // buffer as the A operand of the PV MMA (no shared-memory round trip)
  const uint32_t tm_s[2] = {tmem, tmem + 64};
  const uint32_t tm_q = tmem + 128;            // Q (A operand of S = Q K^T): columns [128, 256)
  const uint32_t tm_o = tmem + 256;            // O: columns [256, 512)

  Sched sch;
  sch.init(p, blockIdx.x, gridDim.x);
  bool failed = false;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      int64_t j = 0;        // global tile counter (raw ring)
      for (; !sch.done() && !failed; sch.next(), ++j) {
        const Walk w = sch.current();
        const int stage = static_cast<int>(j % C::RS);
        if (j >= C::RS) failed |= !mbar_wait_bounded(&bars[B_RAW_EMPTY + stage], ((j / C::RS) - 1) & 1);
        const int tok_begin = w.kt * PF_BN;
        const int groups = (min(tok_begin + PF_BN, p.n) - tok_begin + 15) >> 4;
        mbar_arrive_expect_tx(&bars[B_RAW_FULL + stage], static_cast<uint32_t>(groups * 16 * C::CELL));
        uint8_t* dst = smem + C::OFF_RAW + stage * C::RAW_BYTES;
        const uint8_t* head_base = p.cache + static_cast<int64_t>(w.kvh) * p.head_stride;
        for (int gi = 0; gi < groups;) {
          const int tok = tok_begin + gi * 16;
          const int blk = __ldg(p.block_row + tok / p.block_size);
          const int in_blk = tok % p.block_size;
          const int run = min(groups - gi, (p.block_size - in_blk) >> 4);
          bulk_g2s(dst + gi * 16 * C::CELL,
                   head_base + static_cast<int64_t>(blk) * p.block_stride + static_cast<int64_t>(in_blk) * C::CELL,
                   static_cast<uint32_t>(run * 16 * C::CELL), &bars[B_RAW_FULL + stage]);
          gi += run;
        }
      }
      // the copies in flight land before the CTA's shared memory can go away
      for (int64_t k = (j > C::RS ? j - C::RS : 0); k < j; ++k)
        mbar_wait_bounded(&bars[B_RAW_FULL + (k % C::RS)], (k / C::RS) & 1, 100000000ull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_QK = f16_idesc(PF_BM, PF_BN, false);
      constexpr uint32_t ID_PV = f16_idesc(PF_BM, PF_HS, true);
      const uint32_t k_base = smem_u32(smem + C::OFF_K), v_base = smem_u32(smem + C::OFF_V);
      int64_t j = 0;
      int qcount = 0, pieces = 0;
      int64_t pv_pending = -1;  // tile whose PV is still to be issued
      bool pv_first = false, pv_last = false;
      auto issue_pv = [&](int64_t t, bool first) {
        const int b = static_cast<int>(t & 1);
        failed |= !mbar_wait_bounded(&bars[B_V_FULL + b], (t >> 1) & 1);
        failed |= !mbar_wait_bounded(&bars[B_P_FULL + b], (t >> 1) & 1);
        tc_fence_after();
        const uint32_t vb = v_base + b * 32768;
        // P(t) in TMEM, K step s (16 keys) = 8 columns; S(t + 2) overwrites these columns with MMAs issued after
        // these (the tcgen05.mma of one thread execute in issue order)
#pragma unroll
        for (int s = 0; s < 4; ++s)
          umma_f16_ts(tm_o, tm_s[b] + 8 * s, sw128_desc(vb + 2 * s * 1024, 8192, 1024), ID_PV,
                      (first && s == 0) ? 0u : 1u);
        umma_commit(&bars[B_V_FREE + b]);
        umma_commit(&bars[B_O_DONE]);
      };
      for (; !sch.done() && !failed; sch.next(), ++j) {
        const Walk w = sch.current();
        if (w.new_mtile) {
          failed |= !mbar_wait_bounded(&bars[B_Q_FULL], qcount & 1);
          ++qcount;
        }
        // S(j) = Q K(j)^T
        const int b = static_cast<int>(j & 1);
        failed |= !mbar_wait_bounded(&bars[B_K_FULL + b], (j >> 1) & 1);
        // S buffer b last held S(j - 2) and P(j - 2): the PV of that tile, issued before these MMAs, waited for the
        // softmax to finish with it
        tc_fence_after();
        const uint32_t kb = k_base + b * 32768;
#pragma unroll
        for (int s = 0; s < 16; ++s)  // K step s: 16 channels = 8 TMEM columns of Q
          umma_f16_ts(tm_s[b], tm_q + 8 * s, sw128_desc(kb + (s >> 2) * 8192 + (s & 3) * 32, 16, 1024), ID_QK,
                      s > 0 ? 1u : 0u);
        umma_commit(&bars[B_K_FREE + b]);
        umma_commit(&bars[B_S_FULL + b]);
        // Q of this piece is free once S of its last tile is complete: the softmax, which waits for that S before
        // it stores the next piece's Q, needs no other signal
        // O += P(j-1) V(j-1), one tile behind so the softmax of tile j overlaps it
        if (pv_pending >= 0) {
          issue_pv(pv_pending, pv_first);
          pv_pending = -1;
        }
        if (w.first_of_piece && pieces > 0) {
          // O is overwritten by this piece's first PV: the previous piece's epilogue must have read it
          failed |= !mbar_wait_bounded(&bars[B_O_FREE], (pieces - 1) & 1);
        }
        if (w.first_of_piece) ++pieces;
        pv_pending = j;
        pv_first = w.first_of_piece;
        pv_last = w.last_of_piece;
        if (w.last_of_piece) {  // the epilogue waits for this PV: issue it now
          issue_pv(pv_pending, pv_first);
          pv_pending = -1;
        }
      }
      (void)pv_last;
      umma_commit(&bars[B_FINAL]);
      mbar_wait_bounded(&bars[B_FINAL], 0, 100000000ull);
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------------ dequant (warps 2..5)
    // keys:   K_op = (u - zp) * ks * 2^-F  (F: exponent of the tile's largest key scale; 2^F goes to the softmax)
    // values: V_op = (u - zp) * vs * 2^-E  (E: running exponent of the piece's largest value scale; O is rescaled by
    //         the softmax when E grows). Every operand is then <= 15 in magnitude and exact up to one fp16 rounding.
    const int dq = tid - 64;     // 0..127
    const int kr = dq & 63;      // key row of the tile
    const bool is_k = dq < 64;   // warps 2, 3: keys; warps 4, 5: values
    const int wpair = (warp - 2) & 1;
    uint8_t* const kop0 = smem + C::OFF_K;
    uint8_t* const vop0 = smem + C::OFF_V;
    float* xch = reinterpret_cast<float*>(smem + C::OFF_XCH) + (is_k ? 0 : 4);
    int e_run_v = -1000;
    int64_t j = 0;
    for (; !sch.done() && !failed; sch.next(), ++j) {
      const Walk w = sch.current();
      const int stage = static_cast<int>(j % C::RS);
      const int b = static_cast<int>(j & 1);
      if (w.first_of_piece) e_run_v = -1000;
      failed |= !mbar_wait_bounded(&bars[B_RAW_FULL + stage], (j / C::RS) & 1);
      const uint8_t* cell = smem + C::OFF_RAW + stage * C::RAW_BYTES + kr * C::CELL;
      const int tok = w.kt * PF_BN + kr;
      const uint32_t sw = *reinterpret_cast<const uint32_t*>(cell + (is_k ? C::KB : C::KB + 4 + PF_HS / 2));
      const float scl = tok < p.n ? __uint_as_float((FMT == FMT_INT4 || !is_k) ? (sw & 0xFFFFFFF0u) : sw) : 0.f;
      const uint32_t zp = (FMT == FMT_INT4 || !is_k) ? (sw & 0xFu) : 0u;
      // tile maximum of this half's scales (two warps)
      const float wm = warp_max(scl);
      if (lane == 0) xch[b * 2 + wpair] = wm;
      // the two warps of this half leave together if either gave up a wait (a bar.sync has no time bound)
      if (named_bar_or(is_k ? 1 : 2, 64, failed)) {
        failed = true;
        break;
      }
      const float tmax = fmaxf(xch[b * 2], xch[b * 2 + 1]);
      int ex = -1000;
      if (tmax > 0.f) frexpf(tmax, &ex);  // tmax < 2^ex
      if (!is_k) {
        e_run_v = max(e_run_v, ex);
        ex = e_run_v;
      }
      const float q = ex == -1000 ? 0.f : ldexpf(scl, -ex);
      const __half2 qh2 = __floats2half2_rn(q, q);
      const uint32_t q2 = *reinterpret_cast<const uint32_t*>(&qh2);
      if (j >= 2) failed |= !mbar_wait_bounded(&bars[B_SC_FREE + b], ((j >> 1) - 1) & 1);
      if (kr == 0 && (warp == 2 || warp == 4)) {
        float* scb = reinterpret_cast<float*>(smem + C::OFF_SC) + b * 4;
        if (is_k)
          scb[0] = ex == -1000 ? 0.f : ldexpf(1.f, ex);
        else
          scb[1] = __int_as_float(ex);
      }
      // the softmax needs only these factors: release them now, not after the (longer) operand conversion
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[B_SC_FULL + b]);
      const uint32_t lo_b = 0x64006400u | zp | (zp << 16), hi_b = 0xD400D400u | (zp << 4) | (zp << 20);
      // Each thread converts its key row: every 8-byte load of the row is issued before any conversion (the
      // stores below could alias them for the compiler, which would otherwise serialise load -> convert -> store
      // per word). Cells are 8-byte aligned (264 / 392 B) and the 8-byte loads of 16 consecutive rows fall in 16
      // distinct bank pairs; the stores of 8 consecutive rows hit 8 distinct 16-byte bank groups (swizzle).
      const uint32_t rbase = (kr >> 3) * 1024 + (kr & 7) * 128, rxor = (kr & 7) << 4;
      if (is_k) {
        if (j >= 2) failed |= !mbar_wait_bounded(&bars[B_K_FREE + b], ((j >> 1) - 1) & 1);
        uint8_t* const kop = kop0 + b * 32768;
        if constexpr (FMT == FMT_INT4) {
#pragma unroll 1
          for (int kb = 0; kb < 4; ++kb) {  // K-block kb: words 8 kb .. 8 kb + 7 (channels 64 kb ..)
            uint2 kw[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) kw[k] = *reinterpret_cast<const uint2*>(cell + 32 * kb + 8 * k);
            uint8_t* const dst = kop + kb * 8192 + rbase;
#pragma unroll
            for (int i = 0; i < 8; ++i) {  // word: channels 8 (8 kb + i) .. + 7 = chunk i of the K-block
              const uint32_t x = (i & 1) ? kw[i >> 1].y : kw[i >> 1].x;
              const uint32_t x8 = x >> 8;
              uint4 v;
              v.x = hmul2_u32(hsub2_u32(lop3_and_or(x, 0x000F000Fu, 0x64006400u), lo_b), q2);  // channels 0, 4
              v.y = hmul2_u32(hfma2_u32(lop3_and_or(x, 0x00F000F0u, 0x64006400u), 0x2C002C00u, hi_b), q2);  // 1, 5
              v.z = hmul2_u32(hsub2_u32(lop3_and_or(x8, 0x000F000Fu, 0x64006400u), lo_b), q2);  // 2, 6
              v.w = hmul2_u32(hfma2_u32(lop3_and_or(x8, 0x00F000F0u, 0x64006400u), 0x2C002C00u, hi_b), q2);  // 3, 7
              *reinterpret_cast<uint4*>(dst + ((static_cast<uint32_t>(i) << 4) ^ rxor)) = v;
            }
          }
        } else {
#pragma unroll 1
          for (int h = 0; h < 4; ++h) {  // K-block h: codes 64 h .. 64 h + 63, 8 loads of 8 bytes in flight
            uint2 kw[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) kw[k] = *reinterpret_cast<const uint2*>(cell + 64 * h + 8 * k);
#pragma unroll
            for (int k = 0; k < 8; ++k) {  // 8 channels 8 C8 .. 8 C8 + 7 (two words)
              const int C8 = 8 * h + k;
              const uint32_t a = kw[k].x ^ 0x80808080u, c = kw[k].y ^ 0x80808080u;
              uint4 v;  // (1152 + code) - 1152 = code, exact; then the scale
              v.x = hmul2_u32(hsub2_u32(prmt(a, 0x64646464u, 0x4140u), 0x64806480u), q2);
              v.y = hmul2_u32(hsub2_u32(prmt(a, 0x64646464u, 0x4342u), 0x64806480u), q2);
              v.z = hmul2_u32(hsub2_u32(prmt(c, 0x64646464u, 0x4140u), 0x64806480u), q2);
              v.w = hmul2_u32(hsub2_u32(prmt(c, 0x64646464u, 0x4342u), 0x64806480u), q2);
              *reinterpret_cast<uint4*>(kop + (C8 >> 3) * 8192 +
                                        (rbase + ((static_cast<uint32_t>(C8 & 7) << 4) ^ rxor))) = v;
            }
          }
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[B_K_FULL + b]);
      } else {
        if (j >= 2) failed |= !mbar_wait_bounded(&bars[B_V_FREE + b], ((j >> 1) - 1) & 1);
        uint8_t* const vop = vop0 + b * 32768;
        // the value words start 4 bytes past an 8-byte boundary: 8-byte loads from the key scale on give the pairs
        // (key scale, V0), (V1, V2), ..., (V31, value scale)
#pragma unroll 1
        for (int kb = 0; kb < 4; ++kb) {  // N-block kb: words 8 kb .. 8 kb + 7; loads at 8-byte offsets 4 kb ..
          uint2 vw[5];
#pragma unroll
          for (int k = 0; k < 5; ++k) vw[k] = *reinterpret_cast<const uint2*>(cell + C::KB + 32 * kb + 8 * k);
          uint8_t* const dst = vop + kb * 8192 + rbase;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint32_t x = (i & 1) ? vw[(i + 1) >> 1].x : vw[i >> 1].y;
            const uint32_t x8 = x >> 8;
            uint4 v;
            v.x = hmul2_u32(hsub2_u32(lop3_and_or(x, 0x000F000Fu, 0x64006400u), lo_b), q2);
            v.y = hmul2_u32(hfma2_u32(lop3_and_or(x, 0x00F000F0u, 0x64006400u), 0x2C002C00u, hi_b), q2);
            v.z = hmul2_u32(hsub2_u32(lop3_and_or(x8, 0x000F000Fu, 0x64006400u), lo_b), q2);
            v.w = hmul2_u32(hfma2_u32(lop3_and_or(x8, 0x00F000F0u, 0x64006400u), 0x2C002C00u, hi_b), q2);
            *reinterpret_cast<uint4*>(dst + ((static_cast<uint32_t>(i) << 4) ^ rxor)) = v;
          }
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[B_V_FULL + b]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[B_RAW_EMPTY + stage]);
    }
  } else {
    // ------------------------------------------------------------------ softmax / epilogue (warps 6..13)
    // Two warps per TMEM lane quarter (32 query rows): warps 6-9 take keys 0-31 of every tile and channels 0-127 of
    // O, warps 10-13 keys 32-63 and channels 128-255. The two threads of a row agree on its maximum through shared
    // memory (a named barrier per pair of warps) and add their partial sums in the epilogue.
    const int quarter = warp & 3;
    const int half = (warp - 6) >> 2;
    const int row = quarter * 32 + lane;  // TMEM lane = M-tile row
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const int pair_bar = 3 + quarter;     // named barriers 1, 2: dequant pairs
    float* hmax = reinterpret_cast<float*>(smem + C::OFF_HX);  // [buffer][half][row]
    float* hsum = hmax + 2 * 2 * 128;                              // [half][row]
    int64_t j = 0;
    // PV completions seen so far. O_DONE completes one phase per tile (its PV); a parity wait is exact only while
    // the barrier is at most one phase ahead of the phase waited for, so the phases are consumed in order: PV(j - 1)
    // before P(j) is stored (S_FULL(j) already implies PV(j - 2)), PV(j) in the epilogue.
    int64_t pv_seen = 0;
    auto wait_pv = [&](int64_t t) {  // until PV(t) is complete
      for (; pv_seen <= t; ++pv_seen) failed |= !mbar_wait_bounded(&bars[B_O_DONE], static_cast<uint32_t>(pv_seen & 1));
    };
    float m_used = -INFINITY, l = 0.f, qsc = 0.f;
    int e_used = -1000, lim = -1, tok = 0, qh = 0;
    bool row_ok = false;
    int64_t t_in_piece = 0;
    for (; !sch.done() && !failed; sch.next(), ++j) {
      const Walk w = sch.current();
      const int b = static_cast<int>(j & 1);
      if (w.new_mtile) {
        // this thread's half of its row of the piece's Q tile -> TMEM columns 128 + [64 half, 64 half + 64) of its
        // lane (the previous piece's QKs are complete: this thread consumed the S of its last tile)
        const int64_t mt = static_cast<int64_t>(w.kvh) * p.mt_per_kv + w.m;
        const uint4* qrow = reinterpret_cast<const uint4*>(p.qprep + mt * 65536 + row * (PF_HS * 2));
#pragma unroll 1
        for (int c0 = 64 * half; c0 < 64 * half + 64; c0 += 32) {
          uint32_t qw[32];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint4 v = __ldg(qrow + c0 / 4 + i);
            qw[4 * i] = v.x;
            qw[4 * i + 1] = v.y;
            qw[4 * i + 2] = v.z;
            qw[4 * i + 3] = v.w;
          }
          tmem_st32u(tm_q + lane_off + c0, qw);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[B_Q_FULL]);
        qsc = p.qscale[mt * PF_BM + row];
        const int rg = w.m * PF_BM + row;
        row_ok = rg < p.qlen * p.group;
        tok = rg / p.group;
        qh = w.kvh * p.group + rg % p.group;
        lim = row_ok ? min(p.n - 1, p.vis_base + tok) : -1;
      }
      if (w.first_of_piece) {
        m_used = -INFINITY;
        l = 0.f;
        e_used = -1000;
        t_in_piece = 0;
      }
      // this row's scores for keys 32 half .. 32 half + 31 of the tile
      failed |= !mbar_wait_bounded(&bars[B_S_FULL + b], (j >> 1) & 1);
      tc_fence_after();
      float s[32];
      tmem_ld32(tm_s[b] + lane_off + 32 * half, s);
      failed |= !mbar_wait_bounded(&bars[B_SC_FULL + b], (j >> 1) & 1);
      const float* scb = reinterpret_cast<const float*>(smem + C::OFF_SC) + b * 4;
      const float qs_t = qsc * scb[0];               // x 2^F of the key operand
      const int ev = __float_as_int(scb[1]);         // value exponent of this tile's operand
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[B_SC_FREE + b]);
      const int key0 = w.kt * PF_BN + 32 * half;
      const bool masked = w.kt * PF_BN + PF_BN - 1 > min(p.n - 1, p.vis_base);  // some row cannot see some key
      if (masked) {
#pragma unroll
        for (int c = 0; c < 32; ++c)
          if (key0 + c > lim) s[c] = -INFINITY;
      }
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 32; ++c) mx = fmaxf(mx, s[c]);
      hmax[(b * 2 + half) * 128 + row] = mx;
      // the pair leaves together if either gave up a wait (a bar.sync has no time bound)
      if (named_bar_or(pair_bar, 64, failed)) {
        failed = true;
        break;
      }
      mx = fmaxf(mx, hmax[(b * 2 + (half ^ 1)) * 128 + row]);
      const float mrow = mx * qs_t;
      const bool grow = mrow > m_used + PF_SLACK;  // the same in both threads of the row
      const bool vgrow = ev > e_used;              // the same for every thread
      if (__any_sync(0xffffffffu, grow) || vgrow) {
        // rescale this thread's half of the row's O in TMEM (after the previous PV of the piece completed)
        const float m_new = grow ? mrow : m_used;
        const float alpha = m_new == m_used ? 1.f : exp2f(m_used - m_new);
        const float o_range = e_used == -1000 ? 0.f : ldexpf(1.f, e_used - ev);
        const float ao = alpha * o_range;
        if (t_in_piece > 0) {
          wait_pv(j - 1);
          tc_fence_after();
#pragma unroll 1
          for (int c0 = 128 * half; c0 < 128 * half + 128; c0 += 32) {
            float o[32];
            tmem_ld32(tm_o + lane_off + c0, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= ao;
            tmem_st32(tm_o + lane_off + c0, o);
          }
        }
        l *= alpha;
        m_used = m_new;
        e_used = ev;
      }
      // P = 2^(s qs_t - m) <= 2^8 in fp16
      const float base = m_used == -INFINITY ? 0.f : m_used;
      float lsum = 0.f;
      uint32_t pw[16];
      if (masked) {
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          const float p0 = s[c] == -INFINITY ? 0.f : fast_exp2(fmaf(s[c], qs_t, -base));
          const float p1 = s[c + 1] == -INFINITY ? 0.f : fast_exp2(fmaf(s[c + 1], qs_t, -base));
          lsum += p0 + p1;
          const __half2 h = __floats2half2_rn(p0, p1);
          pw[c >> 1] = *reinterpret_cast<const uint32_t*>(&h);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          const float p0 = fast_exp2(fmaf(s[c], qs_t, -base));
          const float p1 = fast_exp2(fmaf(s[c + 1], qs_t, -base));
          lsum += p0 + p1;
          const __half2 h = __floats2half2_rn(p0, p1);
          pw[c >> 1] = *reinterpret_cast<const uint32_t*>(&h);
        }
      }
      l += lsum;
      wait_pv(j - 1);
      // P -> TMEM over columns 16 half + [0, 16) of this tile's S buffer: the A operand of its PV MMA
      tmem_st16u(tm_s[b] + lane_off + 16 * half, pw);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[B_P_FULL + b]);
      ++t_in_piece;

      if (w.last_of_piece) {
        // epilogue: O of this piece -> normalised fp32 partial (channel order restored) + base-2 lse
        hsum[half * 128 + row] = l;
        if (named_bar_or(pair_bar, 64, failed)) {
          failed = true;
          break;
        }
        const float l_row = l + hsum[(half ^ 1) * 128 + row];
        wait_pv(j);
        tc_fence_after();
        const float o_unit = e_used == -1000 ? 0.f : ldexpf(1.f, e_used);
        const float inv = l_row > 0.f ? o_unit / l_row : 0.f;
        const int64_t prow_i = (static_cast<int64_t>(tok) * p.nq + qh) * p.parts + w.piece;
#pragma unroll 1
        for (int c0 = 128 * half; c0 < 128 * half + 128; c0 += 32) {
          float o[32];
          tmem_ld32(tm_o + lane_off + c0, o);
          if (row_ok && w.piece < p.parts) {
            float* dst = p.part_o + prow_i * PF_HS + c0;
#pragma unroll
            for (int g8 = 0; g8 < 4; ++g8) {  // 8 channels per group, operand order [0 4 1 5 2 6 3 7]
              const float* og = o + 8 * g8;
              reinterpret_cast<float4*>(dst + 8 * g8)[0] = make_float4(og[0] * inv, og[2] * inv, og[4] * inv, og[6] * inv);
              reinterpret_cast<float4*>(dst + 8 * g8)[1] = make_float4(og[1] * inv, og[3] * inv, og[5] * inv, og[7] * inv);
            }
          }
        }
        if (half == 0 && row_ok && w.piece < p.parts) p.part_lse[prow_i] = l_row > 0.f ? m_used + log2f(l_row) : -INFINITY;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[B_O_FREE]);
      }
    }
  }

  if (failed) atomicCAS(&g_device_error, DEV_ERR_NONE, DEV_ERR_WAIT_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

}  // namespace qp

using namespace qp;

// Workspace layout of qp_prefill: [qprep nkv*mt*64 KB][qscale nkv*mt*128 f32][part_o qlen*nq*parts*256 f32]
// [part_lse qlen*nq*parts f32], each 256-byte aligned.
static int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }

static void prefill_plan(int qlen, int n, int after, int nkv, int group, int sms, int* mt_per_kv, int64_t* total,
                         int* ctas, int* parts) {
  const int rows = qlen * group;
  *mt_per_kv = (rows + PF_BM - 1) / PF_BM;
  int64_t tot = 0;
  int maxt = 0;
  for (int m = 0; m < *mt_per_kv; ++m) {
    const int r_hi = std::min(rows - 1, m * PF_BM + PF_BM - 1);
    const int t = (std::min(n, n - qlen + after + r_hi / group + 1) + PF_BN - 1) / PF_BN;
    tot += t;
    maxt = std::max(maxt, t);
  }
  tot *= nkv;
  *total = tot;
  *ctas = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(sms, tot)));
  const int64_t per = std::max<int64_t>(1, tot / *ctas);
  *parts = static_cast<int>(std::min<int64_t>(*ctas, (maxt + per - 1) / per + 1));
}

extern "C" int64_t qp_prefill_workspace_bytes(int qlen, int n, int num_q_heads, int num_kv_heads, int head_size,
                                              int tokens_after_keys) {
  if (qlen <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads || tokens_after_keys < 0) return 0;
  const int after = std::min(tokens_after_keys, qlen);
  int mt, ctas, parts;
  int64_t total;
  prefill_plan(qlen, n, after, num_kv_heads, num_q_heads / num_kv_heads, device_sm_count(), &mt, &total, &ctas, &parts);
  const int64_t nt = static_cast<int64_t>(num_kv_heads) * mt;
  return align256(nt * 65536) + align256(nt * PF_BM * 4) +
         align256(static_cast<int64_t>(qlen) * num_q_heads * parts * head_size * 4) +
         align256(static_cast<int64_t>(qlen) * num_q_heads * parts * 4);
}

template <int FMT>
static int launch_prefill_main(const PrefillParams& pp, int ctas, cudaStream_t st) {
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(prefill_kernel<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         PfCfg<FMT>::BYTES);
    if (e != cudaSuccess) return set_error(QP_ERR_CUDA, "prefill smem attribute: %s", cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  prefill_kernel<FMT><<<ctas, PF_THREADS, PfCfg<FMT>::BYTES, st>>>(pp);
  return check_launch("prefill");
}

// declared in qp_decode.cu
extern "C" int qp_merge_attn_partials(int dtype, int head_size, int64_t num_tokens, int num_q_heads, int num_parts,
                                      const float* part_o, int64_t po_stride_token, int64_t po_stride_head,
                                      int64_t po_stride_part, const float* part_lse, int64_t pl_stride_token,
                                      int64_t pl_stride_head, int64_t pl_stride_part, int out_mode, void* out,
                                      int64_t out_stride_token, int64_t out_stride_head, float* lse_out,
                                      const uint32_t* rht_sign_bits, void* stream);

extern "C" int qp_prefill(int fmt, int dtype, const void* q, int64_t q_stride_token, int64_t q_stride_head, void* out,
                          int64_t out_stride_token, int64_t out_stride_head, int qlen, int n,
                          const int32_t* block_row, const void* cache, int block_size, int64_t block_stride,
                          int64_t head_stride, int64_t slot_stride, int64_t k_off, int64_t ks_off, int64_t v_off,
                          int64_t vs_off, int num_q_heads, int num_kv_heads, int head_size, float softmax_scale,
                          const uint32_t* rht_sign_bits, int q_rotated, int tokens_after_keys, int out_mode,
                          float* lse_out, void* workspace, int64_t workspace_bytes, void* stream) {
  if (fmt != FMT_INT4 && fmt != FMT_K8V4) return set_error(QP_ERR_UNSUPPORTED, "prefill: format %d", fmt);
  if (dtype != DT_BF16 && dtype != DT_F16) return set_error(QP_ERR_UNSUPPORTED, "prefill: dtype %d", dtype);
  if (head_size != PF_HS) return set_error(QP_ERR_UNSUPPORTED, "prefill: head size %d (this build: 256)", head_size);
  const int after = std::min(std::max(tokens_after_keys, 0), std::max(qlen, 0));  // >= qlen: nothing masked
  if (tokens_after_keys < 0 || qlen < 0 || n < qlen - after || (qlen > 0 && n <= 0) || num_kv_heads <= 0 ||
      num_q_heads <= 0 || num_q_heads % num_kv_heads)
    return set_error(QP_ERR_INVALID, "prefill: bad sizes (qlen %d, n %d, heads %d/%d)", qlen, n, num_q_heads,
                     num_kv_heads);
  if (qlen == 0) return QP_OK;
  if (out_mode != 0 && out_mode != 1) return set_error(QP_ERR_INVALID, "prefill: out_mode %d", out_mode);
  const int cell = fmt == FMT_INT4 ? PF_HS + 8 : PF_HS * 3 / 2 + 8;
  const int kb = fmt == FMT_INT4 ? PF_HS / 2 : PF_HS;
  if (slot_stride != cell)
    return set_error(QP_ERR_LAYOUT, "prefill: cells of a (block, head) must be contiguous (slot stride %lld)",
                     (long long)slot_stride);
  if (k_off != 0 || ks_off != kb || v_off != kb + 4 || vs_off != kb + 4 + PF_HS / 2)
    return set_error(QP_ERR_LAYOUT, "prefill: unexpected cell field offsets");
  if (block_size <= 0 || block_size % 16 || (reinterpret_cast<uintptr_t>(cache) & 15) || (block_stride & 15) ||
      (head_stride & 15))
    return set_error(QP_ERR_LAYOUT, "prefill: block size must be a multiple of 16 and the cache 16-byte aligned");
  if (!q || !out || !block_row || !cache || !rht_sign_bits || !workspace)
    return set_error(QP_ERR_INVALID, "prefill: null pointer");
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return set_error(QP_ERR_WORKSPACE, "prefill: workspace alignment");
  const int group = num_q_heads / num_kv_heads;
  int mt, ctas, parts;
  int64_t total;
  prefill_plan(qlen, n, after, num_kv_heads, group, device_sm_count(), &mt, &total, &ctas, &parts);
  const int64_t need = qp_prefill_workspace_bytes(qlen, n, num_q_heads, num_kv_heads, head_size, tokens_after_keys);
  if (workspace_bytes < need)
    return set_error(QP_ERR_WORKSPACE, "prefill: workspace of %lld bytes < %lld", (long long)workspace_bytes,
                     (long long)need);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const int64_t nt = static_cast<int64_t>(num_kv_heads) * mt;
  uint8_t* qprep = ws;
  float* qscale = reinterpret_cast<float*>(ws + align256(nt * 65536));
  float* part_o = reinterpret_cast<float*>(ws + align256(nt * 65536) + align256(nt * PF_BM * 4));
  float* part_lse = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(part_o) +
                                             align256(static_cast<int64_t>(qlen) * num_q_heads * parts * PF_HS * 4));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float qk_scale = softmax_scale / static_cast<float>(head_size) * PF_LOG2E;
  const int64_t qrows = nt * PF_BM;
  const int64_t lse_count = static_cast<int64_t>(qlen) * num_q_heads * parts;
  const unsigned qgrid = static_cast<unsigned>((qrows + 7) / 8);
#define QP_QPREP(F, D)                                                                                          \
  prefill_qprep_kernel<F, D><<<qgrid, 256, 0, st>>>(q, q_stride_token, q_stride_head, qlen, num_q_heads,        \
                                                    num_kv_heads, group, mt, rht_sign_bits, q_rotated, qk_scale, \
                                                    qprep, qscale, part_lse, lse_count)
  if (fmt == FMT_INT4) {
    if (dtype == DT_BF16) QP_QPREP(FMT_INT4, DT_BF16); else QP_QPREP(FMT_INT4, DT_F16);
  } else {
    if (dtype == DT_BF16) QP_QPREP(FMT_K8V4, DT_BF16); else QP_QPREP(FMT_K8V4, DT_F16);
  }
#undef QP_QPREP
  int rc = check_launch("prefill q prep");
  if (rc) return rc;

  PrefillParams pp{};
  pp.cache = static_cast<const uint8_t*>(cache);
  pp.block_size = block_size;
  pp.block_stride = block_stride;
  pp.head_stride = head_stride;
  pp.block_row = block_row;
  pp.n = n;
  pp.qlen = qlen;
  pp.vis_base = n - qlen + after;
  pp.nq = num_q_heads;
  pp.nkv = num_kv_heads;
  pp.group = group;
  pp.mt_per_kv = mt;
  pp.qprep = qprep;
  pp.qscale = qscale;
  pp.part_o = part_o;
  pp.part_lse = part_lse;
  pp.parts = parts;
  pp.total_tiles = total;
  rc = fmt == FMT_INT4 ? launch_prefill_main<FMT_INT4>(pp, ctas, st) : launch_prefill_main<FMT_K8V4>(pp, ctas, st);
  if (rc) return rc;
  return qp_merge_attn_partials(dtype, head_size, qlen, num_q_heads, parts, part_o,
                                static_cast<int64_t>(num_q_heads) * parts * PF_HS, static_cast<int64_t>(parts) * PF_HS,
                                PF_HS, part_lse, static_cast<int64_t>(num_q_heads) * parts, parts, 1, out_mode, out,
                                out_stride_token, out_stride_head, lse_out, rht_sign_bits, stream);
}
