// K3: long-chunk prefill over the int4 / k8v4 paged cache on the 5th-generation tensor cores (tcgen05 + TMEM),
// dequantising each key / value tile in shared memory: no scratch unpack of the cache.
//
// Reference behaviour (what this computes): vllm_quantpack/attention/int4_prefill.py:203-232 `prefill_sequence`
// (attention of a chunk of qlen queries, the last qlen positions of a context of n tokens, over the whole cached
// context, causal inside the chunk, RHT domain, scale softmax_scale / head), which the reference runs as 16k-token
// bf16 unpacks + FlashAttention 2 + an fp32 log-sum-exp fold, and the 2D Triton path (int4_kv.py:113-119).
//
// B200 design (one persistent CTA of 18 warps per SM):
//   warp 0      producer: 1-D bulk copies of the raw 264 / 392-byte cells of a 64-key tile (whole 16-key runs) into a
//               ring of raw stages;
//   warp 1      MMA issuer (convergent; one lane chosen by elect.sync issues): S = Q K^T (M 128 rows, N 64 keys,
//               K 256; Q read from TMEM) into TMEM as two interleaved accumulation chains over the two channel halves,
//               then O += P V (M 128, N 256 channels, K 64 keys; P from shared memory) into TMEM, each finished with
//               tcgen05.commit onto mbarriers;
//   warps 2-9   dequant (4 key warps, 4 value warps, one 64-channel block of all 64 keys each) into double-buffered
//               key and value operand tiles (the conversion of tile j + 1 overlaps the MMAs of tile j): raw cells ->
//               fp16 operands in shared memory, 128B-swizzled canonical UMMA layouts. One lop3 turns two nibbles into
//               fp16 and one f16x2 subtract makes the exact (u - zp) (int8 codes for k8v4 keys). Key operands stay
//               exact codes (the 64 key scales of the tile go to shared memory and multiply the scores in fp32); value
//               operands are multiplied by the token's scale over a power of two (the piece's running largest value
//               scale). The channel order inside every 8 channels is [0 4 1 5 2 6 3 7] (what one lop3 pair yields),
//               the same for Q and K (a dot product does not see the order) and undone on O in the epilogue;
//   warps 10-17 softmax: two threads per TMEM lane (= query row), 32 keys each; at the start of each piece they store
//               their row of the prepared Q tile into TMEM (columns 0-127). S is read into registers and released at
//               once (the next tile's QK runs behind the PV of the previous one meanwhile). Scores in log2 units =
//               S x key scale x (softmax_scale / head x log2 e x 2^-row exponent); the running maximum is lazy and
//               per row (P may reach 2^8 before O is rescaled in TMEM, which is rare); P in fp16 goes to shared memory
//               as the A operand of the PV MMA. The epilogue reads O from TMEM and writes fp32 partials + base-2 lse.
// Rows of an M-tile are (query token, query head of the KV head's group) pairs, head fastest: the 6 heads of a group
// share every dequantised key / value tile. The (M-tile, key-tile) space is split evenly over the CTAs (stream-K):
// an M-tile may be finished by two CTAs, whose partials the merge kernel folds (with the inverse RHT).
#include <math.h>
#include <stdlib.h>

#include <algorithm>
#include <vector>

#include "qp_api_internal.h"
#include "qp_common.cuh"
#include "qp_tcgen05.cuh"

namespace qp {

constexpr int PF_HS = 256;
constexpr int PF_BM = 128;  // query rows per M-tile (TMEM lanes)
constexpr int PF_BN = 64;   // keys per tile
constexpr int PF_MAX_CHUNKS = 16;  // key chunks of the walk (Sched); one lane of a warp works out each
static_assert(PF_MAX_CHUNKS <= 32, "chunk shares are computed one per lane");
#ifndef QP_PF_DQ_WARPS
#define QP_PF_DQ_WARPS 8
#endif
// single-CTA kernel: producer, MMA, PF_DQ dequant warps (half keys, half values; each converts 8 / PF_DQ of the
// tile's 64-channel blocks), 8 softmax warps
constexpr int PF_DQ = QP_PF_DQ_WARPS;
static_assert(PF_DQ == 4 || PF_DQ == 8, "dequant warps: 4 or 8");
#ifndef QP_PF_SM_WARPS
#define QP_PF_SM_WARPS 8
#endif
// softmax warps: one or two per TMEM lane quarter (a row's 64 keys and 256 output channels in one thread, or split
// over two)
constexpr int PF_SMW = QP_PF_SM_WARPS;
static_assert(PF_SMW == 4 || PF_SMW == 8, "softmax warps: 4 or 8");
constexpr int PF_HALVES = PF_SMW / 4;
constexpr int PF_SM0 = 2 + PF_DQ;                // first softmax warp
constexpr int PF1_THREADS = 32 * (PF_SM0 + PF_SMW);
// registers per thread one CTA may hold: the register file is split over the 4 sub-partitions (16384 each), and a
// sub-partition hosts every fourth warp
constexpr int PF1_REGS = (16384 / (32 * ((PF1_THREADS / 32 + 3) / 4))) & ~7;
constexpr float PF_SLACK = 8.f;
constexpr float PF_LOG2E = 1.4426950408889634f;

template <int FMT>
struct PfCfg {
  static constexpr int CELL = FMT == FMT_INT4 ? PF_HS + 8 : PF_HS * 3 / 2 + 8;
  static constexpr int KB = FMT == FMT_INT4 ? PF_HS / 2 : PF_HS;  // key bytes in a cell
  static constexpr int RS = FMT == FMT_INT4 ? 4 : 3;               // raw stages
  static constexpr int RAW_BYTES = PF_BN * CELL;
  // shared memory map (operand tiles 1024-byte aligned for the 128B swizzle); Q, S and O live in TMEM
  static constexpr int OFF_K = 0;                       // 2 buffers x 4 K-blocks x 64 keys x 128 B = 64 KB
  static constexpr int OFF_V = OFF_K + 65536;           // 2 buffers x 4 N-blocks x 8 key groups x 1024 B = 64 KB
  static constexpr int OFF_P = OFF_V + 65536;           // P: 128 rows x 64 keys fp16, K-major, 128B-swizzled = 16 KB
  static constexpr int OFF_RAW = OFF_P + 16384;         // RS x RAW_BYTES
  // [2 buffers][64 key scales (fp32), value exponent E, 3 spare] (272 B each)
  static constexpr int SC_STRIDE = 68;
  static constexpr int OFF_SC = OFF_RAW + RS * RAW_BYTES;
  static constexpr int OFF_HX = OFF_SC + 2 * SC_STRIDE * 4;  // softmax pairs: [2 buffers][2 halves][128] row maxima,
                                                         // then [2 halves][128] row sums
  static constexpr int OFF_BAR = OFF_HX + (2 * 2 * 128 + 2 * 128) * 4;
  static constexpr int NBAR = 40;
  static constexpr int OFF_TMEM = OFF_BAR + NBAR * 8;
  static constexpr int OFF_CHUNKS = OFF_TMEM + 16;  // [PF_MAX_CHUNKS] ChunkStart: this CTA's share of every chunk
  static constexpr int BYTES = OFF_CHUNKS + PF_MAX_CHUNKS * 24;
  static_assert(BYTES <= 232448, "dynamic shared memory above the 227 KB a CTA may hold");
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
  B_S_FULL = 18,     // S (both channel halves) of the tile is in TMEM
  B_S_FREE = 19,     // the softmax has read S into registers (8 softmax warps)
  B_P_FULL = 22,     // P of the tile is in shared memory (8 softmax warps)
  B_SC_FULL = 26,    // [2] the tile's 64 key scales are in shared memory (key warps)
  B_SC_FREE = 28,    // [2]
  B_O_DONE = 30,
  B_O_FREE = 31,
  B_FINAL = 32,      // the MMA thread's last commit: every tcgen05.mma done before TMEM is released
  B_SCV_FULL = 33,   // [2] the tile's value exponent E (value warps)
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
  int chunk_tiles;           // key tiles of one key chunk (the walk is chunk-major, see Sched)
  int piece_stride;          // piece slots per key chunk of an M-tile
  int chunks;                // key chunks (<= PF_MAX_CHUNKS)
  int64_t chunk_total[PF_MAX_CHUNKS];  // (M-tile, key-tile) pairs of each chunk over all KV heads
};

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

// Key tiles [*lo, *lo + result) of M-tile m that fall in key chunk j.
__device__ __forceinline__ int run_tiles(const PrefillParams& p, int j, int m, int* lo) {
  const int a = j * p.chunk_tiles;
  *lo = a;
  return max(0, min(mtile_key_tiles(p, m), a + p.chunk_tiles) - a);
}

// Walk of the tiles of this CTA over the (key chunk, KV head, M-tile, key tile) space. Every key chunk is split
// among all CTAs on its own (CTA c takes [T_j c / ctas, T_j (c + 1) / ctas) of chunk j's T_j tiles), and a CTA
// finishes its share of chunk j before it starts on chunk j + 1: the CTAs running at one time work on the same key
// chunk, so each key tile is fetched from HBM about once and the other M-tiles of its KV head read it from L2 (a walk
// with the key tiles of one M-tile innermost had every M-tile re-read its head's whole cache). A run (one M-tile's
// tiles inside one chunk) split by CTA boundaries gives several pieces; piece slots j * piece_stride + i keep the
// pieces of different chunks apart.
struct Walk {
  int kvh, m, kt, kt_end;  // current M-tile and key tile
  int piece;               // partial slot of this CTA's piece of the M-tile
  bool first_of_piece, last_of_piece, new_mtile;
};

// Where a CTA's share of key chunk j starts: run (kvh, m), key tiles [kt, kt_hi) of it, the partial slot and the
// share's tile count (0: no tile of the chunk).
struct ChunkStart {
  int kvh, m, kt, kt_hi, piece, left;
};

__device__ ChunkStart chunk_start(const PrefillParams& p, int j, int cta, int ctas) {
  ChunkStart c{};
  const int64_t T = p.chunk_total[j];
  const int64_t g = T * cta / ctas;
  c.left = static_cast<int>(T * (cta + 1) / ctas - g);
  if (c.left <= 0) return c;
  int64_t start = 0;
  int lo = 0;
  int len = run_tiles(p, j, 0, &lo);
  while (start + len <= g) {  // to the run holding g (empty runs are skipped)
    start += len;
    if (++c.m == p.mt_per_kv) {
      c.m = 0;
      ++c.kvh;
    }
    len = run_tiles(p, j, c.m, &lo);
  }
  c.kt = lo + static_cast<int>(g - start);
  c.kt_hi = lo + len;
  // piece inside the run: CTAs whose share starts inside it before this one. The CTA covering `start` is the largest
  // c0 with T * c0 / ctas <= start; every later run of this CTA in the chunk starts with it (piece 0).
  int c0 = static_cast<int>((start * ctas) / T);
  while (c0 + 1 < ctas && T * (c0 + 1) / ctas <= start) ++c0;
  while (c0 > 0 && T * c0 / ctas > start) --c0;
  c.piece = j * p.piece_stride + (cta - c0);
  return c;
}

// Every warp walks the same schedule each tile, so the walk itself runs in 32-bit counters (the host keeps the
// tile count below 2^31); 64-bit arithmetic is confined to chunk_start.
struct Sched {
  const PrefillParams* p;
  int left;          // tiles of this CTA's share of chunk j not yet walked past, the current one included
  int j, kvh, m;     // current run: key chunk, M-tile
  int kt, kt_hi;     // current key tile inside the M-tile, end of the run
  int first_kt;      // first key tile of this CTA inside the current run
  int piece;         // partial slot of this CTA's piece of the current run
  const ChunkStart* starts;  // [chunks] this CTA's share of each chunk (shared memory)

  __device__ void advance_run() {  // next (KV head, M-tile) inside chunk j
    if (++m == p->mt_per_kv) {
      m = 0;
      ++kvh;
    }
  }

  // Positions the walk at this CTA's share of chunk j, or of the next chunk with a non-empty share (the shares are
  // worked out once per CTA, chunk_start, into shared memory: a copy of that search in every warp role's tile loop
  // cost instruction-cache misses, 9.9 against 7.8 ms per c3 launch).
  __device__ void start_chunk() {
    for (; j < p->chunks; ++j) {
      const ChunkStart c = starts[j];
      if (c.left <= 0) continue;
      left = c.left;
      kvh = c.kvh;
      m = c.m;
      kt = first_kt = c.kt;
      kt_hi = c.kt_hi;
      piece = c.piece;
      return;
    }
    left = 0;
  }

  __device__ void init(const PrefillParams& prm, const ChunkStart* starts_) {
    p = &prm;
    starts = starts_;
    j = 0;
    start_chunk();
  }
  __device__ bool done() const { return left <= 0; }
  __device__ Walk current() const {
    Walk w;
    w.kvh = kvh;
    w.m = m;
    w.kt = kt;
    w.kt_end = kt_hi;
    w.piece = piece;
    w.first_of_piece = kt == first_kt;
    w.last_of_piece = (kt + 1 == kt_hi) || (left == 1);
    w.new_mtile = w.first_of_piece;
    return w;
  }
  __device__ void next() {
    if (--left == 0) {  // this CTA's share of chunk j is done
      ++j;
      start_chunk();
      return;
    }
    if (++kt >= kt_hi) {
      int lo = 0, len = 0;
      do {
        advance_run();
        len = run_tiles(*p, j, m, &lo);
      } while (len == 0);
      kt = first_kt = lo;
      kt_hi = lo + len;
      piece = j * p->piece_stride;
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
  *reinterpret_cast<uint4*>(tile + r * (PF_HS * 2) + lane * 16) = v;  // plain rows, stored into TMEM by the kernel
  if (lane == 0) qs[r] = mr < qlen * group ? ldexpf(qk_scale, -ex) : 0.f;
}

// ---------------------------------------------------------------------------------------------------- main kernel
template <int FMT>
__global__ void __maxnreg__(PF1_REGS) prefill_kernel(const PrefillParams p) {
  using C = PfCfg<FMT>;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_TMEM);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < C::RS; ++s) {
      mbar_init(&bars[B_RAW_FULL + s], 1);
      mbar_init(&bars[B_RAW_EMPTY + s], PF_DQ);
    }
    mbar_init(&bars[B_Q_FULL], PF_SMW);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars[B_K_FULL + b], PF_DQ / 2);
      mbar_init(&bars[B_K_FREE + b], 1);
      mbar_init(&bars[B_V_FULL + b], PF_DQ / 2);
      mbar_init(&bars[B_V_FREE + b], 1);
      mbar_init(&bars[B_SC_FULL + b], PF_DQ / 2);
      mbar_init(&bars[B_SCV_FULL + b], PF_DQ / 2);
      mbar_init(&bars[B_SC_FREE + b], PF_SMW);
    }
    mbar_init(&bars[B_S_FULL], 1);
    mbar_init(&bars[B_S_FREE], PF_SMW);
    mbar_init(&bars[B_P_FULL], PF_SMW);
    mbar_init(&bars[B_O_DONE], 1);
    mbar_init(&bars[B_O_FREE], PF_SMW);
    mbar_init(&bars[B_FINAL], 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  ChunkStart* starts = reinterpret_cast<ChunkStart*>(smem + C::OFF_CHUNKS);
  if (warp == 2 && lane < p.chunks) starts[lane] = chunk_start(p, lane, blockIdx.x, gridDim.x);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // S = Q K^T is two independent accumulation chains, one per half of the channels (the tensor pipe overlaps two
  // chains; one chain of dependent MMAs runs at about 60 % of the rate). The softmax adds the halves.
  const uint32_t tm_q = tmem;                  // Q (A operand of S = Q K^T): columns [0, 128)
  const uint32_t tm_sa = tmem + 128;           // S over channels 0..127: columns [128, 192)
  const uint32_t tm_sb = tmem + 192;           // S over channels 128..255: columns [192, 256)
  const uint32_t tm_o = tmem + 256;            // O: columns [256, 512)

  Sched sch;
  sch.init(p, starts);
  bool failed = false;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      int64_t j = 0;        // global tile counter (raw ring)
      for (; !sch.done() && !failed; sch.next(), ++j) {
        const Walk w = sch.current();
        const int stage = static_cast<int>(j % C::RS);
        if (j >= C::RS) failed |= !mbar_wait_spin(&bars[B_RAW_EMPTY + stage], ((j / C::RS) - 1) & 1);
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
        mbar_wait_spin(&bars[B_RAW_FULL + (k % C::RS)], (k / C::RS) & 1, 100000000ull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    // The whole warp walks the schedule and waits (convergent, so the descriptors and TMEM addresses are warp-uniform
    // values); one elected lane issues. A tcgen05.mma issued from a one-lane branch costs tens of cycles of operand
    // moves each, which starves the tensor pipe.
    constexpr uint32_t ID_QK = f16_idesc(PF_BM, PF_BN, false);
    constexpr uint32_t ID_PV = f16_idesc(PF_BM, PF_HS, true);
    const uint32_t k_base = smem_u32(smem + C::OFF_K), v_base = smem_u32(smem + C::OFF_V);
    const uint32_t p_base = smem_u32(smem + C::OFF_P);
    int64_t j = 0;
    int qcount = 0, pieces = 0;
    int64_t pv_pending = -1;  // tile whose PV is still to be issued
    bool pv_first = false;
    // every lane runs the same bounded waits; the vote keeps the warp's view (and its control flow) uniform
    auto wait_all = [&](uint64_t* bar, uint32_t parity) {
      const bool ok = mbar_wait_spin(bar, parity);
      failed |= __any_sync(0xffffffffu, !ok);
    };
    auto issue_pv = [&](int64_t t, bool first) {
      const int b = static_cast<int>(t & 1);
      wait_all(&bars[B_V_FULL + b], (t >> 1) & 1);
      wait_all(&bars[B_P_FULL], static_cast<uint32_t>(t & 1));
      tc_fence_after();
      const uint32_t vb = v_base + b * 32768;
      if (elect_one()) {
        // P(t) in shared memory, K step s = 16 keys = 32 bytes of each 128-byte row
#pragma unroll
        for (int s = 0; s < 4; ++s)
          umma_f16(tm_o, sw128_desc(p_base + 32 * s, 16, 1024), sw128_desc(vb + 2 * s * 1024, 8192, 1024), ID_PV,
                   (first && s == 0) ? 0u : 1u);
        umma_commit(&bars[B_V_FREE + b]);
        umma_commit(&bars[B_O_DONE]);
      }
      __syncwarp();
    };
    for (; !sch.done() && !failed; sch.next(), ++j) {
      const Walk w = sch.current();
      if (w.new_mtile) {
        wait_all(&bars[B_Q_FULL], qcount & 1);
        ++qcount;
      }
      // S(j) = Q K(j)^T
      const int b = static_cast<int>(j & 1);
      wait_all(&bars[B_K_FULL + b], (j >> 1) & 1);
      // S(j - 1) has been read by the softmax (it releases S before its exponentials: the PV issued just before
      // keeps the tensor pipe busy meanwhile)
      if (j > 0) wait_all(&bars[B_S_FREE], static_cast<uint32_t>((j - 1) & 1));
      tc_fence_after();
      const uint32_t kb = k_base + b * 32768;
      if (elect_one()) {
#pragma unroll
        for (int s = 0; s < 8; ++s) {  // K step s of each half: 16 channels = 8 TMEM columns of Q
          umma_f16_ts(tm_sa, tm_q + 8 * s, sw128_desc(kb + (s >> 2) * 8192 + (s & 3) * 32, 16, 1024), ID_QK,
                      s > 0 ? 1u : 0u);
          umma_f16_ts(tm_sb, tm_q + 64 + 8 * s, sw128_desc(kb + 16384 + (s >> 2) * 8192 + (s & 3) * 32, 16, 1024),
                      ID_QK, s > 0 ? 1u : 0u);
        }
        umma_commit(&bars[B_K_FREE + b]);
        umma_commit(&bars[B_S_FULL]);
      }
      __syncwarp();
      // Q of this piece is free once S of its last tile is complete: the softmax, which waits for that S before
      // it stores the next piece's Q, needs no other signal
      // O += P(j-1) V(j-1), one tile behind so the softmax of tile j overlaps it
      if (pv_pending >= 0) {
        issue_pv(pv_pending, pv_first);
        pv_pending = -1;
      }
      if (w.first_of_piece && pieces > 0) {
        // O is overwritten by this piece's first PV: the previous piece's epilogue must have read it
        wait_all(&bars[B_O_FREE], (pieces - 1) & 1);
      }
      if (w.first_of_piece) ++pieces;
      pv_pending = j;
      pv_first = w.first_of_piece;
      if (w.last_of_piece) {  // the epilogue waits for this PV: issue it now
        issue_pv(pv_pending, pv_first);
        pv_pending = -1;
      }
    }
    if (elect_one()) umma_commit(&bars[B_FINAL]);
    __syncwarp();
    mbar_wait_spin(&bars[B_FINAL], 0, 100000000ull);
  } else if (warp < PF_SM0) {
    // ------------------------------------------------------------------ dequant (warps 2 .. PF_SM0 - 1)
    // keys:   K_op = u - zp (int4) or the int8 code, exact in fp16; the key scale multiplies the score in fp32 in
    //         the softmax. (A scale folded into the operand would be one fp16 rounding shared by all 256 channels of
    //         a key, a relative error of the whole score that the exponential amplifies at large logits.)
    // values: V_op = (u - zp) * vs * 2^-E  (E: running exponent of the piece's largest value scale; O is rescaled by
    //         the softmax when E grows): <= 15 in magnitude, exact up to one fp16 rounding.
    // The first PF_DQ / 2 warps convert the keys, the others the values; each warp takes BPW of the four 64-channel
    // blocks for all 64 rows of the tile (lane l: rows l and l + 32). Every warp sees all 64 scales of its operand:
    // the tile maximum is one warp reduction, with no exchange between warps.
    constexpr int BPW = 8 / PF_DQ;                 // 64-channel blocks per warp
    const int dq = warp - 2;
    const bool is_k = dq < PF_DQ / 2;
    const int dd = dq % (PF_DQ / 2);               // blocks BPW dd .. BPW dd + BPW - 1
    uint8_t* const kop0 = smem + C::OFF_K;
    uint8_t* const vop0 = smem + C::OFF_V;
    const int sc_off = is_k ? C::KB : C::KB + 4 + PF_HS / 2;
    const bool packed = FMT == FMT_INT4 || !is_k;  // the scale carries the zero point in its low 4 mantissa bits
    int e_run_v = -1000;
    int64_t j = 0;
    for (; !sch.done() && !failed; sch.next(), ++j) {
      const Walk w = sch.current();
      const int stage = static_cast<int>(j % C::RS);
      const int b = static_cast<int>(j & 1);
      if (w.first_of_piece) e_run_v = -1000;
      failed |= !mbar_wait_spin(&bars[B_RAW_FULL + stage], (j / C::RS) & 1);
      const uint8_t* const raw = smem + C::OFF_RAW + stage * C::RAW_BYTES;
      const int tok0 = w.kt * PF_BN + lane;
      const uint32_t sw0 = *reinterpret_cast<const uint32_t*>(raw + lane * C::CELL + sc_off);
      const uint32_t sw1 = *reinterpret_cast<const uint32_t*>(raw + (lane + 32) * C::CELL + sc_off);
      const float scl0 = tok0 < p.n ? __uint_as_float(packed ? (sw0 & 0xFFFFFFF0u) : sw0) : 0.f;
      const float scl1 = tok0 + 32 < p.n ? __uint_as_float(packed ? (sw1 & 0xFFFFFFF0u) : sw1) : 0.f;
      int ex = -1000;
      if (!is_k) {
        const float tmax = warp_max(fmaxf(scl0, scl1));  // scales are >= 0
        // tmax < 2^ex (the exponent field; subnormals give -126, still a bound)
        if (tmax > 0.f) ex = static_cast<int>((__float_as_uint(tmax) >> 23) & 0xFFu) - 126;
        e_run_v = max(e_run_v, ex);
        ex = e_run_v;
      }
      const float inv = ex == -1000 ? 0.f : exp2_int(-ex);
      const float q_0 = scl0 * inv, q_1 = scl1 * inv;  // < 1
      const uint32_t zp_0 = packed ? (sw0 & 0xFu) : 0u, zp_1 = packed ? (sw1 & 0xFu) : 0u;
      // int4 (u - zp) exact from the exponent-bias forms (1024 + u) - (1024 + zp) and (1024 + 16 u) / 16 - (64 + zp),
      // int8 codes from (1152 + code) - 1152; values then times their fp16 scale q, rounded once. (Folding the zero
      // point into one fma, u 2^-24 q' - zp q'', rounds the zero-point term on its own: the same error in all
      // channels of a token.)
      const uint32_t q2_0 = h2_bits(q_0), q2_1 = h2_bits(q_1);
      if (j >= 2) failed |= !mbar_wait_spin(&bars[B_SC_FREE + b], ((j >> 1) - 1) & 1);
      if (dd == 0) {
        float* scb = reinterpret_cast<float*>(smem + C::OFF_SC) + b * C::SC_STRIDE;
        if (is_k) {  // the 64 key scales of the tile (0 past the context)
          scb[lane] = scl0;
          scb[lane + 32] = scl1;
        } else if (lane == 0) {
          scb[64] = __int_as_float(ex);
        }
      }
      // the softmax needs only these factors: release them now, not after the (longer) operand conversion
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[is_k ? B_SC_FULL + b : B_SCV_FULL + b]);
      // Each pass converts 64 channels of one row: all its loads are issued before any conversion (the stores could
      // alias them for the compiler, which would otherwise serialise load -> convert -> store per word). Cells are
      // 8-byte aligned (264 / 392 B): the 8-byte loads of 16 consecutive rows fall in 16 distinct bank pairs; the
      // 16-byte stores of 8 consecutive rows hit 8 distinct bank groups (swizzle).
      if (is_k) {
        if (j >= 2) failed |= !mbar_wait_spin(&bars[B_K_FREE + b], ((j >> 1) - 1) & 1);
        uint8_t* const kop = kop0 + b * 32768;
#pragma unroll 1
        for (int it = 0; it < 2 * BPW; ++it) {
          const int r = it / BPW, kb = BPW * dd + it % BPW;  // row lane + 32 r, K-block kb (channels 64 kb ..)
          const int kr = lane + 32 * r;
          const uint8_t* const cell = raw + kr * C::CELL;
          // the row's 128-byte line with its swizzle folded in: chunk i of the row sits at d ^ (i << 4)
          const uint32_t d = static_cast<uint32_t>(kop - smem) + kb * 8192 + (kr >> 3) * 1024 + (kr & 7) * 144;
          if constexpr (FMT == FMT_INT4) {
            const uint32_t zp = r ? zp_1 : zp_0;
            const uint32_t lo_b = 0x64006400u | zp | (zp << 16), hi_b = 0xD400D400u | (zp << 4) | (zp << 20);
            uint2 kw[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) kw[k] = *reinterpret_cast<const uint2*>(cell + 32 * kb + 8 * k);
#pragma unroll
            for (int i = 0; i < 8; ++i) {  // word: channels 8 (8 kb + i) .. + 7 = chunk i of the K-block
              const uint32_t x = (i & 1) ? kw[i >> 1].y : kw[i >> 1].x;
              const uint32_t x8 = x >> 8;
              uint4 v;
              v.x = hsub2_u32(lop3_and_or(x, 0x000F000Fu, 0x64006400u), lo_b);                      // channels 0, 4
              v.y = hfma2_u32(lop3_and_or(x, 0x00F000F0u, 0x64006400u), 0x2C002C00u, hi_b);         // 1, 5
              v.z = hsub2_u32(lop3_and_or(x8, 0x000F000Fu, 0x64006400u), lo_b);                     // 2, 6
              v.w = hfma2_u32(lop3_and_or(x8, 0x00F000F0u, 0x64006400u), 0x2C002C00u, hi_b);        // 3, 7
              *reinterpret_cast<uint4*>(smem + (d ^ (static_cast<uint32_t>(i) << 4))) = v;
            }
          } else {
            uint2 kw[8];  // codes 64 kb .. 64 kb + 63
#pragma unroll
            for (int k = 0; k < 8; ++k) kw[k] = *reinterpret_cast<const uint2*>(cell + 64 * kb + 8 * k);
#pragma unroll
            for (int k = 0; k < 8; ++k) {  // chunk k: channels 8 (8 kb + k) .. + 7 (two words)
              const uint32_t a = kw[k].x ^ 0x80808080u, cc = kw[k].y ^ 0x80808080u;
              uint4 v;  // (1152 + code) - 1152 = code, exact
              v.x = hsub2_u32(prmt(a, 0x64646464u, 0x4140u), 0x64806480u);
              v.y = hsub2_u32(prmt(a, 0x64646464u, 0x4342u), 0x64806480u);
              v.z = hsub2_u32(prmt(cc, 0x64646464u, 0x4140u), 0x64806480u);
              v.w = hsub2_u32(prmt(cc, 0x64646464u, 0x4342u), 0x64806480u);
              *reinterpret_cast<uint4*>(smem + (d ^ (static_cast<uint32_t>(k) << 4))) = v;
            }
          }
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[B_K_FULL + b]);
      } else {
        if (j >= 2) failed |= !mbar_wait_spin(&bars[B_V_FREE + b], ((j >> 1) - 1) & 1);
        uint8_t* const vop = vop0 + b * 32768;
#pragma unroll 1
        for (int it = 0; it < 2 * BPW; ++it) {
          const int r = it / BPW, kb = BPW * dd + it % BPW;  // row lane + 32 r, N-block kb (channels 64 kb ..)
          const int kr = lane + 32 * r;
          const uint8_t* const cell = raw + kr * C::CELL;
          const uint32_t q2 = r ? q2_1 : q2_0, zp = r ? zp_1 : zp_0;
          const uint32_t lo_b = 0x64006400u | zp | (zp << 16), hi_b = 0xD400D400u | (zp << 4) | (zp << 20);
          const uint32_t d = static_cast<uint32_t>(vop - smem) + kb * 8192 + (kr >> 3) * 1024 + (kr & 7) * 144;
          // the value words start 4 bytes past an 8-byte boundary: 8-byte loads from the key scale on give the
          // pairs (key scale, V0), (V1, V2), ..., (V31, value scale)
          uint2 vw[5];
#pragma unroll
          for (int k = 0; k < 5; ++k) vw[k] = *reinterpret_cast<const uint2*>(cell + C::KB + 32 * kb + 8 * k);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint32_t x = (i & 1) ? vw[(i + 1) >> 1].x : vw[i >> 1].y;
            const uint32_t x8 = x >> 8;
            uint4 v;
            v.x = hmul2_u32(hsub2_u32(lop3_and_or(x, 0x000F000Fu, 0x64006400u), lo_b), q2);
            v.y = hmul2_u32(hfma2_u32(lop3_and_or(x, 0x00F000F0u, 0x64006400u), 0x2C002C00u, hi_b), q2);
            v.z = hmul2_u32(hsub2_u32(lop3_and_or(x8, 0x000F000Fu, 0x64006400u), lo_b), q2);
            v.w = hmul2_u32(hfma2_u32(lop3_and_or(x8, 0x00F000F0u, 0x64006400u), 0x2C002C00u, hi_b), q2);
            *reinterpret_cast<uint4*>(smem + (d ^ (static_cast<uint32_t>(i) << 4))) = v;
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
    // ------------------------------------------------------------------ softmax / epilogue (warps PF_SM0 ..)
    // (waits with the suspend hint: polling softmax warps would take issue slots from the dequant warps)
    // PF_HALVES warps per TMEM lane quarter (32 query rows; a warp reaches the quarter warp % 4). With two, the first
    // four warps take keys 0-31 of every tile and channels 0-127 of O, the last four keys 32-63 and channels
    // 128-255, and the two threads of a row agree on its maximum through shared memory (a named barrier per pair of
    // warps) and add their partial sums in the epilogue; with one, a thread owns its whole row.
    constexpr int KPT = PF_BN / PF_HALVES;   // keys of a tile per thread
    constexpr int CPT = PF_HS / PF_HALVES;   // output channels per thread
    const int quarter = warp & 3;
    const int half = (warp - PF_SM0) >> 2;   // 0 .. PF_HALVES - 1
    const int row = quarter * 32 + lane;     // TMEM lane = M-tile row
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const int pair_bar = 3 + quarter;        // named barriers 3 .. 6: the two warps of a lane quarter
    float* hmax = reinterpret_cast<float*>(smem + C::OFF_HX);  // [buffer][half][row]
    float* hsum = hmax + 2 * 2 * 128;                           // [half][row]
    (void)pair_bar;
    (void)hmax;
    (void)hsum;
    int64_t j = 0;
    // PV completions seen so far. O_DONE completes one phase per tile (its PV); a parity wait is exact only while
    // the barrier is at most one phase ahead of the phase waited for, so the phases are consumed in order: PV(j - 1)
    // before P(j) is stored (PV(j) cannot complete before P(j) exists), PV(j) in the epilogue.
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
        // this thread's share of its row of the piece's Q tile -> TMEM columns (128 / PF_HALVES) half + [0, 128 /
        // PF_HALVES) of its lane (the previous piece's QKs are complete: this thread consumed the S of its last tile)
        const int64_t mt = static_cast<int64_t>(w.kvh) * p.mt_per_kv + w.m;
        const uint4* qrow = reinterpret_cast<const uint4*>(p.qprep + mt * 65536 + row * (PF_HS * 2));
#pragma unroll 1
        for (int c0 = (128 / PF_HALVES) * half; c0 < (128 / PF_HALVES) * (half + 1); c0 += 32) {
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
      // this row's scores for keys KPT half .. KPT half + KPT - 1 of the tile (sum of the two channel-half
      // accumulators), then S is released to the next tile's QK
      failed |= !mbar_wait_bounded(&bars[B_S_FULL], static_cast<uint32_t>(j & 1));
      tc_fence_after();
      float s[KPT];
#pragma unroll
      for (int kk = 0; kk < KPT / 32; ++kk) {
        float t32[32];
        tmem_ld32_sum2(tm_sa + lane_off + KPT * half + 32 * kk, tm_sb + lane_off + KPT * half + 32 * kk, t32);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[32 * kk + i] = t32[i];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[B_S_FREE]);
      failed |= !mbar_wait_bounded(&bars[B_SC_FULL + b], (j >> 1) & 1);
      const float* scb = reinterpret_cast<const float*>(smem + C::OFF_SC) + b * C::SC_STRIDE;
      // the scores in fp32: key operand (exact codes) . Q, times the key's scale
#pragma unroll
      for (int c4 = 0; c4 < KPT; c4 += 4) {
        const float4 f = *reinterpret_cast<const float4*>(scb + KPT * half + c4);
        s[c4] *= f.x;
        s[c4 + 1] *= f.y;
        s[c4 + 2] *= f.z;
        s[c4 + 3] *= f.w;
      }
      const float qs_t = qsc;
      const int key0 = w.kt * PF_BN + KPT * half;
      const bool masked = w.kt * PF_BN + PF_BN - 1 > min(p.n - 1, p.vis_base);  // some row cannot see some key
      if (masked) {
#pragma unroll
        for (int c = 0; c < KPT; ++c)
          if (key0 + c > lim) s[c] = -INFINITY;
      }
      float mx4[4] = {s[0], s[1], s[2], s[3]};  // four independent chains
#pragma unroll
      for (int c = 4; c < KPT; ++c) mx4[c & 3] = fmaxf(mx4[c & 3], s[c]);
      float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      if constexpr (PF_HALVES == 2) {
        hmax[(b * 2 + half) * 128 + row] = mx;
        // the pair leaves together if either gave up a wait (a bar.sync has no time bound)
        if (named_bar_or(pair_bar, 64, failed)) {
          failed = true;
          break;
        }
        mx = fmaxf(mx, hmax[(b * 2 + (half ^ 1)) * 128 + row]);
      }
      const float mrow = mx * qs_t;
      const bool grow = mrow > m_used + PF_SLACK;  // the same in both threads of the row
      float alpha = 1.f;
      if (grow) {
        alpha = exp2f(m_used - mrow);
        m_used = mrow;
        l *= alpha;
      }
      // P = 2^(s qs_t - m) <= 2^8 in fp16
      const float base = m_used == -INFINITY ? 0.f : m_used;
      float ls4[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pw[KPT / 2];
      if (masked) {
#pragma unroll
        for (int c = 0; c < KPT; c += 2) {
          const float p0 = s[c] == -INFINITY ? 0.f : fast_exp2(fmaf(s[c], qs_t, -base));
          const float p1 = s[c + 1] == -INFINITY ? 0.f : fast_exp2(fmaf(s[c + 1], qs_t, -base));
          ls4[(c >> 1) & 3] += p0 + p1;
          const __half2 h = __floats2half2_rn(p0, p1);
          pw[c >> 1] = *reinterpret_cast<const uint32_t*>(&h);
        }
      } else {
#pragma unroll
        for (int c = 0; c < KPT; c += 2) {
          const float p0 = fast_exp2(fmaf(s[c], qs_t, -base));
          const float p1 = fast_exp2(fmaf(s[c + 1], qs_t, -base));
          ls4[(c >> 1) & 3] += p0 + p1;
          const __half2 h = __floats2half2_rn(p0, p1);
          pw[c >> 1] = *reinterpret_cast<const uint32_t*>(&h);
        }
      }
      l += (ls4[0] + ls4[1]) + (ls4[2] + ls4[3]);
      // the value exponent is needed only now, for the O rescale: the value warps publish it separately, so the
      // exponentials above do not wait for them
      failed |= !mbar_wait_bounded(&bars[B_SCV_FULL + b], (j >> 1) & 1);
      const int ev = __float_as_int(scb[64]);  // value exponent of this tile's operand
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[B_SC_FREE + b]);
      const bool vgrow = ev > e_used;  // the same for every thread
      wait_pv(j - 1);  // PV(j - 1) has read P(j - 1) and added into O
      if (__any_sync(0xffffffffu, alpha != 1.f) || vgrow) {
        // rescale this thread's channels of the row's O in TMEM: new running maximum and / or value exponent
        const float ao = alpha * (!vgrow ? 1.f : e_used == -1000 ? 0.f : ldexpf(1.f, e_used - ev));
        if (t_in_piece > 0) {
          tc_fence_after();
#pragma unroll 1
          for (int c0 = CPT * half; c0 < CPT * (half + 1); c0 += 32) {
            float o[32];
            tmem_ld32(tm_o + lane_off + c0, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= ao;
            tmem_st32(tm_o + lane_off + c0, o);
          }
        }
        if (vgrow) e_used = ev;
      }
      // P -> shared memory, row `row`, keys KPT half .. + KPT - 1 = 16-byte chunks (KPT / 8) half .. of the row (the
      // A operand of the PV MMA, K-major, 128B-swizzled; the 8 rows of a store phase hit 8 distinct bank groups)
      {
        uint8_t* const prow = smem + C::OFF_P;
#pragma unroll
        for (int i = 0; i < KPT / 8; ++i)
          *reinterpret_cast<uint4*>(prow + sw128_off(row, (KPT / 8) * half + i)) =
              make_uint4(pw[4 * i], pw[4 * i + 1], pw[4 * i + 2], pw[4 * i + 3]);
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[B_P_FULL]);
      ++t_in_piece;

      if (w.last_of_piece) {
        // epilogue: O of this piece -> normalised fp32 partial (channel order restored) + base-2 lse
        float l_row = l;
        if constexpr (PF_HALVES == 2) {
          hsum[half * 128 + row] = l;
          if (named_bar_or(pair_bar, 64, failed)) {
            failed = true;
            break;
          }
          l_row += hsum[(half ^ 1) * 128 + row];
        }
        wait_pv(j);
        tc_fence_after();
        const float o_unit = e_used == -1000 ? 0.f : ldexpf(1.f, e_used);  // value operand x 2^-E
        const float inv = l_row > 0.f ? o_unit / l_row : 0.f;
        const int64_t prow_i = (static_cast<int64_t>(tok) * p.nq + qh) * p.parts + w.piece;
#pragma unroll 1
        for (int c0 = CPT * half; c0 < CPT * (half + 1); c0 += 32) {
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

// Key chunks of a chunk prefill: the cache of all KV heads in pieces of at most 80 MB, so that the chunk the CTAs work
// on stays in the 126 MB L2; at most PF_MAX_CHUNKS. Measured at c3 (242 MB): 8.05 ms with 80 MB chunks, 8.22 with
// 40 MB, 8.58 with 20 MB (more pieces to fold and more piece epilogues), 8.06 with one contiguous split (10 GB of
// DRAM reads, which this kernel, bound by its CUDA-core work, does not feel yet).
static int prefill_chunks(int n, int nkv, int cell) {
  const int64_t bytes = static_cast<int64_t>(n) * nkv * cell;
  const int64_t c = (bytes + (80ll << 20) - 1) / (80ll << 20);
  return static_cast<int>(std::min<int64_t>(PF_MAX_CHUNKS, std::max<int64_t>(1, c)));
}

struct PrefillPlan {
  int mt_per_kv, ctas, parts, chunk_tiles, piece_stride, chunks;
  int64_t total;
  int64_t chunk_total[PF_MAX_CHUNKS];
};

static PrefillPlan prefill_plan(int qlen, int n, int after, int nkv, int group, int sms, int cell) {
  PrefillPlan pl{};
  const int rows = qlen * group;
  pl.mt_per_kv = (rows + PF_BM - 1) / PF_BM;
  std::vector<int> tiles(pl.mt_per_kv);
  int64_t tot = 0;
  int maxt = 0;
  for (int m = 0; m < pl.mt_per_kv; ++m) {
    const int r_hi = std::min(rows - 1, m * PF_BM + PF_BM - 1);
    tiles[m] = (std::min(n, n - qlen + after + r_hi / group + 1) + PF_BN - 1) / PF_BN;
    tot += tiles[m];
    maxt = std::max(maxt, tiles[m]);
  }
  tot *= nkv;
  pl.total = tot;
  pl.ctas = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(sms, tot)));
  const int want = prefill_chunks(n, nkv, cell);
  pl.chunk_tiles = std::max(1, (maxt + want - 1) / want);
  pl.chunks = (maxt + pl.chunk_tiles - 1) / pl.chunk_tiles;
  // chunk j's tiles, then the pieces of each of its runs: the CTAs covering it under chunk j's own split (the CTA of
  // tile g: the largest c with T_j * c / ctas <= g)
  int stride = 1;
  for (int j = 0; j < pl.chunks; ++j) {
    const int a = j * pl.chunk_tiles;
    int64_t T = 0;
    for (int m = 0; m < pl.mt_per_kv; ++m) T += std::max(0, std::min(tiles[m], a + pl.chunk_tiles) - a);
    T *= nkv;
    pl.chunk_total[j] = T;
    auto cta_of = [&](int64_t g) {
      int c = static_cast<int>(g * pl.ctas / std::max<int64_t>(1, T));
      while (c + 1 < pl.ctas && T * (c + 1) / pl.ctas <= g) ++c;
      while (c > 0 && T * c / pl.ctas > g) --c;
      return c;
    };
    int64_t start = 0;
    for (int h = 0; h < nkv; ++h)
      for (int m = 0; m < pl.mt_per_kv; ++m) {
        const int len = std::max(0, std::min(tiles[m], a + pl.chunk_tiles) - a);
        if (len > 0) stride = std::max(stride, cta_of(start + len - 1) - cta_of(start) + 1);
        start += len;
      }
  }
  pl.piece_stride = stride;
  pl.parts = pl.chunks * stride;
  return pl;
}

static int64_t prefill_ws_bytes(int qlen, int nq, int64_t nt, int parts) {
  return align256(nt * 65536) + align256(nt * PF_BM * 4) +
         align256(static_cast<int64_t>(qlen) * nq * parts * PF_HS * 4) +
         align256(static_cast<int64_t>(qlen) * nq * parts * 4);
}

extern "C" int64_t qp_prefill_workspace_bytes(int qlen, int n, int num_q_heads, int num_kv_heads, int head_size,
                                              int tokens_after_keys) {
  if (qlen <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads || tokens_after_keys < 0) return 0;
  if (head_size == 512) return decode_chunk_workspace_bytes(qlen, n, num_q_heads, num_kv_heads, head_size);
  const int after = std::min(tokens_after_keys, qlen);
  const int group = num_q_heads / num_kv_heads;
  // either cache format (the chunk count depends on the cell size)
  int64_t need = 0;
  for (int cell : {PF_HS + 8, PF_HS * 3 / 2 + 8}) {
    const PrefillPlan pl = prefill_plan(qlen, n, after, num_kv_heads, group, device_sm_count(), cell);
    need = std::max(need, prefill_ws_bytes(qlen, num_q_heads, static_cast<int64_t>(num_kv_heads) * pl.mt_per_kv,
                                           pl.parts));
  }
  return need;
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
  prefill_kernel<FMT><<<ctas, PF1_THREADS, PfCfg<FMT>::BYTES, st>>>(pp);
  return check_launch("prefill");
}

// ---------------------------------------------------------------------------------------------------- piece fold
// The pieces of every M-tile (one per CTA that worked on it, a few at most) folded by log-sum-exp, with the inverse
// RHT (out_mode 0) or as the fp32 RHT-domain output and its base-2 lse (out_mode 1): one warp per (token, query head)
// row, lane s reading piece s's lse, lane l holding channels 8 l .. 8 l + 7 (the layout of the warp's 256-point WHT).
// The general merge (K2) runs one 512-thread CTA per row, sized for decode's hundred splits; over the prefill's
// tens of thousands of rows of a few pieces each its per-CTA overhead dominated.
constexpr int FOLD_WARPS = 8;
constexpr int FOLD_MAX_PARTS = 32;

template <int DT>
__global__ void __launch_bounds__(32 * FOLD_WARPS) prefill_fold_kernel(const float* part_o, const float* part_lse,
                                                                        int64_t rows, int nq, int parts, int mode,
                                                                        void* out, int64_t out_st, int64_t out_sh,
                                                                        float* lse_out, const uint32_t* sign_bits,
                                                                        float out_scale) {
  const int lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * FOLD_WARPS + (threadIdx.x >> 5);  // token * nq + head
  if (r >= rows) return;
  const int64_t tok = r / nq;
  const int qh = static_cast<int>(r % nq);
  const float l_me = lane < parts ? part_lse[r * parts + lane] : -INFINITY;  // absent pieces hold -inf
  const float M = warp_max(l_me);
  const float w_me = (M == -INFINITY || l_me == -INFINITY) ? 0.f : exp2f(l_me - M);
  const float T = warp_sum(w_me);
  const float* po = part_o + r * parts * PF_HS + 8 * lane;
  float x[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = 0.f;
  for (int s = 0; s < parts; ++s) {
    const float w = __shfl_sync(0xffffffffu, w_me, s);
    if (w != 0.f) {  // the same in every lane; an absent piece's partial is never read
      const float4 a = *reinterpret_cast<const float4*>(po + s * PF_HS);
      const float4 b = *reinterpret_cast<const float4*>(po + s * PF_HS + 4);
      x[0] = fmaf(w, a.x, x[0]);
      x[1] = fmaf(w, a.y, x[1]);
      x[2] = fmaf(w, a.z, x[2]);
      x[3] = fmaf(w, a.w, x[3]);
      x[4] = fmaf(w, b.x, x[4]);
      x[5] = fmaf(w, b.y, x[5]);
      x[6] = fmaf(w, b.z, x[6]);
      x[7] = fmaf(w, b.w, x[7]);
    }
  }
  const float inv = T > 0.f ? 1.f / T : 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] *= inv;
  if (mode == 1) {
    float* dst = reinterpret_cast<float*>(out) + tok * out_st + qh * out_sh + 8 * lane;
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[i] = x[i];
    if (lane == 0 && lse_out) lse_out[r] = T > 0.f ? M + log2f(T) : -INFINITY;
    return;
  }
  warp_wht<8>(x, lane);
  apply_signs<8>(x, sign_bits, lane);
  using EL = Elem<DT>;
  typename EL::T* dst = reinterpret_cast<typename EL::T*>(out) + tok * out_st + qh * out_sh + 8 * lane;
#pragma unroll
  for (int i = 0; i < 8; ++i) dst[i] = EL::from_f(x[i] * out_scale);
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
  if (head_size != PF_HS && head_size != 512)
    return set_error(QP_ERR_UNSUPPORTED, "prefill: head size %d (this build: 256, 512)", head_size);
  const int after = std::min(std::max(tokens_after_keys, 0), std::max(qlen, 0));  // >= qlen: nothing masked
  if (tokens_after_keys < 0 || qlen < 0 || n < qlen - after || (qlen > 0 && n <= 0) || num_kv_heads <= 0 ||
      num_q_heads <= 0 || num_q_heads % num_kv_heads)
    return set_error(QP_ERR_INVALID, "prefill: bad sizes (qlen %d, n %d, heads %d/%d)", qlen, n, num_q_heads,
                     num_kv_heads);
  if (qlen == 0) return QP_OK;
  if (out_mode != 0 && out_mode != 1) return set_error(QP_ERR_INVALID, "prefill: out_mode %d", out_mode);
  if (head_size == 512) {  // O^T of a 128-query tile would need all of TMEM: the split-KV kernel's chunk mode
    if (!q || !out || !block_row || !cache || !rht_sign_bits || !workspace)
      return set_error(QP_ERR_INVALID, "prefill: null pointer");
    return decode_chunk_prefill(fmt, dtype, q, q_stride_token, q_stride_head, out, out_stride_token, out_stride_head,
                                qlen, n, block_row, cache, block_size, block_stride, head_stride, slot_stride, k_off,
                                ks_off, v_off, vs_off, num_q_heads, num_kv_heads, head_size, softmax_scale,
                                rht_sign_bits, q_rotated, tokens_after_keys, out_mode, lse_out, workspace,
                                workspace_bytes, stream);
  }
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
  const PrefillPlan pl = prefill_plan(qlen, n, after, num_kv_heads, group, device_sm_count(), cell);
  const int mt = pl.mt_per_kv, ctas = pl.ctas, parts = pl.parts;
  const int64_t total = pl.total;
  if (total >= (int64_t(1) << 31))  // the kernel walks its schedule in 32-bit counters
    return set_error(QP_ERR_UNSUPPORTED, "prefill: %lld (128-query, 64-key) tiles exceed the 2^31 the schedule counts",
                     (long long)total);
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
#define QP_QPREP(F, D)                                                                                         \
  prefill_qprep_kernel<F, D><<<qgrid, 256, 0, st>>>(q, q_stride_token, q_stride_head, qlen, num_q_heads,   \
                                                        num_kv_heads, group, mt, rht_sign_bits, q_rotated,      \
                                                        qk_scale, qprep, qscale, part_lse, lse_count)
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
  pp.chunk_tiles = pl.chunk_tiles;
  pp.piece_stride = pl.piece_stride;
  pp.chunks = pl.chunks;
  for (int j = 0; j < pl.chunks; ++j) pp.chunk_total[j] = pl.chunk_total[j];
  rc = fmt == FMT_INT4 ? launch_prefill_main<FMT_INT4>(pp, ctas, st) : launch_prefill_main<FMT_K8V4>(pp, ctas, st);
  if (rc) return rc;
  if (parts <= FOLD_MAX_PARTS) {
    if (!out || (out_mode == 0 && !rht_sign_bits)) return set_error(QP_ERR_INVALID, "prefill: null output / signs");
    const int64_t rows = static_cast<int64_t>(qlen) * num_q_heads;
    const unsigned grid = static_cast<unsigned>((rows + FOLD_WARPS - 1) / FOLD_WARPS);
    const float out_scale = 1.f / static_cast<float>(head_size);
    if (dtype == DT_BF16)
      prefill_fold_kernel<DT_BF16><<<grid, 32 * FOLD_WARPS, 0, st>>>(part_o, part_lse, rows, num_q_heads, parts,
                                                                     out_mode, out, out_stride_token,
                                                                     out_stride_head, lse_out, rht_sign_bits,
                                                                     out_scale);
    else
      prefill_fold_kernel<DT_F16><<<grid, 32 * FOLD_WARPS, 0, st>>>(part_o, part_lse, rows, num_q_heads, parts,
                                                                    out_mode, out, out_stride_token, out_stride_head,
                                                                    lse_out, rht_sign_bits, out_scale);
    return check_launch("prefill fold");
  }
  return qp_merge_attn_partials(dtype, head_size, qlen, num_q_heads, parts, part_o,
                                static_cast<int64_t>(num_q_heads) * parts * PF_HS, static_cast<int64_t>(parts) * PF_HS,
                                PF_HS, part_lse, static_cast<int64_t>(num_q_heads) * parts, parts, 1, out_mode, out,
                                out_stride_token, out_stride_head, lse_out, rht_sign_bits, stream);
}
