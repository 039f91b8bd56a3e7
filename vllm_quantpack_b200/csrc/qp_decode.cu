// K1: split-KV paged decode over an int4_per_token_head / k8v4_per_token_head cache, up to 32 query rows
//     (qlen x query heads per KV head) per KV head, 64-token tiles; and K2: log-sum-exp merge of the segments with
//     the inverse RHT fused in.
//
// Reference behaviour (what this computes, not how): the split-KV 3D path of vLLM's int4 kernel as the plugin
// configures it (vllm_quantpack/attention/int4_kv.py:98-122: 64-token tiles, every query token of a step in one
// program, segments sized to the SM count) and vLLM's reduce_segments (vllm/v1/attention/ops/
// triton_unified_attention.py:645-732 in vLLM 0.22). Scores S = (Q.u - Q_sum zp) k_scale scale, P_v = P v_scale,
// out += P_v16 u - sum(P_v16 zp) with the same rounded P_v16 in both terms (int4_kv.py:80-94).
//
// B200 design:
// - one CTA (4 warps) per (split, KV head, sequence); the segment's cells stream through a 2-stage shared-memory
//   ring filled by 1-D bulk copies (TMA engine), each warp copying its own 16-token group of a tile, completing on
//   mbarriers;
// - K0q (a small kernel before K1) rotates (RHT) and scales every query row once into fp16 with a per-row power of
//   two, its channels permuted so that the nibble extraction below needs no shuffles (odd, high-nibble, channels
//   carry a factor 1/16), and stores it as the exact shared-memory image of the row; K1 starts under programmatic
//   dependent launch, issues its first cache copies, then waits for K0q and fetches its rows with one bulk copy;
// - QK: mma.sync m16n8k16 with the keys as M (16 tokens per warp) and the query rows as N (8 per n-tile). Key
//   nibbles become fp16 by the exponent-bias trick ((w & 0x000F000F) | 0x64006400 = 1024 + u): one lop3 per two
//   values, the bias removed once per score (Q.1024 is a per-row constant);
// - softmax in log2 units with the row max exchanged through shared memory, the V scale folded into P (P_v16 in fp16
//   with a running power-of-two range);
// - PV: mma.sync with the head dimension as M (64 channels per warp) and the query rows as N; the value nibbles of
//   two tokens are interleaved by prmt so each register holds one channel of two tokens, converted to the exact
//   fp16 (u - zp) of each token. The zero point sits in the operand, so the accumulator that runs over the whole
//   segment only ever holds the signal; the reference subtracts sum(P_v16 zp) once per tile instead
//   (int4_kv.py:90-92), which a running accumulator over many tiles cannot do without its rounding bias showing;
// - each split writes its normalised partial O (fp32, RHT domain) and its log2-sum-exp; K2 folds the splits and
//   applies the inverse RHT / head, launched with programmatic dependent launch so its launch overlaps K1.
#include <math.h>

#include "qp_api_internal.h"
#include "qp_common.cuh"

namespace qp {

constexpr int DEC_TILE = 64;
constexpr int DEC_STAGES = 2;
constexpr int DEC_THREADS = 128;
constexpr int DEC_HS = 256;
constexpr int DEC_MAX_ROWS = 32;
constexpr int Q_STRIDE = DEC_HS * 2 + 16;  // bytes per Q row in shared memory (conflict-free ldmatrix)
constexpr float LOG2E = 1.4426950408889634f;

struct DecodeParams {
  const void* q;
  int64_t q_st, q_sh;  // element strides of q (token, head)
  const int32_t* cu_seqlens_q;
  const int32_t* seqused_k;
  const int32_t* block_table;
  int64_t bt_stride;
  const uint8_t* cache;
  int block_size;
  int64_t block_stride, head_stride;  // bytes; cells of one (block, head) are contiguous (slot stride == cell)
  int ks_off, v_off, vs_off;
  int nq, nkv, group;  // query heads, KV heads, query heads per KV head
  float qk_scale;      // softmax_scale / head_size * log2(e)
  const uint32_t* sign_bits;
  int q_rotated;  // q already in the RHT domain
  const uint8_t* qrec;  // prepared query rows: [kv head][token][query head of the group] x Q_STRIDE bytes
  int64_t num_tokens;
  int tokens_after;  // sequence tokens after this call's keys (held by other ranks), clamped to max_seqlen_q
  int num_splits;
  float* part_o;    // [tokens][nq][splits][HS]
  float* part_lse;  // [tokens][nq][splits], log2 units
};

template <int FMT>
struct Cell {
  static constexpr int BYTES = FMT == FMT_INT4 ? DEC_HS + 8 : DEC_HS * 3 / 2 + 8;
};

template <int NT>
struct PLayout {
  // P^T in shared memory: [64 tokens][8 NT rows] fp16, row stride chosen for conflict-free ldmatrix.trans
  static constexpr int STRIDE = NT == 1 ? 16 : (NT == 2 ? 48 : (NT == 3 ? 48 : 80));
};

template <int FMT, int NT>
struct DecSmem {
  static constexpr int CELL = Cell<FMT>::BYTES;
  static constexpr int ROWS = 8 * NT;  // query rows held (padded to whole n-tiles)
  static constexpr int STAGE_BYTES = DEC_TILE * CELL;
  static constexpr int P_BYTES = DEC_TILE * PLayout<NT>::STRIDE;
  static constexpr int OFF_STAGES = 0;
  static constexpr int OFF_Q = OFF_STAGES + DEC_STAGES * STAGE_BYTES;
  static constexpr int OFF_P = OFF_Q + ROWS * Q_STRIDE;       // 2 buffers (alternate tiles)
  static constexpr int OFF_RED = OFF_P + 2 * P_BYTES;         // [ROWS][4 warps] f32 (row max, then l)
  static constexpr int OFF_VS = OFF_RED + ROWS * 4 * 4;       // [4] f32 (value-scale max per warp)
  static constexpr int OFF_ZB = OFF_VS + 16;                  // [2 buffers][lo, hi][64] u16 zero-point biases
  static constexpr int OFF_BAR = (OFF_ZB + 2 * 2 * DEC_TILE * 2 + 7) / 8 * 8;
  static constexpr int BYTES = OFF_BAR + (DEC_STAGES + 1) * 8;  // stage barriers, then the Q-rows barrier
};

// k index (0..255) of the QK MMA that carries channel c (see the fragment mapping in decode_kernel).
template <int FMT>
__device__ __forceinline__ int qk_k_of_channel(int c) {
  if constexpr (FMT == FMT_INT4) {
    // word W = 8 t + j of the key row feeds k-steps 2j (h = 0) and 2j + 1 (h = 1) of lane quad t; inside the word,
    // nibble r = (2h + f) + 4e is element e of register f.
    const int W = c >> 3, r = c & 7;
    const int t = W >> 3, j = W & 7;
    const int h = (r & 3) >> 1, f = r & 1, e = r >> 2;
    return 16 * (2 * j + h) + 2 * t + e + 8 * f;
  } else {
    // word W of the int8 key row: k-step s = W & 7 (W < 32) or 8 + (W & 7) (W >= 32) of lane quad t = (W >> 3) & 3;
    // byte 2f + e is element e of register f.
    const int W = c >> 2;
    const int f = (c >> 1) & 1, e = c & 1;
    const int t = (W >> 3) & 3;
    const int s = (W < 32 ? 0 : 8) + (W & 7);
    return 16 * s + 2 * t + e + 8 * f;
  }
}

// Row of P^T (the PV MMA's k index inside the tile) that holds tile-local token tau: lane quad t of k-step kk reads
// tokens 16 kk + 4 t + {0, 1, 2, 3} as k = 2 t, 2 t + 1, 2 t + 8, 2 t + 9.
__device__ __forceinline__ int pv_k_of_token(int tau) {
  const int kk = tau >> 4, u = tau & 15;
  const int t = u >> 2, f = (u >> 1) & 1, e = u & 1;
  return 16 * kk + 2 * t + e + 8 * f;
}

// fp16 pair -> exact (nibble - zero point) of two tokens a, b: the low-nibble form (1024 + u) minus (1024 + zp), the
// high-nibble form (1024 + 16 u) / 16 - (64 + zp). The zero point enters the operand itself (not a correction summed
// apart), so the fp32 accumulator only ever holds the signal sum P (u - zp).
__device__ __forceinline__ uint32_t nib_lo(uint32_t x, uint32_t lo_bias) {
  return hsub2_u32(lop3_and_or(x, 0x000F000Fu, 0x64006400u), lo_bias);
}
__device__ __forceinline__ uint32_t nib_hi(uint32_t x, uint32_t hi_bias) {
  return hfma2_u32(lop3_and_or(x, 0x00F000F0u, 0x64006400u), 0x2C002C00u /* 1/16 */, hi_bias);
}

// Online softmax with a lazy maximum: P = exp2(s - m_used) is allowed up to 2^RESCALE_SLACK, so the O accumulators
// are rescaled only when a row maximum grows by more than that (rare after the first tiles), not every tile. Every
// thread checks its own scores against m_used; only when some score (or value scale) leaves the allowed range does
// the CTA take the slow path that exchanges the exact tile maxima.
constexpr float RESCALE_SLACK = 8.f;


// ---------------------------------------------------------------------------------------------------- K0q
// One warp per (query token, query head): the row as the decode kernel holds it in shared memory (Q_STRIDE bytes):
// 256 fp16 in the k order of the QK MMA, scaled by a power of two (|q| < 2^14), odd int4 channels x 1/16; then the
// row's score scale (softmax_scale / head x log2 e x 2^-exponent), its bias sum (Q . 1024 / 64 / 1152 per channel
// kind) and its plain sum, as fp32 at byte 512. Written once per call; every split of the row's KV head reads it.
template <int FMT, int DT>
__global__ void __launch_bounds__(256) decode_qprep_kernel(const void* q, int64_t q_st, int64_t q_sh, int64_t T,
                                                           int nq, int nkv, const uint32_t* sign_bits, int q_rotated,
                                                           float qk_scale, uint8_t* qrec) {
  asm volatile("griddepcontrol.launch_dependents;");
  using EL = Elem<DT>;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= T * nq) return;
  const int64_t tok = row / nq;
  const int qh = static_cast<int>(row % nq);
  const int group = nq / nkv, kvh = qh / group, hg = qh % group;
  uint8_t* rec = qrec + ((static_cast<int64_t>(kvh) * T + tok) * group + hg) * Q_STRIDE;
  __half* qrow = reinterpret_cast<__half*>(rec);
  const typename EL::T* src = reinterpret_cast<const typename EL::T*>(q) + tok * q_st + qh * q_sh + lane * 8;
  float x[8];
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
  int ex = 0;
  if (am > 0.f) {
    frexpf(am, &ex);  // am < 2^ex
    ex = 14 - ex;     // am * 2^ex in [2^13, 2^14)
  }
  float cq = 0.f, qs = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = lane * 8 + i;
    const __half h = __float2half_rn(ldexpf(x[i], ex));
    const float hv = __half2float(h);
    qs += hv;
    if constexpr (FMT == FMT_INT4) {
      const bool odd = c & 1;
      cq += odd ? 64.f * hv : 1024.f * hv;
      qrow[qk_k_of_channel<FMT>(c)] = odd ? __float2half_rn(hv * 0.0625f) : h;
    } else {
      cq += 1152.f * hv;
      qrow[qk_k_of_channel<FMT>(c)] = h;
    }
  }
  cq = warp_sum(cq);
  qs = warp_sum(qs);
  if (lane == 0) {
    float* rc = reinterpret_cast<float*>(rec + 2 * DEC_HS);
    rc[0] = ldexpf(qk_scale, -ex);
    rc[1] = cq;
    rc[2] = qs;
    rc[3] = 0.f;
  }
}

template <int FMT, int DT, int NT>
__global__ void __launch_bounds__(DEC_THREADS, NT == 4 ? 2 : 3) decode_kernel(const DecodeParams p) {
  using SM = DecSmem<FMT, NT>;
  constexpr int CELL = SM::CELL;
  constexpr int ROWS = SM::ROWS;
  constexpr int PSTRIDE = PLayout<NT>::STRIDE;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* stages = smem + SM::OFF_STAGES;
  uint8_t* qsm = smem + SM::OFF_Q;
  float* red = reinterpret_cast<float*>(smem + SM::OFF_RED);
  float* red_vs = reinterpret_cast<float*>(smem + SM::OFF_VS);
  uint16_t* zbuf = reinterpret_cast<uint16_t*>(smem + SM::OFF_ZB);  // [buf][lo/hi][64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::OFF_BAR);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int split = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;

  // Let the merge kernel (launched with programmatic stream serialization) start its launch now; it waits for this
  // grid's completion before reading anything.
  asm volatile("griddepcontrol.launch_dependents;");

  const int q0 = p.cu_seqlens_q[seq];
  const int qlen = p.cu_seqlens_q[seq + 1] - q0;
  const int n = p.seqused_k[seq];
  const int rows = qlen * p.group;
  if (qlen <= 0) return;

  const int n_tiles = (n + DEC_TILE - 1) / DEC_TILE;
  const int tps = (n_tiles + p.num_splits - 1) / p.num_splits;
  const int tile0 = split * tps;
  const int ntl = max(0, min(tile0 + tps, n_tiles) - tile0);

  if (ntl == 0) {  // empty segment: lse = -inf
    for (int r = tid; r < rows; r += DEC_THREADS) {
      const int tok = q0 + r / p.group, qh = kvh * p.group + r % p.group;
      p.part_lse[(static_cast<int64_t>(tok) * p.nq + qh) * p.num_splits + split] = -INFINITY;
    }
    return;
  }

  const int32_t* btab = p.block_table + static_cast<int64_t>(seq) * p.bt_stride;
  const uint8_t* head_base = p.cache + static_cast<int64_t>(kvh) * p.head_stride;

  // --- copies: warp w copies 16-token group w of every tile (block_size % 16 == 0, so a group never crosses a block),
  // one bulk copy each, arriving with its byte count on the tile's stage barrier (4 arrivals per phase). The group's
  // block-table index and in-block offset advance by one tile at a time (no division in the loop); its block entry
  // is loaded one tile ahead.
  int gb_tok = tile0 * DEC_TILE + 16 * warp;  // first token of this warp's group of the tile to fetch next
  int gb_idx = gb_tok / p.block_size;
  int gb_off = gb_tok - gb_idx * p.block_size;
  auto advance_group = [&]() {
    gb_tok += DEC_TILE;
    gb_off += DEC_TILE;
    while (gb_off >= p.block_size) {
      gb_off -= p.block_size;
      ++gb_idx;
    }
  };
  auto fetch_block = [&](int i) { return (i < ntl && gb_tok < n) ? __ldg(btab + gb_idx) : -1; };
  auto issue_group = [&](int stage, int blk, int inb) {
    if (lane == 0) {
      if (blk >= 0) {
        mbar_arrive_expect_tx(&bars[stage], static_cast<uint32_t>(16 * CELL));
        bulk_g2s(stages + stage * SM::STAGE_BYTES + warp * 16 * CELL,
                 head_base + static_cast<int64_t>(blk) * p.block_stride + static_cast<int64_t>(inb) * CELL,
                 static_cast<uint32_t>(16 * CELL), &bars[stage]);
      } else {
        mbar_arrive(&bars[stage]);
      }
    }
  };

  if (tid == 0) {
    for (int s = 0; s < DEC_STAGES; ++s) mbar_init(&bars[s], 4);
    mbar_init(&bars[DEC_STAGES], 1);
    fence_mbar_init();
  }
  __syncthreads();
  const int issued0 = min(ntl, DEC_STAGES);
  int issued = issued0;  // tiles whose copies every warp has issued
  {
    int blk[DEC_STAGES], off[DEC_STAGES];
#pragma unroll
    for (int i = 0; i < DEC_STAGES; ++i) {
      blk[i] = fetch_block(i);
      off[i] = gb_off;
      advance_group();
    }
#pragma unroll
    for (int i = 0; i < DEC_STAGES; ++i)
      if (i < issued0) issue_group(i, blk[i], off[i]);
  }
  int next_blk = fetch_block(issued), next_inb = gb_off;  // this warp's group of tile `issued`

  // --- Q rows: prepared by K0q (programmatic dependent launch: wait for it only now) --------------------------
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (tid == 0) {
    const uint8_t* src = p.qrec + ((static_cast<int64_t>(kvh) * p.num_tokens + q0) * p.group) * Q_STRIDE;
    mbar_arrive_expect_tx(&bars[DEC_STAGES], static_cast<uint32_t>(rows * Q_STRIDE));
    bulk_g2s(qsm, src, static_cast<uint32_t>(rows * Q_STRIDE), &bars[DEC_STAGES]);
  }
  for (int idx = rows * (Q_STRIDE / 16) + tid; idx < ROWS * (Q_STRIDE / 16); idx += DEC_THREADS)
    reinterpret_cast<uint4*>(qsm)[idx] = make_uint4(0u, 0u, 0u, 0u);  // padding rows: zero
  bool failed = !mbar_wait_bounded(&bars[DEC_STAGES], 0);
  __syncthreads();

  // --- per-thread state: this thread's query rows are r = 8 nt + 2 t + e ------------------------------------
  float qsc[NT][2], qcq[NT][2], qsum[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float* rc = reinterpret_cast<const float*>(qsm + (8 * nt + 2 * t + e) * Q_STRIDE + 2 * DEC_HS);
      qsc[nt][e] = rc[0];
      qcq[nt][e] = rc[1];
      qsum[nt][e] = rc[2];
    }
  float o[4][NT][4];
#pragma unroll
  for (int mt = 0; mt < 4; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int c = 0; c < 4; ++c) o[mt][nt][c] = 0.f;
  float m_used[NT][2], l_part[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      m_used[nt][e] = -INFINITY;
      l_part[nt][e] = 0.f;
    }
  int e_run = -1000;    // running power-of-two range of P_v (value scales): every value scale < 2^e_run
  float pv_mul = 0.f;   // 2^-e_run
  float v_limit = 0.f;  // 2^e_run
  // query token i sits at position n - qlen + i + tokens_after of the keys; keys >= causal_from are hidden from some
  // row or lie past the context
  const int vis_base = n - qlen + p.tokens_after;  // last key query token 0 sees (before clamping to n - 1)
  const int causal_from = min(n, vis_base + 1);
  const uint32_t qsm_base = smem_u32(qsm);
  const int tau_a = 16 * warp + g, tau_b = tau_a + 8;
  const int pk_a = pv_k_of_token(tau_a) * PSTRIDE, pk_b = pv_k_of_token(tau_b) * PSTRIDE;
  int fail_tile = ntl;

  int stage = 0;         // i % DEC_STAGES
  uint32_t sphase = 0;   // (i / DEC_STAGES) & 1
  for (int i = 0; i < ntl; ++i) {
    const int buf = i & 1;
    uint8_t* psm = smem + SM::OFF_P + buf * SM::P_BYTES;
    uint16_t* zb_lo = zbuf + buf * 2 * DEC_TILE;
    uint16_t* zb_hi = zb_lo + DEC_TILE;
    // A thread whose wait runs out keeps going on whatever the stage holds (nothing reaches global memory before
    // the epilogue); the CTA leaves together at barrier (B), so no thread skips a __syncthreads.
    failed |= !mbar_wait_bounded(&bars[stage], sphase);
    const uint8_t* tile = stages + stage * SM::STAGE_BYTES;
    const int tok_base = (tile0 + i) * DEC_TILE;

    // ---------------- QK: warp handles tokens 16 warp + [0, 16) ----------------
    float sacc[NT][4], sacc2[NT][4];  // two accumulator chains (even / odd k-steps), summed after the loop
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int c = 0; c < 4; ++c) sacc[nt][c] = sacc2[nt][c] = 0.f;
    const uint8_t* rowg = tile + tau_a * CELL;
    const uint8_t* rowg8 = rowg + 8 * CELL;
    if constexpr (FMT == FMT_INT4) {
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const uint2 wa = *reinterpret_cast<const uint2*>(rowg + 4 * (8 * t + 2 * jj));
        const uint2 wb = *reinterpret_cast<const uint2*>(rowg8 + 4 * (8 * t + 2 * jj));
#pragma unroll
        for (int hw = 0; hw < 2; ++hw) {
          const int j = 2 * jj + hw;
          const uint32_t xa = hw ? wa.y : wa.x, xb = hw ? wb.y : wb.x;
          const uint32_t xa8 = xa >> 8, xb8 = xb >> 8;
          uint32_t A0[4], A1[4];  // k-steps 2j (h = 0) and 2j + 1 (h = 1)
          A0[0] = lop3_and_or(xa, 0x000F000Fu, 0x64006400u);
          A0[1] = lop3_and_or(xb, 0x000F000Fu, 0x64006400u);
          A0[2] = lop3_and_or(xa, 0x00F000F0u, 0x64006400u);
          A0[3] = lop3_and_or(xb, 0x00F000F0u, 0x64006400u);
          A1[0] = lop3_and_or(xa8, 0x000F000Fu, 0x64006400u);
          A1[1] = lop3_and_or(xb8, 0x000F000Fu, 0x64006400u);
          A1[2] = lop3_and_or(xa8, 0x00F000F0u, 0x64006400u);
          A1[3] = lop3_and_or(xb8, 0x00F000F0u, 0x64006400u);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            uint32_t b0, b1, b2, b3;
            ldmatrix_x4(b0, b1, b2, b3, qsm_base + (8 * nt + (lane & 7)) * Q_STRIDE + (32 * j + 8 * (lane >> 3)) * 2);
            mma_f16_16816(sacc[nt], A0, b0, b1);
            mma_f16_16816(sacc2[nt], A1, b2, b3);
          }
        }
      }
    } else {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int wbase = half * 32 + 8 * t + 2 * jj;  // words wbase, wbase + 1 = k-steps s0, s0 + 1
          const int s0 = half * 8 + 2 * jj;
          const uint2 wa = *reinterpret_cast<const uint2*>(rowg + 4 * wbase);
          const uint2 wb = *reinterpret_cast<const uint2*>(rowg8 + 4 * wbase);
          uint32_t A[2][4];
#pragma unroll
          for (int hw = 0; hw < 2; ++hw) {
            const uint32_t xa = (hw ? wa.y : wa.x) ^ 0x80808080u, xb = (hw ? wb.y : wb.x) ^ 0x80808080u;
            A[hw][0] = prmt(xa, 0x64646464u, 0x4140u);  // {1024 + 128 + c0, 1024 + 128 + c1}
            A[hw][1] = prmt(xb, 0x64646464u, 0x4140u);
            A[hw][2] = prmt(xa, 0x64646464u, 0x4342u);  // {.. + c2, .. + c3}
            A[hw][3] = prmt(xb, 0x64646464u, 0x4342u);
          }
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            uint32_t b0, b1, b2, b3;
            ldmatrix_x4(b0, b1, b2, b3, qsm_base + (8 * nt + (lane & 7)) * Q_STRIDE + (16 * s0 + 8 * (lane >> 3)) * 2);
            mma_f16_16816(sacc[nt], A[0], b0, b1);
            mma_f16_16816(sacc2[nt], A[1], b2, b3);
          }
        }
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int c = 0; c < 4; ++c) sacc[nt][c] += sacc2[nt][c];

    // ---------------- scores (log2 units) and masks ----------------
    const int tok_a = tok_base + tau_a, tok_b = tok_base + tau_b;
    const uint32_t kwa = *reinterpret_cast<const uint32_t*>(tile + tau_a * CELL + p.ks_off);
    const uint32_t kwb = *reinterpret_cast<const uint32_t*>(tile + tau_b * CELL + p.ks_off);
    const uint32_t vwa = *reinterpret_cast<const uint32_t*>(tile + tau_a * CELL + p.vs_off);
    const uint32_t vwb = *reinterpret_cast<const uint32_t*>(tile + tau_b * CELL + p.vs_off);
    float ks_a, ks_b, kz_a = 0.f, kz_b = 0.f;
    if constexpr (FMT == FMT_INT4) {
      ks_a = __uint_as_float(kwa & 0xFFFFFFF0u);
      ks_b = __uint_as_float(kwb & 0xFFFFFFF0u);
      kz_a = static_cast<float>(kwa & 0xFu);
      kz_b = static_cast<float>(kwb & 0xFu);
    } else {
      ks_a = __uint_as_float(kwa);
      ks_b = __uint_as_float(kwb);
    }
    // value scales of this thread's two tokens (tokens past the end count as scale 0)
    const float vs_a = tok_a < n ? __uint_as_float(vwa & 0xFFFFFFF0u) : 0.f;
    const float vs_b = tok_b < n ? __uint_as_float(vwb & 0xFFFFFFF0u) : 0.f;
    if (t == 0) {  // zero-point biases of the value operand, per token (read by the PV phase after barrier B)
      zb_lo[tau_a] = static_cast<uint16_t>(0x6400u | (vwa & 0xFu));
      zb_lo[tau_b] = static_cast<uint16_t>(0x6400u | (vwb & 0xFu));
      zb_hi[tau_a] = static_cast<uint16_t>(0xD400u | ((vwa & 0xFu) << 4));
      zb_hi[tau_b] = static_cast<uint16_t>(0xD400u | ((vwb & 0xFu) << 4));
    }
    const bool need_mask = tok_base + DEC_TILE > causal_from;
    float sc[NT][4];
    bool grow = vs_a >= v_limit || vs_b >= v_limit;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float s0 = (sacc[nt][e] - fmaf(kz_a, qsum[nt][e], qcq[nt][e])) * (ks_a * qsc[nt][e]);
        float s1 = (sacc[nt][2 + e] - fmaf(kz_b, qsum[nt][e], qcq[nt][e])) * (ks_b * qsc[nt][e]);
        if (need_mask) {
          const int r = 8 * nt + 2 * t + e;
          const int lim = r < rows ? min(n - 1, vis_base + r / p.group) : -1;  // last key this row sees
          if (tok_a > lim) s0 = -INFINITY;                                      // also past the context
          if (tok_b > lim) s1 = -INFINITY;
        }
        sc[nt][e] = s0;
        sc[nt][2 + e] = s1;
        grow |= fmaxf(s0, s1) > m_used[nt][e] + RESCALE_SLACK;
      }
    }

    // ---------------- P with the current maximum and value range (optimistic) ----------------
    float psum[NT][2];
    auto make_p = [&]() {
      const float va = vs_a * pv_mul, vb = vs_b * pv_mul;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float pv[4];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float base = m_used[nt][e] == -INFINITY ? 0.f : m_used[nt][e];
          const float pa = fast_exp2(sc[nt][e] - base);
          const float pb = fast_exp2(sc[nt][2 + e] - base);
          psum[nt][e] = pa + pb;
          pv[e] = pa * va;
          pv[2 + e] = pb * vb;
        }
        // P_v rounded to fp16: the operand of the PV MMA
        *reinterpret_cast<__half2*>(psm + pk_a + (8 * nt + 2 * t) * 2) = __floats2half2_rn(pv[0], pv[1]);
        *reinterpret_cast<__half2*>(psm + pk_b + (8 * nt + 2 * t) * 2) = __floats2half2_rn(pv[2], pv[3]);
      }
    };
    make_p();

    // this thread's value words for the PV phase: word 8 warp + g of tokens 16 kk + 4 t + j
    uint32_t vw[4][4];
    {
      const uint8_t* vbase = tile + p.v_off + 4 * (8 * warp + g);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
#pragma unroll
        for (int j = 0; j < 4; ++j) vw[kk][j] = *reinterpret_cast<const uint32_t*>(vbase + (16 * kk + 4 * t + j) * CELL);
    }

    // (B) P^T and the zero-point biases visible; the stage is no longer read
    if (__syncthreads_or(grow || failed)) {
      if (__syncthreads_or(failed)) {
        failed = true;
        fail_tile = i;
        break;
      }
      // slow path: exact tile maxima and value range, rescale, recompute P
      float tm[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float mx = fmaxf(sc[nt][e], sc[nt][2 + e]);
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
          tm[nt][e] = mx;
          if (g == 0) red[(8 * nt + 2 * t + e) * 4 + warp] = mx;
        }
      const float vm = warp_max(fmaxf(vs_a, vs_b));
      if (lane == 0) red_vs[warp] = vm;
      __syncthreads();
      const float4 vv = *reinterpret_cast<const float4*>(red_vs);
      const float vmax = fmaxf(fmaxf(vv.x, vv.y), fmaxf(vv.z, vv.w));
      int e_tile = -1000;
      if (vmax > 0.f) frexpf(vmax, &e_tile);  // vmax < 2^e_tile
      const int e_new = max(e_run, e_tile);
      const float o_range = e_run == -1000 ? 0.f : ldexpf(1.f, e_run - e_new);
      e_run = e_new;
      pv_mul = e_new == -1000 ? 0.f : ldexpf(1.f, -e_new);
      v_limit = e_new == -1000 ? 0.f : ldexpf(1.f, e_new);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float4 mv = *reinterpret_cast<const float4*>(red + (8 * nt + 2 * t + e) * 4);
          const float mt_ = fmaxf(fmaxf(mv.x, mv.y), fmaxf(mv.z, mv.w));
          const float m_new = mt_ > m_used[nt][e] + RESCALE_SLACK ? mt_ : m_used[nt][e];
          const float alpha = m_new == m_used[nt][e] ? 1.f : fast_exp2(m_used[nt][e] - m_new);
          m_used[nt][e] = m_new;
          const float ao = alpha * o_range;
          l_part[nt][e] *= alpha;
#pragma unroll
          for (int mt = 0; mt < 4; ++mt) {
            o[mt][nt][e] *= ao;
            o[mt][nt][2 + e] *= ao;
          }
        }
      (void)tm;
      make_p();
      __syncthreads();  // the recomputed P^T visible
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) l_part[nt][e] += psum[nt][e];

    // the stage is free: every warp refills its group with tile i + DEC_STAGES
    if (issued < ntl) {
      issue_group(stage, next_blk, next_inb);  // issued == i + DEC_STAGES: the stage of this tile
      advance_group();
      ++issued;
      next_blk = fetch_block(issued);
      next_inb = gb_off;
    }
    if (++stage == DEC_STAGES) {
      stage = 0;
      sphase ^= 1u;
    }

    // ---------------- PV: warp handles channels 64 warp + [0, 64) ----------------
    const uint32_t psm_base = smem_u32(psm);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t bf[NT][2];
      {
        const int mi = lane >> 3;
        const int krow = 16 * kk + (mi & 1) * 8 + (lane & 7);
        if constexpr (NT == 1) {
          ldmatrix_x2_trans(bf[0][0], bf[0][1], psm_base + krow * PSTRIDE);
        } else {
          ldmatrix_x4_trans(bf[0][0], bf[0][1], bf[1][0], bf[1][1], psm_base + krow * PSTRIDE + (mi >> 1) * 16);
          if constexpr (NT == 3) {
            ldmatrix_x2_trans(bf[2][0], bf[2][1], psm_base + krow * PSTRIDE + 32);
          } else if constexpr (NT == 4) {
            ldmatrix_x4_trans(bf[2][0], bf[2][1], bf[3][0], bf[3][1], psm_base + krow * PSTRIDE + 32 + (mi >> 1) * 16);
          }
        }
      }
      const int tau0 = 16 * kk + 4 * t;
      const uint2 blo = *reinterpret_cast<const uint2*>(zb_lo + tau0);  // {tau0, tau0+1}, {tau0+2, tau0+3}
      const uint2 bhi = *reinterpret_cast<const uint2*>(zb_hi + tau0);
      // f = 0: tokens (tau0, tau0 + 1); f = 1: tokens (tau0 + 2, tau0 + 3)
      uint32_t vr[2][8];  // [f][channel offset 0..7]
#pragma unroll
      for (int f = 0; f < 2; ++f) {
        const uint32_t wa = vw[kk][2 * f], wb = vw[kk][2 * f + 1];
        const uint32_t lo_b = f ? blo.y : blo.x, hi_b = f ? bhi.y : bhi.x;
        const uint32_t x = prmt(wa, wb, 0x5410u), y = prmt(wa, wb, 0x7632u);
        const uint32_t x8 = x >> 8, y8 = y >> 8;
        vr[f][0] = nib_lo(x, lo_b);
        vr[f][1] = nib_hi(x, hi_b);
        vr[f][2] = nib_lo(x8, lo_b);
        vr[f][3] = nib_hi(x8, hi_b);
        vr[f][4] = nib_lo(y, lo_b);
        vr[f][5] = nib_hi(y, hi_b);
        vr[f][6] = nib_lo(y8, lo_b);
        vr[f][7] = nib_hi(y8, hi_b);
      }
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        const uint32_t A[4] = {vr[0][2 * mt], vr[0][2 * mt + 1], vr[1][2 * mt], vr[1][2 * mt + 1]};
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_f16_16816(o[mt][nt], A, bf[nt][0], bf[nt][1]);
      }
    }
  }

  if (failed) {
    // give the copies still in flight a bounded chance to land before the CTA's shared memory goes away
    if (tid == 0) {
      for (int j = fail_tile; j < issued; ++j)
        mbar_wait_bounded(&bars[j % DEC_STAGES], (j / DEC_STAGES) & 1, 100000000ull);
      mbar_wait_bounded(&bars[DEC_STAGES], 0, 100000000ull);
    }
    __syncthreads();
    return;
  }

  // --- epilogue: totals of l, normalised partial O and lse ---------------------------------------------------
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float l = l_part[nt][e];
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
      l_part[nt][e] = l;
    }
  __syncthreads();
  if (g == 0) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) red[(8 * nt + 2 * t + e) * 4 + warp] = l_part[nt][e];
  }
  __syncthreads();
  const float o_unit = e_run == -1000 ? 0.f : ldexpf(1.f, e_run);
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int r = 8 * nt + 2 * t + e;
      if (r >= rows) continue;
      const float4 lv = *reinterpret_cast<const float4*>(red + r * 4);
      const float l = (lv.x + lv.y) + (lv.z + lv.w);
      const int tok = q0 + r / p.group, qh = kvh * p.group + r % p.group;
      const int64_t prow = (static_cast<int64_t>(tok) * p.nq + qh) * p.num_splits + split;
      const float inv = l > 0.f ? o_unit / l : 0.f;
      float v[8];
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        v[2 * mt] = o[mt][nt][e] * inv;
        v[2 * mt + 1] = o[mt][nt][2 + e] * inv;
      }
      float4* dst = reinterpret_cast<float4*>(p.part_o + prow * DEC_HS + 64 * warp + 8 * g);
      dst[0] = make_float4(v[0], v[1], v[2], v[3]);
      dst[1] = make_float4(v[4], v[5], v[6], v[7]);
      if (warp == 0 && g == 0) p.part_lse[prow] = l > 0.f ? m_used[nt][e] + log2f(l) : -INFINITY;
    }
}

// ---------------------------------------------------------------------------------------------------- K2 merge
struct MergeParams {
  const float* part_o;
  const float* part_lse;     // log2 units
  int64_t po_t, po_h, po_s;  // element strides of part_o (token, head, part); channel stride 1
  int64_t pl_t, pl_h, pl_s;
  int num_splits;
  int nq;
  int mode;  // 0: inverse RHT / head, cast to the model dtype; 1: fp32 RHT-domain O and lse (log2) out
  void* out;
  int64_t out_st, out_sh;  // element strides of out
  float* lse_out;          // mode 1 (may be null)
  int64_t lo_t, lo_h;
  const uint32_t* sign_bits;
  float out_scale;  // multiplies the output (mode 0: 1 / head)
};

constexpr int MERGE_THREADS = 512;

template <int DT, int HS>
__global__ void __launch_bounds__(MERGE_THREADS) merge_kernel(const MergeParams p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  constexpr int C4 = HS / 4;              // float4 groups per row
  constexpr int SG = MERGE_THREADS / C4;  // split groups
  constexpr int NW = MERGE_THREADS / 32;
  __shared__ float w_sm[1024];
  __shared__ __align__(16) float acc_sm[SG][HS];
  __shared__ float red[NW];
  __shared__ float tot_sm;
  const int tok = blockIdx.x, qh = blockIdx.y, tid = threadIdx.x;
  const float* lse = p.part_lse + tok * p.pl_t + qh * p.pl_h;
  float mx = -INFINITY;
  for (int s = tid; s < p.num_splits; s += MERGE_THREADS) mx = fmaxf(mx, lse[s * p.pl_s]);
  mx = warp_max(mx);
  if ((tid & 31) == 0) red[tid >> 5] = mx;
  __syncthreads();
  float M = red[0];
#pragma unroll
  for (int i = 1; i < NW; ++i) M = fmaxf(M, red[i]);
  float tot = 0.f;
  for (int s = tid; s < p.num_splits; s += MERGE_THREADS) {
    const float l = lse[s * p.pl_s];
    const float w = (M == -INFINITY || l == -INFINITY) ? 0.f : exp2f(l - M);
    w_sm[s] = w;
    tot += w;
  }
  tot = warp_sum(tot);
  __syncthreads();
  if ((tid & 31) == 0) red[tid >> 5] = tot;
  __syncthreads();
  if (tid == 0) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NW; ++i) s += red[i];
    tot_sm = s;
  }
  const int c4 = tid % C4, sg = tid / C4;
  float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
  const float* po = p.part_o + tok * p.po_t + qh * p.po_h + 4 * c4;
  // 8 partials per round, loads issued before any is used (the partials are L2-resident: latency-bound)
  for (int s0 = sg; s0 < p.num_splits; s0 += 8 * SG) {
    float4 v[8];
    float w[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int s = s0 + k * SG;
      w[k] = s < p.num_splits ? w_sm[s] : 0.f;
      v[k] = w[k] != 0.f ? *reinterpret_cast<const float4*>(po + s * p.po_s) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      a.x = fmaf(w[k], v[k].x, a.x);
      a.y = fmaf(w[k], v[k].y, a.y);
      a.z = fmaf(w[k], v[k].z, a.z);
      a.w = fmaf(w[k], v[k].w, a.w);
    }
  }
  *reinterpret_cast<float4*>(&acc_sm[sg][4 * c4]) = a;
  __syncthreads();
  const float T = tot_sm;
  const float inv = T > 0.f ? 1.f / T : 0.f;
  if (p.mode == 1) {
    for (int c = tid; c < HS; c += MERGE_THREADS) {
      float v = 0.f;
#pragma unroll
      for (int s = 0; s < SG; ++s) v += acc_sm[s][c];
      reinterpret_cast<float*>(p.out)[tok * p.out_st + qh * p.out_sh + c] = v * inv;
    }
    if (tid == 0 && p.lse_out) p.lse_out[tok * p.lo_t + qh * p.lo_h] = T > 0.f ? M + log2f(T) : -INFINITY;
    return;
  }
  if (tid < 32) {
    constexpr int E = HS / 32;
    float x[E];
#pragma unroll
    for (int i = 0; i < E; ++i) {
      float v = 0.f;
#pragma unroll
      for (int s = 0; s < SG; ++s) v += acc_sm[s][tid * E + i];
      x[i] = v * inv;
    }
    warp_wht<E>(x, tid);
    apply_signs<E>(x, p.sign_bits, tid);
    using EL = Elem<DT>;
    typename EL::T* dst = reinterpret_cast<typename EL::T*>(p.out) + tok * p.out_st + qh * p.out_sh + tid * E;
#pragma unroll
    for (int i = 0; i < E; ++i) dst[i] = EL::from_f(x[i] * p.out_scale);
  }
}

template <int DT, int HS>
static int launch_merge(const MergeParams& mp, int num_tokens, cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(num_tokens), static_cast<unsigned>(mp.nq));
  cfg.blockDim = dim3(MERGE_THREADS);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, merge_kernel<DT, HS>, mp);
  if (e != cudaSuccess) return set_error(QP_ERR_CUDA, "merge launch: %s", cudaGetErrorString(e));
  return QP_OK;
}

static int merge_dispatch(const MergeParams& mp, int dtype, int head_size, int64_t num_tokens, cudaStream_t st,
                          bool pdl) {
  if (num_tokens == 0) return QP_OK;
  if (mp.num_splits > 1024) return set_error(QP_ERR_UNSUPPORTED, "merge: %d partials > 1024", mp.num_splits);
  if (num_tokens > 0x7fffffff) return set_error(QP_ERR_UNSUPPORTED, "merge: too many tokens");
  const int nt = static_cast<int>(num_tokens);
  switch (head_size) {
    case 256:
      return dtype == DT_BF16 ? launch_merge<DT_BF16, 256>(mp, nt, st, pdl) : launch_merge<DT_F16, 256>(mp, nt, st, pdl);
    case 512:
      return dtype == DT_BF16 ? launch_merge<DT_BF16, 512>(mp, nt, st, pdl) : launch_merge<DT_F16, 512>(mp, nt, st, pdl);
    case 128:
      return dtype == DT_BF16 ? launch_merge<DT_BF16, 128>(mp, nt, st, pdl) : launch_merge<DT_F16, 128>(mp, nt, st, pdl);
    default:
      return set_error(QP_ERR_UNSUPPORTED, "merge: head size %d", head_size);
  }
}

template <int FMT, int DT, int NT>
static int launch_decode_t(const DecodeParams& dp, int num_seqs, cudaStream_t st) {
  using SM = DecSmem<FMT, NT>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(decode_kernel<FMT, DT, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, SM::BYTES);
    if (e != cudaSuccess) return set_error(QP_ERR_CUDA, "decode smem attribute: %s", cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  // programmatic dependent launch: the CTAs start their cache copies while K0q finishes (they wait for it before
  // reading the query rows)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(dp.num_splits), static_cast<unsigned>(dp.nkv), static_cast<unsigned>(num_seqs));
  cfg.blockDim = dim3(DEC_THREADS);
  cfg.dynamicSmemBytes = SM::BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, decode_kernel<FMT, DT, NT>, dp);
  if (e != cudaSuccess) return set_error(QP_ERR_CUDA, "decode launch: %s", cudaGetErrorString(e));
  return QP_OK;
}

template <int FMT, int DT>
static int launch_decode_nt(const DecodeParams& dp, int nt, int num_seqs, cudaStream_t st) {
  switch (nt) {
    case 1: return launch_decode_t<FMT, DT, 1>(dp, num_seqs, st);
    case 2: return launch_decode_t<FMT, DT, 2>(dp, num_seqs, st);
    case 3: return launch_decode_t<FMT, DT, 3>(dp, num_seqs, st);
    default: return launch_decode_t<FMT, DT, 4>(dp, num_seqs, st);
  }
}

}  // namespace qp

using namespace qp;

// Split-count heuristic: whole waves of 3 CTAs per SM, a fixed cost per CTA, at least 4 tiles per split.
extern "C" int qp_decode_num_splits(int num_seqs, int num_kv_heads, int max_seqlen_k, int sm_count) {
  if (sm_count <= 0) sm_count = device_sm_count();
  const int pairs = max(1, num_seqs * num_kv_heads);
  const int tiles = max(1, (max_seqlen_k + DEC_TILE - 1) / DEC_TILE);
  const int slots = 3 * sm_count;
  const int max_splits = max(1, min(1024, tiles / 4));
  int best = 1;
  double best_cost = 1e30;
  for (int s = 1; s <= max_splits; ++s) {
    const long ctas = static_cast<long>(pairs) * s;
    const long waves = (ctas + slots - 1) / slots;
    const double cost = waves * (static_cast<double>((tiles + s - 1) / s) + 6.0);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

// Workspace of qp_paged_decode: [part_o rows x head fp32][part_lse rows fp32, 256-aligned][prepared query rows
// tokens x q heads x Q_STRIDE bytes], rows = tokens x q heads x splits.
static int64_t decode_qrec_offset(int64_t num_q_tokens, int num_q_heads, int head_size, int num_splits) {
  const int64_t rows = num_q_tokens * num_q_heads * static_cast<int64_t>(num_splits);
  return rows * head_size * 4 + ((rows * 4 + 255) / 256) * 256;
}

extern "C" int64_t qp_decode_workspace_bytes(int64_t num_q_tokens, int num_q_heads, int head_size, int num_splits) {
  return decode_qrec_offset(num_q_tokens, num_q_heads, head_size, num_splits) +
         num_q_tokens * num_q_heads * static_cast<int64_t>(Q_STRIDE);
}

extern "C" int qp_paged_decode(int fmt, int dtype, const void* q, int64_t q_stride_token, int64_t q_stride_head,
                               void* out, int64_t out_stride_token, int64_t out_stride_head, int64_t num_q_tokens,
                               int num_seqs, const int32_t* cu_seqlens_q, const int32_t* seqused_k, int max_seqlen_q,
                               const int32_t* block_table, int64_t block_table_stride, const void* cache,
                               int block_size, int64_t block_stride, int64_t head_stride, int64_t slot_stride,
                               int64_t k_off, int64_t ks_off, int64_t v_off, int64_t vs_off, int num_q_heads,
                               int num_kv_heads, int head_size, float softmax_scale, const uint32_t* rht_sign_bits,
                               int q_rotated, int tokens_after_keys, int out_mode, float* lse_out, int num_splits,
                               void* workspace, int64_t workspace_bytes, void* stream) {
  if (fmt != FMT_INT4 && fmt != FMT_K8V4) return set_error(QP_ERR_UNSUPPORTED, "decode: format %d", fmt);
  if (dtype != DT_BF16 && dtype != DT_F16) return set_error(QP_ERR_UNSUPPORTED, "decode: dtype %d", dtype);
  if (head_size != DEC_HS) return set_error(QP_ERR_UNSUPPORTED, "decode: head size %d (this build: 256)", head_size);
  if (num_seqs < 0 || num_q_tokens < 0 || num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads)
    return set_error(QP_ERR_INVALID, "decode: bad sizes (seqs %d, tokens %lld, heads %d/%d)", num_seqs,
                     (long long)num_q_tokens, num_q_heads, num_kv_heads);
  if (num_seqs == 0 || num_q_tokens == 0) return QP_OK;
  if (num_seqs > 65535 || num_kv_heads > 65535) return set_error(QP_ERR_UNSUPPORTED, "decode: grid too large");
  const int group = num_q_heads / num_kv_heads;
  if (max_seqlen_q < 1 || max_seqlen_q * group > DEC_MAX_ROWS)
    return set_error(QP_ERR_UNSUPPORTED, "decode: %d query tokens x %d heads per KV head > %d rows", max_seqlen_q,
                     group, DEC_MAX_ROWS);
  if (out_mode < 0 || out_mode > 2) return set_error(QP_ERR_INVALID, "decode: out_mode %d", out_mode);
  if (tokens_after_keys < 0) return set_error(QP_ERR_INVALID, "decode: tokens_after_keys %d", tokens_after_keys);
  const int cell = fmt == FMT_INT4 ? DEC_HS + 8 : DEC_HS * 3 / 2 + 8;
  if (slot_stride != cell)
    return set_error(QP_ERR_LAYOUT, "decode: cells of a (block, head) must be contiguous (slot stride %lld, cell %d)",
                     (long long)slot_stride, cell);
  const int kb = fmt == FMT_INT4 ? DEC_HS / 2 : DEC_HS;
  if (k_off != 0 || ks_off != kb || v_off != kb + 4 || vs_off != kb + 4 + DEC_HS / 2)
    return set_error(QP_ERR_LAYOUT, "decode: unexpected cell field offsets");
  if (block_size <= 0 || block_size % 16 || (reinterpret_cast<uintptr_t>(cache) & 15) || (block_stride & 15) ||
      (head_stride & 15))
    return set_error(QP_ERR_LAYOUT, "decode: block size must be a multiple of 16 and the cache 16-byte aligned");
  if (num_splits <= 0) return set_error(QP_ERR_INVALID, "decode: num_splits %d", num_splits);
  if (num_splits > 1024) return set_error(QP_ERR_UNSUPPORTED, "decode: num_splits %d > 1024", num_splits);
  if (!q || !out || !cu_seqlens_q || !seqused_k || !block_table || !cache || !rht_sign_bits || !workspace)
    return set_error(QP_ERR_INVALID, "decode: null pointer");
  if ((reinterpret_cast<uintptr_t>(workspace) & 15) ||
      workspace_bytes < qp_decode_workspace_bytes(num_q_tokens, num_q_heads, head_size, num_splits))
    return set_error(QP_ERR_WORKSPACE, "decode: workspace of %lld bytes < %lld", (long long)workspace_bytes,
                     (long long)qp_decode_workspace_bytes(num_q_tokens, num_q_heads, head_size, num_splits));

  DecodeParams dp{};
  dp.q = q;
  dp.q_st = q_stride_token;
  dp.q_sh = q_stride_head;
  dp.cu_seqlens_q = cu_seqlens_q;
  dp.seqused_k = seqused_k;
  dp.block_table = block_table;
  dp.bt_stride = block_table_stride;
  dp.cache = static_cast<const uint8_t*>(cache);
  dp.block_size = block_size;
  dp.block_stride = block_stride;
  dp.head_stride = head_stride;
  dp.ks_off = static_cast<int>(ks_off);
  dp.v_off = static_cast<int>(v_off);
  dp.vs_off = static_cast<int>(vs_off);
  dp.nq = num_q_heads;
  dp.nkv = num_kv_heads;
  dp.group = group;
  dp.qk_scale = softmax_scale / static_cast<float>(head_size) * LOG2E;
  dp.sign_bits = rht_sign_bits;
  dp.q_rotated = q_rotated;
  dp.qrec = static_cast<const uint8_t*>(workspace) +
            decode_qrec_offset(num_q_tokens, num_q_heads, head_size, num_splits);
  dp.num_tokens = num_q_tokens;
  dp.tokens_after = tokens_after_keys < max_seqlen_q ? tokens_after_keys : max_seqlen_q;  // >= qlen - 1: no mask
  dp.num_splits = num_splits;
  const int64_t rows = num_q_tokens * num_q_heads * static_cast<int64_t>(num_splits);
  dp.part_o = static_cast<float*>(workspace);
  dp.part_lse = dp.part_o + rows * head_size;

  const int nt = (max_seqlen_q * group + 7) / 8;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  {
    uint8_t* qrec = const_cast<uint8_t*>(dp.qrec);
    const int64_t qrows = num_q_tokens * num_q_heads;
    if ((qrows + 7) / 8 > 0x7fffffff) return set_error(QP_ERR_UNSUPPORTED, "decode: too many query rows");
    const unsigned qgrid = static_cast<unsigned>((qrows + 7) / 8);
#define QP_DQPREP(F, D)                                                                                      \
  decode_qprep_kernel<F, D><<<qgrid, 256, 0, st>>>(q, q_stride_token, q_stride_head, num_q_tokens, num_q_heads, \
                                                   num_kv_heads, rht_sign_bits, q_rotated, dp.qk_scale, qrec)
    if (fmt == FMT_INT4) {
      if (dtype == DT_BF16) QP_DQPREP(FMT_INT4, DT_BF16); else QP_DQPREP(FMT_INT4, DT_F16);
    } else {
      if (dtype == DT_BF16) QP_DQPREP(FMT_K8V4, DT_BF16); else QP_DQPREP(FMT_K8V4, DT_F16);
    }
#undef QP_DQPREP
    const int rc0 = check_launch("decode q prep");
    if (rc0) return rc0;
  }
  int rc;
  if (fmt == FMT_INT4)
    rc = dtype == DT_BF16 ? launch_decode_nt<FMT_INT4, DT_BF16>(dp, nt, num_seqs, st)
                          : launch_decode_nt<FMT_INT4, DT_F16>(dp, nt, num_seqs, st);
  else
    rc = dtype == DT_BF16 ? launch_decode_nt<FMT_K8V4, DT_BF16>(dp, nt, num_seqs, st)
                          : launch_decode_nt<FMT_K8V4, DT_F16>(dp, nt, num_seqs, st);
  if (rc) return rc;
  if (out_mode == 2) return QP_OK;  // split partials stay in the workspace

  MergeParams mp{};
  mp.part_o = dp.part_o;
  mp.part_lse = dp.part_lse;
  mp.po_t = static_cast<int64_t>(num_q_heads) * num_splits * head_size;
  mp.po_h = static_cast<int64_t>(num_splits) * head_size;
  mp.po_s = head_size;
  mp.pl_t = static_cast<int64_t>(num_q_heads) * num_splits;
  mp.pl_h = num_splits;
  mp.pl_s = 1;
  mp.num_splits = num_splits;
  mp.nq = num_q_heads;
  mp.mode = out_mode;
  mp.out = out;
  mp.out_st = out_stride_token;
  mp.out_sh = out_stride_head;
  mp.lse_out = lse_out;
  mp.lo_t = num_q_heads;
  mp.lo_h = 1;
  mp.sign_bits = rht_sign_bits;
  mp.out_scale = 1.f / static_cast<float>(head_size);
  return merge_dispatch(mp, dtype, head_size, num_q_tokens, st, true);
}

extern "C" int qp_merge_attn_partials(int dtype, int head_size, int64_t num_tokens, int num_q_heads, int num_parts,
                                      const float* part_o, int64_t po_stride_token, int64_t po_stride_head,
                                      int64_t po_stride_part, const float* part_lse, int64_t pl_stride_token,
                                      int64_t pl_stride_head, int64_t pl_stride_part, int out_mode, void* out,
                                      int64_t out_stride_token, int64_t out_stride_head, float* lse_out,
                                      const uint32_t* rht_sign_bits, void* stream) {
  if (num_tokens < 0 || num_q_heads <= 0 || num_parts <= 0) return set_error(QP_ERR_INVALID, "merge: bad sizes");
  if (num_tokens == 0) return QP_OK;
  if (out_mode != 0 && out_mode != 1) return set_error(QP_ERR_INVALID, "merge: out_mode %d", out_mode);
  if (out_mode == 0 && dtype != DT_BF16 && dtype != DT_F16)
    return set_error(QP_ERR_UNSUPPORTED, "merge: dtype %d", dtype);
  if (!part_o || !part_lse || !out || (out_mode == 0 && !rht_sign_bits))
    return set_error(QP_ERR_INVALID, "merge: null pointer");
  if (((po_stride_token | po_stride_head | po_stride_part) & 3) || (reinterpret_cast<uintptr_t>(part_o) & 15))
    return set_error(QP_ERR_LAYOUT, "merge: partial rows must be 16-byte aligned");
  MergeParams mp{};
  mp.part_o = part_o;
  mp.part_lse = part_lse;
  mp.po_t = po_stride_token;
  mp.po_h = po_stride_head;
  mp.po_s = po_stride_part;
  mp.pl_t = pl_stride_token;
  mp.pl_h = pl_stride_head;
  mp.pl_s = pl_stride_part;
  mp.num_splits = num_parts;
  mp.nq = num_q_heads;
  mp.mode = out_mode;
  mp.out = out;
  mp.out_st = out_stride_token;
  mp.out_sh = out_stride_head;
  mp.lse_out = lse_out;
  mp.lo_t = num_q_heads;
  mp.lo_h = 1;
  mp.sign_bits = rht_sign_bits;
  mp.out_scale = 1.f / static_cast<float>(head_size);
  return merge_dispatch(mp, out_mode == 1 ? DT_BF16 : dtype, head_size, num_tokens, static_cast<cudaStream_t>(stream),
                        false);
}

// ---------------------------------------------------------------------------------------------------------------
// Split-KV decode for callers that cannot allocate device memory.
//
// Some hosts of this library never call cudaMalloc once they are running: an engine that hands all device memory to
// its own pool at start-up and forbids allocations afterwards, or embedded C code with no device allocator at all.
// qp_paged_decode needs a workspace for its split partials; this variant takes it from a fixed array that lives in
// the library itself (QP_STATIC_DECODE_SCRATCH_BYTES, 32 MiB), so the call allocates nothing.
// - The array is reserved on every GPU that loads this library, for as long as the process lives.
// - Its device address is looked up (cudaGetSymbolAddress) on the first call on each device, with that device
//   current; make that first call before any stream capture.
// - Every call on a device uses the same array and it keeps the last call's contents. Nothing in it has to start at
//   zero (each call writes every partial it later reads), but calls that overlap on the GPU (two streams, two host
//   threads) race on it: serialize them.
// - Sizes whose partials exceed the array are rejected with QP_ERR_WORKSPACE.
static constexpr int64_t kStaticDecodeScratchBytes = 32ll << 20;
static __device__ __align__(256) uint8_t g_static_decode_scratch[kStaticDecodeScratchBytes];
static void* g_static_decode_scratch_addr[64] = {};

extern "C" int qp_paged_decode_static(int fmt, int dtype, const void* q, int64_t q_stride_token,
                                      int64_t q_stride_head, void* out, int64_t out_stride_token,
                                      int64_t out_stride_head, int64_t num_q_tokens, int num_seqs,
                                      const int32_t* cu_seqlens_q, const int32_t* seqused_k, int max_seqlen_q,
                                      const int32_t* block_table, int64_t block_table_stride, const void* cache,
                                      int block_size, int64_t block_stride, int64_t head_stride, int64_t slot_stride,
                                      int64_t k_off, int64_t ks_off, int64_t v_off, int64_t vs_off, int num_q_heads,
                                      int num_kv_heads, int head_size, float softmax_scale,
                                      const uint32_t* rht_sign_bits, int q_rotated, int out_mode, float* lse_out,
                                      int num_splits, void* stream) {
  const int64_t need = qp_decode_workspace_bytes(num_q_tokens, num_q_heads, head_size, num_splits);
  if (need > kStaticDecodeScratchBytes)
    return set_error(QP_ERR_WORKSPACE,
                     "decode (static scratch): the split partials need %lld bytes, the library's static scratch "
                     "holds %lld; lower num_splits or the batch, or call qp_paged_decode with a workspace",
                     (long long)need, (long long)kStaticDecodeScratchBytes);
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(QP_ERR_CUDA, "decode (static scratch): cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_error(QP_ERR_UNSUPPORTED, "decode (static scratch): device %d >= 64", dev);
  if (g_static_decode_scratch_addr[dev] == nullptr) {
    void* addr = nullptr;
    e = cudaGetSymbolAddress(&addr, g_static_decode_scratch);
    if (e != cudaSuccess || addr == nullptr)
      return set_error(QP_ERR_CUDA, "decode (static scratch): cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_static_decode_scratch_addr[dev] = addr;
  }
  return qp_paged_decode(fmt, dtype, q, q_stride_token, q_stride_head, out, out_stride_token, out_stride_head,
                         num_q_tokens, num_seqs, cu_seqlens_q, seqused_k, max_seqlen_q, block_table,
                         block_table_stride, cache, block_size, block_stride, head_stride, slot_stride, k_off, ks_off,
                         v_off, vs_off, num_q_heads, num_kv_heads, head_size, softmax_scale, rht_sign_bits, q_rotated,
                         0, out_mode, lse_out, num_splits, g_static_decode_scratch_addr[dev], kStaticDecodeScratchBytes,
                         stream);
}
