// K1: split-KV paged decode over an int4_per_token_head / k8v4_per_token_head cache, up to 32 query rows
//     (qlen x query heads per KV head) per KV head, head size 256 or 512, on the 5th-generation tensor cores
//     (tcgen05 + TMEM); K0q: the query preparation it reads; K2: log-sum-exp merge of the segments with the inverse
//     RHT and the attention sinks fused in. At head 512 the same kernel also serves chunk prefill, as decodes of a
//     few query tokens each over the chunk's causal prefixes (qp_prefill), and at both head sizes the short chunks of
//     a step in one launch (qp_prefill_varlen). A second instantiation (FEAT) applies vLLM's sliding window and logit
//     softcap.
//
// Reference behaviour (what this computes, not how): the split-KV 3D path of vLLM's int4 kernel as the plugin
// configures it (vllm_quantpack/attention/int4_kv.py:98-122: every query token of a step in one program, segments
// sized to the SM count) and vLLM's reduce_segments (vllm/v1/attention/ops/triton_unified_attention.py:645-732 in
// vLLM 0.22). Scores S = (Q.u - Q_sum zp) k_scale scale, out = sum_t P_t v_scale_t (u_t - zp_t) / sum_t P_t
// (int4_kv.py:80-94; k8v4 keys: S = Q.k8 k_scale scale, int4_kv.py:127-146).
//
// B200 design. Decode has 24 query rows per KV head (4 tokens x 6 heads) against 128 keys per tile, so the MMAs
// are thin (N = 32). A thin MMA runs at the tensor pipe's full rate only when its wide operand comes from TMEM
// (measured on this part: M 128 x N 32 x K 16 in 16 cycles with A in TMEM, 40 with A in shared memory, whose
// bandwidth the A operand then saturates). So the keys are the M dimension and both cache operands live in TMEM:
//   S^T (128 keys x N rows)          = K_op (TMEM, 128 keys x HS channels)          x Q^T (shared memory, N x HS)
//   O^T (HS/128 x 128 channels x N)  = V^T_op (TMEM, HS/128 x 128 channels x keys)  x P^T (shared memory, N x keys)
// One CTA of 15 warps (19 at head 256 with up to 24 rows) per SM (it holds all 512 TMEM columns) per (split, KV
// head, sequence):
//   warp 0      producer: 1-D bulk copies (TMA engine, no tensor map, no multicast) of the tile's raw cells, whole
//               16-token groups, into a ring of raw stages (a stage holds the tile, or at head 512 half of it);
//   warps 1, 14 MMA issuers (convergent; elect.sync picks the lane), on different SM sub-partitions: warp 1 the
//               HS/16 QK MMAs of a tile into a double-buffered S, warp 14 the PV MMAs, each group finished with
//               tcgen05.commit onto mbarriers;
//   warps 2-5   key operand: thread = key = TMEM lane; one AND per channel pair makes the int4 codes fp16
//               subnormals (u x 2^-24, 16 u x 2^-24 for high nibbles, whose query channels K0q divides by 16); k8v4
//               codes become c + 128 the same way (one XOR per word, one prmt per pair). The zero point (int4) or the
//               bias 128 (k8v4) comes off in the MMA: one more MMA of K 16 per tile, A = -zp x 2^-14 from shared
//               memory, B = the query row's sum split into three fp16 terms. The operand is
//               written in 256-channel chunks (128 TMEM columns) into a ring of two chunk slots (one at head 512
//               with 32 rows, where TMEM has no room for two), so the conversion of one chunk overlaps the MMAs of
//               the other. The key / value scales go to shared memory for the softmax, the value zero points as
//               paired fp16 operand biases;
//   warps 6-9   value operand (and 15-18, a second set converting every other slot, at head 256 with <= 24 rows):
//               V^T written with tcgen05.st.16x256b, whose thread layout (lanes i/4 and 8 + i/4,
//               column pair 2(i%4)) puts one channel of four consecutive keys in each thread: one 32-bit word of
//               each of four keys, interleaved by prmt, becomes the exact fp16 (u - zp) of every (channel, key).
//               The zero point sits in the operand, so the running O accumulator only holds the signal; two value
//               slots (64 keys at head 256; 32 at head 512, where O^T takes four channel tiles) let the conversion
//               of one slot overlap the MMAs of the other;
//   warps 10-13 softmax: thread = key; scores in log2 units from S^T, a lazy per-row maximum (P may reach 2^8
//               before O is rescaled, which happens in TMEM and rarely), P x value scale in fp16 with a running
//               power-of-two range written as P^T, MN-major (a key's rows contiguous: 8 rows per 16-byte store);
//               per-thread row sums reduced once at the end; the epilogue reads O^T and writes the normalised
//               partial and its log2-sum-exp.
// Every wait is bounded (a timeout records an error word and the roles leave; the softmax warps leave together).
#include <math.h>

#include <algorithm>
#include <atomic>
#include <type_traits>

#include "qp_api_internal.h"
#include "qp_common.cuh"
#include "qp_tcgen05.cuh"

namespace qp {

constexpr int DEC_TILE = 128;  // keys per tile (TMEM lanes of the QK accumulator)
constexpr int P_KGROUP = 128;                    // bytes between the 8-key groups of P^T (LBO of its descriptor)
constexpr int P_NGROUP = DEC_TILE / 8 * P_KGROUP;  // bytes between its 8-row groups (SBO)
constexpr int DEC_MAX_ROWS = 32;
#ifndef QP_DEC_SMX_HALVES
#define QP_DEC_SMX_HALVES 1
#endif
constexpr int SMX_HALVES = QP_DEC_SMX_HALVES;  // softmax warps per TMEM lane quarter (each takes RL / halves rows)
static_assert(SMX_HALVES == 1 || SMX_HALVES == 2, "one or two softmax warps per lane quarter");

// warp 0 producer, 1 QK issuer, 2-5 key operand, 6-9 value operand, 10.. softmax (SMX_HALVES per lane quarter), then
// the PV issuer and, at head 256 with up to 24 rows, a second set of four value-operand warps (W_VB..). The two MMA
// issuers sit on different SM sub-partitions: issuing a tcgen05.mma takes that sub-partition's issue slots from the
// operand warps beside it, and with all 32 MMAs of a tile on one sub-partition its value warp fell 1,500 cycles
// behind the other three every tile (clock64 stamps per role). The value conversion sets the tile period, so where
// the registers allow (96 a thread; the softmax of 32 rows would spill) two warps per lane quarter share it, each set
// converting one of the tile's two value slots (c2a, same box: 99.1 -> 90.3 us; splitting every slot between the
// sets instead measured 91.1, with twice the slot hand-offs per warp).
constexpr int W_MMA = 1, W_VAL = 6, W_SMX = 10, W_PV = W_SMX + 4 * SMX_HALVES, W_VB = W_PV + 1;
constexpr int SMX_THREADS = 32 * 4 * SMX_HALVES;

template <int HS, int RL>
struct DecWarps {
  static constexpr int VSETS = (HS == 256 && RL <= 24) ? 2 : 1;  // value-operand warp sets
  static constexpr int WARPS = W_VB + 4 * (VSETS - 1);
  static constexpr int THREADS = 32 * WARPS;
  // registers per thread one CTA may hold: each SM sub-partition's 16384 registers host every fourth warp
  static constexpr int REGS = (16384 / (32 * ((WARPS + 3) / 4))) & ~7;
};
// prepared query row: HS fp16 in operand order, then 4 fp32 (row scale, three zero words)
constexpr int q_rec_bytes(int hs) { return hs * 2 + 16; }
constexpr float LOG2E = 1.4426950408889634f;
constexpr float RESCALE_SLACK = 8.f;
constexpr int BAR_SMX = 1;  // named barrier of the softmax warps

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
  int nq, nkv, group;  // query heads, KV heads, query heads per KV head
  float qk_scale;      // softmax_scale / head_size * log2(e)
  const uint32_t* sign_bits;
  int q_rotated;        // q already in the RHT domain
  const uint8_t* qrec;  // prepared query rows: [kv head][token][query head of the group] x q_rec_bytes(HS)
  int64_t num_tokens;
  int tokens_after;  // sequence tokens after this call's keys (held by other ranks), clamped to the query tokens
  // chunk_q > 0: the num_tokens query tokens are ONE sequence's chunk (its last positions, causal among themselves)
  // over chunk_n cached keys through block-table row 0, served as sub-sequences of chunk_q tokens (grid z), each
  // reading only the keys its last token sees. cu_seqlens_q / seqused_k are not read.
  int chunk_q, chunk_n;
  // subseq != null: sequence z of the grid is subseq[z] = {first query token, query tokens, keys its last token
  // sees, block-table row}, causal inside it (built on the device by varlen_table_kernel; entries past the real ones
  // hold 0 query tokens). cu_seqlens_q / seqused_k are not read.
  const int4* subseq;
  // window > 0: vLLM's SLIDING_WINDOW (1 + window_size[0]): a query token whose last visible key is p sees the keys
  // [p - window + 1, p] only (vllm/v1/attention/ops/triton_attention_helpers.py:196-218, vLLM 0.22)
  int window;
  // softcap > 0: every score S (natural units) becomes softcap x tanh(S / softcap) before the softmax, vLLM's
  // apply_softcap (vllm/v1/attention/ops/triton_attention_helpers.py:28-36, triton_unified_attention.py:513-514)
  float softcap;
  int num_splits;
  float* part_o;    // [tokens][nq][splits][HS]
  float* part_lse;  // [tokens][nq][splits], log2 units
};

template <int FMT, int HS>
struct Cell {
  static constexpr int KB = FMT == FMT_INT4 ? HS / 2 : HS;  // key bytes
  static constexpr int BYTES = KB + 8 + HS / 2;
  static constexpr int KS = KB, V = KB + 4, VS = KB + 4 + HS / 2;  // field offsets
};

// TMEM columns (512) of the head size's operands and accumulators.
//   HS 256: key operand chunks at [0, 128) and [384, 512); two 64-key value slots (two channel tiles of 32 columns)
//           at [128, 256); S (2 x NR) and O^T (2 channel tiles x NR) from 256.
//   HS 512: key operand chunks (channels 0-255, then 256-511 of a tile) in AKS slots of 128 columns from 0; two
//           32-key value slots (four channel tiles of 16 columns) after them; S and O^T (4 channel tiles x NR) last.
//           At NR 32 only one key slot fits (448 columns; the key conversion of a chunk then waits for the previous
//           chunk's QK MMAs). Two key slots would leave room for 16-key value slots only: the value warps then release
//           a raw stage only once the PV MMAs of its tile have started, after the next tile's QK, which needs two fresh
//           raw stages first, so the three-stage k8v4 ring would deadlock; with int4's four stages that plan runs,
//           but measured slower (262k-token decode 0.214 against 0.193 ms, 1024-query prefill 30.1 against 25.1 ms).
template <int HS, int NR>
struct DecTmem {
  static constexpr int NCH = HS / 256;                         // key operand chunks per tile
  static constexpr int MT = HS / 128;                          // channel tiles of V^T and O^T
  static constexpr int AKS = (HS == 256 || NR <= 16) ? 2 : 1;  // key operand chunk slots
  static constexpr int VK = HS == 256 ? 64 : 32;               // keys per value slot
  static constexpr int VSLOTS = DEC_TILE / VK;                 // value slots per tile
  static constexpr int SLOT = MT * VK / 2;                     // TMEM columns of a value slot
  static constexpr uint32_t AK0 = 0, AK1 = HS == 256 ? 384 : 128;
  static constexpr uint32_t AV = HS == 256 ? 128 : 128 * AKS;
  static constexpr uint32_t S = AV + 2 * SLOT;
  static constexpr uint32_t O = S + 2 * NR;  // channel tile t at O + NR t
  static_assert(HS == 256 || HS == 512, "head size 256 or 512");
  static_assert(O + MT * NR <= (HS == 256 ? AK1 : 512u), "TMEM columns overlap");
  static_assert(VK % 16 == 0 && DEC_TILE % VK == 0, "value slots of whole 16-key blocks");
};

template <int FMT, int HS, int NR>
struct DecSmem {
  static constexpr int CELL = Cell<FMT, HS>::BYTES;
  static constexpr int SK = HS == 256 ? DEC_TILE : DEC_TILE / 2;  // keys per raw stage
  static constexpr int SPT = DEC_TILE / SK;                        // raw stages per tile
  static constexpr int RS = FMT == FMT_INT4 ? 4 : 3;               // raw stages
  static constexpr int KPS = HS == 256 ? RS : 3;                   // tiles of key / value scales in flight
  static constexpr int RAW = SK * CELL;
  static constexpr int ATOM = NR * 128;  // one 64-element column of 128B-swizzle atoms over the NR rows
  // Q: HS / 64 atoms, K-major; then one more atom whose first 16 k hold the zero-point correction terms (K0q)
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_QZ = OFF_Q + HS / 64 * ATOM;
  static constexpr int OFF_P = OFF_QZ + ATOM;              // P^T: 2 buffers x 2 ATOM (128 keys), MN-major (p_off)
  static constexpr int OFF_RAW = OFF_P + 4 * ATOM;         // RS raw stages
  // P^T (the B operand of the PV MMAs) is MN-major without swizzle: core matrices of 8 keys x 8 rows, 128 bytes
  // (key k at 16 k, row r at 2 r), the 16 key groups of a tile P_KGROUP apart, the row groups P_NGROUP apart; byte
  // offset of (buffer b, row, key) from OFF_P
  static __device__ __forceinline__ int p_off(int b, int row, int key) {
    return b * 2 * ATOM + (row >> 3) * P_NGROUP + (key >> 3) * P_KGROUP + (key & 7) * 16 + (row & 7) * 2;
  }
  static constexpr int OFF_KP = OFF_RAW + RS * RAW;        // [KPS][128] float4: key scale, key zp, value scale
  static constexpr int OFF_ZB = OFF_KP + KPS * 128 * 16;   // [KPS][128] u32: paired value zero-point operand biases
  static constexpr int OFF_RP = OFF_ZB + KPS * 128 * 4;    // [2][NR] float2: row scale, row maximum
  static constexpr int OFF_LIM = OFF_RP + 2 * NR * 8;      // [NR] int: last key the row sees
  static constexpr int OFF_WLO = OFF_LIM + NR * 4;         // [NR] int: first key the row sees (sliding window), or -1
  // [8] value-scale maxima, [NR] O factors, [NR] float2 (row-sum factor, exp-argument shift)
  static constexpr int OFF_RED = OFF_WLO + NR * 4;
  static constexpr int OFF_SB = (OFF_RED + (8 + NR + 2 * NR) * 4 + 15) / 16 * 16;  // [NR][128] f32 scores
  // the A operand of the zero-point correction MMA: 128 keys x 16 k fp16, K-major without swizzle (the 8-key groups
  // AZ_MGROUP apart, the two 8-k halves AZ_KHALF apart), one buffer per key-operand slot (int4: the key's zero point
  // changes every tile) or one constant buffer (k8v4)
  static constexpr int AZ_MGROUP = 128, AZ_KHALF = 2048, AZ_BYTES = 4096;
  static constexpr int AZB = FMT == FMT_INT4 ? 2 : 1;
  static constexpr int OFF_AZ = (OFF_SB + NR * 128 * 4 + 127) / 128 * 128;
  static constexpr int OFF_BAR = OFF_AZ + AZB * AZ_BYTES;
  static constexpr int NBAR = 40;
  static constexpr int OFF_TMEM = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_TMEM + 16;
  static_assert(BYTES <= 232448, "dynamic shared memory above the 227 KB a CTA may hold");
  static_assert(RAW % 16 == 0 && OFF_RAW % 1024 == 0, "bulk copy destinations must be 16-byte aligned");
  static_assert(RS <= 4 && KPS <= 4, "barrier slots");
};

// barrier slots
enum {
  D_RAW_FULL = 0,    // [RS <= 4] a raw stage landed
  D_RAW_EMPTY = 4,   // [RS] the key warps of its keys and the value warps are done with it
  D_Q_FULL = 8,      // Q^T is in shared memory (every softmax warp)
  D_AK_FULL = 9,     // [2] key operand chunk in TMEM (4 key warps)
  D_AK_FREE = 11,    // [2] its QK MMAs completed (commit)
  D_KP_FULL = 13,    // [KPS <= 4] the tile's scales and zero-point biases are in shared memory (4 key warps)
  D_KP_FREE = 17,    // [KPS] the softmax and the value warps read them
  D_AV_FULL = 21,    // [2] value operand slot in TMEM (4 value warps)
  D_AV_FREE = 23,    // [2] its PV MMAs completed (commit)
  D_S_FULL = 25,     // [2] S^T of the tile is in TMEM (commit)
  D_S_FREE = 27,     // [2] the softmax read it (every softmax warp)
  D_P_FULL = 29,     // [2] P^T of the tile is in shared memory (every softmax warp)
  D_PV_DONE = 31,    // [2] PV(j) completed: barrier j & 1, one phase per two tiles (commit)
  D_FINAL = 33,      // every MMA issued has completed (before TMEM is released)
};

// fp16 pair -> exact (nibble - zero point) of two keys a, b: the low-nibble form (1024 + u) minus (1024 + zp), the
// high-nibble form (1024 + 16 u) / 16 - (64 + zp).
__device__ __forceinline__ uint32_t nib_lo(uint32_t x, uint32_t lo_bias) {
  return hsub2_u32(lop3_and_or(x, 0x000F000Fu, 0x64006400u), lo_bias);
}
__device__ __forceinline__ uint32_t nib_hi(uint32_t x, uint32_t hi_bias) {
  return hfma2_u32(lop3_and_or(x, 0x00F000F0u, 0x64006400u), 0x2C002C00u /* 1/16 */, hi_bias);
}

// Key operand codes as fp16 subnormals (bits = value x 2^24), one AND per pair of channels: int4 low nibbles give
// u x 2^-24, high nibbles 16 u x 2^-24 (K0q divides the query's high-nibble channels by 16, exactly); k8v4 codes c
// biased to c + 128 by one XOR, two bytes per prmt. The MMA then sums exact products u q 2^-24 (tcgen05 kind::f16
// takes subnormal inputs), and the zero point (int4: per key; k8v4: the bias 128) comes off through one more MMA of
// K 16 per tile: A = -zp x 2^-14 in three k, B = the query row's sum of its effective channels x 2^-10 split into
// three fp16 terms (K0q), so that A B = -zp 2^-24 sum(q).
constexpr uint32_t KEY_SUB_LO = 0x000F000Fu, KEY_SUB_HI = 0x00F000F0u;

template <int NR>
__device__ __forceinline__ void tmem_ld_rows(uint32_t taddr, float (&v)[NR]) {
  tmem_ld_cols<NR>(taddr, v);
}
template <int NR>
__device__ __forceinline__ void tmem_st_rows(uint32_t taddr, const float (&v)[NR]) {
  if constexpr (NR == 32) tmem_st32(taddr, v);
  else tmem_st16(taddr, v);
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// capl x tanh(t / capl) for a score t in log2 units (capl = softcap x log2 e, cap_k = 2 log2 e / capl), from
// tanh(y) = 1 - 2 / (e^{2y} + 1) taken on |y| and given t's sign: absolute error ~1e-7 x capl, which is what a softmax
// argument needs (no cancellation matters once it is multiplied back by capl); e^{2|y|} = 2^{|t| cap_k}, its exponent
// held below 64 so the quotient stays finite.
__device__ __forceinline__ float softcap_log2(float t, float capl, float cap_k) {
  const float a = fast_exp2(fminf(fabsf(t) * cap_k, 64.f));
  return copysignf(capl * (1.f - __fdividef(2.f, a + 1.f)), t);
}

// k index (0..HS-1) of the QK operand that carries channel c. int4: column j = 4 w + m of a key's TMEM lane holds
// the pair lop3'd from word w (shifted right 8 for m >= 2; low nibbles for even m, high for odd), i.e. channels
// 8 w + m (low half) and 8 w + m + 4 (high half); k8v4: the natural order (prmt takes bytes 0, 1 then 2, 3).
template <int FMT>
__host__ __device__ __forceinline__ int qk_k_of_channel(int c) {
  if constexpr (FMT == FMT_INT4) return 8 * (c >> 3) + 2 * (c & 3) + ((c >> 2) & 1);
  else return c;
}

// ---------------------------------------------------------------------------------------------------- K0q
// One warp per (query token, query head): the row as K1 reads it (q_rec_bytes(HS)): HS fp16 in the k order of the
// QK operand, scaled by a power of two (|q| < 2^14; int4: the high-nibble channels by a further 2^-4); then the
// fp32 row scale A (softmax_scale / head x log2 e x 2^(24 - exponent)), the three fp16 terms of the zero-point
// correction (the row's sum x 2^-10) and zeros. Written once per call; every split of the row's KV head reads it.
template <int FMT, int DT, int HS>
__global__ void __launch_bounds__(256) decode_qprep_kernel(const void* q, int64_t q_st, int64_t q_sh, int64_t T,
                                                           int nq, int nkv, const uint32_t* sign_bits, int q_rotated,
                                                           float qk_scale, uint8_t* qrec) {
  asm volatile("griddepcontrol.launch_dependents;");
  using EL = Elem<DT>;
  constexpr int E = HS / 32;  // elements per lane
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= T * nq) return;
  const int64_t tok = row / nq;
  const int qh = static_cast<int>(row % nq);
  const int group = nq / nkv, kvh = qh / group, hg = qh % group;
  uint8_t* rec = qrec + ((static_cast<int64_t>(kvh) * T + tok) * group + hg) * q_rec_bytes(HS);
  __half* qrow = reinterpret_cast<__half*>(rec);
  const typename EL::T* src = reinterpret_cast<const typename EL::T*>(q) + tok * q_st + qh * q_sh + lane * E;
  float x[E];
#pragma unroll
  for (int i = 0; i < E; ++i) x[i] = EL::to_f(src[i]);
  if (!q_rotated) {
    apply_signs<E>(x, sign_bits, lane);
    warp_wht<E>(x, lane);
  }
  float am = 0.f;
#pragma unroll
  for (int i = 0; i < E; ++i) am = fmaxf(am, fabsf(x[i]));
  am = warp_max(am);
  int ex = 0;
  if (am > 0.f) {
    frexpf(am, &ex);  // am < 2^ex
    ex = 14 - ex;     // am * 2^ex in [2^13, 2^14)
  }
  // int4: the high-nibble (odd) channels meet operand codes 16 u x 2^-24, so they carry q / 16 (a power of two:
  // exact); ysum: the row's sum of the channel values the MMA effectively multiplies by u x 2^-24
  float ysum = 0.f;
#pragma unroll
  for (int i = 0; i < E; ++i) {
    const int c = lane * E + i;
    const bool hi = FMT == FMT_INT4 && (c & 1);
    const __half h = __float2half_rn(ldexpf(x[i], hi ? ex - 4 : ex));
    qrow[qk_k_of_channel<FMT>(c)] = h;
    ysum += hi ? 16.f * __half2float(h) : __half2float(h);
  }
  ysum = warp_sum(ysum);
  if (lane == 0) {
    float* rc = reinterpret_cast<float*>(rec + 2 * HS);
    rc[0] = ldexpf(qk_scale, 24 - ex);  // the MMA's scores carry 2^-24
    // ysum x 2^-10 (|.| < 2^12) as three fp16 terms, each the rounding of what the terms before it left
    const float y = ldexpf(ysum, -10);
    const __half h1 = __float2half_rn(y);
    const float r1 = y - __half2float(h1);
    const __half h2 = __float2half_rn(r1);
    const __half h3 = __float2half_rn(r1 - __half2float(h2));
    uint32_t* rz = reinterpret_cast<uint32_t*>(rc + 1);
    rz[0] = static_cast<uint32_t>(__half_as_ushort(h1)) | (static_cast<uint32_t>(__half_as_ushort(h2)) << 16);
    rz[1] = __half_as_ushort(h3);
    rz[2] = 0u;
  }
}

// ---------------------------------------------------------------------------------------------------- K1
// FEAT: the launch applies a sliding window (p.window > 0) and / or a logit softcap (p.softcap > 0); the
// instantiations without FEAT carry none of their code
template <int FMT, int DT, int HS, int NR, int RL, bool FEAT>
__global__ void __maxnreg__((DecWarps<HS, RL>::REGS)) decode_kernel(const DecodeParams p) {
  using SM = DecSmem<FMT, HS, NR>;
  using CL = Cell<FMT, HS>;
  using TM = DecTmem<HS, NR>;
  static_assert(TM::VK >= 32 || DecSmem<FMT, HS, NR>::RS >= 4, "16-key value slots need a four-stage raw ring");
  constexpr int CELL = SM::CELL, RS = SM::RS, KPS = SM::KPS, SK = SM::SK, SPT = SM::SPT;
  constexpr int NCH = TM::NCH, MT = TM::MT, VK = TM::VK, VSLOTS = TM::VSLOTS, AKS = TM::AKS;
  constexpr int QREC = q_rec_bytes(HS);
  constexpr int VSETS = DecWarps<HS, RL>::VSETS, THREADS = DecWarps<HS, RL>::THREADS;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + SM::OFF_TMEM);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;

  // Let the merge kernel (launched with programmatic stream serialization) start its launch now; it waits for this
  // grid's completion before reading anything.
  asm volatile("griddepcontrol.launch_dependents;");

  // the sequence's query tokens [q0, q0 + qlen), its keys [0, n), the last key its first token sees (before clamping
  // to n - 1) and its block-table row
  int q0, qlen, n, vis_base;
  const int32_t* btab;
  if (p.subseq != nullptr) {
    const int4 e = p.subseq[seq];
    q0 = e.x;
    qlen = e.y;
    n = e.z;
    vis_base = n - qlen;
    btab = p.block_table + static_cast<int64_t>(e.w) * p.bt_stride;
  } else if (p.chunk_q > 0) {
    q0 = seq * p.chunk_q;
    qlen = min(p.chunk_q, static_cast<int>(p.num_tokens) - q0);
    vis_base = p.chunk_n - static_cast<int>(p.num_tokens) + q0 + p.tokens_after;
    n = min(p.chunk_n, vis_base + qlen);
    btab = p.block_table;
  } else {
    q0 = p.cu_seqlens_q[seq];
    qlen = p.cu_seqlens_q[seq + 1] - q0;
    n = p.seqused_k[seq];
    vis_base = n - qlen + p.tokens_after;
    btab = p.block_table + static_cast<int64_t>(seq) * p.bt_stride;
  }
  const int rows = qlen * p.group;
  if (qlen <= 0) return;
  // with a sliding window the splits share the tiles from the one holding the first token's first key: the later
  // tokens' windows start at most qlen - 1 <= 31 keys further on, so inside the first two tiles of that range
  const int win_lo = (FEAT && p.window > 0) ? max(0, vis_base - p.window + 1) : 0;
  const int tile_lo = win_lo / DEC_TILE;
  const int n_tiles = (n + DEC_TILE - 1) / DEC_TILE;
  const int tps = max(0, (n_tiles - tile_lo + p.num_splits - 1) / p.num_splits);
  const int tile0 = tile_lo + split * tps;
  const int ntl = max(0, min(tile0 + tps, n_tiles) - tile0);
  if (ntl == 0) {  // empty segment: lse = -inf
    for (int r = tid; r < rows; r += THREADS) {
      const int tok = q0 + r / p.group, qh = kvh * p.group + r % p.group;
      p.part_lse[(static_cast<int64_t>(tok) * p.nq + qh) * p.num_splits + split] = -INFINITY;
    }
    return;
  }

  if (tid == 0) {
    for (int s = 0; s < RS; ++s) {
      mbar_init(&bars[D_RAW_FULL + s], 1);
      mbar_init(&bars[D_RAW_EMPTY + s], 4 / SPT + 4 * VSETS);  // the key warps of the stage's keys, every value warp
    }
    for (int s = 0; s < KPS; ++s) {
      mbar_init(&bars[D_KP_FULL + s], 4);
      mbar_init(&bars[D_KP_FREE + s], 4 * VSETS + 4 * SMX_HALVES);
    }
    mbar_init(&bars[D_Q_FULL], 4 * SMX_HALVES);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars[D_AK_FULL + b], 4);
      mbar_init(&bars[D_AK_FREE + b], 1);
      mbar_init(&bars[D_AV_FULL + b], 4);
      mbar_init(&bars[D_AV_FREE + b], 1);
      mbar_init(&bars[D_S_FULL + b], 1);
      mbar_init(&bars[D_S_FREE + b], 4 * SMX_HALVES);
      mbar_init(&bars[D_P_FULL + b], 4 * SMX_HALVES);
    }
    mbar_init(&bars[D_PV_DONE], 1);
    mbar_init(&bars[D_PV_DONE + 1], 1);
    mbar_init(&bars[D_FINAL], 2);  // one commit per MMA issuer
    fence_mbar_init();
  }
  if (warp == W_MMA) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool failed = false;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    // Fill u of the ring holds keys [(u % SPT) SK, + SK) of tile u / SPT. Lane j copies 16-token group j of it
    // (block_size % 16 == 0, so a group never crosses a block); its block-table entry is loaded one fill ahead, so
    // the lookups of a fill are in flight together. A fill past the context lands at once (no bytes expected).
    const uint8_t* head_base = p.cache + static_cast<int64_t>(kvh) * p.head_stride;
    const int nu = ntl * SPT;
    auto first_key = [&](int u) { return (tile0 + u / SPT) * DEC_TILE + (u % SPT) * SK; };
    auto block_of = [&](int u) {
      const int tok = first_key(u) + 16 * lane;
      return (lane < SK / 16 && u < nu && tok < n) ? __ldg(btab + tok / p.block_size) : -1;
    };
    int next_blk = block_of(0);
    int u = 0;
    for (; u < nu; ++u) {
      const int stage = u % RS;
      if (u >= RS && __any_sync(0xffffffffu, !mbar_wait_bounded(&bars[D_RAW_EMPTY + stage], ((u / RS) - 1) & 1)))
        break;
      const int blk = next_blk;
      next_blk = block_of(u + 1);
      const int tb = first_key(u);
      const int groups = max(0, (min(tb + SK, n) - tb + 15) >> 4);
      if (lane == 0) mbar_arrive_expect_tx(&bars[D_RAW_FULL + stage], static_cast<uint32_t>(groups * 16 * CELL));
      __syncwarp();
      if (lane < groups) {
        const int tok = tb + 16 * lane;
        const int in_blk = tok - (tok / p.block_size) * p.block_size;
        bulk_g2s(smem + SM::OFF_RAW + stage * SM::RAW + lane * 16 * CELL,
                 head_base + static_cast<int64_t>(blk) * p.block_stride + static_cast<int64_t>(in_blk) * CELL,
                 static_cast<uint32_t>(16 * CELL), &bars[D_RAW_FULL + stage]);
      }
    }
    // the copies in flight land before the CTA's shared memory can go away
    if (lane == 0)
      for (int k = max(0, u - RS); k < u; ++k)
        mbar_wait_bounded(&bars[D_RAW_FULL + k % RS], (k / RS) & 1, 100000000ull);
  } else if (warp == W_MMA || warp == W_PV) {
    // ------------------------------------------------------------------ MMA issuers (QK, PV)
    // The whole warp waits (convergent, so descriptors and TMEM addresses are warp-uniform); one elected lane issues.
    constexpr uint32_t ID = f16_idesc(128, NR, false);      // QK: B = Q^T, K-major
    constexpr uint32_t ID_PV = f16_idesc(128, NR, true);    // PV: B = P^T, MN-major
    // Every B operand descriptor is the base descriptor of its buffer plus a compile-time start-address offset (the
    // 14-bit start field holds address / 16 and every shared-memory address here is below 256 KB, so the add
    // never carries out of it): one integer add per MMA.
    const uint64_t q_desc = sw128_desc(smem_u32(smem + SM::OFF_Q), 16, 1024);
    const uint64_t p_desc = interleave_desc(smem_u32(smem + SM::OFF_P), P_KGROUP, P_NGROUP);
    const uint64_t az_desc = interleave_desc(smem_u32(smem + SM::OFF_AZ), SM::AZ_KHALF, SM::AZ_MGROUP);
    const uint64_t qz_desc = sw128_desc(smem_u32(smem + SM::OFF_QZ), 16, 1024);
    auto wait_all = [&](uint64_t* bar, uint32_t parity) {
      const bool ok = mbar_wait_spin(bar, parity);
      failed |= __any_sync(0xffffffffu, !ok);
    };
    // O^T += V^T(j) P^T(j), slot by slot (the value warps refill a slot as soon as its MMAs complete)
    auto issue_pv = [&](int j) {
      const int bj = j & 1;
      wait_all(&bars[D_P_FULL + bj], (j >> 1) & 1);
      const uint64_t pd = p_desc + static_cast<uint64_t>(SM::p_off(bj, 0, 0) >> 4);
#pragma unroll
      for (int h = 0; h < VSLOTS; ++h) {  // slot h: keys [h VK, h VK + VK) of the tile, TMEM slot k & 1
        if (failed) break;
        const int k = j * VSLOTS + h, sl = k & 1;
        wait_all(&bars[D_AV_FULL + sl], (k >> 1) & 1);
        if (failed) break;
        tc_fence_after();
        if (elect_one()) {
#pragma unroll
          for (int c = 0; c < MT; ++c)
#pragma unroll
            for (int s = 0; s < VK / 16; ++s) {
              const int key = h * VK + 16 * s;
              umma_f16_ts(tmem + (TM::O + NR * c), tmem + (TM::AV + TM::SLOT * sl + (VK / 2) * c + 8 * s),
                          pd + static_cast<uint64_t>(SM::p_off(0, 0, key) >> 4), ID_PV,
                          (h | s) ? 1u : static_cast<uint32_t>(j));
            }
          umma_commit(&bars[D_AV_FREE + sl]);
        }
        __syncwarp();
      }
      if (elect_one()) umma_commit(&bars[D_PV_DONE + bj]);
      __syncwarp();
    };
    if (warp == W_PV) {
      for (int j = 0; j < ntl && !failed; ++j) issue_pv(j);
      if (elect_one()) umma_commit(&bars[D_FINAL]);
      __syncwarp();
    } else {
    wait_all(&bars[D_Q_FULL], 0);
    for (int i = 0; i < ntl && !failed; ++i) {
      const int b = i & 1;
      const uint32_t sd = tmem + TM::S + NR * b;
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) {  // key operand chunk ch: channels [256 ch, 256 ch + 256), slot k % AKS
        const int k = i * NCH + ch, sl = k % AKS;
        wait_all(&bars[D_AK_FULL + sl], (k / AKS) & 1);
        if (ch == 0 && i >= 2) wait_all(&bars[D_S_FREE + b], ((i - 2) >> 1) & 1);  // S buffer b read by the softmax
        if (failed) break;
        tc_fence_after();
        const uint32_t ak = tmem + (sl ? TM::AK1 : TM::AK0);
        if (elect_one()) {
#pragma unroll
          for (int s = 0; s < 16; ++s)
            umma_f16_ts(sd, ak + 8 * s,
                        q_desc + static_cast<uint64_t>(((4 * ch + (s >> 2)) * SM::ATOM + (s & 3) * 32) >> 4), ID,
                        (ch | s) ? 1u : 0u);
          if (ch == 0)  // the zero-point correction: S^T += A_z (smem, this slot's buffer) x Q_z^T
            umma_f16(sd, az_desc + static_cast<uint64_t>(((sl % SM::AZB) * SM::AZ_BYTES) >> 4), qz_desc, ID, 1u);
          umma_commit(&bars[D_AK_FREE + sl]);
          if (ch == NCH - 1) umma_commit(&bars[D_S_FULL + b]);
        }
        __syncwarp();
      }
    }
    if (elect_one()) umma_commit(&bars[D_FINAL]);
    __syncwarp();
    mbar_wait_spin(&bars[D_FINAL], 0, 100000000ull);  // both issuers' MMAs have completed
    }
  } else if (warp < W_VAL) {
    // ------------------------------------------------------------------ key operand (thread = key = TMEM lane)
    const int q = warp & 3, kl = 32 * q + lane;
    const int part = q / (4 / SPT);  // the raw stage of this warp's keys within the tile
    const uint32_t lane_off = static_cast<uint32_t>(32 * q) << 16;
    float4* kp = reinterpret_cast<float4*>(smem + SM::OFF_KP);
    uint32_t* zb = reinterpret_cast<uint32_t*>(smem + SM::OFF_ZB);
    // this key's row of the correction MMA's A: k 8-15 zero in every buffer; k8v4: k 0-2 the constant -128 x 2^-14
    uint8_t* const az = smem + SM::OFF_AZ + (kl >> 3) * SM::AZ_MGROUP + (kl & 7) * 16;
#pragma unroll
    for (int b = 0; b < SM::AZB; ++b) {
      *reinterpret_cast<uint4*>(az + b * SM::AZ_BYTES + SM::AZ_KHALF) = make_uint4(0u, 0u, 0u, 0u);
      if constexpr (FMT != FMT_INT4)
        *reinterpret_cast<uint4*>(az + b * SM::AZ_BYTES) = make_uint4(0xA000A000u, 0x0000A000u, 0u, 0u);
    }
    fence_async_smem();  // read by the MMAs (async proxy) after the first key-operand barrier
    for (int i = 0; i < ntl; ++i) {
      const int u = i * SPT + part, stage = u % RS, ki = i % KPS;
      bool ok = mbar_wait_spin(&bars[D_RAW_FULL + stage], (u / RS) & 1);
      if (i >= KPS) ok = ok && mbar_wait_spin(&bars[D_KP_FREE + ki], ((i / KPS) - 1) & 1);
      if (__any_sync(0xffffffffu, !ok)) {
        failed = true;
        break;
      }
      const uint8_t* cell = smem + SM::OFF_RAW + stage * SM::RAW + (kl - part * SK) * CELL;
      const uint32_t kw = *reinterpret_cast<const uint32_t*>(cell + CL::KS);
      const uint32_t vw = *reinterpret_cast<const uint32_t*>(cell + CL::VS);
      const bool valid = (tile0 + i) * DEC_TILE + kl < n;
      float ks, kz = 0.f;
      if constexpr (FMT == FMT_INT4) {
        ks = __uint_as_float(kw & 0xFFFFFFF0u);
        kz = static_cast<float>(kw & 0xFu);
      } else {
        ks = __uint_as_float(kw);
      }
      kp[ki * 128 + kl] = make_float4(ks, kz, valid ? __uint_as_float(vw & 0xFFFFFFF0u) : 0.f, 0.f);
      // value zero-point operand biases of the key pair (a even, a + 1): key a stores {1024 + zp_a, 1024 + zp_b},
      // key a + 1 stores {-(64 + zp_a), -(64 + zp_b)} (fp16 pairs, low half = key a)
      {
        const uint32_t vz = vw & 0xFu;
        const uint32_t lo16 = 0x6400u | vz, hi16 = 0xD400u | (vz << 4);
        const uint32_t other = __shfl_xor_sync(0xffffffffu, (lane & 1) ? lo16 : hi16, 1);
        zb[ki * 128 + kl] = (lane & 1) ? (other | (hi16 << 16)) : (lo16 | (other << 16));
      }
      // int4: -zp x 2^-14 as fp16 (exact: zp < 16), the key's k 0-2 of the correction MMA's A
      uint32_t zneg = 0u;
      if constexpr (FMT == FMT_INT4) zneg = __half_as_ushort(__float2half_rn(-ldexpf(kz, -14)));
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) {  // 256 channels (128 TMEM columns) per chunk
        const int k = i * NCH + ch, sl = k % AKS;
        if (k >= AKS && __any_sync(0xffffffffu, !mbar_wait_spin(&bars[D_AK_FREE + sl], ((k - AKS) / AKS) & 1))) {
          failed = true;
          break;
        }
        tc_fence_after();
        if constexpr (FMT == FMT_INT4) {  // its buffer is free with the slot: the correction MMA goes with chunk 0
          if (ch == 0)
            *reinterpret_cast<uint4*>(az + (sl % SM::AZB) * SM::AZ_BYTES) =
                make_uint4(zneg | (zneg << 16), zneg, 0u, 0u);
        }
        const uint32_t dst = tmem + (sl ? TM::AK1 : TM::AK0) + lane_off;
        const uint8_t* kc = cell + ch * (CL::KB / NCH);
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {  // 32 TMEM columns (64 channels) per store (a loop: instruction-cache size)
          uint32_t a[32];
          if constexpr (FMT == FMT_INT4) {
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4) {
              const uint2 w2 = *reinterpret_cast<const uint2*>(kc + 32 * c + 8 * k4);
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const uint32_t w = e ? w2.y : w2.x, w8 = w >> 8;
                const int j = 8 * k4 + 4 * e;
                a[j + 0] = w & KEY_SUB_LO;   // channels 8 w' + {0, 4}: u x 2^-24
                a[j + 1] = w & KEY_SUB_HI;   // {1, 5}: 16 u x 2^-24
                a[j + 2] = w8 & KEY_SUB_LO;  // {2, 6}
                a[j + 3] = w8 & KEY_SUB_HI;  // {3, 7}
              }
            }
          } else {
#pragma unroll
            for (int k8 = 0; k8 < 8; ++k8) {
              const uint2 w2 = *reinterpret_cast<const uint2*>(kc + 64 * c + 8 * k8);
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const uint32_t x = (e ? w2.y : w2.x) ^ 0x80808080u;
                const int j = 4 * k8 + 2 * e;
                // {c0 + 128, c1 + 128} x 2^-24
                a[j] = prmt(x, 0u, 0x4140u);
                a[j + 1] = prmt(x, 0u, 0x4342u);
              }
            }
          }
          tmem_st32u(dst + 32 * c, a);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        if constexpr (FMT == FMT_INT4) {
          if (ch == 0) fence_async_smem();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[D_AK_FULL + sl]);
      }
      if (failed) break;
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bars[D_KP_FULL + ki]);
        mbar_arrive(&bars[D_RAW_EMPTY + stage]);
      }
    }
  } else if (warp < W_SMX || warp >= W_VB) {
    // ------------------------------------------------------------------ value operand (V^T, lane = channel)
    // Thread (g, t) of quarter q converts the words wv = 8 (q HS/256 + v) + g, v < HS/256 (channels 8 wv + [0, 8)),
    // of keys 4 t + [0, 4) of every 16-key block. Lane 32 q + g + 8 m of channel tile 2 v + c holds channel
    // 8 wv + 4 c + m = 64 (q HS/256 + v) + 8 g + 4 c + m.
    constexpr int WPT = HS / 256;
    constexpr int NB = VK >= 32 ? 2 : 1;  // 16-key blocks per TMEM store
    const int q = warp & 3, g = lane >> 2, t = lane & 3;
    constexpr int KBN = VK / (16 * NB);  // block groups (one TMEM store each) per slot
    // with two sets, set s converts the slots h = s, s + 2, ...: each warp hands over one slot per tile
    static_assert(VSETS == 1 || (VSLOTS % VSETS == 0 && SPT == 1), "value slots split evenly over the warp sets");
    const int h0 = warp >= W_VB ? 1 : 0;
    const uint32_t* zb = reinterpret_cast<const uint32_t*>(smem + SM::OFF_ZB);
    for (int i = 0; i < ntl && !failed; ++i) {
      const int ki = i % KPS;
      if (__any_sync(0xffffffffu, !mbar_wait_spin(&bars[D_KP_FULL + ki], (i / KPS) & 1))) {
        failed = true;
        break;
      }
      int stage = 0;
#pragma unroll 1
      for (int h = h0; h < VSLOTS; h += VSETS) {  // slot h: keys [h VK, h VK + VK) of the tile, TMEM slot k & 1
        const int part = h * VK / SK;
        if ((h * VK) % SK == 0 || h == h0) {  // the slot starts a raw stage, or this warp's first slot
          const int u = i * SPT + part;
          stage = u % RS;
          if (__any_sync(0xffffffffu, !mbar_wait_spin(&bars[D_RAW_FULL + stage], (u / RS) & 1))) {
            failed = true;
            break;
          }
        }
        const int k = i * VSLOTS + h, sl = k & 1;
        if (k >= 2 && __any_sync(0xffffffffu, !mbar_wait_spin(&bars[D_AV_FREE + sl], ((k - 2) >> 1) & 1))) {
          failed = true;
          break;
        }
        tc_fence_after();
        const uint8_t* raw = smem + SM::OFF_RAW + stage * SM::RAW + CL::V + 32 * q * WPT + 4 * g;
#pragma unroll
        for (int v = 0; v < WPT; ++v) {
#pragma unroll 1
          for (int kb = 0; kb < KBN; ++kb) {  // a loop, not unrolled: instruction-cache size
            uint32_t r[4][4 * NB];  // [store (channel tile 2 v + c, lane half lb)][registers]
#pragma unroll
            for (int rr = 0; rr < NB; ++rr) {
              const int kt = h * VK + 16 * (NB * kb + rr) + 4 * t;  // first of the thread's 4 keys in the tile
              const uint8_t* src = raw + 32 * v + (kt - part * SK) * CELL;
              uint32_t w[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) w[j] = *reinterpret_cast<const uint32_t*>(src + j * CELL);
              const uint4 bz = *reinterpret_cast<const uint4*>(zb + ki * 128 + kt);
#pragma unroll
              for (int f = 0; f < 2; ++f) {
                const uint32_t lo_b = f ? bz.z : bz.x, hi_b = f ? bz.w : bz.y;
                const uint32_t x = prmt(w[2 * f], w[2 * f + 1], 0x5410u), y = prmt(w[2 * f], w[2 * f + 1], 0x7632u);
                const uint32_t x8 = x >> 8, y8 = y >> 8;
                r[0][4 * rr + f] = nib_lo(x, lo_b);       // channel tile 2 v, m 0
                r[0][4 * rr + 2 + f] = nib_hi(x, hi_b);   // tile 2 v, m 1
                r[1][4 * rr + f] = nib_lo(x8, lo_b);      // tile 2 v, m 2
                r[1][4 * rr + 2 + f] = nib_hi(x8, hi_b);  // tile 2 v, m 3
                r[2][4 * rr + f] = nib_lo(y, lo_b);       // tile 2 v + 1, m 0
                r[2][4 * rr + 2 + f] = nib_hi(y, hi_b);
                r[3][4 * rr + f] = nib_lo(y8, lo_b);
                r[3][4 * rr + 2 + f] = nib_hi(y8, hi_b);
              }
            }
#pragma unroll
            for (int st = 0; st < 4; ++st) {
              const int c = st >> 1, lb = st & 1;
              const uint32_t addr = tmem + (static_cast<uint32_t>(32 * q + 16 * lb) << 16) + TM::AV + TM::SLOT * sl +
                                    (VK / 2) * (2 * v + c) + 8 * NB * kb;
              if constexpr (NB == 2) tmem_st_16x256b_x2(addr, r[st]);
              else tmem_st_16x256b_x1(addr, r[st]);
            }
          }
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&bars[D_AV_FULL + sl]);
          // the stage's last slot (with two sets, each warp's last slot of the tile's single stage)
          if (VSETS == 2 ? h + VSETS >= VSLOTS : ((h + 1) * VK) % SK == 0) mbar_arrive(&bars[D_RAW_EMPTY + stage]);
        }
      }
      if (failed) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[D_KP_FREE + ki]);
    }
  } else {
    // ------------------------------------------------------------------ softmax (thread = key = TMEM lane)
    // SMX_HALVES warps per lane quarter, each taking RL / SMX_HALVES of the rows (RL a multiple of 8 covering the
    // launch's largest row count), with compile-time row indices and no per-row branch. Row states live in rp[].y: the row maximum
    // (log2 units), 0 before the first tile (whose rescale path always runs, since no value range is known yet), and
    // +inf for a row past the sequence's rows or one with no key in this split (keys visible to a row are a prefix of
    // the context, so such a row never gets one later): its scores are -inf and its probabilities 0. The scores are
    // kept as exp arguments (score minus the row maximum), so the exponentials read no shared memory.
    const int q = warp & 3, kl = 32 * q + lane, stid = tid - 32 * W_SMX;
    const int hf = (warp - W_SMX) >> 2;
    const uint32_t lane_off = static_cast<uint32_t>(32 * q) << 16;
    float2* rp = reinterpret_cast<float2*>(smem + SM::OFF_RP);  // [2][NR]: row scale, row maximum
    int* lim = reinterpret_cast<int*>(smem + SM::OFF_LIM);
    int* wlo = reinterpret_cast<int*>(smem + SM::OFF_WLO);
    float* red_vs = reinterpret_cast<float*>(smem + SM::OFF_RED);  // [softmax warps]
    float* frow = red_vs + 8;                                                // [NR]
    float2* adj = reinterpret_cast<float2*>(frow + NR);                      // [NR]
    float* sb = reinterpret_cast<float*>(smem + SM::OFF_SB);                 // [NR][128]
    const float4* kp = reinterpret_cast<const float4*>(smem + SM::OFF_KP);
    const int causal_from = min(n, vis_base + 1);
    // sliding window: the last token's first key; a tile starting at or before it holds keys below some row's window
    // (masked path), and a row whose window starts after the split's first tile opens there
    const int win_hi = (FEAT && p.window > 0) ? vis_base + qlen - p.window : -1;
    // softcap in log2 units (the scores here are log2 e x the natural ones) and the factor of its exponential
    const float capl = FEAT ? p.softcap * LOG2E : 0.f;
    const float cap_k = capl > 0.f ? 2.f * LOG2E / capl : 0.f;
    // query rows (prepared by K0q: programmatic dependent launch, wait for it only now) -> Q^T operand, K-major
    // 128B-swizzled; row constants
    asm volatile("griddepcontrol.wait;" ::: "memory");
    {
      const uint8_t* qsrc = p.qrec + ((static_cast<int64_t>(kvh) * p.num_tokens + q0) * p.group) * QREC;
      for (int idx = stid; idx < NR * (HS / 8); idx += SMX_THREADS) {
        const int r = idx / (HS / 8), ch = idx % (HS / 8);  // 16-byte chunk ch (8 channels) of row r
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (r < rows) v = *reinterpret_cast<const uint4*>(qsrc + r * QREC + 16 * ch);
        *reinterpret_cast<uint4*>(smem + SM::OFF_Q + (ch >> 3) * SM::ATOM + sw128_off(r, ch & 7)) = v;
      }
      for (int idx = stid; idx < NR * 2; idx += SMX_THREADS) {  // k 0-15 of the correction atom: terms, zeros
        const int r = idx >> 1, ch = idx & 1;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (r < rows && ch == 0) {
          const uint32_t* rz = reinterpret_cast<const uint32_t*>(qsrc + r * QREC + 2 * HS + 4);
          v = make_uint4(rz[0], rz[1], 0u, 0u);
        }
        *reinterpret_cast<uint4*>(smem + SM::OFF_QZ + sw128_off(r, ch)) = v;
      }
      for (int r = stid; r < NR; r += SMX_THREADS) {
        float2 c = make_float2(0.f, INFINITY);
        if (r < rows) c = make_float2(*reinterpret_cast<const float*>(qsrc + r * QREC + 2 * HS), 0.f);
        rp[r] = c;
        rp[NR + r] = c;
        lim[r] = r < rows ? min(n - 1, vis_base + r / p.group) : -1;
        wlo[r] = (FEAT && p.window > 0 && r < rows) ? vis_base + r / p.group - p.window + 1 : -1;
        frow[r] = 1.f;
      }
      // P^T rows RL .. NR - 1 (whole 8-row groups: RL is a multiple of 8) are read by the MMAs but never written by
      // the loops below: zero them once, in both buffers
      if constexpr (RL < NR) {
        for (int idx = stid; idx < 2 * (NR - RL) / 8 * DEC_TILE; idx += SMX_THREADS) {
          const int b = idx / ((NR - RL) / 8 * DEC_TILE), rem = idx % ((NR - RL) / 8 * DEC_TILE);
          *reinterpret_cast<uint4*>(smem + SM::OFF_P + SM::p_off(b, RL + rem / DEC_TILE * 8, rem % DEC_TILE)) =
              make_uint4(0u, 0u, 0u, 0u);
        }
      }
    }
    fence_async_smem();
    named_bar_or(BAR_SMX, SMX_THREADS, false);  // row constants visible to every softmax thread
    if (lane == 0) mbar_arrive(&bars[D_Q_FULL]);

    auto role = [&](auto half) {
      constexpr int RH = RL / SMX_HALVES, R0 = decltype(half)::value * RH;  // this warp's rows [R0, R0 + RH)
      float l[RH];
#pragma unroll
      for (int r = 0; r < RH; ++r) l[r] = 0.f;
      int mb = 0;           // current row-state buffer
      int e_run = -1000;    // running power-of-two range of the value scales: every one < 2^e_run
      float pv_mul = 0.f;   // 2^-e_run
      float v_limit = 0.f;  // 2^e_run
      for (int i = 0; i < ntl; ++i) {
        const int b = i & 1;
        const int ki = i % KPS;
        bool ok = mbar_wait_bounded(&bars[D_S_FULL + b], (i >> 1) & 1);
        ok = ok && mbar_wait_bounded(&bars[D_KP_FULL + ki], (i / KPS) & 1);
        failed |= __any_sync(0xffffffffu, !ok);
        float s[RH];
        if (!failed) {
          tc_fence_after();
          tmem_ld_cols<RH>(tmem + TM::S + NR * b + R0 + lane_off, s);
        } else {
#pragma unroll
          for (int r = 0; r < RH; ++r) s[r] = 0.f;
        }
        tc_fence_before();
        const float4 kv = kp[ki * 128 + kl];  // key scale, key zero point, value scale (0 past the context)
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&bars[D_S_FREE + b]);
          mbar_arrive(&bars[D_KP_FREE + ki]);
        }
        const int tok = (tile0 + i) * DEC_TILE + kl;
        // exp arguments: score (log2 units) minus the row maximum; emax: the largest one
        float emax = -INFINITY;
        bool opening = false;  // a row not opened yet (sliding window) has a key in this tile
        auto logits = [&](auto masked, auto windowed) {
#pragma unroll
          for (int r = 0; r < RH; ++r) {
            if (r % 4 == 0 && r > 0) asm volatile("" ::: "memory");  // 4 rows' constants in flight at a time
            const float2 c = rp[mb * NR + R0 + r];  // row scale, row maximum
            if constexpr (FEAT) {
              // A row with no key of this split so far (-inf: FEAT only) takes its scores as they are and sends the
              // tile down the slow path, which opens it; with a window, such a row meets no tile but masked ones
              // before it opens (its first key is at most win_hi), without one it never gets a key (causality).
              const bool fresh = c.y == -INFINITY;
              float t = s[r] * kv.x * c.x;  // the score, log2 units
              if (capl > 0.f) t = softcap_log2(t, capl, cap_k);
              float e = t - (fresh ? 0.f : c.y);
              if constexpr (decltype(masked)::value) {
                // outside the row's keys (its window, when the tile reaches below one) or past the context
                if (tok > lim[R0 + r] || (decltype(windowed)::value && tok < wlo[R0 + r])) e = -INFINITY;
              }
              opening |= fresh && e != -INFINITY;
              s[r] = e;
            } else {
              float e = fmaf(s[r] * kv.x, c.x, -c.y);
              if constexpr (decltype(masked)::value) {
                if (tok > lim[R0 + r]) e = -INFINITY;  // past the row's last key or the context
              }
              s[r] = e;
            }
            emax = fmaxf(emax, s[r]);
          }
        };
        const int tile_start = (tile0 + i) * DEC_TILE;
        if constexpr (FEAT) {
          if (tile_start <= win_hi) logits(std::true_type{}, std::true_type{});
          else if (tile_start + DEC_TILE > causal_from) logits(std::true_type{}, std::false_type{});
          else logits(std::false_type{}, std::false_type{});
        } else {
          if (tile_start + DEC_TILE > causal_from) logits(std::true_type{}, std::false_type{});
          else logits(std::false_type{}, std::false_type{});
        }
        const bool grow = emax > RESCALE_SLACK || kv.z >= v_limit || opening;
        bool rescale = false;
        // every softmax thread takes the same barriers: a wait that ran out is folded into the vote
        if (named_bar_or(BAR_SMX, SMX_THREADS, grow || failed)) {
          if (named_bar_or(BAR_SMX, SMX_THREADS, failed)) {
            failed = true;
            break;
          }
          // slow path: exact tile maxima and value range, new row states, rescale factors. The exp arguments go
          // through shared memory, so that thread r can take row r's maximum over the 128 keys.
#pragma unroll
          for (int r = 0; r < RH; ++r) sb[(R0 + r) * 128 + kl] = s[r];
          {
            const float vm = warp_max(kv.z);
            if (lane == 0) red_vs[warp - W_SMX] = vm;
          }
          named_bar_or(BAR_SMX, SMX_THREADS, false);
          float vmax = red_vs[0];
#pragma unroll
          for (int k = 1; k < 4 * SMX_HALVES; ++k) vmax = fmaxf(vmax, red_vs[k]);
          // e_tile: vmax < 2^e_tile (value scales are normal, positive fp32: exponent field + 1 - bias)
          const int e_tile = vmax > 0.f ? static_cast<int>((__float_as_uint(vmax) >> 23) & 0xFFu) - 126 : -1000;
          const bool first = e_run == -1000;
          const int e_new = max(e_run, e_tile);
          const float o_range = first ? 0.f : exp2_int(max(e_run - e_new, -149));
          e_run = e_new;
          pv_mul = e_new == -1000 ? 0.f : exp2_int(-e_new);
          v_limit = e_new == -1000 ? 0.f : exp2_int(e_new);
          float f = 1.f;
          if (stid < RL) {  // thread r: row r
            const int r = stid;
            float2 c = rp[mb * NR + r];
            float2 ad = make_float2(1.f, 0.f);
            if (c.y != INFINITY) {  // an open row of the sequence, or one not opened yet (-inf)
              float mx = -INFINITY;
              const float4* row = reinterpret_cast<const float4*>(sb + r * 128);
#pragma unroll 8
              for (int k = 0; k < 32; ++k) {
                const float4 v = row[(k + r) & 31];  // rotated start: threads read different banks
                mx = fmaxf(mx, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
              }
              if constexpr (FEAT) {
                const bool fresh = first || c.y == -INFINITY;  // no key of this split seen yet
                const float cy = c.y == -INFINITY ? 0.f : c.y;  // what the exp arguments were taken against
                const float mt = mx + cy;                        // the tile's largest score
                float mn = c.y;
                // a row without a key so far stays unopened (-inf) when a window may start its keys further on,
                // and is closed otherwise (its keys are a prefix of the context)
                if (fresh) mn = mt != -INFINITY ? mt : (p.window > 0 ? -INFINITY : INFINITY);
                else if (mt > c.y + RESCALE_SLACK) mn = mt;
                if (mn != c.y) {
                  ad.x = fresh ? 0.f : fast_exp2(c.y - mn);
                  ad.y = (mn == -INFINITY || mn == INFINITY) ? -INFINITY : cy - mn;  // -inf: no key, P = 0
                  c.y = mn;
                }
              } else {
                const float mt = mx + c.y;  // the tile's largest score
                float mn = c.y;
                if (first) mn = mt == -INFINITY ? INFINITY : mt;  // no key in this split: the row is closed
                else if (mt > c.y + RESCALE_SLACK) mn = mt;
                if (mn != c.y) {
                  ad.x = first ? 0.f : fast_exp2(c.y - mn);
                  ad.y = c.y - mn;  // -inf for a row that closes
                  c.y = mn;
                }
              }
              f = ad.x * o_range;
            }
            rp[(mb ^ 1) * NR + r] = c;
            frow[r] = f;
            adj[r] = ad;
          }
          rescale = named_bar_or(BAR_SMX, SMX_THREADS, f != 1.f);  // new row states and factors visible
#pragma unroll
          for (int r = 0; r < RH; ++r) {  // the arguments come back from shared memory: no registers held across
            const float2 ad = adj[R0 + r];
            s[r] = sb[(R0 + r) * 128 + kl] + ad.y;
            l[r] *= ad.x;
          }
          mb ^= 1;
        }
        // P^T buffer b is free once PV(i - 2) has completed; O may be rescaled once PV(i - 1) has. (PV(j) completes
        // phase j / 2 of barrier j % 2, which cannot move on before this thread has stored P(j + 2).)
        if (i >= 2) failed |= !mbar_wait_bounded(&bars[D_PV_DONE + b], ((i - 2) >> 1) & 1);
        if (rescale && i >= 1) failed |= !mbar_wait_bounded(&bars[D_PV_DONE + (b ^ 1)], ((i - 1) >> 1) & 1);
        tc_fence_after();
        const float vsp = kv.z * pv_mul;
        // P^T of this thread's key: the rows of an 8-row group are 16 contiguous bytes (MN-major), so two rows
        // convert in one instruction and eight go out in one 16-byte store
        uint8_t* pb = smem + SM::OFF_P + SM::p_off(b, R0, kl);
        if constexpr (RH % 8 == 0 && R0 % 8 == 0) {
#pragma unroll
          for (int g = 0; g < RH / 8; ++g) {
            uint32_t w[4];
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              const int r = 8 * g + 2 * h;
              const float p0 = fast_exp2(s[r]), p1 = fast_exp2(s[r + 1]);
              l[r] += p0;
              l[r + 1] += p1;
              const __half2 v = __floats2half2_rn(p0 * vsp, p1 * vsp);
              w[h] = *reinterpret_cast<const uint32_t*>(&v);
            }
            *reinterpret_cast<uint4*>(pb + g * P_NGROUP) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        } else {
#pragma unroll
          for (int r = 0; r < RH; ++r) {
            const float pe = fast_exp2(s[r]);
            l[r] += pe;
            *reinterpret_cast<__half*>(smem + SM::OFF_P + SM::p_off(b, R0 + r, kl)) = __float2half_rn(pe * vsp);
          }
        }
        if (rescale && i >= 1) {  // before PV(i), which waits for this tile's P
#pragma unroll 1
          for (int c = 0; c < MT; ++c) {
            float o[RH];
            tmem_ld_cols<RH>(tmem + TM::O + NR * c + R0 + lane_off, o);
#pragma unroll
            for (int r = 0; r < RH; ++r) o[r] *= frow[R0 + r];
            tmem_st_cols<RH>(tmem + TM::O + NR * c + R0 + lane_off, o);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
          }
        }
        fence_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[D_P_FULL + b]);
      }
      // ---- epilogue: row sums (thread r adds row r's 128 partial sums), normalised partial O (channel order
      // undone) and its lse
      if (named_bar_or(BAR_SMX, SMX_THREADS, failed)) return;
#pragma unroll
      for (int r = 0; r < RH; ++r) sb[(R0 + r) * 128 + kl] = l[r];
      named_bar_or(BAR_SMX, SMX_THREADS, false);
      if (stid < NR) {
        const int r = stid;
        float inv = 0.f;
        if (r < rows) {
          float lt = 0.f;
          const float4* row = reinterpret_cast<const float4*>(sb + r * 128);
#pragma unroll 8
          for (int k = 0; k < 32; ++k) {
            const float4 v = row[(k + r) & 31];
            lt += (v.x + v.y) + (v.z + v.w);
          }
          const float o_unit = e_run == -1000 ? 0.f : exp2_int(e_run);
          inv = lt > 0.f ? o_unit / lt : 0.f;
          const int tok = q0 + r / p.group, qh = kvh * p.group + r % p.group;
          p.part_lse[(static_cast<int64_t>(tok) * p.nq + qh) * p.num_splits + split] =
              lt > 0.f ? rp[mb * NR + r].y + log2f(lt) : -INFINITY;
        }
        frow[r] = inv;
      }
      named_bar_or(BAR_SMX, SMX_THREADS, false);
      const bool ok = mbar_wait_bounded(&bars[D_PV_DONE + ((ntl - 1) & 1)], ((ntl - 1) >> 1) & 1);
      tc_fence_after();
      const int g = lane & 7, mm = lane >> 3;
      const int64_t head_step = static_cast<int64_t>(p.num_splits) * HS;
      const int64_t tok_step = (static_cast<int64_t>(p.nq) - p.group + 1) * head_step;
      const int tok0 = q0 + R0 / p.group, hg0 = R0 % p.group;
#pragma unroll 1
      for (int c = 0; c < MT && ok; ++c) {  // channel tile c: channels 64 (q HS/256 + c / 2) + 8 g + 4 (c % 2) + mm
        float o[RH];
        tmem_ld_cols<RH>(tmem + TM::O + NR * c + R0 + lane_off, o);
        float* dst = p.part_o + ((static_cast<int64_t>(tok0) * p.nq + kvh * p.group + hg0) * p.num_splits + split) *
                                    HS + 64 * (q * (HS / 256) + (c >> 1)) + 8 * g + 4 * (c & 1) + mm;
        int hg = hg0;
#pragma unroll
        for (int r = 0; r < RH; ++r) {
          if (R0 + r < rows) *dst = o[r] * frow[R0 + r];
          dst += (++hg == p.group) ? tok_step : head_step;  // next query head, or the next token's first head
          if (hg == p.group) hg = 0;
        }
      }
    };
    if constexpr (SMX_HALVES == 1) {
      role(std::integral_constant<int, 0>{});
    } else {
      if (hf == 0) role(std::integral_constant<int, 0>{});
      else role(std::integral_constant<int, 1>{});
    }
  }

  // every role is done with TMEM (the MMA warp saw its last commit complete)
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == W_MMA) tmem_dealloc(tmem, 512);
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
  // mode 0, may be null: per query head, a sink logit (natural units) whose exp joins every row's softmax
  // denominator once, vLLM's attention sinks (vllm/v1/attention/ops/triton_attention_helpers.py:108-138: the row
  // maximum starts at the sink with sum 1 in one segment only; triton_unified_attention.py:356-359)
  const float* sinks;
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
  const float sink = p.sinks != nullptr ? p.sinks[qh] * LOG2E : -INFINITY;  // base 2, like the partials' lse
  M = fmaxf(M, sink);
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
    float s = sink == -INFINITY ? 0.f : exp2f(sink - M);  // the sink: in the denominator only
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

template <int FMT, int DT, int HS, int RL, bool FEAT>
static int launch_decode_t(const DecodeParams& dp, int grid_z, cudaStream_t st) {
  constexpr int NR = RL <= 16 ? 16 : 32;  // the MMAs' N: a multiple of 16 at M 128
  using SM = DecSmem<FMT, HS, NR>;
  static std::atomic<bool> configured[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(decode_kernel<FMT, DT, HS, NR, RL, FEAT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, SM::BYTES);
    if (e != cudaSuccess) return set_error(QP_ERR_CUDA, "decode smem attribute: %s", cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) configured[dev].store(true, std::memory_order_release);
  }
  // programmatic dependent launch: the CTAs start their cache copies while K0q finishes (the softmax warps wait for
  // it before reading the query rows)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(dp.num_splits), static_cast<unsigned>(dp.nkv), static_cast<unsigned>(grid_z));
  cfg.blockDim = dim3(DecWarps<HS, RL>::THREADS);
  cfg.dynamicSmemBytes = SM::BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, decode_kernel<FMT, DT, HS, NR, RL, FEAT>, dp);
  if (e != cudaSuccess) return set_error(QP_ERR_CUDA, "decode launch: %s", cudaGetErrorString(e));
  return QP_OK;
}

// K0q, then K1 with the smallest row count (a multiple of 8) that covers `rows`
template <int FMT, int DT, int HS>
static int launch_decode_hs(const DecodeParams& dp, int rows, int grid_z, cudaStream_t st) {
  const int64_t qrows = dp.num_tokens * dp.nq;
  if ((qrows + 7) / 8 > 0x7fffffff) return set_error(QP_ERR_UNSUPPORTED, "decode: too many query rows");
  decode_qprep_kernel<FMT, DT, HS><<<static_cast<unsigned>((qrows + 7) / 8), 256, 0, st>>>(
      dp.q, dp.q_st, dp.q_sh, dp.num_tokens, dp.nq, dp.nkv, dp.sign_bits, dp.q_rotated, dp.qk_scale,
      const_cast<uint8_t*>(dp.qrec));
  const int rc = check_launch("decode q prep");
  if (rc) return rc;
  if (dp.window > 0 || dp.softcap > 0.f) {
    if (rows <= 8) return launch_decode_t<FMT, DT, HS, 8, true>(dp, grid_z, st);
    if (rows <= 16) return launch_decode_t<FMT, DT, HS, 16, true>(dp, grid_z, st);
    if (rows <= 24) return launch_decode_t<FMT, DT, HS, 24, true>(dp, grid_z, st);
    return launch_decode_t<FMT, DT, HS, 32, true>(dp, grid_z, st);
  }
  if (rows <= 8) return launch_decode_t<FMT, DT, HS, 8, false>(dp, grid_z, st);
  if (rows <= 16) return launch_decode_t<FMT, DT, HS, 16, false>(dp, grid_z, st);
  if (rows <= 24) return launch_decode_t<FMT, DT, HS, 24, false>(dp, grid_z, st);
  return launch_decode_t<FMT, DT, HS, 32, false>(dp, grid_z, st);
}

template <int FMT>
static int launch_decode_fmt(int dtype, int hs, const DecodeParams& dp, int rows, int grid_z, cudaStream_t st) {
  if (hs == 512)
    return dtype == DT_BF16 ? launch_decode_hs<FMT, DT_BF16, 512>(dp, rows, grid_z, st)
                            : launch_decode_hs<FMT, DT_F16, 512>(dp, rows, grid_z, st);
  return dtype == DT_BF16 ? launch_decode_hs<FMT, DT_BF16, 256>(dp, rows, grid_z, st)
                          : launch_decode_hs<FMT, DT_F16, 256>(dp, rows, grid_z, st);
}

static int launch_decode(int fmt, int dtype, int hs, const DecodeParams& dp, int rows, int grid_z, cudaStream_t st) {
  return fmt == FMT_INT4 ? launch_decode_fmt<FMT_INT4>(dtype, hs, dp, rows, grid_z, st)
                         : launch_decode_fmt<FMT_K8V4>(dtype, hs, dp, rows, grid_z, st);
}

}  // namespace qp

using namespace qp;

// Split-count heuristic: one CTA per SM (a CTA holds all of TMEM), whole waves, a fixed cost of about two tiles per
// CTA (pipeline fill and drain, epilogue), 128-key tiles.
extern "C" int qp_decode_num_splits(int num_seqs, int num_kv_heads, int max_seqlen_k, int sm_count) {
  if (sm_count <= 0) sm_count = device_sm_count();
  const int pairs = max(1, num_seqs * num_kv_heads);
  const int tiles = max(1, (max_seqlen_k + DEC_TILE - 1) / DEC_TILE);
  const int max_splits = max(1, min(1024, tiles / 2));
  int best = 1;
  double best_cost = 1e30;
  for (int s = 1; s <= max_splits; ++s) {
    const long ctas = static_cast<long>(pairs) * s;
    const long waves = (ctas + sm_count - 1) / sm_count;
    const double cost = waves * (static_cast<double>((tiles + s - 1) / s) + 2.0);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

// Workspace of qp_paged_decode: [part_o rows x head fp32][part_lse rows fp32, 256-aligned][prepared query rows
// tokens x q heads x q_rec_bytes(head) bytes], rows = tokens x q heads x splits.
static int64_t decode_qrec_offset(int64_t num_q_tokens, int num_q_heads, int head_size, int num_splits) {
  const int64_t rows = num_q_tokens * num_q_heads * static_cast<int64_t>(num_splits);
  return rows * head_size * 4 + ((rows * 4 + 255) / 256) * 256;
}

extern "C" int64_t qp_decode_workspace_bytes(int64_t num_q_tokens, int num_q_heads, int head_size, int num_splits) {
  return decode_qrec_offset(num_q_tokens, num_q_heads, head_size, num_splits) +
         num_q_tokens * num_q_heads * static_cast<int64_t>(q_rec_bytes(head_size));
}

// Checks shared by the decode entry points: formats, head size, cache layout.
static int decode_check_cache(const char* who, int fmt, int dtype, int head_size, const void* cache, int block_size,
                              int64_t block_stride, int64_t head_stride, int64_t slot_stride, int64_t k_off,
                              int64_t ks_off, int64_t v_off, int64_t vs_off) {
  if (fmt != FMT_INT4 && fmt != FMT_K8V4) return set_error(QP_ERR_UNSUPPORTED, "%s: format %d", who, fmt);
  if (dtype != DT_BF16 && dtype != DT_F16) return set_error(QP_ERR_UNSUPPORTED, "%s: dtype %d", who, dtype);
  if (head_size != 256 && head_size != 512)
    return set_error(QP_ERR_UNSUPPORTED, "%s: head size %d (this build: 256, 512)", who, head_size);
  const int kb = fmt == FMT_INT4 ? head_size / 2 : head_size;
  const int cell = kb + 8 + head_size / 2;
  if (slot_stride != cell)
    return set_error(QP_ERR_LAYOUT, "%s: cells of a (block, head) must be contiguous (slot stride %lld, cell %d)", who,
                     (long long)slot_stride, cell);
  if (k_off != 0 || ks_off != kb || v_off != kb + 4 || vs_off != kb + 4 + head_size / 2)
    return set_error(QP_ERR_LAYOUT, "%s: unexpected cell field offsets", who);
  if (block_size <= 0 || block_size % 16 || (reinterpret_cast<uintptr_t>(cache) & 15) || (block_stride & 15) ||
      (head_stride & 15))
    return set_error(QP_ERR_LAYOUT, "%s: block size must be a multiple of 16 and the cache 16-byte aligned", who);
  return QP_OK;
}

static MergeParams decode_merge_params(const DecodeParams& dp, int head_size, int out_mode, void* out,
                                       int64_t out_stride_token, int64_t out_stride_head, float* lse_out,
                                       const float* sinks = nullptr) {
  MergeParams mp{};
  mp.part_o = dp.part_o;
  mp.part_lse = dp.part_lse;
  mp.po_t = static_cast<int64_t>(dp.nq) * dp.num_splits * head_size;
  mp.po_h = static_cast<int64_t>(dp.num_splits) * head_size;
  mp.po_s = head_size;
  mp.pl_t = static_cast<int64_t>(dp.nq) * dp.num_splits;
  mp.pl_h = dp.num_splits;
  mp.pl_s = 1;
  mp.num_splits = dp.num_splits;
  mp.nq = dp.nq;
  mp.mode = out_mode;
  mp.out = out;
  mp.out_st = out_stride_token;
  mp.out_sh = out_stride_head;
  mp.lse_out = lse_out;
  mp.lo_t = dp.nq;
  mp.lo_h = 1;
  mp.sign_bits = dp.sign_bits;
  mp.out_scale = 1.f / static_cast<float>(head_size);
  mp.sinks = sinks;
  return mp;
}

// Points dp's partials and prepared query rows into `workspace` (qp_decode_workspace_bytes layout).
static void decode_bind_workspace(DecodeParams& dp, void* workspace, int head_size) {
  const int64_t rows = dp.num_tokens * dp.nq * static_cast<int64_t>(dp.num_splits);
  dp.part_o = static_cast<float*>(workspace);
  dp.part_lse = dp.part_o + rows * head_size;
  dp.qrec = static_cast<const uint8_t*>(workspace) + decode_qrec_offset(dp.num_tokens, dp.nq, head_size, dp.num_splits);
}

extern "C" int qp_paged_decode(int fmt, int dtype, const void* q, int64_t q_stride_token, int64_t q_stride_head,
                               void* out, int64_t out_stride_token, int64_t out_stride_head, int64_t num_q_tokens,
                               int num_seqs, const int32_t* cu_seqlens_q, const int32_t* seqused_k, int max_seqlen_q,
                               const int32_t* block_table, int64_t block_table_stride, const void* cache,
                               int block_size, int64_t block_stride, int64_t head_stride, int64_t slot_stride,
                               int64_t k_off, int64_t ks_off, int64_t v_off, int64_t vs_off, int num_q_heads,
                               int num_kv_heads, int head_size, float softmax_scale, const uint32_t* rht_sign_bits,
                               int q_rotated, int tokens_after_keys, int sliding_window, float softcap,
                               const float* sinks, int out_mode, float* lse_out, int num_splits, void* workspace,
                               int64_t workspace_bytes, void* stream) {
  int rc = decode_check_cache("decode", fmt, dtype, head_size, cache, block_size, block_stride, head_stride,
                              slot_stride, k_off, ks_off, v_off, vs_off);
  if (rc) return rc;
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
  if (sliding_window < 0) return set_error(QP_ERR_INVALID, "decode: sliding_window %d", sliding_window);
  if (!(softcap >= 0.f) || isinf(softcap)) return set_error(QP_ERR_INVALID, "decode: softcap %g", softcap);
  if (sinks && out_mode != 0)
    return set_error(QP_ERR_INVALID, "decode: sinks need out_mode 0 (a partial must not carry them: they count once)");
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
  dp.nq = num_q_heads;
  dp.nkv = num_kv_heads;
  dp.group = group;
  dp.qk_scale = softmax_scale / static_cast<float>(head_size) * LOG2E;
  dp.sign_bits = rht_sign_bits;
  dp.q_rotated = q_rotated;
  dp.num_tokens = num_q_tokens;
  // a window wider than any context here (2^30 keys) masks nothing
  const int window = sliding_window >= (1 << 30) ? 0 : sliding_window;
  // tokens after the keys change the causal mask up to qlen - 1 of them, a window's mask up to qlen + window - 1
  dp.tokens_after = static_cast<int>(std::min<int64_t>(tokens_after_keys, static_cast<int64_t>(max_seqlen_q) + window));
  dp.window = window;
  dp.softcap = softcap;
  dp.num_splits = num_splits;
  decode_bind_workspace(dp, workspace, head_size);

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  rc = launch_decode(fmt, dtype, head_size, dp, max_seqlen_q * group, num_seqs, st);
  if (rc) return rc;
  if (out_mode == 2) return QP_OK;  // split partials stay in the workspace
  return merge_dispatch(decode_merge_params(dp, head_size, out_mode, out, out_stride_token, out_stride_head, lse_out,
                                          sinks),
                        dtype, head_size, num_q_tokens, st, true);
}

// ---------------------------------------------------------------------------------------------------------------
// Chunk prefill through K1 (the head-512 path of qp_prefill): the chunk's qlen query tokens become sub-sequences of
// chunk_q = 32 / group tokens (32 query rows each), every one a split-KV decode over the keys its last token sees.
// The sub-sequences of one KV head start on the same key tiles and move through them at the same pace, so the keys
// are read from HBM about once and shared through L2.
static int chunk_q_of(int group) { return group > DEC_MAX_ROWS ? 0 : DEC_MAX_ROWS / group; }

static int chunk_num_splits(int qlen, int n, int num_q_heads, int num_kv_heads) {
  const int cq = chunk_q_of(num_q_heads / num_kv_heads);
  return qp_decode_num_splits((qlen + cq - 1) / cq, num_kv_heads, n, 0);
}

int64_t decode_chunk_workspace_bytes(int qlen, int n, int num_q_heads, int num_kv_heads, int head_size) {
  if (qlen <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads || !chunk_q_of(num_q_heads / num_kv_heads))
    return 0;
  return qp_decode_workspace_bytes(qlen, num_q_heads, head_size, chunk_num_splits(qlen, n, num_q_heads, num_kv_heads));
}

int decode_chunk_prefill(int fmt, int dtype, const void* q, int64_t q_stride_token, int64_t q_stride_head, void* out,
                         int64_t out_stride_token, int64_t out_stride_head, int qlen, int n, const int32_t* block_row,
                         const void* cache, int block_size, int64_t block_stride, int64_t head_stride,
                         int64_t slot_stride, int64_t k_off, int64_t ks_off, int64_t v_off, int64_t vs_off,
                         int num_q_heads, int num_kv_heads, int head_size, float softmax_scale,
                         const uint32_t* rht_sign_bits, int q_rotated, int tokens_after_keys, int out_mode,
                         float* lse_out, void* workspace, int64_t workspace_bytes, void* stream) {
  int rc = decode_check_cache("prefill", fmt, dtype, head_size, cache, block_size, block_stride, head_stride,
                              slot_stride, k_off, ks_off, v_off, vs_off);
  if (rc) return rc;
  const int group = num_q_heads / num_kv_heads;
  const int cq = chunk_q_of(group);
  if (!cq) return set_error(QP_ERR_UNSUPPORTED, "prefill: %d query heads per KV head > %d", group, DEC_MAX_ROWS);
  const int subs = (qlen + cq - 1) / cq;
  if (subs > 65535 || num_kv_heads > 65535) return set_error(QP_ERR_UNSUPPORTED, "prefill: grid too large");
  const int splits = chunk_num_splits(qlen, n, num_q_heads, num_kv_heads);
  const int64_t need = qp_decode_workspace_bytes(qlen, num_q_heads, head_size, splits);
  if ((reinterpret_cast<uintptr_t>(workspace) & 15) || workspace_bytes < need)
    return set_error(QP_ERR_WORKSPACE, "prefill: workspace of %lld bytes < %lld", (long long)workspace_bytes,
                     (long long)need);
  DecodeParams dp{};
  dp.q = q;
  dp.q_st = q_stride_token;
  dp.q_sh = q_stride_head;
  dp.block_table = block_row;
  dp.cache = static_cast<const uint8_t*>(cache);
  dp.block_size = block_size;
  dp.block_stride = block_stride;
  dp.head_stride = head_stride;
  dp.nq = num_q_heads;
  dp.nkv = num_kv_heads;
  dp.group = group;
  dp.qk_scale = softmax_scale / static_cast<float>(head_size) * LOG2E;
  dp.sign_bits = rht_sign_bits;
  dp.q_rotated = q_rotated;
  dp.num_tokens = qlen;
  dp.tokens_after = tokens_after_keys < qlen ? tokens_after_keys : qlen;  // >= qlen: nothing masked
  dp.chunk_q = cq;
  dp.chunk_n = n;
  dp.num_splits = splits;
  decode_bind_workspace(dp, workspace, head_size);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  rc = launch_decode(fmt, dtype, head_size, dp, cq * group, subs, st);
  if (rc) return rc;
  return merge_dispatch(decode_merge_params(dp, head_size, out_mode, out, out_stride_token, out_stride_head, lse_out),
                        dtype, head_size, qlen, st, true);
}

// ---------------------------------------------------------------------------------------------------------------
// Short prefill chunks of several sequences in one launch of K1 (the counterpart of the reference's Triton 2D
// sub-batch for every chunk that is not long, int4_kv.py:313-323). Chunk i (query tokens [cu[i], cu[i + 1]), its
// last token seeing used[i] keys through block-table row i) becomes ceil(qlen_i / cq) sub-sequences of cq = 32 /
// group tokens, causal inside each; the table is built on the device from the same length tensors, so the call reads
// nothing back to the host. The grid holds an upper bound of sub-sequences computed from host-known sizes; entries
// past the real ones hold 0 query tokens and their CTAs return at once.
__global__ void __launch_bounds__(32) varlen_table_kernel(const int32_t* cu, const int32_t* used, int num_chunks,
                                                          int cq, int upper, int4* table) {
  const int lane = threadIdx.x;
  int base = 0;
  for (int c0 = 0; c0 < num_chunks; c0 += 32) {  // 32 chunks at a time, offsets by a warp scan
    const int i = c0 + lane;
    int q0 = 0, ql = 0, n = 0;
    if (i < num_chunks) {
      q0 = cu[i];
      ql = max(0, cu[i + 1] - q0);
      n = used[i];
    }
    const int ns = (ql + cq - 1) / cq;
    int incl = ns;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += t;
    }
    const int off = base + incl - ns;
    for (int j = 0; j < ns && off + j < upper; ++j) {
      const int a = j * cq, len = min(cq, ql - a);
      table[off + j] = make_int4(q0 + a, len, n - ql + a + len, i);  // keys seen by the sub-sequence's last token
    }
    base += __shfl_sync(0xffffffffu, incl, 31);
  }
  for (int e = base + lane; e < upper; e += 32) table[e] = make_int4(0, 0, 0, 0);
}

static int varlen_upper(int64_t num_q_tokens, int num_chunks, int cq) {
  return static_cast<int>((num_q_tokens + cq - 1) / cq + num_chunks);
}

// [decode workspace of the tokens at the launch's split count][sub-sequence table, upper x 16 B]
static void varlen_sizes(int64_t num_q_tokens, int num_chunks, int num_q_heads, int num_kv_heads, int head_size,
                         int max_seqlen_k, int* upper, int* splits, int64_t* table_off) {
  const int cq = chunk_q_of(num_q_heads / num_kv_heads);
  *upper = varlen_upper(num_q_tokens, num_chunks, cq);
  *splits = qp_decode_num_splits(*upper, num_kv_heads, max_seqlen_k, 0);
  *table_off = (qp_decode_workspace_bytes(num_q_tokens, num_q_heads, head_size, *splits) + 15) / 16 * 16;
}

extern "C" int64_t qp_prefill_varlen_workspace_bytes(int64_t num_q_tokens, int num_chunks, int num_q_heads,
                                                     int num_kv_heads, int head_size, int max_seqlen_k) {
  if (num_q_tokens <= 0 || num_chunks <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads ||
      !chunk_q_of(num_q_heads / num_kv_heads))
    return 0;
  int upper = 0, splits = 0;
  int64_t off = 0;
  varlen_sizes(num_q_tokens, num_chunks, num_q_heads, num_kv_heads, head_size, max_seqlen_k, &upper, &splits, &off);
  return off + static_cast<int64_t>(upper) * 16;
}

extern "C" int qp_prefill_varlen(int fmt, int dtype, const void* q, int64_t q_stride_token, int64_t q_stride_head,
                                 void* out, int64_t out_stride_token, int64_t out_stride_head, int64_t num_q_tokens,
                                 int num_chunks, const int32_t* cu_seqlens_q, const int32_t* seqused_k,
                                 int max_seqlen_k, const int32_t* block_table, int64_t block_table_stride,
                                 const void* cache, int block_size, int64_t block_stride, int64_t head_stride,
                                 int64_t slot_stride, int64_t k_off, int64_t ks_off, int64_t v_off, int64_t vs_off,
                                 int num_q_heads, int num_kv_heads, int head_size, float softmax_scale,
                                 const uint32_t* rht_sign_bits, int q_rotated, int sliding_window, float softcap,
                                 const float* sinks, int out_mode, float* lse_out, void* workspace,
                                 int64_t workspace_bytes, void* stream) {
  int rc = decode_check_cache("prefill varlen", fmt, dtype, head_size, cache, block_size, block_stride, head_stride,
                              slot_stride, k_off, ks_off, v_off, vs_off);
  if (rc) return rc;
  if (num_chunks < 0 || num_q_tokens < 0 || num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads ||
      max_seqlen_k < 0)
    return set_error(QP_ERR_INVALID, "prefill varlen: bad sizes (chunks %d, tokens %lld, heads %d/%d)", num_chunks,
                     (long long)num_q_tokens, num_q_heads, num_kv_heads);
  if (num_chunks == 0 || num_q_tokens == 0) return QP_OK;
  if (out_mode != 0 && out_mode != 1) return set_error(QP_ERR_INVALID, "prefill varlen: out_mode %d", out_mode);
  if (sliding_window < 0) return set_error(QP_ERR_INVALID, "prefill varlen: sliding_window %d", sliding_window);
  if (!(softcap >= 0.f) || isinf(softcap)) return set_error(QP_ERR_INVALID, "prefill varlen: softcap %g", softcap);
  if (sinks && out_mode != 0)
    return set_error(QP_ERR_INVALID, "prefill varlen: sinks need out_mode 0 (a partial must not carry them)");
  const int group = num_q_heads / num_kv_heads;
  const int cq = chunk_q_of(group);
  if (!cq) return set_error(QP_ERR_UNSUPPORTED, "prefill varlen: %d query heads per KV head > %d", group, DEC_MAX_ROWS);
  if (num_q_tokens > 0x7fffffff || varlen_upper(num_q_tokens, num_chunks, cq) > 65535 || num_kv_heads > 65535)
    return set_error(QP_ERR_UNSUPPORTED, "prefill varlen: grid too large (%lld tokens, %d chunks)",
                     (long long)num_q_tokens, num_chunks);
  if (!q || !out || !cu_seqlens_q || !seqused_k || !block_table || !cache || !rht_sign_bits || !workspace)
    return set_error(QP_ERR_INVALID, "prefill varlen: null pointer");
  int upper = 0, splits = 0;
  int64_t table_off = 0;
  varlen_sizes(num_q_tokens, num_chunks, num_q_heads, num_kv_heads, head_size, max_seqlen_k, &upper, &splits,
               &table_off);
  const int64_t need = table_off + static_cast<int64_t>(upper) * 16;
  if ((reinterpret_cast<uintptr_t>(workspace) & 15) || workspace_bytes < need)
    return set_error(QP_ERR_WORKSPACE, "prefill varlen: workspace of %lld bytes < %lld", (long long)workspace_bytes,
                     (long long)need);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int4* table = reinterpret_cast<int4*>(static_cast<uint8_t*>(workspace) + table_off);
  varlen_table_kernel<<<1, 32, 0, st>>>(cu_seqlens_q, seqused_k, num_chunks, cq, upper, table);
  rc = check_launch("prefill varlen table");
  if (rc) return rc;
  DecodeParams dp{};
  dp.q = q;
  dp.q_st = q_stride_token;
  dp.q_sh = q_stride_head;
  dp.block_table = block_table;
  dp.bt_stride = block_table_stride;
  dp.cache = static_cast<const uint8_t*>(cache);
  dp.block_size = block_size;
  dp.block_stride = block_stride;
  dp.head_stride = head_stride;
  dp.nq = num_q_heads;
  dp.nkv = num_kv_heads;
  dp.group = group;
  dp.qk_scale = softmax_scale / static_cast<float>(head_size) * LOG2E;
  dp.sign_bits = rht_sign_bits;
  dp.q_rotated = q_rotated;
  dp.num_tokens = num_q_tokens;
  dp.subseq = table;
  dp.window = sliding_window >= (1 << 30) ? 0 : sliding_window;
  dp.softcap = softcap;
  dp.num_splits = splits;
  decode_bind_workspace(dp, workspace, head_size);
  rc = launch_decode(fmt, dtype, head_size, dp, cq * group, upper, st);
  if (rc) return rc;
  return merge_dispatch(decode_merge_params(dp, head_size, out_mode, out, out_stride_token, out_stride_head, lse_out,
                                          sinks),
                        dtype, head_size, num_q_tokens, st, true);
}

// ---------------------------------------------------------------------------------------------------------------
// Rank fold of a sequence split over GPUs, reading the peers' partials over NVLink (K2p). Every rank keeps its own
// partial [O (tokens, q heads, hs) fp32 | lse (tokens, q heads) base-2] in an exchange buffer that all ranks have
// mapped (symmetric memory: the same layout at `bases[r]` for rank r, this rank's own included):
//   [flags: 2 x P uint32, padded to flag_bytes][partial of parity 0][partial of parity 1]
// Call e (epoch e, parity e & 1): the kernel that wrote this rank's partial of parity e & 1 has completed (stream
// order), so CTA 0 publishes it by storing e into flag [parity][rank] of every rank (a system-scope release); each
// CTA waits (acquire, bounded) until every rank's flag [parity][r] holds e, then folds the P partials of its rows,
// read straight from the owners' buffers (plain peer loads, no multicast, no library kernel on peer memory). Two
// parities suffice: a rank writes its parity-p partial again two calls later, after its fold of the call between,
// which waited for every peer's flag of that call, which each peer stores only after its own fold of this call has
// completed. The fold: one warp per (token, query head) row, lane l holding channels [l E, l E + E), E = hs / 32
// (the layout of the warp's Hadamard transform); mode 0 applies the inverse RHT and 1 / hs and casts, mode 1 writes
// the fp32 RHT-domain output and the folded lse. Replaces the NCCL all-gather + K2 of the split (one launch, no
// host involvement); a wait that runs out records DEV_ERR_WAIT_TIMEOUT and the CTA leaves.
struct PeerFoldParams {
  const uint64_t* bases;  // [P] device address of every rank's exchange buffer
  int P, rank, parity;
  uint32_t epoch;
  int64_t part_off;       // bytes from a base to the partial of parity 0
  int64_t part_bytes;     // bytes of one partial (the parity stride)
  int64_t rows;           // tokens x q heads
  int nq, mode;
  void* out;
  int64_t out_st, out_sh;
  float* lse_out;
  const uint32_t* sign_bits;
  float out_scale;
};

constexpr int PF_FOLD_WARPS = 8;
constexpr int PEER_MAX = 32;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <int DT, int HS>
__global__ void __launch_bounds__(32 * PF_FOLD_WARPS) peer_fold_kernel(const PeerFoldParams p) {
  constexpr int E = HS / 32;
  const int lane = threadIdx.x & 31;
  if (blockIdx.x == 0 && threadIdx.x < p.P) {  // publish this rank's partial to every rank
    __threadfence_system();
    uint32_t* f = reinterpret_cast<uint32_t*>(p.bases[threadIdx.x]) + p.parity * p.P + p.rank;
    st_release_sys(f, p.epoch);
  }
  bool ok = true;
  if (threadIdx.x < p.P && threadIdx.x != p.rank) {  // every peer's partial of this call is published
    const uint32_t* f = reinterpret_cast<const uint32_t*>(p.bases[p.rank]) + p.parity * p.P + threadIdx.x;
    if (ld_acquire_sys(f) != p.epoch) {
      const uint64_t t0 = global_timer_ns();
      while (ld_acquire_sys(f) != p.epoch) {
        if (global_timer_ns() - t0 > 2000000000ull) {
          atomicCAS(&g_device_error, DEV_ERR_NONE, DEV_ERR_WAIT_TIMEOUT);
          ok = false;
          break;
        }
      }
    }
  }
  if (__syncthreads_or(!ok)) return;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * PF_FOLD_WARPS + (threadIdx.x >> 5);  // token * nq + head
  if (r >= p.rows) return;
  const int64_t lse_off = p.part_off + p.parity * p.part_bytes + p.rows * HS * 4;
  const int64_t o_off = p.part_off + p.parity * p.part_bytes + r * HS * 4;
  const float l_me = lane < p.P ? *reinterpret_cast<const float*>(p.bases[lane] + lse_off + r * 4) : -INFINITY;
  const float M = warp_max(l_me);
  const float w_me = (M == -INFINITY || l_me == -INFINITY) ? 0.f : exp2f(l_me - M);
  const float T = warp_sum(w_me);
  float x[E];
#pragma unroll
  for (int i = 0; i < E; ++i) x[i] = 0.f;
  for (int s = 0; s < p.P; ++s) {
    const float w = __shfl_sync(0xffffffffu, w_me, s);
    if (w != 0.f) {  // the same in every lane; a rank with no key for the row contributes nothing
      const float4* po = reinterpret_cast<const float4*>(p.bases[s] + o_off) + lane * (E / 4);
#pragma unroll
      for (int i = 0; i < E / 4; ++i) {
        const float4 a = po[i];
        x[4 * i] = fmaf(w, a.x, x[4 * i]);
        x[4 * i + 1] = fmaf(w, a.y, x[4 * i + 1]);
        x[4 * i + 2] = fmaf(w, a.z, x[4 * i + 2]);
        x[4 * i + 3] = fmaf(w, a.w, x[4 * i + 3]);
      }
    }
  }
  const float inv = T > 0.f ? 1.f / T : 0.f;
#pragma unroll
  for (int i = 0; i < E; ++i) x[i] *= inv;
  const int64_t tok = r / p.nq;
  const int qh = static_cast<int>(r % p.nq);
  if (p.mode == 1) {
    float* dst = reinterpret_cast<float*>(p.out) + tok * p.out_st + qh * p.out_sh + E * lane;
#pragma unroll
    for (int i = 0; i < E; ++i) dst[i] = x[i];
    if (lane == 0 && p.lse_out) p.lse_out[r] = T > 0.f ? M + log2f(T) : -INFINITY;
    return;
  }
  warp_wht<E>(x, lane);
  apply_signs<E>(x, p.sign_bits, lane);
  using EL = Elem<DT>;
  typename EL::T* dst = reinterpret_cast<typename EL::T*>(p.out) + tok * p.out_st + qh * p.out_sh + E * lane;
#pragma unroll
  for (int i = 0; i < E; ++i) dst[i] = EL::from_f(x[i] * p.out_scale);
}

// Bytes of a rank's exchange buffer for K2p: flags (2 x P uint32, padded to 256 bytes) and two partials.
static int64_t peer_flag_bytes(int P) { return (2 * static_cast<int64_t>(P) * 4 + 255) / 256 * 256; }
static int64_t peer_part_bytes(int64_t num_tokens, int nq, int hs) {
  const int64_t rows = num_tokens * nq;
  return (rows * hs * 4 + rows * 4 + 255) / 256 * 256;
}

extern "C" int64_t qp_peer_exchange_bytes(int num_ranks, int64_t num_tokens, int num_q_heads, int head_size) {
  if (num_ranks <= 0 || num_tokens < 0 || num_q_heads <= 0) return 0;
  return peer_flag_bytes(num_ranks) + 2 * peer_part_bytes(num_tokens, num_q_heads, head_size);
}

extern "C" int64_t qp_peer_partial_offset(int num_ranks, int64_t num_tokens, int num_q_heads, int head_size,
                                          int parity) {
  return peer_flag_bytes(num_ranks) + (parity & 1) * peer_part_bytes(num_tokens, num_q_heads, head_size);
}

extern "C" int qp_fold_peer_partials(int dtype, int head_size, int64_t num_tokens, int num_q_heads, int num_ranks,
                                     int rank, const uint64_t* bases, uint32_t epoch, int out_mode, void* out,
                                     int64_t out_stride_token, int64_t out_stride_head, float* lse_out,
                                     const uint32_t* rht_sign_bits, void* stream) {
  if (num_tokens < 0 || num_q_heads <= 0 || num_ranks <= 0 || rank < 0 || rank >= num_ranks)
    return set_error(QP_ERR_INVALID, "fold peers: bad sizes");
  if (num_ranks > PEER_MAX) return set_error(QP_ERR_UNSUPPORTED, "fold peers: %d ranks > %d", num_ranks, PEER_MAX);
  if (head_size != 256 && head_size != 512 && head_size != 128)
    return set_error(QP_ERR_UNSUPPORTED, "fold peers: head size %d", head_size);
  if (out_mode != 0 && out_mode != 1) return set_error(QP_ERR_INVALID, "fold peers: out_mode %d", out_mode);
  if (out_mode == 0 && dtype != DT_BF16 && dtype != DT_F16) return set_error(QP_ERR_UNSUPPORTED, "fold peers: dtype");
  if (!bases || !out || (out_mode == 0 && !rht_sign_bits)) return set_error(QP_ERR_INVALID, "fold peers: null pointer");
  if (num_tokens == 0) return QP_OK;
  PeerFoldParams fp{};
  fp.bases = bases;
  fp.P = num_ranks;
  fp.rank = rank;
  fp.parity = static_cast<int>(epoch & 1u);
  fp.epoch = epoch;
  fp.part_off = peer_flag_bytes(num_ranks);
  fp.part_bytes = peer_part_bytes(num_tokens, num_q_heads, head_size);
  fp.rows = num_tokens * num_q_heads;
  fp.nq = num_q_heads;
  fp.mode = out_mode;
  fp.out = out;
  fp.out_st = out_stride_token;
  fp.out_sh = out_stride_head;
  fp.lse_out = lse_out;
  fp.sign_bits = rht_sign_bits;
  fp.out_scale = 1.f / static_cast<float>(head_size);
  const int64_t grid = (fp.rows + PF_FOLD_WARPS - 1) / PF_FOLD_WARPS;
  if (grid > 0x7fffffff) return set_error(QP_ERR_UNSUPPORTED, "fold peers: too many rows");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 g(static_cast<unsigned>(grid)), b(32 * PF_FOLD_WARPS);
  const bool bf = out_mode == 1 || dtype == DT_BF16;
  switch (head_size) {
    case 128: if (bf) peer_fold_kernel<DT_BF16, 128><<<g, b, 0, st>>>(fp); else peer_fold_kernel<DT_F16, 128><<<g, b, 0, st>>>(fp); break;
    case 256: if (bf) peer_fold_kernel<DT_BF16, 256><<<g, b, 0, st>>>(fp); else peer_fold_kernel<DT_F16, 256><<<g, b, 0, st>>>(fp); break;
    default: if (bf) peer_fold_kernel<DT_BF16, 512><<<g, b, 0, st>>>(fp); else peer_fold_kernel<DT_F16, 512><<<g, b, 0, st>>>(fp); break;
  }
  return check_launch("fold peers");
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
//   zero (each call writes every partial and query row it later reads), but calls that overlap on the GPU (two
//   streams, two host threads) race on it: serialize them.
// - The array holds the split partials and the prepared query rows (qp_decode_workspace_bytes); sizes that need
//   more are rejected with QP_ERR_WORKSPACE.
// - Only out_mode 0 and 1 are served (out_mode 2 would leave the partials where no caller can reach them), and the
//   causal mask assumes the keys given are the sequence's last ones (tokens_after_keys = 0): an ordinary single-GPU
//   decode, not a sequence-parallel rank holding an earlier range.
static constexpr int64_t kStaticDecodeScratchBytes = 32ll << 20;
static __device__ __align__(256) uint8_t g_static_decode_scratch[kStaticDecodeScratchBytes];
static std::atomic<void*> g_static_decode_scratch_addr[64];

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
  if (out_mode != 0 && out_mode != 1)
    return set_error(QP_ERR_INVALID, "decode (static scratch): out_mode %d (0 or 1: the partials stay private)",
                     out_mode);
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
  void* scratch = g_static_decode_scratch_addr[dev].load(std::memory_order_acquire);
  if (scratch == nullptr) {
    // two host threads may both look it up the first time; they store the same address
    e = cudaGetSymbolAddress(&scratch, g_static_decode_scratch);
    if (e != cudaSuccess || scratch == nullptr)
      return set_error(QP_ERR_CUDA, "decode (static scratch): cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_static_decode_scratch_addr[dev].store(scratch, std::memory_order_release);
  }
  return qp_paged_decode(fmt, dtype, q, q_stride_token, q_stride_head, out, out_stride_token, out_stride_head,
                         num_q_tokens, num_seqs, cu_seqlens_q, seqused_k, max_seqlen_q, block_table,
                         block_table_stride, cache, block_size, block_stride, head_stride, slot_stride, k_off, ks_off,
                         v_off, vs_off, num_q_heads, num_kv_heads, head_size, softmax_scale, rht_sign_bits, q_rotated,
                         0, 0, 0.f, nullptr, out_mode, lse_out, num_splits, scratch, kStaticDecodeScratchBytes,
                         stream);
}
