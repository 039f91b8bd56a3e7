/* quantpack_b200: B200-native (sm_100a) quantized KV-cache attention, C ABI.
 *
 * Replaces the hot path of the vLLM plugin jramirez-uab/vllm-quantpack 0.1.8: the int4_per_token_head and
 * k8v4_per_token_head cache write, split-KV paged decode with up to 4 MTP query tokens (with vLLM's sliding window,
 * logit softcap and attention sinks where a layer has them), long-chunk prefill, the short chunks of a step in one
 * launch and the log-sum-exp merge of attention partials. The reference's hot path is Python calling Triton
 * kernels; each entry point below names the reference function it stands in for (paths inside the reference
 * project).
 *
 * Conventions for every function:
 * - all pointers are device pointers unless stated; `stream` is a cudaStream_t (NULL = legacy default stream);
 * - calls are asynchronous on `stream` and never allocate or synchronize (qp_device_error excepted);
 * - return 0 on success, a QP_ERR_* code otherwise, with a message in qp_last_error() (thread-local);
 * - `dtype` is QP_DTYPE_BF16 or QP_DTYPE_F16 (the model dtype of keys, values, queries and outputs);
 * - strides are in elements for model-dtype tensors and in bytes for the cache;
 * - cache cell of (block b, KV head h, slot s) at cache + b*block_stride + h*head_stride + s*slot_stride, with the
 *   fields at k_off (key codes), ks_off (key scale word), v_off (value nibbles), vs_off (value scale word):
 *     int4: [K hs/2 | K scale f32 | V hs/2 | V scale f32]    (tests/test_int4_kv.py:95-103)
 *     k8v4: [K hs int8 | K scale f32 | V hs/2 | V scale f32]  (vllm_quantpack/attention/k8v4_kv.py:10-11, 41-65)
 *   An int4 scale word carries the 4-bit zero point in its low mantissa bits; low nibble = even channel.
 * - rht_sign_bits: head_size/32 uint32 words, bit i set where the randomized-Hadamard sign d_i is -1.
 */
#ifndef QUANTPACK_B200_H
#define QUANTPACK_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QP_DTYPE_BF16 0
#define QP_DTYPE_F16 1
#define QP_FMT_INT4 0
#define QP_FMT_K8V4 1

#define QP_OK 0
#define QP_ERR_INVALID 1
#define QP_ERR_UNSUPPORTED 2
#define QP_ERR_LAYOUT 3
#define QP_ERR_WORKSPACE 4
#define QP_ERR_CUDA 5

/* Library version (100 = 1.0.0). No counterpart in the reference (a Python package). */
int qp_version(void);

/* Message of the last failed call on this thread. No counterpart in the reference (Python exceptions). */
const char* qp_last_error(void);

/* Reads and clears the device error word of the current device (synchronous): *code != 0 when a kernel gave up a
 * bounded wait (it then returned early instead of hanging). No counterpart in the reference (its Triton kernels
 * have no waits). */
int qp_device_error(int* code);

/* int4_per_token_head cache write: y = RHT(x) rounded to dtype, then per (token, KV head) asymmetric 4-bit codes
 * with an fp32 scale carrying the zero point, for keys and values. Tokens with slot_mapping[t] < 0 are skipped.
 * rotate = 0 takes key / value as already rotated (the contract of the reference's `_store_k8v4` kernel, whose
 * `store` wrapper rotates first).
 * Replaces the stock vLLM `reshape_and_cache_int4(key, value, key_cache, value_cache, slot_mapping, *,
 * k_scale_cache, v_scale_cache)` that the plugin calls at vllm_quantpack/attention/k8v4_kv.py:152-155 (and the
 * tests at tests/test_int4_kv.py:112); the quantizer is the one of vllm_quantpack/attention/k8v4_ops.py:44-63. */
int qp_reshape_and_cache_int4(const void* key, const void* value, int dtype, int64_t num_tokens, int num_kv_heads,
                              int head_size, int64_t key_stride_token, int64_t key_stride_head,
                              int64_t value_stride_token, int64_t value_stride_head, const int64_t* slot_mapping,
                              void* cache, int block_size, int64_t block_stride, int64_t head_stride,
                              int64_t slot_stride, int64_t k_off, int64_t ks_off, int64_t v_off, int64_t vs_off,
                              const uint32_t* rht_sign_bits, int rotate, void* stream);

/* k8v4_per_token_head cache write: keys int8 with scale absmax/127, values as int4, both after the RHT.
 * Replaces vllm_quantpack/attention/k8v4_kv.py:68-86 (`store`: single_rht + `_store_k8v4`,
 * vllm_quantpack/attention/k8v4_ops.py:10-63). Same arguments as qp_reshape_and_cache_int4. */
int qp_reshape_and_cache_k8v4(const void* key, const void* value, int dtype, int64_t num_tokens, int num_kv_heads,
                              int head_size, int64_t key_stride_token, int64_t key_stride_head,
                              int64_t value_stride_token, int64_t value_stride_head, const int64_t* slot_mapping,
                              void* cache, int block_size, int64_t block_stride, int64_t head_stride,
                              int64_t slot_stride, int64_t k_off, int64_t ks_off, int64_t v_off, int64_t vs_off,
                              const uint32_t* rht_sign_bits, int rotate, void* stream);

/* Randomized Hadamard transform of `rows` fp32 rows of head_size: forward y = H (d * x), inverse x = d * (H y),
 * unnormalised. Replaces the stock `single_rht(x, inverse=False)` called at vllm_quantpack/attention/int4_kv.py:326,
 * 329 and k8v4_kv.py:71-72. x and y may alias. */
int qp_single_rht(const float* x, float* y, int64_t rows, int head_size, int inverse, const uint32_t* rht_sign_bits,
                  void* stream);

/* Split-KV count the decode uses for a batch on a GPU with sm_count SMs (<= 0: the current device's). Stands in for
 * `segments_for` / `decode_tiles` (vllm_quantpack/attention/int4_kv.py:66-78). */
int qp_decode_num_splits(int num_seqs, int num_kv_heads, int max_seqlen_k, int sm_count);

/* Bytes of workspace qp_paged_decode needs (the split-KV partials). Stands in for the segment buffers vLLM's
 * metadata builder allocates (vllm_quantpack/attention/int4_kv.py:229-257). */
int64_t qp_decode_workspace_bytes(int64_t num_q_tokens, int num_q_heads, int head_size, int num_splits);

/* Split-KV paged decode: for every sequence b, query tokens cu_seqlens_q[b] .. cu_seqlens_q[b+1]-1 (the last ones
 * of a context of seqused_k[b] tokens, causal among themselves) attend to the cached context through
 * block_table[b]. q (tokens, num_q_heads, head_size) in dtype; out likewise. max_seqlen_q * (num_q_heads /
 * num_kv_heads) <= 32. The RHT is applied to q (unless q_rotated) and inverted on the output, which is divided by
 * head_size; scores use softmax_scale / head_size (vllm_quantpack/attention/int4_kv.py:326-329).
 * tokens_after_keys: tokens of every sequence that follow its seqused_k cached keys here (a sequence-parallel rank
 * holding an earlier range of the sequence): query token i then sees key k iff k <= seqused_k - qlen + i +
 * tokens_after_keys; 0 for an ordinary call, >= qlen - 1 lifts the causal mask.
 * sliding_window: vLLM's SLIDING_WINDOW (1 + window_size[0]; 0 = none): query token i whose last visible key is p
 * sees the keys [p - sliding_window + 1, p] only, as the stock kernel masks them (vllm/v1/attention/ops/
 * triton_attention_helpers.py:196-218 and triton_unified_attention.py:533-536, vLLM 0.22); the splits then cover
 * only the tiles of the window, so num_splits should come from min(context, window + max_seqlen_q + 127).
 * softcap: vLLM's logit softcap (0 = none): every score S = softmax_scale / head_size x q.k becomes
 * softcap x tanh(S / softcap) before the softmax (vllm/v1/attention/ops/triton_attention_helpers.py:28-36,
 * triton_unified_attention.py:513-514, vLLM 0.22).
 * sinks: null, or num_q_heads fp32 sink logits (natural units, out_mode 0 only): exp(sink) joins every row's softmax
 * denominator once, as vLLM's attention sinks (triton_attention_helpers.py:108-138: the row maximum starts at the
 * sink with sum 1, in one segment only).
 * out_mode 0: out in dtype, model domain. out_mode 1: out fp32 in the RHT domain and lse_out (tokens, num_q_heads)
 * the base-2 log-sum-exp of the scaled scores (the partial a sequence-parallel rank exchanges). out_mode 2: the
 * split partials only, left in the workspace as part_o (tokens, num_q_heads, num_splits, head_size) fp32 followed by
 * part_lse (tokens, num_q_heads, num_splits) base-2, for a caller that folds them with qp_merge_attn_partials.
 * Replaces the plugin's split-KV decode: the patched `_launch_packed_attn` (int4_kv.py:98-122, 212-216) with its 3D
 * kernel `_attn_packed_qp` / `_attn_k8v4_qp` (int4_kv.py:80-146) and vLLM's reduce_segments, reached through
 * `unified_attention_int4` (int4_kv.py:294-307). Needs HND cells (slot_stride == cell bytes), block_size % 16 == 0,
 * head_size 256 or 512, a 16-byte aligned cache and qp_decode_workspace_bytes() of workspace. */
int qp_paged_decode(int fmt, int dtype, const void* q, int64_t q_stride_token, int64_t q_stride_head, void* out,
                    int64_t out_stride_token, int64_t out_stride_head, int64_t num_q_tokens, int num_seqs,
                    const int32_t* cu_seqlens_q, const int32_t* seqused_k, int max_seqlen_q,
                    const int32_t* block_table, int64_t block_table_stride, const void* cache, int block_size,
                    int64_t block_stride, int64_t head_stride, int64_t slot_stride, int64_t k_off, int64_t ks_off,
                    int64_t v_off, int64_t vs_off, int num_q_heads, int num_kv_heads, int head_size,
                    float softmax_scale, const uint32_t* rht_sign_bits, int q_rotated, int tokens_after_keys,
                    int sliding_window, float softcap, const float* sinks, int out_mode, float* lse_out,
                    int num_splits, void* workspace, int64_t workspace_bytes, void* stream);

/* Bytes of workspace qp_prefill needs for a chunk of qlen queries over a context of n tokens (prepared query tiles
 * and per-piece partials). */
int64_t qp_prefill_workspace_bytes(int qlen, int n, int num_q_heads, int num_kv_heads, int head_size,
                                   int tokens_after_keys);

/* Long-chunk prefill of one sequence: the qlen queries q (the last qlen positions of a context of n tokens, causal
 * among themselves) attend to the whole cached context through block_row (that sequence's block-table row), on the
 * tcgen05 tensor cores with every key / value tile dequantised in shared memory (no scratch unpack of the cache).
 * out_mode / lse_out / q_rotated / tokens_after_keys as in qp_paged_decode (n >= qlen - tokens_after_keys);
 * head_size 256, or 512 (there the chunk runs on the split-KV decode kernel as decodes of 32 / (query heads per KV
 * head) tokens over its causal prefixes: O of a 128-query tile alone would fill TMEM); HND cells,
 * block_size % 16 == 0.
 * Replaces vllm_quantpack/attention/int4_prefill.py:203-232 `prefill_sequence` (16k-token bf16 unpacks +
 * FlashAttention 2 + log-sum-exp fold) and the Triton 2D path of int4_kv.py:113-119, reached through
 * `unified_attention_int4` (int4_kv.py:308-329). */
int qp_prefill(int fmt, int dtype, const void* q, int64_t q_stride_token, int64_t q_stride_head, void* out,
               int64_t out_stride_token, int64_t out_stride_head, int qlen, int n, const int32_t* block_row,
               const void* cache, int block_size, int64_t block_stride, int64_t head_stride, int64_t slot_stride,
               int64_t k_off, int64_t ks_off, int64_t v_off, int64_t vs_off, int num_q_heads, int num_kv_heads,
               int head_size, float softmax_scale, const uint32_t* rht_sign_bits, int q_rotated,
               int tokens_after_keys, int out_mode, float* lse_out, void* workspace, int64_t workspace_bytes,
               void* stream);

/* Bytes of workspace qp_prefill_varlen needs (its split partials, prepared query rows and sub-sequence table). */
int64_t qp_prefill_varlen_workspace_bytes(int64_t num_q_tokens, int num_chunks, int num_q_heads, int num_kv_heads,
                                          int head_size, int max_seqlen_k);

/* Short prefill chunks of several sequences in one launch: chunk i's query tokens q[cu_seqlens_q[i] ..
 * cu_seqlens_q[i + 1]) are the last positions of its context of seqused_k[i] cached tokens (causal among themselves),
 * read through block_table[i]; cu_seqlens_q / seqused_k are device int32 arrays (num_chunks + 1 / num_chunks) that
 * the call never reads back to the host. max_seqlen_k bounds the keys any query token sees (seqused_k, or with a
 * sliding window min(seqused_k, sliding_window + 158)); it sizes the split count and the workspace. The chunks run
 * on the split-KV decode kernel as sub-sequences of 32 / (query heads per KV head) tokens. out / out_mode / lse_out /
 * q_rotated / sliding_window / softcap / sinks as in qp_paged_decode (out_mode 0 or 1); head_size 256 or 512; HND cells,
 * block_size % 16 == 0.
 * Replaces the Triton 2D sub-batch that the plugin runs for every chunk that is not long (int4_kv.py:113-119,
 * 313-323). */
int qp_prefill_varlen(int fmt, int dtype, const void* q, int64_t q_stride_token, int64_t q_stride_head, void* out,
                      int64_t out_stride_token, int64_t out_stride_head, int64_t num_q_tokens, int num_chunks,
                      const int32_t* cu_seqlens_q, const int32_t* seqused_k, int max_seqlen_k,
                      const int32_t* block_table, int64_t block_table_stride, const void* cache, int block_size,
                      int64_t block_stride, int64_t head_stride, int64_t slot_stride, int64_t k_off, int64_t ks_off,
                      int64_t v_off, int64_t vs_off, int num_q_heads, int num_kv_heads, int head_size,
                      float softmax_scale, const uint32_t* rht_sign_bits, int q_rotated, int sliding_window,
                      float softcap, const float* sinks, int out_mode, float* lse_out, void* workspace,
                      int64_t workspace_bytes, void* stream);

/* Bytes of the library's static decode scratch used by qp_paged_decode_static. */
#define QP_STATIC_DECODE_SCRATCH_BYTES (32ll << 20)

/* qp_paged_decode without a workspace argument, for callers that cannot allocate device memory (an engine that owns
 * every byte of device memory in its own pool, embedded code with no device allocator). The split partials go to a
 * fixed 32 MiB array inside the library, reserved on every GPU that loads it until the process exits; calls whose
 * partials (qp_decode_workspace_bytes) exceed it return QP_ERR_WORKSPACE. The first call on a device looks the array
 * up (cudaGetSymbolAddress) with that device current: make it before any stream capture. All calls on a device share
 * the array and it keeps the last call's contents (nothing in it needs to start at zero); calls that overlap on the
 * GPU race on it, so serialize them. The array holds the split partials and the prepared query rows. Only out_mode 0
 * and 1 are served (QP_ERR_INVALID for 2: the partials would stay where no caller can reach them), and the keys are
 * taken as the sequence's last ones (tokens_after_keys 0) with no sliding window, softcap or sinks: a single-GPU
 * decode, not a rank of a sequence split.
 * Allocates nothing. No counterpart in the reference. */
int qp_paged_decode_static(int fmt, int dtype, const void* q, int64_t q_stride_token, int64_t q_stride_head,
                           void* out, int64_t out_stride_token, int64_t out_stride_head, int64_t num_q_tokens,
                           int num_seqs, const int32_t* cu_seqlens_q, const int32_t* seqused_k, int max_seqlen_q,
                           const int32_t* block_table, int64_t block_table_stride, const void* cache, int block_size,
                           int64_t block_stride, int64_t head_stride, int64_t slot_stride, int64_t k_off,
                           int64_t ks_off, int64_t v_off, int64_t vs_off, int num_q_heads, int num_kv_heads,
                           int head_size, float softmax_scale, const uint32_t* rht_sign_bits, int q_rotated,
                           int out_mode, float* lse_out, int num_splits, void* stream);

/* Bytes of one rank's exchange buffer for qp_fold_peer_partials (num_ranks flags per parity, two partials), and the
 * offset of its partial of a parity ([O (tokens, q heads, hs) fp32 | lse (tokens, q heads) fp32 base-2]). */
int64_t qp_peer_exchange_bytes(int num_ranks, int64_t num_tokens, int num_q_heads, int head_size);
int64_t qp_peer_partial_offset(int num_ranks, int64_t num_tokens, int num_q_heads, int head_size, int parity);

/* Rank fold of a sequence split over GPUs without a collective: every rank has written its partial of call `epoch`
 * (out_mode 1 of qp_paged_decode / qp_prefill) at qp_peer_partial_offset(..., epoch & 1) of its own exchange buffer,
 * and bases (a device array of num_ranks addresses) holds every rank's buffer as mapped here (NVLink peer memory,
 * e.g. torch symmetric memory; the flags zeroed before the first call, epochs counting up from 1). The kernel
 * publishes this rank's partial through a flag in every buffer, waits (bounded: QP device error on timeout) for the
 * other ranks' flags and folds the num_ranks partials read over NVLink into `out` (out_mode 0: model domain in dtype;
 * 1: fp32 RHT domain + lse_out). Replaces the NCCL all-gather + qp_merge_attn_partials of the split; no counterpart
 * in the reference (which serves one GPU). */
int qp_fold_peer_partials(int dtype, int head_size, int64_t num_tokens, int num_q_heads, int num_ranks, int rank,
                          const uint64_t* bases, uint32_t epoch, int out_mode, void* out, int64_t out_stride_token,
                          int64_t out_stride_head, float* lse_out, const uint32_t* rht_sign_bits, void* stream);

/* Log-sum-exp fold of num_parts attention partials per (token, query head): part_o fp32 (RHT domain, normalised),
 * part_lse base-2. out_mode 0: inverse RHT / head_size into `out` in dtype; out_mode 1: fp32 RHT-domain O into
 * `out` and the folded lse into lse_out. Replaces the fold of vllm_quantpack/attention/int4_prefill.py:223-230 and
 * vLLM's reduce_segments (vllm/v1/attention/ops/triton_unified_attention.py:645-732, vLLM 0.22); also the merge of a
 * sequence split over ranks. */
int qp_merge_attn_partials(int dtype, int head_size, int64_t num_tokens, int num_q_heads, int num_parts,
                           const float* part_o, int64_t po_stride_token, int64_t po_stride_head,
                           int64_t po_stride_part, const float* part_lse, int64_t pl_stride_token,
                           int64_t pl_stride_head, int64_t pl_stride_part, int out_mode, void* out,
                           int64_t out_stride_token, int64_t out_stride_head, float* lse_out,
                           const uint32_t* rht_sign_bits, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QUANTPACK_B200_H */
