"""Long-context prefill over the packed int4 / k8v4 KV cache, on the B200 tensor cores.

Mirrors the plugin module vllm_quantpack/attention/int4_prefill.py: the same routing thresholds and the same
`prefill_sequence` contract (queries already RHT-rotated, output in the RHT domain in the queries' dtype). The
reference unpacks the cache to bf16 in 16k-token segments and runs FlashAttention 2 over each, folding them by
log-sum-exp; here one tcgen05 kernel (csrc/qp_prefill.cu) reads the packed cells once, dequantises each 64-key tile
in shared memory and accumulates in TMEM, with no scratch segment. SEGMENT is kept only as a name callers may read.
"""
import torch

from . import ops

MAX_HEAD = 256       # largest head size of the B200 prefill kernel (the reference's FlashAttention limit too)
SEGMENT = 16384      # the reference's unpack segment; the B200 kernel needs no scratch segment
MIN_QUERY = 64       # chunks at least this long count as long prefills (int4_prefill.py:21)
MIN_CONTEXT = 8192   # with at least this much context (int4_prefill.py:22)


def prefill_sequence(q_rot, k_cache, v_cache, k_scales, v_scales, block_row, n, softmax_scale, fa=None):
    """Attention of q_rot (the chunk's queries, RHT-rotated, the last len(q_rot) positions of a context of n tokens)
    over the whole cached context; returns the RHT-domain output in q_rot's dtype.

    softmax_scale is the scale applied to the rotated dot products (the caller passes softmax_scale / head, as
    vllm_quantpack/attention/int4_kv.py:327-328 does). `fa` (the reference's FlashAttention function) is accepted
    and unused. Replaces int4_prefill.py:203-232."""
    qlen, nq, hs = q_rot.shape
    out = torch.empty((qlen, nq, hs), dtype=torch.float32, device=q_rot.device)
    lse = torch.empty((qlen, nq), dtype=torch.float32, device=q_rot.device)
    if block_row.dtype != torch.int32:
        block_row = block_row.to(torch.int32)
    ops.prefill(q_rot, k_cache, v_cache, out, block_row=block_row.contiguous(), n=int(n),
                softmax_scale=float(softmax_scale) * hs, k_scale_cache=k_scales, v_scale_cache=v_scales,
                q_rotated=True, out_fp32_lse=lse)
    return out.to(q_rot.dtype)


def prefill_sequence_i8(q_rot, k_cache, v_cache, k_scales, v_scales, block_row, n, softmax_scale):
    """The reference's single-kernel prefill (int4_prefill.py:95-200) has the same contract; on B200 it is the same
    tensor-core kernel as prefill_sequence."""
    return prefill_sequence(q_rot, k_cache, v_cache, k_scales, v_scales, block_row, n, softmax_scale)
