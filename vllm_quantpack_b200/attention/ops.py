"""B200 ops behind the plugin's patch points: cache write, split-KV decode, RHT and partial merge.

These are the functions the stock vLLM int4 module (`vllm.v1.attention.ops.int4_per_token_head`, vLLM >= 0.31)
exposes and the plugin patches (vllm_quantpack/attention/int4_kv.py:39, 212-216, 294-333;
vllm_quantpack/attention/k8v4_kv.py:152-163), with the same names, arguments and tensor views, each one a thin
launch of a CUDA kernel of libquantpack_b200.so on the current stream. There is no CPU path: on a machine without
the library or a GPU every op raises.
"""
import threading

import torch

from .. import _lib
from . import rht

_DTYPES = {torch.bfloat16: 0, torch.float16: 1}
FMT_INT4, FMT_K8V4 = 0, 1
MAX_Q_DECODE_ROWS = 32      # query rows (tokens x query heads per KV head) one decode CTA holds


def _stream(device):
    return torch.cuda.current_stream(device).cuda_stream


def _sinks_ptr(sinks, nq, mode):
    """Device pointer of fp32 sink logits (one per query head), or None. Sinks count once in a row's softmax, so
    only the model-domain output (mode 0) can take them, never a partial."""
    if sinks is None:
        return None
    if mode != 0:
        raise ValueError("sinks apply to the model-domain output only, not to partials")
    if sinks.dim() != 1 or sinks.shape[0] != nq:
        raise ValueError(f"sinks must have one logit per query head ({nq}), got {tuple(sinks.shape)}")
    if sinks.dtype != torch.float32 or not sinks.is_contiguous():
        # a temporary on the current stream: torch's caching allocator hands its memory to a later allocation only
        # in stream order, after the merge kernel that reads it
        sinks = sinks.float().contiguous()
    return sinks.data_ptr()


def _dtype_code(t, what):
    code = _DTYPES.get(t.dtype)
    if code is None:
        raise TypeError(f"{what}: dtype {t.dtype} (bf16 or fp16 expected)")
    return code


class CacheLayout:
    """Byte layout of a paged int4 / k8v4 cache, derived from the four views vLLM passes (`of` keeps the layouts it
    derived, keyed by everything they are derived from, so a call on the same cache pays for the checks once).

    int4 views (tests/test_int4_kv.py:95-103): key / value (blocks, block size, KV heads, hs/2 + 4) uint8 over cells
    [K | K scale | V | V scale]; k8v4 views (vllm_quantpack/attention/k8v4_kv.py:41-65): key (..., hs) int8, value
    (..., hs/2) uint8. Scale views are fp32 (blocks, block size, KV heads) over the same storage."""

    def __init__(self, k_cache, v_cache, k_scale_cache, v_scale_cache, head_size):
        if k_cache.dtype == torch.int8:
            self.fmt, kb = FMT_K8V4, head_size
        elif k_cache.dtype == torch.uint8:
            self.fmt, kb = FMT_INT4, head_size // 2
        else:
            raise TypeError(f"key cache dtype {k_cache.dtype}: uint8 (int4) or int8 (k8v4) expected")
        if k_cache.dim() != 4 or v_cache.dim() != 4:
            raise ValueError("cache views must be (blocks, block size, KV heads, bytes)")
        self.nblocks, self.block_size, self.nkv = k_cache.shape[0], k_cache.shape[1], k_cache.shape[2]
        self.head_size = head_size
        base = k_cache.data_ptr()
        self.base = base
        self.block_stride, self.slot_stride, self.head_stride = (int(s) for s in k_cache.stride()[:3])
        self.k_off = 0
        self.ks_off = k_scale_cache.data_ptr() - base
        self.v_off = v_cache.data_ptr() - base
        self.vs_off = v_scale_cache.data_ptr() - base
        self.cell = kb + 8 + head_size // 2
        if (tuple(v_cache.stride()[:3]) != (self.block_stride, self.slot_stride, self.head_stride)
                or tuple(v_cache.shape[:3]) != tuple(k_cache.shape[:3])):
            raise ValueError("key and value cache views disagree on blocks / slots / heads")
        for sc in (k_scale_cache, v_scale_cache):
            if sc.dtype != torch.float32 or tuple(sc.shape) != (self.nblocks, self.block_size, self.nkv):
                raise ValueError("scale views must be fp32 (blocks, block size, KV heads)")
            if tuple(4 * s for s in sc.stride()) != (self.block_stride, self.slot_stride, self.head_stride):
                raise ValueError("scale views must share the cache's strides")
        if self.ks_off != kb or self.v_off != kb + 4 or self.vs_off != kb + 4 + head_size // 2:
            raise ValueError(f"cell fields at K 0, K scale {self.ks_off}, V {self.v_off}, V scale {self.vs_off}: "
                             f"expected 0, {kb}, {kb + 4}, {kb + 4 + head_size // 2}")

    _known = {}

    @classmethod
    def of(cls, k_cache, v_cache, k_scale_cache, v_scale_cache, head_size):
        """The layout of these views: a derived one when every input to the derivation (addresses, dtypes, shapes,
        strides, head size) matches, else a new one (checked; only valid layouts are kept)."""
        key = (k_cache.data_ptr(), v_cache.data_ptr(), k_scale_cache.data_ptr(), v_scale_cache.data_ptr(),
               k_cache.dtype, v_cache.dtype, k_scale_cache.dtype, v_scale_cache.dtype, k_cache.shape, v_cache.shape,
               k_scale_cache.shape, v_scale_cache.shape, k_cache.stride(), v_cache.stride(), k_scale_cache.stride(),
               v_scale_cache.stride(), head_size)
        lay = cls._known.get(key)
        if lay is None:
            lay = cls(k_cache, v_cache, k_scale_cache, v_scale_cache, head_size)
            if len(cls._known) >= 256:
                cls._known.clear()
            cls._known[key] = lay
        return lay

    def args(self):
        return (self.base, self.block_size, self.block_stride, self.head_stride, self.slot_stride, self.k_off,
                self.ks_off, self.v_off, self.vs_off)

    @property
    def hnd(self):
        return self.slot_stride == self.cell


# ------------------------------------------------------------------------------------------------------ RHT


def single_rht(x, inverse=False):
    """Randomized Hadamard transform over the last axis of fp32 `x` (unnormalised; see rht.py). Returns fp32."""
    if x.dtype != torch.float32:
        raise TypeError("single_rht takes fp32 (as the callers pass x.float())")
    hs = x.shape[-1]
    xc = x.contiguous()
    y = torch.empty_like(xc)
    rows = xc.numel() // hs if hs else 0
    _lib.call("qp_single_rht", xc.data_ptr(), y.data_ptr(), rows, hs, int(bool(inverse)),
              rht.device_sign_bits(hs, x.device).data_ptr(), _stream(x.device))
    return y


# ------------------------------------------------------------------------------------------------------ cache write


def reshape_and_cache_int4(key, value, key_cache, value_cache, slot_mapping, *, k_scale_cache, v_scale_cache,
                           rotate=True):
    """Rotate, quantize and write key / value (tokens, KV heads, hs) into the cache; slots < 0 are skipped.
    A uint8 key view is the int4 cache, an int8 one k8v4 (vllm_quantpack/attention/k8v4_kv.py:36-38, 152-157).
    rotate=False takes key / value as already in the RHT domain (the `_store_k8v4` kernel contract)."""
    hs = key.shape[-1]
    if value.shape[-1] != hs:
        raise ValueError(f"key head size {hs} != value head size {value.shape[-1]}")
    if key.stride(-1) != 1 or value.stride(-1) != 1:
        raise ValueError("key / value rows must be contiguous")
    lay = CacheLayout.of(key_cache, value_cache, k_scale_cache, v_scale_cache, hs)
    if slot_mapping.dtype != torch.int64:
        slot_mapping = slot_mapping.to(torch.int64)
    slot_mapping = slot_mapping.contiguous()
    dt = _dtype_code(key, "reshape_and_cache_int4")
    if value.dtype != key.dtype:
        raise TypeError("key and value dtypes differ")
    name = "qp_reshape_and_cache_int4" if lay.fmt == FMT_INT4 else "qp_reshape_and_cache_k8v4"
    _lib.call(name, key.data_ptr(), value.data_ptr(), dt, key.shape[0], key.shape[1], hs, key.stride(0),
              key.stride(1), value.stride(0), value.stride(1), slot_mapping.data_ptr(), *lay.args(),
              rht.device_sign_bits(hs, key.device).data_ptr(), int(bool(rotate)), _stream(key.device))


# ------------------------------------------------------------------------------------------------------ decode

_ws_lock = threading.Lock()
_workspaces = {}


_retired = []


def workspace(device, nbytes):
    """A per-device scratch buffer for the split-KV partials, grown geometrically and kept for the process. A
    buffer that is outgrown stays allocated too: a CUDA graph captured earlier may still hold its address. Growing
    it inside a CUDA-graph capture allocates from the graph's pool: reserve the largest size before capturing."""
    key = str(torch.device(device))
    ws = _workspaces.get(key)
    if ws is not None and ws.numel() >= nbytes:  # the common case: no growth, no lock
        return ws
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            if ws is not None:
                _retired.append(ws)
            size = max(nbytes, 2 * (ws.numel() if ws is not None else 0), 1 << 20)
            ws = torch.empty(size, dtype=torch.uint8, device=device)
            _workspaces[key] = ws
    return ws


_sm_counts = {}


def sm_count(device):
    key = str(torch.device(device))
    n = _sm_counts.get(key)
    if n is None:
        n = _sm_counts[key] = torch.cuda.get_device_properties(device).multi_processor_count
    return n


VARLEN_MAX_Q = 32   # query tokens of a varlen sub-sequence at most (32 query rows per KV head)


def window_keys(max_seqlen_k, sliding_window, max_q):
    """Keys the split count is sized for: the context, or with a sliding window the span of the tiles a request's
    windows cover (its first token's window start to its last token, plus a partial tile)."""
    max_seqlen_k = int(max_seqlen_k)
    if sliding_window and sliding_window > 0:
        return min(max_seqlen_k, int(sliding_window) + int(max_q) - 1 + 127)
    return max_seqlen_k


_sizes = {}   # host-side size arithmetic of the library, by its arguments


def _memo(fn_name, *args):
    key = (fn_name,) + args
    v = _sizes.get(key)
    if v is None:
        if len(_sizes) >= 4096:
            _sizes.clear()
        v = _sizes[key] = getattr(_lib.load(), fn_name)(*args)
    return v


def decode_num_splits(num_seqs, num_kv_heads, max_seqlen_k, sms):
    return _memo("qp_decode_num_splits", int(num_seqs), int(num_kv_heads), int(max_seqlen_k), int(sms))


def paged_decode(q, key_cache, value_cache, out, *, cu_seqlens_q, max_seqlen_q, seqused_k, max_seqlen_k,
                 softmax_scale, block_table, k_scale_cache, v_scale_cache, num_splits=None, q_rotated=False,
                 out_fp32_lse=None, ws=None, partials_only=False, tokens_after_keys=0, sliding_window=0,
                 softcap=0.0, sinks=None):
    """Split-KV decode of up to 32 query rows per KV head (4 MTP tokens x 6 heads) over the paged cache.

    q / out (tokens, query heads, hs). When `out_fp32_lse` is a tensor (tokens, query heads) fp32, `out` must be fp32
    and receives the RHT-domain output with its base-2 log-sum-exp in `out_fp32_lse` (the partial a sequence-parallel
    rank exchanges); otherwise `out` gets the model-domain output in q's dtype. partials_only=True launches the split
    kernel alone and leaves its partials in the workspace (returned). tokens_after_keys: sequence tokens that follow
    the cached keys given here (a sequence-parallel rank holding an earlier range): query token i of a sequence sees
    key k iff k <= seqused_k - qlen + i + tokens_after_keys. sliding_window: vLLM's SLIDING_WINDOW (1 +
    window_size[0], 0 = none): that token then sees only the keys k > its last key - sliding_window. softcap > 0:
    vLLM's logit softcap, every score S becomes softcap * tanh(S / softcap). sinks: None or (query heads,) sink
    logits whose exp joins every row's softmax denominator (vLLM's attention sinks; model-domain output only)."""
    hs = q.shape[-1]
    nq = q.shape[1]
    lay = CacheLayout.of(key_cache, value_cache, k_scale_cache, v_scale_cache, hs)
    nkv = lay.nkv
    num_seqs = cu_seqlens_q.shape[0] - 1
    if num_splits is None:
        num_splits = decode_num_splits(num_seqs, nkv, window_keys(max_seqlen_k, sliding_window, max_seqlen_q),
                                       sm_count(q.device))
    wbytes = _memo("qp_decode_workspace_bytes", int(q.shape[0]), int(nq), int(hs), int(num_splits))
    if ws is None:
        ws = workspace(q.device, wbytes)
    for name, t in (("cu_seqlens_q", cu_seqlens_q), ("seqused_k", seqused_k), ("block_table", block_table)):
        if t.dtype != torch.int32:
            raise TypeError(f"{name} must be int32")
    if cu_seqlens_q.stride(0) != 1 or seqused_k.stride(0) != 1 or block_table.stride(-1) != 1:
        raise ValueError("cu_seqlens_q, seqused_k and block_table rows must be contiguous")
    if q.stride(-1) != 1 or out.stride(-1) != 1:
        raise ValueError("q / out rows must be contiguous")
    dt = _dtype_code(q, "paged_decode")
    if partials_only:
        mode, lse_ptr = 2, None
    elif out_fp32_lse is not None:
        if out.dtype != torch.float32 or out_fp32_lse.dtype != torch.float32:
            raise TypeError("out and lse must be fp32 for the RHT-domain output")
        if not out_fp32_lse.is_contiguous():
            raise ValueError("lse must be contiguous (tokens, query heads)")
        mode, lse_ptr = 1, out_fp32_lse.data_ptr()
    else:
        if out.dtype != q.dtype:
            raise TypeError("out dtype must match q")
        mode, lse_ptr = 0, None
    _lib.call("qp_paged_decode", lay.fmt, dt, q.data_ptr(), q.stride(0), q.stride(1), out.data_ptr(), out.stride(0),
              out.stride(1), q.shape[0], num_seqs, cu_seqlens_q.data_ptr(), seqused_k.data_ptr(), int(max_seqlen_q),
              block_table.data_ptr(), block_table.stride(0), *lay.args(), nq, nkv, hs, float(softmax_scale),
              rht.device_sign_bits(hs, q.device).data_ptr(), int(bool(q_rotated)), int(tokens_after_keys),
              int(sliding_window), float(softcap or 0.0), _sinks_ptr(sinks, nq, mode), mode, lse_ptr, int(num_splits),
              ws.data_ptr(), ws.numel() * ws.element_size(), _stream(q.device))
    return ws if partials_only else out


def merge_attn_partials(part_o, part_lse, out, lse_out=None):
    """Fold P partials part_o (P, tokens, heads, hs) fp32 / part_lse (P, tokens, heads) base-2 into `out`: in the
    model domain (inverse RHT / head, out's dtype) or, with `lse_out`, fp32 in the RHT domain plus the folded lse."""
    P, T, H, hs = part_o.shape
    if part_o.dtype != torch.float32 or part_lse.dtype != torch.float32:
        raise TypeError("partials must be fp32")
    if part_o.stride(-1) != 1:
        raise ValueError("partial rows must be contiguous")
    if lse_out is not None:
        if out.dtype != torch.float32 or not lse_out.is_contiguous():
            raise TypeError("out must be fp32 and lse_out contiguous")
        mode, dt, lptr, sbits = 1, 0, lse_out.data_ptr(), None
    else:
        mode, dt, lptr = 0, _dtype_code(out, "merge_attn_partials"), None
        sbits = rht.device_sign_bits(hs, out.device).data_ptr()
    _lib.call("qp_merge_attn_partials", dt, hs, T, H, P, part_o.data_ptr(), part_o.stride(1), part_o.stride(2),
              part_o.stride(0), part_lse.data_ptr(), part_lse.stride(1), part_lse.stride(2), part_lse.stride(0), mode,
              out.data_ptr(), out.stride(0), out.stride(1), lptr, sbits, _stream(out.device))
    return out


def fold_peer_partials(bases, rank, world, epoch, num_tokens, num_heads, head_size, out, lse_out=None):
    """Rank fold over NVLink (qp_fold_peer_partials): `bases` an int64 device tensor of the ranks' exchange buffer
    addresses, every rank's partial of call `epoch` already in its own buffer."""
    if lse_out is not None:
        if out.dtype != torch.float32 or not lse_out.is_contiguous():
            raise TypeError("out must be fp32 and lse_out contiguous")
        mode, dt, lptr, sbits = 1, 0, lse_out.data_ptr(), None
    else:
        mode, dt, lptr = 0, _dtype_code(out, "fold_peer_partials"), None
        sbits = rht.device_sign_bits(head_size, out.device).data_ptr()
    if out.stride(-1) != 1:
        raise ValueError("out rows must be contiguous")
    _lib.call("qp_fold_peer_partials", dt, head_size, num_tokens, num_heads, world, rank, bases.data_ptr(),
              epoch & 0xFFFFFFFF, mode, out.data_ptr(), out.stride(0), out.stride(1), lptr, sbits, _stream(out.device))
    return out


# ------------------------------------------------------------------------------------------------------ prefill


def prefill(q, key_cache, value_cache, out, *, block_row, n, softmax_scale, k_scale_cache, v_scale_cache,
            q_rotated=False, out_fp32_lse=None, ws=None, tokens_after_keys=0):
    """Chunk prefill of one sequence on the tensor cores: q (qlen, query heads, hs) are the last qlen positions of a
    context of n cached tokens (causal among themselves); block_row is the sequence's int32 block-table row.
    `out` gets the model-domain output in q's dtype, or with `out_fp32_lse` the fp32 RHT-domain output and its
    base-2 lse (vllm_quantpack/attention/int4_prefill.py:203-232 returns the RHT-domain output for rotated queries).
    tokens_after_keys as in paged_decode (n >= qlen - tokens_after_keys)."""
    hs, nq, qlen = q.shape[-1], q.shape[1], q.shape[0]
    lay = CacheLayout.of(key_cache, value_cache, k_scale_cache, v_scale_cache, hs)
    if block_row.dtype != torch.int32 or block_row.stride(-1) != 1:
        raise TypeError("block_row must be a contiguous int32 row")
    if q.stride(-1) != 1 or out.stride(-1) != 1:
        raise ValueError("q / out rows must be contiguous")
    dt = _dtype_code(q, "prefill")
    wbytes = _lib.load().qp_prefill_workspace_bytes(qlen, int(n), nq, lay.nkv, hs, int(tokens_after_keys))
    if ws is None:
        ws = workspace(q.device, wbytes)
    if out_fp32_lse is not None:
        if out.dtype != torch.float32 or out_fp32_lse.dtype != torch.float32 or not out_fp32_lse.is_contiguous():
            raise TypeError("out and lse must be fp32 (lse contiguous) for the RHT-domain output")
        mode, lse_ptr = 1, out_fp32_lse.data_ptr()
    else:
        if out.dtype != q.dtype:
            raise TypeError("out dtype must match q")
        mode, lse_ptr = 0, None
    _lib.call("qp_prefill", lay.fmt, dt, q.data_ptr(), q.stride(0), q.stride(1), out.data_ptr(), out.stride(0),
              out.stride(1), qlen, int(n), block_row.data_ptr(), *lay.args(), nq, lay.nkv, hs, float(softmax_scale),
              rht.device_sign_bits(hs, q.device).data_ptr(), int(bool(q_rotated)), int(tokens_after_keys), mode,
              lse_ptr, ws.data_ptr(), ws.numel() * ws.element_size(), _stream(q.device))
    return out


def prefill_varlen(q, key_cache, value_cache, out, *, cu_seqlens_q, seqused_k, max_seqlen_k, block_table,
                   softmax_scale, k_scale_cache, v_scale_cache, q_rotated=False, out_fp32_lse=None, ws=None,
                   sliding_window=0, softcap=0.0, sinks=None):
    """Several short prefill chunks in ONE launch (the reference's Triton sub-batch of the chunks that are not long,
    vllm_quantpack/attention/int4_kv.py:313-323): request i's query tokens q[cu_seqlens_q[i]:cu_seqlens_q[i + 1]] are
    the last positions of its context of seqused_k[i] cached tokens, causal among themselves, read through
    block_table[i]. Split on the device into sub-sequences of 32 / group tokens for the split-KV kernel, so nothing
    is read back to the host; max_seqlen_k (a host int, an upper bound of seqused_k) sizes the split count.
    `out` as in prefill; sliding_window, softcap and sinks as in paged_decode."""
    hs, nq, T = q.shape[-1], q.shape[1], q.shape[0]
    lay = CacheLayout.of(key_cache, value_cache, k_scale_cache, v_scale_cache, hs)
    for name, t in (("cu_seqlens_q", cu_seqlens_q), ("seqused_k", seqused_k), ("block_table", block_table)):
        if t.dtype != torch.int32 or t.stride(-1) != 1:
            raise TypeError(f"{name} must be int32 with contiguous rows")
    if q.stride(-1) != 1 or out.stride(-1) != 1:
        raise ValueError("q / out rows must be contiguous")
    dt = _dtype_code(q, "prefill_varlen")
    chunks = seqused_k.shape[0]
    lib = _lib.load()
    max_k = window_keys(max_seqlen_k, sliding_window, VARLEN_MAX_Q)
    wbytes = lib.qp_prefill_varlen_workspace_bytes(T, chunks, nq, lay.nkv, hs, max_k)
    if ws is None:
        ws = workspace(q.device, wbytes)
    if out_fp32_lse is not None:
        if out.dtype != torch.float32 or out_fp32_lse.dtype != torch.float32 or not out_fp32_lse.is_contiguous():
            raise TypeError("out and lse must be fp32 (lse contiguous) for the RHT-domain output")
        mode, lse_ptr = 1, out_fp32_lse.data_ptr()
    else:
        if out.dtype != q.dtype:
            raise TypeError("out dtype must match q")
        mode, lse_ptr = 0, None
    _lib.call("qp_prefill_varlen", lay.fmt, dt, q.data_ptr(), q.stride(0), q.stride(1), out.data_ptr(),
              out.stride(0), out.stride(1), T, chunks, cu_seqlens_q.data_ptr(), seqused_k.data_ptr(),
              max_k, block_table.data_ptr(), block_table.stride(0), *lay.args(), nq, lay.nkv, hs,
              float(softmax_scale), rht.device_sign_bits(hs, q.device).data_ptr(), int(bool(q_rotated)),
              int(sliding_window), float(softcap or 0.0), _sinks_ptr(sinks, nq, mode), mode, lse_ptr, ws.data_ptr(),
              ws.numel() * ws.element_size(), _stream(q.device))
    return out
