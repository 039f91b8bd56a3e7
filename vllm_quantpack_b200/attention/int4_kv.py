"""int4_per_token_head / k8v4_per_token_head attention on vLLM's Triton backend, served by B200 kernels.

The drop-in counterpart of the plugin module vllm_quantpack/attention/int4_kv.py. The reference generates a patched
copy of vLLM's Triton kernel and launcher; this module instead replaces the stock module's entry points
(`vllm.v1.attention.ops.int4_per_token_head`) with thin launches of libquantpack_b200.so:

  unified_attention_int4   decode steps (<= MAX_Q_SPLIT_KV query tokens per request, graph-capturable, no host
                           sync) -> split-KV decode kernel + merge; steps with prefill chunks -> one host read of the
                           step's lengths per step, decode rows as a sub-batch, each long chunk -> the tcgen05
                           prefill kernel, all other chunks -> one varlen launch of the split-KV kernel
                           (int4_kv.py:281-333: long chunks to FlashAttention, the rest to one Triton sub-batch)
  reshape_and_cache_int4   fused RHT + quantize + pack store, int4 and k8v4 (k8v4_kv.py:152-163)
  single_rht               the transform both of the above apply, so any stock path left in use stays consistent

Head sizes 256 and 512 (Gemma 4's global layers, int4_kv.py:302-305) are served. Calls the B200 path does not cover
(sliding window, softcap, sinks, ALiBi, qq_bias, FP8 output, mm_prefix ranges, another head size) go to the stock
`unified_attention_int4`, unchanged, for an int4 cache, and raise for a k8v4 cache (no stock kernel reads it). The
stock `_launch_packed_attn` is left in place: only that stock path reaches it. The same environment switches are honoured:
VLLM_QUANTPACK_INT4_KV=0 (no patch), VLLM_QUANTPACK_INT4_FA_PREFILL=0 (prefill chunks stay stock),
VLLM_QUANTPACK_INT4_DECODE="tile,warps,segments[,rows]" (segments: split count of the decode, "auto" = per call),
VLLM_QUANTPACK_INT4_TILES (accepted; the B200 prefill tiles are fixed at 128 x 64).
"""
import contextlib
import importlib
import itertools
import os

import torch

MODULE = "vllm.v1.attention.ops.int4_per_token_head"
PACKED_DTYPES = ("int4_per_token_head", "k8v4_per_token_head")   # caches served by the B200 kernels
MAX_Q_SPLIT_KV = 4               # MTP / EAGLE verification with up to 3 draft tokens
MAX_DECODE_ROWS = 32             # query tokens x query heads per KV head one decode CTA holds
LONG_ROWS = 2048                 # query rows (tokens x heads per KV head) that make a chunk long at any context
HEAD_SIZES = (256, 512)          # head sizes of the attention kernels
PREFILL_TILES_DEFAULT = (128, 64, 10, 1)   # (BLOCK_M, TILE, warps, CTAs per SM) of the tcgen05 prefill kernel
DECODE_TILES_DEFAULT = (64, 4, "auto")
DECODE_MAX_M = 32
MIN_SEGMENTS, MAX_SEGMENTS = 16, 128


def prefill_tiles(major):
    """The prefill tiling, for the reference's VLLM_QUANTPACK_INT4_TILES override (int4_kv.py:67-71). The B200
    kernel's tiles are fixed; an override is reported and not applied."""
    env = os.environ.get("VLLM_QUANTPACK_INT4_TILES")
    if env:
        return tuple(int(x) for x in env.split(","))
    return PREFILL_TILES_DEFAULT


def segments_for(sms):
    """Split-KV segments per sequence vLLM's metadata builder sizes its buffers for (int4_kv.py:74-77): next power
    of two of SMs / 4, between 16 and 128."""
    n = 1 << max(0, -(-sms // 4) - 1).bit_length()
    return min(MAX_SEGMENTS, max(MIN_SEGMENTS, n))


def decode_tiles(sms):
    """(tile, warps, segments[, rows]) of the split-KV decode (int4_kv.py:80-85 semantics). The B200 decode kernel
    runs 64-token tiles with 4 warps whatever the tuple says; an integer segment count fixes its split count,
    "auto" lets `qp_decode_num_splits` choose per call (reported here as segments_for(sms))."""
    env = os.environ.get("VLLM_QUANTPACK_INT4_DECODE")
    tile, warps, segments, *max_m = env.split(",") if env else DECODE_TILES_DEFAULT
    segments = segments_for(sms) if str(segments).strip() == "auto" else int(segments)
    return (int(tile), int(warps), segments) + tuple(int(m) for m in max_m[:1])


def decode_splits_override():
    """The decode split count fixed by VLLM_QUANTPACK_INT4_DECODE, or None for the per-call choice."""
    env = os.environ.get("VLLM_QUANTPACK_INT4_DECODE")
    if not env:
        return None
    parts = env.split(",")
    if len(parts) < 3 or parts[2].strip() == "auto":
        return None
    return int(parts[2])


def _plain(q, alibi_slopes, qq_bias, output_scale, mm_prefix_range):
    """True when the call uses no feature outside the B200 kernels (the reference's list, int4_kv.py:304-305, less
    the sliding window, the softcap and the sinks, which the split-KV kernel and its merge apply)."""
    return alibi_slopes is None and qq_bias is None and output_scale is None and mm_prefix_range is None \
        and q.shape[2] in HEAD_SIZES


def sliding_window_of(window_size):
    """vLLM's SLIDING_WINDOW from the window_size argument (1 + left window, 0 for none): a query token at position p
    sees keys p - SLIDING_WINDOW + 1 .. p (vllm/v1/attention/ops/triton_unified_attention.py:855, 1008, vLLM 0.22;
    the right window is not applied there either)."""
    if window_size is None or window_size[0] < 0:
        return 0
    return 1 + int(window_size[0])


def _forward_step():
    """vLLM's forward context of the running step, or None outside one (tests, eager calls)."""
    try:
        from vllm.forward_context import get_forward_context, is_forward_context_available
        return get_forward_context() if is_forward_context_available() else None
    except Exception:
        return None


class StepPlan:
    """How one forward step's requests split over the kernels, worked out once per step and reused by every attention
    layer of it (they all get the same cu_seqlens_q / seqused_k tensors): the lengths come to the host in ONE read
    (the two tensors concatenated on the GPU), and the sub-batch index tensors go to the GPU from pinned memory
    without a wait. The reference reads both lists per step (int4_kv.py:260-278) and rebuilds its sub-batch indices
    per layer; here the second and later layers of a step touch no host memory at all."""

    def __init__(self, cu_seqlens_q, seqused_k, group, prefill_on, head_size=256, long_chunks=True):
        nseq = seqused_k.shape[0]
        both = torch.cat([cu_seqlens_q.to(torch.int64), seqused_k.to(torch.int64)]).tolist()
        self.cu, self.used = both[:nseq + 1], both[nseq + 1:]
        self.dec, self.pre, self.short, self.stock = split_step(self.cu, self.used, group, prefill_on, head_size,
                                                                long_chunks)
        dev = cu_seqlens_q.device
        self.dec_batch = _SubBatch(self.dec, self.cu, self.used, dev) if self.dec else None
        self.short_batch = _SubBatch(self.short, self.cu, self.used, dev) if self.short else None
        self.stock_batch = _SubBatch(self.stock, self.cu, self.used, dev) if self.stock else None

    @staticmethod
    def of(cu_seqlens_q, seqused_k, group, prefill_on, head_size=256, long_chunks=True):
        """The step's plan, kept on vLLM's forward context (keyed by the length tensors themselves: another KV-cache
        group of the same step gets other tensors)."""
        step = _forward_step()
        plans = getattr(step, "_quantpack_b200_plans", None) if step is not None else None
        key = (id(cu_seqlens_q), id(seqused_k), group, prefill_on, head_size, long_chunks)
        if plans is not None and key in plans and plans[key][0] is cu_seqlens_q and plans[key][1] is seqused_k:
            return plans[key][2]
        plan = StepPlan(cu_seqlens_q, seqused_k, group, prefill_on, head_size, long_chunks)
        if step is not None:
            try:
                if plans is None:
                    plans = step._quantpack_b200_plans = {}
                plans[key] = (cu_seqlens_q, seqused_k, plan)
            except Exception:
                pass
        return plan


class _SubBatch:
    """Requests `idx` of a step as a batch of their own: gather rows / per-request tensors, scatter the output."""

    def __init__(self, idx, cu, used, device):
        lens = [cu[i + 1] - cu[i] for i in idx]
        rows = [r for i in idx for r in range(cu[i], cu[i + 1])]
        def to_dev(x, dt):
            t = torch.tensor(x, dtype=dt)
            return t.pin_memory().to(device, non_blocking=True) if device.type == "cuda" else t.to(device)

        self.rows = to_dev(rows, torch.int64)
        self.sel = to_dev(idx, torch.int64)
        self.cu = to_dev([0, *itertools.accumulate(lens)], torch.int32)
        self.max_q, self.max_k = max(lens), max(used[i] for i in idx)

    def run(self, fn, q, out, args):
        """fn(q_rows, out_rows, args) with the sub-batch's own lengths, block table and query rows."""
        sub_out = torch.empty((self.rows.shape[0],) + tuple(out.shape[1:]), dtype=out.dtype, device=out.device)
        sub = dict(args, cu_seqlens_q=self.cu, max_seqlen_q=self.max_q, seqused_k=args["seqused_k"][self.sel],
                   block_table=args["block_table"][self.sel], max_seqlen_k=self.max_k)
        fn(q[self.rows], sub_out, sub)
        out[self.rows] = sub_out


def split_step(cu, used, group, prefill_on=True, head_size=256, long_chunks=True):
    """Requests of one step by path: (decode, long, short, stock) index lists. Decode: 1..MAX_Q_SPLIT_KV query tokens
    whose rows fit one decode CTA. The other requests with queries are prefill chunks: long ones (at least MIN_QUERY
    tokens over at least MIN_CONTEXT cached tokens, or enough query rows to fill the machine on their own; head 256)
    each go to the tcgen05 prefill kernel, the rest together to one varlen launch of the split-KV kernel, as the
    reference sends its long chunks to FlashAttention and the rest to one Triton sub-batch (int4_kv.py:313-323).
    long_chunks=False (a sliding-window, softcap or sink layer: the prefill kernel has none of them) sends every
    chunk to the varlen launch. With prefill routing off every chunk goes to the stock path. Requests without queries are left out."""
    from .int4_prefill import MIN_CONTEXT, MIN_QUERY
    dec, long, short, stock = [], [], [], []
    for i in range(len(used)):
        ql = cu[i + 1] - cu[i]
        if ql <= 0:
            continue
        if ql <= MAX_Q_SPLIT_KV and ql * group <= MAX_DECODE_ROWS:
            dec.append(i)
        elif not prefill_on:
            stock.append(i)
        elif long_chunks and head_size == 256 and ql >= MIN_QUERY and (used[i] >= MIN_CONTEXT or
                                                                       ql * group >= LONG_ROWS):
            long.append(i)
        else:
            short.append(i)
    return dec, long, short, stock


def make_unified_attention(stock_unified, prefill_on=True):
    """The replacement of `unified_attention_int4` (signature of int4_kv.py:294-301), falling back to
    `stock_unified` for int4 calls the B200 kernels do not cover. A k8v4 cache has no stock kernel to fall back to
    (the stock int4 kernel would read its int8 keys as nibbles), so such a call raises instead. A sliding-window,
    softcap or sink layer runs on the split-KV kernel: decodes as usual, every prefill chunk in the varlen launch."""
    from . import k8v4_kv, ops
    # VLLM_QUANTPACK_INT4_DECODE is read once, when the replacement is made (the plugin reads its knobs at patch
    # time, int4_kv.py:190-226), not in every layer's call
    splits = decode_splits_override()

    def unified_attention_int4(q, k_cache, v_cache, out, *, cu_seqlens_q, max_seqlen_q, seqused_k, max_seqlen_k,
                               softmax_scale, window_size, block_table, softcap, sinks, alibi_slopes, use_alibi_sqrt,
                               qq_bias, output_scale, mm_prefix_range, k_scale_cache, v_scale_cache, **kw):
        def stock_args():
            return dict(cu_seqlens_q=cu_seqlens_q, max_seqlen_q=max_seqlen_q, seqused_k=seqused_k,
                        max_seqlen_k=max_seqlen_k, softmax_scale=softmax_scale, window_size=window_size,
                        block_table=block_table, softcap=softcap, sinks=sinks, alibi_slopes=alibi_slopes,
                        use_alibi_sqrt=use_alibi_sqrt, qq_bias=qq_bias, output_scale=output_scale,
                        mm_prefix_range=mm_prefix_range, k_scale_cache=k_scale_cache, v_scale_cache=v_scale_cache,
                        **kw)

        if not _plain(q, alibi_slopes, qq_bias, output_scale, mm_prefix_range):
            if k8v4_kv.is_k8v4(k_cache):
                raise NotImplementedError(
                    f"{k8v4_kv.NAME}: ALiBi, qq_bias, FP8 output, mm_prefix ranges and head sizes other than "
                    f"{HEAD_SIZES} are not served by the B200 kernels, and vLLM's stock int4 kernel cannot read a "
                    f"k8v4 cache")
            return stock_unified(q, k_cache, v_cache, out, **stock_args())
        group = q.shape[1] // k_cache.shape[2]
        window = sliding_window_of(window_size)
        cap = float(softcap) if softcap and softcap > 0 else 0.0

        def decode(qs, outs, a):
            ops.paged_decode(qs, k_cache, v_cache, outs, cu_seqlens_q=a["cu_seqlens_q"],
                             max_seqlen_q=a["max_seqlen_q"], seqused_k=a["seqused_k"], max_seqlen_k=a["max_seqlen_k"],
                             softmax_scale=softmax_scale, block_table=a["block_table"], k_scale_cache=k_scale_cache,
                             v_scale_cache=v_scale_cache, num_splits=splits, sliding_window=window, softcap=cap,
                             sinks=sinks)

        if max_seqlen_q <= MAX_Q_SPLIT_KV and max_seqlen_q * group <= MAX_DECODE_ROWS:
            # a decode step: no host read of the lengths (CUDA-graph capturable)
            ops.paged_decode(q, k_cache, v_cache, out, cu_seqlens_q=cu_seqlens_q, max_seqlen_q=max_seqlen_q,
                             seqused_k=seqused_k, max_seqlen_k=max_seqlen_k, softmax_scale=softmax_scale,
                             block_table=block_table, k_scale_cache=k_scale_cache, v_scale_cache=v_scale_cache,
                             num_splits=splits, sliding_window=window, softcap=cap, sinks=sinks)
            return None
        args = stock_args()
        plan = StepPlan.of(cu_seqlens_q, seqused_k, group, prefill_on, q.shape[2],
                           long_chunks=window == 0 and cap == 0.0 and sinks is None)
        if plan.dec_batch is not None:
            plan.dec_batch.run(decode, q, out, args)
        if plan.short_batch is not None:
            plan.short_batch.run(
                lambda qs, outs, a: ops.prefill_varlen(
                    qs, k_cache, v_cache, outs, cu_seqlens_q=a["cu_seqlens_q"], seqused_k=a["seqused_k"],
                    max_seqlen_k=a["max_seqlen_k"], block_table=a["block_table"], softmax_scale=softmax_scale,
                    k_scale_cache=k_scale_cache, v_scale_cache=v_scale_cache, sliding_window=window, softcap=cap,
                    sinks=sinks), q, out, args)
        if plan.stock_batch is not None:
            if k8v4_kv.is_k8v4(k_cache):
                raise NotImplementedError(f"{k8v4_kv.NAME}: prefill chunks need the B200 prefill kernel "
                                          f"(VLLM_QUANTPACK_INT4_FA_PREFILL=0 leaves them to the stock int4 kernel)")
            plan.stock_batch.run(lambda qs, outs, a: stock_unified(qs, k_cache, v_cache, outs, **a), q, out, args)
        cu, used = plan.cu, plan.used
        for i in plan.pre:
            ops.prefill(q[cu[i]:cu[i + 1]], k_cache, v_cache, out[cu[i]:cu[i + 1]], block_row=block_table[i],
                        n=used[i], softmax_scale=softmax_scale, k_scale_cache=k_scale_cache,
                        v_scale_cache=v_scale_cache)
        return out

    unified_attention_int4._quantpack = True           # the plugin's idempotence marker (int4_kv.py:198, 215)
    unified_attention_int4._quantpack_b200 = True      # this build's (the reference's own patch also sets _quantpack)
    return unified_attention_int4


def make_reshape_and_cache(stock_store):
    """The replacement of `reshape_and_cache_int4` (k8v4_kv.py:152-163): the fused B200 store for int4 (uint8 views)
    and k8v4 (int8 views) caches. Head sizes other than 128 / 256 / 512 go to the stock store (int4) or raise
    (k8v4, which the stock store does not know)."""
    from . import k8v4_kv, ops

    def reshape_and_cache_int4(key, value, key_cache, value_cache, slot_mapping, *, k_scale_cache, v_scale_cache):
        if key.shape[-1] not in (128, 256, 512) or value.shape[-1] != key.shape[-1]:
            if k8v4_kv.is_k8v4(key_cache):
                raise ValueError(f"{k8v4_kv.NAME}: head sizes {key.shape[-1]} / {value.shape[-1]} not supported")
            return stock_store(key, value, key_cache, value_cache, slot_mapping, k_scale_cache=k_scale_cache,
                               v_scale_cache=v_scale_cache)
        ops.reshape_and_cache_int4(key, value, key_cache, value_cache, slot_mapping, k_scale_cache=k_scale_cache,
                                   v_scale_cache=v_scale_cache)

    reshape_and_cache_int4._quantpack = True           # the plugin's idempotence marker (int4_kv.py:198, 215)
    reshape_and_cache_int4._quantpack_b200 = True      # this build's (the reference's own patch also sets _quantpack)
    return reshape_and_cache_int4


def make_single_rht():
    from . import ops

    def single_rht(x, inverse=False):
        return ops.single_rht(x.float(), inverse=inverse)

    single_rht._quantpack = True           # the plugin's idempotence marker (int4_kv.py:198, 215)
    single_rht._quantpack_b200 = True      # this build's (the reference's own patch also sets _quantpack)
    return single_rht


def _b200_ready():
    """SM count of device 0; raises unless the B200 library loads and device 0 is an sm_100 GPU."""
    import torch

    from .. import _lib
    _lib.load()
    if not torch.cuda.is_available():
        raise RuntimeError("no CUDA device")
    cap = torch.cuda.get_device_capability(0)
    if cap[0] != 10:
        raise RuntimeError(f"compute capability {cap[0]}.{cap[1]}: the B200 kernels need sm_100")
    return torch.cuda.get_device_properties(0).multi_processor_count


def patch_int4_kv(logger):
    """Install the B200 ops into the stock int4 module (int4_kv.py:190-226). Returns True when patched (or already
    patched), False when disabled, when vLLM lacks the int4 mode, or when the B200 library / GPU is unavailable (the
    stock path then stays, with a warning)."""
    if os.environ.get("VLLM_QUANTPACK_INT4_KV", "1") == "0":
        return False
    try:
        stock = importlib.import_module(MODULE)
    except Exception as e:      # vLLM without the int4 KV mode
        logger.debug("vllm-quantpack-b200: int4 KV attention not patched (%s)", e)
        return False
    if getattr(getattr(stock, "unified_attention_int4", None), "_quantpack_b200", False):
        return True
    try:
        sms = _b200_ready()
        decode = decode_tiles(sms)
        if os.environ.get("VLLM_QUANTPACK_INT4_TILES"):
            logger.info("vllm-quantpack-b200: VLLM_QUANTPACK_INT4_TILES ignored (fixed 128 x 64 tcgen05 tiles)")
        if decode[:2] != (64, 4):
            logger.info("vllm-quantpack-b200: decode tile / warps %s ignored (fixed 64-token tiles, 4 warps)",
                        decode[:2])
        prefill_on = os.environ.get("VLLM_QUANTPACK_INT4_FA_PREFILL", "1") != "0"
        unified = make_unified_attention(stock.unified_attention_int4, prefill_on=prefill_on)
        store = make_reshape_and_cache(stock.reshape_and_cache_int4)
        rht_fn = make_single_rht()
    except Exception as e:
        logger.warning("vllm-quantpack-b200: int4_per_token_head attention left stock (%s)", e)
        return False
    from . import k8v4_kv
    stock.single_rht = rht_fn
    stock.reshape_and_cache_int4 = store
    stock.unified_attention_int4 = unified
    segments = _patch_decode_segments(decode[2], logger)
    k8v4 = k8v4_kv.patch_backend(stock, logger) and k8v4_kv.register_dtype(logger)
    logger.info("vllm-quantpack-b200: int4_per_token_head KV attention on B200 kernels (split-KV decode up to %d "
                "tokens, %s splits; tcgen05 prefill%s; segment buffers for %s)", MAX_Q_SPLIT_KV,
                decode[2] if decode_splits_override() else "auto", "" if prefill_on else " off",
                segments or "stock")
    if k8v4:
        logger.info("vllm-quantpack-b200: KV cache dtype %s available (int8 keys, int4 values)", k8v4_kv.NAME)
    return True


@contextlib.contextmanager
def _segment_count(module, segments):
    """vLLM's Triton metadata builder reads the module constant NUM_PAR_SOFTMAX_SEGMENTS once, while it allocates its
    split-KV segment buffers: hold it at `segments` for that long."""
    old = module.NUM_PAR_SOFTMAX_SEGMENTS
    module.NUM_PAR_SOFTMAX_SEGMENTS = segments
    try:
        yield
    finally:
        module.NUM_PAR_SOFTMAX_SEGMENTS = old


def _patch_decode_segments(segments, logger):
    """Builders of int4 / k8v4 caches allocate vLLM's split-KV segment buffers for `segments` segments (the buffers
    the stock fallback kernel writes; int4_kv.py:229-257), and reserve this process's decode workspace on their device
    for the largest decode batch they plan (seq_threshold_3D query rows at the largest split count), so that CUDA-graph
    capture never grows it. Returns the segment count in use, 0 when the builder is left stock."""
    if segments < 1 or segments & (segments - 1):
        logger.warning("vllm-quantpack-b200: int4 split-KV segments must be a power of two, got %d: left stock",
                       segments)
        return 0
    try:
        from vllm.v1.attention.backends import triton_attn
        cls = triton_attn.TritonAttentionMetadataBuilder
        triton_attn.NUM_PAR_SOFTMAX_SEGMENTS   # the constant the wrapper sets must exist
    except Exception as e:
        logger.info("vllm-quantpack-b200: int4 split-KV segments left stock (%s)", e)
        return 0
    original = cls.__init__
    if getattr(original, "_quantpack_b200", False):
        return segments

    def init(builder, kv_cache_spec, layer_names, vllm_config, device):
        packed = vllm_config.cache_config.cache_dtype in PACKED_DTYPES
        with _segment_count(triton_attn, segments) if packed else contextlib.nullcontext():
            original(builder, kv_cache_spec, layer_names, vllm_config, device)
        if packed:
            reserve_decode_workspace(builder, vllm_config, device)

    init._quantpack = True
    init._quantpack_b200 = True
    cls.__init__ = init
    return segments


def reserve_decode_workspace(builder, vllm_config, device):
    """Grow the decode workspace of `device` to the builder's largest decode batch (best effort: the sizes come
    from vLLM attributes that may be absent, in which case the workspace grows on first use)."""
    try:
        from .. import _lib
        from . import ops
        rows = int(getattr(builder, "seq_threshold_3D"))
        model = vllm_config.model_config
        nq = int(model.get_num_attention_heads(vllm_config.parallel_config))
        nkv = int(model.get_num_kv_heads(vllm_config.parallel_config))
        max_len = int(getattr(model, "max_model_len", 1 << 20))
        try:
            head = int(model.get_head_size())
        except Exception:
            head = max(HEAD_SIZES)
        ops.workspace(device, decode_workspace_bound(rows, nq, nkv, max_len, ops.sm_count(device), head))
    except Exception:
        pass


def decode_workspace_bound(max_tokens, num_q_heads, num_kv_heads, max_seqlen_k, sms, head_size=max(HEAD_SIZES)):
    """Largest decode workspace (bytes) a batch of at most `max_tokens` query tokens can need: over every batch size,
    the tokens it can hold times the split count the library (or the environment) gives it."""
    from .. import _lib
    lib = _lib.load()
    fixed = decode_splits_override()
    worst = 0
    for seqs in range(1, max(1, max_tokens) + 1):
        splits = fixed or lib.qp_decode_num_splits(seqs, num_kv_heads, max_seqlen_k, sms)
        tokens = min(max_tokens, MAX_Q_SPLIT_KV * seqs)
        worst = max(worst, lib.qp_decode_workspace_bytes(tokens, num_q_heads, head_size, splits))
    return worst
