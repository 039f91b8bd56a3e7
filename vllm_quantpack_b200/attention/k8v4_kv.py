"""k8v4_per_token_head KV cache: int8 keys and int4 values, both in the randomized-Hadamard domain.

The cache format is the reference plugin's (vllm_quantpack/attention/k8v4_kv.py:1-30): per (token, KV head) one cell
[K hs int8 | K scale f32 | V hs/2 bytes | V scale f32] = 1.5 hs + 8 bytes (392 at hs 256; the int4 cell is 264). The
value half is byte for byte the int4 cell's value half (nibbles, fp32 scale with the 4-bit zero point in its low
mantissa bits). vLLM owns the cache and reads it through four strided views, so those views, the cell size and the
dtype registration are the drop-in contract; the store and both attention kernels are this build's
(`ops.reshape_and_cache_int4` / `paged_decode` / `prefill` dispatch on the int8 key view).

Here the cell is described once (`CellFormat`) and every view is cut from it with `as_strided`; the vLLM glue wraps
the three backend methods through one helper instead of per-method closures.
"""
import dataclasses

import torch

NAME = "k8v4_per_token_head"


@dataclasses.dataclass(frozen=True)
class CellFormat:
    """Byte layout of one (token, KV head) cell: key codes, key scale, value codes, value scale, in that order."""

    key_bytes: int
    value_bytes: int
    scale_bytes: int = 4

    @property
    def key_scale_at(self):
        return self.key_bytes

    @property
    def value_at(self):
        return self.key_bytes + self.scale_bytes

    @property
    def value_scale_at(self):
        return self.value_at + self.value_bytes

    @property
    def size(self):
        return self.value_scale_at + self.scale_bytes


def k8v4_cell(head_size, head_size_v=None):
    """The k8v4 cell: one int8 per key channel, two value channels per byte (k8v4_kv.py:31-33)."""
    return CellFormat(head_size, (head_size if head_size_v is None else head_size_v) // 2)


def cell_bytes(head_size, head_size_v):
    """Bytes of one (token, KV head) k8v4 cell."""
    return k8v4_cell(head_size, head_size_v).size


def is_k8v4(key_cache):
    """A k8v4 key view is int8; the int4 cache's views are uint8 (k8v4_kv.py:36-38)."""
    return key_cache.dtype == torch.int8


def views(kv_cache, head_size, head_size_v=None):
    """(key, value, key scale, value scale) views of the logical (blocks, KV heads, block size, cell) int8 cache.

    key (blocks, block size, KV heads, hs) int8; value (..., hs_v / 2) uint8; scales (blocks, block size, KV heads)
    fp32, all over the cache's own storage. Only the cache's strides are used, so a physically NHD cache works too.
    These are the views vLLM's Triton backend hands to the store and the attention ops (k8v4_kv.py:41-65)."""
    fmt = k8v4_cell(head_size, head_size_v)
    nblocks, nkv, block_size, cell = kv_cache.shape
    if kv_cache.element_size() != 1 or cell != fmt.size:
        raise ValueError(f"{NAME}: cache cell of {cell} x {kv_cache.element_size()} bytes, expected {fmt.size} for "
                         f"head sizes {head_size} / {head_size_v if head_size_v is not None else head_size}")
    s_block, s_head, s_slot, _ = kv_cache.stride()  # bytes (one-byte elements)
    base = kv_cache.storage_offset()
    if any(x % 4 for x in (s_block, s_head, s_slot, base, fmt.key_scale_at, fmt.value_scale_at)):
        raise ValueError(f"{NAME}: fp32 scales are not 4-byte aligned (strides {tuple(kv_cache.stride())}, head "
                         f"{head_size})")
    shape, stride = (nblocks, block_size, nkv), (s_block, s_slot, s_head)
    key = kv_cache.as_strided(shape + (fmt.key_bytes,), stride + (1,), base)
    value = kv_cache.view(torch.uint8).as_strided(shape + (fmt.value_bytes,), stride + (1,), base + fmt.value_at)
    words = torch.empty(0, dtype=torch.float32, device=kv_cache.device).set_(kv_cache.untyped_storage())

    def scales(at):
        return words.as_strided(shape, tuple(x // 4 for x in stride), (base + at) // 4)

    return key, value, scales(fmt.key_scale_at), scales(fmt.value_scale_at)


def store(key, value, key_cache, value_cache, slot_mapping, *, k_scale_cache, v_scale_cache):
    """Rotate (RHT), quantize and write key / value into the k8v4 cache views in one fused kernel (the reference
    rotates in torch and then launches its Triton store, k8v4_kv.py:68-86)."""
    from . import ops
    if value.shape[2] % 2:
        raise ValueError(f"{NAME}: odd value head size {value.shape[2]}")
    ops.reshape_and_cache_int4(key, value, key_cache, value_cache, slot_mapping, k_scale_cache=k_scale_cache,
                               v_scale_cache=v_scale_cache)


# ---------------------------------------------------------------------------------------------------- vLLM glue
def _dtype_handler(mode):
    """The handler vLLM's kv-cache dtype registry takes: storage dtype int8, vLLM's int4 per-token-head mode, so
    every generic per-token-head path of vLLM (scales, the Triton backend, packed-attention dispatch) serves it."""
    return type("K8v4PerTokenHead", (), {"name": NAME, "torch_dtype": lambda self: torch.int8,
                                         "quant_mode": lambda self: mode})


def register_dtype(logger):
    """Make `--kv-cache-dtype k8v4_per_token_head` valid (k8v4_kv.py:89-110). False on a vLLM without the dtype
    registry (the option then stays unknown to vLLM)."""
    try:
        from vllm.config import cache as cache_config
        from vllm.v1.kv_cache_interface import KVQuantMode
        mode = KVQuantMode.INT4_PER_TOKEN_HEAD
        known = cache_config.get_kv_cache_dtype_handler(NAME)
        registrar = cache_config.register_kv_cache_dtype
    except Exception as e:
        logger.debug("vllm-quantpack-b200: no kv-cache dtype registry, %s unavailable (%s)", NAME, e)
        return False
    if known is None:
        registrar(NAME)(_dtype_handler(mode))
    return True


def _mark(fn):
    fn._quantpack = True           # the plugin's idempotence marker
    fn._quantpack_b200 = True      # this build's
    return fn


def _wrap(owner, name, body):
    """Replace the method `owner.name` by one that calls body(stock_method, self, *args)."""
    stock = getattr(owner, name)

    def method(self, *args, **kwargs):
        return body(stock, self, *args, **kwargs)

    method.__name__ = name
    setattr(owner, name, _mark(method))


def _ensure_scale_views(stock, impl, kv_cache):
    """TritonAttentionImpl._ensure_scale_caches: a k8v4 layer's scale caches are views into its cache cells,
    initialised to 1 like vLLM's own per-token-head scales."""
    if impl.kv_cache_dtype != NAME:
        return stock(impl, kv_cache)
    if impl._k_scale_cache is None:
        *_, key_scales, value_scales = views(kv_cache, impl.head_size)
        key_scales.fill_(1.0)
        value_scales.fill_(1.0)
        impl._k_scale_cache, impl._v_scale_cache = key_scales, value_scales


def _key_value_views(stock, impl, kv_cache):
    """TritonAttentionImpl._pth_key_value_caches: the int8 key and uint8 value views of a k8v4 cache."""
    if impl.kv_cache_dtype != NAME:
        return stock(impl, kv_cache)
    impl._ensure_scale_caches(kv_cache)
    key, value, _, _ = views(kv_cache, impl.head_size)
    return key, value


def patch_backend(stock_module, logger):
    """Teach vLLM's Triton backend the k8v4 page cell and views (k8v4_kv.py:113-166): the attention spec gets the
    k8v4 cell size (vLLM's int4 mode with int8 storage), and the layer's key / value / scale views are cut from the
    cell. The store and read paths are the B200 ops int4_kv.patch_int4_kv installed, which dispatch on the key
    view's dtype. Returns False when this vLLM lacks the pieces (logged)."""
    try:
        from vllm.v1.attention.backends import triton_attn
        from vllm.v1.kv_cache_interface import KVQuantMode
        backend, impl = triton_attn.TritonAttentionBackend, triton_attn.TritonAttentionImpl
        mode = KVQuantMode.INT4_PER_TOKEN_HEAD
        stock_spec = backend.customize_spec.__func__
        for name in ("_ensure_scale_caches", "_pth_key_value_caches"):
            getattr(impl, name)
        dtypes = backend.supported_kv_cache_dtypes
    except Exception as e:
        logger.warning("vllm-quantpack-b200: %s not available on this vLLM (%s)", NAME, e)
        return False
    if getattr(impl._pth_key_value_caches, "_quantpack_b200", False):
        return True

    def customize_spec(cls, spec):
        if spec.state_content_bytes is None and spec.kv_quant_mode == mode and spec.dtype == torch.int8:
            return dataclasses.replace(spec, state_content_bytes=cell_bytes(spec.head_size, spec.head_size_v))
        return stock_spec(cls, spec)

    backend.customize_spec = classmethod(_mark(customize_spec))
    _wrap(impl, "_ensure_scale_caches", _ensure_scale_views)
    _wrap(impl, "_pth_key_value_caches", _key_value_views)
    if NAME not in dtypes:
        dtypes.append(NAME)
    return True
