"""k8v4_per_token_head KV cache: int8 keys and int4 values, both in the randomized-Hadamard domain.

Same page cell, views, dtype registration and backend patches as the reference plugin
(vllm_quantpack/attention/k8v4_kv.py), with the store running on the B200 store kernel instead of Triton.

Page cell, head size hs: [K hs int8 | K scale f32 | V hs/2 bytes | V scale f32] = 1.5 hs + 8 bytes (392 at hs 256;
int4 264). The value half is exactly the int4 cell's value half (nibbles, fp32 scale with the 4-bit zero point in its
low mantissa bits). The format is identified by the int8 storage dtype (the stock int4 cache is uint8).
"""
import torch

NAME = "k8v4_per_token_head"
SCALE_BYTES = 4


def cell_bytes(head_size, head_size_v):
    """Bytes of one (token, KV head) cell: int8 key, packed value, one fp32 scale each (k8v4_kv.py:31-33)."""
    return head_size + head_size_v // 2 + 2 * SCALE_BYTES


def is_k8v4(key_cache):
    """True for the key view of a k8v4 cache (the int4 cache views are uint8) (k8v4_kv.py:36-38)."""
    return key_cache.dtype == torch.int8


def views(kv_cache, head_size, head_size_v=None):
    """(key, value, key scale, value scale) views of the logical (blocks, KV heads, block size, cell) int8 cache.

    key (blocks, block size, KV heads, hs) int8; value (..., hs_v / 2) uint8; scales (blocks, block size, KV heads)
    fp32 over the same storage. The cache may be physically NHD: only its strides are used (k8v4_kv.py:41-65)."""
    head_size_v = head_size if head_size_v is None else head_size_v
    nblocks, nkv, block_size, cell = kv_cache.shape
    if kv_cache.element_size() != 1 or cell != cell_bytes(head_size, head_size_v):
        raise ValueError(f"{NAME}: cache cell of {cell} x {kv_cache.element_size()} bytes, expected "
                         f"{cell_bytes(head_size, head_size_v)} for head sizes {head_size} / {head_size_v}")
    v_at = head_size + SCALE_BYTES
    t = kv_cache.transpose(1, 2)
    key = t[..., :head_size]
    value = t[..., v_at:v_at + head_size_v // 2].view(torch.uint8)
    st = kv_cache.stride()
    if any(s % 4 for s in st[:3]) or kv_cache.storage_offset() % 4 or head_size % 4 or (head_size_v // 2) % 4:
        raise ValueError(f"{NAME}: fp32 scales are not 4-byte aligned (strides {tuple(st)}, head {head_size})")
    base = torch.tensor([], dtype=torch.float32, device=kv_cache.device).set_(kv_cache.untyped_storage())
    off = kv_cache.storage_offset() // 4

    def scales(byte_at):
        return torch.as_strided(base, (nblocks, block_size, nkv), (st[0] // 4, st[2] // 4, st[1] // 4),
                                off + byte_at // 4)

    return key, value, scales(head_size), scales(v_at + head_size_v // 2)


def store(key, value, key_cache, value_cache, slot_mapping, *, k_scale_cache, v_scale_cache):
    """Rotate (RHT), quantize and write key / value into the k8v4 cache views in one fused kernel
    (replaces k8v4_kv.py:68-86, which rotates in torch and then launches `_store_k8v4`)."""
    from . import ops
    if value.shape[2] % 2:
        raise ValueError(f"{NAME}: odd value head size {value.shape[2]}")
    ops.reshape_and_cache_int4(key, value, key_cache, value_cache, slot_mapping, k_scale_cache=k_scale_cache,
                               v_scale_cache=v_scale_cache)


def register_dtype(logger):
    """Make `--kv-cache-dtype k8v4_per_token_head` a valid option. False on a vLLM without the dtype registry
    (k8v4_kv.py:89-110)."""
    try:
        from vllm.config import cache as cache_config
        from vllm.v1.kv_cache_interface import KVQuantMode
        registry, lookup = cache_config.register_kv_cache_dtype, cache_config.get_kv_cache_dtype_handler
        mode = KVQuantMode.INT4_PER_TOKEN_HEAD
    except Exception as e:
        logger.debug("vllm-quantpack-b200: %s not registered (%s)", NAME, e)
        return False
    if lookup(NAME) is None:
        class Handler:
            name = NAME

            def torch_dtype(self):
                return torch.int8

            def quant_mode(self):
                return mode

        registry(NAME)(Handler)
    return True


def patch_backend(stock, logger):
    """Teach vLLM's Triton backend the k8v4 page cell and views (k8v4_kv.py:113-166). The store and read paths are
    the B200 ops installed by int4_kv.patch_int4_kv, which dispatch on the key view's dtype."""
    try:
        from vllm.v1.attention.backends import triton_attn
        from vllm.v1.kv_cache_interface import KVQuantMode
        backend, impl = triton_attn.TritonAttentionBackend, triton_attn.TritonAttentionImpl
        stock_spec = backend.customize_spec.__func__
        stock_scales, stock_views = impl._ensure_scale_caches, impl._pth_key_value_caches
        supported = backend.supported_kv_cache_dtypes
    except Exception as e:
        logger.warning("vllm-quantpack-b200: %s not available on this vLLM (%s)", NAME, e)
        return False
    if getattr(stock_scales, "_quantpack_b200", False):
        return True

    def customize_spec(cls, spec):
        if (spec.state_content_bytes is None and spec.kv_quant_mode == KVQuantMode.INT4_PER_TOKEN_HEAD
                and spec.dtype == torch.int8):
            from dataclasses import replace
            return replace(spec, state_content_bytes=cell_bytes(spec.head_size, spec.head_size_v))
        return stock_spec(cls, spec)

    def _ensure_scale_caches(self, kv_cache):
        if self.kv_cache_dtype != NAME:
            return stock_scales(self, kv_cache)
        if self._k_scale_cache is None:
            _, _, ks, vs = views(kv_cache, self.head_size)
            ks.fill_(1.0)
            vs.fill_(1.0)
            self._k_scale_cache, self._v_scale_cache = ks, vs

    def _pth_key_value_caches(self, kv_cache):
        if self.kv_cache_dtype != NAME:
            return stock_views(self, kv_cache)
        self._ensure_scale_caches(kv_cache)
        key, value, _, _ = views(kv_cache, self.head_size)
        return key, value

    _ensure_scale_caches._quantpack_b200 = True
    backend.customize_spec = classmethod(customize_spec)
    impl._ensure_scale_caches = _ensure_scale_caches
    impl._pth_key_value_caches = _pth_key_value_caches
    if NAME not in supported:
        supported.append(NAME)
    return True
