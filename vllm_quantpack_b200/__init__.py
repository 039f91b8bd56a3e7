"""vllm-quantpack-b200: the int4_per_token_head / k8v4_per_token_head KV-cache attention of vllm-quantpack on B200
(sm_100a) kernels.

Installed as a vLLM general plugin (entry point `vllm.general_plugins`, name `quantpack_b200`). `register()` patches
vLLM's int4 KV-cache module with the B200 ops (attention/int4_kv.py) and registers `--kv-cache-dtype
k8v4_per_token_head`, as vllm_quantpack/__init__.py:51-56 does through `patch_int4_kv`. The plugin's other parts
(EXL3 weights, model families, TurboQuant) are not part of this package. The reference plugin may stay installed for
them; whichever int4 patch runs last owns the module, so list this plugin last in VLLM_PLUGINS (or set
VLLM_QUANTPACK_INT4_KV=0 for neither; VLLM_QUANTPACK_B200=0 disables this one alone).
"""
__version__ = "0.1.0"


def _logger():
    try:
        from vllm.logger import init_logger
        return init_logger("vllm.quantpack_b200")
    except Exception:
        import logging
        return logging.getLogger("vllm.quantpack_b200")


def register():
    """vLLM plugin entry point. Returns True when the B200 attention path is installed."""
    import os
    logger = _logger()
    if os.environ.get("VLLM_QUANTPACK_B200", "1") == "0":
        logger.info("vllm-quantpack-b200: disabled by VLLM_QUANTPACK_B200=0")
        return False
    from .attention.int4_kv import patch_int4_kv
    try:
        return patch_int4_kv(logger)
    except Exception as e:      # never take the engine down from a plugin: the stock path stays
        logger.warning("vllm-quantpack-b200: not installed (%s)", e)
        return False
