"""ctypes binding of libquantpack_b200.so (the C ABI declared in include/quantpack_b200.h).

There is no fallback: if the library is missing or does not load, every op raises. Build it with
`python -m vllm_quantpack_b200.build` (nvcc, sm_100a)."""
import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libquantpack_b200.so")

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_F = ctypes.c_float

# name -> (restype, argtypes); must match include/quantpack_b200.h
SIGNATURES = {
    "qp_version": (_I, []),
    "qp_last_error": (ctypes.c_char_p, []),
    "qp_device_error": (_I, [ctypes.POINTER(ctypes.c_int)]),
    "qp_reshape_and_cache_int4": (_I, [_P, _P, _I, _L, _I, _I, _L, _L, _L, _L, _P, _P, _I, _L, _L, _L, _L, _L, _L, _L,
                                       _P, _I, _P]),
    "qp_reshape_and_cache_k8v4": (_I, [_P, _P, _I, _L, _I, _I, _L, _L, _L, _L, _P, _P, _I, _L, _L, _L, _L, _L, _L, _L,
                                       _P, _I, _P]),
    "qp_single_rht": (_I, [_P, _P, _L, _I, _I, _P, _P]),
    "qp_decode_num_splits": (_I, [_I, _I, _I, _I]),
    "qp_decode_workspace_bytes": (_L, [_L, _I, _I, _I]),
    "qp_paged_decode": (_I, [_I, _I, _P, _L, _L, _P, _L, _L, _L, _I, _P, _P, _I, _P, _L, _P, _I, _L, _L, _L, _L, _L,
                             _L, _L, _I, _I, _I, _F, _P, _I, _I, _I, _F, _P, _I, _P, _I, _P, _L, _P]),
    "qp_paged_decode_static": (_I, [_I, _I, _P, _L, _L, _P, _L, _L, _L, _I, _P, _P, _I, _P, _L, _P, _I, _L, _L, _L, _L,
                                    _L, _L, _L, _I, _I, _I, _F, _P, _I, _I, _P, _I, _P]),
    "qp_prefill_workspace_bytes": (_L, [_I, _I, _I, _I, _I, _I]),
    "qp_prefill": (_I, [_I, _I, _P, _L, _L, _P, _L, _L, _I, _I, _P, _P, _I, _L, _L, _L, _L, _L, _L, _L, _I, _I, _I, _F,
                        _P, _I, _I, _I, _P, _P, _L, _P]),
    "qp_prefill_varlen_workspace_bytes": (_L, [_L, _I, _I, _I, _I, _I]),
    "qp_prefill_varlen": (_I, [_I, _I, _P, _L, _L, _P, _L, _L, _L, _I, _P, _P, _I, _P, _L, _P, _I, _L, _L, _L, _L, _L,
                               _L, _L, _I, _I, _I, _F, _P, _I, _I, _F, _P, _I, _P, _P, _L, _P]),
    "qp_peer_exchange_bytes": (_L, [_I, _L, _I, _I]),
    "qp_peer_partial_offset": (_L, [_I, _L, _I, _I, _I]),
    "qp_fold_peer_partials": (_I, [_I, _I, _L, _I, _I, _I, _P, ctypes.c_uint32, _I, _P, _L, _L, _P, _P, _P]),
    "qp_merge_attn_partials": (_I, [_I, _I, _L, _I, _I, _P, _L, _L, _L, _P, _L, _L, _L, _I, _P, _L, _L, _P, _P, _P]),
}

_lock = threading.Lock()
_lib = None


class QuantpackError(RuntimeError):
    pass


def load():
    """The loaded library (raises QuantpackError when it is missing: there is no CPU path)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise QuantpackError(f"{LIB_PATH} is missing: build it with `python -m vllm_quantpack_b200.build`")
            try:
                lib = ctypes.CDLL(LIB_PATH)
            except OSError as e:
                raise QuantpackError(f"cannot load {LIB_PATH}: {e}") from e
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def call(name, *args):
    """Call a qp_* entry point; a non-zero return raises QuantpackError with the library's message."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != 0:
        msg = lib.qp_last_error().decode(errors="replace")
        raise QuantpackError(f"{name}: {msg} (code {rc})")
    return rc


def device_error():
    """Read and clear the device error word of the current device (synchronous)."""
    code = ctypes.c_int(0)
    call("qp_device_error", ctypes.byref(code))
    return code.value
