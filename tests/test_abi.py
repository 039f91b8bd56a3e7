"""The C-ABI library builds for sm_100a, loads on a machine without a GPU, and exports every entry point that
include/quantpack_b200.h declares, with the ctypes signatures the Python side binds (no compute call here)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "quantpack_b200.h")


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(qp_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from vllm_quantpack_b200 import _lib, build
    build.build()
    return _lib.load()


def test_header_declares_the_hot_path():
    names = declared()
    for n in ("qp_reshape_and_cache_int4", "qp_reshape_and_cache_k8v4", "qp_paged_decode", "qp_merge_attn_partials",
              "qp_single_rht"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    for name in declared():
        assert hasattr(lib, name), name


def test_python_binding_covers_the_header(lib):
    from vllm_quantpack_b200 import _lib
    assert sorted(_lib.SIGNATURES) == declared()
    src = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    for name, (_, args) in _lib.SIGNATURES.items():
        decl = re.search(name + r"\s*\(([^)]*)\)", src).group(1)
        n_args = 0 if decl.strip() in ("", "void") else decl.count(",") + 1
        assert n_args == len(args), (name, n_args, len(args))


def test_host_side_calls_without_a_gpu(lib):
    assert lib.qp_version() == 100
    # pure host arithmetic: split counts and workspace sizes
    assert lib.qp_decode_num_splits(1, 4, 262144, 148) >= 37
    assert lib.qp_decode_num_splits(1, 4, 64, 148) == 1
    assert lib.qp_decode_workspace_bytes(4, 24, 256, 74) >= 4 * 24 * 74 * 257 * 4
    # argument checks fail before any device work
    rc = lib.qp_paged_decode(0, 0, None, 0, 0, None, 0, 0, 4, 1, None, None, 9, None, 0, None, 16, 0, 0, 264, 0,
                             128, 132, 260, 24, 4, 256, ctypes.c_float(0.0625), None, 0, 0, 0, ctypes.c_float(0.0),
                             None, 0, None, 1, None, 0, None)
    assert rc == 2 and b"rows" in lib.qp_last_error()
