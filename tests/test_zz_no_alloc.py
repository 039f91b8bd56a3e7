"""qp_paged_decode_static: the split-KV decode for callers that cannot allocate device memory.

Some hosts of this library never call cudaMalloc after start-up (an engine that owns all device memory in its own
pool, embedded code with no device allocator), so they cannot hand qp_paged_decode a workspace. The static variant
keeps its split partials in a fixed 32 MiB array inside the library. These tests call it through the C ABI and check
that two calls in a row (the second one finds the first call's partials still in the array) give the output of the
workspace entry point and of the fp64 oracle, within the tolerance of the decode tests; and that a request whose
partials do not fit is refused with a clear error. This file is collected last on purpose."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import quantpack_oracle as qo

import qp_testutil as U

pytestmark = pytest.mark.gpu
TOL = 5e-3          # the decode tests' tolerance (tests/test_decode_gpu.py)


def _static_decode(lib, cache, q, out, cu, used, table, qlen, num_splits, out_mode=0, lse=None):
    from vllm_quantpack_b200.attention import ops, rht
    kc, vc, ks, vs = cache.views
    lay = ops.CacheLayout(kc, vc, ks, vs, U.HS)
    return lib.qp_paged_decode_static(
        lay.fmt, 0, q.data_ptr(), q.stride(0), q.stride(1), out.data_ptr(), out.stride(0), out.stride(1),
        q.shape[0], cu.shape[0] - 1, cu.data_ptr(), used.data_ptr(), qlen, table.data_ptr(), table.stride(0),
        *lay.args(), U.NQ, U.NKV, U.HS, ctypes.c_float(U.HS ** -0.5), rht.device_sign_bits(U.HS, q.device).data_ptr(),
        0, out_mode, None if lse is None else lse.data_ptr(), num_splits,
        torch.cuda.current_stream(q.device).cuda_stream)


def _case(device, fmt, qlens, lens, seed):
    table_np, nblocks = U.block_tables(lens, 16, seed=seed)
    cache = U.Cache(fmt, nblocks, 16, device)
    for i, n in enumerate(lens):
        cache.fill(table_np[i], n, seed=40 + seed + i)
    q = U.to_torch(U.make_queries(qlens, seed=8 + seed), device)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(qlens)]), dtype=torch.int32, device=device)
    used = torch.tensor(lens, dtype=torch.int32, device=device)
    return cache, q, cu, used, torch.from_numpy(table_np).to(device)


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
def test_static_scratch_decode_matches_workspace_decode(device, fmt):
    from vllm_quantpack_b200 import _lib
    from vllm_quantpack_b200.attention import ops
    lib = _lib.load()
    qlens, lens = [4, 1, 3], [20000, 777, 4096]
    table_np, nblocks = U.block_tables(lens, 16)
    cache = U.Cache(fmt, nblocks, 16, device)
    for i, n in enumerate(lens):
        cache.fill(table_np[i], n, seed=40 + i)
    kc, vc, ks, vs = cache.views
    qb = U.make_queries(qlens, seed=8)
    q = U.to_torch(qb, device)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(qlens)]), dtype=torch.int32, device=device)
    used = torch.tensor(lens, dtype=torch.int32, device=device)
    table = torch.from_numpy(table_np).to(device)
    splits = ops.decode_num_splits(len(lens), U.NKV, max(lens), ops.sm_count(device))
    oracle = U.reference(cache.host_bytes(), cache.layout, qb, qlens, lens, table_np)
    want = torch.empty_like(q)
    ops.paged_decode(q, kc, vc, want, cu_seqlens_q=cu, max_seqlen_q=max(qlens), seqused_k=used,
                     max_seqlen_k=max(lens), softmax_scale=U.HS ** -0.5, block_table=table, k_scale_cache=ks,
                     v_scale_cache=vs, num_splits=splits)
    want = want.float().cpu().numpy()
    for call in range(2):
        out = torch.full_like(q, float("nan"))
        rc = _static_decode(lib, cache, q, out, cu, used, table, max(qlens), splits)
        assert rc == 0, lib.qp_last_error().decode()
        torch.cuda.synchronize()
        got = out.float().cpu().numpy()
        assert np.isfinite(got).all(), f"call {call}: output not written"
        err = qo.relerr(got, want)
        assert err < TOL, f"call {call}: static-scratch decode differs from the workspace decode by {err:.3e}"
        err = qo.relerr(got, oracle)
        assert err < TOL, f"call {call}: static-scratch decode differs from the fp64 oracle by {err:.3e}"
        if call == 0:
            # between the two compared calls, a bigger request with more splits and the other cache format fills
            # the array with partials of another shape: the next call must not read any of them
            c2, q2, cu2, used2, t2 = _case(device, "k8v4" if fmt == "int4" else "int4", [4, 4, 4, 4],
                                           [30000, 100, 9000, 64], seed=3)
            o2 = torch.empty_like(q2)
            rc = _static_decode(lib, c2, q2, o2, cu2, used2, t2, 4, 60)   # 16 x 24 x 60 partials: 24 MB
            assert rc == 0, lib.qp_last_error().decode()
    assert _lib.device_error() == 0


def test_static_scratch_rht_domain_output_with_lse(device):
    """out_mode 1 (fp32 RHT-domain output and its base-2 lse, the partial a sequence-parallel rank exchanges)
    against the workspace entry point, twice in a row; out_mode 2 (partials left in the array) is refused."""
    from vllm_quantpack_b200 import _lib
    from vllm_quantpack_b200.attention import ops
    lib = _lib.load()
    qlens, lens = [2, 4], [12000, 3000]
    cache, q, cu, used, table = _case(device, "int4", qlens, lens, seed=5)
    kc, vc, ks, vs = cache.views
    splits = ops.decode_num_splits(len(lens), U.NKV, max(lens), ops.sm_count(device))
    want = torch.empty(q.shape, dtype=torch.float32, device=device)
    want_lse = torch.empty(q.shape[:2], dtype=torch.float32, device=device)
    ops.paged_decode(q, kc, vc, want, cu_seqlens_q=cu, max_seqlen_q=max(qlens), seqused_k=used,
                     max_seqlen_k=max(lens), softmax_scale=U.HS ** -0.5, block_table=table, k_scale_cache=ks,
                     v_scale_cache=vs, num_splits=splits, out_fp32_lse=want_lse)
    for call in range(2):
        out = torch.full_like(want, float("nan"))
        lse = torch.full_like(want_lse, float("nan"))
        rc = _static_decode(lib, cache, q, out, cu, used, table, max(qlens), splits, out_mode=1, lse=lse)
        assert rc == 0, lib.qp_last_error().decode()
        torch.cuda.synchronize()
        assert qo.relerr(out.cpu().numpy(), want.cpu().numpy()) < TOL, f"call {call}"
        assert np.allclose(lse.cpu().numpy(), want_lse.cpu().numpy(), atol=1e-3), f"call {call}: lse"
    rc = _static_decode(lib, cache, q, out, cu, used, table, max(qlens), splits, out_mode=2)
    assert rc == 1 and b"out_mode" in lib.qp_last_error()


def test_static_scratch_refuses_requests_that_do_not_fit(device):
    from vllm_quantpack_b200 import _lib
    lib = _lib.load()
    cache = U.Cache("int4", 4, 16, device)
    q = torch.zeros((4096, U.NQ, U.HS), dtype=torch.bfloat16, device=device)
    out = torch.empty_like(q)
    cu = torch.tensor([0, 4096], dtype=torch.int32, device=device)
    used = torch.tensor([64], dtype=torch.int32, device=device)
    table = torch.zeros((1, 4), dtype=torch.int32, device=device)
    # 4096 tokens x 24 heads x 64 splits of 1 KiB partials is about 6.4 GB: far more than the 32 MiB array
    rc = _static_decode(lib, cache, q, out, cu, used, table, 1, 64)
    assert rc == 4, rc
    assert b"static scratch" in lib.qp_last_error()
