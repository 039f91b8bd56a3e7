"""Short prefill chunks of several requests in ONE launch (ops.prefill_varlen / qp_prefill_varlen), against the fp64
oracle computed from the same cache bytes. The reference runs every chunk that is not long as one Triton sub-batch
(vllm_quantpack/attention/int4_kv.py:313-323); its tests check such steps row by row against fp64
(tests/test_int4_kv.py:214-229). Cases: 32 chunks of 100 tokens (the step the reference's sub-batch exists for),
chunk lengths that are not multiples of the sub-sequence size, first chunks (no past context), head 512, and the
call under torch's sync debug mode (it reads nothing back to the host)."""
import numpy as np
import pytest
import torch

from oracle import quantpack_oracle as qo
from vllm_quantpack_b200 import _lib
from vllm_quantpack_b200.attention import ops

import qp_testutil as U

pytestmark = pytest.mark.gpu
TOL = 5e-3
BS = 16


def step(device, fmt, qlens, lens, nq=U.NQ, nkv=U.NKV, hs=U.HS, seed=0):
    table, nblocks = U.block_tables(lens, BS, seed=seed + 1)
    cache = U.Cache(fmt, nblocks, BS, device, nkv=nkv, hs=hs)
    for i, n in enumerate(lens):
        cache.fill(table[i], n, seed=seed + 100 + i)
    qb = U.make_queries(qlens, seed=seed + 7, nq=nq, hs=hs)
    return cache, table, qb


def run(device, cache, table, qb, qlens, lens):
    kc, vc, ks, vs = cache.views
    q = U.to_torch(qb, device)
    out = torch.full_like(q, float("nan"))
    cu = torch.tensor(np.concatenate([[0], np.cumsum(qlens)]), dtype=torch.int32, device=device)
    ops.prefill_varlen(q, kc, vc, out, cu_seqlens_q=cu, seqused_k=torch.tensor(lens, dtype=torch.int32, device=device),
                       max_seqlen_k=max(lens), block_table=torch.from_numpy(table).to(device),
                       softmax_scale=cache.hs ** -0.5, k_scale_cache=ks, v_scale_cache=vs)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


def check(cache, table, qb, qlens, lens, got, requests):
    """Every row of the chosen requests against the oracle (each request its own causal chunk)."""
    starts = np.concatenate([[0], np.cumsum(qlens)])
    data = cache.host_bytes()
    for i in requests:
        a, b = starts[i], starts[i + 1]
        want = U.reference(data, cache.layout, qb[a:b], [qlens[i]], [lens[i]], table[i:i + 1])
        err = qo.relerr(got[a:b], want)
        assert err < TOL, f"request {i} ({qlens[i]} tokens over {lens[i]}): relative error {err:.3e}"


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
def test_32_chunks_of_100_tokens(device, fmt):
    qlens = [100] * 32
    lens = [300 + 53 * i for i in range(32)]
    cache, table, qb = step(device, fmt, qlens, lens)
    got = run(device, cache, table, qb, qlens, lens)
    assert np.isfinite(got).all(), "a row was not written"
    check(cache, table, qb, qlens, lens, got, [0, 1, 17, 31])
    assert _lib.device_error() == 0


def test_ragged_chunks_and_first_chunks(device):
    """Lengths that leave partial sub-sequences (1, 7, 33, 63 tokens), first chunks (context == chunk) and a short
    chunk over a long context."""
    qlens = [1, 7, 33, 63, 40, 12, 5]
    lens = [1, 7, 2000, 63, 9000, 12, 30000]
    cache, table, qb = step(device, "int4", qlens, lens, seed=2)
    got = run(device, cache, table, qb, qlens, lens)
    assert np.isfinite(got).all()
    check(cache, table, qb, qlens, lens, got, range(len(qlens)))


def test_head_512(device):
    qlens, lens = [37, 4, 100], [5000, 300, 100]
    cache, table, qb = step(device, "k8v4", qlens, lens, nq=16, nkv=2, hs=512, seed=3)
    got = run(device, cache, table, qb, qlens, lens)
    check(cache, table, qb, qlens, lens, got, range(len(qlens)))


def test_varlen_call_does_not_wait_for_the_gpu(device):
    qlens, lens = [20, 50, 9], [400, 1000, 9]
    cache, table, qb = step(device, "int4", qlens, lens, seed=4)
    first = run(device, cache, table, qb, qlens, lens)           # library load, workspace, sign vector
    kc, vc, ks, vs = cache.views
    q = U.to_torch(qb, device)
    out = torch.empty_like(q)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(qlens)]), dtype=torch.int32, device=device)
    used = torch.tensor(lens, dtype=torch.int32, device=device)
    bt = torch.from_numpy(table).to(device)
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        ops.prefill_varlen(q, kc, vc, out, cu_seqlens_q=cu, seqused_k=used, max_seqlen_k=max(lens), block_table=bt,
                           softmax_scale=U.HS ** -0.5, k_scale_cache=ks, v_scale_cache=vs)
    finally:
        torch.cuda.set_sync_debug_mode("default")
    torch.cuda.synchronize()
    assert np.array_equal(out.float().cpu().numpy(), first)
