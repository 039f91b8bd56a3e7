"""Chunk prefill on the tcgen05 tensor cores (K3) against the fp64 oracle computed from the same cache bytes.

Cases follow the reference's prefill tests (tests/test_int4_kv.py:172-191, 318-339; tests/test_k8v4_kv.py:159-173):
chunks of 40 / 256 / 1000 queries, a first chunk (no past context), block sizes 16 and 3072, both cache formats,
fp16, and the full configuration of the benchmark (1024 queries over 229,376 cached tokens). Long cases check a
sample of query rows (every head), each row against its own causal prefix. Bound: relative error < 5e-3."""
import numpy as np
import pytest
import torch

from oracle import quantpack_oracle as qo

import qp_testutil as U
from conftest import golden

pytestmark = pytest.mark.gpu
TOL = 5e-3


def run_prefill(device, cache, table_row, q_bits, n, dtype="bf16"):
    from vllm_quantpack_b200.attention import ops
    kc, vc, ks, vs = cache.views
    q = U.to_torch(q_bits, device, dtype)
    out = torch.empty_like(q)
    ops.prefill(q, kc, vc, out, block_row=torch.from_numpy(np.asarray(table_row, np.int32)).to(device), n=n,
                softmax_scale=cache.hs ** -0.5, k_scale_cache=ks, v_scale_cache=vs)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


def reference_rows(cache_bytes, layout, table_row, q_bits, n, rows, dtype="bf16"):
    """Oracle output of the chunk's query rows `rows`: row i is the last position of a context of n - qlen + i + 1.
    Each run of consecutive rows is one oracle call (its last row's context, causal inside the run)."""
    hs = layout.head_size
    sg = U.signs(hs)
    qlen = q_bits.shape[0]
    out = []
    rows = list(rows)
    a = 0
    while a < len(rows):
        b = a + 1
        while b < len(rows) and rows[b] == rows[b - 1] + 1:
            b += 1
        lo, hi = rows[a], rows[b - 1] + 1
        q_rot = qo.single_rht(qo.to_f32(q_bits[lo:hi], dtype), sg).astype(np.float64)
        o, _ = qo.attention_from_cache(q_rot, cache_bytes, layout, table_row, n - qlen + hi, hs ** -0.5)
        out.append(qo.single_rht(o.astype(np.float32), sg, inverse=True).astype(np.float64) / hs)
        a = b
    return np.concatenate(out)


def prefill_case(device, fmt, qlen, n, bs, dtype="bf16", rows=None, seed=0, **fill_kw):
    table, nblocks = U.block_tables([n], bs, seed=seed + 1)
    cache = U.Cache(fmt, nblocks, bs, device)
    cache.fill(table[0], n, seed=seed, **fill_kw)
    qb = U.make_queries([qlen], seed=seed + 3, dtype=dtype)
    out = run_prefill(device, cache, table[0], qb, n, dtype)
    rows = list(range(qlen)) if rows is None else rows
    ref = reference_rows(cache.host_bytes(), cache.layout, table[0], qb, n, rows, dtype)
    return qo.relerr(out[rows], ref)


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
def test_small_chunk(device, fmt):
    assert prefill_case(device, fmt, 40, 300, 16) < TOL


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
def test_chunk_256_over_16k(device, fmt):
    err = prefill_case(device, fmt, 256, 16384, 16, rows=[0, 1, 63, 64, 127, 128, 200, 255])
    assert err < TOL, err


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
def test_scales_spread_and_rising(device, fmt):
    """Per-token K / V magnitudes spread over four orders of magnitude inside every tile and rising sevenfold along
    the sequence: large, peaked logits (a key scale rounded into the fp16 operand showed here as 7e-3, a zero point
    rounded apart from the scale as 6e-2) and row maxima / value exponents that keep growing (the O rescale paths
    run). Measured 1.8-1.9e-3."""
    err = prefill_case(device, fmt, 256, 8192, 16, rows=[0, 1, 100, 128, 255], spread=2.0, grow=6.0)
    assert err < TOL, err


def test_first_chunk_without_past(device):
    assert prefill_case(device, "int4", 64, 64, 16) < TOL


def test_odd_chunk_block_3072(device):
    err = prefill_case(device, "int4", 1000, 40000, 3072, rows=[0, 333, 500, 999])
    assert err < TOL, err


def test_fp16_model(device):
    assert prefill_case(device, "int4", 100, 2000, 16, dtype="f16") < TOL


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
def test_full_size_chunk(device, fmt):
    """c3: 1024 queries over 229,376 cached tokens (+ the chunk's own 1024), both cache formats. Every row (all 24
    heads) of the first and last 22 tokens: the first and last 128-row M-tiles of every KV head, each summed from
    pieces of every key chunk and of the CTAs that split a chunk's run, plus a middle token."""
    rows = list(range(0, 22)) + [511] + list(range(1002, 1024))
    err = prefill_case(device, fmt, 1024, 229376 + 1024, 16, rows=rows)
    assert err < TOL, err


ATTN = golden("attn_i8.npz")


def test_no_worse_than_reference_kernel(device):
    """Golden case a0 (40 queries x 4 heads over 300 keys): the B200 prefill's error against the oracle is no larger
    than that of the reference's own kernel (`prefill_sequence_i8`) on the same cache and rotated queries."""
    from vllm_quantpack_b200.attention import ops
    nq, nkv, hs, bs, nblocks, n, qlen = (int(x) for x in ATTN["a0.meta"])
    layout = qo.CacheLayout("int4", nblocks, nkv, bs, hs)
    data, table = ATTN["a0.cache"], ATTN["a0.table"]
    q_rot = qo.bf16_to_f32(ATTN["a0.q_rot"])
    K, V = qo.read_sequence(data, layout, table, n)
    ref, lse_ref = qo.attention_rht_domain(q_rot, K, V, n, hs ** -0.5, hs)
    ref_err = qo.relerr(qo.bf16_to_f32(ATTN["a0.out"]), ref)
    kv = torch.from_numpy(data.reshape(nblocks, nkv, bs, hs + 8).copy()).to(device)
    base = torch.tensor([], dtype=torch.float32, device=device).set_(kv.untyped_storage())
    st = [s // 4 for s in kv.stride()]
    ks = torch.as_strided(base, (nblocks, bs, nkv), (st[0], st[2], st[1]), hs // 2 // 4)
    vs = torch.as_strided(base, (nblocks, bs, nkv), (st[0], st[2], st[1]), (hs // 2 + 4 + hs // 2) // 4)
    kc, vc = kv.transpose(1, 2).split(hs // 2 + 4, dim=-1)
    q = U.to_torch(ATTN["a0.q_rot"], device)
    out = torch.empty(q.shape, dtype=torch.float32, device=device)
    lse = torch.empty(q.shape[:2], dtype=torch.float32, device=device)
    ops.prefill(q, kc, vc, out, block_row=torch.from_numpy(table.astype(np.int32)).to(device), n=n,
                softmax_scale=hs ** -0.5, k_scale_cache=ks, v_scale_cache=vs, q_rotated=True, out_fp32_lse=lse)
    torch.cuda.synchronize()
    err = qo.relerr(out.cpu().numpy(), ref)
    assert err <= max(ref_err, 1e-4), f"B200 {err:.3e} vs reference kernel {ref_err:.3e}"
    assert np.allclose(lse.cpu().numpy() / np.log2(np.e), lse_ref, atol=2e-3)


def test_no_device_timeouts(device):
    from vllm_quantpack_b200 import _lib
    prefill_case(device, "int4", 40, 300, 16)
    assert _lib.device_error() == 0
