"""Split-KV paged decode on the GPU (K1 + K2) against the fp64 oracle computed from the same cache bytes.

Cases follow the reference's tests (tests/test_int4_kv.py:172-191, 230-249; tests/test_k8v4_kv.py:159-192):
1-4 query tokens at 16k context, a batch of MTP decodes with 4/3/1/4 tokens, both cache formats, plus edge cases
(contexts shorter than a tile, not a multiple of 16, more splits than tiles, block size 16 and 3072) and the
full-size configurations of the benchmark. Bound: relative error < 5e-3 (0.5 %)."""
import numpy as np
import pytest
import torch

from oracle import quantpack_oracle as qo

import qp_testutil as U
from conftest import golden

pytestmark = pytest.mark.gpu
TOL = 5e-3


def run_case(device, fmt, qlens, lens, bs, dtype="bf16", num_splits=None, seed=0, **fill_kw):
    table, nblocks = U.block_tables(lens, bs, seed=seed + 1)
    cache = U.Cache(fmt, nblocks, bs, device)
    for i, n in enumerate(lens):
        cache.fill(table[i], n, seed=seed + i, **fill_kw)
    qb = U.make_queries(qlens, seed=seed + 5, dtype=dtype)
    out = U.decode(cache, qb, qlens, lens, table, dtype=dtype, num_splits=num_splits)
    ref = U.reference(cache.host_bytes(), cache.layout, qb, qlens, lens, table, dtype=dtype)
    errs = []
    at = 0
    for ql in qlens:
        errs.append(qo.relerr(out[at:at + ql], ref[at:at + ql]))
        at += ql
    return errs


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
@pytest.mark.parametrize("qlen", [1, 2, 3, 4], ids=["decode", "mtp-decode", "mtp2-decode", "mtp3-decode"])
def test_decode_matches_fp64(device, fmt, qlen):
    errs = run_case(device, fmt, [qlen], [16384], 16)
    assert errs[0] < TOL, errs


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
def test_scales_spread_and_rising(device, fmt):
    """Per-token K / V magnitudes spread over four orders of magnitude and rising sevenfold along the context (the
    lazy maximum and the value range both grow: the rescale slow path runs)."""
    errs = run_case(device, fmt, [4], [12000], 16, spread=2.0, grow=6.0)
    assert errs[0] < TOL, errs


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
def test_batched_mtp_decodes(device, fmt):
    """Sequences with 4, 3, 1 and 4 query tokens in one step (tests/test_int4_kv.py:230-249)."""
    errs = run_case(device, fmt, [4, 3, 1, 4], [20000, 9000, 16384, 3072], 16)
    assert max(errs) < TOL, errs


@pytest.mark.parametrize("qlens,lens", [([1], [1]), ([2], [2]), ([4], [5]), ([1], [15]), ([3], [17]), ([4], [64]),
                                        ([4], [65]), ([2], [1000]), ([1, 4, 2], [33, 129, 4097])],
                         ids=["n1", "n2", "n5", "n15", "n17", "n64", "n65", "n1000", "ragged"])
def test_short_and_ragged_contexts(device, qlens, lens):
    errs = run_case(device, "int4", qlens, lens, 16)
    assert max(errs) < TOL, errs


def test_more_splits_than_tiles(device):
    errs = run_case(device, "int4", [4], [300], 16, num_splits=37)
    assert errs[0] < TOL, errs


@pytest.mark.parametrize("bs", [32, 3072])
def test_block_sizes(device, bs):
    errs = run_case(device, "k8v4", [2], [9000], bs)
    assert errs[0] < TOL, errs


def test_fp16_model(device):
    errs = run_case(device, "int4", [4], [5000], 16, dtype="f16")
    assert errs[0] < TOL, errs


def test_split_count_does_not_change_the_result(device):
    """Splits only regroup the same keys: outputs agree within fp32 re-association."""
    table, nblocks = U.block_tables([12345], 16)
    cache = U.Cache("int4", nblocks, 16, device)
    cache.fill(table[0], 12345, seed=9)
    qb = U.make_queries([3])
    outs = [U.decode(cache, qb, [3], [12345], table, num_splits=s) for s in (1, 7, 64, 193)]
    for o in outs[1:]:
        assert qo.relerr(o, outs[0]) < 2e-3


@pytest.mark.parametrize("fmt,qlens,lens", [("int4", [2], [131072]), ("int4", [4], [262144]),
                                            ("k8v4", [4], [262144])],
                         ids=["c1-131k-mtp1", "c2a-262k-mtp3", "c4-k8v4-262k"])
def test_full_size_configs(device, fmt, qlens, lens):
    errs = run_case(device, fmt, qlens, lens, 16)
    assert errs[0] < TOL, errs


def test_batch32_config(device):
    """c2b: 32 requests x 32k context x 2 query tokens (the oracle checks every 8th request)."""
    qlens, lens = [2] * 32, [32768] * 32
    table, nblocks = U.block_tables(lens, 16)
    cache = U.Cache("int4", nblocks, 16, device)
    for i in range(32):
        cache.fill(table[i], lens[i], seed=100 + i)
    qb = U.make_queries(qlens)
    out = U.decode(cache, qb, qlens, lens, table)
    data = cache.host_bytes()
    for i in range(0, 32, 8):
        ref = U.reference(data, cache.layout, qb[2 * i:2 * i + 2], [2], [lens[i]], table[i:i + 1])
        assert qo.relerr(out[2 * i:2 * i + 2], ref) < TOL, i


ATTN = golden("attn_i8.npz")


def test_no_worse_than_reference_kernel(device):
    """On the golden case a1 (3 query tokens x 6 heads, 200 keys), the B200 decode's error against the oracle is no
    larger than that of the reference's own kernel (`prefill_sequence_i8`) on the same cache and rotated queries."""
    from vllm_quantpack_b200.attention import ops
    nq, nkv, hs, bs, nblocks, n, qlen = (int(x) for x in ATTN["a1.meta"])
    layout = qo.CacheLayout("int4", nblocks, nkv, bs, hs)
    data, table = ATTN["a1.cache"], ATTN["a1.table"]
    q_rot = qo.bf16_to_f32(ATTN["a1.q_rot"])
    K, V = qo.read_sequence(data, layout, table, n)
    ref, _ = qo.attention_rht_domain(q_rot, K, V, n, hs ** -0.5, hs)
    ref_err = qo.relerr(qo.bf16_to_f32(ATTN["a1.out"]), ref)
    kv = torch.from_numpy(data.reshape(nblocks, nkv, bs, hs + 8).copy()).to(device)
    base = torch.tensor([], dtype=torch.float32, device=device).set_(kv.untyped_storage())
    st = [s // 4 for s in kv.stride()]
    ks = torch.as_strided(base, (nblocks, bs, nkv), (st[0], st[2], st[1]), hs // 2 // 4)
    vs = torch.as_strided(base, (nblocks, bs, nkv), (st[0], st[2], st[1]), (hs // 2 + 4 + hs // 2) // 4)
    kc, vc = kv.transpose(1, 2).split(hs // 2 + 4, dim=-1)
    q = U.to_torch(ATTN["a1.q_rot"], device)
    out = torch.empty(q.shape, dtype=torch.float32, device=device)
    lse = torch.empty(q.shape[:2], dtype=torch.float32, device=device)
    ops.paged_decode(q, kc, vc, out, cu_seqlens_q=torch.tensor([0, qlen], dtype=torch.int32, device=device),
                     max_seqlen_q=qlen, seqused_k=torch.tensor([n], dtype=torch.int32, device=device), max_seqlen_k=n,
                     softmax_scale=hs ** -0.5, block_table=torch.from_numpy(table.astype(np.int32))[None].to(device),
                     k_scale_cache=ks, v_scale_cache=vs, q_rotated=True, out_fp32_lse=lse)
    torch.cuda.synchronize()
    err = qo.relerr(out.cpu().numpy(), ref)
    assert err <= max(ref_err, 1e-4), f"B200 {err:.3e} vs reference kernel {ref_err:.3e}"
    # the base-2 lse of the RHT-domain partial agrees with the oracle's natural-log lse
    _, lse_ref = qo.attention_rht_domain(q_rot, K, V, n, hs ** -0.5, hs)
    assert np.allclose(lse.cpu().numpy() / np.log2(np.e), lse_ref, atol=2e-3)


def test_no_device_timeouts(device):
    from vllm_quantpack_b200 import _lib
    run_case(device, "int4", [4], [5000], 16)
    assert _lib.device_error() == 0


def test_decode_step_in_cuda_graph(device):
    """The decode path is graph-capturable (no host sync, preallocated workspace): a captured step replays to the
    same output as a direct call, and a replay after new query values reflects them."""
    from vllm_quantpack_b200.attention import ops
    n, qlen = 8192, 4
    table, nblocks = U.block_tables([n], 16)
    cache = U.Cache("int4", nblocks, 16, device)
    cache.fill(table[0], n, seed=2)
    kc, vc, ks, vs = cache.views
    q = U.to_torch(U.make_queries([qlen], seed=4), device)
    out = torch.empty_like(q)
    args = dict(cu_seqlens_q=torch.tensor([0, qlen], dtype=torch.int32, device=device), max_seqlen_q=qlen,
                seqused_k=torch.tensor([n], dtype=torch.int32, device=device), max_seqlen_k=n,
                softmax_scale=U.HS ** -0.5, block_table=torch.from_numpy(table).to(device), k_scale_cache=ks,
                v_scale_cache=vs)
    ops.paged_decode(q, kc, vc, out, **args)  # warm-up: workspace and sign vector allocated outside the capture
    torch.cuda.synchronize()
    ref = out.clone()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g):
            ops.paged_decode(q, kc, vc, out, **args)
    torch.cuda.current_stream().wait_stream(s)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    q.copy_(U.to_torch(U.make_queries([qlen], seed=5), device))
    g.replay()
    direct = torch.empty_like(out)
    ops.paged_decode(q, kc, vc, direct, **args)
    torch.cuda.synchronize()
    assert torch.equal(out, direct) and not torch.equal(out, ref)
