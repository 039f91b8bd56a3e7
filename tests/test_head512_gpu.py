"""Head 512 (Gemma 4's global layers) on the GPU, both cache formats, against the fp64 oracle computed from the same
cache bytes: 16 query heads over 2 KV heads, as the reference's own head-512 tests
(tests/test_int4_kv.py:194-210: int4 prefill of 256 queries over one and three 16k segments;
tests/test_k8v4_kv.py:208-225: k8v4 prefill and a decode). Also the MTP decodes (8, 16 and 32 query rows per KV
head), a ragged batch, chunk prefills whose length is not a multiple of the sub-sequence size, the
sequence-parallel partials (`tokens_after_keys`, out_fp32_lse) and a mixed step through the installed router.
The reference's bound is 1e-2; these use 5e-3."""
import logging
import sys
import types

import numpy as np
import pytest
import torch

from oracle import quantpack_oracle as qo
from vllm_quantpack_b200.attention import ops
from vllm_quantpack_b200.attention import seq_parallel as sp

import qp_testutil as U

pytestmark = pytest.mark.gpu
NQ, NKV, HS, BS = 16, 2, 512, 16
TOL = 5e-3


def setup(device, fmt, lens, seed=0):
    table, nblocks = U.block_tables(lens, BS, seed=seed + 1)
    cache = U.Cache(fmt, nblocks, BS, device, nkv=NKV, hs=HS)
    for i, n in enumerate(lens):
        cache.fill(table[i], n, seed=seed + 10 + i)
    return cache, table


def oracle_rows(cache, row_table, q_bits, n, rows):
    """Model-domain fp64 output of chunk rows `rows` (row i: the last position of a context of n - qlen + i + 1)."""
    data, sg, qlen = cache.host_bytes(), U.signs(HS), q_bits.shape[0]
    out = []
    for i in rows:
        q_rot = qo.single_rht(qo.to_f32(q_bits[i:i + 1], "bf16"), sg).astype(np.float64)
        o, _ = qo.attention_from_cache(q_rot, data, cache.layout, row_table, n - qlen + i + 1, HS ** -0.5)
        out.append(qo.single_rht(o.astype(np.float32), sg, inverse=True).astype(np.float64) / HS)
    return np.concatenate(out)


def prefill(device, cache, row_table, q_bits, n, **kw):
    kc, vc, ks, vs = cache.views
    q = U.to_torch(q_bits, device)
    out = kw.pop("out", None)
    out = torch.empty_like(q) if out is None else out
    ops.prefill(q, kc, vc, out, block_row=torch.from_numpy(np.asarray(row_table, np.int32)).to(device), n=n,
                softmax_scale=HS ** -0.5, k_scale_cache=ks, v_scale_cache=vs, **kw)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
@pytest.mark.parametrize("qlens,lens", [([1], [16384]), ([2, 4, 1], [9000, 16385, 300]), ([4], [40000])],
                         ids=["decode-16k", "ragged-mtp", "mtp4-40k"])
def test_decode_matches_fp64(device, fmt, qlens, lens):
    cache, table = setup(device, fmt, lens)
    qb = U.make_queries(qlens, seed=7, nq=NQ, hs=HS)
    got = U.decode(cache, qb, qlens, lens, table)
    want = U.reference(cache.host_bytes(), cache.layout, qb, qlens, lens, table)
    err = qo.relerr(got, want)
    assert err < TOL, f"{fmt} {qlens}: relative error {err:.3e}"


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
@pytest.mark.parametrize("n", [16384, 40000], ids=["one-segment", "3-segments"])
def test_prefill_256_matches_fp64(device, fmt, n):
    cache, table = setup(device, fmt, [n], seed=2)
    qb = U.make_queries([256], seed=9, nq=NQ, hs=HS)
    got = prefill(device, cache, table[0], qb, n).float().cpu().numpy()
    rows = [0, 1, 2, 3, 4, 5, 127, 128, 200, 254, 255]
    err = qo.relerr(got[rows], oracle_rows(cache, table[0], qb, n, rows))
    assert err < TOL, f"{fmt} n {n}: relative error {err:.3e}"


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
def test_prefill_ragged_chunk_and_first_chunk(device, fmt):
    """37 queries (sub-sequences of 4 tokens, the last one of 1) over 5000 tokens; then a first chunk (no past
    context) of 22 tokens, every row checked."""
    cache, table = setup(device, fmt, [5000], seed=4)
    qb = U.make_queries([37], seed=11, nq=NQ, hs=HS)
    got = prefill(device, cache, table[0], qb, 5000).float().cpu().numpy()
    rows = list(range(37))
    assert qo.relerr(got[rows], oracle_rows(cache, table[0], qb, 5000, rows)) < TOL
    qb = U.make_queries([22], seed=12, nq=NQ, hs=HS)
    got = prefill(device, cache, table[0], qb, 22).float().cpu().numpy()
    rows = list(range(22))
    assert qo.relerr(got[rows], oracle_rows(cache, table[0], qb, 22, rows)) < TOL


def test_prefill_split_by_range_folds_to_the_whole(device):
    """Two emulated sequence-parallel ranks: each prefills its own key range (fp32 RHT-domain partial and base-2 lse,
    the earlier range shifted by `tokens_after_keys`), the merge kernel folds them."""
    n, qlen, world = 6144, 64, 2
    cache, table = setup(device, "k8v4", [n], seed=5)
    qb = U.make_queries([qlen], seed=13, nq=NQ, hs=HS)
    part_o = torch.empty((world, qlen, NQ, HS), dtype=torch.float32, device=device)
    part_lse = torch.empty((world, qlen, NQ), dtype=torch.float32, device=device)
    for r in range(world):
        lo, hi, after = sp.sequence_range(n, r, world)
        prefill(device, cache, table[0][lo // BS:(hi + BS - 1) // BS], qb, hi - lo, out=part_o[r],
                out_fp32_lse=part_lse[r], tokens_after_keys=after)
    out = torch.empty((qlen, NQ, HS), dtype=torch.bfloat16, device=device)
    ops.merge_attn_partials(part_o, part_lse, out)
    torch.cuda.synchronize()
    rows = [0, 1, 31, 62, 63]
    got = out.float().cpu().numpy()[rows]
    assert qo.relerr(got, oracle_rows(cache, table[0], qb, n, rows)) < TOL


@pytest.fixture
def stock(monkeypatch):
    from vllm_quantpack_b200.attention import int4_kv
    mod = types.ModuleType("qp_fake_int4_module_hs512")

    def no_stock(*a, **k):
        raise AssertionError("the stock int4 path was reached")

    mod.unified_attention_int4 = no_stock
    mod.reshape_and_cache_int4 = no_stock
    mod.single_rht = lambda x, inverse=False: x
    mod._launch_packed_attn = no_stock
    monkeypatch.setitem(sys.modules, mod.__name__, mod)
    monkeypatch.setattr(int4_kv, "MODULE", mod.__name__)
    assert int4_kv.patch_int4_kv(logging.getLogger("test")) is True
    return mod


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
def test_mixed_step_through_the_router(device, stock, fmt):
    """A 256-query prefill chunk and an MTP decode in one step at head 512 (tests/test_int4_kv.py:214-229 shape),
    through the installed unified_attention_int4: the B200 kernels serve both, nothing reaches the stock path."""
    qlens, lens = [256, 2], [20000, 9000]
    cache, table = setup(device, fmt, lens, seed=6)
    qb = U.make_queries(qlens, seed=15, nq=NQ, hs=HS)
    q = U.to_torch(qb, device)
    kc, vc, ks, vs = cache.views
    cu = torch.tensor([0, 256, 258], dtype=torch.int32, device=device)
    used = torch.tensor(lens, dtype=torch.int32, device=device)
    out = torch.full_like(q, float("nan"))
    stock.unified_attention_int4(
        q, kc, vc, out, cu_seqlens_q=cu, max_seqlen_q=256, seqused_k=used, max_seqlen_k=max(lens),
        softmax_scale=HS ** -0.5, window_size=(-1, -1), block_table=torch.from_numpy(table).to(device), softcap=0.0,
        sinks=None, alibi_slopes=None, use_alibi_sqrt=False, qq_bias=None, output_scale=None, mm_prefix_range=None,
        k_scale_cache=ks, v_scale_cache=vs)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all(), "a row of the step was not written"
    rows = [0, 100, 255]
    assert qo.relerr(got[rows], oracle_rows(cache, table[0], qb[:256], lens[0], rows)) < TOL
    want = U.reference(cache.host_bytes(), cache.layout, qb[256:], [2], [lens[1]], table[1:2])
    assert qo.relerr(got[256:], want) < TOL
