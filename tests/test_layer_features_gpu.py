"""Sliding-window, softcap and sink layers on the split-KV kernel (K1) and its merge (K2), against the fp64 oracle
computed from the same cache bytes.

vLLM passes window_size = (w, 0) and its int4 kernel (the one the reference patches) masks with SLIDING_WINDOW =
1 + w: the query at position p sees keys p - SLIDING_WINDOW + 1 .. p (vllm/v1/attention/ops/
triton_attention_helpers.py:196-218, triton_unified_attention.py:533-536, vLLM 0.22). The reference serves such layers
on its patched Triton kernel for both cache formats (vllm_quantpack/attention/int4_kv.py:127-146, 302-307). Cases:
windows whose starts for the 4 MTP tokens straddle a 128-key tile (rows that see no key in the first tile of a split
and open in the next), every split count from one split over the whole window to one tile per split, a window of one
key, windows wider than the context, ragged MTP batches, keys whose magnitudes spread and rise (the rescale path),
head 512, the varlen launch of short chunks, a sequence split over two ranges (the window reaching into the earlier
rank's range) and a mixed step through the installed `unified_attention_int4`. The logit softcap (vLLM's
apply_softcap, softcap * tanh(S / softcap): triton_attention_helpers.py:28-36) with caps that bend most scores (3)
and Gemma 2's (50), alone and with a window, in decode, the varlen launch and the router. Attention sinks (vLLM:
the row maximum starts at the sink with sum 1 in one segment, triton_attention_helpers.py:108-138), folded once by
the merge whatever the split count, in decode, varlen and a router step with every feature at once. Bound: relative
error < 5e-3."""
import numpy as np
import pytest
import torch

from oracle import quantpack_oracle as qo
from vllm_quantpack_b200 import _lib
from vllm_quantpack_b200.attention import ops
from vllm_quantpack_b200.attention import seq_parallel as sp

import qp_testutil as U
from test_router_gpu import mixed_step, stock  # noqa: F401  (the stand-in int4 module the router patches)

pytestmark = pytest.mark.gpu
TOL = 5e-3
BS = 16


def build(device, fmt, qlens, lens, nq=U.NQ, nkv=U.NKV, hs=U.HS, seed=0, **fill_kw):
    table, nblocks = U.block_tables(lens, BS, seed=seed + 1)
    cache = U.Cache(fmt, nblocks, BS, device, nkv=nkv, hs=hs)
    for i, n in enumerate(lens):
        cache.fill(table[i], n, seed=seed + i, **fill_kw)
    qb = U.make_queries(qlens, seed=seed + 5, nq=nq, hs=hs)
    return cache, table, qb


def errors(got, ref, qlens):
    starts = np.concatenate([[0], np.cumsum(qlens)])
    return [qo.relerr(got[a:b], ref[a:b]) for a, b in zip(starts[:-1], starts[1:])]


def decode_case(device, fmt, qlens, lens, window, num_splits=None, softcap=0.0, sinks=None, **kw):
    cache, table, qb = build(device, fmt, qlens, lens, **kw)
    got = U.decode(cache, qb, qlens, lens, table, num_splits=num_splits, sliding_window=window, softcap=softcap,
                   sinks=sinks)
    ref = U.reference(cache.host_bytes(), cache.layout, qb, qlens, lens, table, sliding_window=window,
                      softcap=softcap, sinks=sinks)
    assert np.isfinite(got).all()
    return errors(got, ref, qlens)


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
@pytest.mark.parametrize("num_splits", [None, 1, 2, 9], ids=["auto", "one-split", "two-splits", "tile-per-split"])
def test_window_starts_straddle_a_tile(device, fmt, num_splits):
    """4 tokens at 16,380..16,383 with a window of 1023: their first keys 15,358..15,361 straddle the tile at 15,360,
    so the last two tokens' rows see no key of tile 119 and open in tile 120 (or in the next split)."""
    errs = decode_case(device, fmt, [4], [16384], 1023, num_splits=num_splits)
    assert errs[0] < TOL, errs


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
@pytest.mark.parametrize("window", [1, 2, 130, 4097, 16384, 50000])
def test_window_sizes(device, fmt, window):
    errs = decode_case(device, fmt, [4], [16384], window)
    assert errs[0] < TOL, errs


def test_window_equal_to_the_context_is_no_window(device):
    """The windowed kernel variant with a window as wide as the context gives the plain kernel's output up to the
    rounding of the bf16 outputs (it does not fuse the score scaling into one FMA), and both match fp64."""
    cache, table, qb = build(device, "int4", [2], [5000])
    plain = U.decode(cache, qb, [2], [5000], table)
    wide = U.decode(cache, qb, [2], [5000], table, sliding_window=5000)
    assert qo.relerr(wide, plain) < 1e-3
    ref = U.reference(cache.host_bytes(), cache.layout, qb, [2], [5000], table)
    assert qo.relerr(wide, ref) < TOL and qo.relerr(plain, ref) < TOL


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
def test_ragged_mtp_batch(device, fmt):
    """4, 3, 1 and 4 tokens; the third context (100 keys) is shorter than the window."""
    errs = decode_case(device, fmt, [4, 3, 1, 4], [20000, 9000, 100, 3072], 2048, seed=3)
    assert max(errs) < TOL, errs


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
def test_spread_and_rising_scales(device, fmt):
    errs = decode_case(device, fmt, [4], [12000], 1500, spread=2.0, grow=6.0, seed=4)
    assert errs[0] < TOL, errs


def test_head_512(device):
    errs = decode_case(device, "k8v4", [4, 1], [9000, 700], 1023, nq=16, nkv=2, hs=512, seed=5)
    assert max(errs) < TOL, errs


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
@pytest.mark.parametrize("softcap", [3.0, 50.0])
def test_softcap_decode(device, fmt, softcap):
    errs = decode_case(device, fmt, [4, 2], [16384, 3000], 0, softcap=softcap, seed=8)
    assert max(errs) < TOL, errs


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
def test_softcap_with_window(device, fmt):
    errs = decode_case(device, fmt, [4], [16384], 1023, softcap=5.0, seed=9, spread=1.0)
    assert errs[0] < TOL, errs


def sink_logits(seed=11, nq=U.NQ):
    """Per-head sinks from well below the rows' scores to well above them (the sink then takes most of the mass)."""
    return np.random.default_rng(seed).uniform(-3.0, 6.0, nq).astype(np.float32)


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
@pytest.mark.parametrize("num_splits", [None, 1, 7])
def test_sinks_decode(device, fmt, num_splits):
    """The sink joins each row's denominator once, however many splits the merge folds."""
    errs = decode_case(device, fmt, [4, 1], [16384, 700], 0, num_splits=num_splits, sinks=sink_logits(), seed=10)
    assert max(errs) < TOL, errs


def test_sinks_need_the_model_domain_output(device):
    cache, table, qb = build(device, "int4", [1], [100])
    kc, vc, ks, vs = cache.views
    q = U.to_torch(qb, device)
    with pytest.raises(ValueError, match="sinks"):
        ops.paged_decode(q, kc, vc, torch.empty(q.shape, dtype=torch.float32, device=device),
                         cu_seqlens_q=torch.tensor([0, 1], dtype=torch.int32, device=device), max_seqlen_q=1,
                         seqused_k=torch.tensor([100], dtype=torch.int32, device=device), max_seqlen_k=100,
                         softmax_scale=U.HS ** -0.5, block_table=torch.from_numpy(table).to(device), k_scale_cache=ks,
                         v_scale_cache=vs, out_fp32_lse=torch.empty(q.shape[:2], dtype=torch.float32, device=device),
                         sinks=torch.zeros(U.NQ, device=device))


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
@pytest.mark.parametrize("window,softcap,sinks", [(64, 0.0, False), (700, 0.0, False), (0, 4.0, False),
                                                  (700, 4.0, False), (0, 0.0, True), (700, 4.0, True)])
def test_varlen_chunks(device, fmt, window, softcap, sinks):
    """Short chunks in one varlen launch (the long ones too, for a windowed or softcapped layer), first chunks
    included."""
    qlens = [100] * 6 + [37, 250]
    lens = [300 + 411 * i for i in range(6)] + [37, 9000]
    cache, table, qb = build(device, fmt, qlens, lens, seed=6)
    kc, vc, ks, vs = cache.views
    q = U.to_torch(qb, device)
    out = torch.full_like(q, float("nan"))
    cu = torch.tensor(np.concatenate([[0], np.cumsum(qlens)]), dtype=torch.int32, device=device)
    sk = sink_logits() if sinks else None
    ops.prefill_varlen(q, kc, vc, out, cu_seqlens_q=cu, seqused_k=torch.tensor(lens, dtype=torch.int32, device=device),
                       max_seqlen_k=max(lens), block_table=torch.from_numpy(table).to(device),
                       softmax_scale=U.HS ** -0.5, k_scale_cache=ks, v_scale_cache=vs, sliding_window=window,
                       softcap=softcap, sinks=None if sk is None else torch.from_numpy(sk).to(device))
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all(), "a row was not written"
    ref = U.reference(cache.host_bytes(), cache.layout, qb, qlens, lens, table, sliding_window=window,
                      softcap=softcap, sinks=sk)
    errs = errors(got, ref, qlens)
    assert max(errs) < TOL, errs
    assert _lib.device_error() == 0


@pytest.mark.parametrize("window", [2000, 5000])
def test_sequence_split_over_two_ranges(device, window):
    """Ranks holding [0, 4096) and [4096, 8192) of one sequence: rank 0 applies the window through
    tokens_after_keys (5000 reaches into its range, 2000 leaves it no key at all); the folded partials equal the
    windowed decode of the whole sequence."""
    n, qlen, world = 8192, 4, 2
    cache, table, qb = build(device, "int4", [qlen], [n], seed=7)
    kc, vc, ks, vs = cache.views
    q = U.to_torch(qb, device)
    part_o = torch.empty((world, qlen, U.NQ, U.HS), dtype=torch.float32, device=device)
    part_lse = torch.empty((world, qlen, U.NQ), dtype=torch.float32, device=device)
    cu = torch.tensor([0, qlen], dtype=torch.int32, device=device)
    for r in range(world):
        lo, hi, after = sp.sequence_range(n, r, world)
        sub = torch.from_numpy(np.ascontiguousarray(table[0, lo // BS:(hi + BS - 1) // BS])).to(device)
        ops.paged_decode(q, kc, vc, part_o[r], cu_seqlens_q=cu, max_seqlen_q=qlen,
                         seqused_k=torch.tensor([hi - lo], dtype=torch.int32, device=device), max_seqlen_k=hi - lo,
                         softmax_scale=U.HS ** -0.5, block_table=sub[None], k_scale_cache=ks, v_scale_cache=vs,
                         out_fp32_lse=part_lse[r], tokens_after_keys=after, sliding_window=window)
    out = torch.empty_like(q)
    ops.merge_attn_partials(part_o, part_lse, out)
    got = out.float().cpu().numpy()
    ref = U.reference(cache.host_bytes(), cache.layout, qb, [qlen], [n], table, sliding_window=window)
    assert qo.relerr(got, ref) < TOL
    if window == 2000:
        assert torch.isinf(part_lse[0]).all() and (part_lse[0] < 0).all()


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
@pytest.mark.parametrize("softcap,sinks", [(0.0, False), (5.0, False), (5.0, True)],
                         ids=["window", "window-softcap", "window-softcap-sinks"])
def test_mixed_step_through_the_router(device, stock, fmt, softcap, sinks):  # noqa: F811
    """A sliding-window (softcap, sink) layer's step: MTP decodes, a chunk long enough for the prefill kernel (it
    goes to the varlen launch instead: the prefill kernel has none of them) and a short chunk; every sampled row
    against fp64."""
    qlens = [192, 4, 2, 40]
    lens = [12000, 9000, 30000, 300]
    window = 1024
    cache, table, qb, q, kc, vc, args = mixed_step(device, fmt, qlens, lens)
    out = torch.full_like(q, float("nan"))
    sk = sink_logits() if sinks else None
    stock.unified_attention_int4(q, kc, vc, out, **dict(args, window_size=(window - 1, 0), softcap=softcap,
                                                        sinks=None if sk is None else torch.from_numpy(sk).to(device)))
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all(), "a row of the step was not written"
    starts = np.concatenate([[0], np.cumsum(qlens)])
    data, sg, hs = cache.host_bytes(), U.signs(cache.hs), cache.hs
    sample = [0, 95, 191] + list(range(starts[1], starts[3])) + [starts[3], starts[3] + 39]
    want = []
    for r in sample:
        i = int(np.searchsorted(starts, r, side="right") - 1)
        j = r - starts[i]
        q_rot = qo.single_rht(qo.to_f32(qb[r:r + 1], "bf16"), sg).astype(np.float64)
        o, _ = qo.attention_from_cache(q_rot, data, cache.layout, table[i], lens[i] - qlens[i] + j + 1, hs ** -0.5,
                                       sliding_window=window, softcap=softcap, sinks=sk)
        want.append(qo.single_rht(o.astype(np.float32), sg, inverse=True).astype(np.float64) / hs)
    err = qo.relerr(got[sample], np.concatenate(want))
    assert err < TOL, f"{fmt}: relative error {err:.3e}"
    assert _lib.device_error() == 0
