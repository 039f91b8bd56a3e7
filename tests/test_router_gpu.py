"""A real mixed vLLM step through the installed `unified_attention_int4` on the GPU (decode requests, a long prefill
chunk and a short chunk in one call), every row against the fp64 oracle, for both cache formats; and the step's host
behaviour: the first attention layer of a step reads the lengths once, the next layers of the same step never wait
for the GPU (the reference's checks: tests/test_int4_kv.py:213-229, 253-319; tests/test_k8v4_kv.py:177-195).

The stock vLLM int4 module is not in this image, so a stand-in module receives the patch; its own stock functions
fail the test if the B200 router ever falls back to them."""
import logging
import sys
import types

import numpy as np
import pytest
import torch

from oracle import quantpack_oracle as qo

import qp_testutil as U

pytestmark = pytest.mark.gpu
LOG = logging.getLogger("test")
TOL = 5e-3


@pytest.fixture
def stock(monkeypatch):
    from vllm_quantpack_b200.attention import int4_kv
    mod = types.ModuleType("qp_fake_int4_module_gpu")

    def no_stock(*a, **k):
        raise AssertionError("the stock int4 path was reached")

    mod.unified_attention_int4 = no_stock
    mod.reshape_and_cache_int4 = no_stock
    mod.single_rht = lambda x, inverse=False: x
    mod._launch_packed_attn = no_stock
    monkeypatch.setitem(sys.modules, mod.__name__, mod)
    monkeypatch.setattr(int4_kv, "MODULE", mod.__name__)
    assert int4_kv.patch_int4_kv(LOG) is True
    return mod


def vllm_args(cu, used, table, ks, vs):
    return dict(cu_seqlens_q=cu, max_seqlen_q=int((cu[1:] - cu[:-1]).max()), seqused_k=used,
                max_seqlen_k=int(used.max()), softmax_scale=U.HS ** -0.5, window_size=(-1, -1), block_table=table,
                softcap=0.0, sinks=None, alibi_slopes=None, use_alibi_sqrt=False, qq_bias=None, output_scale=None,
                mm_prefix_range=None, k_scale_cache=ks, v_scale_cache=vs, seq_threshold_3D=32,
                num_par_softmax_segments=64, softmax_segm_output=None, softmax_segm_max=None,
                softmax_segm_expsum=None)


def mixed_step(device, fmt, qlens, lens, bs=16):
    table, nblocks = U.block_tables(lens, bs, seed=4)
    cache = U.Cache(fmt, nblocks, bs, device)
    for i, n in enumerate(lens):
        cache.fill(table[i], n, seed=10 + i)
    qb = U.make_queries(qlens, seed=21)
    q = U.to_torch(qb, device)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(qlens)]), dtype=torch.int32, device=device)
    used = torch.tensor(lens, dtype=torch.int32, device=device)
    kc, vc, ks, vs = cache.views
    args = vllm_args(cu, used, torch.from_numpy(table).to(device), ks, vs)
    return cache, table, qb, q, kc, vc, args


def oracle_rows(cache, table, qb, qlens, lens, sample):
    """fp64 output of the step's rows `sample` (global row indices), each against its own causal prefix."""
    data, sg, hs = cache.host_bytes(), U.signs(cache.hs), cache.hs
    starts = np.concatenate([[0], np.cumsum(qlens)])
    out = []
    for r in sample:
        i = int(np.searchsorted(starts, r, side="right") - 1)
        j = r - starts[i]
        q_rot = qo.single_rht(qo.to_f32(qb[r:r + 1], "bf16"), sg).astype(np.float64)
        o, _ = qo.attention_from_cache(q_rot, data, cache.layout, table[i], lens[i] - qlens[i] + j + 1, hs ** -0.5)
        out.append(qo.single_rht(o.astype(np.float32), sg, inverse=True).astype(np.float64) / hs)
    return np.concatenate(out)


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
def test_mixed_step_every_request_matches_fp64(device, stock, fmt):
    # a long prefill chunk, two MTP decodes, a plain decode and a short chunk in one step
    qlens = [192, 4, 2, 1, 40]
    lens = [12000, 9000, 30000, 5000, 300]
    cache, table, qb, q, kc, vc, args = mixed_step(device, fmt, qlens, lens)
    out = torch.full_like(q, float("nan"))
    stock.unified_attention_int4(q, kc, vc, out, **args)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all(), "a row of the step was not written"
    starts = np.concatenate([[0], np.cumsum(qlens)])
    sample = [0, 95, 191] + list(range(starts[1], starts[4])) + [starts[4], starts[4] + 39]
    err = qo.relerr(got[sample], oracle_rows(cache, table, qb, qlens, lens, sample))
    assert err < TOL, f"{fmt}: relative error {err:.3e}"


def test_second_layer_of_a_step_does_not_wait_for_the_gpu(device, stock, monkeypatch):
    """Every attention layer of a step gets the same length tensors: the first may read them to the host once, the
    next ones must not synchronise at all (sync debug mode 'error' raises on any synchronising call)."""
    from vllm_quantpack_b200.attention import int4_kv
    step = types.SimpleNamespace()
    monkeypatch.setattr(int4_kv, "_forward_step", lambda: step)
    qlens, lens = [128, 4, 2], [9000, 3000, 20000]
    cache, table, qb, q, kc, vc, args = mixed_step(device, "int4", qlens, lens)
    first, second = torch.empty_like(q), torch.empty_like(q)
    stock.unified_attention_int4(q, kc, vc, first, **args)
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        stock.unified_attention_int4(q, kc, vc, second, **args)
    finally:
        torch.cuda.set_sync_debug_mode("default")
    torch.cuda.synchronize()
    assert torch.equal(first, second)
    step2 = types.SimpleNamespace()                # a new step reads its own lengths
    monkeypatch.setattr(int4_kv, "_forward_step", lambda: step2)
    args["seqused_k"][2] = 15000
    third = torch.empty_like(q)
    stock.unified_attention_int4(q, kc, vc, third, **dict(args, max_seqlen_k=15000))
    torch.cuda.synchronize()
    sample = [130, 131]
    err = qo.relerr(third.float().cpu().numpy()[sample],
                    oracle_rows(cache, table, qb, qlens, [9000, 3000, 15000], sample))
    assert err < TOL


def test_decode_step_does_not_wait_for_the_gpu(device, stock):
    """A decode-only step never reads lengths: CUDA-graph capturable and free of host synchronisation."""
    qlens, lens = [4, 2, 1], [5000, 20000, 700]
    cache, table, qb, q, kc, vc, args = mixed_step(device, "k8v4", qlens, lens)
    out = torch.empty_like(q)
    stock.unified_attention_int4(q, kc, vc, out, **args)   # first call: library load, workspace, sign vector
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        stock.unified_attention_int4(q, kc, vc, out, **args)
    finally:
        torch.cuda.set_sync_debug_mode("default")
    torch.cuda.synchronize()
    err = qo.relerr(out.float().cpu().numpy(), oracle_rows(cache, table, qb, qlens, lens, list(range(7))))
    assert err < TOL
