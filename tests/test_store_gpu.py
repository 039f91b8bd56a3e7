"""Cache write on the GPU (K0 / K0'). The store divides like the reference's store as compiled by Triton for the GPU
(PTX div.full.f32, and v * (1 / scale) + zp fused into one FMA), and is bit-exact with that kernel
(tests/test_reference_gpu.py runs it). Here it is checked against the IEEE fp32 order of the reference's source (the
oracle, and the golden bytes of the reference run by Triton's interpreter): a scale may differ by a couple of ulp in
any cell (div.full.f32 is within 2 ulp of the IEEE quotient), a code moves by one step only next to a rounding tie
(qo.check_store_agreement: at most 1 % of the codes).
Padding slots skipped, nothing written past the tokens (tests/test_k8v4_kv.py:140-156 of the reference)."""
import numpy as np
import pytest
import torch

from oracle import quantpack_oracle as qo

import qp_testutil as U
from conftest import golden

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
@pytest.mark.parametrize("hs,bs,nhd,dtype", [(256, 16, False, "bf16"), (256, 3072, False, "bf16"),
                                              (128, 32, False, "f16"), (512, 16, False, "bf16"),
                                              (256, 32, True, "bf16")],
                         ids=["hs256-bs16", "hs256-bs3072", "hs128-f16", "hs512", "nhd"])
def test_store_agrees_with_oracle(device, fmt, hs, bs, nhd, dtype):
    if nhd and fmt == "int4":
        pytest.skip("the int4 cache is HND in vLLM")
    T, nkv = 301, 4
    nblocks = (T + bs - 1) // bs + 2
    cache = U.Cache(fmt, nblocks, bs, device, nkv=nkv, hs=hs, nhd=nhd)
    kb, vb = qo.synthetic_kv(T, nkv, hs, seed=11)
    if dtype == "f16":
        kb = qo.f32_to_f16(qo.bf16_to_f32(kb))
        vb = qo.f32_to_f16(qo.bf16_to_f32(vb))
    rng = np.random.default_rng(2)
    slots = rng.permutation(nblocks * bs)[:T].astype(np.int64)
    slots[::7] = -1
    cache.store(kb, vb, slots, dtype=dtype)
    got = cache.host_bytes()
    want = np.zeros_like(got)
    qo.store(fmt, kb, vb, slots, want, cache.layout, U.signs(hs), dtype=dtype)
    U.assert_store_agrees(got, want, cache.layout)


STORE = golden("store_k8v4.npz")


@pytest.mark.parametrize("case", sorted({k.split(".")[0] for k in STORE.files}))
def test_store_agrees_with_interpreted_reference_kernel(device, case):
    """The reference's `_store_k8v4` run by Triton's interpreter (IEEE fp32), from the same pre-rotated inputs."""
    T, nkv, hs, bs, nblocks, nhd = (int(x) for x in STORE[f"{case}.meta"])
    cache = U.Cache("k8v4", nblocks, bs, device, nkv=nkv, hs=hs, nhd=bool(nhd))
    cache.store(STORE[f"{case}.k"], STORE[f"{case}.v"], STORE[f"{case}.slots"], rotate=False)
    U.assert_store_agrees(cache.host_bytes(), STORE[f"{case}.cache"], cache.layout)


@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
def test_padding_slots_and_bounds(device, fmt):
    bs, T = 16, 40
    cache = U.Cache(fmt, 8, bs, device)
    kb, vb = qo.synthetic_kv(T, U.NKV, U.HS, seed=3)
    cache.store(kb, vb, np.arange(T))
    before = cache.host_bytes().copy()
    layout = cache.layout
    # nothing written past the tokens
    for slot in range(T, 8 * bs):
        for h in range(U.NKV):
            c = layout.cell_at(slot, h)
            assert not before[c:c + layout.cell].any()
    cache.store(kb[:8], vb[:8], np.full(8, -1))          # padding slots are skipped
    assert np.array_equal(cache.host_bytes(), before)


def test_error_bands_of_the_stored_cache(device):
    """k8v4 keys ~1 % and values ~10 % relative error against the rotated inputs (reference bands,
    tests/test_k8v4_kv.py:149-151)."""
    n = 4096
    cache = U.Cache("k8v4", n // 16, 16, device)
    kb, vb = qo.synthetic_kv(n, U.NKV, U.HS, seed=0, outlier_frac=0.0)
    cache.store(kb, vb, np.arange(n))
    K, V = qo.read_sequence(cache.host_bytes(), cache.layout, np.arange(n // 16), n)
    kr = qo.single_rht(qo.bf16_to_f32(kb), U.signs(U.HS))
    vr = qo.single_rht(qo.bf16_to_f32(vb), U.signs(U.HS))
    k_err, v_err = qo.relerr(K, kr), qo.relerr(V, vr)
    assert k_err < 0.02, k_err
    assert 0.05 < v_err < 0.2, v_err


def test_single_rht_matches_oracle(device):
    from vllm_quantpack_b200.attention import ops
    for hs in (128, 256, 512):
        x = np.random.default_rng(hs).standard_normal((37, hs)).astype(np.float32)
        xt = torch.from_numpy(x).to(device)
        y = ops.single_rht(xt).cpu().numpy()
        assert np.array_equal(y, qo.single_rht(x, U.signs(hs)))
        z = ops.single_rht(torch.from_numpy(y).to(device), inverse=True).cpu().numpy()
        assert np.array_equal(z, qo.single_rht(y, U.signs(hs), inverse=True))
