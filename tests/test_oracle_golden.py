"""The CPU oracle against golden vectors produced by the reference's own kernels (tests/golden/make_golden.py).

These pin the oracle before anything is checked against it: the quantizer byte for byte (`_store_k8v4`,
vllm_quantpack/attention/k8v4_ops.py:10-63), dequantisation (`_unpack_segment[_i8]`,
vllm_quantpack/attention/int4_prefill.py:25-68) and the attention math within the reference's own bound
(`prefill_sequence_i8`, int4_prefill.py:176-200; bound 1e-2 as tests/test_int4_kv.py:339)."""
import numpy as np
import pytest

from oracle import quantpack_oracle as qo

from conftest import golden


def _cases(fname):
    data = golden(fname)
    return data, sorted({k.split(".")[0] for k in data.files})


STORE, STORE_CASES = _cases("store_k8v4.npz")


def oracle_store_golden(case):
    """The oracle's k8v4 store of a golden case's pre-rotated inputs, into a fresh cache buffer."""
    d = {k: STORE[f"{case}.{k}"] for k in ("k", "v", "slots", "cache", "meta")}
    T, nkv, hs, bs, nblocks, nhd = (int(x) for x in d["meta"])
    layout = qo.CacheLayout("k8v4", nblocks, nkv, bs, hs, nhd=bool(nhd))
    cache = np.zeros(layout.nbytes, dtype=np.uint8)
    qo.store("k8v4", d["k"], d["v"], d["slots"], cache, layout, None, rotate=False)
    return cache, d


@pytest.mark.parametrize("case", STORE_CASES)
def test_store_quantizer_is_bit_exact(case):
    cache, d = oracle_store_golden(case)
    assert cache.size == d["cache"].size
    bad = np.flatnonzero(cache != d["cache"])
    assert bad.size == 0, f"{bad.size} bytes differ, first at {bad[:8]}"


def test_store_golden_covers_padding_and_edges():
    slots = STORE["s0.slots"]
    assert (slots < 0).any() and (slots >= 0).any()
    k = qo.bf16_to_f32(STORE["s0.k"])
    assert (k[:, 0] == 0).all(axis=-1).any()           # an all-zero row: scale clamps to 1e-6


UNPACK, _ = _cases("unpack.npz")


def _gather(cache, layout, table, start, length, off, nbytes):
    pos = start + np.arange(length)
    blk = table[pos // layout.block_size]
    s = pos % layout.block_size
    base = blk[:, None] * layout.block_stride + np.arange(layout.nkv)[None] * layout.head_stride + \
        s[:, None] * layout.slot_stride
    return cache[base[..., None] + off + np.arange(nbytes)]


def _trunc_bf16(x):
    """The Triton interpreter casts fp32 -> bf16 by truncation (compiled Triton rounds to nearest even): the golden
    unpack outputs are the fp32 dequantised values truncated to bf16, so that is what is compared."""
    return (np.asarray(x, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def test_unpack_int4_matches_dequantisation():
    nkv, hs, bs, nblocks, start, length = (int(x) for x in UNPACK["u_int4.meta"])
    layout = qo.CacheLayout("int4", nblocks, nkv, bs, hs)
    cache, table = UNPACK["u_int4.cache"], UNPACK["u_int4.table"]
    for name, off, soff in (("k", layout.k_off, layout.ks_off), ("v", layout.v_off, layout.vs_off)):
        packed = _gather(cache, layout, table, start, length, off, hs // 2)
        word = _gather(cache, layout, table, start, length, soff, 4).copy().view(np.uint32)[..., 0]
        u = np.stack((packed & 0xF, packed >> 4), -1).reshape(length, nkv, hs).astype(np.float32)
        zp = (word & 0xF).astype(np.float32)
        sc = (word & np.uint32(0xFFFFFFF0)).view(np.float32)
        got = _trunc_bf16(((u - zp[..., None]).astype(np.float32) * sc[..., None]).astype(np.float32))
        assert np.array_equal(got, UNPACK[f"u_int4.{name}"]), name
        ref = qo.bf16_to_f32(UNPACK[f"u_int4.{name}"])
        assert np.allclose(qo.dequant_int4(packed, word), ref, rtol=1e-2, atol=1e-6)


def test_unpack_int8_matches_dequantisation():
    nkv, hs, bs, nblocks, start, length = (int(x) for x in UNPACK["u_int8.meta"])
    layout = qo.CacheLayout("k8v4", nblocks, nkv, bs, hs)
    cache, table = UNPACK["u_int8.cache"], UNPACK["u_int8.table"]
    codes = _gather(cache, layout, table, start, length, layout.k_off, hs).view(np.int8)
    sc = _gather(cache, layout, table, start, length, layout.ks_off, 4).copy().view(np.float32)[..., 0]
    got = _trunc_bf16((codes.astype(np.float32) * sc[..., None]).astype(np.float32))
    assert np.array_equal(got, UNPACK["u_int8.k"])


ATTN, ATTN_CASES = _cases("attn_i8.npz")


def golden_attention_case(case):
    """(layout, cache, table, q_rot fp32, n, reference kernel output fp32) of an attention golden case."""
    nq, nkv, hs, bs, nblocks, n, qlen = (int(x) for x in ATTN[f"{case}.meta"])
    layout = qo.CacheLayout("int4", nblocks, nkv, bs, hs)
    return (layout, ATTN[f"{case}.cache"], ATTN[f"{case}.table"], qo.bf16_to_f32(ATTN[f"{case}.q_rot"]), n,
            qo.bf16_to_f32(ATTN[f"{case}.out"]))


@pytest.mark.parametrize("case", ATTN_CASES)
def test_attention_oracle_agrees_with_reference_kernel(case):
    layout, cache, table, q_rot, n, out = golden_attention_case(case)
    hs = layout.head_size
    K, V = qo.read_sequence(cache, layout, table, n)
    ref, _ = qo.attention_rht_domain(q_rot, K, V, n, hs ** -0.5, hs)
    err = qo.relerr(out, ref)
    assert err < 1e-2, f"reference i8 kernel vs oracle: {err:.3e}"


def test_rht_is_an_involution_up_to_head():
    hs = 256
    signs = qo.rht_signs(hs)
    assert set(np.unique(signs)) == {-1.0, 1.0}
    x = np.random.default_rng(0).standard_normal((5, hs)).astype(np.float32)
    y = qo.single_rht(qo.single_rht(x, signs), signs, inverse=True) / hs
    assert np.allclose(y, x, atol=1e-5)
    bits = qo.rht_sign_bits(hs)
    unpacked = np.array([(bits[i // 32] >> (i % 32)) & 1 for i in range(hs)])
    assert np.array_equal(unpacked == 1, signs < 0)


def test_merge_of_partials_equals_whole_attention():
    rng = np.random.default_rng(3)
    nq, nkv, hs, n, qlen = 4, 2, 64, 97, 3
    K = rng.standard_normal((n, nkv, hs))
    V = rng.standard_normal((n, nkv, hs))
    q = rng.standard_normal((qlen, nq, hs)) * 4
    whole, lse = qo.attention_rht_domain(q, K, V, n, hs ** -0.5, hs)
    o1, l1 = qo.attention_rht_domain(q, K[:40], V[:40], n, hs ** -0.5, hs)
    # the second part is a context of n - 40 tokens: the same causal positions relative to its own keys
    o2, l2 = qo.attention_rht_domain(q, K[40:], V[40:], n - 40, hs ** -0.5, hs)
    merged, mlse = qo.merge_partials(np.stack([o1, o2]), np.stack([l1, l2]))
    assert np.allclose(merged, whole, atol=1e-12)
    assert np.allclose(mlse, lse, atol=1e-12)


@pytest.mark.parametrize("window", [1, 3, 64, 129, 500])
def test_sliding_window_keeps_the_last_window_keys_of_each_query(window):
    """vLLM's SLIDING_WINDOW (1 + window_size[0]): the query at position p sees keys p - window + 1 .. p, restated
    here as the attention over exactly those keys, per query token."""
    rng = np.random.default_rng(3)
    n, qlen, nq, nkv, hs = 300, 4, 4, 2, 32
    K = rng.standard_normal((n, nkv, hs))
    V = rng.standard_normal((n, nkv, hs))
    q = rng.standard_normal((qlen, nq, hs))
    got, lse = qo.attention_rht_domain(q, K, V, n, hs ** -0.5, hs, window)
    for i in range(qlen):
        p = n - qlen + i
        lo = max(0, p - window + 1)
        want, wl = qo.attention_rht_domain(q[i:i + 1], K[lo:p + 1], V[lo:p + 1], p + 1 - lo, hs ** -0.5, hs)
        np.testing.assert_allclose(got[i], want[0], rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(lse[i], wl[0], rtol=1e-12)
    whole, _ = qo.attention_rht_domain(q, K, V, n, hs ** -0.5, hs)
    if window >= n:
        np.testing.assert_allclose(got, whole, rtol=1e-12, atol=1e-12)
    else:
        assert not np.allclose(got, whole)


@pytest.mark.parametrize("window", [5, 100, 1000])
def test_streamed_oracle_skips_only_chunks_outside_every_window(window):
    """attention_from_cache reads the keys in chunks and skips the chunks before the first query's window: the same
    result as the attention over the whole dequantised sequence."""
    hs, nkv, nq, bs, n, qlen = 32, 2, 4, 16, 400, 3
    nblocks = n // bs + 2
    layout = qo.CacheLayout("int4", nblocks, nkv, bs, hs)
    cache = np.zeros(nblocks * nkv * bs * layout.cell, dtype=np.uint8)
    kb, vb = qo.synthetic_kv(n, nkv, hs, seed=1)
    table = np.random.default_rng(2).permutation(nblocks)[: n // bs].astype(np.int32)
    pos = np.arange(n)
    qo.store("int4", kb, vb, table[pos // bs].astype(np.int64) * bs + pos % bs, cache, layout, qo.rht_signs(hs))
    q = np.random.default_rng(4).standard_normal((qlen, nq, hs))
    got, gl = qo.attention_from_cache(q, cache, layout, table, n, hs ** -0.5, chunk=64, sliding_window=window)
    K, V = qo.read_sequence(cache, layout, table, n)
    want, wl = qo.attention_rht_domain(q, K, V, n, hs ** -0.5, hs, window)
    np.testing.assert_allclose(got, want, rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(gl, wl, rtol=1e-10)


@pytest.mark.parametrize("softcap", [3.0, 50.0])
def test_softcap_is_tanh_of_the_scaled_score(softcap):
    """vLLM's apply_softcap: softcap * tanh(S / softcap) on the scaled score, before the softmax; restated here as an
    explicit softmax over the capped scores."""
    rng = np.random.default_rng(8)
    n, qlen, nq, nkv, hs = 200, 2, 2, 1, 16
    K = rng.standard_normal((n, nkv, hs)) * 3
    V = rng.standard_normal((n, nkv, hs))
    q = rng.standard_normal((qlen, nq, hs)) * 3
    got, _ = qo.attention_rht_domain(q, K, V, n, hs ** -0.5, hs, 0, softcap)
    for i in range(qlen):
        p = n - qlen + i
        for h in range(nq):
            s = K[:p + 1, 0] @ q[i, h] * (hs ** -0.5 / hs)
            s = softcap * np.tanh(s / softcap)
            w = np.exp(s - s.max())
            np.testing.assert_allclose(got[i, h], w @ V[:p + 1, 0] / w.sum(), rtol=1e-12, atol=1e-12)


def test_sinks_join_the_denominator_once():
    """A sink is a virtual key with logit sink_h and value 0 in every row's softmax (vLLM's attention sinks); folded
    after the keys, also when the keys come in chunks (attention_from_cache folds the chunks first)."""
    rng = np.random.default_rng(9)
    n, qlen, nq, nkv, hs = 150, 3, 4, 2, 16
    K = rng.standard_normal((n, nkv, hs)) * 2
    V = rng.standard_normal((n, nkv, hs))
    q = rng.standard_normal((qlen, nq, hs)) * 2
    sinks = np.array([-3.0, 0.0, 2.5, 40.0])
    got, lse = qo.attention_rht_domain(q, K, V, n, hs ** -0.5, hs, sinks=sinks)
    for i in range(qlen):
        p = n - qlen + i
        for h in range(nq):
            s = np.append(K[:p + 1, h // 2] @ q[i, h] * (hs ** -0.5 / hs), sinks[h])
            w = np.exp(s - s.max())
            vals = np.vstack([V[:p + 1, h // 2], np.zeros(hs)])
            np.testing.assert_allclose(got[i, h], w @ vals / w.sum(), rtol=1e-10, atol=1e-14)
            np.testing.assert_allclose(lse[i, h], s.max() + np.log(w.sum()), rtol=1e-12)
    plain, plain_lse = qo.attention_rht_domain(q, K, V, n, hs ** -0.5, hs)
    halves = [qo.attention_rht_domain(q, K[a:b], V[a:b], n - a, hs ** -0.5, hs) for a, b in ((0, 70), (70, n))]
    o, l = qo.merge_partials(np.stack([h[0] for h in halves]), np.stack([h[1] for h in halves]))
    np.testing.assert_allclose(qo.apply_sinks(o, l, sinks)[0], got, rtol=1e-10, atol=1e-14)
