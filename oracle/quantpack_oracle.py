"""CPU oracle for the quantized KV-cache attention path. TEST INFRASTRUCTURE ONLY.

Only `tests/`, `__graft_entry__.smoke()` and the `cpu_baseline` / `--impl reference` legs of `bench.py` may import
this module, and only as the checker or the timed CPU baseline. The product path (`vllm_quantpack_b200`) never
imports it and has no CPU fallback.

What it restates, with the reference line each function follows (paths inside jramirez-uab/vllm-quantpack 0.1.8):

- round half away from zero: `vllm_quantpack/attention/k8v4_ops.py:5-8` (fp32 add of +-0.5, then truncation);
- int8 key quantizer (absmax / 127, IEEE division per element): `k8v4_ops.py:33-42`;
- int4 quantizer (min/max scale, zero point in the scale's low mantissa bits, multiply by the fp32 reciprocal,
  then add the zero point as a separate fp32 add): `k8v4_ops.py:44-63`. The stock int4 store
  (`reshape_and_cache_int4`, vLLM >= 0.31, not in this container) uses the same formula for keys and values
  (`k8v4_ops.py:7` "as vLLM's int4 store"; the key dequantisation in `tests/test_int4_kv.py:119-123` is the value one);
- dequantisation: `vllm_quantpack/attention/int4_prefill.py:42-46` (int4) and `:66-67` (int8 keys);
- fp64 attention of the last `qlen` positions of a context of `n` tokens from the cache, RHT domain,
  scale `softmax_scale / head`, inverse RHT divided by `head`: `tests/test_int4_kv.py:115-133`,
  `tests/test_k8v4_kv.py:112-133`;
- log-sum-exp fold of attention partials: `int4_prefill.py:223-230` and vLLM's `reduce_segments`
  (`vllm/v1/attention/ops/triton_unified_attention.py:645-732` in vLLM 0.22).

The randomized Hadamard transform (`single_rht`, called at `int4_kv.py:326,329` and `k8v4_kv.py:71-72`) lives in
the stock vLLM module, which is absent here: its sign vector and seed are unknown, so the RHT is PARITY UNPINNED.
This build defines it as y = H (d * x), H the unnormalised Sylvester Hadamard matrix evaluated by fp32 butterflies
with strides 1, 2, 4, ..., head/2 in that order, and d_i = -1 where bit 63 of splitmix64(seed * 2**32 + i) is set.
Every attention check is invariant to the choice (the same transform is applied on both sides), and the store's
quantizer is pinned by the reference's own `_store_k8v4` on pre-rotated inputs (tests/golden).

bf16 values are carried as uint16 bit patterns; fp32 <-> bf16 conversion is round-to-nearest-even.
"""
import numpy as np

F32 = np.float32

# ---------------------------------------------------------------------------------------------------- bf16 helpers


def bf16_to_f32(bits):
    """uint16 bf16 bit patterns -> float32 (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x):
    """float32 -> uint16 bf16 bits, round to nearest even (finite inputs; NaN stays NaN)."""
    xf = np.asarray(x, dtype=np.float32)
    u = xf.view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)
    r = np.where(np.isnan(xf), (u >> np.uint32(16)) | np.uint32(0x40), r)
    return r.astype(np.uint16)


def f16_to_f32(bits):
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def f32_to_f16(x):
    return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def to_f32(bits, dtype):
    """Model-dtype bits ('bf16' or 'f16') -> float32."""
    return bf16_to_f32(bits) if dtype == "bf16" else f16_to_f32(bits)


def from_f32(x, dtype):
    return f32_to_bf16(x) if dtype == "bf16" else f32_to_f16(x)


# ---------------------------------------------------------------------------------------------------- RHT

_M64 = (1 << 64) - 1


def _splitmix64(z):
    z = (z + 0x9E3779B97F4A7C15) & _M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
    return z ^ (z >> 31)


def rht_signs(head_size, seed=0):
    """The RHT sign vector d (+1 / -1 as float32) of this build (see the module docstring)."""
    return np.array([-1.0 if _splitmix64((seed << 32) + i) >> 63 else 1.0 for i in range(head_size)], dtype=F32)


def rht_sign_bits(head_size, seed=0):
    """d packed as uint32 words, bit i set where d_i = -1 (the layout the CUDA kernels take)."""
    d = rht_signs(head_size, seed)
    words = np.zeros((head_size + 31) // 32, dtype=np.uint32)
    for i in range(head_size):
        if d[i] < 0:
            words[i // 32] |= np.uint32(1 << (i % 32))
    return words


def wht_f32(x):
    """Unnormalised Walsh-Hadamard transform over the last axis in fp32, butterflies of stride 1, 2, 4, ... ."""
    x = np.array(x, dtype=F32, copy=True)
    n = x.shape[-1]
    lead = x.shape[:-1]
    h = 1
    while h < n:
        y = x.reshape(lead + (n // (2 * h), 2, h))
        a, b = y[..., 0, :], y[..., 1, :]
        x = np.stack((a + b, a - b), axis=-2).reshape(lead + (n,)).astype(F32)
        h *= 2
    return x


def single_rht(x, signs, inverse=False):
    """Forward: H (d * x). Inverse: d * (H x). Unnormalised: inverse(forward(x)) = head * x."""
    x = np.asarray(x, dtype=F32)
    if inverse:
        return (wht_f32(x) * signs).astype(F32)
    return wht_f32(x * signs)


# ---------------------------------------------------------------------------------------------------- quantizers


def round_half_away(x):
    """`k8v4_ops.py:5-8`: where(x >= 0, int(x + 0.5), int(x - 0.5)), the +-0.5 added in fp32."""
    x = np.asarray(x, dtype=F32)
    up = (x + F32(0.5)).astype(F32)
    dn = (x - F32(0.5)).astype(F32)
    return np.where(x >= 0, np.trunc(up), np.trunc(dn)).astype(F32)


def quant_int4(x):
    """Rows of x (..., hs) float32 -> (packed uint8 (..., hs/2), scale word uint32 (...)). `k8v4_ops.py:44-63`."""
    x = np.asarray(x, dtype=F32)
    mn = x.min(axis=-1)
    mx = x.max(axis=-1)
    scale = np.maximum(((mx - mn).astype(F32) / F32(15.0)).astype(F32), F32(1e-6)).astype(F32)
    zp = np.clip(round_half_away((-mn).astype(F32) / scale), F32(0.0), F32(15.0)).astype(F32)
    inv = (F32(1.0) / scale).astype(F32)
    prod = (x * inv[..., None]).astype(F32)
    q = np.clip(round_half_away((prod + zp[..., None]).astype(F32)), 0.0, 15.0).astype(np.uint8)
    packed = (q[..., 0::2] & 0xF) | ((q[..., 1::2] & 0xF) << 4)
    word = (scale.view(np.uint32) & np.uint32(0xFFFFFFF0)) | (zp.astype(np.uint32) & np.uint32(0xF))
    return packed.astype(np.uint8), word.astype(np.uint32)


def quant_int8(x):
    """Rows of x (..., hs) float32 -> (int8 codes (..., hs), fp32 scale (...)). `k8v4_ops.py:33-42`."""
    x = np.asarray(x, dtype=F32)
    scale = np.maximum((np.abs(x).max(axis=-1) / F32(127.0)).astype(F32), F32(1e-6)).astype(F32)
    q = np.clip(round_half_away((x / scale[..., None]).astype(F32)), -127.0, 127.0).astype(np.int8)
    return q, scale


def dequant_int4(packed, word):
    """(nibble - zero point) * scale, low nibble = even channel, in fp64. `int4_prefill.py:42-46`."""
    packed = np.asarray(packed, dtype=np.uint8)
    word = np.asarray(word, dtype=np.uint32)
    u = np.stack((packed & 0xF, packed >> 4), axis=-1).reshape(packed.shape[:-1] + (2 * packed.shape[-1],))
    zp = (word & np.uint32(0xF)).astype(np.float64)
    scale = (word & np.uint32(0xFFFFFFF0)).view(np.float32).astype(np.float64)
    return (u.astype(np.float64) - zp[..., None]) * scale[..., None]


def dequant_int8(codes, scale):
    """int8 * scale in fp64. `int4_prefill.py:66-67`."""
    return np.asarray(codes, dtype=np.int8).astype(np.float64) * np.asarray(scale, dtype=np.float32)[..., None]


# ---------------------------------------------------------------------------------------------------- cache model


class CacheLayout:
    """Byte layout of a paged cache: cell of one (block, KV head, slot) at
    base + block * block_stride + head * head_stride + slot * slot_stride, with the four fields at k_off, ks_off,
    v_off, vs_off inside the cell. int4: [K hs/2 | K scale | V hs/2 | V scale] (tests/test_int4_kv.py:95-103);
    k8v4: [K hs int8 | K scale | V hs/2 | V scale] (vllm_quantpack/attention/k8v4_kv.py:10-11, 41-65)."""

    def __init__(self, fmt, nblocks, nkv, block_size, head_size, nhd=False):
        self.fmt, self.nblocks, self.nkv, self.block_size, self.head_size = fmt, nblocks, nkv, block_size, head_size
        kb = head_size // 2 if fmt == "int4" else head_size
        self.k_off, self.ks_off = 0, kb
        self.v_off = kb + 4
        self.vs_off = kb + 4 + head_size // 2
        self.cell = kb + 8 + head_size // 2
        if nhd:
            self.slot_stride, self.head_stride = nkv * self.cell, self.cell
        else:
            self.slot_stride, self.head_stride = self.cell, block_size * self.cell
        self.block_stride = nkv * block_size * self.cell
        self.nbytes = nblocks * self.block_stride

    def cell_at(self, slot, head):
        blk, s = divmod(int(slot), self.block_size)
        return blk * self.block_stride + head * self.head_stride + s * self.slot_stride


def quantize_rows(fmt, k, v):
    """(key codes bytes, key scale word, value nibbles, value scale word) of rotated fp32 rows (..., hs)."""
    if fmt == "int4":
        kq, kw = quant_int4(k)
    else:
        kq, ks = quant_int8(k)
        kq, kw = kq.view(np.uint8), ks.view(np.uint32)
    vq, vw = quant_int4(v)
    return kq, kw, vq, vw


def store(fmt, key_bits, value_bits, slots, cache, layout, signs, dtype="bf16", rotate=True):
    """Rotate, quantize and write (tokens, kv heads, hs) key / value into the uint8 cache buffer `cache`.

    The RHT output is rounded to the model dtype before quantizing, as `k8v4_kv.py:71-72` does
    (`single_rht(key.float()).to(key.dtype)`). Slots < 0 are skipped (`k8v4_ops.py:23-24`)."""
    k = to_f32(key_bits, dtype)
    v = to_f32(value_bits, dtype)
    if rotate:
        k = to_f32(from_f32(single_rht(k, signs), dtype), dtype)
        v = to_f32(from_f32(single_rht(v, signs), dtype), dtype)
    kq, kw, vq, vw = quantize_rows(fmt, k, v)
    T, nkv, _ = k.shape
    for t in range(T):
        if slots[t] < 0:
            continue
        for h in range(nkv):
            c = layout.cell_at(slots[t], h)
            cache[c + layout.k_off:c + layout.k_off + kq.shape[-1]] = kq[t, h]
            cache[c + layout.ks_off:c + layout.ks_off + 4] = kw[t, h:h + 1].view(np.uint8)
            cache[c + layout.v_off:c + layout.v_off + vq.shape[-1]] = vq[t, h]
            cache[c + layout.vs_off:c + layout.vs_off + 4] = vw[t, h:h + 1].view(np.uint8)


def read_sequence(cache, layout, block_row, n):
    """(K, V) fp64 (n, kv heads, hs) in the RHT domain of the first n positions of one sequence."""
    hs, nkv = layout.head_size, layout.nkv
    pos = np.arange(n)
    blk = np.asarray(block_row, dtype=np.int64)[pos // layout.block_size]
    s = pos % layout.block_size
    base = blk[:, None] * layout.block_stride + np.arange(nkv)[None, :] * layout.head_stride + \
        s[:, None] * layout.slot_stride

    def gather(off, nbytes):
        return cache[base[..., None] + off + np.arange(nbytes)]

    kb = hs // 2 if layout.fmt == "int4" else hs
    kraw = gather(layout.k_off, kb)
    kw = gather(layout.ks_off, 4).copy().view(np.uint32)[..., 0]
    vraw = gather(layout.v_off, hs // 2)
    vw = gather(layout.vs_off, 4).copy().view(np.uint32)[..., 0]
    if layout.fmt == "int4":
        K = dequant_int4(kraw, kw)
    else:
        K = dequant_int8(kraw.view(np.int8), kw.view(np.float32))
    V = dequant_int4(vraw, vw)
    return K, V


# ---------------------------------------------------------------------------------------------------- attention


def attention_rht_domain(q_rot, K, V, n, softmax_scale, head_size, sliding_window=0, softcap=0.0, sinks=None):
    """fp64 attention of q_rot (qlen, nq, hs), the last qlen positions of a context of n tokens, over the cached
    K, V (n, nkv, hs) in the RHT domain, scale softmax_scale / head. Returns (out (qlen, nq, hs), lse (qlen, nq)) with
    lse the natural-log log-sum-exp of the scaled scores. `tests/test_int4_kv.py:127-132`. sliding_window > 0 (vLLM's
    SLIDING_WINDOW = 1 + window_size[0]): the query at position p sees only keys k with p - k < sliding_window, the
    stock kernel's mask (vllm/v1/attention/ops/triton_unified_attention.py:533-536 and triton_attention_helpers.py:
    203-218, vLLM 0.22, whose int4 kernel the reference patches). softcap > 0: every scaled score S becomes
    softcap * tanh(S / softcap) before the mask and the softmax (apply_softcap, triton_attention_helpers.py:28-36,
    applied at triton_unified_attention.py:513-514). sinks (nq,): see apply_sinks."""
    q_rot = np.asarray(q_rot, dtype=np.float64)
    qlen, nq, hs = q_rot.shape
    nkv = K.shape[1]
    g = nq // nkv
    pos = n - qlen + np.arange(qlen)
    keys = np.arange(K.shape[0])
    out = np.zeros((qlen, nq, hs))
    lse = np.full((qlen, nq), -np.inf)
    for h in range(nq):
        s = q_rot[:, h] @ K[:, h // g].T * (softmax_scale / head_size)
        if softcap > 0:
            s = softcap * np.tanh(s / softcap)
        s = np.where(keys[None, :] > pos[:, None], -np.inf, s)
        if sliding_window > 0:
            s = np.where(pos[:, None] - keys[None, :] >= sliding_window, -np.inf, s)
        m = s.max(axis=1, keepdims=True) if s.shape[1] else np.full((qlen, 1), -np.inf)
        ok = np.isfinite(m[:, 0])
        m = np.where(np.isfinite(m), m, 0.0)
        p = np.exp(s - m)
        l = p.sum(axis=1)
        safe = np.where(l > 0, l, 1.0)
        out[:, h] = np.where(ok[:, None], (p @ V[:, h // g]) / safe[:, None], 0.0)
        lse[:, h] = np.where(ok, m[:, 0] + np.log(safe), -np.inf)
    return apply_sinks(out, lse, sinks)


def apply_sinks(out, lse, sinks):
    """Attention sinks: per query head a logit (natural units) whose exp joins the softmax denominator of every row
    once and adds nothing to the numerator (vLLM: the row maximum starts at the sink with sum 1,
    vllm/v1/attention/ops/triton_attention_helpers.py:108-138, triton_unified_attention.py:356-359). Takes the
    attention over the keys, out (..., nq, hs) with natural-log lse (..., nq); returns both with the sink folded."""
    if sinks is None:
        return out, lse
    s = np.asarray(sinks, dtype=np.float64)
    tot = np.logaddexp(lse, s)
    w = np.where(np.isfinite(lse), np.exp(lse - tot), 0.0)
    return out * w[..., None], tot


def attention(q, K, V, n, softmax_scale, signs, dtype="bf16", sliding_window=0, softcap=0.0, sinks=None):
    """Attention output in the model domain, fp64: RHT(q) -> attention -> inverse RHT / head.
    `tests/test_int4_kv.py:126-133` (q rotated in fp32, output rotated back in fp32 then divided by head)."""
    qf = to_f32(q, dtype)
    hs = qf.shape[-1]
    q_rot = single_rht(qf, signs).astype(np.float64)
    o, _ = attention_rht_domain(q_rot, K, V, n, softmax_scale, hs, sliding_window, softcap, sinks)
    return single_rht(o.astype(F32), signs, inverse=True).astype(np.float64) / hs


def merge_partials(outs, lses):
    """Fold attention partials (P, ..., hs) with natural-log lse (P, ...) by log-sum-exp.
    `int4_prefill.py:223-230`; `triton_unified_attention.py:693-725` (vLLM 0.22)."""
    outs = np.asarray(outs, dtype=np.float64)
    lses = np.asarray(lses, dtype=np.float64)
    m = lses.max(axis=0)
    m = np.where(np.isfinite(m), m, 0.0)
    w = np.exp(lses - m)
    tot = w.sum(axis=0)
    safe = np.where(tot > 0, tot, 1.0)
    o = (outs * w[..., None]).sum(axis=0) / safe[..., None]
    return np.where((tot > 0)[..., None], o, 0.0), np.where(tot > 0, m + np.log(safe), -np.inf)


def relerr(o, ref):
    """||o - ref|| / ||ref||, as `tests/test_int4_kv.py:160-161`."""
    o = np.asarray(o, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.linalg.norm(o - ref) / np.linalg.norm(ref))


def check_store_agreement(got, want, layout, max_code_frac=0.01):
    """Compare cache bytes `got` written by a store that divides like the reference's COMPILED store (Triton lowers
    the fp32 `/` of `k8v4_ops.py:33-63` to PTX div.full.f32, within 2 ulp of the IEEE quotient, and fuses
    v * (1 / scale) + zp into one FMA) with `want`, this module's IEEE fp32 restatement of the same source. A scale
    may differ by a couple of ulp in any cell; a code moves only where its quotient sits next to a rounding tie.
    Raises AssertionError unless every code is within one step, every scale within 2 ulp (int4: the word with its
    zero-point bits masked within 2 x 16, the zero point within 1) and at most `max_code_frac` of the codes differ.
    Returns (cells that differ, codes that differ)."""
    hs, cell = layout.head_size, layout.cell
    kb = hs if layout.fmt == "k8v4" else hs // 2
    g = np.asarray(got, np.uint8).reshape(-1, cell)
    w = np.asarray(want, np.uint8).reshape(-1, cell)

    def nibbles(x):
        return np.concatenate([(x & 0xF).astype(np.int16), (x >> 4).astype(np.int16)], axis=1)

    def words(x, at):
        return x[:, at:at + 4].copy().view(np.uint32)[:, 0].astype(np.int64)

    def scale_word(at, what):
        gw, ww = words(g, at), words(w, at)
        if layout.fmt == "k8v4" and at == kb:
            assert np.abs(gw - ww).max(initial=0) <= 2, f"a {what} scale moved by more than 2 ulp"
            return
        assert np.abs((gw & ~0xF) - (ww & ~0xF)).max(initial=0) <= 32, f"a {what} scale moved by more than 2 ulp"
        assert np.abs((gw & 0xF) - (ww & 0xF)).max(initial=0) <= 1, f"a {what} zero point moved by more than one"

    if layout.fmt == "k8v4":
        dk = np.abs(g[:, :kb].view(np.int8).astype(np.int16) - w[:, :kb].view(np.int8).astype(np.int16))
    else:
        dk = np.abs(nibbles(g[:, :kb]) - nibbles(w[:, :kb]))
    assert dk.max(initial=0) <= 1, "a key code moved by more than one step"
    scale_word(kb, "key")
    v0 = kb + 4
    dv = np.abs(nibbles(g[:, v0:v0 + hs // 2]) - nibbles(w[:, v0:v0 + hs // 2]))
    assert dv.max(initial=0) <= 1, "a value code moved by more than one step"
    scale_word(v0 + hs // 2, "value")
    codes = int((dk != 0).sum() + (dv != 0).sum())
    total = dk.size + dv.size
    assert codes <= max_code_frac * total, f"{codes} of {total} codes differ"
    return int((g != w).any(axis=1).sum()), codes


# ---------------------------------------------------------------------------------------------------- inputs


def synthetic_kv(n, nkv, hs, seed=0, outlier_frac=0.02, outlier_gain=8.0):
    """bf16 bits (n, nkv, hs) ~ N(0, 1) with `outlier_frac` of the channels of every KV head scaled by
    `outlier_gain` (seeded), the input distribution of the measured configurations."""
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((n, nkv, hs), dtype=np.float32)
    v = rng.standard_normal((n, nkv, hs), dtype=np.float32)
    nout = max(1, int(round(outlier_frac * hs)))
    for h in range(nkv):
        ch = rng.choice(hs, nout, replace=False)
        k[:, h, ch] *= outlier_gain
        v[:, h, ch] *= outlier_gain
    return f32_to_bf16(k), f32_to_bf16(v)


def read_range(cache, layout, block_row, start, end):
    """(K, V) fp64 of positions [start, end) of one sequence (see read_sequence)."""
    hs, nkv = layout.head_size, layout.nkv
    pos = np.arange(start, end)
    blk = np.asarray(block_row, dtype=np.int64)[pos // layout.block_size]
    s = pos % layout.block_size
    base = blk[:, None] * layout.block_stride + np.arange(nkv)[None, :] * layout.head_stride + \
        s[:, None] * layout.slot_stride

    def gather(off, nbytes):
        return cache[base[..., None] + off + np.arange(nbytes)]

    kb = hs // 2 if layout.fmt == "int4" else hs
    kraw = gather(layout.k_off, kb)
    kw = gather(layout.ks_off, 4).copy().view(np.uint32)[..., 0]
    vraw = gather(layout.v_off, hs // 2)
    vw = gather(layout.vs_off, 4).copy().view(np.uint32)[..., 0]
    K = dequant_int4(kraw, kw) if layout.fmt == "int4" else dequant_int8(kraw.view(np.int8), kw.view(np.float32))
    return K, dequant_int4(vraw, vw)


def attention_from_cache(q_rot, cache, layout, block_row, n, softmax_scale, chunk=16384, sliding_window=0,
                         softcap=0.0, sinks=None):
    """attention_rht_domain over the cached context of one sequence, streamed in chunks of keys and folded by
    log-sum-exp (memory bounded for long contexts). Returns (out, natural-log lse)."""
    hs = layout.head_size
    outs, lses = [], []
    first = 0
    if sliding_window > 0:  # chunks wholly before the first query's window hold no visible key
        first = max(0, n - q_rot.shape[0] - sliding_window + 1) // chunk * chunk
    for start in range(first, max(n, 1), chunk):
        end = min(n, start + chunk)
        K, V = read_range(cache, layout, block_row, start, end)
        o, l = attention_rht_domain(q_rot, K, V, n - start, softmax_scale, hs, sliding_window, softcap)
        outs.append(o)
        lses.append(l)
    o, l = merge_partials(np.stack(outs), np.stack(lses))
    return apply_sinks(o, l, sinks)  # once, after the chunks are folded
