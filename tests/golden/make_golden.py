"""Generate the golden vectors in tests/golden/ from the reference's own kernels (run once, in a container that has
the reference checkout; the outputs are committed and the GPU box never needs the reference).

    REFERENCE=/path/to/vllm-quantpack python tests/golden/make_golden.py

It runs the reference's Triton kernels under TRITON_INTERPRET=1 (CPU, IEEE fp32, no FMA contraction):
- `_store_k8v4` (vllm_quantpack/attention/k8v4_ops.py:10-63) on pre-rotated bf16 keys / values: int8 keys and the
  int4 value half, which is the int4 quantizer of both halves of the int4 cache;
- `_unpack_segment` / `_unpack_segment_i8` (vllm_quantpack/attention/int4_prefill.py:25-68): dequantisation through
  a shuffled block table;
- `prefill_sequence_i8` (int4_prefill.py:176-200): the reference's single-kernel attention over the raw int4 cache,
  whose output pins the attention oracle within the reference's own bound (tests/test_int4_kv.py:339: 1e-2).
"""
import os
import sys

import numpy as np

os.environ["TRITON_INTERPRET"] = "1"
REF = os.environ.get("REFERENCE")
if not REF:
    sys.exit("set REFERENCE to the reference checkout (the directory holding vllm_quantpack/)")
sys.path.insert(0, REF)
HERE = os.path.dirname(os.path.abspath(__file__))

import torch  # noqa: E402

from vllm_quantpack.attention import int4_prefill, k8v4_kv, k8v4_ops  # noqa: E402


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def _edge_rows(hs, g):
    """Rows that exercise the quantizer's corner cases: constant, zero, one-sided, tiny, huge, exact .5 steps."""
    rows = [
        torch.zeros(hs),
        torch.full((hs,), 3.25),
        torch.full((hs,), -2.0),
        torch.rand(hs, generator=g) * 5 + 1,                 # all positive: zero point clamps at 0
        -(torch.rand(hs, generator=g) * 5 + 1),              # all negative: zero point clamps at 15
        torch.randn(hs, generator=g) * 1e-7,                 # below the 1e-6 scale floor
        torch.randn(hs, generator=g) * 3e4,
        (torch.arange(hs) % 31 - 15).float() * 0.5,          # many exact half steps
        torch.linspace(-7.5, 7.5, hs),
    ]
    return torch.stack(rows)


def _store(k, v, kc, vc, ks, vs, slots, bs, hs):
    k8v4_ops._store_k8v4[(k.shape[0], k.shape[1])](
        k, v, kc, vc, ks, vs, slots,
        k.stride(0), k.stride(1), v.stride(0), v.stride(1),
        kc.stride(0), kc.stride(1), kc.stride(2), vc.stride(0), vc.stride(1), vc.stride(2),
        ks.stride(0), ks.stride(1), ks.stride(2), vs.stride(0), vs.stride(1), vs.stride(2),
        block_size=bs, head_size=hs, head_size_v=hs, HEAD_PADDED=hs, HALF_PADDED=hs // 2)


def store_cases():
    out = {}
    g = torch.Generator().manual_seed(1234)
    cases = [("s0", 37, 4, 256, 16, False), ("s1", 19, 2, 128, 32, False), ("s2", 11, 2, 512, 16, True),
             ("s3", 40, 2, 256, 32, True)]
    for name, T, nkv, hs, bs, nhd in cases:
        k = torch.randn((T, nkv, hs), generator=g) * (1 + 15 * torch.rand((T, nkv, 1), generator=g))
        v = torch.randn((T, nkv, hs), generator=g) * (1 + 15 * torch.rand((T, nkv, 1), generator=g))
        e = _edge_rows(hs, g)
        k[: min(T, len(e)), 0] = e[: min(T, len(e))]
        v[: min(T, len(e)), nkv - 1] = e[: min(T, len(e))].flip(0)
        k = k.to(torch.bfloat16)
        v = v.to(torch.bfloat16)
        nblocks = (T + bs - 1) // bs + 2
        cell = k8v4_kv.cell_bytes(hs, hs)
        if nhd:
            kv = torch.zeros((nblocks, bs, nkv, cell), dtype=torch.int8).transpose(1, 2)
        else:
            kv = torch.zeros((nblocks, nkv, bs, cell), dtype=torch.int8)
        kc, vc, ks, vs = k8v4_kv.views(kv, hs)
        slots = torch.randperm(nblocks * bs, generator=g)[:T]
        slots[::5] = -1                                         # padding slots: skipped
        _store(k, v, kc, vc, ks, vs, slots, bs, hs)
        phys = kv.transpose(1, 2) if nhd else kv                # back to the allocation order
        out[name] = dict(k=_bits(k), v=_bits(v), slots=slots.numpy().astype(np.int64),
                         cache=phys.contiguous().numpy().view(np.uint8).reshape(-1).copy(),
                         meta=np.array([T, nkv, hs, bs, nblocks, int(nhd)], dtype=np.int64))
    return out


def _int4_cache(nblocks, nkv, bs, hs, g):
    """A random int4 cache in the layout of tests/test_int4_kv.py:95-103 with valid scale words."""
    phs = hs // 2 + 4
    kv = torch.randint(0, 256, (nblocks, nkv, bs, 2 * phs), dtype=torch.uint8, generator=g)
    words = kv.view(torch.int32).view(nblocks, nkv, bs, 2 * phs // 4)
    for at in (hs // 2 // 4, (phs + hs // 2) // 4):
        sc = (torch.rand((nblocks, nkv, bs), generator=g) * 2 + 0.05).view(torch.int32)
        zp = torch.randint(0, 16, (nblocks, nkv, bs), dtype=torch.int32, generator=g)
        words[..., at] = (sc & -16) | zp
    base = torch.tensor([], dtype=torch.float32).set_(kv.untyped_storage())
    st = [s // 4 for s in kv.stride()]
    ks = torch.as_strided(base, (nblocks, bs, nkv), (st[0], st[2], st[1]), hs // 2 // 4)
    vs = torch.as_strided(base, (nblocks, bs, nkv), (st[0], st[2], st[1]), (phs + hs // 2) // 4)
    kc, vc = kv.transpose(1, 2).split(phs, dim=-1)
    return kv, (kc, vc, ks, vs)


def unpack_cases():
    out = {}
    g = torch.Generator().manual_seed(99)
    nkv, hs, bs, nblocks = 2, 256, 16, 12
    kv, (kc, vc, ks, vs) = _int4_cache(nblocks, nkv, bs, hs, g)
    table = torch.randperm(nblocks, generator=g).to(torch.int32)
    start, length = 21, 130
    kbuf = torch.zeros((length, nkv, hs), dtype=torch.bfloat16)
    vbuf = torch.zeros_like(kbuf)
    int4_prefill.unpack_segment(kc, ks, table, start, length, kbuf)
    int4_prefill.unpack_segment(vc, vs, table, start, length, vbuf)
    out["u_int4"] = dict(cache=kv.numpy().reshape(-1).copy(), table=table.numpy().astype(np.int64),
                         meta=np.array([nkv, hs, bs, nblocks, start, length], dtype=np.int64),
                         k=_bits(kbuf), v=_bits(vbuf))
    cell = k8v4_kv.cell_bytes(hs, hs)
    kv8 = torch.randint(-128, 128, (nblocks, nkv, bs, cell), dtype=torch.int8, generator=g)
    kc8, vc8, ks8, vs8 = k8v4_kv.views(kv8, hs)
    ks8.copy_(torch.rand(ks8.shape, generator=g) * 0.1 + 1e-3)
    kbuf8 = torch.zeros((length, nkv, hs), dtype=torch.bfloat16)
    int4_prefill.unpack_segment(kc8, ks8, table, start, length, kbuf8)
    out["u_int8"] = dict(cache=kv8.numpy().view(np.uint8).reshape(-1).copy(), table=table.numpy().astype(np.int64),
                         meta=np.array([nkv, hs, bs, nblocks, start, length], dtype=np.int64), k=_bits(kbuf8))
    return out


def attention_cases():
    """`prefill_sequence_i8` over a stored cache: (q_rot, cache, table) -> output in the RHT domain."""
    out = {}
    g = torch.Generator().manual_seed(7)
    for name, nq, nkv, hs, bs, n, qlen in (("a0", 4, 2, 256, 16, 300, 40), ("a1", 6, 1, 256, 32, 200, 3)):
        nblocks = (n + bs - 1) // bs + 3
        cell = k8v4_kv.cell_bytes(hs, hs)
        # K and V each go through the reference's store; the int4 value half of each k8v4 cell (the int4 formula)
        # is copied into the key or value half of the int4 cell.
        kv = torch.zeros((nblocks, nkv, bs, hs + 8), dtype=torch.uint8)
        phs = hs // 2 + 4
        kc, vc = kv.transpose(1, 2).split(phs, dim=-1)
        table = (torch.randperm(nblocks - 3, generator=g) + 3).to(torch.int32)   # blocks 0..2 never used
        pos = torch.arange(n)
        slots = table[pos // bs].long() * bs + pos % bs
        for half in (0, 1):
            x = (torch.randn((n, nkv, hs), generator=g) * 4).to(torch.bfloat16)
            tmp = torch.zeros((nblocks, nkv, bs, cell), dtype=torch.int8)
            tk, tv, tks, tvs = k8v4_kv.views(tmp, hs)
            _store(x, x, tk, tv, tks, tvs, slots, bs, hs)
            src = tmp.view(torch.uint8)[..., hs + 4:]           # [V hs/2 | V scale]: one int4 half-cell
            (kc if half == 0 else vc).copy_(src.transpose(1, 2))
        base = torch.tensor([], dtype=torch.float32).set_(kv.untyped_storage())
        st = [s // 4 for s in kv.stride()]
        ks = torch.as_strided(base, (nblocks, bs, nkv), (st[0], st[2], st[1]), hs // 2 // 4)
        vs = torch.as_strided(base, (nblocks, bs, nkv), (st[0], st[2], st[1]), (phs + hs // 2) // 4)
        q_rot = (torch.randn((qlen, nq, hs), generator=g) * 16).to(torch.bfloat16)
        o = int4_prefill.prefill_sequence_i8(q_rot, kc, vc, ks, vs, table, n, hs ** -0.5 / hs,
                                             block_m=16, block_n=16, num_warps=1, num_stages=1)
        out[name] = dict(cache=kv.numpy().reshape(-1).copy(), table=table.numpy().astype(np.int64),
                         q_rot=_bits(q_rot), out=_bits(o),
                         meta=np.array([nq, nkv, hs, bs, nblocks, n, qlen], dtype=np.int64))
    return out


def main():
    for fname, fn in (("store_k8v4.npz", store_cases), ("unpack.npz", unpack_cases),
                      ("attn_i8.npz", attention_cases)):
        cases = fn()
        flat = {f"{c}.{k}": v for c, d in cases.items() for k, v in d.items()}
        np.savez_compressed(os.path.join(HERE, fname), **flat)
        print(fname, sorted(cases), sum(v.nbytes for v in flat.values()), "bytes")


if __name__ == "__main__":
    main()
