"""Shared helpers of the GPU tests: caches in the reference's layouts, seeded fills through the B200 store, and the
CPU oracle evaluated on the bytes the GPU wrote (as the reference's tests compute their fp64 reference from the same
cache, tests/test_int4_kv.py:115-133)."""
import numpy as np
import torch

from oracle import quantpack_oracle as qo
from vllm_quantpack_b200.attention import k8v4_kv, ops

NQ, NKV, HS = 24, 4, 256                 # Qwen3.8-27B full-attention layers (tests/test_int4_kv.py:92)
SIGNS = {}


def signs(hs):
    if hs not in SIGNS:
        SIGNS[hs] = qo.rht_signs(hs)
    return SIGNS[hs]


def to_torch(bits, device, dtype="bf16"):
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16))
    return t.view(torch.bfloat16 if dtype == "bf16" else torch.float16).to(device)


def to_bits(t):
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


class Cache:
    """A paged cache in vLLM's layout: int4 as tests/test_int4_kv.py:95-103, k8v4 through k8v4_kv.views."""

    def __init__(self, fmt, nblocks, block_size, device, nkv=NKV, hs=HS, nhd=False):
        self.fmt, self.nblocks, self.block_size, self.nkv, self.hs, self.nhd = fmt, nblocks, block_size, nkv, hs, nhd
        if fmt == "int4":
            assert not nhd
            phs = hs // 2 + 4
            kv = torch.zeros((nblocks, nkv, block_size, 2 * phs), dtype=torch.uint8, device=device)
            base = torch.tensor([], dtype=torch.float32, device=device).set_(kv.untyped_storage())
            st = [s // 4 for s in kv.stride()]
            ks = torch.as_strided(base, (nblocks, block_size, nkv), (st[0], st[2], st[1]), hs // 2 // 4)
            vs = torch.as_strided(base, (nblocks, block_size, nkv), (st[0], st[2], st[1]), (phs + hs // 2) // 4)
            kc, vc = kv.transpose(1, 2).split(phs, dim=-1)
            self.phys = kv
        else:
            cell = k8v4_kv.cell_bytes(hs, hs)
            if nhd:
                self.phys = torch.zeros((nblocks, block_size, nkv, cell), dtype=torch.int8, device=device)
                kv = self.phys.transpose(1, 2)
            else:
                kv = self.phys = torch.zeros((nblocks, nkv, block_size, cell), dtype=torch.int8, device=device)
            kc, vc, ks, vs = k8v4_kv.views(kv, hs)
        self.views = (kc, vc, ks, vs)
        self.layout = qo.CacheLayout(fmt, nblocks, nkv, block_size, hs, nhd=nhd)

    def host_bytes(self):
        torch.cuda.synchronize()
        return self.phys.contiguous().view(torch.uint8).cpu().numpy().reshape(-1)

    def store(self, k_bits, v_bits, slots, dtype="bf16", rotate=True):
        kc, vc, ks, vs = self.views
        dev = kc.device
        k = to_torch(k_bits, dev, dtype)
        v = to_torch(v_bits, dev, dtype)
        ops.reshape_and_cache_int4(k, v, kc, vc, torch.as_tensor(slots, device=dev), k_scale_cache=ks,
                                   v_scale_cache=vs, rotate=rotate)

    def fill(self, block_row, n, seed, chunk=32768, spread=0.0, grow=0.0):
        """Store n seeded tokens (synthetic K/V with outlier channels) at positions 0..n-1 of block_row.
        spread > 0 scales each (token, head) of K and of V by 10^u, u ~ U(-spread, spread) (scales that differ by
        orders of magnitude inside one tile); grow > 0 multiplies position i by 1 + grow i / n (row maxima and value
        scales that keep rising, so the kernels' rescale paths run)."""
        row = np.asarray(block_row, dtype=np.int64)
        rng = np.random.default_rng(seed + 77)
        for s in range(0, n, chunk):
            e = min(n, s + chunk)
            kb, vb = qo.synthetic_kv(e - s, self.nkv, self.hs, seed=seed * 1000 + s // chunk)
            if spread > 0 or grow > 0:
                fk = np.ones((e - s, self.nkv, 1), np.float32)
                fv = np.ones((e - s, self.nkv, 1), np.float32)
                if spread > 0:
                    fk *= 10.0 ** rng.uniform(-spread, spread, fk.shape).astype(np.float32)
                    fv *= 10.0 ** rng.uniform(-spread, spread, fv.shape).astype(np.float32)
                if grow > 0:
                    g = (1.0 + grow * np.arange(s, e, dtype=np.float32) / n)[:, None, None]
                    fk *= g
                    fv *= g
                kb = qo.from_f32(qo.to_f32(kb, "bf16") * fk, "bf16")
                vb = qo.from_f32(qo.to_f32(vb, "bf16") * fv, "bf16")
            pos = np.arange(s, e)
            slots = row[pos // self.block_size] * self.block_size + pos % self.block_size
            self.store(kb, vb, slots)


def block_tables(lens, block_size, seed=1, spare=3):
    """Random block tables over a shuffled pool: a permutation of blocks (seeded) dealt to the sequences."""
    need = [(n + block_size - 1) // block_size for n in lens]
    total = sum(need) + spare
    perm = np.random.default_rng(seed).permutation(total)
    width = max(need) if need else 1
    table = np.zeros((len(lens), max(width, 1)), dtype=np.int32)
    at = 0
    for i, nb in enumerate(need):
        table[i, :nb] = perm[at:at + nb]
        at += nb
    return table, total


def make_queries(qlens, seed=5, nq=NQ, hs=HS, dtype="bf16"):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((sum(qlens), nq, hs), dtype=np.float32)
    return qo.from_f32(q, dtype)


def decode(cache, q_bits, qlens, lens, table, dtype="bf16", num_splits=None, device="cuda", sliding_window=0,
           softcap=0.0, sinks=None):
    """Run the B200 split-KV decode; returns the output as float32 numpy (tokens, nq, hs)."""
    kc, vc, ks, vs = cache.views
    q = to_torch(q_bits, device, dtype)
    out = torch.empty_like(q)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(qlens)]), dtype=torch.int32, device=device)
    ops.paged_decode(q, kc, vc, out, cu_seqlens_q=cu, max_seqlen_q=max(qlens),
                     seqused_k=torch.tensor(lens, dtype=torch.int32, device=device), max_seqlen_k=max(lens),
                     softmax_scale=cache.hs ** -0.5, block_table=torch.from_numpy(table).to(device),
                     k_scale_cache=ks, v_scale_cache=vs, num_splits=num_splits, sliding_window=sliding_window,
                     softcap=softcap, sinks=None if sinks is None else torch.tensor(sinks, device=device))
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


def reference(cache_bytes, layout, q_bits, qlens, lens, table, dtype="bf16", sliding_window=0, softcap=0.0,
              sinks=None):
    """fp64 oracle output (tokens, nq, hs) in the model domain, per sequence, from the cache bytes."""
    hs = layout.head_size
    sg = signs(hs)
    outs = []
    at = 0
    for i, (ql, n) in enumerate(zip(qlens, lens)):
        qf = qo.to_f32(q_bits[at:at + ql], dtype)
        q_rot = qo.single_rht(qf, sg).astype(np.float64)
        o, _ = qo.attention_from_cache(q_rot, cache_bytes, layout, table[i], n, hs ** -0.5,
                                       sliding_window=sliding_window, softcap=softcap, sinks=sinks)
        outs.append(qo.single_rht(o.astype(np.float32), sg, inverse=True).astype(np.float64) / hs)
        at += ql
    return np.concatenate(outs)


def assert_store_agrees(got, want, layout):
    """Cache bytes `got` (this build's store, which divides like the reference's compiled store) against `want` (the
    IEEE fp32 order of the reference's source: the oracle, or the reference run by Triton's interpreter): scales
    within 2 ulp, codes within one step and at most 1 % of them moved (qo.check_store_agreement). Returns the number
    of cells that differ."""
    return qo.check_store_agreement(got, want, layout)[0]
