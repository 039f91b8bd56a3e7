"""Parity against the reference's own kernels as they run on the B200 (not its Triton interpreter).

- Store: the reference's `_store_k8v4` (vllm_quantpack/attention/k8v4_ops.py:10-63), compiled by Triton for this GPU
  and launched through the reference's own `k8v4_kv.store` (k8v4_kv.py:68-86), against this build's store on the same
  pre-rotated bf16 rows: the k8v4 cells byte for byte, and the int4 cells against the reference's value half (the
  int4 formula; k8v4_ops.py:44-63), for the keys and the values. The golden vectors under tests/golden come from the
  interpreter (IEEE fp32, no contraction); this checks that compiled Triton writes the same bytes.
- Prefill: the reference's production long-chunk path `prefill_sequence` (int4_prefill.py:203-232: 16k-token bf16
  unpacks + FlashAttention 2 with LSE + fp32 fold) on the very cache this build's prefill reads. This build's error
  against the fp64 oracle must be no larger than the reference's. vLLM's own FA2 build carries sm_80 code only, so the
  image's flash_attn 2.8 varlen forward (the same FA2 kernel family, with the same arguments) stands in for it.

Skipped when the reference is not installed in baseline/_ref (python -m pip install --no-index --no-deps --target
baseline/_ref <reference checkout>) or cannot be imported (no Triton / vLLM)."""
import os
import sys

import numpy as np
import pytest
import torch

from oracle import quantpack_oracle as qo

import qp_testutil as U

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")


def reference_module(name):
    if not os.path.isdir(os.path.join(REF, "vllm_quantpack")):
        pytest.skip("reference not installed in baseline/_ref")
    if REF not in sys.path:
        sys.path.insert(0, REF)
    try:
        return __import__(f"vllm_quantpack.attention.{name}", fromlist=[name])
    except Exception as e:  # no Triton / vLLM in this environment
        pytest.skip(f"reference module {name} not importable: {e}")


class _Identity:
    """The reference's store rotates through `stock.single_rht`; the rows given here are already rotated."""

    @staticmethod
    def single_rht(x, inverse=False):
        return x


def edge_rows(nkv, hs):
    """Rows the quantizers treat specially: all equal, zero, huge and tiny magnitudes, one outlier, codes on the
    grid, half-step ties."""
    rows = np.zeros((8, nkv, hs), np.float32)
    rows[0] = 3.0                                                  # constant: scale floor 1e-6
    rows[2] = np.linspace(-6.0e4, 6.0e4, hs)                        # near the bf16 range
    rows[3] = np.linspace(-1e-5, 1e-5, hs)                          # below the scale floor
    rows[4, :, 7] = 100.0                                           # one outlier
    rows[5] = np.tile(np.arange(16, dtype=np.float32), hs // 16)    # codes exactly on the grid
    rows[6] = np.linspace(-7.5, 7.5, hs)
    rows[7] = -np.linspace(0.0, 1.0, hs) ** 3
    return qo.from_f32(rows, "bf16")


def store_inputs(n, nkv, hs, seed):
    kb, vb = qo.synthetic_kv(n, nkv, hs, seed=seed)
    e = edge_rows(nkv, hs)
    return np.concatenate([kb, e]), np.concatenate([vb, e[::-1]])


@pytest.mark.parametrize("bs", [16, 3072])
def test_k8v4_store_bytes_match_compiled_reference(device, bs):
    rk = reference_module("k8v4_kv")
    n_tok, nkv, hs = 600, U.NKV, U.HS
    kb, vb = store_inputs(n_tok - 8, nkv, hs, seed=11)
    nblocks = (n_tok + bs - 1) // bs + 2
    slots = np.random.default_rng(3).permutation(nblocks * bs)[:n_tok].astype(np.int64)
    slots[::37] = -1                                                # padding slots: nothing written
    ours = U.Cache("k8v4", nblocks, bs, device)
    ours.store(kb, vb, slots, rotate=False)
    theirs = torch.zeros_like(ours.phys)
    kc, vc, ks, vs = rk.views(theirs, hs)
    rk.store(_Identity, U.to_torch(kb, device), U.to_torch(vb, device), kc, vc,
             torch.from_numpy(slots).to(device), k_scale_cache=ks, v_scale_cache=vs)
    a, b = ours.host_bytes(), theirs.view(torch.uint8).cpu().numpy().reshape(-1)
    diff = np.flatnonzero(a != b)
    assert diff.size == 0, f"{diff.size} bytes differ from the compiled reference store, first at {diff[:8]}"


def test_int4_store_bytes_match_compiled_reference_value_half(device):
    """The int4 cell's key and value halves are the int4 formula the reference's store applies to its value half."""
    rk = reference_module("k8v4_kv")
    n_tok, nkv, hs, bs = 400, U.NKV, U.HS, 16
    kb, vb = store_inputs(n_tok - 8, nkv, hs, seed=12)
    nblocks = n_tok // bs + 2
    slots = np.random.default_rng(4).permutation(nblocks * bs)[:n_tok].astype(np.int64)
    ours = U.Cache("int4", nblocks, bs, device)
    ours.store(kb, vb, slots, rotate=False)
    mine = ours.host_bytes().reshape(nblocks, nkv, bs, hs + 8)
    for half, rows in ((0, kb), (1, vb)):
        theirs = torch.zeros((nblocks, nkv, bs, rk.cell_bytes(hs, hs)), dtype=torch.int8, device=device)
        kc, vc, ks, vs = rk.views(theirs, hs)
        rk.store(_Identity, U.to_torch(kb, device), U.to_torch(rows, device), kc, vc,
                 torch.from_numpy(slots).to(device), k_scale_cache=ks, v_scale_cache=vs)
        want = theirs.view(torch.uint8).cpu().numpy()[..., hs + 4:]   # value nibbles + value scale word
        got = mine[..., half * (hs // 2 + 4):(half + 1) * (hs // 2 + 4)]
        diff = int((want != got).sum())
        assert diff == 0, f"{'key' if half == 0 else 'value'} half: {diff} bytes differ from the compiled reference"


def fa2_varlen():
    """The reference calls vLLM's FA2 with fa_version=2 and gets (out, lse); flash_attn 2.8's varlen forward."""
    try:
        from flash_attn import flash_attn_varlen_func
    except Exception as e:
        pytest.skip(f"flash_attn not importable: {e}")

    def fa(q, k, v, *, max_seqlen_q, cu_seqlens_q, max_seqlen_k, cu_seqlens_k, softmax_scale, causal,
           return_softmax_lse, fa_version):
        out, lse, _ = flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                                             softmax_scale=softmax_scale, causal=causal, return_attn_probs=True)
        return out, lse

    return fa


@pytest.mark.parametrize("fmt,qlen,n,bs,rows", [
    ("int4", 256, 40000, 3072, list(range(0, 256, 17)) + [255]),
    ("k8v4", 256, 40000, 3072, list(range(0, 256, 17)) + [255]),
    ("int4", 1024, 230400, 16, [0, 127, 128, 511, 512, 1023]),
], ids=["int4-40k", "k8v4-40k", "int4-c3"])
def test_prefill_no_worse_than_reference_fa2_path(device, fmt, qlen, n, bs, rows):
    from vllm_quantpack_b200.attention import ops
    rp = reference_module("int4_prefill")
    fa = fa2_varlen()
    table, nblocks = U.block_tables([n], bs, seed=2)
    cache = U.Cache(fmt, nblocks, bs, device)
    cache.fill(table[0], n, seed=5)
    qb = U.make_queries([qlen], seed=9)
    q = U.to_torch(qb, device)
    kc, vc, ks, vs = cache.views
    row = torch.from_numpy(table[0].astype(np.int32)).to(device)
    hs = cache.hs
    ours = torch.empty_like(q)
    ops.prefill(q, kc, vc, ours, block_row=row, n=n, softmax_scale=hs ** -0.5, k_scale_cache=ks, v_scale_cache=vs)
    q_rot = ops.single_rht(q.float()).to(q.dtype)
    o = rp.prefill_sequence(q_rot, kc, vc, ks, vs, row, n, hs ** -0.5 / hs, fa)
    theirs = ops.single_rht(o.float(), inverse=True) / hs
    torch.cuda.synchronize()
    data, sg, want = cache.host_bytes(), U.signs(hs), []
    for i in rows:
        qr = qo.single_rht(qo.to_f32(qb[i:i + 1], "bf16"), sg).astype(np.float64)
        out_i, _ = qo.attention_from_cache(qr, data, cache.layout, table[0], n - qlen + i + 1, hs ** -0.5)
        want.append(qo.single_rht(out_i.astype(np.float32), sg, inverse=True).astype(np.float64) / hs)
    want = np.concatenate(want)
    err_ours = qo.relerr(ours.float().cpu().numpy()[rows], want)
    err_ref = qo.relerr(theirs.cpu().numpy()[rows], want)
    print(f"{fmt} qlen {qlen} n {n}: B200 prefill {err_ours:.3e}, reference FA2 path {err_ref:.3e}")
    assert err_ours <= err_ref, f"B200 prefill {err_ours:.3e} > reference {err_ref:.3e}"
