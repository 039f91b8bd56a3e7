"""Sequence-parallel attention on the GPU: the kernels' causal shift (`tokens_after_keys`) and the fold of per-range
partials reproduce the attention of the whole sequence.

One GPU: the ranks are emulated in one process (each range decoded / prefilled through its own slice of the block
table, partials stacked and folded by the merge kernel). Two or more GPUs: `seq_parallel_worker.py` under torchrun,
one rank per GPU, NCCL all-gather of the packed partials."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from oracle import quantpack_oracle as qo
from vllm_quantpack_b200.attention import ops
from vllm_quantpack_b200.attention import seq_parallel as sp

import qp_testutil as U

pytestmark = pytest.mark.gpu
TOL = 5e-3
BS = 16


def _setup(device, fmt, n, seed=0):
    table, nblocks = U.block_tables([n], BS, seed=seed + 1)
    cache = U.Cache(fmt, nblocks, BS, device)
    cache.fill(table[0], n, seed=seed)
    return cache, table


def _sub_table(table, lo, hi, device):
    assert lo % BS == 0
    return torch.from_numpy(np.ascontiguousarray(table[0, lo // BS:(hi + BS - 1) // BS])).to(device)


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("fmt", ["int4", "k8v4"])
def test_decode_split_by_range(device, fmt, world):
    n, qlen = 8192, 4
    cache, table = _setup(device, fmt, n)
    kc, vc, ks, vs = cache.views
    qb = U.make_queries([qlen], seed=7)
    q = U.to_torch(qb, device)
    part_o = torch.empty((world, qlen, U.NQ, U.HS), dtype=torch.float32, device=device)
    part_lse = torch.empty((world, qlen, U.NQ), dtype=torch.float32, device=device)
    cu = torch.tensor([0, qlen], dtype=torch.int32, device=device)
    for r in range(world):
        lo, hi, after = sp.sequence_range(n, r, world)
        ops.paged_decode(q, kc, vc, part_o[r], cu_seqlens_q=cu, max_seqlen_q=qlen,
                         seqused_k=torch.tensor([hi - lo], dtype=torch.int32, device=device), max_seqlen_k=hi - lo,
                         softmax_scale=U.HS ** -0.5, block_table=_sub_table(table, lo, hi, device)[None],
                         k_scale_cache=ks, v_scale_cache=vs, out_fp32_lse=part_lse[r], tokens_after_keys=after)
    out = torch.empty_like(q)
    ops.merge_attn_partials(part_o, part_lse, out)
    got = out.float().cpu().numpy()
    whole = U.decode(cache, qb, [qlen], [n], table)
    ref = U.reference(cache.host_bytes(), cache.layout, qb, [qlen], [n], table)
    assert qo.relerr(got, ref) < TOL
    assert qo.relerr(got, whole) < 2e-3  # same kernels, different split points


@pytest.mark.parametrize("world", [2, 4])
def test_prefill_split_by_range(device, world):
    n, qlen = 4096, 128
    cache, table = _setup(device, "int4", n, seed=3)
    kc, vc, ks, vs = cache.views
    qb = U.make_queries([qlen], seed=9)
    q = U.to_torch(qb, device)
    part_o = torch.empty((world, qlen, U.NQ, U.HS), dtype=torch.float32, device=device)
    part_lse = torch.empty((world, qlen, U.NQ), dtype=torch.float32, device=device)
    for r in range(world):
        lo, hi, after = sp.sequence_range(n, r, world)
        ops.prefill(q, kc, vc, part_o[r], block_row=_sub_table(table, lo, hi, device), n=hi - lo,
                    softmax_scale=U.HS ** -0.5, k_scale_cache=ks, v_scale_cache=vs, out_fp32_lse=part_lse[r],
                    tokens_after_keys=after)
    out = torch.empty_like(q)
    ops.merge_attn_partials(part_o, part_lse, out)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    rows = [0, 1, 64, 127]
    sg = U.signs(U.HS)
    data = cache.host_bytes()
    ref = []
    for i in rows:
        q_rot = qo.single_rht(qo.to_f32(qb[i:i + 1], "bf16"), sg).astype(np.float64)
        o, _ = qo.attention_from_cache(q_rot, data, cache.layout, table[0], n - qlen + i + 1, U.HS ** -0.5)
        ref.append(qo.single_rht(o.astype(np.float32), sg, inverse=True).astype(np.float64) / U.HS)
    assert qo.relerr(got[rows], np.concatenate(ref)) < TOL


def test_nccl_ranks(device):
    """One rank per GPU over NCCL (torchrun): the sequence-parallel decode and prefill agree with the whole-sequence
    kernels run on rank 0."""
    ngpu = torch.cuda.device_count()
    if ngpu < 2:
        pytest.skip("one GPU: the ranks are covered by the emulated tests above")
    world = min(ngpu, 4)
    here = os.path.dirname(os.path.abspath(__file__))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", "--master-port=29561",
           os.path.join(here, "seq_parallel_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "seq_parallel ok" in r.stdout
