"""Host side of the sequence-parallel split (CPU, gloo ranks): the range partition, the causal shift each rank
applies, the packed [O | lse] exchange and the log-sum-exp fold reproduce the attention of the whole sequence.

Each rank's partial comes from the fp64 oracle over its own key range (the product computes it with the decode or
prefill kernel, checked against the same rule on a GPU in test_seq_parallel_gpu.py); the exchange is the product's
`PartialExchange` over a gloo process group."""
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import quantpack_oracle as qo
from vllm_quantpack_b200.attention import seq_parallel as sp

LOG2E = math.log2(math.e)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(n_total, qlen, nq=6, nkv=2, hs=64, seed=0):
    rng = np.random.default_rng(seed)
    K = rng.standard_normal((n_total, nkv, hs))
    V = rng.standard_normal((n_total, nkv, hs))
    q = rng.standard_normal((qlen, nq, hs)) * 2.0
    return q, K, V


def _worker(rank, world, port, n_total, qlen, result_dir, window=0):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, K, V = _case(n_total, qlen)
        hs = q.shape[-1]
        lo, hi, after = sp.sequence_range(n_total, rank, world)
        # this rank's partial: its keys only, query token i at local position (hi - lo) + after - qlen + i (with a
        # sliding window, a rank may hold none of a token's keys: lse -inf, folded with weight 0)
        o, lse = qo.attention_rht_domain(q, K[lo:hi], V[lo:hi], (hi - lo) + after, hs ** -0.5, hs, window)
        x = sp.PartialExchange(dist.group.WORLD, qlen, q.shape[1], hs, "cpu")
        x.o.copy_(torch.from_numpy(o))
        x.lse.copy_(torch.from_numpy(lse * LOG2E))  # the kernels exchange base-2 lse
        part_o, part_lse = x.gather()
        assert part_o.shape == (world, qlen, q.shape[1], hs) and part_lse.shape == (world, qlen, q.shape[1])
        assert part_o.stride(0) % 4 == 0  # each rank's partial starts 16-byte aligned (merge kernel requirement)
        folded, flse = qo.merge_partials(part_o.double().numpy(), part_lse.double().numpy() / LOG2E)
        np.save(os.path.join(result_dir, f"r{rank}.npy"), np.concatenate([folded.ravel(), flse.ravel()]))
    finally:
        dist.destroy_process_group()


def test_sequence_range_partition():
    for n, world in ((262144, 8), (1000, 3), (5, 2), (7, 1)):
        got = [sp.sequence_range(n, r, world) for r in range(world)]
        assert got[0][0] == 0 and got[-1][1] == n and got[-1][2] == 0
        for (lo, hi, after), (lo2, _, _) in zip(got, got[1:]):
            assert hi == lo2 and after == n - hi
    with pytest.raises(ValueError):
        sp.sequence_range(10, 2, 2)


@pytest.mark.parametrize("world,n_total,qlen,window", [(2, 900, 4, 0), (2, 640, 64, 0), (3, 1000, 3, 0),
                                                       (2, 900, 4, 300), (3, 1000, 3, 500), (2, 640, 64, 400)])
def test_exchange_and_fold_match_whole_sequence(tmp_path, world, n_total, qlen, window):
    """With a sliding window the earlier ranks see fewer keys, or none (900 / 300: rank 0 holds no key of any
    token's window)."""
    mp.spawn(_worker, args=(world, _free_port(), n_total, qlen, str(tmp_path), window), nprocs=world, join=True)
    q, K, V = _case(n_total, qlen)
    hs = q.shape[-1]
    ref, ref_lse = qo.attention_rht_domain(q, K, V, n_total, hs ** -0.5, hs, window)
    for r in range(world):
        got = np.load(tmp_path / f"r{r}.npy")
        o, lse = got[: ref.size].reshape(ref.shape), got[ref.size:].reshape(ref_lse.shape)
        # the exchange carries fp32: agreement to fp32 rounding of the partials
        assert qo.relerr(o, ref) < 1e-6
        assert np.allclose(lse, ref_lse, atol=1e-5)
