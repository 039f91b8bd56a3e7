"""One rank of the multi-GPU sequence-parallel check (launched by test_seq_parallel_gpu.py under torchrun, one
process per GPU, NCCL). Every rank writes the same seeded sequence into its own cache, attends over its own range
only through `SequenceParallelAttention`, and compares the folded result with the whole-sequence kernels run
locally. Rank 0 prints `seq_parallel ok` when every rank agrees."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(HERE))

import qp_testutil as U  # noqa: E402
from oracle import quantpack_oracle as qo  # noqa: E402
from vllm_quantpack_b200.attention import ops  # noqa: E402
from vllm_quantpack_b200.attention import seq_parallel as sp  # noqa: E402

BS = 16


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=device)
    rank, world = dist.get_rank(), dist.get_world_size()
    errs = []
    try:
        n = 16384
        table, nblocks = U.block_tables([n], BS, seed=1)
        cache = U.Cache("int4", nblocks, BS, device)
        cache.fill(table[0], n, seed=0)
        kc, vc, ks, vs = cache.views
        lo, hi, after = sp.sequence_range(n, rank, world)
        sub = torch.from_numpy(np.ascontiguousarray(table[0, lo // BS:(hi + BS - 1) // BS])).to(device)

        qlen = 4
        cu = torch.tensor([0, qlen], dtype=torch.int32, device=device)
        whole = None
        # the NVLink fold (symmetric memory; every rank reads the others' partials) and the NCCL all-gather; three
        # calls in a row with other queries each, so the fold's two partial parities both serve twice
        for peer in (None, False):
            runner = sp.SequenceParallelAttention(dist.group.WORLD, qlen, U.NQ, U.HS, device, peer=peer)
            if rank == 0:
                print(f"exchange: {'NVLink fold' if runner.peer is not None else 'NCCL all-gather'}", flush=True)
            for call in range(3):
                q = U.to_torch(U.make_queries([qlen], seed=7 + call), device)
                out = torch.empty_like(q)
                runner.decode(q, kc, vc, out, cu_seqlens_q=cu, max_seqlen_q=qlen,
                              seqused_k=torch.tensor([hi - lo], dtype=torch.int32, device=device),
                              max_seqlen_k=hi - lo, softmax_scale=U.HS ** -0.5, block_table=sub[None],
                              k_scale_cache=ks, v_scale_cache=vs, tokens_after_keys=after)
                whole = torch.empty_like(q)
                ops.paged_decode(q, kc, vc, whole, cu_seqlens_q=cu, max_seqlen_q=qlen,
                                 seqused_k=torch.tensor([n], dtype=torch.int32, device=device), max_seqlen_k=n,
                                 softmax_scale=U.HS ** -0.5, block_table=torch.from_numpy(table).to(device),
                                 k_scale_cache=ks, v_scale_cache=vs)
                errs.append(qo.relerr(out.float().cpu().numpy(), whole.float().cpu().numpy()))

        qlen = 256
        for peer in (None, False):
            q = U.to_torch(U.make_queries([qlen], seed=9), device)
            runner = sp.SequenceParallelAttention(dist.group.WORLD, qlen, U.NQ, U.HS, device, peer=peer)
            out = torch.empty_like(q)
            runner.prefill(q, kc, vc, out, block_row=sub, n=hi - lo, softmax_scale=U.HS ** -0.5, k_scale_cache=ks,
                           v_scale_cache=vs, tokens_after_keys=after)
            whole = torch.empty_like(q)
            ops.prefill(q, kc, vc, whole, block_row=torch.from_numpy(table[0]).to(device), n=n,
                        softmax_scale=U.HS ** -0.5, k_scale_cache=ks, v_scale_cache=vs)
            errs.append(qo.relerr(out.float().cpu().numpy(), whole.float().cpu().numpy()))
        from vllm_quantpack_b200 import _lib
        if _lib.device_error() != 0:
            raise RuntimeError("a kernel gave up a bounded wait")
        ok = all(e < 2e-3 for e in errs)
    except Exception as exc:  # every rank still takes part in the final all-reduce
        print(f"rank {rank}: {exc!r}", flush=True)
        ok = False
    flag = torch.tensor([0 if ok else 1], dtype=torch.int32, device=device)
    dist.all_reduce(flag)
    print(f"rank {rank}: relerr vs whole-sequence kernels {errs}", flush=True)
    dist.destroy_process_group()
    if flag.item():
        sys.exit(1)
    if rank == 0:
        print("seq_parallel ok", flush=True)


if __name__ == "__main__":
    main()
