"""Benchmark of the B200 quantized KV-cache attention (prints one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--workload c2a|c1|c2b|c3|c4]

Metric: 262k-context int4-KV decode, query tokens per second of one attention-layer call, and the
HBM bandwidth it reaches. A step is one attention call (split-KV decode + segment merge) over a resident paged cache
of synthetic data (K, V ~ N(0, 1) with 2 % outlier channels x8, written by the B200 store; q ~ N(0, 1); seeds 0 / 1),
with a random block table over a shuffled pool. Workloads:
  c2a  int4, 1 request, context 262144, 4 query tokens (3 MTP drafts)     [default, the N=1 headline]
  c1   int4, 1 request, context 131072, 2 query tokens
  c2b  int4, 32 requests x context 32768, 2 query tokens
  c4   k8v4, 1 request, context 262144, 4 query tokens
  c3   int4 prefill: a 1024-query chunk over 229,376 cached tokens (+ its own 1024), causal in the chunk; metric
       prefill tokens per second and the dense tensor throughput it reaches
At N > 1 each rank serves its own request(s) of the workload (batch sharded by request, no collective: weak
scaling); the line also carries `seq_parallel`: one request split by sequence range over the N ranks, each rank's
partial (O, LSE) all-gathered over NCCL and merged (strong scaling of a single request).

The cache (>= 138 MB) is larger than L2 and L2 is flushed (256 MB written, then another 256 MB read so that the
write-back of the dirty lines happens before the timed region) before every timed step; each step is timed
on the device with CUDA events on the launching stream, max over ranks.

`--impl reference` times the reference algorithm on the host cores instead: the CPU oracle (a restatement of the
reference's fp64 attention-from-cache, tests/test_int4_kv.py:115-133) on a bounded sample of the workload.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

NQ, NKV, HS, BS = 24, 4, 256, 16
WORKLOADS = {
    "c2a": dict(fmt="int4", seqs=1, ctx=262144, qlen=4),
    "c1": dict(fmt="int4", seqs=1, ctx=131072, qlen=2),
    "c2b": dict(fmt="int4", seqs=32, ctx=32768, qlen=2),
    "c4": dict(fmt="k8v4", seqs=1, ctx=262144, qlen=4),
    "c3": dict(fmt="int4", seqs=1, ctx=229376 + 1024, qlen=1024, prefill=True),
}
CELL = {"int4": HS + 8, "k8v4": HS * 3 // 2 + 8}
# DRAM bytes (read + write) per launch of the dominant kernel, from one ncu capture of that workload (profiles/):
# decode_kernel at c2a, prefill_kernel at c3 (the workloads whose dominant kernel was captured).
TRAFFIC = {"c2a": 277.01e6 + 3.97e6, "c3": 9.940e9 + 0.0340e9}


def algorithmic_bytes(w, seqs=None):
    """Bytes one attention call must move: every cached cell once, plus q and out (bf16)."""
    seqs = w["seqs"] if seqs is None else seqs
    return seqs * (w["ctx"] * NKV * CELL[w["fmt"]] + 2 * w["qlen"] * NQ * HS * 2)


def prefill_flops(w):
    """QK and PV flops of one chunk, causal counted exactly: 4 * nq * hs * sum_i (ctx - qlen + i + 1)."""
    ctx, qlen = w["ctx"], w["qlen"]
    return 4 * NQ * HS * (qlen * (ctx - qlen) + qlen * (qlen + 1) // 2)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            d = json.load(fh)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except (ValueError, IndexError):
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------------------------------- setup


def build_request(torch, ops, w, device, seqs, seed=0):
    """A paged cache holding `seqs` requests of the workload, filled through the B200 store, plus the call args."""
    from vllm_quantpack_b200.attention import k8v4_kv
    ctx, qlen, fmt = w["ctx"], w["qlen"], w["fmt"]
    nb_per = (ctx + BS - 1) // BS
    nblocks = seqs * nb_per + 8
    perm = torch.randperm(nblocks, generator=torch.Generator().manual_seed(seed + 1)).to(torch.int32)
    table = perm[: seqs * nb_per].view(seqs, nb_per).to(device)
    if fmt == "int4":
        phs = HS // 2 + 4
        kv = torch.empty((nblocks, NKV, BS, 2 * phs), dtype=torch.uint8, device=device)
        base = torch.tensor([], dtype=torch.float32, device=device).set_(kv.untyped_storage())
        st = [s // 4 for s in kv.stride()]
        ks = torch.as_strided(base, (nblocks, BS, NKV), (st[0], st[2], st[1]), HS // 2 // 4)
        vs = torch.as_strided(base, (nblocks, BS, NKV), (st[0], st[2], st[1]), (phs + HS // 2) // 4)
        kc, vc = kv.transpose(1, 2).split(phs, dim=-1)
    else:
        kv = torch.empty((nblocks, NKV, BS, k8v4_kv.cell_bytes(HS, HS)), dtype=torch.int8, device=device)
        kc, vc, ks, vs = k8v4_kv.views(kv, HS)
    g = torch.Generator(device=device).manual_seed(seed)
    chan = torch.randperm(HS, generator=torch.Generator().manual_seed(seed))[: max(1, round(0.02 * HS))].to(device)
    chunk = 32768
    for s in range(seqs):
        for t0 in range(0, ctx, chunk):
            t1 = min(ctx, t0 + chunk)
            k = torch.randn((t1 - t0, NKV, HS), generator=g, device=device)
            v = torch.randn((t1 - t0, NKV, HS), generator=g, device=device)
            k[..., chan] *= 8
            v[..., chan] *= 8
            pos = torch.arange(t0, t1, device=device)
            slots = table[s, pos // BS].long() * BS + pos % BS
            ops.reshape_and_cache_int4(k.to(torch.bfloat16), v.to(torch.bfloat16), kc, vc, slots, k_scale_cache=ks,
                                       v_scale_cache=vs)
    q = torch.randn((seqs * qlen, NQ, HS), generator=g, device=device).to(torch.bfloat16)
    cu = torch.arange(0, seqs * qlen + 1, qlen, dtype=torch.int32, device=device)
    used = torch.full((seqs,), ctx, dtype=torch.int32, device=device)
    return dict(kv=kv, views=(kc, vc, ks, vs), table=table, q=q, cu=cu, used=used, seqs=seqs)


FLUSH_BYTES = 256 << 20   # each half of the flush buffer is twice the 126 MB L2


def l2_flush(flush):
    """Evict L2: write one half of `flush` (> L2), then read the other half (> L2), so the dirty lines of the write
    are written back here and not during the next timed step (a write-only flush leaves ~126 MB of dirty lines whose
    write-back the timed kernel would pay)."""
    import torch
    half = flush.numel() // 2
    flush[:half].zero_()
    flush[half:].view(torch.int64).sum()


def timed_steps(torch, fn, steps, warmup, flush):
    """Run `warmup` untimed steps, then `steps` steps each timed by CUDA events (L2 flushed before each)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(steps):
        l2_flush(flush)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b))
    return times


# ---------------------------------------------------------------------------------------------------- CPU arm


def cpu_sample(w, budget_s=15.0):
    """Time the CPU oracle (fp64 attention from the cache bytes, all host threads for the BLAS part) on a bounded
    sample of the workload: the same head shape over a 16,384-token context, scaled to the full workload by the
    number of (query, key) pairs (the work is linear in them). A decode sample keeps the workload's query tokens; a
    prefill chunk is sampled by 16 query tokens. Returns (tokens/s of the full workload, sample description,
    threads)."""
    from oracle import quantpack_oracle as qo
    ctx = 16384
    qlen = 16 if w.get("prefill") else w["qlen"]

    def pairs(q, n):  # (query, key) pairs of q queries that are the last q positions of an n-token context
        return q * (n - q) + q * (q + 1) // 2

    fmt = w["fmt"]
    layout = qo.CacheLayout(fmt, ctx // BS, NKV, BS, HS)
    cache = np.zeros(layout.nbytes, dtype=np.uint8)
    kb, vb = qo.synthetic_kv(ctx, NKV, HS, seed=0)
    qo.store(fmt, kb, vb, np.arange(ctx), cache, layout, qo.rht_signs(HS))
    table = np.arange(ctx // BS)
    q = qo.f32_to_bf16(np.random.default_rng(1).standard_normal((qlen, NQ, HS)).astype(np.float32))
    signs = qo.rht_signs(HS)
    reps, t0 = 0, time.perf_counter()
    while True:
        q_rot = qo.single_rht(qo.bf16_to_f32(q), signs).astype(np.float64)
        o, _ = qo.attention_from_cache(q_rot, cache, layout, table, ctx, HS ** -0.5)
        qo.single_rht(o.astype(np.float32), signs, inverse=True)
        reps += 1
        el = time.perf_counter() - t0
        if el > budget_s or reps >= 50:
            break
    scale = w["seqs"] * pairs(w["qlen"], w["ctx"]) / pairs(qlen, ctx)
    per_call_full = el / reps * scale
    tok_s = w["seqs"] * w["qlen"] / per_call_full
    desc = (f"{reps} calls of 1 request x {qlen} query tokens over a {ctx}-token context, scaled x{scale:.1f} by "
            f"(query, key) pairs to {w['seqs']} x {w['qlen']} tokens over {w['ctx']}")
    return tok_s, desc, os.cpu_count()


def run_reference(args, w, rank, world):
    if rank != 0:
        return
    steps = []
    for _ in range(args.warmup):
        cpu_sample(w, budget_s=1.0)
    desc = cores = None
    for _ in range(args.steps):
        v, desc, cores = cpu_sample(w, budget_s=max(2.0, 20.0 / max(1, args.steps)))
        steps.append(v)
    value = statistics.median(steps)
    line = {"impl": "reference", "metric": "prefill_tok_s" if w.get("prefill") else "decode_tok_s", "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * w["qlen"] * w["seqs"] / value,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": args.workload, **w, "nq": NQ, "nkv": NKV, "head_size": HS, "block_size": BS},
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": "port", "sample": desc},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------------- GPU arm


def run_prefill(args, w, rank, world, local_rank):
    """Chunk prefill (c3): one request, qlen queries over the cached context, on the tensor cores."""
    import torch
    from vllm_quantpack_b200 import _lib
    from vllm_quantpack_b200.attention import ops
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    R = build_request(torch, ops, w, device, 1, seed=rank)
    kc, vc, ks, vs = R["views"]
    q = R["q"]
    out = torch.empty_like(q)
    row = R["table"][0].contiguous()
    call = dict(block_row=row, n=w["ctx"], softmax_scale=HS ** -0.5, k_scale_cache=ks, v_scale_cache=vs)
    flush = torch.empty(2 * FLUSH_BYTES, dtype=torch.uint8, device=device)
    q_host = q.cpu().pin_memory()
    out_host = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    q_dev = torch.empty_like(q)

    def step():
        ops.prefill(q, kc, vc, out, **call)

    def e2e_step():
        q_dev.copy_(q_host, non_blocking=True)
        ops.prefill(q_dev, kc, vc, out, **call)
        out_host.copy_(out, non_blocking=True)

    with Clocks(local_rank) as clk:
        t = timed_steps(torch, step, args.steps, args.warmup, flush)
    t_e2e = timed_steps(torch, e2e_step, args.steps, args.warmup, flush)
    dev_err = _lib.device_error()
    ms, ms_e = statistics.mean(t), statistics.mean(t_e2e)
    if rank != 0:
        return
    flops = prefill_flops(w)
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            peak, kind = float(json.load(fh)["bf16_tflops"]), "measured"
    except Exception:
        peak, kind = 1590.0, "fallback"
    achieved = flops / (ms * 1e-3) / 1e12
    cpu = None
    if not args.no_cpu:
        v, desc, cores = cpu_sample(w)
        cpu = {"value": v, "unit": "tok/s", "cores": cores, "kind": "port", "sample": desc}
    line = {"metric": "prefill_tok_s", "value": w["qlen"] / (ms * 1e-3), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int4+f16", "data": "synthetic",
            "config": {"workload": args.workload, **w, "nq": NQ, "nkv": NKV, "head_size": HS, "block_size": BS,
                       "l2": "flushed before every step (256 MB write, then 256 MB read); cache larger than L2"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": TRAFFIC.get(args.workload),
                         "traffic_unit": "bytes per launch (ncu dram__bytes_read + write)",
                         "kernel": "prefill_kernel (q prep + piece fold included)",
                         "algorithmic_flops_per_launch": flops, "peak_kind": kind},
            "cpu_baseline": cpu,
            "e2e": {"value": w["qlen"] / (ms_e * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": q.numel() * 2,
                    "d2h_bytes_per_step": out.numel() * 2},
            "gpu_launches": 3 * args.steps, "clocks": clk.summary(), "device_error": dev_err}
    print(json.dumps(line), flush=True)


def run_b200(args, w, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from vllm_quantpack_b200 import _lib
    from vllm_quantpack_b200.attention import ops
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    seqs = w["seqs"]
    R = build_request(torch, ops, w, device, seqs, seed=rank)
    kc, vc, ks, vs = R["views"]
    q, cu, used, table = R["q"], R["cu"], R["used"], R["table"]
    out = torch.empty_like(q)
    nsplit = ops.decode_num_splits(seqs, NKV, w["ctx"], ops.sm_count(device))
    call = dict(cu_seqlens_q=cu, max_seqlen_q=w["qlen"], seqused_k=used, max_seqlen_k=w["ctx"],
                softmax_scale=HS ** -0.5, block_table=table, k_scale_cache=ks, v_scale_cache=vs, num_splits=nsplit)
    flush = torch.empty(2 * FLUSH_BYTES, dtype=torch.uint8, device=device)

    def step():
        ops.paged_decode(q, kc, vc, out, **call)

    def kernel_only():
        ops.paged_decode(q, kc, vc, out, partials_only=True, **call)

    # e2e: host q (pinned) -> device, the public op, out -> pinned host; cache resident in HBM
    q_host = q.cpu().pin_memory()
    out_host = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    q_dev = torch.empty_like(q)

    def e2e_step():
        q_dev.copy_(q_host, non_blocking=True)
        ops.paged_decode(q_dev, kc, vc, out, **call)
        out_host.copy_(out, non_blocking=True)

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(local_rank) as clk:
        t_step = timed_steps(torch, step, args.steps, args.warmup, flush)
    t_kernel = timed_steps(torch, kernel_only, args.steps, args.warmup, flush)
    t_e2e = timed_steps(torch, e2e_step, args.steps, args.warmup, flush)
    torch.cuda.synchronize()
    dev_err = _lib.device_error()
    ms = statistics.mean(t_step)
    ms_k = statistics.mean(t_kernel)
    ms_e = statistics.mean(t_e2e)
    if world > 1:
        t = torch.tensor([ms, ms_k, ms_e], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_k, ms_e = t.tolist()
    seq_parallel = run_seq_parallel(args, torch, dist, ops, w, device, rank, world, flush) if world > 1 else None
    if rank != 0:
        return
    tokens = world * seqs * w["qlen"]
    bytes_call = algorithmic_bytes(w)
    peak, peak_kind = peaks()
    achieved = bytes_call / (ms_k * 1e-3) / 1e9
    cpu = None
    if world == 1 and not args.no_cpu:
        v, desc, cores = cpu_sample(w)
        cpu = {"value": v, "unit": "tok/s", "cores": cores, "kind": "port", "sample": desc}
    line = {
        "metric": "decode_tok_s", "value": tokens / (ms * 1e-3), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int4+f16" if w["fmt"] == "int4" else "k8v4+f16",
        "data": "synthetic",
        "config": {"workload": args.workload, **w, "nq": NQ, "nkv": NKV, "head_size": HS, "block_size": BS,
                   "num_splits": nsplit, "parallelism": f"requests sharded over {world} GPU(s)" if world > 1 else
                   "1 GPU", "l2": "flushed before every step (256 MB write, then 256 MB read); cache larger than L2"},
        "hbm_gbs": bytes_call * world / (ms * 1e-3) / 1e9 / world,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": TRAFFIC.get(args.workload),
                     "traffic_unit": "bytes per launch (ncu dram__bytes_read + write)",
                     "kernel": "decode_kernel (split-KV, with its query-row prep kernel, without the merge)",
                     "algorithmic_bytes_per_launch": bytes_call, "kernel_ms": ms_k, "peak_kind": peak_kind},
        "cpu_baseline": cpu,
        "e2e": {"value": tokens / (ms_e * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": q.numel() * 2,
                "d2h_bytes_per_step": out.numel() * 2},
        "gpu_launches": 3 * args.steps,  # query prep, split-KV decode, merge
        "clocks": clk.summary(),
        "device_error": dev_err,
        "x16_layers_ms": ms * 16,
    }
    if seq_parallel is not None:
        line["seq_parallel"] = seq_parallel
    print(json.dumps(line), flush=True)


def run_seq_parallel(args, torch, dist, ops, w, device, rank, world, flush):
    """One request of the workload split by sequence range over the ranks: rank r holds cached tokens
    [r * ctx / N, (r + 1) * ctx / N), computes its partial (O fp32 in the RHT domain, base-2 LSE) for all query
    tokens (causal mask shifted by the tokens held after its range), the partials are all-gathered over NCCL and
    every rank folds them (the same fold as the split-KV merge)."""
    from vllm_quantpack_b200.attention import seq_parallel as sp
    lo, hi, after = sp.sequence_range(w["ctx"], rank, world)
    part = dict(w)
    part["ctx"] = hi - lo
    R = build_request(torch, ops, part, device, 1, seed=100 + rank)
    dist.broadcast(R["q"], 0)  # one request: every rank holds the same query tokens
    kc, vc, ks, vs = R["views"]
    runner = sp.SequenceParallelAttention(dist.group.WORLD, R["q"].shape[0], NQ, HS, device)
    out = torch.empty_like(R["q"])
    nsplit = ops.decode_num_splits(1, NKV, part["ctx"], ops.sm_count(device))
    call = dict(cu_seqlens_q=R["cu"], max_seqlen_q=w["qlen"], seqused_k=R["used"], max_seqlen_k=part["ctx"],
                softmax_scale=HS ** -0.5, block_table=R["table"], k_scale_cache=ks, v_scale_cache=vs,
                num_splits=nsplit, tokens_after_keys=after)

    def step():
        runner.decode(R["q"], kc, vc, out, **call)

    dist.barrier()
    t = timed_steps(torch, step, args.steps, args.warmup, flush)
    ms = torch.tensor([statistics.mean(t)], dtype=torch.float64, device=device)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = ms.item()
    return {"value": w["qlen"] / (ms * 1e-3), "unit": "tok/s", "ms_per_step": ms, "scaling": "strong",
            "context_per_rank": part["ctx"], "collective": "NCCL all_gather of [O fp32 | LSE] per rank"}


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="c2a", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline sample")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    w = WORKLOADS[args.workload]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    if args.impl == "reference":
        return run_reference(args, w, rank, world)
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if w.get("prefill"):
            run_prefill(args, w, rank, world, local_rank)
        else:
            run_b200(args, w, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
