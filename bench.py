"""Benchmark of the B200 quantized KV-cache attention (prints one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--workload c2a|c1|c2b|c3|c4]
                    [--no-cpu] [--no-prefill]

Metric: 262k-context int4-KV decode, query tokens per second of one attention-layer call and the
HBM bandwidth it reaches; prefill tokens per second and the tensor throughput it reaches. A step is one attention call
over a resident paged cache of synthetic data (K, V ~ N(0, 1) with 2 % outlier channels x8, written by the B200
store; q ~ N(0, 1); seeded), with a random block table over a shuffled pool. Workloads:
  c2a  int4, 1 request, context 262144, 4 query tokens (3 MTP drafts)     [default, the headline]
  c1   int4, 1 request, context 131072, 2 query tokens
  c2b  int4, 32 requests x context 32768, 2 query tokens
  c4   k8v4, 1 request, context 262144, 4 query tokens
  c3   int4 prefill: a 1024-query chunk over 229,376 cached tokens (+ its own 1024), causal in the chunk
The default c2a line also carries `prefill`: the c3 chunk measured the same way (its own roofline, e2e and clocks),
and, next to it, the reference's own production prefill (its `prefill_sequence`, FlashAttention 2) timed on the same
cache bytes when the reference is installed in baseline/_ref.

At N > 1 (one process per GPU) the headline is ONE request split by sequence range over the N GPUs: rank r holds
cached tokens [r ctx / N, (r + 1) ctx / N), attends every query token over its range, and the partial (O, LSE) are
all-gathered over NCCL and folded (strong scaling). The side key `batch_sharded` has each GPU serve its own full
request(s) with no collective (weak scaling). The prefill chunk is split the same way.

The caches (>= 138 MB) are larger than L2 and L2 is flushed (256 MB written, then another 256 MB read so that the
write-back of the dirty lines happens before the timed region) before every timed step; each step is timed on the
device with CUDA events on the launching stream, max over ranks. Clocks are sampled while at least one second of
back-to-back steps and then the timed steps run.

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
TRAFFIC = {"c2a": 277.01e6 + 7.30e6, "c3": 1700.8e6 + 120.2e6}


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
LEAD_CYCLES = 100_000     # ~50 us of device spin before each start event: the host enqueues the whole step behind it


def l2_flush(flush):
    """Evict L2: write one half of `flush` (> L2), then read the other half (> L2), so the dirty lines of the write
    are written back here and not during the next timed step (a write-only flush leaves ~126 MB of dirty lines whose
    write-back the timed kernel would pay)."""
    import torch
    half = flush.numel() // 2
    flush[:half].zero_()
    flush[half:].view(torch.int64).sum()


def sustain(torch, fn, seconds=1.0):
    """Back-to-back steps for at least `seconds` (the clock sampler sees the GPU under this load, not idle)."""
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    n = 0
    while time.perf_counter() - t0 < seconds:
        for _ in range(16):
            fn()
        n += 16
        torch.cuda.synchronize()
    return n


def timed_steps(torch, fn, steps, warmup, flush, align=None, lead=True):
    """Run `warmup` untimed steps, then `steps` steps each timed by CUDA events (L2 flushed before each). With several
    ranks, `align` (a one-element all-reduce on the stream) runs after the flush and before the start event, so that
    every rank starts its timed step when the slowest rank has finished its flush: a step with a collective inside
    otherwise also times the other rank's flush and host-launch skew. A short device spin (LEAD_CYCLES) then runs
    before the start event, so that the host has enqueued the step's launches by the time the device reaches it and
    the events time the device work, not the host's launch latency; lead=False (the end-to-end loops) leaves it out,
    so that those times keep whatever launch latency the host adds."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(steps):
        l2_flush(flush)
        if align is not None:
            align()
        if lead:
            torch.cuda._sleep(LEAD_CYCLES)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b))
    return times


def exchange_name(runner):
    if runner is not None and runner.peer is not None:
        return "[O | LSE] partials folded by one kernel reading the peers' buffers over NVLink (symmetric memory)"
    return "NCCL all-gather of [O | LSE] partials + merge kernel"


def rank_aligner(torch, dist, world, device):
    """None on one GPU; else a callable that all-reduces one element over the default group on the current stream."""
    if world == 1:
        return None
    one = torch.ones(1, device=device)
    return lambda: dist.all_reduce(one)


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


def tensor_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            return float(json.load(fh)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def max_over_ranks(torch, dist, world, device, values):
    if world == 1:
        return values
    t = torch.tensor(values, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def reference_fa2_prefill(torch, ops, R, w, flush, args):
    """The reference's production long-chunk prefill (vllm_quantpack/attention/int4_prefill.py:203-232: 16k-token
    bf16 unpacks + FlashAttention 2 + fp32 fold, run through its own `prefill_sequence`) on the same cache bytes and
    the same rotated queries, timed like this build's prefill. vLLM's FA2 build carries sm_80 code only; the image's
    flash_attn 2.8 varlen forward stands in for it. None when the reference (baseline/_ref) or flash_attn is absent."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "vllm_quantpack")):
        return {"unavailable": "reference not installed in baseline/_ref"}
    try:
        if ref not in sys.path:
            sys.path.insert(0, ref)
        from vllm_quantpack.attention import int4_prefill as rp
        from flash_attn import flash_attn_varlen_func
    except Exception as e:
        return {"unavailable": f"reference prefill not importable: {e}"[:200]}

    def fa(q, k, v, *, max_seqlen_q, cu_seqlens_q, max_seqlen_k, cu_seqlens_k, softmax_scale, causal,
           return_softmax_lse, fa_version):
        o, lse, _ = flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                                           softmax_scale=softmax_scale, causal=causal, return_attn_probs=True)
        return o, lse

    kc, vc, ks, vs = R["views"]
    row = R["table"][0].contiguous()
    q_rot = ops.single_rht(R["q"].float()).to(R["q"].dtype)

    def step():
        rp.prefill_sequence(q_rot, kc, vc, ks, vs, row, w["ctx"], HS ** -0.5 / HS, fa)

    t = timed_steps(torch, step, max(3, args.steps // 2), 3, flush)
    ms = statistics.mean(t)
    return {"ms_per_step": ms, "value": w["qlen"] / (ms * 1e-3), "unit": "tok/s",
            "path": "reference prefill_sequence (Triton unpack + flash_attn 2.8 varlen FA2 + fp32 fold)"}


def measure_prefill(args, torch, dist, ops, lib, w, device, rank, world, flush, with_reference):
    """Chunk prefill (c3) on the tensor cores. N = 1: the whole chunk. N > 1: the request's cached context split by
    sequence range over the ranks (each rank attends every query of the chunk over its range; [O | LSE] partials
    all-gathered over NCCL and folded), strong scaling of the one chunk. Returns the JSON object (rank 0)."""
    from vllm_quantpack_b200.attention import seq_parallel as sp
    lo, hi, after = sp.sequence_range(w["ctx"], rank, world)
    part = dict(w, ctx=hi - lo)
    R = build_request(torch, ops, part, device, 1, seed=7 + rank)
    if world > 1:
        dist.broadcast(R["q"], 0)
    kc, vc, ks, vs = R["views"]
    q = R["q"]
    out = torch.empty_like(q)
    call = dict(block_row=R["table"][0].contiguous(), n=part["ctx"], softmax_scale=HS ** -0.5, k_scale_cache=ks,
                v_scale_cache=vs)
    runner = sp.SequenceParallelAttention(dist.group.WORLD, q.shape[0], NQ, HS, device) if world > 1 else None
    align = rank_aligner(torch, dist, world, device)
    q_host = q.cpu().pin_memory()
    out_host = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    q_dev = torch.empty_like(q)

    def kernel_only():          # this rank's chunk prefill over its range
        if runner is None:
            ops.prefill(q, kc, vc, out, **call)
        else:
            ops.prefill(q, kc, vc, runner.scratch()[0], out_fp32_lse=runner.scratch()[1], tokens_after_keys=after,
                        **call)

    def step():
        if runner is None:
            ops.prefill(q, kc, vc, out, **call)
        else:
            runner.prefill(q, kc, vc, out, tokens_after_keys=after, **call)

    def e2e_step():
        q_dev.copy_(q_host, non_blocking=True)
        if runner is None:
            ops.prefill(q_dev, kc, vc, out, **call)
        else:
            runner.prefill(q_dev, kc, vc, out, tokens_after_keys=after, **call)
        out_host.copy_(out, non_blocking=True)

    if world > 1:
        dist.barrier()
    with Clocks(device.index) as clk:
        sustain(torch, step, 1.0)
        t = timed_steps(torch, step, args.steps, args.warmup, flush, align)
    t_k = timed_steps(torch, kernel_only, args.steps, args.warmup, flush, align)
    t_e = timed_steps(torch, e2e_step, args.steps, args.warmup, flush, align, lead=False)
    ms, ms_k, ms_e = max_over_ranks(torch, dist, world, device,
                                    [statistics.mean(t), statistics.mean(t_k), statistics.mean(t_e)])
    refl = reference_fa2_prefill(torch, ops, R, w, flush, args) if with_reference and world == 1 else None
    dev_err = lib.device_error()
    if rank != 0:
        return None
    peak, kind = tensor_peak()
    achieved = prefill_flops(w) / world / (ms_k * 1e-3) / 1e12
    obj = {"metric": "prefill_tok_s", "value": w["qlen"] / (ms * 1e-3), "unit": "tok/s", "ms_per_step": ms,
           "higher_is_better": True, "scaling": "strong" if world > 1 else "single chunk",
           "config": {"workload": "c3", **w, "nq": NQ, "nkv": NKV, "head_size": HS, "block_size": BS,
                      "parallelism": f"context split by sequence range over {world} GPUs, {exchange_name(runner)}"
                      if world > 1 else "1 GPU",
                      "l2": "flushed before every step; cache larger than L2",
                      "timing": "CUDA events; a ~50 us device spin before each start event hides host launch latency (not in e2e)"},
           "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                        "frac": achieved / peak, "traffic": TRAFFIC.get("c3") if world == 1 else None,
                        "traffic_unit": "bytes per launch (ncu dram__bytes_read + write)",
                        "kernel": "prefill_kernel (q prep + piece fold included)" + (
                            "; per rank: its range, flops of the whole chunk / N" if world > 1 else ""),
                        "algorithmic_flops_per_launch": prefill_flops(w) / world, "kernel_ms": ms_k,
                        "peak_kind": kind},
           "e2e": {"value": w["qlen"] / (ms_e * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": q.numel() * 2,
                   "d2h_bytes_per_step": out.numel() * 2},
           "gpu_launches": (3 if world == 1 else 4) * args.steps, "clocks": clk.summary(), "device_error": dev_err}
    if refl is not None:
        if "ms_per_step" in refl:
            refl["speedup_of_this_build"] = refl["ms_per_step"] / ms
        obj["reference_gpu"] = refl
    return obj


def run_prefill(args, w, rank, world, local_rank):
    """--workload c3: the chunk prefill as the headline line."""
    import torch
    import torch.distributed as dist
    from vllm_quantpack_b200 import _lib
    from vllm_quantpack_b200.attention import ops
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    flush = torch.empty(2 * FLUSH_BYTES, dtype=torch.uint8, device=device)
    obj = measure_prefill(args, torch, dist, ops, _lib, w, device, rank, world, flush, with_reference=True)
    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu:
        v, desc, cores = cpu_sample(w)
        cpu = {"value": v, "unit": "tok/s", "cores": cores, "kind": "port", "sample": desc}
    line = {"metric": obj.pop("metric"), "value": obj.pop("value"), "unit": obj.pop("unit"), "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": obj.pop("ms_per_step"),
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
            "dtype": "int4+f16", "data": "synthetic", "config": obj.pop("config"), "cpu_baseline": cpu, **obj}
    print(json.dumps(line), flush=True)


def decode_request_step(torch, ops, R, w, nsplit, runner=None, after=0):
    """(step, kernel_only, e2e_step, q, out) closures of one decode call over the request(s) of R."""
    kc, vc, ks, vs = R["views"]
    q, cu, used, table = R["q"], R["cu"], R["used"], R["table"]
    out = torch.empty_like(q)
    ctx = int(R["ctx"])
    call = dict(cu_seqlens_q=cu, max_seqlen_q=w["qlen"], seqused_k=used, max_seqlen_k=ctx,
                softmax_scale=HS ** -0.5, block_table=table, k_scale_cache=ks, v_scale_cache=vs, num_splits=nsplit)
    q_host = q.cpu().pin_memory()
    out_host = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    q_dev = torch.empty_like(q)

    def run(qq):
        if runner is None:
            ops.paged_decode(qq, kc, vc, out, **call)
        else:
            runner.decode(qq, kc, vc, out, tokens_after_keys=after, **call)

    def step():
        run(q)

    def kernel_only():
        if runner is None:
            ops.paged_decode(q, kc, vc, out, partials_only=True, **call)
        else:
            ops.paged_decode(q, kc, vc, runner.scratch()[0], out_fp32_lse=runner.scratch()[1], tokens_after_keys=after,
                             partials_only=True, **call)

    def e2e_step():
        q_dev.copy_(q_host, non_blocking=True)
        run(q_dev)
        out_host.copy_(out, non_blocking=True)

    return step, kernel_only, e2e_step, q, out


def run_b200(args, w, rank, world, local_rank):
    """Decode workloads. N = 1: one call over the workload's request(s). N > 1: the headline is ONE request of the
    workload split by sequence range over the N GPUs (strong scaling: partial (O, LSE) all-gathered over NCCL and
    folded); the requests sharded over the GPUs (weak scaling, no collective) are the side key `batch_sharded`."""
    import torch
    import torch.distributed as dist
    from vllm_quantpack_b200 import _lib
    from vllm_quantpack_b200.attention import ops
    from vllm_quantpack_b200.attention import seq_parallel as sp
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    flush = torch.empty(2 * FLUSH_BYTES, dtype=torch.uint8, device=device)
    align = rank_aligner(torch, dist, world, device)
    seqs = w["seqs"]
    sms = ops.sm_count(device)
    # the headline request(s): the whole workload (N = 1), or this rank's sequence range of it (N > 1)
    if world == 1:
        part, after, runner = dict(w), 0, None
        R = build_request(torch, ops, part, device, seqs, seed=0)
    else:
        lo, hi, after = sp.sequence_range(w["ctx"], rank, world)
        part = dict(w, ctx=hi - lo)
        R = build_request(torch, ops, part, device, seqs, seed=100 + rank)
        dist.broadcast(R["q"], 0)  # the same query tokens on every rank
        runner = sp.SequenceParallelAttention(dist.group.WORLD, R["q"].shape[0], NQ, HS, device)
    R["ctx"] = part["ctx"]
    nsplit = ops.decode_num_splits(seqs, NKV, part["ctx"], sms)
    step, kernel_only, e2e_step, q, out = decode_request_step(torch, ops, R, w, nsplit, runner, after)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(local_rank) as clk:
        sustain(torch, step, 1.0)
        t_step = timed_steps(torch, step, args.steps, args.warmup, flush, align)
    t_kernel = timed_steps(torch, kernel_only, args.steps, args.warmup, flush, align)
    t_e2e = timed_steps(torch, e2e_step, args.steps, args.warmup, flush, align, lead=False)
    torch.cuda.synchronize()
    ms, ms_k, ms_e = max_over_ranks(torch, dist, world, device,
                                    [statistics.mean(t_step), statistics.mean(t_kernel), statistics.mean(t_e2e)])
    batch = None
    if world > 1:   # side key: each rank serves its own full request(s) of the workload, no collective
        del R
        Rb = build_request(torch, ops, w, device, seqs, seed=rank)
        Rb["ctx"] = w["ctx"]
        nb = ops.decode_num_splits(seqs, NKV, w["ctx"], sms)
        bstep, _, _, _, _ = decode_request_step(torch, ops, Rb, w, nb)
        dist.barrier()
        tb = timed_steps(torch, bstep, args.steps, args.warmup, flush, align)
        (msb,) = max_over_ranks(torch, dist, world, device, [statistics.mean(tb)])
        batch = {"value": world * seqs * w["qlen"] / (msb * 1e-3), "unit": "tok/s", "ms_per_step": msb,
                 "scaling": "weak", "parallelism": f"requests sharded over {world} GPUs, no collective"}
        del Rb
    pf = None
    if args.workload == "c2a" and not args.no_prefill:
        pf = measure_prefill(args, torch, dist, ops, _lib, WORKLOADS["c3"], device, rank, world, flush,
                             with_reference=not args.no_cpu)
    dev_err = _lib.device_error()
    if rank != 0:
        return
    tokens = seqs * w["qlen"]
    bytes_rank = algorithmic_bytes(part)
    peak, peak_kind = peaks()
    achieved = bytes_rank / (ms_k * 1e-3) / 1e9
    cpu = None
    if world == 1 and not args.no_cpu:
        v, desc, cores = cpu_sample(w)
        cpu = {"value": v, "unit": "tok/s", "cores": cores, "kind": "port", "sample": desc}
    line = {
        "metric": "decode_tok_s", "value": tokens / (ms * 1e-3), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "dtype": "int4+f16" if w["fmt"] == "int4" else "k8v4+f16", "data": "synthetic",
        "config": {"workload": args.workload, **w, "nq": NQ, "nkv": NKV, "head_size": HS, "block_size": BS,
                   "num_splits": nsplit, "parallelism": f"one request split by sequence range over {world} GPUs "
                   f"({part['ctx']} tokens each), {exchange_name(runner)}" if world > 1 else "1 GPU",
                   "l2": "flushed before every step (256 MB write, then 256 MB read); cache larger than L2",
                   "timing": "CUDA events; a ~50 us device spin before each start event hides host launch latency (not in e2e)"},
        "hbm_gbs": bytes_rank / (ms * 1e-3) / 1e9,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": TRAFFIC.get(args.workload) if world == 1 else None,
                     "traffic_unit": "bytes per launch (ncu dram__bytes_read + write)",
                     "kernel": "decode_kernel (split-KV, with its query-row prep kernel, without the merge)" + (
                         "; per rank over its range" if world > 1 else ""),
                     "algorithmic_bytes_per_launch": bytes_rank, "kernel_ms": ms_k, "peak_kind": peak_kind},
        "cpu_baseline": cpu,
        "e2e": {"value": tokens / (ms_e * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": q.numel() * 2,
                "d2h_bytes_per_step": out.numel() * 2},
        "gpu_launches": 3 * args.steps,  # query prep, split-KV decode, merge
        "clocks": clk.summary(),
        "device_error": dev_err,
        "x16_layers_ms": ms * 16,
    }
    if batch is not None:
        line["batch_sharded"] = batch
    if pf is not None:
        line["prefill"] = pf
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="c2a", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline sample (and the reference prefill)")
    ap.add_argument("--no-prefill", action="store_true", help="c2a: leave out the nested c3 prefill object")
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
