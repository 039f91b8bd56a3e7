"""The plugin boundary on the CPU: registration, environment switches, the segment table, the k8v4 page cell and
views, and the routing of `unified_attention_int4` (decode batch / prefill chunks / stock fallback) with the
kernels replaced by recorders. Mirrors the reference's CPU tests (tests/test_int4_kv.py:1-87,
tests/test_k8v4_kv.py:16-53); the kernels themselves are checked on a GPU in test_*_gpu.py."""
import logging
import sys
import tomllib
import types

import pytest
import torch

import vllm_quantpack_b200
from vllm_quantpack_b200.attention import int4_kv, int4_prefill, k8v4_kv, ops

LOG = logging.getLogger("test")
NQ, NKV, HS = 24, 4, 256


# ---------------------------------------------------------------- registration and switches
def test_entry_point_names_register():
    with open(__file__.rsplit("/tests/", 1)[0] + "/pyproject.toml", "rb") as fh:
        eps = tomllib.load(fh)["project"]["entry-points"]["vllm.general_plugins"]
    assert eps == {"quantpack_b200": "vllm_quantpack_b200:register"}
    assert callable(vllm_quantpack_b200.register)


def test_register_can_be_disabled(monkeypatch):
    monkeypatch.setenv("VLLM_QUANTPACK_B200", "0")
    assert vllm_quantpack_b200.register() is False


def test_disabled_by_environment(monkeypatch):
    monkeypatch.setenv("VLLM_QUANTPACK_INT4_KV", "0")
    assert int4_kv.patch_int4_kv(LOG) is False


def test_vllm_without_int4_mode_leaves_everything(monkeypatch):
    monkeypatch.setattr(int4_kv, "MODULE", "vllm_quantpack_b200_no_such_module")
    assert int4_kv.patch_int4_kv(LOG) is False


def _fake_stock(monkeypatch):
    """A stand-in for vllm.v1.attention.ops.int4_per_token_head with recording stock functions."""
    mod = types.ModuleType("qp_fake_int4_module")
    mod.calls = []
    mod.unified_attention_int4 = lambda *a, **k: mod.calls.append(("unified", a, k))
    mod.reshape_and_cache_int4 = lambda *a, **k: mod.calls.append(("store", a, k))
    mod.single_rht = lambda x, inverse=False: x
    mod._launch_packed_attn = lambda **k: mod.calls.append(("launch", k))
    monkeypatch.setitem(sys.modules, mod.__name__, mod)
    monkeypatch.setattr(int4_kv, "MODULE", mod.__name__)
    return mod


def test_no_b200_library_or_gpu_leaves_stock(monkeypatch):
    mod = _fake_stock(monkeypatch)
    before = (mod.unified_attention_int4, mod.reshape_and_cache_int4, mod.single_rht, mod._launch_packed_attn)

    def not_ready():
        raise RuntimeError("no CUDA device")

    monkeypatch.setattr(int4_kv, "_b200_ready", not_ready)
    assert int4_kv.patch_int4_kv(LOG) is False
    assert (mod.unified_attention_int4, mod.reshape_and_cache_int4, mod.single_rht, mod._launch_packed_attn) == before


def test_patch_installs_marked_ops_once(monkeypatch):
    mod = _fake_stock(monkeypatch)
    launch = mod._launch_packed_attn
    monkeypatch.setattr(int4_kv, "_b200_ready", lambda: 148)
    assert int4_kv.patch_int4_kv(LOG) is True
    for fn in (mod.unified_attention_int4, mod.reshape_and_cache_int4, mod.single_rht):
        assert fn._quantpack and fn._quantpack_b200
    assert mod._launch_packed_attn is launch   # only the stock path reaches the stock launcher
    installed = mod.unified_attention_int4
    assert int4_kv.patch_int4_kv(LOG) is True and mod.unified_attention_int4 is installed


# ---------------------------------------------------------------- segment buffers and tiles
def _fake_triton_attn(monkeypatch):
    """A stand-in for vllm.v1.attention.backends.triton_attn whose builder records the segment count it saw."""
    mod = types.ModuleType("vllm.v1.attention.backends.triton_attn")
    mod.NUM_PAR_SOFTMAX_SEGMENTS = 16

    class Builder:
        def __init__(self, kv_cache_spec, layer_names, vllm_config, device):
            self.num_par_softmax_segments = mod.NUM_PAR_SOFTMAX_SEGMENTS

    mod.TritonAttentionMetadataBuilder = Builder
    for name in ("vllm", "vllm.v1", "vllm.v1.attention", "vllm.v1.attention.backends"):
        monkeypatch.setitem(sys.modules, name, sys.modules.get(name) or types.ModuleType(name))
    monkeypatch.setitem(sys.modules, mod.__name__, mod)
    monkeypatch.setattr(sys.modules["vllm.v1.attention.backends"], "triton_attn", mod, raising=False)
    return mod


def _config(dtype):
    return types.SimpleNamespace(cache_config=types.SimpleNamespace(cache_dtype=dtype))


def test_decode_segments_only_for_packed_caches(monkeypatch):
    mod = _fake_triton_attn(monkeypatch)
    assert int4_kv._patch_decode_segments(64, LOG) == 64
    B = mod.TritonAttentionMetadataBuilder
    assert B(None, [], _config("int4_per_token_head"), None).num_par_softmax_segments == 64
    assert B(None, [], _config("k8v4_per_token_head"), None).num_par_softmax_segments == 64
    assert B(None, [], _config("auto"), None).num_par_softmax_segments == 16
    assert mod.NUM_PAR_SOFTMAX_SEGMENTS == 16


def test_decode_segments_not_power_of_two_left_stock(monkeypatch):
    mod = _fake_triton_attn(monkeypatch)
    assert int4_kv._patch_decode_segments(48, LOG) == 0
    assert mod.TritonAttentionMetadataBuilder(None, [], _config("int4_per_token_head"),
                                              None).num_par_softmax_segments == 16


def test_decode_override_from_environment(monkeypatch):
    monkeypatch.setenv("VLLM_QUANTPACK_INT4_DECODE", "32,8,32")
    assert int4_kv.decode_tiles(188) == (32, 8, 32)
    assert int4_kv.decode_splits_override() == 32
    monkeypatch.setenv("VLLM_QUANTPACK_INT4_DECODE", "64,4,auto")
    assert int4_kv.decode_tiles(84) == (64, 4, 32)
    assert int4_kv.decode_splits_override() is None


def test_decode_override_accepts_query_row_cap(monkeypatch):
    monkeypatch.setenv("VLLM_QUANTPACK_INT4_DECODE", "64,4,auto,16")
    assert int4_kv.decode_tiles(188) == (64, 4, 64, 16)
    monkeypatch.setenv("VLLM_QUANTPACK_INT4_DECODE", "64,4,32,32")
    assert int4_kv.decode_tiles(84) == (64, 4, 32, 32)


@pytest.mark.parametrize("sms,segments", [(188, 64), (84, 32), (36, 16), (8, 16), (132, 64), (512, 128),
                                          (148, 64)],
                         ids=["rtx-pro-6000", "a40", "rtx-5060-ti", "tiny", "h100", "cap", "b200"])
def test_segments_follow_sm_count(monkeypatch, sms, segments):
    monkeypatch.delenv("VLLM_QUANTPACK_INT4_DECODE", raising=False)
    assert int4_kv.decode_tiles(sms) == (64, 4, segments)


def test_prefill_tiles_override_is_read(monkeypatch):
    monkeypatch.setenv("VLLM_QUANTPACK_INT4_TILES", "64,64,8,2")
    assert int4_kv.prefill_tiles(10) == (64, 64, 8, 2)
    monkeypatch.delenv("VLLM_QUANTPACK_INT4_TILES")
    assert int4_kv.prefill_tiles(10) == int4_kv.PREFILL_TILES_DEFAULT


def test_prefill_thresholds_match_the_plugin():
    assert (int4_prefill.MAX_HEAD, int4_prefill.SEGMENT, int4_prefill.MIN_QUERY, int4_prefill.MIN_CONTEXT) == \
        (256, 16384, 64, 8192)


def test_decode_workspace_bound_covers_every_batch(monkeypatch):
    monkeypatch.delenv("VLLM_QUANTPACK_INT4_DECODE", raising=False)
    from vllm_quantpack_b200 import _lib
    lib = _lib.load()
    for nq, nkv, hs in ((NQ, NKV, HS), (16, 2, 512)):
        bound = int4_kv.decode_workspace_bound(64, nq, nkv, 262144, 148, hs)
        for seqs in (1, 2, 5, 16, 64):
            tokens = min(64, 4 * seqs)
            need = lib.qp_decode_workspace_bytes(tokens, nq, hs, lib.qp_decode_num_splits(seqs, nkv, 262144, 148))
            assert need <= bound
        assert bound < hs << 18   # tens of MB (64 MB at head 256), not the 1024-split worst case


# ---------------------------------------------------------------- k8v4 page cell and views
def test_cell_is_key_bytes_plus_packed_value_plus_two_scales():
    assert k8v4_kv.cell_bytes(256, 256) == 392
    assert k8v4_kv.cell_bytes(128, 64) == 168


@pytest.mark.parametrize("layout", ["hnd", "nhd"])
def test_views_cover_the_cell_without_overlap(layout):
    nb, nkv, bs, hs = 3, 2, 4, 16
    cell = k8v4_kv.cell_bytes(hs, hs)
    if layout == "hnd":
        kv = torch.zeros((nb, nkv, bs, cell), dtype=torch.int8)
    else:
        kv = torch.zeros((nb, bs, nkv, cell), dtype=torch.int8).transpose(1, 2)
    key, value, ks, vs = k8v4_kv.views(kv, hs)
    assert key.shape == (nb, bs, nkv, hs) and key.dtype == torch.int8
    assert value.shape == (nb, bs, nkv, hs // 2) and value.dtype == torch.uint8
    assert ks.shape == vs.shape == (nb, bs, nkv) and ks.dtype == torch.float32
    key.fill_(1)
    ks.view(torch.int32).fill_(0x02020202)
    value.fill_(3)
    vs.view(torch.int32).fill_(0x04040404)
    want = torch.tensor([1] * hs + [2] * 4 + [3] * (hs // 2) + [4] * 4, dtype=torch.int8)
    assert (kv == want).all()
    ks[1, 2, 1] = 7.0
    assert kv[1, 1, 2, hs:hs + 4].view(torch.float32).item() == 7.0


def test_views_reject_another_cell_size():
    with pytest.raises(ValueError, match="expected 392"):
        k8v4_kv.views(torch.zeros((1, 4, 16, 264), dtype=torch.int8), 256)


def test_int4_cache_views_are_not_taken_for_k8v4():
    assert not k8v4_kv.is_k8v4(torch.zeros(1, dtype=torch.uint8))
    assert k8v4_kv.is_k8v4(torch.zeros(1, dtype=torch.int8))


def test_cache_layout_from_views_matches_cells():
    kv = torch.zeros((5, NKV, 16, k8v4_kv.cell_bytes(HS, HS)), dtype=torch.int8)
    lay = ops.CacheLayout(*k8v4_kv.views(kv, HS), HS)
    assert (lay.fmt, lay.cell, lay.ks_off, lay.v_off, lay.vs_off, lay.hnd) == (ops.FMT_K8V4, 392, 256, 260, 388, True)
    phs = HS // 2 + 4
    kv4 = torch.zeros((5, NKV, 16, 2 * phs), dtype=torch.uint8)
    base = torch.tensor([], dtype=torch.float32).set_(kv4.untyped_storage())
    st = [s // 4 for s in kv4.stride()]
    ks = torch.as_strided(base, (5, 16, NKV), (st[0], st[2], st[1]), HS // 2 // 4)
    vs = torch.as_strided(base, (5, 16, NKV), (st[0], st[2], st[1]), (phs + HS // 2) // 4)
    kc, vc = kv4.transpose(1, 2).split(phs, dim=-1)
    lay = ops.CacheLayout(kc, vc, ks, vs, HS)
    assert (lay.fmt, lay.cell, lay.ks_off, lay.v_off, lay.vs_off) == (ops.FMT_INT4, 264, 128, 132, 260)
    with pytest.raises(ValueError):
        ops.CacheLayout(kc, vc, vs, ks, HS)      # scale views swapped: fields out of place


# ---------------------------------------------------------------- routing of unified_attention_int4
class Recorder:
    """Replaces ops.paged_decode / ops.prefill: records each launch and writes the request index + 1 into out."""

    def __init__(self, monkeypatch):
        self.calls = []
        self.windows = []   # the sliding_window of every decode / varlen launch
        monkeypatch.setattr(ops, "paged_decode", self.decode)
        monkeypatch.setattr(ops, "prefill", self.prefill)
        monkeypatch.setattr(ops, "prefill_varlen", self.varlen)

    def decode(self, q, kc, vc, out, *, cu_seqlens_q, seqused_k, block_table, max_seqlen_q, num_splits, **kw):
        self.calls.append(("decode", q.shape[0], cu_seqlens_q.tolist(), seqused_k.tolist(), max_seqlen_q,
                           num_splits))
        self.windows.append(kw.get("sliding_window", 0))
        for b in range(len(seqused_k)):
            out[cu_seqlens_q[b]:cu_seqlens_q[b + 1]] = float(block_table[b, 0])
        return out

    def prefill(self, q, kc, vc, out, *, block_row, n, **kw):
        self.calls.append(("prefill", q.shape[0], n))
        out[:] = float(block_row[0])
        return out

    def varlen(self, q, kc, vc, out, *, cu_seqlens_q, seqused_k, max_seqlen_k, block_table, **kw):
        self.calls.append(("varlen", q.shape[0], cu_seqlens_q.tolist(), seqused_k.tolist(), max_seqlen_k))
        self.windows.append(kw.get("sliding_window", 0))
        for b in range(len(seqused_k)):
            out[cu_seqlens_q[b]:cu_seqlens_q[b + 1]] = float(block_table[b, 0])
        return out


def _step(qlens, used, window=(-1, -1), dtype=torch.float32, nq=NQ, nkv=NKV, hs=HS):
    T = sum(qlens)
    cu = torch.tensor([0] + list(torch.tensor(qlens).cumsum(0)), dtype=torch.int32)
    q = torch.randn((T + 3, nq, hs), dtype=dtype)   # 3 padding rows past cu[-1] stay untouched
    out = torch.full_like(q, -7.0)
    table = torch.tensor([[i + 1] + [0] * 3 for i in range(len(qlens))], dtype=torch.int32)
    kc = torch.zeros((4, 16, nkv, hs // 2 + 4), dtype=torch.uint8)
    args = dict(cu_seqlens_q=cu, max_seqlen_q=max(qlens), seqused_k=torch.tensor(used, dtype=torch.int32),
                max_seqlen_k=max(used), softmax_scale=hs ** -0.5, window_size=window, block_table=table,
                softcap=0.0, sinks=None, alibi_slopes=None, use_alibi_sqrt=False, qq_bias=None, output_scale=None,
                mm_prefix_range=None, k_scale_cache=None, v_scale_cache=None, seq_threshold_3D=32,
                num_par_softmax_segments=64, softmax_segm_output=None, softmax_segm_max=None,
                softmax_segm_expsum=None)
    return q, kc, out, args


def _stock_recorder():
    calls = []

    def stock(q, k, v, out, **kw):
        calls.append((q.shape[0], kw["cu_seqlens_q"].tolist(), kw["seqused_k"].tolist()))
        out[:] = 99.0
    return stock, calls


def test_decode_step_is_one_launch_without_host_read(monkeypatch):
    rec = Recorder(monkeypatch)
    stock, stock_calls = _stock_recorder()
    fn = int4_kv.make_unified_attention(stock)
    monkeypatch.setattr(int4_kv.StepPlan, "of", lambda *a: pytest.fail("decode steps must not read lengths"))
    q, kc, out, args = _step([4, 3, 1, 0, 4], [20000, 9000, 16384, 5, 3072])
    fn(q, kc, kc, out, **args)
    assert rec.calls == [("decode", q.shape[0], [0, 4, 7, 8, 8, 12], [20000, 9000, 16384, 5, 3072], 4, None)]
    assert not stock_calls
    assert (out[:4] == 1).all() and (out[4:7] == 2).all() and (out[7] == 3).all() and (out[8:12] == 5).all()
    assert (out[12:] == -7).all()


def test_mixed_step_splits_decode_prefill(monkeypatch):
    rec = Recorder(monkeypatch)
    stock, stock_calls = _stock_recorder()
    fn = int4_kv.make_unified_attention(stock)
    q, kc, out, args = _step([256, 2, 4, 40], [40000, 20000, 100, 300])
    fn(q, kc, kc, out, **args)
    assert ("decode", 6, [0, 2, 6], [20000, 100], 4, None) in rec.calls
    assert ("prefill", 256, 40000) in rec.calls and ("varlen", 40, [0, 40], [300], 300) in rec.calls
    assert len(rec.calls) == 3 and not stock_calls
    assert (out[:256] == 1).all() and (out[256:258] == 2).all() and (out[258:262] == 3).all()
    assert (out[262:302] == 4).all() and (out[302:] == -7).all()


def test_unsupported_features_go_to_the_stock_path(monkeypatch):
    rec = Recorder(monkeypatch)
    stock, stock_calls = _stock_recorder()
    fn = int4_kv.make_unified_attention(stock)
    q, kc, out, args = _step([4], [5000])
    fn(q, kc, kc, out, **dict(args, alibi_slopes=torch.zeros(NQ)))
    assert not rec.calls and len(stock_calls) == 1
    fn(q, kc, kc, out, **dict(args, qq_bias=torch.zeros(4, 4)))
    assert not rec.calls and len(stock_calls) == 2


def test_sliding_window_layers_run_on_the_split_kv_kernel(monkeypatch):
    """window_size (w, 0) is vLLM's SLIDING_WINDOW = w + 1: decodes take it to the split-KV kernel, and every prefill
    chunk (the long one too: the tcgen05 prefill kernel has no window) goes to the one varlen launch."""
    rec = Recorder(monkeypatch)
    stock, stock_calls = _stock_recorder()
    fn = int4_kv.make_unified_attention(stock)
    q, kc, out, args = _step([4, 1], [5000, 700], window=(1023, 0))
    fn(q, kc, kc, out, **args)
    assert rec.calls == [("decode", q.shape[0], [0, 4, 5], [5000, 700], 4, None)] and rec.windows == [1024]
    rec.calls.clear()
    rec.windows.clear()
    q, kc, out, args = _step([256, 2, 40], [40000, 20000, 300], window=(511, 0))
    fn(q, kc, kc, out, **args)
    assert ("decode", 2, [0, 2], [20000], 2, None) in rec.calls
    assert ("varlen", 296, [0, 256, 296], [40000, 300], 40000) in rec.calls
    assert len(rec.calls) == 2 and rec.windows == [512, 512] and not stock_calls
    assert (out[:256] == 1).all() and (out[256:258] == 2).all() and (out[258:298] == 3).all()
    # no window: (-1, -1); the same step then sends the long chunk to the prefill kernel
    rec.calls.clear()
    q, kc, out, args = _step([256, 2, 40], [40000, 20000, 300])
    fn(q, kc, kc, out, **args)
    assert ("prefill", 256, 40000) in rec.calls and len(rec.calls) == 3
    assert int4_kv.sliding_window_of((-1, -1)) == 0 and int4_kv.sliding_window_of(None) == 0
    assert int4_kv.sliding_window_of((0, 0)) == 1


def test_softcap_layers_run_on_the_split_kv_kernel(monkeypatch):
    """A logit softcap (Gemma-2-style layers) is applied by the split-KV kernel: decodes carry it, and every chunk of
    the step (the long one too: the prefill kernel has no softcap) goes to the varlen launch."""
    rec = Recorder(monkeypatch)
    stock, stock_calls = _stock_recorder()
    fn = int4_kv.make_unified_attention(stock)
    seen = []
    monkeypatch.setattr(ops, "paged_decode", lambda *a, **kw: seen.append(("decode", kw["softcap"], kw["sinks"])))
    monkeypatch.setattr(ops, "prefill_varlen", lambda *a, **kw: seen.append(("varlen", kw["softcap"], kw["sinks"])))
    q, kc, out, args = _step([256, 2, 40], [40000, 20000, 300], window=(4095, 0))
    fn(q, kc, kc, out, **dict(args, softcap=50.0))
    assert sorted(seen) == [("decode", 50.0, None), ("varlen", 50.0, None)] and not rec.calls and not stock_calls
    # sinks (gpt-oss-style layers): the merge folds them in; the long chunk goes to the varlen launch as well
    seen.clear()
    sinks = torch.zeros(NQ)
    q, kc, out, args = _step([256, 2], [40000, 20000])
    fn(q, kc, kc, out, **dict(args, sinks=sinks))
    assert [(c[0], c[2] is sinks) for c in sorted(seen, key=lambda c: c[0])] == [("decode", True), ("varlen", True)]
    assert not stock_calls


def test_head_512_is_served_and_other_head_sizes_go_stock(monkeypatch):
    """Gemma 4 global layers (16 query heads over 2 KV heads, head 512): decodes of up to 4 tokens (32 rows) and
    prefill chunks run on the B200 kernels; a head size the kernels lack (128) stays on the stock int4 path."""
    rec = Recorder(monkeypatch)
    stock, stock_calls = _stock_recorder()
    fn = int4_kv.make_unified_attention(stock)
    q, kc, out, args = _step([4, 1], [16384, 700], nq=16, nkv=2, hs=512)
    fn(q, kc, kc, out, **args)
    assert rec.calls == [("decode", q.shape[0], [0, 4, 5], [16384, 700], 4, None)] and not stock_calls
    rec.calls.clear()
    q, kc, out, args = _step([256, 2], [40000, 9000], nq=16, nkv=2, hs=512)
    fn(q, kc, kc, out, **args)
    assert ("varlen", 256, [0, 256], [40000], 40000) in rec.calls and ("decode", 2, [0, 2], [9000], 2, None) in rec.calls
    assert not stock_calls
    rec.calls.clear()
    q, kc, out, args = _step([4], [5000], hs=128)
    fn(q, kc, kc, out, **args)
    assert not rec.calls and len(stock_calls) == 1


def test_short_chunks_of_a_step_are_one_launch(monkeypatch):
    """32 chunks of 100 tokens over short contexts, a long chunk and a decode in one step: the short chunks are ONE
    varlen launch (the reference's single Triton sub-batch, int4_kv.py:313-323), the long chunk the prefill kernel,
    the decode the split-KV batch; every output row gets its own request's value."""
    rec = Recorder(monkeypatch)
    stock, stock_calls = _stock_recorder()
    fn = int4_kv.make_unified_attention(stock)
    qlens = [100] * 32 + [512, 3]
    used = [300 + 50 * i for i in range(32)] + [600, 20000]
    q, kc, out, args = _step(qlens, used)
    args["block_table"] = torch.arange(1, len(qlens) + 1, dtype=torch.int32)[:, None].repeat(1, 4)
    fn(q, kc, kc, out, **args)
    varlen = [c for c in rec.calls if c[0] == "varlen"]
    assert len(varlen) == 1 and varlen[0][1] == 3200 and varlen[0][2] == list(range(0, 3201, 100))
    assert varlen[0][3] == used[:32] and varlen[0][4] == max(used[:32])
    assert ("prefill", 512, 600) in rec.calls and ("decode", 3, [0, 3], [20000], 3, None) in rec.calls
    assert len(rec.calls) == 3 and not stock_calls
    for i in range(len(qlens)):
        a = sum(qlens[:i])
        assert (out[a:a + qlens[i]] == i + 1).all()


def test_prefill_routing_off_sends_chunks_to_stock(monkeypatch):
    rec = Recorder(monkeypatch)
    stock, stock_calls = _stock_recorder()
    fn = int4_kv.make_unified_attention(stock, prefill_on=False)
    q, kc, out, args = _step([256, 2], [40000, 20000])
    fn(q, kc, kc, out, **args)
    assert rec.calls == [("decode", 2, [0, 2], [20000], 2, None)]
    assert stock_calls == [(256, [0, 256], [40000])]
    assert (out[:256] == 99).all() and (out[256:258] == 2).all()


def test_decode_split_count_from_environment(monkeypatch):
    monkeypatch.setenv("VLLM_QUANTPACK_INT4_DECODE", "64,4,32")
    rec = Recorder(monkeypatch)
    fn = int4_kv.make_unified_attention(_stock_recorder()[0])
    q, kc, out, args = _step([2], [262144])
    fn(q, kc, kc, out, **args)
    assert rec.calls[0][-1] == 32


def test_store_dispatch(monkeypatch):
    calls = []
    monkeypatch.setattr(ops, "reshape_and_cache_int4", lambda *a, **k: calls.append("b200"))
    stock_calls = []
    store = int4_kv.make_reshape_and_cache(lambda *a, **k: stock_calls.append("stock"))
    k = torch.zeros((3, NKV, HS))
    kc8 = torch.zeros((2, 16, NKV, HS), dtype=torch.int8)
    kc4 = torch.zeros((2, 16, NKV, HS // 2), dtype=torch.uint8)
    store(k, k, kc4, kc4, torch.zeros(3, dtype=torch.int64), k_scale_cache=None, v_scale_cache=None)
    store(k, k, kc8, kc8, torch.zeros(3, dtype=torch.int64), k_scale_cache=None, v_scale_cache=None)
    assert calls == ["b200", "b200"] and not stock_calls
    k96 = torch.zeros((3, NKV, 96))
    store(k96, k96, kc4, kc4, torch.zeros(3, dtype=torch.int64), k_scale_cache=None, v_scale_cache=None)
    assert stock_calls == ["stock"]
    with pytest.raises(ValueError, match="k8v4"):
        store(k96, k96, kc8, kc8, torch.zeros(3, dtype=torch.int64), k_scale_cache=None, v_scale_cache=None)


# ---------------------------------------------------------------- k8v4 registration and backend glue (fake vLLM)
def _fake_vllm_for_k8v4(monkeypatch):
    """Stand-ins for the vLLM pieces the k8v4 glue touches: the kv-cache dtype registry, KVQuantMode and the Triton
    attention backend / impl (vllm_quantpack/attention/k8v4_kv.py:89-166 names them)."""
    import dataclasses
    import enum

    ns = types.SimpleNamespace(registry={})
    cache = types.ModuleType("vllm.config.cache")
    cache.get_kv_cache_dtype_handler = lambda name: ns.registry.get(name)
    cache.register_kv_cache_dtype = lambda name: (lambda cls: ns.registry.__setitem__(name, cls) or cls)
    kvi = types.ModuleType("vllm.v1.kv_cache_interface")

    class KVQuantMode(enum.Enum):
        NONE = 0
        INT4_PER_TOKEN_HEAD = 5

    kvi.KVQuantMode = KVQuantMode
    tri = types.ModuleType("vllm.v1.attention.backends.triton_attn")

    @dataclasses.dataclass
    class Spec:
        head_size: int
        head_size_v: int
        dtype: torch.dtype
        kv_quant_mode: object
        state_content_bytes: object = None

    class Backend:
        supported_kv_cache_dtypes = ["auto", "int4_per_token_head"]

        @classmethod
        def customize_spec(cls, spec):
            return dataclasses.replace(spec, state_content_bytes=-1)

    class Impl:
        def __init__(self, dtype, hs):
            self.kv_cache_dtype, self.head_size = dtype, hs
            self._k_scale_cache = self._v_scale_cache = None

        def _ensure_scale_caches(self, kv_cache):
            self._k_scale_cache = "stock"

        def _pth_key_value_caches(self, kv_cache):
            return "stock", "stock"

    tri.TritonAttentionBackend, tri.TritonAttentionImpl = Backend, Impl
    for name in ("vllm", "vllm.config", "vllm.v1", "vllm.v1.attention", "vllm.v1.attention.backends"):
        monkeypatch.setitem(sys.modules, name, types.ModuleType(name))
    for mod in (cache, kvi, tri):
        monkeypatch.setitem(sys.modules, mod.__name__, mod)
    monkeypatch.setattr(sys.modules["vllm.config"], "cache", cache, raising=False)
    monkeypatch.setattr(sys.modules["vllm.v1.attention.backends"], "triton_attn", tri, raising=False)
    ns.Spec, ns.Backend, ns.Impl, ns.mode = Spec, Backend, Impl, KVQuantMode.INT4_PER_TOKEN_HEAD
    return ns


def test_k8v4_dtype_registered_once_with_int8_storage(monkeypatch):
    ns = _fake_vllm_for_k8v4(monkeypatch)
    assert k8v4_kv.register_dtype(LOG) is True
    handler = ns.registry[k8v4_kv.NAME]()
    assert handler.torch_dtype() == torch.int8 and handler.quant_mode() == ns.mode
    first = ns.registry[k8v4_kv.NAME]
    assert k8v4_kv.register_dtype(LOG) is True and ns.registry[k8v4_kv.NAME] is first


def test_k8v4_dtype_not_registered_without_registry(monkeypatch):
    monkeypatch.setitem(sys.modules, "vllm.config.cache", None)
    assert k8v4_kv.register_dtype(LOG) is False


def test_k8v4_backend_patch_sizes_spec_and_serves_views(monkeypatch):
    ns = _fake_vllm_for_k8v4(monkeypatch)
    assert k8v4_kv.patch_backend(None, LOG) is True
    spec = ns.Backend.customize_spec(ns.Spec(256, 256, torch.int8, ns.mode))
    assert spec.state_content_bytes == 392
    assert ns.Backend.customize_spec(ns.Spec(256, 256, torch.uint8, ns.mode)).state_content_bytes == -1  # int4: stock
    assert k8v4_kv.NAME in ns.Backend.supported_kv_cache_dtypes
    kv = torch.zeros((3, NKV, 16, 392), dtype=torch.int8)
    layer = ns.Impl(k8v4_kv.NAME, HS)
    key, value = layer._pth_key_value_caches(kv)
    assert key.dtype == torch.int8 and key.shape == (3, 16, NKV, HS) and value.shape == (3, 16, NKV, HS // 2)
    assert (layer._k_scale_cache == 1).all() and (layer._v_scale_cache == 1).all()
    assert (kv[..., HS:HS + 4].view(torch.float32) == 1).all()      # the scales live inside the cells
    other = ns.Impl("int4_per_token_head", HS)
    assert other._pth_key_value_caches(kv) == ("stock", "stock")
    patched = ns.Impl._pth_key_value_caches
    assert k8v4_kv.patch_backend(None, LOG) is True and ns.Impl._pth_key_value_caches is patched
    assert ns.Backend.supported_kv_cache_dtypes.count(k8v4_kv.NAME) == 1


def test_k8v4_call_outside_the_kernels_raises(monkeypatch):
    """The stock int4 kernel would read a k8v4 cache's int8 keys as nibbles: such calls raise instead."""
    Recorder(monkeypatch)
    stock, stock_calls = _stock_recorder()
    fn = int4_kv.make_unified_attention(stock)
    q, _, out, args = _step([4], [5000])
    kc8 = torch.zeros((4, 16, NKV, HS), dtype=torch.int8)
    with pytest.raises(NotImplementedError, match="k8v4"):
        fn(q, kc8, kc8, out, **dict(args, qq_bias=torch.zeros(4, 4)))
    with pytest.raises(NotImplementedError, match="k8v4"):
        fn(q, kc8, kc8, out, **dict(args, alibi_slopes=torch.zeros(NQ)))
    fn2 = int4_kv.make_unified_attention(stock, prefill_on=False)
    q, _, out, args = _step([256], [40000])
    with pytest.raises(NotImplementedError, match="k8v4"):
        fn2(q, kc8, kc8, out, **args)
    assert not stock_calls


def test_step_plan_is_made_once_per_step(monkeypatch):
    """Every layer of a step gets the same length tensors: only the first layer reads them (one host read)."""
    Recorder(monkeypatch)
    fn = int4_kv.make_unified_attention(_stock_recorder()[0])
    made = []
    init = int4_kv.StepPlan.__init__

    def counting(self, *a):
        made.append(1)
        init(self, *a)

    monkeypatch.setattr(int4_kv.StepPlan, "__init__", counting)
    step = types.SimpleNamespace()
    monkeypatch.setattr(int4_kv, "_forward_step", lambda: step)
    q, kc, out, args = _step([256, 2], [40000, 20000])
    for _ in range(3):
        fn(q, kc, kc, out, **args)
    assert len(made) == 1
    step = types.SimpleNamespace()                     # the next step reads its lengths again
    fn(q, kc, kc, out, **args)
    assert len(made) == 2
    fn(q, kc, kc, out, **dict(args, seqused_k=args["seqused_k"].clone()))   # other tensors, same step: new plan
    assert len(made) == 3


def test_window_sizes_the_split_count_by_the_window():
    """With a sliding window the splits cover only the tiles of the window (plus a partial tile), not the context."""
    assert ops.window_keys(262144, 0, 4) == 262144
    assert ops.window_keys(262144, 1024, 4) == 1024 + 3 + 127
    assert ops.window_keys(500, 1024, 4) == 500
    assert ops.window_keys(262144, 1, 1) == 128


def test_step_split_without_long_chunks():
    """long_chunks=False (window, softcap or sink layers): a chunk that would be long goes with the short ones."""
    cu = [0, 256, 258, 298]
    used = [40000, 20000, 300]
    dec, long, short, stock = int4_kv.split_step(cu, used, group=6)
    assert (dec, long, short, stock) == ([1], [0], [2], [])
    dec, long, short, stock = int4_kv.split_step(cu, used, group=6, long_chunks=False)
    assert (dec, long, short, stock) == ([1], [], [0, 2], [])


def test_sinks_argument_checks():
    """Sinks: one logit per query head, model-domain output only; other dtypes are converted to fp32."""
    assert ops._sinks_ptr(None, NQ, 0) is None
    s32 = torch.zeros(NQ)
    assert ops._sinks_ptr(s32, NQ, 0) == s32.data_ptr()
    assert ops._sinks_ptr(torch.zeros(NQ, dtype=torch.bfloat16), NQ, 0) != 0
    with pytest.raises(ValueError, match="query head"):
        ops._sinks_ptr(torch.zeros(NQ + 1), NQ, 0)
    with pytest.raises(ValueError, match="model-domain"):
        ops._sinks_ptr(s32, NQ, 1)


def test_cache_layout_is_derived_once_per_set_of_views():
    """CacheLayout.of keeps a layout by every input of its derivation: the same views give the same object, a view
    with other strides or offsets is derived (and checked) anew, and an invalid set raises every time."""
    kv4 = torch.zeros((5, NKV, 16, 2 * (HS // 2 + 4)), dtype=torch.uint8)
    base = torch.tensor([], dtype=torch.float32).set_(kv4.untyped_storage())
    st = [s // 4 for s in kv4.stride()]
    phs = HS // 2 + 4
    ks = torch.as_strided(base, (5, 16, NKV), (st[0], st[2], st[1]), HS // 2 // 4)
    vs = torch.as_strided(base, (5, 16, NKV), (st[0], st[2], st[1]), (phs + HS // 2) // 4)
    kc, vc = kv4.transpose(1, 2).split(phs, dim=-1)
    a = ops.CacheLayout.of(kc, vc, ks, vs, HS)
    assert ops.CacheLayout.of(kc, vc, ks, vs, HS) is a
    kc2, vc2 = kv4.transpose(1, 2).split(phs, dim=-1)      # new view objects over the same bytes
    assert ops.CacheLayout.of(kc2, vc2, ks, vs, HS) is a
    for _ in range(2):
        with pytest.raises(ValueError):
            ops.CacheLayout.of(kc, vc, vs, ks, HS)           # scale views swapped
    sub = kc[:4], vc[:4], ks[:4], vs[:4]                     # fewer blocks: another layout
    b = ops.CacheLayout.of(*sub, HS)
    assert b is not a and b.nblocks == 4 and b.args() == a.args()
