"""One long request split over ranks by sequence range: each rank holds a contiguous range of the sequence's cached
tokens in its own paged pool, computes the attention of every query token over that range, and the per-rank
partials (O fp32 in the RHT domain, base-2 log-sum-exp) are combined exactly by their log-sum-exp.

The combine is the fold the plugin applies to its 16k-token prefill segments (vllm_quantpack/attention/
int4_prefill.py:223-230) and vLLM's reduce_segments to decode segments; here the segments live on different GPUs.
The exchange: with torch symmetric memory (every rank maps the others' buffers over NVLink) each rank writes its
partial into its own exchange buffer and one kernel (ops.fold_peer_partials) publishes it through flags and folds
all ranks' partials read straight over NVLink, with no collective; otherwise an all-gather (NCCL) of the packed
[O | lse] buffers and the merge kernel. Causality: query token i of a
chunk of qlen sits at absolute position n_total - qlen + i; a rank whose keys end `after` tokens before n_total sees
key k of its range iff k <= n_local - qlen + i + after, which the kernels apply through `tokens_after_keys`; only the
rank holding the newest tokens (after = 0) masks anything inside a decode step.

There is no TMA multicast and no library kernel reading peer memory: the peer reads are plain loads in this build's
own fold kernel, or the exchange is an NCCL all-gather into this GPU's own buffer.
"""
import warnings

import torch
import torch.distributed as dist

from . import ops


def sequence_range(n_total, rank, world):
    """Cached-token range [lo, hi) of a sequence of n_total tokens held by `rank`, and the tokens after it."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    lo = n_total * rank // world
    hi = n_total * (rank + 1) // world
    return lo, hi, n_total - hi


class PartialExchange:
    """Packs this rank's partial, out (tokens, heads, head) fp32 followed by lse (tokens, heads) fp32, into one
    buffer whose size is a multiple of 16 bytes, and all-gathers it over `group`."""

    def __init__(self, group, num_tokens, num_heads, head_size, device):
        self.group = group
        self.world = dist.get_world_size(group)
        self.shape = (num_tokens, num_heads, head_size)
        self.n_o = num_tokens * num_heads * head_size
        self.n_l = num_tokens * num_heads
        self.chunk = (self.n_o + self.n_l + 3) // 4 * 4
        self.send = torch.zeros(self.chunk, dtype=torch.float32, device=device)
        self.recv = torch.empty(self.world * self.chunk, dtype=torch.float32, device=device)
        self.o = self.send[: self.n_o].view(self.shape)
        self.lse = self.send[self.n_o: self.n_o + self.n_l].view(self.shape[:2])

    def gather(self):
        """All-gather the packed partials; returns part_o (P, tokens, heads, head) and part_lse (P, tokens, heads)
        views of the receive buffer (rank order)."""
        dist.all_gather_into_tensor(self.recv, self.send, group=self.group)
        r = self.recv.view(self.world, self.chunk)
        part_o = r[:, : self.n_o].view(self.world, *self.shape)
        part_lse = r[:, self.n_o: self.n_o + self.n_l].view(self.world, *self.shape[:2])
        return part_o, part_lse


class PeerExchange:
    """This rank's partial in an exchange buffer of torch symmetric memory that every rank of `group` maps; the fold
    kernel reads the other ranks' partials over NVLink. Raises when symmetric memory is unavailable."""

    def __init__(self, group, num_tokens, num_heads, head_size, device):
        import torch.distributed._symmetric_memory as symm_mem
        from .. import _lib
        lib = _lib.load()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.shape = (num_tokens, num_heads, head_size)
        nbytes = lib.qp_peer_exchange_bytes(self.world, num_tokens, num_heads, head_size)
        try:
            with warnings.catch_warnings():  # required before rendezvous by older torch, deprecated by newer
                warnings.simplefilter("ignore", FutureWarning)
                symm_mem.enable_symm_mem_for_group(group.group_name)
        except Exception:
            pass
        self.buf = symm_mem.empty(nbytes // 4, dtype=torch.float32, device=device)
        self.buf.zero_()  # flags start below the first epoch
        handle = symm_mem.rendezvous(self.buf, group)
        self.bases = torch.tensor(list(handle.buffer_ptrs), dtype=torch.int64, device=device)
        torch.cuda.synchronize(device)
        dist.barrier(group)
        self.views = []
        n_o = num_tokens * num_heads * head_size
        for parity in (0, 1):
            off = lib.qp_peer_partial_offset(self.world, num_tokens, num_heads, head_size, parity) // 4
            o = self.buf[off: off + n_o].view(self.shape)
            lse = self.buf[off + n_o: off + n_o + num_tokens * num_heads].view(self.shape[:2])
            self.views.append((o, lse))
        self.epoch = 0

    def next_partial(self):
        """The (O, lse) views this call's partial goes to (the parity of the next epoch)."""
        self.epoch += 1
        return self.views[self.epoch & 1]

    def fold(self, out, lse_out=None):
        return ops.fold_peer_partials(self.bases, self.rank, self.world, self.epoch, *self.shape, out, lse_out)


class SequenceParallelAttention:
    """Decode (<= 4 MTP tokens) or chunk prefill of one request whose cache is split by sequence range over the
    ranks of `group` (`sequence_range`). Every rank passes all query tokens; `out` receives the full attention in
    the model domain on every rank. Buffers are sized once for `num_tokens` query tokens."""

    def __init__(self, group, num_tokens, num_q_heads, head_size, device, peer=None):
        """peer: True = the NVLink fold over symmetric memory (raises when unavailable), False = NCCL all-gather,
        None = the NVLink fold when symmetric memory can be set up on every rank, else NCCL."""
        self.shape = (num_tokens, num_q_heads, head_size)
        self.peer = None
        if peer is not False:
            try:
                self.peer = PeerExchange(group, num_tokens, num_q_heads, head_size, device)
            except Exception:
                if peer:
                    raise
            # every rank must take the same path
            ok = torch.tensor([1 if self.peer is not None else 0], dtype=torch.int32, device=device)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
            if not ok.item():
                self.peer = None
        self.exchange = None if self.peer is not None else PartialExchange(group, num_tokens, num_q_heads,
                                                                           head_size, device)

    def _check(self, q):
        if tuple(q.shape) != self.shape:
            raise ValueError(f"q {tuple(q.shape)}: this runner holds partials for {self.shape}")

    def scratch(self):
        """(O, lse) buffers of a partial that no other rank reads (for timing the kernels alone)."""
        if not hasattr(self, "_scratch"):
            dev = self.peer.buf.device if self.peer is not None else self.exchange.send.device
            self._scratch = (torch.empty(self.shape, dtype=torch.float32, device=dev),
                             torch.empty(self.shape[:2], dtype=torch.float32, device=dev))
        return self._scratch

    def _partial(self):
        """Where this call's partial goes: (O, lse) views."""
        if self.peer is not None:
            return self.peer.next_partial()
        return self.exchange.o, self.exchange.lse

    def combine(self, out):
        if self.peer is not None:
            return self.peer.fold(out)
        part_o, part_lse = self.exchange.gather()
        return ops.merge_attn_partials(part_o, part_lse, out)

    def decode(self, q, key_cache, value_cache, out, *, tokens_after_keys, **decode_args):
        """This rank's split-KV decode over its range (ops.paged_decode arguments, seqused_k = tokens held here),
        then the exchange and fold."""
        self._check(q)
        o, lse = self._partial()
        ops.paged_decode(q, key_cache, value_cache, o, out_fp32_lse=lse, tokens_after_keys=tokens_after_keys,
                         **decode_args)
        return self.combine(out)

    def prefill(self, q, key_cache, value_cache, out, *, tokens_after_keys, **prefill_args):
        """This rank's chunk prefill over its range (ops.prefill arguments, n = tokens held here), then the exchange
        and fold."""
        self._check(q)
        o, lse = self._partial()
        ops.prefill(q, key_cache, value_cache, o, out_fp32_lse=lse, tokens_after_keys=tokens_after_keys,
                    **prefill_args)
        return self.combine(out)
