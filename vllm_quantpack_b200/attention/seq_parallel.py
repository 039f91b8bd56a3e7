"""One long request split over ranks by sequence range: each rank holds a contiguous range of the sequence's cached
tokens in its own paged pool, computes the attention of every query token over that range, and the per-rank
partials (O fp32 in the RHT domain, base-2 log-sum-exp) are combined exactly by their log-sum-exp.

The combine is the fold the plugin applies to its 16k-token prefill segments (vllm_quantpack/attention/
int4_prefill.py:223-230) and vLLM's reduce_segments to decode segments; here the segments live on different GPUs.
One collective per call: an all-gather (NCCL over NVLink) of each rank's packed [O | lse] buffer, then every rank
folds the P partials locally with the merge kernel (inverse RHT and 1/head fused). Causality: query token i of a
chunk of qlen sits at absolute position n_total - qlen + i; a rank whose keys end `after` tokens before n_total sees
key k of its range iff k <= n_local - qlen + i + after, which the kernels apply through `tokens_after_keys`; only the
rank holding the newest tokens (after = 0) masks anything inside a decode step.

There is no TMA multicast and no library kernel reading peer memory: the exchange is a plain NCCL all-gather into
this GPU's own buffer.
"""
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


class SequenceParallelAttention:
    """Decode (<= 4 MTP tokens) or chunk prefill of one request whose cache is split by sequence range over the
    ranks of `group` (`sequence_range`). Every rank passes all query tokens; `out` receives the full attention in
    the model domain on every rank. Buffers are sized once for `num_tokens` query tokens."""

    def __init__(self, group, num_tokens, num_q_heads, head_size, device):
        self.exchange = PartialExchange(group, num_tokens, num_q_heads, head_size, device)

    def _check(self, q):
        if tuple(q.shape) != self.exchange.shape:
            raise ValueError(f"q {tuple(q.shape)}: this runner holds partials for {self.exchange.shape}")

    def combine(self, out):
        part_o, part_lse = self.exchange.gather()
        return ops.merge_attn_partials(part_o, part_lse, out)

    def decode(self, q, key_cache, value_cache, out, *, tokens_after_keys, **decode_args):
        """This rank's split-KV decode over its range (ops.paged_decode arguments, seqused_k = tokens held here),
        then the exchange and fold."""
        self._check(q)
        x = self.exchange
        ops.paged_decode(q, key_cache, value_cache, x.o, out_fp32_lse=x.lse, tokens_after_keys=tokens_after_keys,
                         **decode_args)
        return self.combine(out)

    def prefill(self, q, key_cache, value_cache, out, *, tokens_after_keys, **prefill_args):
        """This rank's chunk prefill over its range (ops.prefill arguments, n = tokens held here), then the exchange
        and fold."""
        self._check(q)
        x = self.exchange
        ops.prefill(q, key_cache, value_cache, x.o, out_fp32_lse=x.lse, tokens_after_keys=tokens_after_keys,
                    **prefill_args)
        return self.combine(out)
