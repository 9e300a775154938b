"""Expert parallelism: one process per GPU, experts of a layer sharded over ranks.

Rank ``r`` of ``G`` owns experts ``[r*E/G, (r+1)*E/G)`` of every layer.  Each
rank routes its own tokens; a layer step is

    router -> permute -> ep_dispatch -> all_to_all(rows, with a count header
           per rank) -> ep_receive -> experts (local, grouped) -> ep_return
           -> all_to_all(rows back) -> combine (ascending expert id)

The exchanged buffers are capacity-padded (``cap = tokens * min(k, E/G)`` rows
per rank pair, plus one header row carrying the pair's expert counts), so the
two all-to-alls have equal splits and no step reads a count back to the host:
the step is a fixed sequence of kernels and two NCCL calls per layer.  Per
token the result equals the single-GPU layer (``model/moe_layer.py:117-211``
of the reference): each expert sees the same rows and the combine runs in the
same order with the same roundings.
"""
from __future__ import annotations

from typing import Sequence

import torch
import torch.distributed as dist

from moeinfra_b200 import kernels


def owner(expert: int, num_experts: int, world: int) -> int:
    """Rank that holds ``expert`` (contiguous blocks of E/G experts)."""
    return expert // (num_experts // world)


def local_experts(rank: int, num_experts: int, world: int) -> list[int]:
    per = num_experts // world
    return list(range(rank * per, (rank + 1) * per))


def capacity(max_tokens: int, top_k: int, num_experts: int, world: int) -> int:
    """Rows one rank can send another: each token reaches at most min(k, E/G) of its experts."""
    return max(1, max_tokens * min(top_k, num_experts // world))


def check_layout(num_experts: int, world: int) -> None:
    if world < 1 or num_experts % world:
        raise ValueError(f"{num_experts} experts cannot be sharded evenly over {world} ranks")


class ExpertParallelMoE:
    """One MoE layer whose experts are sharded over the ranks of ``group``.

    ``router`` is an ``ExpertRouter`` (gate replicated on every rank);
    ``experts`` are this rank's resident NF4 experts in ascending expert id.
    ``max_tokens`` bounds the tokens any rank passes per call (it sizes the
    padded exchange and must be the same on every rank).
    """

    def __init__(self, router, experts: Sequence, rank: int, world_size: int, max_tokens: int,
                 group=None, peer=None, layer_slot: int = 0) -> None:
        """``peer`` (a :class:`~moeinfra_b200.ep_p2p.PeerExchange`, optional) switches both
        exchanges from NCCL all-to-alls to stores into peer memory for calls that fit its
        regions (decode); larger calls (prefill) use NCCL.  ``layer_slot`` picks this layer's
        regions.  Every rank passes the same token count per call; calls with more than
        ``max_tokens`` tokens are refused."""
        self.router = router
        self.num_experts = router.num_experts
        self.top_k = router.num_experts_per_tok
        check_layout(self.num_experts, world_size)
        if len(experts) != self.num_experts // world_size:
            raise ValueError(f"rank {rank} needs {self.num_experts // world_size} experts, "
                             f"got {len(experts)}")
        self.rank, self.world, self.group = rank, world_size, group
        self.max_tokens = max_tokens
        self.cap = capacity(max_tokens, self.top_k, self.num_experts, world_size)
        self.experts = list(experts)
        self.hidden = experts[0].hidden_size
        self.inter = experts[0].intermediate_size
        self._table = kernels.expert_array([ex.nf4_descriptor for ex in self.experts])
        self.peer, self.layer_slot = peer, layer_slot
        # The fused front launch runs one CTA per token, all resident at once.
        self._sms = torch.cuda.get_device_properties(peer.device).multi_processor_count \
            if peer is not None else 0
        self._counters = None  # expert-stage counters the fused front zeroes (decode calls)
        if peer is not None and peer.world != world_size:
            raise ValueError("peer exchange regions belong to another world size")

    def __call__(self, h: torch.Tensor) -> torch.Tensor:
        return self.forward(h)

    def _exchange(self, out: torch.Tensor, inp: torch.Tensor, exchange: bool) -> None:
        if exchange:
            dist.all_to_all_single(out, inp, group=self.group)
        else:  # timing aid: the kernels alone, each rank exchanging with itself
            out.copy_(inp)

    def _cap(self, tokens: int) -> int:
        """Rows per rank pair for a call of ``tokens`` tokens (every rank passes the same count)."""
        return capacity(tokens, self.top_k, self.num_experts, self.world)

    def _dispatch(self, h: torch.Tensor, exchange: bool = True):
        E, G, k = self.num_experts, self.world, self.top_k
        cap = self._cap(h.shape[0])
        _, w, idx = kernels.router_topk(h, self.router.gate_f16(), k, with_logits=False)
        offsets, pair_token, _, pair_slot = kernels.permute(idx, w, E)
        send, slot_ep = kernels.ep_dispatch(h, offsets, pair_token, pair_slot, k, E, G, cap)
        recv = torch.empty_like(send)
        self._exchange(recv, send, exchange)  # rows + count headers
        x_sorted, local_off, recv_counts = kernels.ep_receive(recv, E, G, cap)
        return x_sorted, local_off, recv_counts, slot_ep, idx, w

    @torch.no_grad()
    def received_rows(self, h: torch.Tensor):
        """``(x_sorted, local_offsets)``: the rows this rank's experts get for ``h`` (collective)."""
        x_sorted, local_off, _, _, _, _ = self._dispatch(h.contiguous())
        return x_sorted, local_off

    def exchange_buffers(self, tokens: int):
        """Buffers shaped like one call's two exchanges (for timing the all-to-alls alone)."""
        cap = self._cap(tokens)
        rows_d = self.world * (cap + 1)
        rows_r = self.world * cap
        dev = self.router.gate_f16().device
        return [torch.empty(r, self.hidden, dtype=torch.float16, device=dev)
                for r in (rows_d, rows_d, rows_r, rows_r)]

    def exchange_only(self, bufs) -> None:
        """The layer's two all-to-alls on preallocated buffers, nothing else."""
        send, recv, back, home = bufs
        dist.all_to_all_single(recv, send, group=self.group)
        dist.all_to_all_single(home, back, group=self.group)

    @torch.no_grad()
    def forward(self, h: torch.Tensor, exchange: bool = True) -> torch.Tensor:
        """The layer; ``exchange=False`` (a timing aid) replaces both all-to-alls by local copies."""
        if h.ndim != 2 or h.shape[1] != self.hidden:
            raise ValueError(f"expected [tokens, {self.hidden}] fp16, got {tuple(h.shape)}")
        if h.shape[0] > self.max_tokens:
            raise ValueError(f"{h.shape[0]} tokens exceed max_tokens={self.max_tokens}")
        h = h.contiguous()
        if self.peer is not None and exchange and self._cap(h.shape[0]) <= self.peer.cap:
            return self._forward_p2p(h)
        E, G, cap = self.num_experts, self.world, self._cap(h.shape[0])
        x_sorted, local_off, recv_counts, slot_ep, idx, w = self._dispatch(h, exchange)
        y_sorted = kernels.experts_forward(self._table, local_off, x_sorted, self.hidden, self.inter)
        y_back = kernels.ep_return(y_sorted, recv_counts, E, G, cap)
        y_home = torch.empty_like(y_back)
        self._exchange(y_home, y_back, exchange)
        return kernels.combine(y_home, slot_ep, idx, w)

    def _forward_p2p(self, h: torch.Tensor) -> torch.Tensor:
        """The layer with both exchanges as stores into peer memory (no NCCL call).

        A batch of at most one token per SM takes the fused front launch (router, permute and
        dispatch in one kernel); a receive of at most ``DECODE_MAX_ROWS`` rows hands the expert
        stage's fp32 split partials to the return kernel, which sums them on the way out.  Both
        give the bits of the separate launches."""
        E, G, k, cap = self.num_experts, self.world, self.top_k, self.peer.cap
        R = self.peer.layer(self.layer_slot)
        partials = G * cap <= kernels.DECODE_MAX_ROWS
        counters = None
        if h.shape[0] <= self._sms:
            if partials:  # the front zeroes the expert stage's counters
                if self._counters is None:
                    self._counters = torch.zeros(kernels.expert_counter_words(self.inter),
                                                 dtype=torch.int32, device=h.device)
                counters = self._counters
            w, idx, slot_ep = kernels.ep_front_p2p(h, self.router.gate_f16(), k, E, G, self.rank,
                                                   cap, R.recv_table, R.dflag_table, R.seq_d,
                                                   R.done_d, R.bar, zero=counters)
        else:
            _, w, idx = kernels.router_topk(h, self.router.gate_f16(), k, with_logits=False)
            offsets, pair_token, _, pair_slot = kernels.permute(idx, w, E)
            slot_ep = kernels.ep_dispatch_p2p(h, offsets, pair_token, pair_slot, k, E, G,
                                              self.rank, cap, R.recv_table, R.dflag_table,
                                              R.seq_d, R.done_d)
        x_sorted, local_off, recv_counts = kernels.ep_receive_p2p(R.recv, E, G, cap, R.dflags,
                                                                  R.seq_d)
        if partials:
            part = kernels.experts_forward_partials(self._table, local_off, x_sorted, self.hidden,
                                                    self.inter, counters=counters)
            kernels.ep_return_partials_p2p(part, recv_counts, E, G, self.rank, cap, R.back_table,
                                           R.rflag_table, R.seq_r, R.done_r)
        else:
            y_sorted = kernels.experts_forward(self._table, local_off, x_sorted, self.hidden,
                                               self.inter)
            kernels.ep_return_p2p(y_sorted, recv_counts, E, G, self.rank, cap, R.back_table,
                                  R.rflag_table, R.seq_r, R.done_r)
        return kernels.combine_p2p(R.back, slot_ep, idx, w, G, R.rflags, R.seq_r)

