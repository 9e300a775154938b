"""Expert-parallel exchange restated on the CPU (torch) -- TEST INFRASTRUCTURE ONLY.

The reference runs every expert of a layer on one GPU (``model/moe_layer.py:
117-211``).  The expert-parallel layer must give each expert the same rows (in
ascending token order per source rank) and combine in the same order, so its
exchange is restated here, step for step, with the layout the CUDA kernels
(``moe_ep_dispatch`` / ``moe_ep_receive`` / ``moe_ep_return``) implement:

* rank r of G owns experts [r*E/G, (r+1)*E/G);
* source: rows sorted by expert (stable, ascending token), padded to ``cap``
  rows per destination, then a header row with that destination's expert
  counts (one all-to-all carries both); ``pair_slot_ep`` addresses the
  returned rows;
* owner: rows regrouped by (local expert, source rank, arrival order);
* return: the inverse move, then the ordered combine of the reference.

Used by the gloo (CPU, world_size 2) tests and as the checker of the GPU kernels.
"""
from __future__ import annotations

import torch


def permute(idx: torch.Tensor, E: int):
    """Stable sort of the (token, slot) pairs by expert: offsets, pair_token, pair_slot."""
    T, k = idx.shape
    flat = idx.reshape(-1)
    order = torch.sort(flat, stable=True).indices
    counts = torch.bincount(flat, minlength=E)
    offsets = torch.zeros(E + 1, dtype=torch.int64)
    offsets[1:] = torch.cumsum(counts, 0)
    pair_token = (order // k).to(torch.int64)
    pair_slot = torch.empty_like(order)
    pair_slot[order] = torch.arange(order.numel())
    return offsets, pair_token, pair_slot


def dispatch(h: torch.Tensor, idx: torch.Tensor, E: int, G: int, cap: int):
    """Source side: ``(send [G*(cap+1), H], counts [E], pair_slot_ep [T*k])``.

    Chunk r is cap token rows (padding rows zero) and a header row whose first
    E/G int32 are rank r's expert counts (rest zero).
    """
    El = E // G
    offsets, pair_token, pair_slot = permute(idx, E)
    H = h.shape[1]
    send = torch.zeros(G * (cap + 1), H, dtype=h.dtype)
    for r in range(G):
        lo, hi = int(offsets[r * El]), int(offsets[(r + 1) * El])
        assert hi - lo <= cap
        send[r * (cap + 1):r * (cap + 1) + hi - lo] = h[pair_token[lo:hi]]
    counts = (offsets[1:] - offsets[:-1]).to(torch.int32)
    for r in range(G):
        header = send[r * (cap + 1) + cap].view(torch.int32)
        header[:El] = counts[r * El:(r + 1) * El]
    expert_of = torch.repeat_interleave(torch.arange(E), offsets[1:] - offsets[:-1])
    owner = expert_of[pair_slot] // El
    slot_ep = (owner * cap + pair_slot - offsets[owner * El]).to(torch.int32)
    return send, counts, slot_ep


def header_counts(recv: torch.Tensor, E: int, G: int, cap: int) -> torch.Tensor:
    """Compact counts [E] read from the header row of each source's chunk."""
    El = E // G
    return torch.cat([recv[s * (cap + 1) + cap].view(torch.int32)[:El] for s in range(G)])


def receive_plan(recv_counts: torch.Tensor, E: int, G: int):
    """``(local_offsets [El+1], dst [G][rows]: x_sorted row of each received row)``."""
    El = E // G
    cnt = recv_counts.reshape(G, El).to(torch.int64)
    local_off = [0]
    dst_base = torch.zeros(G, El, dtype=torch.int64)
    acc = 0
    for j in range(El):
        for s in range(G):
            dst_base[s, j] = acc
            acc += int(cnt[s, j])
        local_off.append(acc)
    dst = []
    for s in range(G):
        rows = []
        for j in range(El):
            rows += [int(dst_base[s, j]) + m for m in range(int(cnt[s, j]))]
        dst.append(rows)
    return torch.tensor(local_off, dtype=torch.int32), dst


def receive(recv: torch.Tensor, E: int, G: int, cap: int):
    """``(x_sorted [G*cap, H], local_offsets [El+1], counts [E])`` from a received buffer."""
    counts = header_counts(recv, E, G, cap)
    local_off, dst = receive_plan(counts, E, G)
    x = torch.zeros(G * cap, recv.shape[1], dtype=recv.dtype)
    for s in range(G):
        for i, d in enumerate(dst[s]):
            x[d] = recv[s * (cap + 1) + i]
    return x, local_off, counts


def give_back(y_sorted: torch.Tensor, recv_counts: torch.Tensor, E: int, G: int, cap: int):
    _, dst = receive_plan(recv_counts, E, G)
    y_back = torch.zeros(G * cap, y_sorted.shape[1], dtype=y_sorted.dtype)
    for s in range(G):
        for i, d in enumerate(dst[s]):
            y_back[s * cap + i] = y_sorted[d]
    return y_back


def combine(y_home: torch.Tensor, slot_ep: torch.Tensor, idx: torch.Tensor, w: torch.Tensor):
    """out[t] = fp16(out[t] + fp32(y) * w) over the token's experts in ascending id."""
    T, k = idx.shape
    out = torch.zeros(T, y_home.shape[1], dtype=torch.float16)
    for t in range(T):
        acc = torch.zeros(y_home.shape[1], dtype=torch.float16)
        for j in sorted(range(k), key=lambda j: int(idx[t, j])):
            y = y_home[int(slot_ep[t * k + j])].float()
            acc = (acc.float() + y * w[t, j].float()).to(torch.float16)
        out[t] = acc
    return out
