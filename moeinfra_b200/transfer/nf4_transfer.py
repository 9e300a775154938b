"""Host-to-device copy of a staged expert (API of ``transfer/nf4_transfer.py:8-39``).

The reference issues one ``tensor.to("cuda", non_blocking=True)`` per tensor
under the side stream.  Here the slot's whole slab crosses in ONE
``cudaMemcpyAsync`` on ``stream``; the returned state is device views at the
slab's offsets.  The device buffer is allocated on the copy stream (so the
copy never queues behind compute work) and registered with the caller's
current stream; consumers must order themselves after the copy (an event
recorded on ``stream``).
"""
from __future__ import annotations

import torch

from moeinfra_b200.transfer.reusable_staging import StagingSlot, slab_views


def transfer_staged_expert_to_gpu(slot: StagingSlot, stream: torch.cuda.Stream,
                                  device: torch.device | str | None = None) -> dict:
    if not slot.in_use:
        raise RuntimeError("Slot must be acquired before transfer")
    if slot.slab is None or not slot.layout:
        raise RuntimeError("Slot has no staged expert")
    device = torch.device(device) if device is not None else torch.device(
        "cuda", torch.cuda.current_device())
    with torch.cuda.stream(stream):
        dev = torch.empty(slot.used_bytes, dtype=torch.uint8, device=device)
        dev.copy_(slot.slab[:slot.used_bytes], non_blocking=True)
    # The consumer (current) stream uses the buffer too: keep the allocator from
    # recycling it until that stream's work is done as well.
    dev.record_stream(torch.cuda.current_stream(device))
    return slab_views(dev, slot.layout)


def transfer_pinned_expert_to_gpu(expert, stream: torch.cuda.Stream,
                                  device: torch.device | str | None = None) -> dict:
    """One H2D copy of an expert whose CPU copy lives in a pinned slab (``pin_expert``)."""
    slab = getattr(expert, "pinned_slab", None)
    if slab is None:
        raise RuntimeError("expert has no pinned slab; stage it through a staging slot")
    device = torch.device(device) if device is not None else torch.device(
        "cuda", torch.cuda.current_device())
    nbytes = expert.pinned_bytes
    with torch.cuda.stream(stream):
        dev = torch.empty(nbytes, dtype=torch.uint8, device=device)
        dev.copy_(slab[:nbytes], non_blocking=True)
    dev.record_stream(torch.cuda.current_stream(device))
    return slab_views(dev, expert.pinned_layout)

