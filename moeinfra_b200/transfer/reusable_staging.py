"""Reusable pinned staging slots, one contiguous slab per slot.

API of the reference's ``transfer/reusable_staging.py``
(``ReusablePinnedStagingPool.acquire / stage_expert / mark_transfer_complete /
release / destroy``, ``:20-284``).  A slot is reusable only once the CUDA
event of its last host-to-device copy has completed (``:72-108``).

B200 layout change: the reference pins one buffer per tensor and issues one
copy per tensor (12+ per expert).  Here a slot owns a single pinned slab of
``slot_size_bytes``; every tensor of the staged expert is packed into it at a
256-byte aligned offset, so the whole expert crosses the host link in one
``cudaMemcpyAsync``.  ``slot.tensors`` keeps the reference's
``{projection: {key: tensor}}`` view (views into the slab), and
``slot.layout`` records ``(projection, key, offset, shape, dtype)``.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import torch

from moeinfra_b200.model.nf4_format import canonical_state, check_projection_sizes
from moeinfra_b200.transfer.pinned_memory import PinnedMemoryBudget

SLAB_ALIGN = 256


def _pin_available() -> bool:
    return torch.cuda.is_available()


@dataclass
class StagingSlot:
    slot_id: int
    size_bytes: int
    tensors: dict = field(default_factory=dict)
    in_use: bool = False
    ready_event: Optional[torch.cuda.Event] = None
    expert_key: Optional[tuple[int, int]] = None
    slab: Optional[torch.Tensor] = None          # pinned uint8 [size_bytes]
    layout: list = field(default_factory=list)   # (proj, key, offset, shape, dtype)
    used_bytes: int = 0


def _align(v: int) -> int:
    return (v + SLAB_ALIGN - 1) // SLAB_ALIGN * SLAB_ALIGN


def plan_layout(states: dict) -> tuple[list, int]:
    """Offsets of every tensor of ``{proj: canonical_state}`` in one slab."""
    layout = []
    off = 0
    for proj in ("w1", "w2", "w3"):
        for key, t in states[proj].items():
            if t is None:
                layout.append((proj, key, None, None, None))
                continue
            layout.append((proj, key, off, tuple(t.shape), t.dtype))
            off = _align(off + t.numel() * t.element_size())
    return layout, off


def slab_views(slab: torch.Tensor, layout: list) -> dict:
    """``{proj: {key: tensor-view}}`` of a slab laid out by :func:`plan_layout`."""
    out: dict = {"w1": {}, "w2": {}, "w3": {}}
    for proj, key, off, shape, dtype in layout:
        if off is None:
            out[proj][key] = None
            continue
        nbytes = 1
        for s in shape:
            nbytes *= s
        nbytes *= torch.empty((), dtype=dtype).element_size()
        out[proj][key] = slab[off:off + nbytes].view(dtype).view(shape)
    return out


class ReusablePinnedStagingPool:
    """Bounded reusable pinned-memory slots (event-gated reuse)."""

    _PROJECTIONS = ("w1", "w2", "w3")

    def __init__(self, budget: PinnedMemoryBudget, slot_size_bytes: int):
        if slot_size_bytes <= 0:
            raise ValueError("slot_size_bytes must be positive")
        self.budget = budget
        self.slot_size_bytes = slot_size_bytes
        self._slots: dict[int, StagingSlot] = {}

    @property
    def slot_count(self) -> int:
        return len(self._slots)

    @property
    def active_slots(self) -> int:
        return sum(s.in_use for s in self._slots.values())

    def _create_slot(self, slot_id: int) -> Optional[StagingSlot]:
        if not self.budget.reserve(self.slot_size_bytes):
            return None
        try:
            slab = torch.empty(self.slot_size_bytes, dtype=torch.uint8, pin_memory=_pin_available())
        except Exception:
            self.budget.release(self.slot_size_bytes)
            raise
        slot = StagingSlot(slot_id=slot_id, size_bytes=self.slot_size_bytes, slab=slab)
        self._slots[slot_id] = slot
        return slot

    def acquire(self, wait: bool = False) -> Optional[StagingSlot]:
        """A free slot whose last copy finished, a new slot within budget, or ``None``.

        With ``wait=True`` and no free slot, block on the oldest in-flight copy.
        """
        for slot in self._slots.values():
            if slot.in_use:
                continue
            if slot.ready_event is not None:
                if not slot.ready_event.query():
                    continue
                slot.ready_event = None
            slot.in_use = True
            return slot
        slot = self._create_slot(len(self._slots))
        if slot is not None:
            slot.in_use = True
            return slot
        if wait:
            pending = [s for s in self._slots.values() if not s.in_use and s.ready_event is not None]
            if pending:
                pending[0].ready_event.synchronize()
                return self.acquire(wait=False)
        return None

    def mark_transfer_complete(self, slot: StagingSlot, stream) -> None:
        """Record on ``stream`` the point after which the slot's copy is done."""
        if not slot.in_use:
            raise RuntimeError("Cannot mark an inactive slot")
        event = torch.cuda.Event()
        event.record(stream)
        slot.ready_event = event

    def release(self, slot: StagingSlot) -> None:
        if not slot.in_use:
            raise RuntimeError("Slot is not in use")
        slot.in_use = False

    def destroy(self) -> None:
        self._slots.clear()
        self.budget.used_bytes = 0

    @staticmethod
    def _tensor_bytes(tensor: Optional[torch.Tensor]) -> int:
        return 0 if tensor is None else tensor.numel() * tensor.element_size()

    @classmethod
    def _projection_state(cls, expert, name: str) -> dict:
        """One projection in canonical form (accepts dict or ``.state`` projections)."""
        projection = getattr(expert, name)
        raw = projection if isinstance(projection, dict) else getattr(projection, "state", None)
        if not isinstance(raw, dict):
            raise TypeError(f"Expert projection {name!r} does not expose serialized NF4 state")
        return canonical_state(raw, name)

    @classmethod
    def _expert_staging_size(cls, expert) -> int:
        states = {n: cls._projection_state(expert, n) for n in cls._PROJECTIONS}
        return plan_layout(states)[1]

    def stage_expert(self, slot: StagingSlot, expert, layer_id: int, expert_id: int) -> None:
        """Copy the expert's canonical tensors into the slot's slab (host memcpy)."""
        if not slot.in_use:
            raise RuntimeError("Slot must be acquired before staging")
        states = {n: self._projection_state(expert, n) for n in self._PROJECTIONS}
        hidden = getattr(expert, "hidden_size", None)
        inter = getattr(expert, "intermediate_size", None)
        if hidden is not None and inter is not None:
            # A short or mis-shaped store tensor fails here, on the host.
            for n, (i_f, o_f) in (("w1", (hidden, inter)), ("w3", (hidden, inter)),
                                  ("w2", (inter, hidden))):
                check_projection_sizes(states[n], i_f, o_f, n)
        layout, nbytes = plan_layout(states)
        if nbytes > slot.size_bytes:
            raise ValueError(f"expert needs {nbytes} staging bytes, slot holds {slot.size_bytes}")
        for proj, key, off, shape, dtype in layout:
            if off is None:
                continue
            src = states[proj][key].detach()
            if src.device.type != "cpu":
                src = src.cpu()
            src = src.contiguous().reshape(-1).view(torch.uint8)
            slot.slab[off:off + src.numel()].copy_(src)
        slot.layout = layout
        slot.used_bytes = nbytes
        slot.tensors = slab_views(slot.slab, layout)
        slot.expert_key = (layer_id, expert_id)

    @staticmethod
    def _copy_into_pinned(source: Optional[torch.Tensor],
                          existing: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
        if source is None:
            return None
        if existing is None:
            existing = torch.empty_like(source, pin_memory=_pin_available())
        if existing.shape != source.shape or existing.dtype != source.dtype:
            raise ValueError("Existing staging buffer does not match source tensor")
        existing.copy_(source)
        return existing


def pin_expert(expert) -> int:
    """Move a CPU expert's NF4 tensors into ONE page-locked slab, in place.

    The CPU tier is authoritative and, where host RAM allows, can live in
    pinned memory: a GPU miss is then a single ``cudaMemcpyAsync`` of the slab
    (no pageable -> pinned staging copy of ~95 MB per Mixtral expert).  The
    expert's serialized tensors are rebound to views of the slab (no second
    copy is kept); ``expert.pinned_slab`` / ``pinned_layout`` /
    ``pinned_bytes`` describe it for :func:`~moeinfra_b200.transfer.nf4_transfer.transfer_pinned_expert_to_gpu`.
    Returns the slab size in bytes.
    """
    if getattr(expert, "pinned_slab", None) is not None:
        return expert.pinned_bytes
    states = {n: ReusablePinnedStagingPool._projection_state(expert, n)
              for n in ReusablePinnedStagingPool._PROJECTIONS}
    layout, nbytes = plan_layout(states)
    slab = torch.empty(max(nbytes, 1), dtype=torch.uint8, pin_memory=_pin_available())
    views = slab_views(slab, layout)
    for proj, key, off, shape, dtype in layout:
        if off is not None:
            views[proj][key].copy_(states[proj][key].detach().reshape(shape))
    # Rebind the serialized entries that the canonical keys came from.
    rename = {"absmax": "weight.absmax", "code": "weight.quant_map",
              "state2_absmax": "weight.nested_absmax", "state2_code": "weight.nested_quant_map"}
    for proj in ReusablePinnedStagingPool._PROJECTIONS:
        raw = getattr(expert, proj)
        raw = raw if isinstance(raw, dict) else getattr(raw, "state", None)
        if not isinstance(raw, dict):
            continue
        for key, view in views[proj].items():
            if view is None:
                continue
            for name in (key, rename.get(key)):
                if name in raw and isinstance(raw[name], torch.Tensor) and \
                        raw[name].numel() == view.numel() and raw[name].dtype == view.dtype:
                    raw[name] = view.reshape(raw[name].shape)
                    break
    expert.pinned_slab = slab
    expert.pinned_layout = layout
    expert.pinned_bytes = nbytes
    return nbytes

