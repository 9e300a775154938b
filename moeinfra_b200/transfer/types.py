"""Transfer types (API of the reference's ``transfer/types.py``)."""
from __future__ import annotations

import dataclasses
import enum


class TransferDirection(enum.Enum):
    CPU_TO_GPU = "cpu_to_gpu"
    GPU_TO_CPU = "gpu_to_cpu"


class TransferPriority(enum.Enum):
    HIGH = 0
    NORMAL = 1
    LOW = 2


@dataclasses.dataclass(frozen=True)
class TransferRequest:
    """Move one expert between tiers; the expert object stays with the cache."""

    request_id: str
    layer_id: int
    expert_id: int
    direction: TransferDirection
    priority: TransferPriority
    issued_at: float


@dataclasses.dataclass(frozen=True)
class TransferResult:
    request_id: str
    success: bool
    elapsed_ms: float
    bytes_transferred: int
    error: str | None = None


class TransferStatus(enum.Enum):
    IN_FLIGHT = "in_flight"
    READY = "ready"
    REJECTED = "rejected"
    CANCELLED = "cancelled"


@dataclasses.dataclass
class TransferHandle:
    request_id: str
    layer_id: int
    expert_id: int
    slot: object
    event: object
    status: TransferStatus = TransferStatus.IN_FLIGHT
    gpu_state: object = None
    cpu_expert: object = None
