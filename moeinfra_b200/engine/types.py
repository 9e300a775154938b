"""Engine request/result types (API of the reference's ``engine/types.py``)."""
from __future__ import annotations

import dataclasses
import enum
from typing import Optional

import torch


class PrefetchPolicy(enum.Enum):
    NONE = "none"
    NEXT_LAYER = "next_layer"
    LOOKAHEAD = "lookahead"


@dataclasses.dataclass
class ForwardRequest:
    input_ids: torch.Tensor
    attention_mask: Optional[torch.Tensor] = None
    max_new_tokens: int = 128


@dataclasses.dataclass
class ForwardResult:
    logits: torch.Tensor
    token_ids: list
    ttft_ms: float
    tps: float
    stage_timings: dict
