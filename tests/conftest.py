"""Shared pytest configuration.

``-m gpu`` tests need a CUDA device (a B200) and the in-tree library
``moeinfra_b200/_lib/libmoe_b200.so``; everything else runs on CPU.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built CUDA library")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_cuda = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_cuda = False
    if has_cuda:
        return
    skip = pytest.mark.skip(reason="CUDA device not available")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    return np.load(ROOT / "tests" / "golden" / "golden_reference.npz")


@pytest.fixture
def config() -> dict:
    return {
        "model": {"name": "mistralai/Mixtral-8x7B-v0.1", "num_experts": 8,
                  "num_experts_per_tok": 2, "num_layers": 32, "hidden_size": 4096,
                  "intermediate_size": 14336, "quantization": "int4"},
        "cache": {"gpu_slots": 8, "cpu_slots": 32, "eviction_policy": "lru"},
        "transfer": {"bandwidth_gbps": 8.0, "prefetch_depth": 2, "max_concurrent_transfers": 4},
    }
