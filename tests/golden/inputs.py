"""Seeded input generators shared by the golden generator and the tests.

Shapes and value distributions follow the benchmark configurations: hidden
4096, 8 experts, top-2, gate weights N(0, 0.02) (N(0, 0.05) for the uneven
prefill gate), fp16 hidden states N(0, 1).
"""
from __future__ import annotations

import hashlib

import numpy as np

ROUTER_CASES = {
    "decode_bs1": {"T": 1, "H": 4096, "E": 8, "k": 2, "gate_std": 0.02, "seed": 1},
    "decode_bs64": {"T": 64, "H": 4096, "E": 8, "k": 2, "gate_std": 0.02, "seed": 1},
    "ragged_t17": {"T": 17, "H": 4096, "E": 8, "k": 2, "gate_std": 0.02, "seed": 5},
    "prefill_t4096": {"T": 4096, "H": 4096, "E": 8, "k": 2, "gate_std": 0.05, "seed": 2},
    "small_h64_k1": {"T": 33, "H": 64, "E": 8, "k": 1, "gate_std": 0.3, "seed": 6},
    "e4_k3": {"T": 9, "H": 128, "E": 4, "k": 3, "gate_std": 0.2, "seed": 7},
}

DISPATCH_CASES = {
    "t1_h4096": {"T": 1, "H": 4096, "E": 8, "k": 2, "gate_std": 0.02, "seed": 11},
    "t64_h4096": {"T": 64, "H": 4096, "E": 8, "k": 2, "gate_std": 0.02, "seed": 12},
    "t300_h256": {"T": 300, "H": 256, "E": 8, "k": 2, "gate_std": 0.2, "seed": 13},
    "t5_h128_k1": {"T": 5, "H": 128, "E": 8, "k": 1, "gate_std": 0.2, "seed": 14},
}

ORACLE_LAYER_CASE = {"T": 16, "hidden": 128, "inter": 256, "E": 8, "k": 2,
                     "gate_std": 0.1, "seed": 3}


def sha256_arrays(*arrays: np.ndarray) -> bytes:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.digest()


def router_inputs(case: dict) -> tuple[np.ndarray, np.ndarray]:
    rng = np.random.default_rng(case["seed"])
    wg = (rng.standard_normal((case["E"], case["H"]), dtype=np.float32)
          * np.float32(case["gate_std"])).astype(np.float16)
    h = rng.standard_normal((case["T"], case["H"]), dtype=np.float32).astype(np.float16)
    return h, wg


dispatch_inputs = router_inputs


def fake_expert_scale(e: int) -> float:
    """Per-expert scale of the elementwise stand-in expert."""
    return 0.37 + 0.211 * e


def oracle_layer_inputs(case: dict):
    from oracle import nf4 as onf4

    h, wg = router_inputs({**case, "H": case["hidden"]})
    rng = np.random.default_rng(case["seed"] + 1000)
    experts = [onf4.make_expert(rng, case["hidden"], case["inter"], std=0.05)
               for _ in range(case["E"])]
    return h, wg, experts
