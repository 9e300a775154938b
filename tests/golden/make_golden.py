"""Generate golden vectors from the reference's own Python code.

Run in the build container only (the reference tree is not present on GPU
boxes):  ``python tests/golden/make_golden.py [/path/to/reference]``.

What runs here is the UNMODIFIED reference code:

* ``engine/router.py`` ``ExpertRouter.route_with_logits`` on CPU in fp16
  (it imports only torch);
* ``model/moe_layer.py`` ``MoELayer._forward_tokens`` with a real reference
  ``CacheManager`` and its ``_ensure_expert_on_gpu`` seam returning
  deterministic experts.  ``model/expert.py`` imports bitsandbytes at module
  level, which is not installed; an import-only stub module (no behaviour)
  is placed in ``sys.modules`` for the duration of this script so the
  imports resolve.  No stubbed symbol is ever called.

Inputs are regenerated in the tests from numpy ``default_rng`` seeds; each
fixture stores a SHA-256 of its inputs so a drifting generator is caught.
"""
from __future__ import annotations

import hashlib
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from tests.golden.inputs import (  # noqa: E402
    DISPATCH_CASES, ORACLE_LAYER_CASE, ROUTER_CASES, dispatch_inputs,
    oracle_layer_inputs, router_inputs, sha256_arrays, fake_expert_scale,
)


def _install_bnb_import_stub() -> None:
    bnb = types.ModuleType("bitsandbytes")
    bnb.nn = types.ModuleType("bitsandbytes.nn")
    bnb.functional = types.ModuleType("bitsandbytes.functional")

    class _Unavailable:  # never instantiated by the code paths used here
        def __init__(self, *a, **k):
            raise RuntimeError("bitsandbytes stub: not callable")

    bnb.nn.Linear4bit = _Unavailable
    bnb.nn.Params4bit = _Unavailable
    bnb.functional.QuantState = _Unavailable
    sys.modules["bitsandbytes"] = bnb
    sys.modules["bitsandbytes.nn"] = bnb.nn
    sys.modules["bitsandbytes.functional"] = bnb.functional


def main(ref_root: str) -> None:
    import torch

    _install_bnb_import_stub()
    sys.path.insert(0, ref_root)
    import engine  # noqa: F401  (breaks the reference's model<->engine import cycle)
    from cache.manager import CacheManager
    from cache.types import EvictionPolicy
    from engine.router import ExpertRouter
    from model.moe_layer import MoELayer

    out: dict[str, np.ndarray] = {}

    # 1. Router: logits, weights, indices from the reference on CPU fp16.
    for name, case in ROUTER_CASES.items():
        h, wg = router_inputs(case)
        router = ExpertRouter(torch.from_numpy(wg), num_experts_per_tok=case["k"])
        lg, w, idx = router.route_with_logits(torch.from_numpy(h))
        out[f"router/{name}/inputs_sha"] = np.frombuffer(sha256_arrays(h, wg), np.uint8)
        out[f"router/{name}/logits"] = lg.numpy()
        out[f"router/{name}/weights"] = w.numpy()
        out[f"router/{name}/indices"] = idx.numpy()

    # 2. Dispatch + combine: reference _forward_tokens with elementwise experts
    #    y_e = fp16(fp32(x) * s_e), reproducible exactly on any device.
    def run_layer(h, wg, k, expert_fn):
        router = ExpertRouter(torch.from_numpy(wg), num_experts_per_tok=k)
        cm = CacheManager(gpu_slots=8, cpu_slots=32, policy=EvictionPolicy.LRU)
        moe = MoELayer(layer_id=0, router=router, cache_manager=cm,
                       model_loader=None, transfer_scheduler=None)
        moe._ensure_expert_on_gpu = expert_fn
        return moe._forward_tokens(torch.from_numpy(h))

    for name, case in DISPATCH_CASES.items():
        h, wg = dispatch_inputs(case)

        def fake(e):
            s = fake_expert_scale(e)
            return lambda x: (x.float() * s).half()

        y = run_layer(h, wg, case["k"], fake)
        lg, w, idx = ExpertRouter(torch.from_numpy(wg), case["k"]).route_with_logits(torch.from_numpy(h))
        out[f"dispatch/{name}/inputs_sha"] = np.frombuffer(sha256_arrays(h, wg), np.uint8)
        out[f"dispatch/{name}/output"] = y.numpy()
        out[f"dispatch/{name}/logits"] = lg.numpy()
        out[f"dispatch/{name}/weights"] = w.numpy()
        out[f"dispatch/{name}/indices"] = idx.numpy()

    # 3. Oracle NF4 experts through the reference's dispatch/combine.
    from oracle import nf4 as onf4

    case = ORACLE_LAYER_CASE
    h, wg, experts = oracle_layer_inputs(case)

    def oracle_expert(e):
        return lambda x: torch.from_numpy(
            onf4.expert_forward(x.numpy(), experts[e], case["hidden"], case["inter"]))

    y = run_layer(h, wg, case["k"], oracle_expert)
    lg, w, idx = ExpertRouter(torch.from_numpy(wg), case["k"]).route_with_logits(torch.from_numpy(h))
    out["oracle_layer/inputs_sha"] = np.frombuffer(sha256_arrays(h, wg), np.uint8)
    out["oracle_layer/output"] = y.numpy()
    out["oracle_layer/weights"] = w.numpy()
    out["oracle_layer/indices"] = idx.numpy()

    np.savez_compressed(HERE / "golden_reference.npz", **out)
    print("wrote", HERE / "golden_reference.npz", len(out), "arrays")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("MOE_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: make_golden.py <path to the reference checkout> "
                 "(or set MOE_REFERENCE_ROOT)")
    main(root)
