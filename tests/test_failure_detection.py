"""Failure detection without a GPU fault.

GPU side: a bounded device wait that nothing satisfies gives up after the
configured limit (1 ms here) and the host reads MOE_ERR_TIMEOUT; a launch whose
experts carry different codebooks is flagged on the device (MOE_ERR_CODEBOOK).
Neither traps, faults or holds the GPU: the kernels run to their end and the
status is read at a synchronisation point.

Host side (CPU): the reference reports residency failures as values
(``TransferResult.success/error``, ``transfer/scheduler.py:363-396``) and
``MoELayer`` raises ``RuntimeError`` (``model/moe_layer.py:89-113``); these
tests inject the failures on the host -- a pinned allocation that fails, an
exhausted pinned budget, a missing store file, a corrupt or short store blob.
"""
from __future__ import annotations

import types

import numpy as np
import pytest
import torch

from moeinfra_b200 import _native


# ---------------------------------------------------------------------------
# GPU: bounded waits and device-side argument checks
# ---------------------------------------------------------------------------

@pytest.fixture
def short_wait_limit():
    old = _native.wait_limit_ns()
    _native.set_wait_limit_ns(1_000_000)  # 1 ms
    try:
        yield
    finally:
        _native.set_wait_limit_ns(old)


@pytest.mark.gpu
def test_bounded_wait_times_out_and_reports_status(short_wait_limit):
    from moeinfra_b200 import kernels

    assert _native.take_device_error() == 0
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")  # nothing ever sets it
    waited = kernels.probe_wait(flag, target=1)
    status = _native.stream_check(torch.cuda.current_stream().cuda_stream)
    assert status == _native.MOE_ERR_TIMEOUT
    assert int(waited.item()) >= 1_000_000  # gave up only after the limit
    assert int(waited.item()) < 1_000_000_000
    # The error words were cleared by the check; the context is still usable.
    assert _native.stream_check(torch.cuda.current_stream().cuda_stream) == 0
    with pytest.raises(RuntimeError, match="timed out"):
        kernels.probe_wait(flag, target=1)
        kernels.check_device()


@pytest.mark.gpu
def test_bounded_wait_returns_when_the_flag_is_set(short_wait_limit):
    from moeinfra_b200 import kernels

    flag = torch.ones(1, dtype=torch.int32, device="cuda")
    waited = kernels.probe_wait(flag, target=1)
    kernels.check_device()
    assert int(waited.item()) < 1_000_000


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1, 4, 64])
def test_mixed_codebooks_are_flagged(T):
    """Expert 1 carries a different codebook: the decode and GEMM kernels flag it."""
    from moeinfra_b200 import kernels
    from moeinfra_b200._native import NF4Expert
    from moeinfra_b200.model.nf4_format import nf4_code_tensor

    H, I, E, k = 256, 512, 4, 2
    g = torch.Generator(device="cuda").manual_seed(5)
    code = nf4_code_tensor("cuda")
    other = code.clone()
    other[3] += 1e-3
    keep, descs = [code, other], []
    for e in range(E):
        mats = []
        for rows, cols in ((I, H), (I, H), (H, I)):
            q = torch.randint(0, 256, (rows * cols // 2,), dtype=torch.uint8, device="cuda",
                              generator=g)
            a = torch.rand(rows * cols // 64, device="cuda", generator=g) * 0.05 + 0.01
            qt, at = kernels.nf4_tile16(q, a, rows, cols)
            keep += [qt, at]
            mats.append(kernels.matrix_desc(qt, at, other if e >= 1 else code))
        descs.append(NF4Expert(mats[0], mats[1], mats[2]))
    table = kernels.expert_array(descs)
    # Route every token to every expert so expert 1..3 are active.
    gate = torch.zeros(E, H, dtype=torch.float16, device="cuda")
    h = torch.randn(T, H, generator=g, device="cuda").half()
    kernels.check_device()
    kernels.layer_forward(h, gate, table, E, H, I)
    status = _native.stream_check(torch.cuda.current_stream().cuda_stream)
    assert status == _native.MOE_ERR_CODEBOOK
    # Same codebook everywhere: clean.
    same = kernels.expert_array([NF4Expert(d.w1, d.w3, d.w2) for d in descs[:1]] * E)
    kernels.layer_forward(h, gate, same, E, H, I)
    kernels.check_device()


# ---------------------------------------------------------------------------
# Host-side injection (CPU)
# ---------------------------------------------------------------------------

def _tiny_cpu_expert(hidden=64, inter=128, seed=0):
    from moeinfra_b200.model.expert import PrequantizedNF4Expert
    from moeinfra_b200.model.nf4_format import quantize_linear_state

    rng = torch.Generator().manual_seed(seed)
    states = {}
    for name, shape in (("w1", (inter, hidden)), ("w2", (hidden, inter)), ("w3", (inter, hidden))):
        w = (torch.randn(*shape, generator=rng) * 0.02).to(torch.bfloat16)
        states[name] = quantize_linear_state(w)
    return PrequantizedNF4Expert.from_serialized(states["w1"], states["w2"], states["w3"],
                                                 hidden_size=hidden, intermediate_size=inter)


def test_pinned_allocation_failure_releases_the_budget(monkeypatch):
    from moeinfra_b200.transfer import reusable_staging
    from moeinfra_b200.transfer.pinned_memory import PinnedMemoryBudget
    from moeinfra_b200.transfer.reusable_staging import ReusablePinnedStagingPool

    budget = PinnedMemoryBudget(1 << 20)
    pool = ReusablePinnedStagingPool(budget, 1 << 18)

    def failing_empty(*a, **k):
        raise RuntimeError("injected: cudaHostAlloc failed")

    monkeypatch.setattr(reusable_staging.torch, "empty", failing_empty)
    with pytest.raises(RuntimeError, match="injected"):
        pool.acquire()
    assert budget.used_bytes == 0
    assert pool.slot_count == 0


def test_exhausted_pinned_budget_rejects_async_and_fails_sync_transfer():
    from moeinfra_b200.cache.manager import CacheManager
    from moeinfra_b200.cache.types import EvictionPolicy
    from moeinfra_b200.transfer.pinned_memory import PinnedMemoryBudget
    from moeinfra_b200.transfer.reusable_staging import ReusablePinnedStagingPool
    from moeinfra_b200.transfer.scheduler import TransferScheduler
    from moeinfra_b200.transfer.types import (
        TransferDirection, TransferPriority, TransferRequest, TransferStatus,
    )

    cm = CacheManager(gpu_slots=2, cpu_slots=4, policy=EvictionPolicy.LRU)
    cm.put(0, 0, _tiny_cpu_expert(), device="cpu")
    pool = ReusablePinnedStagingPool(PinnedMemoryBudget(0), 1 << 16)  # nothing fits
    sched = TransferScheduler(cm, bandwidth_gbps=8.0, max_concurrent=2, staging_pool=pool,
                              transfer_stream=object())
    req = TransferRequest(request_id="r0", layer_id=0, expert_id=0,
                          direction=TransferDirection.CPU_TO_GPU, priority=TransferPriority.HIGH,
                          issued_at=0.0)
    handle = sched.submit_async(req)
    assert handle.status == TransferStatus.REJECTED
    assert sched.submit(req)
    result = sched.execute_next()
    assert result is not None and not result.success
    assert "staging slot" in result.error
    assert result.bytes_transferred == 0


def test_missing_store_file_raises_file_not_found(tmp_path):
    from tests.helpers import tiny_loader, write_tiny_checkpoint

    write_tiny_checkpoint(tmp_path)
    store = tmp_path / "experts"
    store.mkdir()
    loader = tiny_loader(tmp_path, [str(store)])
    with pytest.raises(FileNotFoundError, match="layer_01_expert_03"):
        loader.load_expert(1, 3)


@pytest.mark.parametrize("damage", ["short_weight", "short_absmax", "bad_quant_type",
                                    "missing_key"])
def test_corrupt_store_file_is_rejected_on_the_host(tmp_path, damage):
    import json

    from safetensors.torch import save_file

    from moeinfra_b200.model.nf4_format import BLOB_KEY, expert_store_tensors, store_file_name
    from moeinfra_b200.transfer.pinned_memory import PinnedMemoryBudget
    from moeinfra_b200.transfer.reusable_staging import ReusablePinnedStagingPool
    from tests.helpers import tiny_loader, write_tiny_checkpoint

    write_tiny_checkpoint(tmp_path)
    store = tmp_path / "experts"
    tensors = expert_store_tensors(_tiny_cpu_expert())
    if damage == "short_weight":
        tensors["w1.weight"] = tensors["w1.weight"][: tensors["w1.weight"].numel() // 2].clone()
    elif damage == "short_absmax":
        tensors["w2.weight.absmax"] = tensors["w2.weight.absmax"][:-1].clone()
    elif damage == "bad_quant_type":
        meta = {"quant_type": "fp4", "blocksize": 64, "dtype": "bfloat16", "shape": [128, 64]}
        tensors["w3." + BLOB_KEY] = torch.tensor(list(json.dumps(meta).encode()), dtype=torch.uint8)
    else:
        del tensors["w2.weight.quant_map"]
    store.mkdir()
    save_file(tensors, str(store / store_file_name(0, 1)))
    loader = tiny_loader(tmp_path, [str(store)])
    pool = ReusablePinnedStagingPool(PinnedMemoryBudget(1 << 20), 1 << 18)
    with pytest.raises(ValueError):
        expert = loader.load_expert(0, 1)  # a missing key fails here
        slot = pool.acquire()
        pool.stage_expert(slot, expert, 0, 1)  # short tensors / bad metadata fail here


def test_moe_layer_raises_runtime_error_when_residency_fails():
    from moeinfra_b200.model.moe_layer import MoELayer

    class FailingScheduler:
        def submit(self, request):
            return True

        def execute_next(self):
            return types.SimpleNamespace(success=False, error="injected copy failure")

    class Cache:
        def get(self, layer, expert):
            return types.SimpleNamespace(device=torch.device("cpu"))

        def put(self, *a, **k):
            pass

    router = types.SimpleNamespace(num_experts=4, hidden_size=8, num_experts_per_tok=2)
    layer = MoELayer(0, router, Cache(), None, FailingScheduler())
    with pytest.raises(RuntimeError, match="injected copy failure"):
        layer._ensure_expert_on_gpu(1)
