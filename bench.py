#!/usr/bin/env python
"""Mixtral NF4 MoE decode benchmark on B200 (one JSON line on rank 0).

Workload (widened to the Mixtral-8x7B MoE stack): a decode
step runs ``--batch`` tokens (default 1) through 32 Mixtral sparse-MoE layers --
gate 4096->8 fp16, top-2 softmax routing, 8 NF4 SwiGLU experts (hidden 4096,
ffn 14336, 64-element blocks, fp32 absmax) per layer -- all experts resident in
HBM.  Each layer sees the step's hidden states (there is no attention between
the layers, so activations do not drift across 32 layers).  Weights: N(0, 0.02)
from per-(layer, expert, projection) seeds, NF4-quantized on the device.
Tokens: N(0, 1) fp16, a different token per step, so routing changes from step
to step.

Arms:
* default (this build): ``value`` = tokens/s of the device-timed step (CUDA
  graph of the 32 layers' fused kernels, inputs resident); ``e2e`` = the same
  tokens/s through the public API (``MoELayer.forward`` per layer, eager) with
  the step's tokens copied from pinned host memory and the step's result (the
  last layer's output) read back to pinned host memory every step; ``roofline``
  from the expert stage (``moe_experts_forward``: the fused gate/up + SwiGLU and
  down GEMV kernel, then the split reduce) timed on its own with CUDA events;
  ``cpu_baseline`` from the CPU restatement
  (``oracle.cpu_path``) on a bounded sample.
* ``--impl reference``: the CPU restatement of the reference's path timed on
  the host cores (bitsandbytes, which the reference's CPU path needs, is not
  available; the restatement is the port).

Multi-GPU (``torchrun --nproc-per-node N``): expert parallelism -- rank r owns
experts [r*8/N, (r+1)*8/N) of every layer; every rank routes its own batch and
exchanges token rows with NCCL all-to-all (dispatch and combine).  Per-GPU
batch is fixed (weak scaling); ``value`` = all ranks' tokens / max-over-ranks
device time.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

HIDDEN, FFN, EXPERTS, TOP_K, LAYERS = 4096, 14336, 8, 2, 32
PROJ_BYTES = FFN * HIDDEN // 2 + FFN * HIDDEN // 64 * 4 + 16 * 4
EXPERT_BYTES = 3 * PROJ_BYTES          # 99,090,624 B of NF4 weights per expert
METRIC = "Mixtral NF4 decode tok/s (bs1, bs64); expert GEMV HBM GB/s vs peak"
SEED = 1
PROFILE_TRAFFIC = ROOT / "profiles" / "expert_stage_decode_bs1.md"
PROFILE_PREFILL = ROOT / "profiles" / "grouped_gemm_prefill.md"


# ----------------------------------------------------------------------------
# synthetic weights
# ----------------------------------------------------------------------------

def _seed(layer: int, expert: int, proj: int) -> int:
    """Per-(layer, expert, projection) seed; expert -1 is the gate."""
    return SEED * 1_000_003 + layer * 1009 + (expert + 1) * 7 + proj


def make_gate(layer: int, device) -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(_seed(layer, -1, 0))
    return (torch.randn(EXPERTS, HIDDEN, generator=g, device=device) * 0.02).to(torch.float16)


def make_expert_store(layer: int, expert: int, device) -> dict:
    """Store-layout NF4 projections {w1, w3, w2: (packed, absmax, code)} on ``device``."""
    from moeinfra_b200.model.nf4_format import quantize_nf4_packed
    out = {}
    for p, (name, shape) in enumerate((("w1", (FFN, HIDDEN)), ("w3", (FFN, HIDDEN)),
                                       ("w2", (HIDDEN, FFN)))):
        g = torch.Generator(device=device).manual_seed(_seed(layer, expert, p))
        w = (torch.randn(*shape, generator=g, device=device) * 0.02).to(torch.bfloat16)
        out[name] = quantize_nf4_packed(w)
        del w
    return out


def make_tokens(n: int, batch: int, device, rank: int = 0) -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(SEED * 7 + 1_000_000 * rank)
    return torch.randn(n, batch, HIDDEN, generator=g, device=device).to(torch.float16)


class _Shape:
    hidden_size = HIDDEN
    intermediate_size = FFN


def resident_expert(layer: int, expert: int, device):
    from moeinfra_b200.transfer.nf4_reconstruct import ReconstructedNF4Expert
    st = make_expert_store(layer, expert, device)
    gpu_state = {n: {"weight": q, "absmax": a, "code": c, "offset": None}
                 for n, (q, a, c) in st.items()}
    return ReconstructedNF4Expert(_Shape(), gpu_state)


# ----------------------------------------------------------------------------
# clocks during the timed region
# ----------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device_index: int) -> None:
        self.proc = None
        self.path = None
        try:
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            self.target = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:
            self.target = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(prefix="moe_clocks_", suffix=".csv")
        os.close(fd)
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
               "-lms", "100"]
        if self.target:
            cmd += ["-i", self.target]
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(cmd, stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        if self.proc is None or not self.path:
            return None
        sm, smax, reasons = [], [], set()
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) != 7:
                    continue
                try:
                    sm.append(float(parts[0]))
                    smax.append(float(parts[1]))
                except ValueError:
                    continue
                for name, v in zip(self.NAMES, parts[3:]):
                    if v.lower() == "active":
                        reasons.add(name)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax),
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------
# CPU baseline (the reference path restated on the host cores)
# ----------------------------------------------------------------------------

def host_cores() -> int:
    """Host threads this process may run on (torchrun sets OMP_NUM_THREADS=1; ignore it)."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def cpu_layer_sample(steps: int, warmup: int, batch: int, time_budget_s: float | None):
    """Time layer steps of the workload with ``oracle.cpu_path`` on every host core.

    Step i runs ``batch`` new tokens through layer ``i % LAYERS`` (that layer's
    gate; the eight experts' NF4 weights are layer 0's for every layer -- a
    host-memory bound on the sample, stated in its description).  Returns
    ``(tok_per_s of the 32-layer stack, list of per-step seconds, threads)``.
    Weights are generated on the host with the device arm's seeds and
    quantizer (host RNG, so values differ; shapes and distributions match).
    """
    from moeinfra_b200.model.nf4_format import NF4_CODE
    from oracle import cpu_path
    threads = host_cores()
    torch.set_num_threads(threads)
    code = torch.tensor(NF4_CODE, dtype=torch.float32)
    gates = {}
    toks = make_tokens(steps + warmup, batch, "cpu")
    experts: dict[int, dict] = {}

    def step(i):
        layer = i % LAYERS
        if layer not in gates:
            gates[layer] = make_gate(layer, "cpu")
        _, _, idx = cpu_path.route(toks[i], gates[layer], TOP_K)
        table = [None] * EXPERTS
        for e in sorted(set(idx.reshape(-1).tolist())):
            if e not in experts:
                st = make_expert_store(0, e, "cpu")
                experts[e] = {n: {"q": q, "absmax": a} for n, (q, a, _) in st.items()}
            table[e] = experts[e]
        t0 = time.perf_counter()
        cpu_path.layer_forward(toks[i], gates[layer], table, code, HIDDEN, FFN, TOP_K)
        return time.perf_counter() - t0

    for i in range(warmup):
        step(i)
    times = []
    for i in range(warmup, warmup + steps):
        times.append(step(i))
        if time_budget_s is not None and sum(times) > time_budget_s and len(times) >= 2:
            break
    per_layer = sum(times) / len(times)
    return batch / (per_layer * LAYERS), times, threads


def cpu_sample_text(times: list, batch: int) -> str:
    per_layer = sum(times) / len(times)
    return (f"{len(times)} steps, each {batch} token(s) through one of the {LAYERS} MoE layers "
            f"(that layer's gate; layer 0's NF4 experts stand in for every layer's); "
            f"{per_layer:.3f} s per layer step; value = tokens / ({LAYERS} x mean layer-step "
            f"time); oracle.cpu_path torch CPU restatement")


def config_dict(L: int, B: int, world: int) -> dict:
    """The workload description, identical in the device and reference arms."""
    return {
        "workload": f"config 1 (Mixtral MoE layer decode) over a {L}-layer MoE stack, "
                    f"bs{B} per GPU",
        "batch_per_gpu": B, "global_batch": B * world, "layers": L, "hidden": HIDDEN,
        "ffn": FFN, "experts": EXPERTS, "top_k": TOP_K, "parallelism": f"ep{world}",
        "l2": "inputs larger than L2: every step streams each layer's routed experts "
              "(99 MB each, 126 MB L2) once, 32 layers per step",
    }


# ----------------------------------------------------------------------------
# device arm
# ----------------------------------------------------------------------------

def _events():
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def _max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def _barrier(world: int):
    if world > 1:
        torch.distributed.barrier()


def _profile_value(path, key: str):
    """A ``key = number`` line of a committed ncu summary (None if absent)."""
    if not path.exists():
        return None
    m = re.search(key + r"\s*[:=]\s*([0-9.eE+]+)", path.read_text())
    return float(m.group(1)) if m else None


def _profile_traffic():
    """DRAM bytes per expert-stage launch from the committed ncu summary, if any."""
    if not PROFILE_TRAFFIC.exists():
        return None
    m = re.search(r"traffic_per_launch_bytes\s*[:=]\s*([0-9.eE+]+)", PROFILE_TRAFFIC.read_text())
    return float(m.group(1)) if m else None


def run_device(args, rank: int, world: int, local_rank: int):
    from moeinfra_b200 import _native, kernels
    from moeinfra_b200.cache.manager import CacheManager
    from moeinfra_b200.cache.types import EvictionPolicy
    from moeinfra_b200.engine.router import ExpertRouter
    from moeinfra_b200.model.moe_layer import MoELayer

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    L, B, K, W = args.layers, args.batch, args.steps, args.warmup
    torch.backends.cuda.matmul.allow_tf32 = False

    # --- build the resident MoE stack --------------------------------------------
    if world == 1:
        cm = CacheManager(gpu_slots=L * EXPERTS, cpu_slots=0, policy=EvictionPolicy.LRU)
        layers, tables, gates = [], [], []
        for l in range(L):
            gate = make_gate(l, dev)
            for e in range(EXPERTS):
                cm.put(l, e, resident_expert(l, e, dev), device="cuda")
            router = ExpertRouter(gate, num_experts_per_tok=TOP_K)
            layers.append(MoELayer(l, router, cm, None, None))
            gates.append(router.gate_f16())
            tables.append(kernels.expert_array(
                [cm.peek_gpu(l, e).nf4_descriptor for e in range(EXPERTS)]))
        step_fn = None
    else:
        from moeinfra_b200.ep import ExpertParallelMoE, capacity
        from moeinfra_b200.ep_p2p import PeerExchange
        per = EXPERTS // world
        owned = list(range(rank * per, (rank + 1) * per))
        peer = None
        if args.ep_exchange == "p2p":
            peer = PeerExchange(L, world, rank, capacity(B, TOP_K, EXPERTS, world), HIDDEN)
        ep_layers, nccl_layers = [], []
        for l in range(L):
            router = ExpertRouter(make_gate(l, dev), num_experts_per_tok=TOP_K)
            local = [resident_expert(l, e, dev) for e in owned]
            ep_layers.append(ExpertParallelMoE(router, local, rank=rank, world_size=world,
                                               max_tokens=B, peer=peer, layer_slot=l))
            nccl_layers.append(ExpertParallelMoE(router, local, rank=rank, world_size=world,
                                                 max_tokens=B))
        step_fn = ep_layers
        owned_experts = owned
    torch.cuda.synchronize()
    _barrier(world)

    tokens = make_tokens(K + W, B, dev, rank)
    h_static = torch.empty(B, HIDDEN, dtype=torch.float16, device=dev)

    # --- device-timed step -------------------------------------------------------
    graph = None
    if world == 1:
        def one_step():
            return [kernels.layer_forward(h_static, gates[l], tables[l], TOP_K, HIDDEN, FFN)[0]
                    for l in range(L)]
        h_static.copy_(tokens[0])
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            one_step()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        c0 = _native.launch_count()
        with torch.cuda.graph(graph):
            graph_outs = one_step()
        launches_per_step = _native.launch_count() - c0

        def run(i):
            h_static.copy_(tokens[i])
            graph.replay()
    else:
        # One eager step (creates the NCCL communicators and counts the
        # library's kernels), then the whole step -- kernels and the NCCL
        # all-to-alls of every layer -- captured in one CUDA graph.
        c0 = _native.launch_count()
        for lay in step_fn:
            lay(tokens[0])
        torch.cuda.synchronize()
        launches_per_step = _native.launch_count() - c0
        h_static.copy_(tokens[0])
        torch.cuda.synchronize()
        _barrier(world)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for lay in step_fn:
                lay(h_static)
        torch.cuda.synchronize()
        _barrier(world)

        def run(i):
            h_static.copy_(tokens[i])
            graph.replay()

    for i in range(W):
        run(i)
    torch.cuda.synchronize()
    _barrier(world)
    start, end = _events()
    with ClockSampler(local_rank) as clocks:
        _barrier(world)
        torch.cuda.synchronize()
        start.record()
        for i in range(W, W + K):
            run(i)
        end.record()
        torch.cuda.synchronize()
        _barrier(world)
    ms_local = start.elapsed_time(end)
    ms = _max_over_ranks(ms_local, world, dev)
    clk = clocks.summary()

    # weight bytes the timed steps streamed (from the routing of each step's token)
    routed_experts = 0
    if world == 1:
        for i in range(W, W + K):
            for l in range(L):
                _, w_, idx = kernels.router_topk(tokens[i], gates[l], TOP_K, with_logits=False)
                routed_experts += len(set(idx.reshape(-1).tolist()))
    total_tokens = B * K * world
    value = total_tokens / (ms / 1e3)

    # --- expert stage alone (roofline of the dominant kernels) ---------------------
    roof = None
    if world == 1:
        stage_bytes = []
        stage_calls = []
        tok = tokens[W]
        for l in range(L):
            _, _, idx = kernels.router_topk(tok, gates[l], TOP_K, with_logits=False)
            offsets, pair_token, _, _ = kernels.permute(idx.contiguous(),
                                                        torch.ones_like(idx, dtype=torch.float32),
                                                        EXPERTS)
            x_sorted = kernels.gather_rows(tok, pair_token)
            n_exp = len(set(idx.reshape(-1).tolist()))
            stage_bytes.append(n_exp * EXPERT_BYTES + 2 * x_sorted.numel() * 2)
            stage_calls.append((offsets, x_sorted))

        def stage():
            for l in range(L):
                kernels.experts_forward(tables[l], stage_calls[l][0], stage_calls[l][1], HIDDEN, FFN)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            stage()
        torch.cuda.current_stream().wait_stream(s)
        g2 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g2):
            stage()
        reps = max(3, K // 2)
        for _ in range(3):
            g2.replay()
        torch.cuda.synchronize()
        a, b = _events()
        a.record()
        for _ in range(reps):
            g2.replay()
        b.record()
        torch.cuda.synchronize()
        per_launch_s = a.elapsed_time(b) / 1e3 / (reps * L)
        bytes_per_launch = sum(stage_bytes) / L
        achieved = bytes_per_launch / per_launch_s / 1e9
        peak = _measured_peak("hbm_gbs")
        traffic = _profile_traffic()
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak[0], "unit": "GB/s",
                "frac": round(achieved / peak[0], 4), "traffic": traffic,
                "kernel": "expert stage (moe_experts_forward: k_stage_mma, one launch for the "
                          "W1/W3 GEMV+SwiGLU and the W2 split-K GEMV, then the split reduce), "
                          "bs1, per layer",
                "algorithmic_bytes_per_launch": int(bytes_per_launch),
                "launch_us": round(per_launch_s * 1e6, 2), "peak_source": peak[1]}
        del g2

    if world > 1:
        roof = ep_roofline(step_fn, tokens[W], dev, L, K)
        e2e = ep_e2e(step_fn, tokens, dev, L, K, W, world)
        ep_par = ep_parity(step_fn[0], tokens[0], dev, rank)
        ep_split = ep_breakdown(step_fn, nccl_layers, tokens[W], dev, L, K, world)

    # --- end to end through the public API, host buffers -----------------------------
    if world == 1:
        e2e = None
        host_in = torch.empty(K + W, B, HIDDEN, dtype=torch.float16).pin_memory()
        host_in.copy_(tokens.cpu())
        host_out = torch.empty(B, HIDDEN, dtype=torch.float16).pin_memory()
        h_dev = torch.empty(B, HIDDEN, dtype=torch.float16, device=dev)

        def e2e_step(i):
            # The step's input up, every layer through the public API, the
            # step's result (the last layer's output) back.
            h_dev.copy_(host_in[i], non_blocking=True)
            y = None
            for l in range(L):
                y = layers[l].forward(h_dev)
            host_out.copy_(y, non_blocking=True)
            torch.cuda.current_stream().synchronize()

        for i in range(W):
            e2e_step(i)
        a, b = _events()
        a.record()
        for i in range(W, W + K):
            e2e_step(i)
        b.record()
        torch.cuda.synchronize()
        e2e_ms = a.elapsed_time(b)
        e2e = {"value": round(B * K / (e2e_ms / 1e3), 3), "unit": "tok/s",
               "h2d_bytes_per_step": B * HIDDEN * 2, "d2h_bytes_per_step": B * HIDDEN * 2,
               "api": "MoELayer.forward per layer (eager), pinned host in/out"}

    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": world,
        "steps": K, "warmup": W, "ms_per_step": round(ms / K, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16",
        "data": "synthetic: seeded N(0,0.02) weights NF4-quantized on device; N(0,1) fp16 tokens",
        "config": config_dict(L, B, world),
        "gpu_launches": int(launches_per_step * K),
        "clocks": clk,
    }
    line["roofline"] = roof
    line["e2e"] = e2e
    if world == 1:
        line["hbm_gbs_step"] = round(routed_experts * EXPERT_BYTES / (ms / 1e3) / 1e9, 1)
        if not args.no_extra:
            line.update(measure_batches(gates, tables, dev, L, K))
            line["config0"] = measure_config0(tables, dev, K)
            if not args.no_offload:  # the resident stack (25 GB) stays; 180 GB of HBM hold both
                line["config3"] = measure_config3(dev)
    else:
        line["ep_parity"] = ep_par
        line["ep_breakdown"] = ep_split
    if not args.no_extra and not args.no_config4:
        line["config4"] = measure_config4(dev, rank, world)
    # Kernels flag timed-out waits or codebook mismatches on the device: a run
    # whose launches were invalid must not print a number.
    from moeinfra_b200 import kernels as _k
    _k.check_device(dev)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tps, times, thr = cpu_layer_sample(steps=args.cpu_steps, warmup=1, batch=B,
                                           time_budget_s=20.0)
        line["cpu_baseline"] = {"value": round(tps, 5), "unit": "tok/s", "cores": thr,
                                "kind": "port", "sample": cpu_sample_text(times, B)}
    if graph is not None:
        graph.reset()  # a graph holding NCCL calls must go before the process group
        del graph
    if world > 1 and peer is not None:
        torch.cuda.synchronize()
        _barrier(world)
        peer.close()
    return line


def ep_roofline(ep_layers, tok, dev, L: int, K: int):
    """Per-GPU roofline of the local expert stage of the expert-parallel step.

    The rows each rank's experts receive for one step's tokens are produced
    once (router, dispatch, all-to-all); then the local expert stage alone
    (``moe_experts_forward``) is replayed over the L layers in a CUDA graph.
    Algorithmic bytes = this rank's experts that received rows x 99,090,624 B
    (+ rows in/out), per layer.
    """
    from moeinfra_b200 import kernels
    calls, nbytes = [], 0
    for lay in ep_layers:
        x_sorted, local_off = lay.received_rows(tok)
        off = local_off.tolist()
        active = sum(1 for j in range(len(off) - 1) if off[j + 1] > off[j])
        rows = off[-1]
        nbytes += active * EXPERT_BYTES + 2 * rows * HIDDEN * 2
        calls.append((lay, local_off, x_sorted))
    def stage():
        for lay, off_t, xs in calls:
            kernels.experts_forward(lay._table, off_t, xs, HIDDEN, FFN)
    reps = max(3, K // 2)
    ms = _graph_time(stage, reps, dev) / L
    achieved = nbytes / L / (ms / 1e3) / 1e9
    peak = _measured_peak("hbm_gbs")
    world = torch.distributed.get_world_size()
    vals = torch.tensor([achieved, ms], dtype=torch.float64, device=dev)
    lo = vals.clone()
    torch.distributed.all_reduce(lo, op=torch.distributed.ReduceOp.MIN)
    return {"bound": "hbm", "achieved": round(float(lo[0]), 1), "peak": peak[0], "unit": "GB/s",
            "frac": round(float(lo[0]) / peak[0], 4), "traffic": None,
            "kernel": f"local expert stage per GPU (moe_experts_forward on the rows this rank's "
                      f"{EXPERTS // world} expert(s) received), per layer; min over ranks",
            "algorithmic_bytes_per_launch": int(nbytes / L), "launch_us": round(ms * 1e3, 2),
            "peak_source": peak[1]}


def ep_breakdown(ep_layers, nccl_layers, tok, dev, L: int, K: int, world: int):
    """Where an expert-parallel layer's time goes, each variant a CUDA graph of L layers.

    layer: the step as timed (peer-memory exchange unless --ep-exchange nccl);
    layer_nccl: the same layers exchanging through NCCL all-to-alls; kernels:
    the kernels with both exchanges replaced by local copies; a2a: the two
    NCCL all-to-alls per layer alone on buffers of the same shapes.  Per
    layer, max over ranks.
    """
    reps = max(3, K // 2)
    h = tok.contiguous()
    bufs = [lay.exchange_buffers(h.shape[0]) for lay in nccl_layers]
    out = {}
    for name, fn in (
            ("layer_us", lambda: [lay.forward(h) for lay in ep_layers]),
            ("layer_nccl_us", lambda: [lay.forward(h) for lay in nccl_layers]),
            ("kernels_only_us", lambda: [lay.forward(h, exchange=False) for lay in ep_layers]),
            ("a2a_only_us", lambda: [lay.exchange_only(b) for lay, b in zip(nccl_layers, bufs)])):
        _barrier(world)
        ms = _graph_time(fn, reps, dev) / L
        out[name] = round(_max_over_ranks(ms, world, dev) * 1e3, 2)
    out["note"] = ("per layer, CUDA graphs of the 32-layer step; layer uses the peer-memory "
                   "exchange (NVLink stores, flag waits), layer_nccl the NCCL all-to-alls; "
                   "kernels_only replaces both exchanges by local copies, a2a_only runs just the "
                   "two NCCL all-to-alls")
    return out


def ep_e2e(ep_layers, tokens, dev, L: int, K: int, W: int, world: int):
    """The expert-parallel step through its public call, host buffers in and out."""
    B = tokens.shape[1]
    host_in = torch.empty(K + W, B, HIDDEN, dtype=torch.float16).pin_memory()
    host_in.copy_(tokens.cpu())
    host_out = torch.empty(B, HIDDEN, dtype=torch.float16).pin_memory()
    h_dev = torch.empty(B, HIDDEN, dtype=torch.float16, device=dev)

    def step(i):
        h_dev.copy_(host_in[i], non_blocking=True)
        y = None
        for lay in ep_layers:
            y = lay.forward(h_dev)
        host_out.copy_(y, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for i in range(W):
        step(i)
    torch.cuda.synchronize()
    _barrier(world)
    a, b = _events()
    a.record()
    for i in range(W, W + K):
        step(i)
    b.record()
    torch.cuda.synchronize()
    ms = _max_over_ranks(a.elapsed_time(b), world, dev)
    return {"value": round(B * K * world / (ms / 1e3), 3), "unit": "tok/s",
            "h2d_bytes_per_step": B * HIDDEN * 2, "d2h_bytes_per_step": B * HIDDEN * 2,
            "api": "ExpertParallelMoE.forward per layer (eager; token exchange "
                   f"{'through peer memory' if ep_layers[0].peer is not None else 'by NCCL all-to-all'}"
                   "), pinned host in/out per rank; max over ranks"}


def ep_parity(ep_layer0, tok, dev, rank: int):
    """Layer 0 on every rank: the expert-parallel output vs the single-GPU layer.

    Each rank builds all eight experts of layer 0 locally and runs the fused
    single-GPU layer on the global batch (every rank's step-0 tokens, gathered
    in rank order), then compares its own rows with the expert-parallel
    output.  An expert then sees the same tokens in both (the 1-row or
    multi-row weight semantics follow its token count), so the two agree
    exactly; the check allows the layer tolerance (rel-L2 <= 2e-3, max-abs
    <= 1e-2 x max(1,|ref|)).  Worst over ranks.
    """
    from moeinfra_b200 import kernels
    world = torch.distributed.get_world_size()
    full = [resident_expert(0, e, dev) for e in range(EXPERTS)]
    table = kernels.expert_array([x.nf4_descriptor for x in full])
    parts = [torch.empty_like(tok) for _ in range(world)]
    torch.distributed.all_gather(parts, tok.contiguous())
    everyone = torch.cat(parts, 0)
    want_all, _, _ = kernels.layer_forward(everyone, ep_layer0.router.gate_f16(), table, TOP_K,
                                           HIDDEN, FFN)
    B = tok.shape[0]
    want = want_all[rank * B:(rank + 1) * B]
    got = ep_layer0.forward(tok)
    torch.cuda.synchronize()
    d = (got.float() - want.float())
    rel = float(d.norm() / max(float(want.float().norm()), 1e-30))
    mabs = float(d.abs().max())
    scale = max(1.0, float(want.float().abs().max()))
    ok = 1.0 if (rel <= 2e-3 and mabs <= 1e-2 * scale) else 0.0
    v = torch.tensor([rel, mabs, -ok], dtype=torch.float64, device=dev)
    torch.distributed.all_reduce(v, op=torch.distributed.ReduceOp.MAX)
    del full, table
    return {"max_abs": float(v[1]), "rel_l2": float(v[0]), "ok": bool(v[2] < 0),
            "check": "layer 0: expert-parallel rows of each rank vs the single-GPU fused layer "
                     "(all 8 experts local) on every rank's step-0 tokens together; worst over "
                     "ranks"}


class SyntheticMixtral:
    """A ModelLoader stand-in serving a seeded random-init Mixtral-8x7B.

    Dense weights N(0, 0.02) fp16 on the device (norm weights 1), gate as the
    decode workload's (same seeds), experts NF4-quantized on the device from
    the same per-(layer, expert) seeds and handed out as CPU experts whose
    tensors live in one pinned slab each (``pin_expert``).
    """

    def __init__(self, layers: int, device, vocab: int = 32000, pin: bool = True) -> None:
        self.layers, self.device, self.vocab, self.pin = layers, device, vocab, pin

    def load(self) -> None:
        pass

    def _randn(self, *shape, seed: int):
        g = torch.Generator(device=self.device).manual_seed(seed)
        return (torch.randn(*shape, generator=g, device=self.device) * 0.02).to(torch.float16)

    def load_layer(self, l: int):
        from moeinfra_b200.model.types import LayerWeights
        one = torch.ones(HIDDEN, dtype=torch.float16, device=self.device)
        return LayerWeights(input_layernorm=one, q_proj=self._randn(HIDDEN, HIDDEN, seed=5 * l + 1),
                            k_proj=self._randn(1024, HIDDEN, seed=5 * l + 2),
                            v_proj=self._randn(1024, HIDDEN, seed=5 * l + 3),
                            o_proj=self._randn(HIDDEN, HIDDEN, seed=5 * l + 4),
                            post_attention_layernorm=one, moe_gate=make_gate(l, self.device))

    def load_embeddings(self):
        return self._randn(self.vocab, HIDDEN, seed=777)

    def load_final_norm(self):
        return torch.ones(HIDDEN, dtype=torch.float16, device=self.device)

    def load_lm_head(self):
        return self._randn(self.vocab, HIDDEN, seed=778)

    def load_expert(self, l: int, e: int):
        from moeinfra_b200.model.expert import PrequantizedNF4Expert
        from moeinfra_b200.model.nf4_format import BLOB_KEY, pack_blob
        from moeinfra_b200.transfer.reusable_staging import pin_expert
        st = {}
        for name, (q, a, c) in make_expert_store(l, e, self.device).items():
            rows, cols = (FFN, HIDDEN) if name != "w2" else (HIDDEN, FFN)
            st[name] = {"weight": q.cpu(), "weight.absmax": a.cpu(), "weight.quant_map": c.cpu(),
                        BLOB_KEY: pack_blob({"quant_type": "nf4", "blocksize": 64,
                                             "dtype": "bfloat16", "shape": [rows, cols]})}
        ex = PrequantizedNF4Expert.from_serialized(st["w1"], st["w2"], st["w3"], HIDDEN, FFN)
        if self.pin:
            pin_expert(ex)
        return ex


def pinned_h2d_peak_gbs(dev) -> float:
    """Measured pinned host -> device copy bandwidth (1 GiB, best of 3)."""
    n = 1 << 30
    src = torch.empty(n, dtype=torch.uint8).pin_memory()
    dst = torch.empty(n, dtype=torch.uint8, device=dev)
    best = 0.0
    for _ in range(3):
        a, b = _events()
        a.record()
        dst.copy_(src, non_blocking=True)
        b.record()
        torch.cuda.synchronize()
        best = max(best, n / (a.elapsed_time(b) / 1e3) / 1e9)
    del src, dst
    return best


def measure_config3(dev):
    """Config 3: full random-init Mixtral-8x7B, 40-token prompt -> 32 greedy tokens, bs1, offload.

    ``InferenceEngine.generate`` with a 4 GiB GPU expert cache (43 Mixtral
    experts, LRU), every expert in the CPU tier in pinned memory; each miss is
    one H2D copy on the copy stream.  One warm-up generation, then one timed;
    then the same with next-layer prefetch (the layer's routed experts
    requested for the next layer on the copy stream while it computes).
    """
    from moeinfra_b200.engine.engine import InferenceEngine
    from moeinfra_b200.engine.types import ForwardRequest
    from moeinfra_b200.transfer.scheduler import EXECUTE_NEXT_PROFILE
    budget = 4 << 30
    slots = budget // EXPERT_BYTES
    loader = SyntheticMixtral(LAYERS, dev)
    t0 = time.perf_counter()
    cpu_experts = {(l, e): loader.load_expert(l, e) for l in range(LAYERS) for e in range(EXPERTS)}
    setup_s = time.perf_counter() - t0
    peak = pinned_h2d_peak_gbs(dev)

    def run(policy: str):
        cfg = {"model": {"name": None, "num_layers": LAYERS, "num_experts": EXPERTS,
                         "num_experts_per_tok": TOP_K, "hidden_size": HIDDEN,
                         "intermediate_size": FFN, "num_attention_heads": 32,
                         "num_key_value_heads": 8, "vocab_size": 32000, "rope_theta": 1e6,
                         "rms_norm_eps": 1e-5, "device": str(dev)},
               "cache": {"gpu_slots": int(slots), "cpu_slots": LAYERS * EXPERTS,
                         "eviction_policy": "lru", "gpu_budget_bytes": budget},
               "transfer": {"bandwidth_gbps": 50.0, "max_concurrent_transfers": 4,
                            "prefetch_policy": policy, "prefetch_depth": 1},
               "engine": {"max_batch": 1, "max_seq_len": 128}}
        eng = InferenceEngine(cfg, model_loader=loader)
        for (l, e), ex in cpu_experts.items():
            eng.cache_manager.put(l, e, ex, device="cpu")
        g = torch.Generator().manual_seed(3)
        eng.generate(ForwardRequest(input_ids=torch.randint(0, 32000, (1, 40), generator=g),
                                    max_new_tokens=32))  # warm-up
        n0 = len(EXECUTE_NEXT_PROFILE)
        pf0 = eng.prefetch_engine.submitted
        res = eng.generate(ForwardRequest(input_ids=torch.randint(0, 32000, (1, 40), generator=g),
                                          max_new_tokens=32))
        prof = EXECUTE_NEXT_PROFILE[n0:]
        moved = sum(p.get("bytes_transferred", 0) for p in prof)
        prefetched = eng.prefetch_engine.submitted - pf0
        h2d = moved + prefetched * EXPERT_BYTES  # prefetch copies go through submit_async
        total_s = (res.ttft_ms + res.stage_timings["decode"]) / 1e3
        eng.close()
        return res, h2d, total_s, len(prof), prefetched

    res, h2d, total_s, n_sync, _ = run("none")
    gbs = h2d / total_s / 1e9
    out = {"value": round(res.tps, 3), "unit": "tok/s (decode, bs1)",
           "ttft_ms": round(res.ttft_ms, 1), "decode_ms": round(res.stage_timings["decode"], 1),
           "experts_moved": n_sync, "h2d_bytes": int(h2d),
           "h2d_gbs": round(gbs, 2), "pinned_h2d_peak_gbs": round(peak, 2),
           "host_link_frac": round(gbs / peak, 4), "gpu_expert_slots": int(slots),
           "setup_s": round(setup_s, 1),
           "note": "InferenceEngine.generate, 32-layer random-init Mixtral-8x7B, 40 random ids -> "
                   "32 greedy tokens, 4 GiB GPU expert cache (LRU), pinned CPU tier, eager decode"}
    res_p, h2d_p, total_p, n_sync_p, n_pf = run("next_layer")
    out["prefetch_next_layer"] = {
        "value": round(res_p.tps, 3), "ttft_ms": round(res_p.ttft_ms, 1),
        "sync_copies": n_sync_p, "prefetch_copies": n_pf,
        "h2d_gbs": round(h2d_p / total_p / 1e9, 2),
        "note": "same run with PrefetchEngine NEXT_LAYER: the current layer's routed experts "
                "requested for the next layer on the copy stream (random routing predicts few)"}
    del cpu_experts
    torch.cuda.empty_cache()
    return out


def measure_config4(dev, rank: int, world: int):
    """Config 4: the 32-layer Mixtral-8x7B, experts resident and sharded over the GPUs.

    64 sequences x 512 random-id prompt tokens, then 128 greedy tokens; rank r
    serves sequences [r*64/G, (r+1)*64/G) and owns experts [r*8/G, (r+1)*8/G)
    of every layer (one expert per GPU per layer at G = 8).  Prefill exchanges
    tokens with NCCL all-to-alls, decode steps through peer memory inside a
    CUDA graph of the whole step.  One GPU: the same model with every expert
    resident and the fused single-GPU layers.  Times are max over ranks.
    """
    from moeinfra_b200.engine.engine import InferenceEngine
    from moeinfra_b200.engine.types import ForwardRequest
    B, S, N = 64, 512, 128
    Bl = B // world
    cfg = {"model": {"name": None, "num_layers": LAYERS, "num_experts": EXPERTS,
                     "num_experts_per_tok": TOP_K, "hidden_size": HIDDEN, "intermediate_size": FFN,
                     "num_attention_heads": 32, "num_key_value_heads": 8, "vocab_size": 32000,
                     "rope_theta": 1e6, "rms_norm_eps": 1e-5, "device": str(dev)},
           "cache": {"gpu_slots": LAYERS * EXPERTS, "cpu_slots": LAYERS * EXPERTS},
           "transfer": {"bandwidth_gbps": 50.0, "staging_slots": 2},
           "engine": {"max_batch": Bl, "max_seq_len": S + N, "preload_experts": world == 1},
           "parallel": {"expert_parallel": world > 1}}
    loader = SyntheticMixtral(LAYERS, dev, pin=False)
    eng = InferenceEngine(cfg, model_loader=loader)
    g = torch.Generator().manual_seed(4)
    ids = torch.randint(0, 32000, (B, S), generator=g)[rank * Bl:(rank + 1) * Bl]
    eng._initialize_runtime()
    torch.cuda.synchronize()
    _barrier(world)
    res = eng.generate(ForwardRequest(input_ids=ids, max_new_tokens=N))
    prefill = _max_over_ranks(res.ttft_ms, world, dev)
    decode = _max_over_ranks(res.stage_timings["decode"], world, dev)
    graphed = res.stage_timings["cuda_graph_decode"]
    eng.close()
    del eng
    torch.cuda.empty_cache()
    return {"value": round(B * (N - 1) / (decode / 1e3), 1), "unit": "tok/s (decode, bs64 global)",
            "prefill_ms": round(prefill, 1), "prefill_tok_s": round(B * S / (prefill / 1e3), 1),
            "decode_ms": round(decode, 1), "cuda_graph_decode": bool(graphed),
            "sequences_per_gpu": Bl, "note": "InferenceEngine.generate, 32-layer random-init "
            "Mixtral-8x7B, 64 x 512 random ids -> 128 greedy tokens; max over ranks"}


def measure_config0(tables, dev, K: int):
    """Config 0: one Mixtral expert, 16 tokens (``moe_expert_forward``).

    Eight different experts (layer 0's) are cycled so that no expert is
    reused while it could still sit in L2 (99 MB each, 126 MB L2).
    """
    from moeinfra_b200 import _native, kernels
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(16, HIDDEN, generator=g, device=dev).to(torch.float16)
    descs = [tables[0][e] for e in range(EXPERTS)]
    ys = [torch.empty_like(x) for _ in descs]
    lib = _native.lib()
    ws_bytes = lib.moe_expert_workspace_size(16, HIDDEN, FFN)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    import ctypes

    def run():
        s = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        for d, y in zip(descs, ys):
            _native.check(lib.moe_expert_forward(ctypes.byref(d), ctypes.c_void_p(x.data_ptr()),
                                                 16, HIDDEN, FFN, ctypes.c_void_p(y.data_ptr()),
                                                 ctypes.c_void_p(ws.data_ptr()), ws_bytes, s),
                          "moe_expert_forward")
    ms = _graph_time(run, max(3, K // 2), dev) / len(descs)
    nbytes = EXPERT_BYTES + 2 * 16 * HIDDEN * 2
    peak = _measured_peak("hbm_gbs")
    gbs = nbytes / (ms / 1e3) / 1e9
    return {"value": round(gbs, 1), "unit": "GB/s", "us_per_expert": round(ms * 1e3, 2),
            "tokens": 16, "algorithmic_bytes": nbytes,
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak[0],
                         "unit": "GB/s", "frac": round(gbs / peak[0], 4),
                         "peak_source": peak[1]},
            "note": "single SwiGLU expert (hidden 4096, ffn 14336) on 16 fp16 tokens"}


def _graph_time(fn, reps: int, dev) -> float:
    """Mean ms of one replay of a CUDA graph of ``fn`` (captured after a warm-up call)."""
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    a, b = _events()
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / reps
    del g
    return ms


def measure_batches(gates, tables, dev, L: int, K: int):
    """bs64 decode over the stack and config-2 prefill (4096 tokens per layer).

    bs64: one step = 64 tokens through the L layers (CUDA graph), as the bs1 step.
    prefill: 4096 N(0,1) tokens (seed 2) through one layer with an N(0,0.05) gate
    (uneven expert loads), layers cycled; the expert stage (grouped tcgen05
    GEMM) is also timed alone for its tensor-pipe roofline.
    """
    from moeinfra_b200 import kernels
    out = {}
    # --- bs64 decode ---
    B = 64
    toks = make_tokens(2, B, dev, rank=17)
    h64 = toks[0].contiguous()
    ms = _graph_time(lambda: [kernels.layer_forward(h64, gates[l], tables[l], TOP_K, HIDDEN, FFN)
                              for l in range(L)], K, dev)
    touched = 0
    for l in range(L):
        _, _, idx = kernels.router_topk(h64, gates[l], TOP_K, with_logits=False)
        touched += len(set(idx.reshape(-1).tolist()))
    out["bs64"] = {"value": round(B / (ms / 1e3), 2), "unit": "tok/s", "ms_per_step": round(ms, 4),
                   "hbm_gbs": round(touched * EXPERT_BYTES / (ms / 1e3) / 1e9, 1),
                   "experts_touched_per_step": touched,
                   "note": "64 tokens through the stack per step (grouped tcgen05 GEMM path)"}
    # --- prefill, config 2 ---
    T = 4096
    g = torch.Generator(device=dev).manual_seed(2)
    xp = torch.randn(T, HIDDEN, generator=g, device=dev).to(torch.float16)
    gates_pf = [(torch.randn(EXPERTS, HIDDEN, generator=g, device=dev) * 0.05).to(torch.float16)
                for _ in range(min(L, 4))]
    nl = len(gates_pf)

    def prefill():
        for l in range(nl):
            kernels.layer_forward(xp, gates_pf[l], tables[l], TOP_K, HIDDEN, FFN)
    reps = max(2, K // 4)
    ms_pf = _graph_time(prefill, reps, dev) / nl
    pairs = T * TOP_K
    flops = pairs * 2 * 3 * HIDDEN * FFN
    # expert stage alone (two grouped GEMM launches per layer)
    stage_args = []
    for l in range(nl):
        _, w, idx = kernels.router_topk(xp, gates_pf[l], TOP_K, with_logits=False)
        offsets, pair_token, _, _ = kernels.permute(idx, w, EXPERTS)
        stage_args.append((offsets, kernels.gather_rows(xp, pair_token)))
    ms_st = _graph_time(lambda: [kernels.experts_forward(tables[l], stage_args[l][0],
                                                         stage_args[l][1], HIDDEN, FFN)
                                 for l in range(nl)], reps, dev) / nl
    peak = _measured_peak("bf16_tflops")
    tflops = flops / (ms_st / 1e3) / 1e12
    loads = torch.bincount(idx.reshape(-1), minlength=EXPERTS).tolist()
    out["prefill"] = {"value": round(T / (ms_pf / 1e3), 1), "unit": "tok/s per layer",
                      "ms_per_layer": round(ms_pf, 4), "tokens": T,
                      "expert_loads_last_layer": loads,
                      "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": peak[0],
                                   "unit": "TFLOP/s", "frac": round(tflops / peak[0], 4),
                                   "traffic": _profile_value(PROFILE_PREFILL,
                                                             "traffic_per_layer_bytes"),
                                   "kernel": "grouped NF4 GEMM (gate_up + down launches), per layer",
                                   "algorithmic_flop_per_launch": flops,
                                   "launch_us": round(ms_st * 1e3, 1), "peak_source": peak[1]}}
    return out


def _measured_peak(key: str):
    p = ROOT / "MEASURED_PEAKS.json"
    fallback = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
    try:
        v = json.loads(p.read_text())[key]
        return float(v), "measured (MEASURED_PEAKS.json)"
    except Exception:
        return fallback[key], "fallback"


def run_reference(args, world: int):
    """The reference's CPU path (its restatement) on the host cores, for this arm's workload.

    One step = the job's ``batch x world`` tokens through one MoE layer (a
    bounded sample of the 32-layer step; ``ms_per_step`` is that measured
    time), value = tokens / (32 x mean layer-step time).
    """
    B = args.batch * world
    tps, times, thr = cpu_layer_sample(steps=args.steps, warmup=args.warmup, batch=B,
                                       time_budget_s=None)
    sample = cpu_sample_text(times, B)
    return {
        "metric": METRIC, "value": round(tps, 5), "unit": "tok/s", "n_gpus": world,
        "steps": len(times), "warmup": args.warmup,
        "ms_per_step": round(sum(times) / len(times) * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp16",
        "data": "synthetic: seeded N(0,0.02) weights NF4-quantized on host; N(0,1) fp16 tokens",
        "config": config_dict(args.layers, args.batch, world),
        "impl": "reference",
        "cpu_baseline": {"value": round(tps, 5), "unit": "tok/s", "cores": thr, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(tps, 5), "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--cpu-steps", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the bs64, prefill, config-0 and config-3 measurements")
    ap.add_argument("--ep-exchange", choices=("p2p", "nccl"), default="p2p",
                    help="expert-parallel token exchange: stores into peer memory, or NCCL")
    ap.add_argument("--no-config4", action="store_true",
                    help="skip the config-4 (full model, expert-parallel, bs64) measurement")
    ap.add_argument("--no-offload", action="store_true",
                    help="skip the config-3 (full model, CPU-offloaded experts) measurement")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    # stdout carries only the JSON line: libraries that print banners (NCCL's
    # version line on rank 0) write to file descriptor 1, so it goes to stderr
    # for the whole run and the result is written to the saved descriptor.
    sys.stdout.flush()
    json_fd = os.dup(1)
    os.dup2(2, 1)

    def emit(line: dict) -> None:
        os.write(json_fd, (json.dumps(line) + "\n").encode())

    if args.impl == "reference":
        # Under torchrun rank 0 alone runs the CPU sample; the other ranks exit.
        if rank == 0:
            emit(run_reference(args, world))
        return 0

    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=300),
                                             device_id=torch.device("cuda", local_rank))
    try:
        line = run_device(args, rank, world, local_rank)
        if rank == 0:
            emit(line)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
