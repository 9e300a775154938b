"""bench.py's output contract, checked on the CPU: the reference arm's JSON
line (the driver runs it on every box), the warm-up floor, and the profile
figures the default arm reads for its roofline objects."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _bench(*args: str, timeout: int = 600) -> subprocess.CompletedProcess:
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT,
                          capture_output=True, text=True, timeout=timeout)


def test_reference_arm_prints_one_contract_line():
    r = _bench("--impl", "reference", "--steps", "1", "--warmup", "3")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["value"] > 0 and d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_warmup_floor_is_enforced():
    r = _bench("--warmup", "2", timeout=120)
    assert r.returncode != 0
    assert "warmup" in r.stderr


def test_profile_figures_for_the_roofline_objects():
    sys.path.insert(0, str(ROOT))
    import bench

    decode = bench._profile_traffic()
    prefill = bench._profile_value(bench.PROFILE_PREFILL, "traffic_per_layer_bytes")
    # DRAM bytes per launch (decode expert stage) and per layer (prefill GEMMs):
    # at least the algorithmic bytes the kernels must read.
    assert decode is not None and decode >= 198_214_016
    assert prefill is not None and prefill >= 8 * 99_090_624
