"""bench.py's reference arm on the CPU (the oracle port timed on a bounded
sample of config 4): one JSON line with the contract's keys, the same metric,
unit, direction and config as the engine arm, and the algorithmic work counts
the roofline is quoted on."""

import importlib.util
import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def load_bench():
    spec = importlib.util.spec_from_file_location("bench_mod", ROOT / "bench.py")
    b = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(b)
    return b


def test_work_counts():
    b = load_bench()
    # four DiT GEMMs of one layer: 2*M*D*(4D + D + 2F) + 2*M*F*D FLOP = 114.3 MFLOP per row
    assert b.row_forward_flops(1, 0, L=1) == pytest.approx(114_294_784 + 4 * 2048 * 32, rel=1e-9)
    # bf16 operands / weights once, bf16 outputs once, f32 residual read + written by Wo and W2
    assert b.gemm_layer_bytes(54504) == 4_746_698_752
    assert b.GEMM_LAYER_TRAFFIC_PER_ROW * 54504 == pytest.approx(5.751e9, rel=1e-3)


def test_reference_arm_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "0"],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    b = load_bench()
    b.load_pkg()
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "scaling", "vs_baseline",
              "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference"
    assert d["metric"] == b.METRIC and d["unit"] == b.UNIT and d["higher_is_better"] is True
    utts = b.workload()
    assert d["config"] == b.config4_dict(sum(u[3] for u in utts), 1)
    assert d["value"] > 0 and d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["kind"] == "port"
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    # a finite step time consistent with the value (one step = the whole job's audio)
    audio = sum(u[3] for u in utts)
    assert d["ms_per_step"] > 0 and d["ms_per_step"] == pytest.approx(audio / d["value"] * 1000.0, rel=1e-3)
    assert d["cpu_baseline"].get("cpu_model") is not None
