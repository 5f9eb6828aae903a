"""Host-side parts of bench.py that need no GPU: the config-5 memory plan and the reference arm's lines for the
workloads that are not run on the CPU."""

import json
import math
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402
from forgeserve_b200 import ModelConfig  # noqa: E402
from forgeserve_b200.weights import model_shapes  # noqa: E402


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_c5_stage_bytes_cover_the_whole_model(world):
    cfg = ModelConfig(**bench.C5_CFG)
    m = 4
    act = bench.C5["rows"] * bench.C5["seq"] * (3 * cfg.ffn_dim + 2 * cfg.d_model) * 2
    kv = cfg.n_layers * 2 * bench.C5["rows"] * m * 2 * cfg.max_seq_len * cfg.n_kv_heads * cfg.head_dim * 2
    weights = sum(2 * math.prod(shape) for shape in model_shapes(cfg).values())
    total = sum(bench.c5_stage_bytes(cfg, world, r, m) for r in range(world))
    assert total == weights + kv + world * act
    assert weights / 1e9 == pytest.approx(141.1, abs=0.2)          # 70.6 B parameters in bf16, untied head


@pytest.mark.parametrize("workload", ["c4", "c5"])
def test_reference_arm_reports_unavailable_workloads(workload):
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", workload],
                         capture_output=True, text=True, timeout=120, cwd=ROOT)
    assert out.returncode == 0, out.stderr
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and "unavailable" in line


def test_reference_arm_runs_config_2_on_the_host_cores():
    """The reference arm on the 1B-shape prefill: the oracle on one of its 16 layers and the head."""
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", "c2",
                          "--steps", "1", "--warmup", "0"], capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert out.returncode == 0, out.stderr
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and "1B-shape" in line["metric"] and line["value"] > 0
    assert line["config"]["seq_len"] == 1024 and line["config"]["microbatches"] == 8
    assert "1 of 16 layers" in line["cpu_baseline"]["sample"]


def test_reference_arm_step_time_is_the_measured_sample():
    """--impl reference: ms_per_step is the time one step of the sample actually took (so steps x ms_per_step fits
    inside the run's wall time); the whole-model extrapolation behind `value` has its own field."""
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", "c2",
                          "--steps", "2", "--warmup", "1"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert res.returncode == 0, res.stderr
    line = json.loads(res.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["cpu_baseline"]["kind"] == "port"
    assert line["ms_per_step"] * (line["steps"] + line["warmup"]) <= line["wall_s"] * 1e3
    assert line["extrapolated_ms_per_row"] > line["ms_per_step"]
    assert math.isclose(line["value"], 1024 / (line["extrapolated_ms_per_row"] / 1e3), rel_tol=1e-3)


def test_sequence_pieces_default_to_the_stage_counts_where_they_pay():
    assert [bench.auto_seq_chunks("c3", n) for n in (1, 2, 4, 8)] == [1, 1, 4, 4]
    assert [bench.auto_seq_chunks("c2", n) for n in (1, 2, 4, 8)] == [1, 1, 2, 2]
    assert bench.auto_seq_chunks("c4", 8) == 1 and bench.auto_seq_chunks("c5", 8) == 1
    from forgeserve_b200.pipeline import seq_pieces
    for w in ("c3", "c2"):          # every default piece keeps >= 2048 GEMM rows
        spec = bench.PREFILL[w]
        for lo, hi in seq_pieces(spec["seq"], bench.auto_seq_chunks(w, 8), spec["rows"]):
            assert spec["rows"] * (hi - lo) >= 2048
