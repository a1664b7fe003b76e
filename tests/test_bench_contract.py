"""CPU check of the JSON line ``bench.py --impl reference`` prints (the
reference's attention path timed on the host: its own module when the
package is installed under baseline/_ref, else the oracle's restatement):
the keys and units the benchmark driver reads. Run in-process on a tiny
workload."""
import argparse
import contextlib
import io
import json

import pytest
import torch

import bench


@pytest.fixture(autouse=True)
def _keep_torch_threads():
    """The reference arm sets torch's thread count; later tests keep theirs."""
    n = torch.get_num_threads()
    yield
    torch.set_num_threads(n)


def test_reference_arm_json_contract(monkeypatch):
    monkeypatch.setenv("RANK", "0")
    monkeypatch.setenv("WORLD_SIZE", "1")
    args = argparse.Namespace(gpus=1, steps=1, warmup=0)
    out = io.StringIO()
    with contextlib.redirect_stdout(out):
        assert bench.run_reference_arm(args, [64, 96]) == 0
    line = json.loads(out.getvalue().strip().splitlines()[-1])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC
    assert line["unit"] == "TFLOP/s" and line["value"] > 0 and line["higher_is_better"] is True
    assert line["cpu_baseline"]["kind"] in ("reference", "port") and line["cpu_baseline"]["cores"] >= 1
    # ms_per_step is the measured time of the step that ran (one sampled layer),
    # and it fits the run: steps x ms_per_step is the timed CPU work
    assert 0 < line["ms_per_step"] < line["extrapolated_full_step_ms"]
    assert line["e2e"] == {"value": line["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert "workload" in line["config"]


def test_reference_arm_other_ranks_exit_quietly(monkeypatch):
    monkeypatch.setenv("RANK", "1")
    monkeypatch.setenv("WORLD_SIZE", "2")
    out = io.StringIO()
    with contextlib.redirect_stdout(out):
        assert bench.run_reference_arm(argparse.Namespace(gpus=2, steps=1, warmup=0), [64]) == 0
    assert out.getvalue() == ""


def test_cpu_baselines_json(monkeypatch):
    """``bench.py --cpu-baselines`` on shrunken workloads: one JSON line with
    config 1 and, for each sparse config, the dense / compute-cache / reuse
    per-layer times of the reference module (or an ``unavailable`` line when
    the reference package is not installed)."""
    monkeypatch.setenv("RANK", "0")
    tiny = {"c3": (2, 4, 4, 2, (64, 64), 32, 0.5, "tiny c3"),
            "c4": (2, 4, 2, 2, (40, 72), 32, 0.5, "tiny c4"),
            "c5": (2, 4, 4, 1, (96, 96), 32, 0.25, "tiny c5")}
    monkeypatch.setattr(bench, "SPARSE_WORKLOADS", tiny)
    out = io.StringIO()
    with contextlib.redirect_stdout(out):
        assert bench.run_cpu_baselines(argparse.Namespace(cpu_budget=0.05)) == 0
    line = json.loads(out.getvalue().strip().splitlines()[-1])
    assert line["impl"] == "reference"
    if "unavailable" in line:
        return
    assert line["cores"] >= 1 and line["c1"]["tflops"] > 0
    for wl in ("c3", "c4", "c5"):
        r = line[wl]
        for key in ("dense_ms_per_layer", "state1_ms_per_layer", "state2_ms_per_layer"):
            assert r[key] > 0, (wl, key)
        assert set(r["extrapolated_full_step_ms"]) >= {"dense", "state1", "state2"}
        assert all(n >= 1 for n in r["n_keep"])
