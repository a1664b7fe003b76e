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
