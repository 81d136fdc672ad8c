"""bench.py's JSON contract, checked on the CPU: the reference arm
(``--impl reference``, the reference's compiled kernels on the host) prints
one JSON line with every key the driver reads, and the library arm refuses
to run without a GPU instead of falling back to the CPU."""
import json
import os
import subprocess
import sys

import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args, timeout=600):
    return subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), *args], cwd=REPO,
                          capture_output=True, text=True, timeout=timeout)


def test_reference_arm_prints_the_contract_line():
    res = _run("--impl", "reference", "--workload", "cfg2", "--steps", "1", "--warmup", "1")
    assert res.returncode == 0, res.stderr[-2000:]
    line = json.loads(res.stdout.strip().splitlines()[-1])
    if "unavailable" in line:
        pytest.skip(f"reference arm unavailable here: {line['unavailable']}")
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config", "e2e",
                "cpu_baseline"):
        assert key in line, key
    assert line["impl"] == "reference"
    # at least 3 timed steps after 1 warm-up, printed as they ran
    assert line["value"] > 0 and line["n_gpus"] == 1 and line["steps"] == 3
    assert line["warmup"] == 1 and line["config"]["global_batch"] == 256
    assert "workload" in line["config"]
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == line["value"] and cb["steps"] == line["steps"]


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU behaviour")
def test_library_arm_fails_loudly_without_a_gpu():
    res = _run("--steps", "1", "--warmup", "1", "--no-cpu-baseline", timeout=300)
    assert res.returncode != 0
    assert res.stdout.strip() == "" or "value" not in res.stdout
