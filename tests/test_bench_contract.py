"""The one-JSON-line output of bench.py: the reference arm on the CPU, the
B200 arm on a GPU (a few steps, without the optional quantizer, kernel,
stack and CPU sections)."""

import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run_bench(*args, timeout=600):
    proc = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), *args], cwd=REPO,
                          capture_output=True, text=True, timeout=timeout)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [ln for ln in proc.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1, proc.stdout[-2000:]
    return json.loads(lines[0])


def _common(line, steps, warmup):
    assert line["metric"].startswith("audio-sec/sec")
    assert line["unit"] == "audio-sec/sec"
    assert line["value"] > 0 and line["ms_per_step"] > 0
    assert (line["steps"], line["warmup"], line["n_gpus"]) == (steps, warmup, 1)
    assert line["higher_is_better"] is True
    assert line["scaling"] == "weak"
    assert line["vs_baseline"] is None
    assert line["dtype"] == "bf16"
    assert "synthetic" in line["data"]
    assert "workload" in line["config"]
    e2e = line["e2e"]
    assert e2e["unit"] == line["unit"] and e2e["value"] > 0
    assert {"h2d_bytes_per_step", "d2h_bytes_per_step"} <= set(e2e)


def test_reference_arm_line():
    line = _run_bench("--impl", "reference", "--steps", "1", "--warmup", "0")
    _common(line, 1, 0)
    assert line["impl"] == "reference"
    cpu = line["cpu_baseline"]
    assert cpu["kind"] in ("port", "reference") and cpu["cores"] >= 1 and cpu["sample"]
    assert cpu["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0


@pytest.mark.gpu
def test_b200_arm_line(cuda_device):
    line = _run_bench("--steps", "2", "--warmup", "3", "--no-cpu", "--no-stack", "--no-kernels",
                      "--no-quantizer")
    _common(line, 2, 3)
    assert "impl" not in line
    roof = line["roofline"]
    assert roof["bound"] in ("hbm", "tensor")
    assert roof["unit"] in ("GB/s", "TFLOP/s")
    assert roof["achieved"] > 0 and roof["peak"] > 0
    assert roof["frac"] == pytest.approx(roof["achieved"] / roof["peak"])
    assert "traffic" in roof
    # 125 chunks per step, 97 library kernels per chunk (1 + 24 layers x 4:
    # the attention with the rotary inside, two residual + LayerNorm passes,
    # the gated activation)
    assert line["gpu_launches"] == 2 * 125 * 97
    assert line["roofline"]["step"]["frac"] > 0
    assert {"sm_mhz", "sm_max_mhz", "reasons"} <= set(line["clocks"])
    assert line["outputs_verified"] is True
    assert line["e2e"]["h2d_bytes_per_step"] > 0 and line["e2e"]["d2h_bytes_per_step"] > 0
