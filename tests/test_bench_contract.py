"""bench.py's output contract, checked on CPU.

* The reference arm (`--impl reference`, rank 0: the reference's own
  pure-PyTorch code from baseline/_ref, or the numpy restatement) prints one
  JSON line with the keys the driver reads, on a tiny token sample so the
  test takes seconds.
* The algorithmic-bytes model is the reference's (scripts/benchmark_kernels.py:
  64-105): 6,609,174,528 bytes for the six kernels at T=65536, C=1024, plus
  this build's grad_W write in K1's backward.
"""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("kind", ["reference", "port"])
def test_reference_arm_prints_the_contract_line(kind):
    if kind == "reference" and not (ROOT / "baseline" / "_ref" / "flash_mhc").is_dir():
        pytest.skip("the reference is not installed in baseline/_ref")
    r = subprocess.run(
        [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
         "--warmup", "1", "--ref-kind", kind, "--ref-tokens", "256", "--no-configs0",
         "--cpu-tokens-per-worker", "16"],
        capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["cpu_baseline"]["kind"] == kind
    # the same workload description as the GPU arm
    sys.path.insert(0, str(ROOT))
    import bench

    assert line["config"] == bench.workload_config(65536, 1024, 1)
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
              "higher_is_better", "config", "cpu_baseline", "e2e"):
        assert k in line, k
    assert line["value"] > 0 and line["unit"] == "tokens/s" and line["higher_is_better"] is True
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["kind"] in ("port", "reference") and cb["cores"] >= 1
    assert cb["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_bytes_model_is_the_reference_model():
    sys.path.insert(0, str(ROOT))
    import bench

    bm = bench.bytes_model(65536, 1024)
    grad_w_write = 32 * 4096 * 2
    assert sum(bm.values()) - grad_w_write == 6_609_174_528
    assert bm["k4_bwd"] == 1_889_533_952
