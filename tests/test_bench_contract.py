"""bench.py's reference arm (``--impl reference``): the JSON line the driver reads.

The arm times the reference's own CPU attention (src/cpu.cpp compiled into
oracle/_ref/, or the C restatement of it when that is not built) on a bounded
sample of the workload, so it runs on a machine without a GPU.  Under torchrun
only rank 0 works and prints; the other ranks exit 0 without output.
"""

import json
import os
import subprocess
import sys

from tests.conftest import ROOT


def _bench(args, env_extra=None):
    env = dict(os.environ)
    env.pop("RANK", None)
    env.pop("WORLD_SIZE", None)
    env.pop("LOCAL_RANK", None)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=600)


def _json_lines(stdout):
    return [json.loads(line) for line in stdout.splitlines() if line.startswith("{")]


def test_reference_arm_prints_one_contract_line():
    r = _bench(["--impl", "reference", "--steps", "1", "--warmup", "0"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _json_lines(r.stdout)
    assert len(lines) == 1
    d = lines[0]
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "dtype", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["unit"] == "TFLOP/s" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["config"]["workload"].startswith("SigLIP-shaped")
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    cpu = d["cpu_baseline"]
    assert cpu["kind"] in ("reference", "port") and cpu["cores"] >= 1 and cpu["value"] == d["value"]
    assert cpu["sample"]


def test_reference_arm_other_ranks_exit_without_output():
    for config in ("c2", "c5"):
        r = _bench(["--impl", "reference", "--config", config, "--gpus", "2", "--steps", "1", "--warmup", "0"],
                   {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
        assert r.returncode == 0, r.stderr[-2000:]
        assert _json_lines(r.stdout) == []
