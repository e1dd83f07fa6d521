"""bench.py's reference arm on CPU: the JSON line the driver reads.

``bench.py --impl reference`` times the CPU restatement of the linear block
(oracle/, OpenMP on every host core) on a bounded sample and prints one line
with the same metric, unit and config keys as the GPU arm; under torchrun
only rank 0 runs it and the other ranks exit 0 without output.  No GPU is
touched on this path.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _bench(*args, env=None, timeout=600):
    e = dict(os.environ)
    e.update(env or {})
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, env=e,
                          capture_output=True, text=True, timeout=timeout)


def _lines(out: str) -> list[dict]:
    return [json.loads(ln) for ln in out.splitlines() if ln.startswith("{")]


def test_reference_arm_prints_one_contract_line():
    r = _bench("--impl", "reference", "--steps", "1", "--warmup", "0")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _lines(r.stdout)
    assert len(lines) == 1, r.stdout
    d = lines[0]
    assert d["impl"] == "reference"
    assert d["metric"].startswith("encrypted linear-block ciphertexts/s")
    assert d["unit"] == "ciphertexts/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and abs(d["ms_per_step"] - 1000.0 / d["value"]) < 1e-9 * d["ms_per_step"]
    cpu = d["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["cores"] >= 1 and cpu["value"] == d["value"]
    assert "oracle" in cpu["sample"].lower()
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    r = _bench("--impl", "reference", "--steps", "1", "--warmup", "0",
               env={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert not _lines(r.stdout)


def test_reference_arm_uses_every_core_under_torchrun():
    """torchrun exports OMP_NUM_THREADS=1; the arm times the oracle with every
    host core all the same."""

    r = _bench("--impl", "reference", "--steps", "1", "--warmup", "0",
               env={"OMP_NUM_THREADS": "1", "RANK": "0", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert _lines(r.stdout)[0]["cpu_baseline"]["cores"] == (os.cpu_count() or 1)


def test_unrestated_workload_reports_unavailable():
    r = _bench("--impl", "reference", "--workload", "mlp", "--steps", "1", "--warmup", "0")
    assert r.returncode == 0, r.stderr[-2000:]
    d = _lines(r.stdout)[-1]
    assert d["impl"] == "reference" and "unavailable" in d
