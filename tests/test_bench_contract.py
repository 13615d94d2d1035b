"""bench.py's JSON contract on the CPU: the reference arm (`--impl reference`,
the oracle port timed on the host cores) prints one line with the keys the
driver reads, and ranks other than 0 of a multi-GPU launch exit 0 silently.

The reference arm builds the benchmark geometry's embedding table on the host
(248320 x 2560 F32), so this test takes about a minute.
"""
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _run(args, env=None, timeout=900):
    e = dict(os.environ)
    e.update(env or {})
    return subprocess.run([sys.executable, str(ROOT / "bench.py")] + args, cwd=ROOT, env=e,
                          capture_output=True, text=True, timeout=timeout)


def test_reference_arm_prints_the_contract_line():
    r = _run(["--impl", "reference", "--steps", "1", "--warmup", "3", "--layers", "2",
              "--cpu-sample-tokens", "16"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == "prefill tok/s" and d["unit"] == "tok/s"
    assert d["value"] > 0 and d["ms_per_step"] > 0 and d["higher_is_better"] is True
    assert d["steps"] == 1 and d["warmup"] == 3 and d["n_gpus"] == 1 and d["scaling"] == "strong"
    assert "workload" in d["config"] and d["vs_baseline"] is None
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert d["finite"] is True
    # The reference arm runs the oracle alone: the product library is never
    # mapped into its process.
    assert d["native_libraries"] == ["oracle/liboracle.so"], d["native_libraries"]


def test_reference_arm_other_ranks_exit_silently():
    r = _run(["--impl", "reference", "--gpus", "2"], env={"RANK": "1", "WORLD_SIZE": "2"}, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [l for l in r.stdout.splitlines() if l.startswith("{")]
