"""bench.py's reference arm (--impl reference) on CPU: the reference path's CPU restatement on
the configs[1] workload, one JSON line with the contract's keys; under torchrun, ranks other than
0 print nothing and exit 0."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    # a small sample (4 blocks from a 4-block host pool): these tests check the line's contract
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "2",
                          "--warmup", "1", "--blocks", "4", "--cpu-pool", "4"], capture_output=True, text=True,
                         env=env, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    return [l for l in out.stdout.splitlines() if l.startswith("{")]


def test_reference_arm_line():
    lines = _run({"RANK": "0"})
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["value"] > 0 and d["unit"] == "GB/s"
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]


def test_reference_arm_other_ranks_silent():
    assert _run({"RANK": "1"}) == []


def test_serving_ttft_is_measured_in_the_closed_loop_steady_state():
    """A timed request's TTFT runs from the same client's previous first token, `clients` rounds
    earlier, warm-up rounds included; a warm-up shorter than one client cycle is refused."""
    sys.path.insert(0, ROOT)
    import bench

    done = [float(t) for t in range(10)]  # one request per round, first token at t = round
    assert bench.closed_loop_ttft(done, warm=4, clients=3) == [3.0] * 6
    done = done[:7] + [8.5, 9.5, 10.5]  # round 7 takes 2.5: the requests finishing after it wait longer
    assert bench.closed_loop_ttft(done, warm=4, clients=3) == [3.0, 3.0, 3.0, 4.5, 4.5, 4.5]
    with pytest.raises(ValueError):
        bench.closed_loop_ttft(done, warm=2, clients=3)
