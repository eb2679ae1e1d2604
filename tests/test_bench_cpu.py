"""bench.py's reference arm on the CPU: one JSON line with the contract's keys, the reference's own decide_many as the
CPU path when the reference package is installed next to the repository (baseline/_ref), the port otherwise."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_config1_prints_one_line():
    env = dict(os.environ, OMP_NUM_THREADS="4")
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--config", "1", "--steps", "1",
                          "--warmup", "1"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["value"] > 0 and line["higher_is_better"] is True
    assert line["e2e"]["value"] == line["value"] and line["e2e"]["h2d_bytes_per_step"] == 0
    installed = os.path.isdir(os.path.join(ROOT, "baseline", "_ref", "opendecider"))
    assert line["cpu_baseline"]["kind"] == ("reference" if installed else "port")
    if installed:
        assert line["port_cross_check"]["value"] > 0 and "decide_many" in line["cpu_baseline"]["sample"]


def test_reference_request_schema():
    """Synthetic questions map onto the reference's request schema (choice options, noul without options, score
    levels), which its pydantic DecideRequest validates."""
    sys.path.insert(0, ROOT)
    import bench
    from opendecider_b200 import synthetic as syn
    reqs, _ = syn.decision_requests(4, seed=0, n_requests=1)
    qs = {q.type: bench.RefCpuSample._question(q) for q in reqs[0].questions}
    assert set(qs) == {"choice", "noul", "score"}
    assert "options" not in qs["noul"] and qs["score"]["levels"] and qs["choice"]["options"]
