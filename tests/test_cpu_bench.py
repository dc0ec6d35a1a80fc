"""The benchmark's reference arm runs on the host cores alone; its JSON line
must keep the contract the round-end driver parses (one line, the metric and
unit of the GPU arm, impl "reference", a cpu_baseline and an e2e object)."""

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("workload", ["mlvc_dec_1080p_8s", "block_stack", "entropy_1080p"])
def test_reference_arm_prints_one_contract_line(workload):
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", workload,
                          "--steps", "2", "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "frames/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 2 and d["warmup"] == 3
    assert d["cpu_baseline"]["kind"] in ("reference", "port") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_bench_rejects_short_warmup():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--warmup", "2"], capture_output=True, text=True,
                         timeout=120, cwd=ROOT)
    assert out.returncode != 0 and "--warmup must be >= 3" in out.stderr


def test_default_workload_is_the_metric_configuration():
    """The default workload is BASELINE config 5 (1080p, 8 independent
    streams), and both arms report it under the same metric and scaling."""
    sys.path.insert(0, str(ROOT))
    import bench
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    d = json.loads([l for l in out.stdout.splitlines() if l.startswith("{")][0])
    assert d["metric"] == bench.STREAMS_METRIC and d["scaling"] == "strong"
    assert d["config"]["workload"] == bench.STREAMS_DESC and d["config"]["global_batch"] == bench.STREAMS == 8


def test_reference_arm_other_ranks_exit_quietly():
    """Under torchrun with N > 1 only rank 0 runs the reference arm."""
    import os
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "3"], capture_output=True, text=True, timeout=300, cwd=ROOT, env=env)
    assert out.returncode == 0 and not [l for l in out.stdout.splitlines() if l.startswith("{")]


def test_ranks_get_disjoint_host_cores():
    """Under torchrun each rank keeps its own share of the host cores (no
    migration or contention between the ranks' host threads)."""
    import ast
    import os
    cores = sorted(os.sched_getaffinity(0))
    if len(cores) < 2:
        pytest.skip("one host core")
    got = []
    for rank in (0, 1):
        code = f"import sys; sys.path.insert(0, {str(ROOT)!r}); import bench; print(bench.pin_host_cores({rank}, 2))"
        out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120, cwd=ROOT)
        assert out.returncode == 0, out.stderr[-2000:]
        got.append(set(ast.literal_eval(out.stdout.strip().splitlines()[-1])))
    assert got[0] and got[1] and not (got[0] & got[1]) and (got[0] | got[1]) <= set(cores)
