"""The bench's JSON contract on the host (no GPU): the reference arm's line
carries the keys and the config dict the GPU arm prints, and the single-op
timing sizes its input copies to exceed twice the L2."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

BASE_KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
             "scaling", "vs_baseline", "dtype", "data", "config", "e2e", "cpu_baseline", "impl"}


def _reference_line(workload, steps=3):
    env = dict(os.environ, OMP_NUM_THREADS="1")  # the arm must use every host core regardless
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", workload,
                          "--steps", str(steps), "--warmup", "3"], capture_output=True, text=True, env=env,
                         cwd=ROOT, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout
    return json.loads(lines[0])


@pytest.mark.parametrize("workload", ["q8gemm", "w8a8"])
def test_reference_arm_line(workload):
    import bench
    from oracle import oracle as orc
    line = _reference_line(workload)
    assert BASE_KEYS <= set(line), BASE_KEYS - set(line)
    assert line["impl"] == "reference"
    assert line["config"] == bench.config_dict(workload, 1)  # the GPU arm prints the same dict
    assert line["value"] > 0 and line["higher_is_better"] is True
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["cpu_baseline"]["kind"] == "port"
    assert line["cpu_baseline"]["cores"] == orc.host_cores()


def test_input_copies_exceed_twice_l2():
    import bench

    class Fake:
        def __init__(self, weight_bytes):
            self.weight_bytes = weight_bytes

    for fp in (1e6, 11.7e6, 60e6, 123e6, 2e9):
        wl = Fake(fp)
        c = bench.input_copies(wl)
        assert 1 <= c <= 32
        assert c == 32 or c * bench.footprint_bytes(wl) >= 2 * bench.L2_BYTES
        assert c == 1 or (c - 1) * bench.footprint_bytes(wl) < 2 * bench.L2_BYTES
