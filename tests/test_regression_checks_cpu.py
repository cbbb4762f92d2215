"""The data-parallel VL regression checks (image rank + text-only rank lockstep; joint SFT +
decision steps train the projector) on two gloo ranks with a small random VL model."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("check", ["mixed", "decision"])
def test_regression_check_passes_on_two_ranks(check):
    port = 29700 + (os.getpid() + (check == "decision")) % 200
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", str(port), "-m", "trida_stack_b200.parallel.regression_checks", check, "--tiny", "--cpu",
           "--steps", "3"]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600,
                       env=dict(os.environ, OMP_NUM_THREADS="1"))
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert f"{check} check: PASS" in r.stdout
    assert r.stdout.count("ranks agree True") == 6
