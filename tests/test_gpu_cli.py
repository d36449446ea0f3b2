"""The command-line checks (the reference engine's cuda-info / cuda-check / cuda-check-moe /
cuda-bench) run through the loader on a GPU and pass."""
import subprocess

import pytest

from katali_lab_b200.build import CHECK

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cmd", ["info", "check", "check-moe", "bench"])
def test_check_cli(cmd):
    r = subprocess.run([CHECK, cmd], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.strip()
