"""The measurement tools of the package (CPU): each module imports and its
command line parses (`--help`), so the commands quoted in the profile
summaries stay runnable."""
import os
import subprocess
import sys

import pytest

PKG = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "forword.c_b200")


@pytest.mark.parametrize("mod", ["fwb.gemm_bench", "fwb.matvec_bench", "fwb.phase_trace"])
def test_tool_command_line_parses(mod):
    env = dict(os.environ, PYTHONPATH=PKG + os.pathsep + os.environ.get("PYTHONPATH", ""))
    r = subprocess.run([sys.executable, "-m", mod, "--help"], capture_output=True, text=True, env=env, timeout=120)
    assert r.returncode == 0, r.stderr
    assert "usage" in r.stdout
