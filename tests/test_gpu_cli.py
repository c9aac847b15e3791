"""Drop-in check: forword.c's own CLI (main.c and its host C, unchanged)
linked with forword.c_b200/shim/transformer_b200.c against the CUDA library
produces the same greedy output as the reference CLI built from its own
sources.

Both executables are built on the build machine (`make -C forword.c_b200 cli`
and `make -C oracle ref`, which need forword.c's sources) and travel prebuilt;
the test skips when either is absent.
"""
import os
import subprocess

import pytest

import pyoracle
from fwb import configs, gguf_synth, native

pytestmark = pytest.mark.gpu
B200_CLI = os.path.join(native.PKG_DIR, "_build", "forword-b200")


@pytest.fixture(scope="module")
def clis(built):
    if native.product().fwb_device_count() < 1:
        pytest.skip("no CUDA device")
    missing = [p for p in (B200_CLI, pyoracle.REF_CLI) if not os.path.exists(p)]
    if missing:
        pytest.skip(f"CLI not built: {missing}")
    return B200_CLI, pyoracle.REF_CLI


def _run(exe, args):
    r = subprocess.run([exe] + args, capture_output=True, text=True, timeout=600)
    return r.returncode, r.stdout, r.stderr


@pytest.mark.parametrize("cfg,seed", [(configs.SMALL_MIXED, 21), (configs.TINY, 22)])
def test_cli_greedy_output_identical(clis, model_dir, cfg, seed):
    path = gguf_synth.write_model(os.path.join(model_dir, f"cli-{cfg.name}-{seed}.gguf"), cfg, seed=seed)
    args = [path, "--temp", "0", "--rep-pen", "1", "--no-template", "--max-tokens", "24",
            "--ctx", "128", "t1 t2 t3 t17 t99"]
    rc_b, out_b, err_b = _run(clis[0], args)
    rc_r, out_r, err_r = _run(clis[1], args)
    assert rc_r == 0, err_r
    assert rc_b == 0, err_b
    assert "Generated" in out_r + err_r
    assert out_b == out_r


def test_cli_reports_bad_model_like_reference(clis, tmp_path):
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"not a gguf file at all")
    rc_b, _, err_b = _run(clis[0], [str(bad), "--max-tokens", "1", "x"])
    rc_r, _, err_r = _run(clis[1], [str(bad), "--max-tokens", "1", "x"])
    assert rc_b == rc_r != 0
    assert err_b.splitlines()[0] == err_r.splitlines()[0]
