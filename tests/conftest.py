"""Shared test setup.

Markers: `gpu` — needs a CUDA device (run with -m gpu on a B200).
CPU tests (-m "not gpu") cover the oracle against golden vectors and the
compiled reference, the host logic, and that the C-ABI library loads and
exports its declared symbols.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "forword.c_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a CUDA GPU (B200)")


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    d = os.environ.get("FWB_MODEL_DIR")
    if d:
        os.makedirs(d, exist_ok=True)
        return d
    return str(tmp_path_factory.mktemp("models"))


@pytest.fixture(scope="session")
def built():
    """Build the product library, the synth helper and the oracle (no-op when
    already built; the GPU box receives them prebuilt)."""
    import subprocess
    from fwb import native
    if not (os.path.exists(native.PRODUCT_SO) and os.path.exists(native.SYNTH_SO)):
        subprocess.run(["make", "-C", native.PKG_DIR, "-j8"], check=True, capture_output=True)
    import pyoracle
    if not os.path.exists(pyoracle.ORACLE_SO):
        pyoracle.build()
    return True


@pytest.fixture(scope="session")
def gpu_available():
    try:
        from fwb import native
        return native.product().fwb_device_count() > 0
    except Exception:
        return False
