"""quant_matvec_static (include/forword_b200.h): quant_matvec staged through
the library's fixed device array instead of per-call allocations.

Kept in its own file, collected after every other test module, so that it is
exercised both alone and after the rest of the suite has used the device.
It compares against quant_matvec, the existing entry point, on two calls in
a row with different inputs (so state left over from the first call would
show), for each quant type; the results must be bit-identical (same kernel,
same launch plan).
"""
import ctypes

import numpy as np
import pytest

from fwb import configs, gguf_synth, native
from fwb.model import quant_matvec

pytestmark = pytest.mark.gpu
_fp = ctypes.POINTER(ctypes.c_float)


@pytest.fixture(scope="module")
def lib(built):
    lib = native.product()
    if lib.fwb_device_count() < 1:
        pytest.skip("no CUDA device")
    fn = lib.quant_matvec_static
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint32, _fp, _fp,
                   ctypes.c_size_t, ctypes.c_size_t]
    return lib


def _static(lib, w, t, x, n_out):
    y = np.full(n_out, np.nan, dtype=np.float32)
    rc = lib.quant_matvec_static(w.ctypes.data, w.nbytes, t, x.ctypes.data_as(_fp),
                                 y.ctypes.data_as(_fp), x.size, n_out)
    return rc, y


@pytest.mark.parametrize("t,rows,cols", [(configs.Q4_0, 4096, 4096), (configs.Q5_0, 1000, 4096),
                                         (configs.Q8_0, 4096, 4096), (configs.Q8_0, 77, 288)])
def test_two_calls_match_quant_matvec(lib, t, rows, cols):
    for call in range(2):
        seed = 1000 * call + rows
        w = gguf_synth.random_matrix(t, rows, cols, seed=seed, mode=1)
        x = gguf_synth.normal_vector(cols, seed=seed + 1)
        want = quant_matvec(w, t, x, rows)
        rc, got = _static(lib, w, t, x, rows)
        assert rc == 0, lib.fwb_last_error().decode()
        assert np.array_equal(got, want), f"call {call}: max diff {np.abs(got - want).max()}"


def test_rejects_calls_beyond_the_static_scratch(lib):
    rows, cols = 14336, 4096  # Q8_0: 62.4 MB of rows > 32 MiB
    w = np.zeros(rows * cols // 32 * 34, dtype=np.uint8)
    x = np.zeros(cols, dtype=np.float32)
    rc, _ = _static(lib, w, configs.Q8_0, x, rows)
    assert rc == -1
    msg = lib.fwb_last_error().decode()
    assert "static scratch" in msg and "33554432" in msg


def test_rejects_bad_arguments_like_quant_matvec(lib):
    w = np.zeros(18 * 4, dtype=np.uint8)
    x = np.zeros(32, dtype=np.float32)
    assert _static(lib, w, 3, x, 4)[0] == -1          # unsupported type
    assert _static(lib, w, configs.Q4_0, x[:16], 4)[0] == -1  # input not a multiple of 32
    assert _static(lib, w[:40], configs.Q4_0, x, 4)[0] == -1  # weights too small
