"""GPU parity of the kernels behind the C ABI against the oracle.

Dequantisation: bit-exact.  Matvec: the reference sums fp32 products in its
own order and this build computes each 32-block dot exactly on fixed-point
inputs (22-bit per block), so outputs differ by rounding only; the test
bound is |y - y_ref| <= 2e-5 * sum_j |w_j x_j| + 1e-6 per row (the
magnitude of the terms, i.e. a relative error of 2e-5 of the dot product's
absolute mass).
"""
import ctypes

import numpy as np
import pytest

import pyoracle
from fwb import configs, gguf_synth, native
from fwb.model import quant_matvec

pytestmark = pytest.mark.gpu

TYPES = [configs.Q4_0, configs.Q5_0, configs.Q8_0]
BB = {configs.Q4_0: 18, configs.Q5_0: 22, configs.Q8_0: 34}


@pytest.fixture(scope="module")
def lib(built):
    lib = native.product()
    if lib.fwb_device_count() < 1:
        pytest.skip("no CUDA device")
    return lib


def _abs_mass(w, t, x, rows):
    deq = pyoracle.dequant(w, t, rows * x.size).reshape(rows, x.size).astype(np.float64)
    return np.abs(deq) @ np.abs(x.astype(np.float64))


def check_matvec(y, y_ref, mass):
    err = np.abs(y.astype(np.float64) - y_ref.astype(np.float64))
    bound = 2e-5 * mass + 1e-6
    bad = np.nonzero(err > bound)[0]
    assert bad.size == 0, f"{bad.size} rows out of tolerance, worst ratio {np.max(err / bound):.3g}"


@pytest.mark.parametrize("t", TYPES)
def test_dequant_bit_exact_gguf_py_blocks(lib, t):
    import os
    import torch
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "quant_gguf_py.npz"))
    name = {configs.Q4_0: "q4_0", configs.Q5_0: "q5_0", configs.Q8_0: "q8_0"}[t]
    raw = g[name + "_bytes"]
    n = raw.size // BB[t] * 32
    dw = torch.from_numpy(raw.copy()).cuda()
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    assert lib.quant_dequant_dev(dw.data_ptr(), raw.size, t, out.data_ptr(), n,
                                 torch.cuda.current_stream().cuda_stream) == 0
    got = out.cpu().numpy()
    want = pyoracle.dequant(raw, t, n)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert np.array_equal(got.view(np.uint32), g[name + "_deq"].view(np.uint32))


@pytest.mark.parametrize("t", TYPES)
def test_dequant_bit_exact_random(lib, t):
    import torch
    rows, cols = 257, 1024
    raw = gguf_synth.random_matrix(t, rows, cols, seed=17, mode=1)
    n = rows * cols
    dw = torch.from_numpy(raw).cuda()
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    assert lib.quant_dequant_dev(dw.data_ptr(), raw.size, t, out.data_ptr(), n, None) == 0
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), pyoracle.dequant(raw, t, n).view(np.uint32))


SHAPES = [(1, 32), (3, 64), (7, 288), (37, 512), (149, 768), (300, 4096), (4096, 4096),
          (1024, 4096), (4096, 14336), (129, 8192), (33, 28672)]


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_quant_matvec_host_vs_oracle(lib, t, rows, cols):
    w = gguf_synth.random_matrix(t, rows, cols, seed=rows * 31 + cols, mode=1)
    x = gguf_synth.normal_vector(cols, seed=cols)
    y = quant_matvec(w, t, x, rows)
    y_ref = pyoracle.quant_matvec(w, t, x, rows)
    check_matvec(y, y_ref, _abs_mass(w, t, x, rows))


@pytest.mark.parametrize("t", TYPES)
def test_quant_matvec_dev_normal_weights(lib, t):
    """N(0, 0.02)-quantised weights (the model distribution), device API."""
    import torch
    rows, cols = 14336, 4096
    w = gguf_synth.random_matrix(t, rows, cols, seed=3, mode=0, lo=0.0, hi=0.02)
    x = gguf_synth.normal_vector(cols, seed=4)
    dw, dx = torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()
    dy = torch.empty(rows, dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert lib.quant_matvec_dev(dw.data_ptr(), w.size, t, dx.data_ptr(), dy.data_ptr(), cols, rows, st) == 0
    torch.cuda.synchronize()
    y_ref = pyoracle.quant_matvec(w, t, x, rows)
    check_matvec(dy.cpu().numpy(), y_ref, _abs_mass(w, t, x, rows))


def test_quant_matvec_dev_unaligned_weight_pointer(lib):
    """Weights starting 2 bytes into an allocation (2-byte aligned only)."""
    import torch
    t, rows, cols = configs.Q4_0, 100, 4096
    w = gguf_synth.random_matrix(t, rows, cols, seed=8, mode=1)
    buf = torch.zeros(w.size + 64, dtype=torch.uint8, device="cuda")
    buf[2:2 + w.size] = torch.from_numpy(w).cuda()
    x = gguf_synth.normal_vector(cols, seed=9)
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty(rows, dtype=torch.float32, device="cuda")
    # the exact row bytes do not reach the 16-byte boundary after the rows: refused
    assert lib.quant_matvec_dev(buf.data_ptr() + 2, w.size, t, dx.data_ptr(), dy.data_ptr(), cols, rows,
                                None) == -1
    assert b"16-byte boundary" in lib.fwb_last_error()
    assert lib.quant_matvec_dev(buf.data_ptr() + 2, w.size + 14, t, dx.data_ptr(), dy.data_ptr(), cols, rows,
                                None) == 0
    assert lib.quant_device_status(None) == 0
    torch.cuda.synchronize()
    check_matvec(dy.cpu().numpy(), pyoracle.quant_matvec(w, t, x, rows), _abs_mass(w, t, x, rows))


def test_quant_matvec_odd_pointer_rejected(lib):
    import torch
    buf = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    x = torch.zeros(32, device="cuda")
    y = torch.zeros(1, device="cuda")
    assert lib.quant_matvec_dev(buf.data_ptr() + 1, 18, configs.Q4_0, x.data_ptr(), y.data_ptr(), 32, 1,
                                None) == -1


def test_quant_matvec_kat_64(lib):
    """test_runner.c:161-178 through the GPU: 1x32, d = 1, q = 2, x = 1 -> 64."""
    blk = np.zeros(34, np.uint8)
    blk[1] = 0x3C
    blk[2:] = 2
    y = quant_matvec(blk, configs.Q8_0, np.ones(32, np.float32), 1)
    assert y[0] == 64.0


def test_quant_matvec_zero_and_nonfinite_inputs(lib):
    t, rows, cols = configs.Q8_0, 5, 256
    w = gguf_synth.random_matrix(t, rows, cols, seed=1, mode=1)
    x = np.zeros(cols, np.float32)
    assert np.all(quant_matvec(w, t, x, rows) == 0)
    x[3] = np.inf
    y = quant_matvec(w, t, x, rows)
    assert not np.any(np.isfinite(y))
