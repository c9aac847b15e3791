"""GPU tests of the tensor-core dequant-GEMM (quant_gemm_dev, the prompt
path's batched linear layer) against a plain float64 (numpy) reference.

The kernel rounds the dequantised weights ((q - 8) * d, bit-exact with the
reference decoders) and the activations to fp16 and accumulates in fp32.
Two references: (1) the same fp16-rounded operands multiplied in float64 --
the only difference is fp32 summation order, bound 4e-5 of each output's
absolute mass (sum_k |w_k x_k|); (2) the exact fp32 weights -- the fp16
rounding of the weights adds at most 2^-11 relative per product, bound
1e-3 of the absolute mass.
"""
import numpy as np
import pytest

import pyoracle
from fwb import configs, gguf_synth, native

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib(built):
    lib = native.product()
    if lib.fwb_device_count() < 1:
        pytest.skip("no CUDA device")
    return lib


def _run(lib, w, x16, rows, cols, accumulate=False, y0=None):
    import torch
    m = x16.shape[0]
    dw = torch.from_numpy(w).cuda()
    dx = torch.from_numpy(x16.view(np.uint16).copy()).cuda()
    dy = torch.from_numpy(y0.copy()).cuda() if y0 is not None else torch.full((m, rows), float("nan"), device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.quant_gemm_dev(dw.data_ptr(), w.size, configs.Q4_0, dx.data_ptr(), dy.data_ptr(), cols, rows, m,
                            int(accumulate), st)
    assert rc == 0, lib.fwb_last_error().decode()
    torch.cuda.synchronize()
    return dy.cpu().numpy()


@pytest.mark.parametrize("m,rows,cols", [(1, 128, 64), (128, 128, 128), (77, 384, 4096), (300, 200, 512),
                                         (512, 1024, 4096)])
def test_quant_gemm_q4_0_matches_fp32_reference(lib, m, rows, cols):
    w = gguf_synth.random_matrix(configs.Q4_0, rows, cols, seed=11 + m, mode=0, lo=0.0, hi=0.02)
    rng = np.random.default_rng(m * 7 + cols)
    x16 = rng.standard_normal((m, cols)).astype(np.float16)
    y = _run(lib, w, x16, rows, cols)
    deq = pyoracle.dequant(w, configs.Q4_0, rows * cols).reshape(rows, cols)
    x = x16.astype(np.float64)
    mass = np.abs(x) @ np.abs(deq.astype(np.float64)).T
    ref16 = x @ deq.astype(np.float16).astype(np.float64).T
    ref32 = x @ deq.astype(np.float64).T
    assert np.isfinite(y).all()
    assert (np.abs(y - ref16) <= 4e-5 * mass + 1e-6).all(), np.max(np.abs(y - ref16) / (mass + 1e-6))
    assert (np.abs(y - ref32) <= 1e-3 * mass + 1e-6).all(), np.max(np.abs(y - ref32) / (mass + 1e-6))


def test_quant_gemm_accumulate_adds_into_output(lib):
    m, rows, cols = 130, 256, 256
    w = gguf_synth.random_matrix(configs.Q4_0, rows, cols, seed=5, mode=0, lo=0.0, hi=0.02)
    x16 = np.random.default_rng(1).standard_normal((m, cols)).astype(np.float16)
    y0 = np.random.default_rng(2).standard_normal((m, rows)).astype(np.float32)
    y = _run(lib, w, x16, rows, cols)
    y_acc = _run(lib, w, x16, rows, cols, accumulate=True, y0=y0)
    assert np.array_equal(y_acc, (y0 + y).astype(np.float32))


def test_quant_gemm_rejects_unsupported(lib):
    import torch
    buf = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    out = torch.zeros(1 << 14, dtype=torch.float32, device="cuda")
    # Q8_0 is not on the tensor-core path; K not a multiple of 64
    assert lib.quant_gemm_dev(buf.data_ptr(), buf.numel(), configs.Q8_0, buf.data_ptr(), out.data_ptr(), 64, 8, 1, 0,
                              None) == -1
    assert lib.quant_gemm_dev(buf.data_ptr(), buf.numel(), configs.Q4_0, buf.data_ptr(), out.data_ptr(), 32, 8, 1, 0,
                              None) == -1
