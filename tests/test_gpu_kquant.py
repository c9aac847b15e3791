"""GPU checks of the Q5_1 / Q4_K / Q6_K paths against the compiled
reference (its own decoders and quant_matvec, quant.c / quant_matvec.c):

* dequantisation bit-exact (quant_dequant_dev vs q5_1/q4_k/q6_k_decode);
* quant_matvec within 2e-5 of each row's absolute mass of the reference's;
* decode of models with these types -- a Q4_K_M-style mix (Q4_K attention,
  gate, up and embedding, Q6_K v, down and head: the v rows then run as a
  GEMV of their own) and an all-Q5_1 model -- against the reference's
  transformer_forward, teacher-forced, greedy tokens identical.
"""
import os

import numpy as np
import pytest

import pyoracle
from fwb import configs, gguf_synth, native
from fwb.model import Model, quant_matvec
from parity import assert_logits_close

pytestmark = pytest.mark.gpu
KTYPES = [configs.Q5_1, configs.Q4_K, configs.Q6_K]


@pytest.fixture(scope="module")
def lib(built):
    lib = native.product()
    if lib.fwb_device_count() < 1:
        pytest.skip("no CUDA device")
    if not pyoracle.ref_available():
        pytest.skip("compiled reference not built")
    return lib


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("t", KTYPES)
def test_dequant_bit_exact_against_reference_decoders(lib, t, mode):
    import torch
    rows, cols = 64, 1024
    w = gguf_synth.random_matrix(t, rows, cols, seed=11 + mode, mode=mode, lo=0.0 if mode == 0 else 1e-3,
                                 hi=0.02 if mode == 0 else 1e-2)
    n = rows * cols
    dw = torch.from_numpy(w).cuda()
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    assert lib.quant_dequant_dev(dw.data_ptr(), w.size, t, out.data_ptr(), n, None) == 0
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    want = pyoracle.ref_dequant(w, t, n)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("rows,cols", [(256, 4096), (1000, 1024), (4096, 14336)])
@pytest.mark.parametrize("t", KTYPES)
def test_quant_matvec_against_reference(lib, t, rows, cols):
    w = gguf_synth.random_matrix(t, rows, cols, seed=rows + t, mode=1)
    x = gguf_synth.normal_vector(cols, seed=cols + t)
    y = quant_matvec(w, t, x, rows)
    y_ref = pyoracle.quant_matvec(w, t, x, rows, use_ref=True)
    deq = pyoracle.ref_dequant(w, t, rows * cols).reshape(rows, cols).astype(np.float64)
    mass = np.abs(deq) @ np.abs(x.astype(np.float64))
    err = np.abs(y.astype(np.float64) - y_ref.astype(np.float64))
    bound = 2e-5 * mass + 1e-6
    assert (err <= bound).all(), f"worst ratio {np.max(err / bound):.3g}"


@pytest.mark.parametrize("cfg,seed", [(configs.SMALL_KQUANT, 71), (configs.SMALL_Q5_1, 72)])
def test_decode_against_reference(lib, model_dir, cfg, seed):
    path = gguf_synth.write_model(os.path.join(model_dir, f"{cfg.name}-{seed}.gguf"), cfg, seed=seed)
    ref = pyoracle.RefModel(path, 0)
    tok = 5
    with Model(path) as m:
        for pos in range(16):
            want = ref.forward(tok, pos)
            got = m.forward(tok, pos)
            assert_logits_close(got, want, f"{cfg.name} step {pos}")
            assert int(np.argmax(got)) == int(np.argmax(want)), f"greedy token differs at step {pos}"
            tok = int(np.argmax(want))
    ref.close()
