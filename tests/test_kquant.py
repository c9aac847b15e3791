"""CPU checks of the K-quant and Q5_1 support: the synthetic writer's blocks
(fwb/synth.c) are valid GGML blocks -- the compiled reference's decoders
(quant.c) and gguf-py 0.19.0 (llama.cpp's own Python decoders) read the same
values from them -- and the reference's quant_matvec runs on them."""
import numpy as np
import pytest

import pyoracle
from fwb import configs, gguf_synth

KTYPES = [configs.Q5_1, configs.Q4_K, configs.Q6_K]


@pytest.fixture(scope="module")
def ref(built):
    if not pyoracle.ref_available():
        pytest.skip("compiled reference not built")
    return True


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("t", KTYPES)
def test_reference_and_gguf_py_decode_the_same_values(ref, t, mode):
    import gguf
    rows, cols = 8, 512
    lo, hi = (0.0, 0.02) if mode == 0 else (1e-3, 1e-2)
    w = gguf_synth.random_matrix(t, rows, cols, seed=5, mode=mode, lo=lo, hi=hi)
    ours = pyoracle.ref_dequant(w, t, rows * cols)
    theirs = gguf.quants.dequantize(w.reshape(1, -1), gguf.GGMLQuantizationType(t)).reshape(-1).astype(np.float32)
    assert np.isfinite(ours).all()
    assert np.allclose(ours, theirs, rtol=1e-6, atol=1e-7), np.abs(ours - theirs).max()


@pytest.mark.parametrize("t", KTYPES)
def test_quantisers_follow_the_weights(ref, t):
    """mode 0 (model weights): the decoded values track the N(0, 0.02) values
    they were quantised from (a loose check that the encoder is sane)."""
    rows, cols = 4, 1024
    w = gguf_synth.random_matrix(t, rows, cols, seed=9, mode=0, lo=0.0, hi=0.02)
    deq = pyoracle.ref_dequant(w, t, rows * cols)
    assert 0.01 < float(np.std(deq)) < 0.03
    assert abs(float(np.mean(deq))) < 0.005


@pytest.mark.parametrize("t", KTYPES)
def test_reference_quant_matvec_runs(ref, t):
    rows, cols = 16, 512
    w = gguf_synth.random_matrix(t, rows, cols, seed=3, mode=1)
    x = gguf_synth.normal_vector(cols, seed=4)
    y = pyoracle.quant_matvec(w, t, x, rows, use_ref=True)
    deq = pyoracle.ref_dequant(w, t, rows * cols).reshape(rows, cols).astype(np.float64)
    assert np.allclose(y, deq @ x.astype(np.float64), rtol=1e-4, atol=1e-4)
