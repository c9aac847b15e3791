"""CPU tests of the oracle: the restatement (oracle/fwd_oracle.c) against
the reference's own known-answer tests, against gguf-py's GGML decoders, and
against the compiled reference (live when oracle/_ref exists, and through the
committed golden fixtures everywhere)."""
import os
import subprocess

import numpy as np
import pytest

import pyoracle
from fwb import configs, gguf_synth

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def orc(built):
    return pyoracle.oracle_lib()


def _f(a):
    return a.ctypes.data_as(pyoracle._fp)


# --- known-answer tests restated from the reference's test_runner.c ----------

def test_kat_q8_0_decode(orc):
    # test_runner.c:110-126: d = 1.0 (0x3C00), q = i - 16 -> i - 16
    blk = np.zeros(34, np.uint8)
    blk[0], blk[1] = 0x00, 0x3C
    blk[2:] = (np.arange(32) - 16).astype(np.int8).view(np.uint8)
    out = pyoracle.dequant(blk, configs.Q8_0, 32)
    assert np.array_equal(out, np.arange(32, dtype=np.float32) - 16)


def test_kat_q8_0_matvec(orc):
    # test_runner.c:161-178: 1x32, d = 1, q = 2, x = 1 -> 64
    blk = np.zeros(34, np.uint8)
    blk[1] = 0x3C
    blk[2:] = 2
    y = pyoracle.quant_matvec(blk, configs.Q8_0, np.ones(32, np.float32), 1)
    assert abs(y[0] - 64.0) < 1e-4


def test_kat_rms_norm_unit_rms(orc):
    # test_runner.c:30-41
    x = np.array([1, 2, 3, 4], np.float32)
    w = np.ones(4, np.float32)
    out = np.zeros(4, np.float32)
    orc.orc_rms_norm(_f(x), _f(w), _f(out), 4, 1e-5)
    assert abs(float(np.mean(out.astype(np.float64) ** 2)) - 1.0) < 1e-4


def test_kat_rope_pos0_identity(orc):
    # test_runner.c:60-90
    hd, ctx = 64, 16
    c = np.zeros(ctx * hd // 2, np.float32)
    s = np.zeros_like(c)
    orc.orc_rope_tables(_f(c), _f(s), ctx, hd, 10000.0)
    assert np.all(np.abs(c[: hd // 2] - 1) < 1e-6) and np.all(np.abs(s[: hd // 2]) < 1e-6)
    qk = np.arange(1, 65, dtype=np.float32)
    q0 = qk.copy()
    orc.orc_rope_apply(_f(qk), 0, 1, hd, _f(c), _f(s))
    assert np.all(np.abs(qk - q0) < 1e-5)


def test_kat_argmax(orc):
    # test_runner.c:93-96, plus the lowest-index-wins tie rule of sampler.c:28-32
    x = np.array([1, 2, 3, 4, 5], np.float32)
    assert orc.orc_argmax(_f(x), 5) == 4
    y = np.array([0, 3, 1, 3], np.float32)
    assert orc.orc_argmax(_f(y), 4) == 1


def test_kat_fp16_subnormal(orc):
    # quant.c:22-55: subnormal-correct fp16 conversion
    for h in (0x0001, 0x03FF, 0x8001, 0x3C00, 0x7BFF, 0xFBFF, 0x0000, 0x8000):
        want = np.array([h], np.uint16).view(np.float16).astype(np.float32)[0]
        assert orc.orc_f16_to_f32(h) == want


# --- gguf-py golden vectors (pins Q4_0, which the reference lacks) -----------

@pytest.mark.parametrize("name,t", [("q4_0", configs.Q4_0), ("q5_0", configs.Q5_0), ("q8_0", configs.Q8_0)])
def test_dequant_matches_gguf_py(orc, name, t):
    g = np.load(os.path.join(GOLDEN, "quant_gguf_py.npz"))
    raw, deq = g[name + "_bytes"], g[name + "_deq"]
    out = pyoracle.dequant(raw, t, deq.size)
    # bit-exact: both are one fp32 product d * q per value
    assert np.array_equal(out.view(np.uint32), deq.view(np.uint32))


# --- the compiled reference itself ---------------------------------------------

@pytest.mark.skipif(not os.path.exists(pyoracle.REF_UNIT_TEST), reason="oracle/_ref not built here")
def test_reference_unit_tests_pass():
    r = subprocess.run([pyoracle.REF_UNIT_TEST], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and "ALL TESTS PASSED" in r.stdout


@pytest.mark.parametrize("tag", ["tied_q8_0", "mixed", "q4_0"])
@pytest.mark.parametrize("variant", ["plain", "kvprefill"])
def test_oracle_matches_reference_golden(built, model_dir, tag, variant):
    """The restatement reproduces the compiled reference's logits on the
    golden models (recorded by tests/golden/make_golden.py)."""
    import make_golden as mg
    g = np.load(os.path.join(GOLDEN, f"ref_decode_{tag}_{variant}.npz"))
    cfg, seed = mg.GOLDEN_MODELS[tag]
    path = gguf_synth.write_model(os.path.join(model_dir, f"golden_{tag}.gguf"), cfg, seed=seed)
    assert mg.sha256(path) == str(g["sha256"]), "synthetic model bytes changed"
    m = pyoracle.OracleModel(path)
    pos0 = int(g["pos0"])
    if variant == "kvprefill":
        for layer in range(cfg.n_layer):
            k, v = mg.prefill_kv(cfg, layer, pos0, seed)
            m.kv_load(layer, 0, k, v)
    tok = int(g["first"])
    for i, (ref_tok, ref_lg) in enumerate(zip(g["tokens"], g["logits"])):
        lg = m.forward(tok, pos0 + i)
        assert np.array_equal(lg, ref_lg), f"step {i}: max diff {np.abs(lg - ref_lg).max()}"
        tok = int(ref_tok)


@pytest.mark.skipif(not pyoracle.ref_available(), reason="oracle/_ref not built here")
@pytest.mark.parametrize("t", [configs.Q4_0, configs.Q5_0, configs.Q8_0])
def test_oracle_matvec_matches_reference(built, t):
    rows, cols = 37, 512
    w = gguf_synth.random_matrix(t, rows, cols, seed=5, mode=1)
    x = gguf_synth.normal_vector(cols, seed=6)
    a = pyoracle.quant_matvec(w, t, x, rows)
    b = pyoracle.quant_matvec(w, t, x, rows, use_ref=True)
    assert np.array_equal(a, b)


@pytest.mark.skipif(not pyoracle.ref_available(), reason="oracle/_ref not built here")
def test_reference_config_matches_reader(built, model_dir):
    """model_config_load's view of a synthetic file (the reference's own
    parser) agrees with the shape the file was written with."""
    import ctypes
    cfg = configs.SMALL_MIXED
    path = gguf_synth.write_model(os.path.join(model_dir, "cfgcheck.gguf"), cfg, seed=3)
    u = (ctypes.c_uint32 * 10)()
    f = (ctypes.c_float * 3)()
    assert pyoracle.ref_lib().refh_config(path.encode(), u, f) == 0
    assert list(u)[1:9] == [cfg.n_vocab, cfg.n_ctx, cfg.n_embd, cfg.n_layer, cfg.n_head,
                            cfg.n_head_kv, cfg.n_ff, cfg.head_dim]
    assert abs(f[0] - cfg.eps) < 1e-12 and f[1] == np.float32(cfg.rope_base)
