"""End-to-end decode parity of the CUDA path (fwb_forward & co., through the
C ABI) against the compiled reference's golden logits and the oracle.

Per step: logits max-abs <= 1e-2 and relative L2 <= 1e-3 (parity.py);
greedy tokens identical (teacher-forced on the reference's stream, with the
reference's top-1/top-2 gap reported on any mismatch).
"""
import dataclasses
import os

import numpy as np
import pytest

import make_golden as mg
import pyoracle
from fwb import configs, gguf_synth, native
from fwb.model import Model
from parity import assert_logits_close, greedy_compare

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def gpu(built):
    if native.product().fwb_device_count() < 1:
        pytest.skip("no CUDA device")
    return True


def _model_path(model_dir, cfg, seed, tag=None):
    return gguf_synth.write_model(os.path.join(model_dir, f"{tag or cfg.name}-{seed}.gguf"), cfg, seed=seed)


@pytest.mark.parametrize("tag", ["tied_q8_0", "mixed", "q4_0"])
@pytest.mark.parametrize("variant", ["plain", "kvprefill"])
def test_decode_matches_reference_golden(gpu, model_dir, tag, variant):
    g = np.load(os.path.join(GOLDEN, f"ref_decode_{tag}_{variant}.npz"))
    cfg, seed = mg.GOLDEN_MODELS[tag]
    path = _model_path(model_dir, cfg, seed, f"golden_{tag}")
    assert mg.sha256(path) == str(g["sha256"])
    pos0 = int(g["pos0"])
    with Model(path) as m:
        if variant == "kvprefill":
            for layer in range(cfg.n_layer):
                k, v = mg.prefill_kv(cfg, layer, pos0, seed)
                m.kv_load(layer, 0, k, v)
        tok = int(g["first"])
        for i, (ref_tok, ref_lg) in enumerate(zip(g["tokens"], g["logits"])):
            lg = m.forward(tok, pos0 + i)
            assert_logits_close(lg, ref_lg, f"step {i}")
            assert int(np.argmax(lg)) == int(ref_tok), f"greedy token differs at step {i}"
            tok = int(ref_tok)


def test_tiny_config_prompt_and_128_greedy_tokens(gpu, model_dir):
    """Benchmark config 1: tiny llama, Q8_0, tied embeddings, ctx 256;
    16-token uniform-random prompt, then 128 greedy tokens."""
    cfg = configs.TINY
    path = _model_path(model_dir, cfg, 101)
    rng = np.random.default_rng(7)
    prompt = [int(t) for t in rng.integers(0, cfg.n_vocab, 16)]
    orc = pyoracle.OracleModel(path)
    with Model(path) as m:
        for p, t in enumerate(prompt[:-1]):
            assert_logits_close(m.forward(t, p), orc.forward(t, p), f"prompt {p}")
        mism, wa, wr, gap = greedy_compare(m.forward, orc.forward, prompt[-1], len(prompt) - 1, 129)
    assert not mism, f"greedy mismatches (step, gpu, ref, ref top-2 gap): {mism}"
    assert wa <= 1e-2 and wr <= 1e-3
    print(f"tiny: worst max-abs {wa:.3g} rel {wr:.3g}; min ref top-2 gap {gap:.3g}")


def test_generate_greedy_equals_stepwise(gpu, model_dir):
    cfg = configs.SMALL_Q4_0
    path = _model_path(model_dir, cfg, 202)
    with Model(path) as m:
        toks = m.generate_greedy(11, 0, 40)
    with Model(path) as m:
        t, step = 11, []
        for p in range(40):
            t = m.forward_argmax(t, p)
            step.append(t)
    assert list(toks) == step


def test_kv_load_read_round_trip(gpu, model_dir):
    cfg = configs.SMALL_MIXED
    path = _model_path(model_dir, cfg, 203)
    rng = np.random.default_rng(3)
    with Model(path) as m:
        k = rng.standard_normal((50, cfg.n_head_kv, cfg.head_dim)).astype(np.float32)
        v = rng.standard_normal((50, cfg.n_head_kv, cfg.head_dim)).astype(np.float32)
        m.kv_load(1, 17, k, v)
        k2, v2 = m.kv_read(1, 17, 50)
        assert np.array_equal(k, k2) and np.array_equal(v, v2)


def test_step_writes_kv_like_reference(gpu, model_dir):
    """K/V rows appended by the decode step (RoPE'd K, raw V) match the oracle's cache."""
    cfg = configs.SMALL_Q4_0
    path = _model_path(model_dir, cfg, 204)
    orc = pyoracle.OracleModel(path)
    with Model(path) as m:
        tok = 3
        for p in range(6):
            m.forward(tok, p)
            tok = int(np.argmax(orc.forward(tok, p)))
        for layer in range(cfg.n_layer):
            k, v = m.kv_read(layer, 0, 6)
            ko = np.zeros_like(k)
            vo = np.zeros_like(v)
            assert orc.lib.orc_kv_read(orc.h, layer, 0, 6, pyoracle._f(ko), pyoracle._f(vo)) == 0
            for a, b in ((k, ko), (v, vo)):
                err = np.abs(a - b).max() / max(np.abs(b).max(), 1e-6)
                assert err < 1e-4, f"layer {layer} kv rel err {err}"


def test_error_paths_match_reference(gpu, model_dir):
    cfg = configs.SMALL_Q4_0
    path = _model_path(model_dir, cfg, 205)
    with Model(path, max_ctx=64) as m:
        assert m.kv_ctx == 64
        assert m.try_forward(1, 64) == -1          # pos >= kv_ctx (transformer.c:156-159)
        assert m.try_forward(cfg.n_vocab, 0) == -1  # token >= n_vocab (transformer.c:161-164)
        assert m.try_forward(1, 0) == 0             # the model stays usable
    with Model(path, max_ctx=10**6) as m:
        assert m.kv_ctx == cfg.n_ctx                # max_ctx clamped to n_ctx (transformer.c:46-47)
    with Model(path, max_ctx=0) as m:
        assert m.kv_ctx == min(cfg.n_ctx, 4096)     # 0 -> min(n_ctx, 4096) (transformer.c:43-45)


# --- full-width layers (8B and 70B widths, few layers, oracle in seconds) ----------

WIDE = [
    dataclasses.replace(configs.LLAMA8B_Q4_0, name="w8b-q4_0-2l", n_layer=2, n_ctx=1024),
    dataclasses.replace(configs.LLAMA8B_MIXED, name="w8b-mixed-1l", n_layer=1, n_ctx=8192),
    dataclasses.replace(configs.LLAMA70B_Q4_0, name="w70b-q4_0-1l", n_layer=1, n_vocab=32000, n_ctx=512),
]


@pytest.mark.parametrize("cfg", WIDE, ids=lambda c: c.name)
def test_full_width_layers_vs_oracle(gpu, model_dir, cfg):
    path = _model_path(model_dir, cfg, 301)
    orc = pyoracle.OracleModel(path, max_ctx=cfg.n_ctx)
    pos0 = 0
    with Model(path, max_ctx=cfg.n_ctx) as m:
        if cfg.t_gate == configs.Q5_0:  # config 4 style: long pre-filled KV (fp16 values)
            pos0 = 8000
            rng = np.random.default_rng(5)
            for layer in range(cfg.n_layer):
                shape = (pos0, cfg.n_head_kv, cfg.head_dim)
                k = rng.standard_normal(shape).astype(np.float16).astype(np.float32)
                v = rng.standard_normal(shape).astype(np.float16).astype(np.float32)
                m.kv_load(layer, 0, k, v)
                orc.kv_load(layer, 0, k, v)
        mism, wa, wr, gap = greedy_compare(m.forward, orc.forward, 5, pos0, 3)
    assert not mism, f"greedy mismatches: {mism}"
    print(f"{cfg.name}: worst max-abs {wa:.3g} rel {wr:.3g} min gap {gap:.3g}")
    assert wa <= 1e-2 and wr <= 1e-3


def test_long_context_more_than_32_splits_vs_oracle(gpu, model_dir):
    """Two KV heads and 3000 pre-filled positions: the attention splits each
    head over more than 32 CTAs (the merge's second round of loads)."""
    cfg = dataclasses.replace(configs.SMALL_Q4_0, name="small-q4_0-ctx4k", n_ctx=4096)
    path = _model_path(model_dir, cfg, 302)
    orc = pyoracle.OracleModel(path, max_ctx=cfg.n_ctx)
    pos0 = 3000
    with Model(path, max_ctx=cfg.n_ctx) as m:
        rng = np.random.default_rng(6)
        for layer in range(cfg.n_layer):
            shape = (pos0, cfg.n_head_kv, cfg.head_dim)
            k = rng.standard_normal(shape).astype(np.float32)
            v = rng.standard_normal(shape).astype(np.float32)
            m.kv_load(layer, 0, k, v)
            orc.kv_load(layer, 0, k, v)
        mism, wa, wr, gap = greedy_compare(m.forward, orc.forward, 5, pos0, 4)
    assert not mism, f"greedy mismatches: {mism}"
    assert wa <= 1e-2 and wr <= 1e-3


@pytest.mark.parametrize("tag", ["mixed", "q4_0"])
def test_half_row_stages_match_reference_golden(gpu, model_dir, monkeypatch, tag):
    """The persistent kernel's two-rows-per-thread GEMV stages (used when the
    four-row ring does not fit shared memory, as for the 70B shapes), forced
    on a small model: the reference's golden logits and greedy tokens."""
    monkeypatch.setenv("FWB_HALF_ROWS", "1")
    g = np.load(os.path.join(GOLDEN, f"ref_decode_{tag}_plain.npz"))
    cfg, seed = mg.GOLDEN_MODELS[tag]
    path = _model_path(model_dir, cfg, seed, f"golden_{tag}")
    pos0 = int(g["pos0"])
    with Model(path) as m:
        tok = int(g["first"])
        for i, (ref_tok, ref_lg) in enumerate(zip(g["tokens"], g["logits"])):
            lg = m.forward(tok, pos0 + i)
            assert_logits_close(lg, ref_lg, f"step {i}")
            assert int(np.argmax(lg)) == int(ref_tok), f"greedy token differs at step {i}"
            tok = int(ref_tok)
