"""Prompt processing (fwb_prefill, through the C ABI) against the oracle.

fwb_prefill(tokens, pos0) must leave the model where n calls of the decode
step would: the last token's logits within the decode tolerance of the
oracle fed token by token (parity.py: max-abs <= 1e-2, relative L2 <= 1e-3),
and a KV cache from which greedy decoding continues with the oracle's tokens.
The batched layers round GEMM inputs to fp16, so the bound is the same
tolerance, not equality with the per-token path.
"""
import dataclasses
import os

import numpy as np
import pytest

import pyoracle
from fwb import configs, gguf_synth, native
from fwb.model import Model
from parity import assert_logits_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu(built):
    if native.product().fwb_device_count() < 1:
        pytest.skip("no CUDA device")
    return True


def _check(path, tokens, pos0, n_after, ctx):
    orc = pyoracle.OracleModel(path)
    want = None
    for i, t in enumerate(tokens):
        want = orc.forward(int(t), pos0 + i)
    with Model(path, max_ctx=ctx) as m:
        if pos0:  # positions before pos0 come from the decode step
            pre = np.random.default_rng(9).integers(0, m.n_vocab, pos0)
            o2 = pyoracle.OracleModel(path)
            for i, t in enumerate(pre):
                m.forward(int(t), i)
                o2.forward(int(t), i)
            for i, t in enumerate(tokens):
                want = o2.forward(int(t), pos0 + i)
            orc.close()
            orc = o2
        got = m.prefill(tokens, pos0)
        assert_logits_close(got, want, "last prompt token")
        tok = int(np.argmax(want))
        for i in range(n_after):
            pos = pos0 + len(tokens) + i
            g = m.forward(tok, pos)
            w = orc.forward(tok, pos)
            assert_logits_close(g, w, f"decode step {i} after the prompt")
            tok = int(np.argmax(w))
    orc.close()


@pytest.mark.parametrize("n,pos0", [(2, 0), (37, 0), (130, 0), (64, 40)])
def test_prefill_q4_0_matches_oracle(gpu, tmp_path, n, pos0):
    path = gguf_synth.write_model(str(tmp_path / "pf.gguf"), configs.SMALL_Q4_0, seed=51)
    tokens = np.random.default_rng(n).integers(0, configs.SMALL_Q4_0.n_vocab, n)
    _check(path, tokens, pos0, 4, 512)


# the prompt attention's variants: tensor cores for head_dim 128 at query
# groups 1, 4 and 8 (the 8B / 70B groups; group 2 is SMALL_Q4_0 above), the
# CUDA-core flash kernel for head_dim 64, the per-(token, KV head) kernel for
# other head dims; 150 tokens span several query and key tiles
@pytest.mark.parametrize("n_embd,n_head,n_kv", [(1024, 8, 8), (1024, 8, 2), (1024, 8, 1), (512, 8, 2),
                                                (256, 8, 4)])
def test_prefill_attention_shapes(gpu, tmp_path, n_embd, n_head, n_kv):
    cfg = dataclasses.replace(configs.SMALL_Q4_0, name=f"pf-{n_embd}-{n_head}-{n_kv}", n_embd=n_embd,
                              n_head=n_head, n_head_kv=n_kv, n_ff=2 * n_embd)
    path = gguf_synth.write_model(str(tmp_path / f"{cfg.name}.gguf"), cfg, seed=55)
    tokens = np.random.default_rng(n_embd + n_kv).integers(0, cfg.n_vocab, 150)
    _check(path, tokens, 0, 2, 512)


def test_prefill_more_tokens_than_a_chunk(gpu, tmp_path):
    cfg = dataclasses.replace(configs.SMALL_Q4_0, name="small-q4_0-ctx1k", n_ctx=1024)
    path = gguf_synth.write_model(str(tmp_path / "pf1k.gguf"), cfg, seed=52)
    tokens = np.random.default_rng(3).integers(0, cfg.n_vocab, 700)
    _check(path, tokens, 0, 2, 1024)


def test_prefill_mixed_types_take_the_decode_path(gpu, tmp_path):
    path = gguf_synth.write_model(str(tmp_path / "pfm.gguf"), configs.SMALL_MIXED, seed=53)
    tokens = np.random.default_rng(4).integers(0, configs.SMALL_MIXED.n_vocab, 20)
    _check(path, tokens, 0, 2, 512)


def test_prefill_rejects_bad_arguments(gpu, tmp_path):
    path = gguf_synth.write_model(str(tmp_path / "pfe.gguf"), configs.SMALL_Q4_0, seed=54)
    with Model(path, max_ctx=64) as m:
        with pytest.raises(Exception, match="KV cache"):
            m.prefill(np.zeros(65, dtype=np.uint32), 0)
        with pytest.raises(Exception, match="out of range"):
            m.prefill(np.array([1, m.n_vocab], dtype=np.uint32), 0)
