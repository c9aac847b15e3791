"""GPU edge cases of the decode step against the reference's semantics.

* Greedy token with NaN / +-inf logits: sampler_argmax (sampler.c:28-32)
  starts at index 0 and moves on a strict '>' only, so a NaN logit never
  wins, a NaN at index 0 is never beaten (token 0), and the first of equal
  maxima (+inf included) wins.  The device argmax is checked against that
  rule applied to the device's own logits row.  The non-finite logits are
  made by patching block scales of the head (fp16 NaN / +inf) in the file.
* A model without output_norm.weight: the head reads x unnormalised
  (transformer.c:304-306), checked against the oracle.
"""
import os

import numpy as np
import pytest

import pyoracle
from fwb import configs, gguf_synth, native
from fwb.model import Model
from parity import assert_logits_close

pytestmark = pytest.mark.gpu

F16_NAN, F16_INF = 0x7E00, 0x7C00


@pytest.fixture(scope="module")
def gpu(built):
    if native.product().fwb_device_count() < 1:
        pytest.skip("no CUDA device")
    return True


def ref_argmax(logits: np.ndarray) -> int:
    """sampler_argmax (sampler.c:28-32) restated: first index, strict '>'."""
    best = 0
    for i in range(1, logits.size):
        if logits[i] > logits[best]:
            best = i
    return best


def _patch_head_scales(path: str, cfg, rows_blocks: dict) -> None:
    """Set the fp16 scale of given (row -> list of block indices, or 'all')
    of output.weight (Q4_0: 18-byte blocks, scale in the first 2 bytes)."""
    import gguf
    r = gguf.GGUFReader(path)
    t = next(t for t in r.tensors if t.name == "output.weight")
    off = int(t.data_offset)
    bpr = cfg.n_embd // 32
    mm = np.memmap(path, dtype=np.uint8, mode="r+")
    for row, (blocks, bits) in rows_blocks.items():
        for b in (range(bpr) if blocks == "all" else blocks):
            o = off + (row * bpr + b) * 18
            mm[o] = bits & 0xFF
            mm[o + 1] = bits >> 8
            if blocks != "all":  # the row's other blocks contribute exactly 0
                for b2 in range(bpr):
                    if b2 not in blocks:
                        o2 = off + (row * bpr + b2) * 18
                        mm[o2] = 0
                        mm[o2 + 1] = 0
    mm.flush()
    del mm


@pytest.mark.parametrize("case", ["nan_at_0", "nan_elsewhere", "inf_rows"])
def test_device_argmax_follows_sampler_argmax(gpu, model_dir, case):
    cfg = configs.SMALL_Q4_0
    path = gguf_synth.write_model(os.path.join(model_dir, f"argmax_{case}.gguf"), cfg, seed=77)
    if case == "nan_at_0":
        patch = {0: ("all", F16_NAN)}
    elif case == "nan_elsewhere":
        patch = {3: ("all", F16_NAN), 100: ("all", F16_NAN)}
    else:  # one block of +inf scale per row: that row's logit is +-inf (NaN if its block dot is 0)
        patch = {5: ([0], F16_INF), 9: ([1], F16_INF), 40: ([2], F16_INF), 41: ([3], F16_INF)}
    _patch_head_scales(path, cfg, patch)
    with Model(path) as m:
        tok = 7
        for pos in range(6):
            lg = m.forward(tok, pos)
            want = ref_argmax(lg)
            got = m.forward_argmax(tok, pos)
            assert got == want, f"pos {pos}: device token {got}, sampler_argmax {want}"
            if case == "nan_at_0":
                assert np.isnan(lg[0]) and got == 0
            if case == "nan_elsewhere":
                assert np.isnan(lg[3]) and np.isnan(lg[100])
            tok = (got * 31 + 5) % cfg.n_vocab  # vary the input
        if case == "inf_rows":
            assert np.isinf(lg[[5, 9, 40, 41]]).any()


def test_model_without_output_norm(gpu, model_dir):
    cfg = configs.SMALL_NO_OUT_NORM
    path = gguf_synth.write_model(os.path.join(model_dir, "no_out_norm.gguf"), cfg, seed=12)
    orc = pyoracle.OracleModel(path)
    with Model(path) as m:
        tok = 3
        for pos in range(5):
            lg = m.forward(tok, pos)
            want = orc.forward(tok, pos)
            assert_logits_close(lg, want, f"step {pos}")
            tok = int(np.argmax(want))
    orc.close()
