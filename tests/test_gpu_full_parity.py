"""Full-depth parity at the benchmark configurations against the compiled
reference's own goldens (tests/golden/ref_full_*.npz, make_golden.py full).

Each model is regenerated from its seed and checked against the golden's
sha256, then driven the way forword.c's main loop drives transformer_forward
(main.c:143-218, transformer.c:149-326): the 8-token prompt one token at a
time, then 64 decode steps.

* Teacher-forced: every step is fed the reference's own greedy token, so
  every step compares logits on identical inputs: the greedy token must be
  the reference's (the reference's top-1/top-2 gap is reported otherwise),
  the reference's 32 largest logits must agree within max-abs 1e-2, the
  logits' L2 norm within 1e-3 relative, and at steps 0, 31 and 63 the whole
  row within max-abs 1e-2 and relative L2 1e-3.
* Free-running: fwb_generate_greedy from the same state must produce the
  reference's 64 greedy tokens exactly.

Models: the Llama-3-8B-shaped Q4_0 model behind the bench's headline (32
layers), the 8B mixed Q8_0/Q5_0 model after an 8000-position K/V pre-fill
(benchmark configuration 4), and the first 8 layers of the Llama-70B shape
with its full vocabulary on one GPU and tensor-parallel over 2 GPUs.
Models are cached in $FWB_MODEL_DIR (default /tmp/fwb_models), shared
with bench.py.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

import make_golden as mg
from fwb import gguf_synth, native
from fwb.model import Model
from parity import LOGIT_ABS, assert_logits_close

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")
MODEL_DIR = os.environ.get("FWB_MODEL_DIR", "/tmp/fwb_models")


def load_golden(tag: str):
    p = os.path.join(GOLDEN, f"ref_full_{tag}.npz")
    if not os.path.exists(p):
        pytest.skip(f"no golden {p}")
    return np.load(p)


# (configuration name, layers kept) each full golden's model is generated from
SOURCE = {"llama8b_q4_0": ("llama8b-q4_0", 0), "llama8b_mixed": ("llama8b-mixed", 0),
          "llama70b_q4_0_8layer": ("llama70b-q4_0", 8)}


def model_for(tag: str, g) -> str:
    name, layers = SOURCE[tag]
    path = gguf_synth.cached_model_subprocess(name, int(g["seed"]), MODEL_DIR, layers=layers)
    assert mg.sha256(path) == str(g["sha256"]), f"{path}: model bytes differ from the golden's"
    return path


def check_teacher_forced(forward, g, where: str):
    """forward(tok, pos) -> logits.  Returns the worst (max-abs, rel) seen."""
    tokens = g["tokens"]
    tok, pos0 = int(g["prompt"][-1]), int(g["pos_first"])
    rows = {int(s): r for s, r in zip(g["row_steps"], g["rows"])}
    mism, worst = [], 0.0
    for i in range(len(tokens)):
        lg = forward(tok, pos0 + i)
        assert np.all(np.isfinite(lg)), f"{where} step {i}: non-finite logits"
        idx, val = g["top_idx"][i], g["top_val"][i]
        d = float(np.abs(lg[idx].astype(np.float64) - val.astype(np.float64)).max())
        worst = max(worst, d)
        assert d <= LOGIT_ABS, f"{where} step {i}: top-32 logits differ by {d:.3g}"
        n = float(np.linalg.norm(lg.astype(np.float64)))
        assert abs(n - float(g["norm"][i])) <= 1e-3 * float(g["norm"][i]), f"{where} step {i}: norm {n} vs {g['norm'][i]}"
        if i in rows:
            assert_logits_close(lg, rows[i], f"{where} step {i}")
        if int(np.argmax(lg)) != int(tokens[i]):
            mism.append((i, int(np.argmax(lg)), int(tokens[i]), float(val[0] - val[1])))
        tok = int(tokens[i])
    assert not mism, f"{where}: greedy tokens differ (step, gpu, ref, ref top-2 gap): {mism}"
    return worst


@pytest.fixture(scope="module")
def gpu(built):
    if native.product().fwb_device_count() < 1:
        pytest.skip("no CUDA device")
    return True


@pytest.mark.parametrize("tag", ["llama8b_q4_0", "llama8b_mixed", "llama70b_q4_0_8layer"])
def test_full_depth_matches_reference(gpu, tag):
    g = load_golden(tag)
    path = model_for(tag, g)
    cfg, seed, n_pre, kv_ctx = mg.FULL_MODELS[tag]
    with Model(path, max_ctx=int(g["kv_ctx"])) as m:
        for layer in range(cfg.n_layer if n_pre else 0):
            k, v = mg.prefill_kv(cfg, layer, n_pre, seed)
            m.kv_load(layer, 0, k, v)
        pos = n_pre
        for t in g["prompt"][:-1]:
            m.forward(int(t), pos)
            pos += 1
        worst = check_teacher_forced(m.forward, g, tag)
        gen = m.generate_greedy(int(g["prompt"][-1]), int(g["pos_first"]), len(g["tokens"]))
    assert np.array_equal(gen, g["tokens"]), f"{tag}: free-running greedy tokens differ: {gen} vs {g['tokens']}"
    print(f"{tag}: 64 teacher-forced steps, worst top-32 |diff| {worst:.3g}; 64 free-running tokens identical")


def test_70b_slice_tensor_parallel_2(gpu, tmp_path):
    """The 70B slice split over 2 GPUs (column/row splits, NVLink all-reduce
    inside the decode kernel) against the same reference golden."""
    if native.product().fwb_device_count() < 2:
        pytest.skip("needs 2 GPUs")
    tag = "llama70b_q4_0_8layer"
    g = load_golden(tag)
    path = model_for(tag, g)
    out = str(tmp_path / "tp_full.npz")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
                        "--master-addr=127.0.0.1", "--master-port=29541", os.path.join(HERE, "tp_worker.py"),
                        path, out, "golden", os.path.join(GOLDEN, f"ref_full_{tag}.npz")],
                       env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = np.load(out)
    steps = iter(res["logits"])
    check_teacher_forced(lambda tok, pos: next(steps), g, "tp2")
    gen = res["gen"]
    assert (gen == gen[0]).all(), "ranks disagree on the greedy tokens"
    assert np.array_equal(gen[0], g["tokens"]), "tp2: free-running greedy tokens differ"
