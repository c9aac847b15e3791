"""Tensor-parallel decode on 2, 4 and 8 GPUs (each case skipped with fewer
GPUs): every rank runs
its slice of the model in its own process, the partial sums after o-proj and
down-proj are added over NVLink inside the persistent kernel, and rank 0's
logits (its own slice plus the peers', gathered by the library) must match
the oracle running the whole model on the CPU, step by step, within the
decode tolerance; greedy generation must give the same tokens on every rank
and match the oracle's greedy continuation (teacher forcing on ties).
"""
import os
import subprocess
import sys

import numpy as np
import pytest

import pyoracle
from fwb import configs, gguf_synth, native
from parity import assert_logits_close

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("cfg,seed,world", [(configs.SMALL_Q4_0, 41, 2), (configs.SMALL_MIXED, 42, 2),
                                            (configs.SMALL_TP8, 43, 4), (configs.SMALL_TP8, 44, 8)])
def test_tp_matches_oracle(built, tmp_path, cfg, seed, world):
    if native.product().fwb_device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    path = gguf_synth.write_model(str(tmp_path / "tp.gguf"), cfg, seed=seed)
    out = str(tmp_path / "tp.npz")
    steps = 12
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
                        "--master-addr=127.0.0.1", "--master-port=29533", os.path.join(HERE, "tp_worker.py"),
                        path, out, str(steps)], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    g = np.load(out)
    orc = pyoracle.OracleModel(path)
    for i, t in enumerate(g["tokens"]):
        want = orc.forward(int(t), i)
        assert_logits_close(g["logits"][i], want, f"step {i}")
    gen = g["gen"]
    assert (gen == gen[0]).all(), "ranks disagree on the greedy tokens"
    tok = int(g["tokens"][-1])
    for i, got in enumerate(gen[0]):
        want = int(np.argmax(orc.forward(tok, steps + i)))
        assert int(got) == want, f"greedy step {i}"
        tok = want
    orc.close()
