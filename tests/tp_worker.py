"""One rank of a tensor-parallel decode check, launched by test_gpu_tp.py
through torch.distributed.run (one process per GPU).

    python -m torch.distributed.run --nproc-per-node N tests/tp_worker.py MODEL OUT.npz STEPS
    python -m torch.distributed.run --nproc-per-node N tests/tp_worker.py MODEL OUT.npz golden GOLDEN.npz

Feeds the same token stream to every rank (teacher forcing from a fixed
seed), records rank 0's full logits per step (gathered over NVLink by the
library), then runs greedy generation on every rank; rank 0 writes
everything to OUT.npz.  Handles travel over a gloo group (bytes only).
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "forword.c_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from fwb import tp  # noqa: E402


def golden_mode(path: str, out: str, golden: str, rank: int, world: int, local: int):
    """Drive the model like test_gpu_full_parity does on one GPU: the
    golden's prompt one token at a time, then the reference's greedy tokens
    teacher-forced (rank 0 keeps the logits), then free-running greedy."""
    g = np.load(golden)
    m = tp.open_model(path, int(g["kv_ctx"]), rank, world, local)
    pos = int(g["n_prefill"])
    for t in g["prompt"][:-1]:
        m.forward(int(t), pos)
        pos += 1
    tok = int(g["prompt"][-1])
    logits = np.zeros((len(g["tokens"]), m.n_vocab), dtype=np.float32)
    for i, t in enumerate(g["tokens"]):
        logits[i] = m.forward(tok, pos + i)
        tok = int(t)
    gen = m.generate_greedy(int(g["prompt"][-1]), pos, len(g["tokens"]))
    allgen = [None] * world
    dist.all_gather_object(allgen, gen.tolist())
    if rank == 0:
        np.savez(out, logits=logits, gen=np.array(allgen, dtype=np.uint32))
    m.close()


def main():
    path, out = sys.argv[1], sys.argv[2]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dist.init_process_group("gloo")
    torch.cuda.set_device(local)
    if sys.argv[3] == "golden":
        golden_mode(path, out, sys.argv[4], rank, world, local)
        dist.barrier()
        dist.destroy_process_group()
        return
    steps = int(sys.argv[3])
    m = tp.open_model(path, 0, rank, world, local)
    toks = np.random.default_rng(3).integers(0, m.n_vocab, steps)
    logits = np.zeros((steps, m.n_vocab), dtype=np.float32)
    for i, t in enumerate(toks):
        logits[i] = m.forward(int(t), i)
    gen = m.generate_greedy(int(toks[-1]), steps, 24)
    allgen = [None] * world
    dist.all_gather_object(allgen, gen.tolist())
    if rank == 0:
        np.savez(out, tokens=toks, logits=logits, gen=np.array(allgen, dtype=np.uint32))
    m.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
