"""One rank of a tensor-parallel decode check, launched by test_gpu_tp.py
through torch.distributed.run (one process per GPU).

    python -m torch.distributed.run --nproc-per-node N tests/tp_worker.py MODEL OUT.npz STEPS

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


def main():
    path, out, steps = sys.argv[1], sys.argv[2], int(sys.argv[3])
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dist.init_process_group("gloo")
    torch.cuda.set_device(local)
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
