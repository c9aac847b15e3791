"""Tensor-parallel host logic, on CPU (no GPU needed).

* The slice every rank keeps of every tensor (fwb_tp_shard, the rule the
  model upload uses) reassembles the whole tensor: row splits concatenate,
  column splits (attn_output, ffn_down) join row by row.  Checked with 2 and
  4 gloo ranks in separate processes, each extracting its own slices.
* The all-reduce identity behind the split: the ranks' partial products of
  attn_output / ffn_down (their input-column slices times their slices of
  the input) sum to the whole product, with the oracle's quant_matvec.
* The exchange of IPC handles returns every rank's handle in rank order.
"""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import pyoracle
from fwb import configs, gguf_synth
from fwb.model import FwbError, tp_shard
from fwb.tp import gather_handles

CFG = configs.SMALL_Q4_0  # 4 heads / 2 KV heads, ff 1024, vocab 2048: splits in 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture(scope="module")
def model(built, tmp_path_factory):
    d = tmp_path_factory.mktemp("tp")
    return gguf_synth.write_model(str(d / "tp.gguf"), CFG, seed=31)


def _tensors(cfg=CFG):
    names = [("token_embd.weight", False), ("output.weight", True), ("output_norm.weight", False)]
    for l in range(cfg.n_layer):
        for t in ("attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "ffn_norm", "ffn_gate",
                  "ffn_up", "ffn_down"):
            names.append((f"blk.{l}.{t}.weight", False))
    return names


def _col_split(name: str) -> bool:
    return name.endswith("attn_output.weight") or name.endswith("ffn_down.weight")


def _shard_worker(rank, world, port, path, cfg_name, errq):
    try:
        cfg = configs.CONFIGS[cfg_name]
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        mine = {n: tp_shard(path, n, rank, world, as_head=h).tobytes() for n, h in _tensors(cfg)}
        allp = [None] * world
        dist.all_gather_object(allp, mine)
        handles = gather_handles(bytes([rank]) * 64)
        assert handles == [bytes([q]) * 64 for q in range(world)]
        if rank == 0:
            for n, h in _tensors(cfg):
                full = tp_shard(path, n, 0, 1, as_head=h)
                parts = [np.frombuffer(p[n], dtype=np.uint8) for p in allp]
                if _col_split(n):
                    rows = cfg.n_embd
                    got = np.concatenate([p.reshape(rows, -1) for p in parts], axis=1).reshape(-1)
                elif n.endswith("norm.weight") or n == "token_embd.weight":
                    assert all(np.array_equal(p, full) for p in parts), n  # whole on every rank
                    continue
                else:
                    got = np.concatenate(parts)
                assert np.array_equal(got, full), n
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.parametrize("world", [2, 4])
def test_ranks_reassemble_every_tensor(built, tmp_path, world):
    cfg = CFG if world == 2 else configs.SMALL_TP8
    model = gguf_synth.write_model(str(tmp_path / f"tp{world}.gguf"), cfg, seed=30 + world)
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_shard_worker, args=(r, world, port, model, cfg.name, errq)) for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=300)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not errs, errs
    assert all(p.exitcode == 0 for p in ps), [p.exitcode for p in ps]


@pytest.mark.parametrize("tensor,width", [("blk.0.attn_output.weight", CFG.n_head * CFG.head_dim),
                                          ("blk.1.ffn_down.weight", CFG.n_ff)])
def test_partial_products_sum_to_the_whole(model, tensor, width):
    world = 2
    x = gguf_synth.normal_vector(width, seed=5)
    full = tp_shard(model, tensor, 0, 1)
    want = pyoracle.quant_matvec(full, configs.Q4_0, x, CFG.n_embd)
    got = np.zeros(CFG.n_embd, dtype=np.float64)
    w = width // world
    for r in range(world):
        part = tp_shard(model, tensor, r, world)
        got += pyoracle.quant_matvec(part, configs.Q4_0, x[r * w:(r + 1) * w].copy(), CFG.n_embd)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5 * np.abs(want).max())


def test_rejects_splits_that_do_not_divide(model):
    with pytest.raises(FwbError):
        tp_shard(model, "blk.0.attn_k.weight", 0, 4)  # 2 KV heads over 4 ranks
