"""Standalone quantised matvec microbenchmark (batch 1), through the C ABI.

    python -m fwb.matvec_bench [--types q4_0,q5_0,q8_0] [--shapes 4096x4096,...]
                               [--iters 50] [--seed 1]

Benchmark configuration 2 of the decode path: x ~ N(0, 1) fp32; weights in
GGUF Q4_0 / Q5_0 / Q8_0 block layout with uniform-random quants and fp16
scales d ~ U(1e-3, 1e-2); shapes (rows x cols) 4096x4096, 14336x4096,
4096x14336 and 128256x4096.  Each launch is `quant_matvec_dev` on device
buffers.  Enough copies of the weight matrix are kept on the device that
consecutive launches read different copies and more than the 126 MB L2, so
every launch streams its weights from HBM.  Time per launch: CUDA events
around `iters` launches on one stream.  Algorithmic bytes per launch: weight
bytes + 4 * (rows + cols).  One JSON line per (type, shape).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import sys

import numpy as np

from . import configs, gguf_synth, native

TYPES = {"q4_0": configs.Q4_0, "q5_0": configs.Q5_0, "q8_0": configs.Q8_0}
SHAPES = [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]
L2_BYTES = 126 * 2**20


def run(types, shapes, iters: int, seed: int, out=sys.stdout) -> list[dict]:
    import torch

    lib = native.product()
    if lib.fwb_device_count() < 1:
        raise RuntimeError("no CUDA device")
    stream = torch.cuda.current_stream()
    results = []
    for tname in types:
        t = TYPES[tname]
        for rows, cols in shapes:
            w = gguf_synth.random_matrix(t, rows, cols, seed=seed, mode=1)
            ncopy = max(2, -(-4 * L2_BYTES // w.nbytes))
            dws = [torch.from_numpy(w).cuda() for _ in range(ncopy)]
            x = torch.from_numpy(gguf_synth.normal_vector(cols, seed=seed + 1)).cuda()
            y = torch.empty(rows, device="cuda")

            def launch(i):
                rc = lib.quant_matvec_dev(dws[i % ncopy].data_ptr(), w.nbytes, t, x.data_ptr(),
                                          y.data_ptr(), cols, rows, ctypes.c_void_p(stream.cuda_stream))
                if rc != 0:
                    raise RuntimeError(lib.fwb_last_error().decode())

            for i in range(5):
                launch(i)
            torch.cuda.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for i in range(iters):
                launch(i)
            e1.record(stream)
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / iters
            nbytes = w.nbytes + 4 * (rows + cols)
            r = {"type": tname, "rows": rows, "cols": cols, "us_per_launch": us,
                 "bytes": nbytes, "gbs": nbytes / us / 1e3, "copies": ncopy}
            results.append(r)
            print(json.dumps(r), file=out, flush=True)
            del dws
            torch.cuda.empty_cache()
    return results


def main() -> None:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--types", default="q4_0,q5_0,q8_0")
    p.add_argument("--shapes", default=",".join(f"{r}x{c}" for r, c in SHAPES))
    p.add_argument("--iters", type=int, default=50)
    p.add_argument("--seed", type=int, default=1)
    a = p.parse_args()
    shapes = [tuple(int(v) for v in s.split("x")) for s in a.shapes.split(",")]
    run(a.types.split(","), shapes, a.iters, a.seed)


if __name__ == "__main__":
    main()
