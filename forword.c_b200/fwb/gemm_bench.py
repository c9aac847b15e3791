"""Tensor-core dequant-GEMM microbenchmark (the prompt path's linear layers).

    python -m fwb.gemm_bench [--tokens 512] [--shapes 6144x4096,...] [--iters 20]

Q4_0 weights (GGUF block layout, N(0, 0.02) quantised) times M fp16 token
rows through `quant_gemm_dev`.  Shapes (rows x cols) default to the 8B
model's QKV, o-proj, gate/up and down matrices.  Time per launch: CUDA events
around --iters launches on one stream after 3 warm-up launches.  FLOPs per
launch: 2 * M * rows * cols.  One JSON line per shape.
"""
from __future__ import annotations

import argparse
import json
import sys

from . import configs, gguf_synth, native

SHAPES = [(6144, 4096), (4096, 4096), (14336, 4096), (4096, 14336)]


def run(tokens: int, shapes, iters: int, out=sys.stdout) -> list[dict]:
    import torch

    lib = native.product()
    if lib.fwb_device_count() < 1:
        raise RuntimeError("no CUDA device")
    stream = torch.cuda.current_stream()
    res = []
    for rows, cols in shapes:
        w = gguf_synth.random_matrix(configs.Q4_0, rows, cols, seed=1, mode=0, lo=0.0, hi=0.02)
        dw = torch.from_numpy(w).cuda()
        x = torch.randn(tokens, cols, device="cuda").half()
        y = torch.empty(tokens, rows, device="cuda")

        def launch():
            rc = lib.quant_gemm_dev(dw.data_ptr(), w.nbytes, configs.Q4_0, x.data_ptr(), y.data_ptr(), cols, rows,
                                    tokens, 0, stream.cuda_stream)
            if rc != 0:
                raise RuntimeError(lib.fwb_last_error().decode())

        for _ in range(3):
            launch()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(iters):
            launch()
        e1.record(stream)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / iters
        r = {"rows": rows, "cols": cols, "tokens": tokens, "us_per_launch": us,
             "tflops": 2.0 * tokens * rows * cols / us / 1e6, "weight_gbs": w.nbytes / us / 1e3}
        res.append(r)
        print(json.dumps(r), file=out, flush=True)
    return res


def main() -> None:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--tokens", type=int, default=512)
    p.add_argument("--shapes", default=",".join(f"{r}x{c}" for r, c in SHAPES))
    p.add_argument("--iters", type=int, default=20)
    a = p.parse_args()
    run(a.tokens, [tuple(int(v) for v in s.split("x")) for s in a.shapes.split(",")], a.iters)


if __name__ == "__main__":
    main()
