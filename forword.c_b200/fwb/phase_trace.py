"""Phase timeline of the persistent decode kernel, through the C ABI.

    python -m fwb.phase_trace [--config llama8b-q4_0] [--layers 8] [--pos 600]
                              [--prefill-kv] [--steps 8] [--seed 1]

Opens the synthetic model of `--config` (its first `--layers` layers) with
FWB_TRACE=1, brings the K/V cache to position `--pos` (decode steps from
position 0, or with `--prefill-kv` the seeded fp16-rounded N(0, 1) rows of
benchmark configuration 4 through `fwb_kv_load`), runs 4 greedy warm-up
steps and then `--steps` traced ones, and prints per phase kind (the phase
name without its layer prefix) the mean time CTA 0 spent in the phase and
waiting at the barrier after it (`fwb_trace_read`: GPU global timer).  A
tracing aid: tracing adds timer reads and stores, so these times are not
bench values.
"""
from __future__ import annotations

import argparse
import ctypes
import os
import sys

import numpy as np

from . import configs, gguf_synth


def main() -> None:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--config", default="llama8b-q4_0", choices=sorted(configs.CONFIGS))
    p.add_argument("--layers", type=int, default=8)
    p.add_argument("--pos", type=int, default=600)
    p.add_argument("--prefill-kv", action="store_true")
    p.add_argument("--steps", type=int, default=8)
    p.add_argument("--seed", type=int, default=1)
    p.add_argument("--model-dir", default=None)
    args = p.parse_args()
    os.environ["FWB_TRACE"] = "1"  # read by fwb_model_open
    from .model import Model

    base = configs.CONFIGS[args.config]
    cfg = configs.with_layers(base, args.layers) if args.layers else base
    path = gguf_synth.cached_model_subprocess(base.name, args.seed, args.model_dir, layers=args.layers)
    with Model(path, max_ctx=args.pos + args.steps + 64) as m:
        lib = m.lib
        lib.fwb_trace_read.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint64), ctypes.c_size_t,
                                       ctypes.c_char_p, ctypes.c_size_t]
        tok = 1
        if args.prefill_kv:
            for layer in range(cfg.n_layer):
                k, v = gguf_synth.kv_prefill_values(cfg, layer, args.pos, args.seed)
                m.kv_load(layer, 0, k, v)
        else:
            for i in range(args.pos):
                tok = m.forward_argmax(tok, i)
        for i in range(4):
            tok = m.forward_argmax(tok, args.pos + i)
        acc: dict[str, list] = {}
        n = 16384
        buf = (ctypes.c_uint64 * n)()
        names = ctypes.create_string_buffer(64 * n)
        for s in range(args.steps):
            tok = m.forward_argmax(tok, args.pos + 4 + s)
            k = lib.fwb_trace_read(m.h, buf, n, names, 64)
            if k < 0:
                raise SystemExit("fwb_trace_read failed (is the decode kernel persistent?)")
            t = np.array(buf[:k], dtype=np.float64)
            for j in range((k - 1) // 2):
                name = names.raw[64 * j:64 * j + 64].split(b"\0")[0].decode()
                a = acc.setdefault(name.split(".", 1)[-1], [0.0, 0.0, 0])
                a[0] += t[2 * j + 1] - t[2 * j]
                a[1] += t[2 * j + 2] - t[2 * j + 1]
                a[2] += 1
    total = sum(a[0] + a[1] for a in acc.values()) / args.steps
    print(f"{cfg.name}: {total / 1e3:.1f} us per traced step at positions {args.pos + 4}..{args.pos + 3 + args.steps}")
    for name, a in acc.items():
        print(f"  {name:18s} work {a[0] / a[2] / 1e3:7.2f} us  barrier {a[1] / a[2] / 1e3:6.2f} us  "
              f"(x{a[2] // args.steps} per step)")


if __name__ == "__main__":
    sys.exit(main())
