"""A small decode case for profilers (ncu captures of decode_kernel).

    python -m fwb.profile_case [--config llama8b-q4_0] [--layers 4] [--pos 600]
                               [--steps 6] [--seed 1]

Writes (once, cached) a seeded synthetic GGUF of the named configuration
with only --layers layers, then runs --steps greedy decode steps through the
C ABI starting at position --pos.  Every layer has the full model's shapes,
so the kernel runs the same phases and code as the full model, with a weight
footprint small enough for multi-pass profiler captures.
"""
from __future__ import annotations

import argparse
from dataclasses import replace

from . import configs, gguf_synth
from .model import Model


def main() -> None:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--config", default="llama8b-q4_0", choices=sorted(configs.CONFIGS))
    p.add_argument("--layers", type=int, default=4)
    p.add_argument("--pos", type=int, default=600)
    p.add_argument("--steps", type=int, default=6)
    p.add_argument("--seed", type=int, default=1)
    a = p.parse_args()
    base = configs.CONFIGS[a.config]
    cfg = replace(base, name=f"{base.name}-{a.layers}layer", n_layer=a.layers)
    path = gguf_synth.cached_model(cfg, seed=a.seed)
    m = Model(path, max_ctx=max(1024, a.pos + a.steps + 1))
    tok = 1
    for i in range(a.steps):
        tok = m.forward_argmax(tok, a.pos + i)
    print("ok", tok)


if __name__ == "__main__":
    main()
