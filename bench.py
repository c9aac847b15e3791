#!/usr/bin/env python3
"""Batch-1 decode benchmark of forword.c's per-token forward on B200.

Workload (N=1, benchmark configuration 3): the Llama-3-8B-shaped decoder with every linear weight in
GGUF Q4_0 (embedding and norms fp32), random-init N(0, 0.02) from a seed and
written as a GGUF file.  A 512-token uniform-random prompt goes through
fwb_prefill (all prompt tokens through each layer together on the tensor
cores; the reference feeds a prompt one token at a time, main.c:145-151; the
prompt is timed separately, the `prefill` key), then greedy decode runs at
batch 1: W untimed warm-up tokens, then K timed tokens.
One step = one token = one `transformer_forward` (one launch of the
persistent decode kernel).

Arms
  --impl b200       (default) the CUDA library through its C ABI
                    (include/forword_b200.h):
                    value  device-timed greedy decode, the token chosen on the
                           device feeds the next step; weights resident in HBM.
                    e2e    `fwb_forward` per token with host buffers: token/pos
                           copied in, the full logits row copied out to pinned
                           host memory, the next token picked on the host
                           (sampler_argmax, sampler.c:28-32) — what the
                           reference's main loop does with transformer_forward.
  --impl reference  the reference's own CPU decode step (its sources compiled
                    by oracle/Makefile into oracle/_ref, else the oracle's C
                    restatement), same model and positions, timed on the host.

Multi-GPU (--gpus N under torchrun): the Llama-70B-shaped Q4_0 model (benchmark
configuration 5) decodes tensor-parallel over the N GPUs: every rank holds
its slices of the weights, and the partial sums after o-proj and down-proj
are added over NVLink inside the decode kernel.  One decode stream for the
box ("scaling": "strong"); value = tokens/s of that stream, timed on the
device on every rank, max over ranks.

Every weight byte of a step is streamed from HBM (4.2 GB per token on one GPU
for the 8B model, 39 GB / N per GPU for the 70B model, against a 126 MB L2),
so no explicit L2 flush is needed between steps.
"""
from __future__ import annotations

import argparse
import csv
import datetime
import io
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "forword.c_b200"))

import numpy as np  # noqa: E402

from fwb import configs, gguf_synth  # noqa: E402

METRIC = "batch-1 decode tokens/s per box"
UNIT = "tokens/s"
MODEL_SEED = 1
PROMPT_SEED = 2024


class Workload:
    """The benchmark configuration one run measures.

    N = 1: configuration 3 -- the Llama-3-8B shape, every linear weight Q4_0,
    512-token prompt, greedy decode on one GPU.
    N > 1: configuration 5 -- the Llama-70B shape, every linear weight Q4_0,
    256-token prompt, greedy decode tensor-parallel over the N GPUs (one
    decode stream for the whole box: strong scaling).
    --workload long-context (N = 1): configuration 4 -- the 8B shape with
    Q8_0 attention / down / head and Q5_0 gate / up, context 8192 with the
    K/V cache pre-filled at positions [0, 8000) with fp16-rounded N(0, 1)
    values, then greedy decode from position 8000.
    """

    def __init__(self, world: int, layers: int = 0, kind: str = "default"):
        self.tp = world > 1
        self.long = kind == "long-context"
        if self.long and self.tp:
            raise SystemExit("--workload long-context runs on one GPU")
        self.base = (configs.LLAMA8B_MIXED if self.long else
                     configs.LLAMA70B_Q4_0 if self.tp else configs.LLAMA8B_Q4_0)
        self.cfg = configs.with_layers(self.base, layers) if layers else self.base
        self.prompt = 8000 if self.long else 256 if self.tp else 512
        if self.long:
            shape = "Llama-3-8B-shaped decoder, Q8_0 attention/down/head and Q5_0 gate/up"
            feed = "K/V cache pre-filled at 8000 positions with fp16-rounded N(0,1) values (fwb_kv_load)"
        else:
            shape = ("Llama-70B" if self.tp else "Llama-3-8B") + "-shaped decoder, all linear weights Q4_0"
            feed = f"{self.prompt}-token random prompt (" + ("one decode step per token" if self.tp
                                                            else "fwb_prefill") + ")"
        if layers:
            shape += f" (first {layers} layers only: a profiler case, not a bench value)"
        self.text = (f"{shape}, fp32 embedding/norms, random-init N(0,0.02); {feed}, then "
                     f"greedy decode at batch 1" + (f", tensor parallel over {world} GPUs" if self.tp else ""))

    def prompt_ids(self) -> np.ndarray:
        if self.long:  # no prompt tokens: the first decode step is fed this token
            return np.array([1], dtype=np.uint32)
        return np.random.default_rng(PROMPT_SEED).integers(0, self.cfg.n_vocab, self.prompt).astype(np.uint32)

    def kv_prefill(self, load) -> None:
        """load(layer, pos0, k, v) for the long-context pre-fill (no-op otherwise)."""
        if not self.long:
            return
        for layer in range(self.cfg.n_layer):
            k, v = gguf_synth.kv_prefill_values(self.cfg, layer, self.prompt, MODEL_SEED)
            load(layer, 0, k, v)

    def kv_bytes_per_position(self, world: int = 1) -> int:
        c = self.cfg
        return 2 * c.n_layer * (c.n_head_kv // world) * c.head_dim * 4

    def config(self, world: int, k_steps: int, w_steps: int, kv_ctx: int) -> dict:
        cfg = {
            "workload": self.text,
            "model": self.cfg.name,
            "global_batch": 1,
            "prompt_tokens": 0 if self.long else self.prompt,
            "decode_positions": [self.prompt + w_steps, self.prompt + w_steps + k_steps],
            "kv_ctx": kv_ctx,
            "parallelism": f"tensor parallel x{world}" if world > 1 else "single GPU",
            "l2": "inputs larger than L2: every step streams the model's quantised weights "
                  f"({self.cfg.weight_bytes_per_token() / 1e9:.1f} GB per token)",
        }
        if self.long:
            cfg["kv_prefill_positions"] = self.prompt
        return cfg


def _args():
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=256, help="timed decode tokens per rank")
    p.add_argument("--warmup", type=int, default=8, help="untimed decode tokens before timing")
    p.add_argument("--impl", choices=("b200", "reference"), default="b200")
    p.add_argument("--no-cpu-baseline", action="store_true",
                   help="skip the timed reference sample in the b200 arm")
    p.add_argument("--cpu-budget-s", type=float, default=15.0,
                   help="CPU seconds for the reference sample inside the b200 arm")
    p.add_argument("--ref-budget-s", type=float, default=300.0,
                   help="cap on the timed CPU seconds of the --impl reference arm")
    p.add_argument("--model-dir", default=None, help="where the synthetic GGUF is cached")
    p.add_argument("--layers", type=int, default=0,
                   help="profiler case: the same model with only its first N layers (not a bench value)")
    p.add_argument("--workload", choices=("default", "long-context"), default="default",
                   help="long-context: benchmark configuration 4 (8B mixed quants, 8000 pre-filled positions)")
    return p.parse_args()


def _peaks() -> tuple[float, str]:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def _dist():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def _model_path(args, wl: Workload) -> str:
    """The cached synthetic GGUF, written (once) by a child process: neither
    arm loads the generator library."""
    return gguf_synth.cached_model_subprocess(wl.base.name, MODEL_SEED, args.model_dir, layers=args.layers)


def _kv_ctx(wl: Workload, k_steps: int, w_steps: int) -> int:
    """KV length both arms allocate: the prompt (or pre-filled positions),
    the warm-up and the timed decode steps (the b200 arm's e2e pass decodes
    the timed positions again)."""
    if wl.long:
        return 8192
    need = wl.prompt + w_steps + k_steps + 1
    return max(1024, 1 << (need - 1).bit_length())


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
_CLOCK_FIELDS = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class ClockSampler:
    """nvidia-smi sampled every 20 ms for one device (read-only queries)."""

    def __init__(self, device: int):
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(device), f"--query-gpu={_CLOCK_FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        self.t0 = self.t1 = None

    def mark_start(self):
        self.t0 = datetime.datetime.now()

    def mark_end(self):
        self.t1 = datetime.datetime.now()

    def finish(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = []
        for r in csv.reader(io.StringIO(out)):
            if len(r) < 9:
                continue
            r = [c.strip() for c in r]
            try:
                ts = datetime.datetime.strptime(r[0], "%Y/%m/%d %H:%M:%S.%f")
                rows.append((ts, float(r[1]), float(r[2]), r[5:9]))
            except ValueError:
                continue
        inside = [x for x in rows if self.t0 and self.t1 and self.t0 <= x[0] <= self.t1]
        use = inside or rows
        if not use:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({names[i] for x in use for i, v in enumerate(x[3]) if v == "Active"})
        return {"sm_mhz": statistics.median(x[1] for x in use), "sm_max_mhz": max(x[2] for x in use),
                "reasons": reasons, "samples": len(use),
                "window": "timed region" if inside else "whole run (no sample inside the timed region)"}


# ---------------------------------------------------------------------------
# reference CPU step (the baseline; never the product path)
# ---------------------------------------------------------------------------
def _reference_model(path: str, kv_ctx: int):
    """The reference decode step on the host: compiled reference when built, else the port."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pyoracle
    if pyoracle.ref_available():
        return pyoracle.RefModel(path, max_ctx=kv_ctx), "reference"
    return pyoracle.OracleModel(path, max_ctx=kv_ctx), "port"


def _time_reference(path: str, wl: Workload, kv_ctx: int, warm: int, n_max: int, budget_s: float):
    """Decode steps of the reference on the host, at the positions the b200
    arm decodes: a K/V pre-fill of the prompt's positions [0, P), `warm`
    untimed steps at P.., then up to n_max timed steps (fewer if budget_s runs
    out).  The prompt's K/V rows are written directly (N(0,1) values) instead
    of running the prompt on the CPU (about an hour for the 8B model); each
    timed step then does the same weight streaming and the same attention
    length as the b200 arm's step at that position.
    Returns (tokens/s, steps timed, kind, seconds, first timed position)."""
    c, P = wl.cfg, wl.prompt
    ref, kind = _reference_model(path, kv_ctx)
    if wl.long:
        wl.kv_prefill(ref.kv_load)
    else:
        rng = np.random.default_rng(7)
        for layer in range(c.n_layer):
            k = rng.standard_normal((P, c.n_head_kv, c.head_dim), dtype=np.float32)
            v = rng.standard_normal((P, c.n_head_kv, c.head_dim), dtype=np.float32)
            ref.kv_load(layer, 0, k, v)
    tok, pos = int(wl.prompt_ids()[-1]), P
    for _ in range(warm):
        tok = int(np.argmax(ref.forward(tok, pos)))
        pos += 1
    first, n, t0 = pos, 0, time.perf_counter()
    while n < n_max:
        tok = int(np.argmax(ref.forward(tok, pos)))
        pos += 1
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    ref.close()
    return n / dt, n, kind, dt, first


def run_reference(args) -> None:
    """The reference's own CPU decode step on the b200 arm's workload: same
    model file, same K/V length, same warm-up count and decode positions."""
    rank, world, _ = _dist()
    if rank != 0:
        return
    wl = Workload(args.gpus, args.layers, args.workload)
    path = _model_path(args, wl)
    K, W = args.steps, args.warmup
    kv_ctx = _kv_ctx(wl, K, W)
    tps, n, kind, dt, first = _time_reference(path, wl, kv_ctx, W, K, args.ref_budget_s)
    sample = (f"{n} greedy decode steps of the {wl.cfg.name} model at positions {first}..{first + n - 1} "
              f"after a {wl.prompt}-position K/V pre-fill and {W} untimed warm-up steps"
              + ("" if n == K else f" ({K} requested, cut at the {args.ref_budget_s:.0f} s cap)"))
    line = {
        "metric": METRIC, "value": tps, "unit": UNIT, "n_gpus": args.gpus, "steps": n,
        "warmup": W, "ms_per_step": dt / n * 1e3, "higher_is_better": True,
        "scaling": "strong" if wl.tp else "weak",
        "vs_baseline": None, "dtype": "fp32", "data": "synthetic (seeded random weights and prompt)",
        "config": wl.config(args.gpus, K, W, kv_ctx), "impl": "reference",
        "cpu_baseline": {"value": tps, "unit": UNIT, "cores": 1, "kind": kind, "sample": sample,
                         "host_cores": os.cpu_count(),
                         "note": "the reference decode step is single-threaded by design"},
        "e2e": {"value": tps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# the B200 arm
# ---------------------------------------------------------------------------
def run_b200(args) -> None:
    import torch
    import torch.distributed as dist

    from fwb import tp
    from fwb.model import Model

    rank, world, local = _dist()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    wl = Workload(world, args.layers, args.workload)
    torch.cuda.set_device(local)
    if world > 1:
        # host coordination only (IPC handles, barriers, the max over ranks):
        # the decode path's exchange runs over NVLink inside the kernel
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=1800))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    if rank == 0:
        path = _model_path(args, wl)
    barrier()
    if rank != 0:
        path = _model_path(args, wl)

    K, W = args.steps, args.warmup
    if K < 1 or W < 0:
        raise SystemExit("--steps must be >= 1 and --warmup >= 0")
    P = wl.prompt
    kv_ctx = _kv_ctx(wl, K, W)
    if kv_ctx > wl.cfg.n_ctx:
        raise SystemExit(f"--steps/--warmup need more than n_ctx {wl.cfg.n_ctx} positions")

    t_open = time.perf_counter()
    m = tp.open_model(path, kv_ctx, rank, world, local) if world > 1 else Model(path, max_ctx=kv_ctx, device=local)
    open_s = time.perf_counter() - t_open
    up_s, up_bytes = m.load_stats
    stream = torch.cuda.ExternalStream(m.stream, device=torch.device(f"cuda:{local}"))

    # prompt.  One GPU: fwb_prefill (the prompt's tokens through each layer
    # together on the tensor cores), once to warm up (scratch allocation) and
    # once timed; tensor parallel: one forward per token, as the reference's
    # main loop.
    prefill = None
    prompt = wl.prompt_ids()
    if wl.long:
        wl.kv_prefill(m.kv_load)
        tok = int(prompt[0])
    elif world == 1:
        m.prefill(prompt, 0)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        logits = m.prefill(prompt, 0)
        pf_s = time.perf_counter() - t0
        tok = int(np.argmax(logits))
        flops = 2.0 * wl.cfg.prefill_gemm_params() * (P - 1)
        prefill = {"tokens": P, "ms": pf_s * 1e3, "tokens_per_s": P / pf_s,
                   "gemm_tflops": flops / pf_s / 1e12,
                   "api": "fwb_prefill with host tokens and the last token's host logits (wall clock): "
                          "P-1 tokens through the tensor-core path (GEMMs on fp16 weight copies made at the first "
                          "call, tcgen05 attention), the last through the decode step"}
    else:
        tok = 0
        for i, t in enumerate(prompt):
            tok = m.forward_argmax(int(t), i)
    pos = P

    # warm-up
    if W:
        toks = m.generate_greedy(tok, pos, W)
        tok, pos = int(toks[-1]), pos + W
    torch.cuda.synchronize()

    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        time.sleep(1.0)  # let nvidia-smi start sampling

    # ---- device-timed greedy decode: K steps, weights resident in HBM ----
    pos_timed = pos
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    if clocks:
        clocks.mark_start()
    e0.record(stream)
    toks = m.generate_greedy(tok, pos, K)
    e1.record(stream)
    torch.cuda.synchronize()
    if clocks:
        clocks.mark_end()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1))
    tok, pos = int(toks[-1]), pos + K

    # ---- end to end through fwb_forward with host buffers (every rank gets
    # ---- the full logits and picks the same token), over the same positions
    # ---- as the device-timed pass (a few warm-up positions before them)
    logits = torch.empty(m.n_vocab, dtype=torch.float32, pin_memory=True).numpy()
    w2 = min(W, 3)
    pos = pos_timed - w2
    for _ in range(w2):  # first use of the pinned logits path
        m.forward(tok, pos, out=logits)
        tok, pos = int(np.argmax(logits)), pos + 1
    barrier()
    torch.cuda.synchronize()
    f0 = torch.cuda.Event(enable_timing=True)
    f1 = torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(K):
        m.forward(tok, pos, out=logits)
        tok, pos = int(np.argmax(logits)), pos + 1
    f1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms_e2e = max_over_ranks(f0.elapsed_time(f1))

    kernels = m.kernels_per_step
    weight_bytes = m.weight_bytes  # this rank's slices
    m.close()
    clk = clocks.finish() if clocks else None

    if rank == 0:
        peak, peak_kind = _peaks()
        # algorithmic bytes of one decode-kernel launch on one GPU at position
        # p: every weight byte of its slices once, its K/V rows 0..p once, the
        # new K/V row, its logits
        kvp = wl.kv_bytes_per_position(world)
        mean_pos = pos_timed + (K - 1) / 2.0
        step_bytes = weight_bytes + kvp * (mean_pos + 1) + kvp + 4 * wl.cfg.n_vocab // world
        launch_s = ms / 1e3 / K
        achieved = step_bytes / launch_s / 1e9
        line = {
            "metric": METRIC, "value": K / (ms / 1e3), "unit": UNIT, "n_gpus": world,
            "steps": K, "warmup": W, "ms_per_step": ms / K, "higher_is_better": True,
            "scaling": "strong" if wl.tp else "weak", "vs_baseline": None,
            "dtype": "q4_0 weights x 24-bit block fixed-point activations (three dp4a byte planes, exact "
                     "integer block sums), fp32 accumulate",
            "data": "synthetic (seeded random weights and prompt)",
            "config": wl.config(world, K, W, kv_ctx),
            "roofline": {
                "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "peak_source": f"hbm_gbs ({peak_kind})",
                "traffic": None if wl.tp or args.layers else _ncu_traffic()[0],
                "traffic_source": None if wl.tp or args.layers else _ncu_traffic()[1],
                "kernel": "decode_kernel (persistent, one launch per token" +
                          (", per GPU)" if wl.tp else ")"),
                "bytes_per_launch": step_bytes,
                "frac_weights_only": weight_bytes / launch_s / 1e9 / peak,
                "launch_time": "events over the K timed launches / K (includes the 8-byte "
                               "step-counter memset node of each graph)",
            },
            "e2e": {"value": K / (ms_e2e / 1e3), "unit": UNIT,
                    "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 4 * wl.cfg.n_vocab + 8,
                    "api": "fwb_forward (transformer_forward) with pinned host logits, host argmax"},
            "clocks": clk,
            "gpu_launches": kernels * K,
        }
        line["load"] = {"bytes": up_bytes, "upload_s": up_s, "gb_per_s": up_bytes / max(up_s, 1e-9) / 1e9,
                        "open_s": open_s,
                        "what": "fwb_model_open: tensor upload from the GGUF mapping (page cache) through pinned "
                                "staging filled by parallel host threads" + (", this rank's slices" if wl.tp else "")
                                + "; open_s adds parsing, allocation and the CUDA-graph capture"}
        if prefill:
            line["prefill"] = prefill
        if wl.tp:
            line["roofline"]["note"] = ("per GPU: its weight slices; the box-wide tokens/s is the value "
                                        "(one decode stream across all GPUs)")
        if world == 1 and not args.no_cpu_baseline:
            tps, n, kind, dt, first = _time_reference(path, wl, kv_ctx, 1, 1 << 30, args.cpu_budget_s)
            line["cpu_baseline"] = {
                "value": tps, "unit": UNIT, "cores": 1, "kind": kind, "host_cores": os.cpu_count(),
                "sample": f"{n} greedy decode steps of the same model at positions "
                          f"{first}..{first + n - 1} after a {P}-position K/V pre-fill and 1 "
                          f"warm-up step ({dt:.1f} s)"}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def _ncu_traffic():
    """DRAM bytes per decode-kernel launch, read from the committed ncu summary
    (not measured in this run: ncu cannot run inside the timed bench), with
    the summary's statement of which kernel source it was captured on."""
    p = os.path.join(ROOT, "profiles", "decode_kernel_8b_q4_0.md")
    val, src = None, None
    try:
        with open(p) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    val = float(line.split(":", 1)[1])
                if line.startswith("kernel_source:"):
                    src = line.split(":", 1)[1].strip()
    except OSError:
        pass
    if val is None:
        return None, None
    return val, f"from profiles/decode_kernel_8b_q4_0.md (ncu capture; {src or 'kernel source not stated'})"


def main() -> None:
    args = _args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
