"""Generate the committed golden fixtures of tests/golden/.

Run in a container that has the reference sources (for oracle/_ref) and the
gguf-py package:  python tests/golden/make_golden.py

quant_gguf_py.npz
    Q4_0 / Q5_0 / Q8_0 blocks quantised by gguf-py (llama.cpp's gguf-py
    0.19.0, gguf.quants.quantize) from seeded normals, plus hand-made blocks
    with special fp16 scales (subnormal, negative, zero, large), and gguf-py's
    own dequantisation of every block.  Pins the Q4_0 restatement (the
    reference has no Q4_0 decoder) and the Q5_0 / Q8_0 decoders against an
    independent implementation of the GGML formats.

ref_full_<model>.npz   (python tests/golden/make_golden.py full <model>)
    The compiled reference at the benchmark configurations, full depth: the
    Llama-3-8B-shaped Q4_0 model (the bench's model: same seed), the 8B mixed
    Q8_0/Q5_0 model after an 8000-position K/V pre-fill (fp16-rounded N(0,1),
    prefill_kv), and the first 8 layers of the Llama-70B-shaped Q4_0 model
    with its full 128256-entry vocabulary.  An 8-token seeded prompt goes
    through transformer_forward one token at a time, then 64 greedy steps.
    Stored: the model's sha256, the prompt, the 64 greedy tokens, per step
    the 32 largest logits (index and value) and the logits' L2 norm, and the
    full logits row at steps 0, 31 and 63.  Each model takes minutes to
    hours of single-threaded reference time.

ref_decode_<model>.npz
    The compiled reference's own transformer_forward (oracle/_ref) on seeded
    synthetic GGUFs: the sha256 of the model bytes, the greedy token stream
    and the logits of every step.  For Q4_0 the reference runs with the
    patch-free Q4_0 add-on of oracle/ref_q4_0_addon.c.  The `kvprefill`
    variant first writes fp16-rounded N(0,1) K/V into positions [0, 96)
    through the reference's kv_k / kv_v.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "forword.c_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

from fwb import configs, gguf_synth  # noqa: E402

GOLDEN_MODELS = {
    "tied_q8_0": (configs.SMALL_TIED_Q8, 11),
    "mixed": (configs.SMALL_MIXED, 12),
    "q4_0": (configs.SMALL_Q4_0, 13),
}
STEPS = 24
FIRST_TOKEN = 7
PREFILL = 96


def sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def prefill_kv(cfg, layer: int, n: int, seed: int):
    return gguf_synth.kv_prefill_values(cfg, layer, n, seed)


def make_quant():
    import gguf
    from gguf import quants
    rng = np.random.default_rng(2024)
    out = {}
    for name, t in (("q4_0", gguf.GGMLQuantizationType.Q4_0),
                    ("q5_0", gguf.GGMLQuantizationType.Q5_0),
                    ("q8_0", gguf.GGMLQuantizationType.Q8_0)):
        x = (rng.standard_normal((64, 256)) * rng.uniform(1e-4, 10.0, (64, 1))).astype(np.float32)
        q = np.ascontiguousarray(quants.quantize(x, t)).reshape(-1)
        bb = {"q4_0": 18, "q5_0": 22, "q8_0": 34}[name]
        blocks = q.reshape(-1, bb).copy()
        # special fp16 scales: subnormal, negative, zero, large, max normal
        for i, d in enumerate((0x0001, 0x03FF, 0xBC00, 0x0000, 0x7BFF, 0x3C00)):
            blocks[i, 0] = d & 0xFF
            blocks[i, 1] = d >> 8
        raw = blocks.reshape(-1)
        deq = quants.dequantize(raw.reshape(1, -1), t).reshape(-1).astype(np.float32)
        out[name + "_bytes"] = raw
        out[name + "_deq"] = deq
    np.savez_compressed(os.path.join(HERE, "quant_gguf_py.npz"), **out)


def make_decode(tmp: str):
    import pyoracle
    for tag, (cfg, seed) in GOLDEN_MODELS.items():
        path = gguf_synth.write_model(os.path.join(tmp, f"{tag}.gguf"), cfg, seed=seed)
        for variant in ("plain", "kvprefill"):
            ref = pyoracle.RefModel(path, 0)
            pos0 = 0
            if variant == "kvprefill":
                for layer in range(cfg.n_layer):
                    k, v = prefill_kv(cfg, layer, PREFILL, seed)
                    ref.kv_load(layer, 0, k, v)
                pos0 = PREFILL
            tok = FIRST_TOKEN
            toks, logits = [], []
            for i in range(STEPS):
                lg = ref.forward(tok, pos0 + i)
                logits.append(lg)
                tok = int(np.argmax(lg))
                toks.append(tok)
            ref.close()
            np.savez_compressed(os.path.join(HERE, f"ref_decode_{tag}_{variant}.npz"),
                                sha256=np.array(sha256(path)), seed=np.array(seed),
                                first=np.array(FIRST_TOKEN), pos0=np.array(pos0),
                                tokens=np.array(toks, np.uint32), logits=np.stack(logits))


# full-depth models of the benchmark configurations: (shape, seed, K/V
# pre-fill positions, kv_ctx)
FULL_MODELS = {
    "llama8b_q4_0": (configs.LLAMA8B_Q4_0, 1, 0, 128),
    "llama8b_mixed": (configs.LLAMA8B_MIXED, 1, 8000, 8192),
    "llama70b_q4_0_8layer": (configs.with_layers(configs.LLAMA70B_Q4_0, 8), 1, 0, 128),
}
FULL_PROMPT = 8
FULL_STEPS = 64
FULL_TOPK = 32
FULL_ROWS = (0, 31, 63)  # steps whose whole logits row is stored


def full_prompt(cfg, seed: int) -> np.ndarray:
    return np.random.default_rng(seed + 77).integers(0, cfg.n_vocab, FULL_PROMPT).astype(np.uint32)


def topk(lg: np.ndarray, k: int = FULL_TOPK) -> tuple[np.ndarray, np.ndarray]:
    """Indices (value descending, index ascending on ties) and values."""
    idx = np.lexsort((np.arange(lg.size), -lg.astype(np.float64)))[:k]
    return idx.astype(np.uint32), lg[idx]


def make_full(tag: str, directory: str) -> str:
    """Golden of one full-depth model (see the module docstring)."""
    import pyoracle
    cfg, seed, n_pre, kv_ctx = FULL_MODELS[tag]
    path = gguf_synth.cached_model(cfg, seed=seed, directory=directory)
    ref = pyoracle.RefModel(path, kv_ctx)
    for layer in range(cfg.n_layer if n_pre else 0):
        k, v = prefill_kv(cfg, layer, n_pre, seed)
        ref.kv_load(layer, 0, k, v)
    prompt = full_prompt(cfg, seed)
    pos = n_pre
    for t in prompt[:-1]:
        ref.forward(int(t), pos)
        pos += 1
    tok = int(prompt[-1])
    toks, tidx, tval, norms, rows = [], [], [], [], []
    for i in range(FULL_STEPS):
        lg = ref.forward(tok, pos + i)
        a, b = topk(lg)
        tidx.append(a)
        tval.append(b)
        norms.append(np.linalg.norm(lg.astype(np.float64)))
        if i in FULL_ROWS:
            rows.append(lg.copy())
        tok = int(np.argmax(lg))
        toks.append(tok)
        print(f"{tag}: step {i} token {tok}", flush=True)
    ref.close()
    out = os.path.join(HERE, f"ref_full_{tag}.npz")
    np.savez_compressed(out, sha256=np.array(sha256(path)), seed=np.array(seed), n_prefill=np.array(n_pre),
                        kv_ctx=np.array(kv_ctx), prompt=prompt, pos_first=np.array(pos),
                        tokens=np.array(toks, np.uint32), top_idx=np.stack(tidx), top_val=np.stack(tval),
                        norm=np.array(norms), row_steps=np.array(FULL_ROWS), rows=np.stack(rows))
    return out


if __name__ == "__main__":
    import tempfile
    if len(sys.argv) > 2 and sys.argv[1] == "full":
        print("written", make_full(sys.argv[2], sys.argv[3] if len(sys.argv) > 3 else "/tmp/fwb_models"))
        sys.exit(0)
    make_quant()
    with tempfile.TemporaryDirectory() as tmp:
        make_decode(tmp)
    print("golden fixtures written to", HERE)
