"""Seeded synthetic GGUF (v3) writer for the benchmark and test models.

The container follows the GGUF v3 layout forword.c's gguf.c:256-353 parses:
header, metadata key/values, tensor descriptors (dims[0] = input width,
dims[1] = rows), data section aligned to 32 bytes, each tensor 32-aligned.
Tensor bytes come from libfwb_synth.so (synth.c), a pure function of
(seed, tensor name, element index).

The metadata carries what model_config.c reads for arch "llama" and a
``tokenizer.ggml.tokens`` list (tokenizer.c:191-195 refuses a model without
one): <unk> <s> </s>, the 256 byte tokens <0x00>..<0xFF>, then filler pieces.
"""
from __future__ import annotations

import ctypes
import hashlib
import os
import struct

import numpy as np

from . import native
from .configs import F32, ModelShape, quant_bytes

ALIGN = 32
_GGUF_MAGIC = 0x46554747
_T_U32, _T_F32, _T_STR, _T_ARR = 4, 6, 8, 9


def tensor_key(seed: int, name: str) -> int:
    h = hashlib.blake2b(name.encode(), digest_size=8).digest()
    return (int.from_bytes(h, "little") ^ (seed * 0x9E3779B97F4A7C15)) & (2**64 - 1)


def _s(b: bytearray, s: str) -> None:
    e = s.encode()
    b += struct.pack("<Q", len(e)) + e


def _kv_u32(b, k, v):
    _s(b, k); b += struct.pack("<II", _T_U32, v)


def _kv_f32(b, k, v):
    _s(b, k); b += struct.pack("<If", _T_F32, v)


def _kv_str(b, k, v):
    _s(b, k); b += struct.pack("<I", _T_STR); _s(b, v)


def _kv_str_arr(b, k, items):
    _s(b, k); b += struct.pack("<IIQ", _T_ARR, _T_STR, len(items))
    for it in items:
        _s(b, it)


def vocab_tokens(n: int) -> list[str]:
    base = ["<unk>", "<s>", "</s>"] + [f"<0x{i:02X}>" for i in range(256)]
    toks = base[:n]
    toks += [f"▁t{i}" for i in range(len(toks), n)]
    return toks


def tensor_plan(cfg: ModelShape) -> list[tuple[str, int, int, int, str]]:
    """(name, ggml type, rows, cols, role) in file order; cols = dims[0]."""
    E, F, hd = cfg.n_embd, cfg.n_ff, cfg.head_dim
    plan = [("token_embd.weight", cfg.t_embd, cfg.n_vocab, E, "w")]
    for l in range(cfg.n_layer):
        p = f"blk.{l}."
        plan += [
            (p + "attn_norm.weight", F32, 1, E, "norm"),
            (p + "attn_q.weight", cfg.t_q, cfg.n_head * hd, E, "w"),
            (p + "attn_k.weight", cfg.t_k, cfg.n_head_kv * hd, E, "w"),
            (p + "attn_v.weight", cfg.t_v, cfg.n_head_kv * hd, E, "w"),
            (p + "attn_output.weight", cfg.t_o, E, cfg.n_head * hd, "w"),
            (p + "ffn_norm.weight", F32, 1, E, "norm"),
            (p + "ffn_gate.weight", cfg.t_gate, F, E, "w"),
            (p + "ffn_up.weight", cfg.t_up, F, E, "w"),
            (p + "ffn_down.weight", cfg.t_down, E, F, "w"),
        ]
    if cfg.out_norm:
        plan.append(("output_norm.weight", F32, 1, E, "norm"))
    if not cfg.tied:
        plan.append(("output.weight", cfg.t_out, cfg.n_vocab, E, "w"))
    return plan


def _nbytes(t: int, rows: int, cols: int) -> int:
    return quant_bytes(t, rows * cols)


def write_model(path: str, cfg: ModelShape, seed: int = 1234) -> str:
    """Write cfg as a GGUF file at path (overwrites).  Returns path."""
    lib = native.synth_lib()
    meta = bytearray()
    kvs = []
    a = "llama"
    kvs.append(lambda b: _kv_str(b, "general.architecture", a))
    kvs.append(lambda b: _kv_str(b, "general.name", cfg.name))
    kvs.append(lambda b: _kv_u32(b, "general.alignment", ALIGN))
    kvs.append(lambda b: _kv_u32(b, f"{a}.context_length", cfg.n_ctx))
    kvs.append(lambda b: _kv_u32(b, f"{a}.embedding_length", cfg.n_embd))
    kvs.append(lambda b: _kv_u32(b, f"{a}.block_count", cfg.n_layer))
    kvs.append(lambda b: _kv_u32(b, f"{a}.feed_forward_length", cfg.n_ff))
    kvs.append(lambda b: _kv_u32(b, f"{a}.attention.head_count", cfg.n_head))
    kvs.append(lambda b: _kv_u32(b, f"{a}.attention.head_count_kv", cfg.n_head_kv))
    kvs.append(lambda b: _kv_f32(b, f"{a}.attention.layer_norm_rms_epsilon", cfg.eps))
    kvs.append(lambda b: _kv_f32(b, f"{a}.rope.freq_base", cfg.rope_base))
    kvs.append(lambda b: _kv_u32(b, f"{a}.rope.dimension_count", cfg.head_dim))
    kvs.append(lambda b: _kv_str(b, "tokenizer.ggml.model", "llama"))
    kvs.append(lambda b: _kv_str_arr(b, "tokenizer.ggml.tokens", vocab_tokens(cfg.n_vocab)))
    kvs.append(lambda b: _kv_u32(b, "tokenizer.ggml.bos_token_id", 1))
    kvs.append(lambda b: _kv_u32(b, "tokenizer.ggml.eos_token_id", 2))
    for f in kvs:
        f(meta)

    plan = tensor_plan(cfg)
    infos = bytearray()
    offsets = []
    off = 0
    for name, t, rows, cols, _ in plan:
        offsets.append(off)
        _s(infos, name)
        if rows == 1:
            infos += struct.pack("<IQ", 1, cols)
        else:
            infos += struct.pack("<IQQ", 2, cols, rows)
        infos += struct.pack("<IQ", t, off)
        off += _nbytes(t, rows, cols)
        off = (off + ALIGN - 1) // ALIGN * ALIGN
    header = struct.pack("<IIQQ", _GGUF_MAGIC, 3, len(plan), len(kvs))
    pre = header + bytes(meta) + bytes(infos)
    data_off = (len(pre) + ALIGN - 1) // ALIGN * ALIGN
    total = data_off + off

    with open(path, "wb") as fh:
        fh.truncate(total)
        fh.write(pre)
    mm = np.memmap(path, dtype=np.uint8, mode="r+", offset=0, shape=(total,))
    base = mm.ctypes.data
    for (name, t, rows, cols, role), o in zip(plan, offsets):
        key = tensor_key(seed, name)
        dst = ctypes.c_void_p(base + data_off + o)
        if role == "norm":
            rc = lib.fwb_synth_fill(dst, F32, cols, 0, 1, key, 1.0, cfg.norm_sd, 0)
        else:
            rc = lib.fwb_synth_fill(dst, t, cols, 0, rows, key, 0.0, cfg.weight_sd, 0)
        if rc != 0:
            raise RuntimeError(f"synth fill failed for {name}")
    mm.flush()
    del mm
    return path


def cached_model(cfg: ModelShape, seed: int = 1234, directory: str | None = None) -> str:
    """Path of cfg's GGUF under directory (default $FWB_MODEL_DIR or /tmp),
    written once per (cfg, seed)."""
    d = directory or os.environ.get("FWB_MODEL_DIR", "/tmp/fwb_models")
    os.makedirs(d, exist_ok=True)
    path = os.path.join(d, f"{cfg.name}-s{seed}.gguf")
    stamp = path + ".ok"
    if not (os.path.exists(path) and os.path.exists(stamp)):
        write_model(path, cfg, seed)
        with open(stamp, "w") as f:
            f.write("ok\n")
    return path


def random_matrix(t: int, rows: int, cols: int, seed: int, mode: int = 1,
                  lo: float = 1e-3, hi: float = 1e-2) -> np.ndarray:
    """Standalone weight matrix bytes (microbench / unit tests).
    mode 1: uniform quants and d ~ U(lo, hi); mode 0: N(lo, hi) quantised."""
    lib = native.synth_lib()
    n = _nbytes(t, rows, cols)
    buf = np.empty(n, dtype=np.uint8)
    rc = lib.fwb_synth_fill(ctypes.c_void_p(buf.ctypes.data), t, cols, 0, rows,
                            tensor_key(seed, f"matrix{t}x{rows}x{cols}"), lo, hi, mode)
    if rc != 0:
        raise ValueError("bad synth arguments")
    return buf


def kv_prefill_values(cfg: ModelShape, layer: int, n: int, seed: int) -> tuple[np.ndarray, np.ndarray]:
    """K and V rows [n][n_head_kv][head_dim] of one layer for a K/V cache
    pre-fill: N(0, 1) rounded to fp16 (benchmark configuration 4), seeded
    per (seed, layer)."""
    rng = np.random.default_rng(seed * 1000 + layer)
    shape = (n, cfg.n_head_kv, cfg.head_dim)
    k = rng.standard_normal(shape).astype(np.float16).astype(np.float32)
    v = rng.standard_normal(shape).astype(np.float16).astype(np.float32)
    return k, v


def normal_vector(n: int, seed: int, mean: float = 0.0, sd: float = 1.0) -> np.ndarray:
    lib = native.synth_lib()
    out = np.empty(n, dtype=np.float32)
    lib.fwb_synth_normal(ctypes.c_void_p(out.ctypes.data), n, tensor_key(seed, "vector"),
                         mean, sd)
    return out


def main(argv: list[str] | None = None) -> None:
    """python -m fwb.gguf_synth CONFIG SEED [DIR]: write (once) the cached
    synthetic model and print its path.  Run as its own process so that a
    caller timing the reference never loads the generator library."""
    import argparse
    from .configs import CONFIGS, with_layers
    p = argparse.ArgumentParser(description=main.__doc__.split("\n")[0])
    p.add_argument("config")
    p.add_argument("seed", type=int)
    p.add_argument("directory", nargs="?", default=None)
    p.add_argument("--layers", type=int, default=0, help="keep only the first N layers (0: all)")
    a = p.parse_args(argv)
    cfg = CONFIGS[a.config]
    if a.layers:
        cfg = with_layers(cfg, a.layers)
    print(cached_model(cfg, seed=a.seed, directory=a.directory))


def cached_model_subprocess(cfg_name: str, seed: int, directory: str | None = None, layers: int = 0) -> str:
    """cached_model in a child process (see main); returns the path."""
    import subprocess
    import sys
    pkg = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    cmd = [sys.executable, "-m", "fwb.gguf_synth", cfg_name, str(seed)]
    if directory:
        cmd.append(directory)
    if layers:
        cmd += ["--layers", str(layers)]
    out = subprocess.run(cmd, check=True, capture_output=True, text=True, cwd=pkg)
    return out.stdout.strip().splitlines()[-1]


if __name__ == "__main__":
    main()
