"""CPU tests of the boundary: the C-ABI library loads and exports every
function include/forword_b200.h declares; host-side argument checks reject
bad calls the way the reference does (quant_matvec.c:270-289) without
touching a GPU; the GGUF writer produces files gguf-py reads back."""
import ctypes
import os
import re

import numpy as np
import pytest

from fwb import configs, gguf_synth, native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions(header: str) -> list[str]:
    src = open(header).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\(", src, flags=re.M)
    return sorted(set(n for n in names if n not in ("if", "defined")))


def test_header_symbols_exported(built):
    lib = ctypes.CDLL(native.PRODUCT_SO)
    names = declared_functions(os.path.join(ROOT, "include", "forword_b200.h"))
    assert "quant_matvec" in names and "fwb_model_open" in names
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_all_headers_symbols_exported(built):
    """Every function declared in any include/*.h is exported by the library."""
    lib = ctypes.CDLL(native.PRODUCT_SO)
    for h in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if not h.endswith(".h"):
            continue
        for n in declared_functions(os.path.join(ROOT, "include", h)):
            assert hasattr(lib, n), f"{h}: {n} not exported"


def test_product_has_no_oracle_dependency(built):
    """The product library links neither oracle library nor any reference object."""
    import subprocess
    out = subprocess.run(["ldd", native.PRODUCT_SO], capture_output=True, text=True).stdout
    assert "oracle" not in out and "forword_ref" not in out
    syms = subprocess.run(["nm", "-D", "--defined-only", native.PRODUCT_SO], capture_output=True,
                          text=True).stdout
    assert "orc_" not in syms and "refh_" not in syms


@pytest.mark.parametrize("args,why", [
    ((None, 1024, 2, True, True, 32, 1), "null weights"),
    ((b"x" * 1024, 1024, 2, False, True, 32, 1), "null input"),
    ((b"x" * 1024, 1024, 2, True, True, 0, 1), "zero input size"),
    ((b"x" * 1024, 1024, 2, True, True, 32, 0), "zero output size"),
    ((b"x" * 1024, 1024, 12, True, True, 256, 1), "unsupported type (Q4_K)"),
    ((b"x" * 1024, 1024, 2, True, True, 48, 1), "input not a multiple of 32"),
    ((b"x" * 17, 17, 2, True, True, 32, 1), "weights too small"),
])
def test_quant_matvec_rejects_bad_arguments(built, args, why):
    """Rejected before any device work, so this runs without a GPU."""
    lib = native.product()
    w, wsz, t, has_x, has_y, n_in, n_out = args
    x = (ctypes.c_float * max(n_in, 1))() if has_x else None
    y = (ctypes.c_float * max(n_out, 1))() if has_y else None
    wp = ctypes.c_char_p(w) if w is not None else None
    rc = lib.quant_matvec(wp, wsz, t, x, y, n_in, n_out)
    assert rc == -1, why
    assert lib.fwb_last_error().decode()


def test_model_open_missing_file_fails_cleanly(built):
    lib = native.product()
    assert not lib.fwb_model_open(b"/nonexistent/model.gguf", 0, 0)
    assert lib.fwb_last_error().decode()
    lib.fwb_model_close(None)  # NULL accepted, like transformer_free


def test_synthetic_gguf_reads_back_with_gguf_py(built, model_dir):
    import gguf
    cfg = configs.SMALL_MIXED
    path = gguf_synth.write_model(os.path.join(model_dir, "rb.gguf"), cfg, seed=9)
    r = gguf.GGUFReader(path)
    names = {t.name: t for t in r.tensors}
    assert len(names) == len(gguf_synth.tensor_plan(cfg))
    t = names["blk.0.ffn_gate.weight"]
    assert int(t.tensor_type) == cfg.t_gate and list(t.shape) == [cfg.n_embd, cfg.n_ff]
    t = names["blk.1.attn_k.weight"]
    assert int(t.tensor_type) == cfg.t_k and list(t.shape) == [cfg.n_embd, cfg.n_head_kv * cfg.head_dim]
    # dequantised bytes of one tensor through gguf-py equal the oracle's decode
    import pyoracle
    t = names["blk.0.attn_q.weight"]
    raw = np.asarray(t.data).reshape(-1).view(np.uint8)
    ours = pyoracle.dequant(np.ascontiguousarray(raw), cfg.t_q, cfg.n_embd * cfg.n_embd)
    theirs = gguf.quants.dequantize(raw.reshape(1, -1), gguf.GGMLQuantizationType(cfg.t_q)).reshape(-1)
    assert np.array_equal(ours, theirs.astype(np.float32))
    f = r.fields
    assert bytes(f["general.architecture"].parts[-1]).decode() == "llama"
    assert int(f["llama.attention.head_count_kv"].parts[-1][0]) == cfg.n_head_kv


def test_synth_is_deterministic_across_row_splits(built):
    lib = native.synth_lib()
    rows, cols = 64, 256
    a = gguf_synth.random_matrix(configs.Q4_0, rows, cols, seed=3, mode=0, lo=0.0, hi=0.02)
    b = np.empty_like(a)
    rb = cols // 32 * 18
    key = gguf_synth.tensor_key(3, f"matrix{configs.Q4_0}x{rows}x{cols}")
    for r0 in range(0, rows, 7):
        r1 = min(rows, r0 + 7)
        lib.fwb_synth_fill(ctypes.c_void_p(b.ctypes.data + r0 * rb), configs.Q4_0, cols, r0, r1, key,
                           0.0, 0.02, 0)
    assert np.array_equal(a, b)


def test_weight_bytes_formula():
    c = configs.LLAMA8B_Q4_0
    # 4.2214 GB of Q4_0 weights incl. the 0.2955 GB head (algorithmic bytes per token)
    assert abs(c.weight_bytes_per_token() / 1e9 - 4.2214) < 0.01


def test_prefill_gemm_params_formula():
    """Weights a prompt token multiplies in fwb_prefill's GEMMs: QKV in every
    layer, o-proj and the FFN in all layers but the last."""
    c = configs.LLAMA8B_Q4_0
    E, F, hd = c.n_embd, c.n_ff, c.head_dim
    q, kv = c.n_head * hd, c.n_head_kv * hd
    want = 32 * (q + 2 * kv) * E + 31 * (q * E + 3 * E * F)
    assert c.prefill_gemm_params() == want
    assert abs(2 * want / 1e9 - 13.57) < 0.01  # GFLOP per prompt token
