"""ctypes access to the oracle libraries — TEST INFRASTRUCTURE ONLY.

Used by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg as the
checker / baseline; the product never imports this module.

  Oracle     oracle/_build/liboracle.so   (my C restatement, fwd_oracle.c)
  Reference  oracle/_ref/libforword_ref.so (forword.c compiled from its own
             sources + the patch-free Q4_0 add-on; present only where it was
             built, travels to the GPU box as a prebuilt file)
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libforword_ref.so")
REF_UNIT_TEST = os.path.join(HERE, "_ref", "unit-test")
REF_CLI = os.path.join(HERE, "_ref", "forword")

_c = ctypes
_fp = _c.POINTER(_c.c_float)
_oracle = None
_ref = None


def build(ref: bool = False) -> None:
    subprocess.run(["make", "-C", HERE, "oracle"], check=True, capture_output=True)
    if ref:
        subprocess.run(["make", "-C", HERE, "ref"], check=True, capture_output=True)


def oracle_lib():
    global _oracle
    if _oracle is None:
        if not os.path.exists(ORACLE_SO):
            build()
        lib = _c.CDLL(ORACLE_SO)
        lib.orc_open.argtypes = [_c.POINTER(_c.c_void_p), _c.c_char_p, _c.c_size_t]
        lib.orc_open.restype = _c.c_int
        lib.orc_close.argtypes = [_c.c_void_p]
        lib.orc_forward.argtypes = [_c.c_void_p, _c.c_uint32, _c.c_size_t, _fp]
        lib.orc_forward.restype = _c.c_int
        lib.orc_dims.argtypes = [_c.c_void_p, _c.POINTER(_c.c_uint32)]
        lib.orc_kv_write.argtypes = [_c.c_void_p, _c.c_size_t, _c.c_size_t, _c.c_size_t, _fp, _fp]
        lib.orc_kv_read.argtypes = [_c.c_void_p, _c.c_size_t, _c.c_size_t, _c.c_size_t, _fp, _fp]
        lib.orc_quant_matvec.argtypes = [_c.c_void_p, _c.c_size_t, _c.c_uint32, _fp, _fp,
                                         _c.c_size_t, _c.c_size_t]
        lib.orc_dequant.argtypes = [_c.c_void_p, _c.c_size_t, _c.c_uint32, _fp, _c.c_size_t]
        lib.orc_f16_to_f32.argtypes = [_c.c_uint16]
        lib.orc_f16_to_f32.restype = _c.c_float
        lib.orc_dot.argtypes = [_fp, _fp, _c.c_size_t]
        lib.orc_dot.restype = _c.c_float
        lib.orc_rms_norm.argtypes = [_fp, _fp, _fp, _c.c_size_t, _c.c_float]
        lib.orc_rope_tables.argtypes = [_fp, _fp, _c.c_size_t, _c.c_size_t, _c.c_float]
        lib.orc_rope_apply.argtypes = [_fp, _c.c_size_t, _c.c_size_t, _c.c_size_t, _fp, _fp]
        lib.orc_argmax.argtypes = [_fp, _c.c_size_t]
        lib.orc_argmax.restype = _c.c_uint32
        _oracle = lib
    return _oracle


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref_lib():
    global _ref
    if _ref is None:
        lib = _c.CDLL(REF_SO)
        lib.refh_open.argtypes = [_c.c_char_p, _c.c_size_t]
        lib.refh_open.restype = _c.c_void_p
        lib.refh_close.argtypes = [_c.c_void_p]
        lib.refh_forward.argtypes = [_c.c_void_p, _c.c_uint32, _c.c_size_t, _fp]
        lib.refh_forward.restype = _c.c_int
        lib.refh_argmax.argtypes = [_c.c_void_p]
        lib.refh_argmax.restype = _c.c_uint32
        lib.refh_dims.argtypes = [_c.c_void_p, _c.POINTER(_c.c_uint32)]
        lib.refh_kv_write.argtypes = [_c.c_void_p, _c.c_size_t, _c.c_size_t, _c.c_size_t, _fp, _fp]
        lib.refh_kv_write.restype = _c.c_int
        lib.refh_kv_read.argtypes = [_c.c_void_p, _c.c_size_t, _c.c_size_t, _c.c_size_t, _fp, _fp]
        lib.refh_config.argtypes = [_c.c_char_p, _c.POINTER(_c.c_uint32), _fp]
        lib.refh_config.restype = _c.c_int
        lib.refh_quant_matvec.argtypes = [_c.c_void_p, _c.c_size_t, _c.c_uint32, _fp, _fp,
                                          _c.c_size_t, _c.c_size_t]
        lib.refh_quant_matvec.restype = _c.c_int
        _ref = lib
    return _ref


def _f(a: np.ndarray):
    return a.ctypes.data_as(_fp)


class _Base:
    dims: list

    @property
    def n_vocab(self):
        return self.dims[0]

    @property
    def kv_ctx(self):
        return self.dims[1]

    @property
    def n_layer(self):
        return self.dims[3]

    @property
    def n_head_kv(self):
        return self.dims[5]

    @property
    def head_dim(self):
        return self.dims[7]


class OracleModel(_Base):
    """My restatement (fwd_oracle.c) of transformer_forward."""

    def __init__(self, path: str, max_ctx: int = 0):
        self.lib = oracle_lib()
        self.h = _c.c_void_p()
        if self.lib.orc_open(_c.byref(self.h), path.encode(), max_ctx) != 0:
            raise RuntimeError(f"oracle cannot open {path}")
        d = (_c.c_uint32 * 8)()
        self.lib.orc_dims(self.h, d)
        self.dims = list(d)

    def forward(self, token: int, pos: int) -> np.ndarray:
        out = np.zeros(self.n_vocab, dtype=np.float32)
        if self.lib.orc_forward(self.h, token, pos, _f(out)) != 0:
            raise RuntimeError("oracle forward failed")
        return out

    def kv_load(self, layer, pos0, k, v):
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        assert self.lib.orc_kv_write(self.h, layer, pos0, k.shape[0], _f(k), _f(v)) == 0

    def close(self):
        if self.h:
            self.lib.orc_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class RefModel(_Base):
    """The compiled reference's own transformer_init / transformer_forward."""

    def __init__(self, path: str, max_ctx: int = 0):
        self.lib = ref_lib()
        self.h = self.lib.refh_open(path.encode(), max_ctx)
        if not self.h:
            raise RuntimeError(f"reference cannot open {path}")
        d = (_c.c_uint32 * 8)()
        self.lib.refh_dims(self.h, d)
        self.dims = list(d)

    def forward(self, token: int, pos: int) -> np.ndarray:
        out = np.zeros(self.n_vocab, dtype=np.float32)
        if self.lib.refh_forward(self.h, token, pos, _f(out)) != 0:
            raise RuntimeError("reference forward failed")
        return out

    def kv_load(self, layer, pos0, k, v):
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        assert self.lib.refh_kv_write(self.h, layer, pos0, k.shape[0], _f(k), _f(v)) == 0

    def close(self):
        if self.h:
            self.lib.refh_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def quant_matvec(w: np.ndarray, t: int, x: np.ndarray, n_out: int, use_ref: bool = False) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.zeros(n_out, np.float32)
    if use_ref:
        rc = ref_lib().refh_quant_matvec(w.ctypes.data, w.nbytes, t, _f(x), _f(y), x.size, n_out)
    else:
        rc = oracle_lib().orc_quant_matvec(w.ctypes.data, w.nbytes, t, _f(x), _f(y), x.size, n_out)
    if rc != 0:
        raise RuntimeError("oracle quant_matvec rejected its arguments")
    return y


_REF_DECODERS = {7: "q5_1_decode", 8: "q8_0_decode", 12: "q4_k_decode", 14: "q6_k_decode"}
_REF_BLOCK = {7: (32, 24), 8: (32, 34), 12: (256, 144), 14: (256, 210)}


def ref_dequant(w: np.ndarray, t: int, n: int) -> np.ndarray:
    """n values of type t decoded by the compiled reference's own decoders
    (quant.c: q5_1_decode, q8_0_decode, q4_k_decode, q6_k_decode)."""
    lib = ref_lib()
    fn = getattr(lib, _REF_DECODERS[t])
    fn.argtypes = [_c.c_void_p, _c.c_size_t, _fp, _c.c_size_t]
    fn.restype = _c.c_int
    bv, bb = _REF_BLOCK[t]
    nbytes = n // bv * bb
    src = np.ascontiguousarray(w[:nbytes])
    out = np.zeros(n, np.float32)
    if fn(src.ctypes.data, nbytes, _f(out), n) != 0:
        raise RuntimeError("reference decoder rejected its arguments")
    return out


def dequant(w: np.ndarray, t: int, n: int) -> np.ndarray:
    out = np.zeros(n, np.float32)
    if oracle_lib().orc_dequant(w.ctypes.data, w.nbytes, t, _f(out), n) != 0:
        raise RuntimeError("oracle dequant rejected its arguments")
    return out
