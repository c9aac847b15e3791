"""Locating and loading the native libraries (ctypes).

``product()``   lib/libforword_b200.so — the CUDA library behind the C ABI of
                include/forword_b200.h.  There is no CPU fallback: if the
                library is missing this raises.
``synth_lib()`` fwb/_build/libfwb_synth.so — synthetic model generator.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))  # forword.c_b200/
REPO = os.path.dirname(PKG_DIR)
PRODUCT_SO = os.path.join(PKG_DIR, "lib", "libforword_b200.so")
SYNTH_SO = os.path.join(PKG_DIR, "fwb", "_build", "libfwb_synth.so")

_c = ctypes
_vp, _sz, _u32, _i32, _u64 = _c.c_void_p, _c.c_size_t, _c.c_uint32, _c.c_int, _c.c_uint64
_fp = _c.POINTER(_c.c_float)

_synth = None
_product = None


def build(target: str = "all") -> None:
    subprocess.run(["make", "-C", PKG_DIR, target, "-j8"], check=True)


def synth_lib():
    global _synth
    if _synth is None:
        if not os.path.exists(SYNTH_SO):
            build("synth")
        lib = _c.CDLL(SYNTH_SO)
        lib.fwb_synth_fill.argtypes = [_vp, _u32, _u64, _u64, _u64, _u64, _c.c_float,
                                       _c.c_float, _i32]
        lib.fwb_synth_fill.restype = _i32
        lib.fwb_synth_normal.argtypes = [_vp, _u64, _u64, _c.c_float, _c.c_float]
        lib.fwb_synth_normal.restype = None
        _synth = lib
    return _synth


def product():
    """The CUDA product library.  Raises if it has not been built."""
    global _product
    if _product is None:
        if not os.path.exists(PRODUCT_SO):
            raise RuntimeError(f"{PRODUCT_SO} is missing: build it with "
                               f"`make -C {PKG_DIR}` (there is no CPU fallback)")
        lib = _c.CDLL(PRODUCT_SO)
        _declare(lib)
        _product = lib
    return _product


def _declare(lib) -> None:
    def sig(name, res, *args):
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = list(args)

    sig("fwb_last_error", _c.c_char_p)
    sig("fwb_device_count", _i32)
    sig("quant_matvec", _i32, _vp, _sz, _u32, _fp, _fp, _sz, _sz)
    sig("quant_matvec_dev", _i32, _vp, _sz, _u32, _vp, _vp, _sz, _sz, _vp)
    sig("quant_gemm_dev", _i32, _vp, _sz, _u32, _vp, _vp, _sz, _sz, _sz, _i32, _vp)
    sig("quant_dequant_dev", _i32, _vp, _sz, _u32, _vp, _sz, _vp)
    sig("quant_device_status", _i32, _vp)
    sig("quant_matvec_static", _i32, _vp, _sz, _u32, _fp, _fp, _sz, _sz)
    sig("fwb_host_alloc", _vp, _sz)
    sig("fwb_host_free", None, _vp)
    sig("fwb_model_open", _vp, _c.c_char_p, _sz, _i32)
    sig("fwb_model_close", None, _vp)
    sig("fwb_model_dims", _i32, _vp, _c.POINTER(_u32))
    sig("fwb_forward", _i32, _vp, _u32, _sz, _fp)
    sig("fwb_prefill", _i32, _vp, _c.POINTER(_u32), _sz, _sz, _c.POINTER(_c.c_float))
    sig("fwb_forward_argmax", _i32, _vp, _u32, _sz, _c.POINTER(_u32))
    sig("fwb_kv_load", _i32, _vp, _sz, _sz, _sz, _fp, _fp)
    sig("fwb_kv_read", _i32, _vp, _sz, _sz, _sz, _fp, _fp)
    sig("fwb_generate_greedy", _i32, _vp, _u32, _sz, _sz, _c.POINTER(_u32))
    sig("fwb_logits_dev", _vp, _vp)
    sig("fwb_sample", _i32, _vp, _c.POINTER(_u32), _sz, _c.c_float, _c.c_float, _c.c_float,
        _c.POINTER(_u64), _c.POINTER(_u32))
    sig("fwb_stream", _vp, _vp)
    sig("fwb_trace_read", _i32, _vp, _c.POINTER(_u64), _sz, _c.c_char_p, _sz)
    sig("fwb_prof_read", _i32, _vp, _c.POINTER(_u64), _sz)
    sig("fwb_trace_cta_read", _i32, _vp, _c.POINTER(_u64), _sz)
    sig("fwb_trace_attn_read", _i32, _vp, _c.POINTER(_u64), _sz)
    sig("fwb_model_weight_bytes", _u64, _vp)
    sig("fwb_model_load_stats", _i32, _vp, _c.POINTER(_c.c_double), _c.POINTER(_u64))
    sig("fwb_model_kernels_per_step", _i32, _vp)
    sig("fwb_model_open_tp", _vp, _c.c_char_p, _sz, _i32, _i32, _i32)
    sig("fwb_tp_handle", _i32, _vp, _vp)
    sig("fwb_tp_connect", _i32, _vp, _vp)
    sig("fwb_tp_shard", _i32, _c.c_char_p, _c.c_char_p, _i32, _i32, _i32, _vp, _sz, _c.POINTER(_sz))
