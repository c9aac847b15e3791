"""Python handle over the C ABI of libforword_b200.so (include/forword_b200.h).

Thin ctypes plumbing only: every call goes to the CUDA library; a missing
library raises (no CPU fallback).
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import native


class FwbError(RuntimeError):
    pass


def _err(lib) -> str:
    return lib.fwb_last_error().decode(errors="replace")


class Model:
    """One decode model on one GPU (transformer_t of forword.c)."""

    def __init__(self, path: str, max_ctx: int = 0, device: int = 0, rank: int = 0, world: int = 1,
                 exchange=None):
        """world > 1: rank `rank` of a tensor-parallel model (one process per
        GPU).  `exchange(handle: bytes) -> list[bytes]` must all-gather the
        64-byte exchange-buffer handles of every rank in rank order (e.g. with
        torch.distributed.all_gather_object); see fwb.tp."""
        self.lib = native.product()
        self.h = None
        self.rank, self.world = rank, world
        if world == 1:
            self.h = self.lib.fwb_model_open(path.encode(), max_ctx, device)
        else:
            self.h = self.lib.fwb_model_open_tp(path.encode(), max_ctx, device, rank, world)
        if not self.h:
            raise FwbError(f"fwb_model_open({path}): {_err(self.lib)}")
        if world > 1:
            if exchange is None:
                raise FwbError("a tensor-parallel model needs an exchange function")
            mine = ctypes.create_string_buffer(64)
            if self.lib.fwb_tp_handle(self.h, mine) != 0:
                raise FwbError(f"fwb_tp_handle: {_err(self.lib)}")
            handles = exchange(mine.raw)
            if len(handles) != world or any(len(x) != 64 for x in handles):
                raise FwbError("exchange must return one 64-byte handle per rank")
            buf = ctypes.create_string_buffer(b"".join(handles), 64 * world)
            if self.lib.fwb_tp_connect(self.h, buf) != 0:
                raise FwbError(f"fwb_tp_connect: {_err(self.lib)}")
        d = (ctypes.c_uint32 * 8)()
        self.lib.fwb_model_dims(self.h, d)
        (self.n_vocab, self.kv_ctx, self.n_embd, self.n_layer, self.n_head, self.n_head_kv,
         self.n_ff, self.head_dim) = list(d)
        self._logits = np.zeros(self.n_vocab, dtype=np.float32)

    def close(self) -> None:
        if self.h:
            self.lib.fwb_model_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def weight_bytes(self) -> int:
        return int(self.lib.fwb_model_weight_bytes(self.h))

    @property
    def load_stats(self) -> tuple[float, int]:
        """(seconds, bytes) of the tensor upload at open (fwb_model_load_stats)."""
        sec = ctypes.c_double()
        nb = ctypes.c_uint64()
        self.lib.fwb_model_load_stats(self.h, ctypes.byref(sec), ctypes.byref(nb))
        return float(sec.value), int(nb.value)

    @property
    def kernels_per_step(self) -> int:
        return int(self.lib.fwb_model_kernels_per_step(self.h))

    @property
    def stream(self) -> int:
        return int(self.lib.fwb_stream(self.h) or 0)

    def forward(self, token: int, pos: int, out: np.ndarray | None = None) -> np.ndarray:
        """transformer_forward: returns (a copy of) the n_vocab logits."""
        dst = self._logits if out is None else out
        rc = self.lib.fwb_forward(self.h, token, pos,
                                  dst.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
        if rc != 0:
            raise FwbError(f"fwb_forward: {_err(self.lib)}")
        return dst.copy() if out is None else dst

    def prefill(self, tokens, pos0: int = 0) -> np.ndarray:
        """fwb_prefill: feed tokens at pos0.. and return the last token's logits."""
        tok = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.zeros(self.n_vocab, dtype=np.float32)
        rc = self.lib.fwb_prefill(self.h, tok.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)), tok.size, pos0,
                                  out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
        if rc != 0:
            raise FwbError(f"fwb_prefill: {_err(self.lib)}")
        return out

    def try_forward(self, token: int, pos: int) -> int:
        """Raw return code of fwb_forward (0 / -1) for error-path tests."""
        return int(self.lib.fwb_forward(self.h, token, pos, None))

    def forward_argmax(self, token: int, pos: int) -> int:
        nxt = ctypes.c_uint32()
        if self.lib.fwb_forward_argmax(self.h, token, pos, ctypes.byref(nxt)) != 0:
            raise FwbError(f"fwb_forward_argmax: {_err(self.lib)}")
        return int(nxt.value)

    def generate_greedy(self, first: int, pos0: int, n: int) -> np.ndarray:
        out = np.zeros(n, dtype=np.uint32)
        rc = self.lib.fwb_generate_greedy(self.h, first, pos0, n,
                                          out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)))
        if rc != 0:
            raise FwbError(f"fwb_generate_greedy: {_err(self.lib)}")
        return out

    def sample(self, history, temperature: float, top_p: float, rep_penalty: float,
               rng_state: int) -> tuple[int, int]:
        """fwb_sample on the last step's device logits: (token, new rng state)."""
        h = np.ascontiguousarray(history, dtype=np.uint32)
        st = ctypes.c_uint64(rng_state)
        tok = ctypes.c_uint32()
        rc = self.lib.fwb_sample(self.h, h.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)), h.size, temperature,
                                 top_p, rep_penalty, ctypes.byref(st), ctypes.byref(tok))
        if rc != 0:
            raise FwbError(f"fwb_sample: {_err(self.lib)}")
        return int(tok.value), int(st.value)

    def kv_load(self, layer: int, pos0: int, k: np.ndarray, v: np.ndarray) -> None:
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        n = k.shape[0]
        fp = ctypes.POINTER(ctypes.c_float)
        if self.lib.fwb_kv_load(self.h, layer, pos0, n, k.ctypes.data_as(fp), v.ctypes.data_as(fp)) != 0:
            raise FwbError(f"fwb_kv_load: {_err(self.lib)}")

    def kv_read(self, layer: int, pos0: int, n: int) -> tuple[np.ndarray, np.ndarray]:
        k = np.zeros((n, self.n_head_kv, self.head_dim), dtype=np.float32)
        v = np.zeros_like(k)
        fp = ctypes.POINTER(ctypes.c_float)
        if self.lib.fwb_kv_read(self.h, layer, pos0, n, k.ctypes.data_as(fp), v.ctypes.data_as(fp)) != 0:
            raise FwbError(f"fwb_kv_read: {_err(self.lib)}")
        return k, v


def tp_shard(path: str, tensor: str, rank: int, world: int, as_head: bool = False) -> np.ndarray:
    """Host-only: the bytes rank `rank` of `world` keeps of `tensor` (fwb_tp_shard)."""
    lib = native.product()
    n = ctypes.c_size_t()
    args = (path.encode(), tensor.encode(), int(as_head), rank, world)
    if lib.fwb_tp_shard(*args, None, 0, ctypes.byref(n)) != 0:
        raise FwbError(f"fwb_tp_shard: {_err(lib)}")
    out = np.empty(n.value, dtype=np.uint8)
    if lib.fwb_tp_shard(*args, out.ctypes.data, out.nbytes, ctypes.byref(n)) != 0:
        raise FwbError(f"fwb_tp_shard: {_err(lib)}")
    return out


def quant_matvec(w: np.ndarray, ggml_type: int, x: np.ndarray, n_out: int) -> np.ndarray:
    """quant_matvec with host buffers (the reference's signature)."""
    lib = native.product()
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(n_out, dtype=np.float32)
    fp = ctypes.POINTER(ctypes.c_float)
    rc = lib.quant_matvec(w.ctypes.data, w.nbytes, ggml_type, x.ctypes.data_as(fp),
                          y.ctypes.data_as(fp), x.size, n_out)
    if rc != 0:
        raise FwbError(f"quant_matvec: {_err(lib)}")
    return y
