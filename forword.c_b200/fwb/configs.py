"""Model shapes: the benchmark spec's configurations plus small test shapes.

Every model is the llama family as forword.c's model_config.c:150-159
configures it: RMSNorm, gated SiLU FFN, adjacent-pair RoPE, no biases.
Quant types are GGML type ids: 0 F32, 2 Q4_0, 6 Q5_0, 8 Q8_0.
"""
from __future__ import annotations

from dataclasses import dataclass, field, replace

F32, Q4_0, Q5_0, Q5_1, Q8_0, Q4_K, Q6_K = 0, 2, 6, 7, 8, 12, 14
TYPE_NAMES = {F32: "F32", Q4_0: "Q4_0", Q5_0: "Q5_0", Q5_1: "Q5_1", Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K"}
BLOCK_BYTES = {Q4_0: 18, Q5_0: 22, Q5_1: 24, Q8_0: 34, Q4_K: 144, Q6_K: 210}
BLOCK_VALUES = {Q4_0: 32, Q5_0: 32, Q5_1: 32, Q8_0: 32, Q4_K: 256, Q6_K: 256}


def quant_bytes(t: int, n: int) -> int:
    """Bytes of n values of ggml type t (n a multiple of the block)."""
    return n * 4 if t == F32 else n // BLOCK_VALUES[t] * BLOCK_BYTES[t]


@dataclass(frozen=True)
class ModelShape:
    name: str
    n_embd: int
    n_layer: int
    n_head: int
    n_head_kv: int
    n_ff: int
    n_vocab: int
    n_ctx: int
    rope_base: float = 10000.0
    eps: float = 1e-5
    tied: bool = False
    out_norm: bool = True   # False: no output_norm.weight (the head reads x unnormalised)
    # ggml type per tensor role
    t_embd: int = F32
    t_q: int = Q4_0
    t_k: int = Q4_0
    t_v: int = Q4_0
    t_o: int = Q4_0
    t_gate: int = Q4_0
    t_up: int = Q4_0
    t_down: int = Q4_0
    t_out: int = Q4_0
    weight_sd: float = 0.02
    norm_sd: float = 0.02
    extra: dict = field(default_factory=dict, compare=False)

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head

    def tensor_bytes(self, t: int, rows: int, cols: int) -> int:
        return quant_bytes(t, rows * cols)

    def weight_bytes_per_token(self) -> int:
        """Algorithmic HBM bytes one decode step must stream: every quantised
        linear weight once (block bytes incl. scales), fp32 norm weights, and
        one embedding row."""
        E, F, hd = self.n_embd, self.n_ff, self.head_dim
        q = self.n_head * hd
        kv = self.n_head_kv * hd
        per_layer = (self.tensor_bytes(self.t_q, q, E) + self.tensor_bytes(self.t_k, kv, E)
                     + self.tensor_bytes(self.t_v, kv, E) + self.tensor_bytes(self.t_o, E, q)
                     + self.tensor_bytes(self.t_gate, F, E) + self.tensor_bytes(self.t_up, F, E)
                     + self.tensor_bytes(self.t_down, E, F) + 2 * E * 4)
        head_t = self.t_embd if self.tied else self.t_out
        head = self.tensor_bytes(head_t, self.n_vocab, E)
        embd_row = self.tensor_bytes(self.t_embd, 1, E)
        return self.n_layer * per_layer + head + E * 4 + embd_row

    def prefill_gemm_params(self) -> int:
        """Weights one prompt token multiplies in the prompt path's GEMMs
        (fwb_prefill): QKV in every layer, o-proj and the FFN in all but the
        last (whose output only feeds the logits).  FLOPs = 2 x this."""
        E, F, hd = self.n_embd, self.n_ff, self.head_dim
        q, kv = self.n_head * hd, self.n_head_kv * hd
        return self.n_layer * (q + 2 * kv) * E + (self.n_layer - 1) * (q * E + 3 * E * F)

    def kv_bytes_per_token(self, n_pos: int) -> int:
        """fp32 K and V bytes the attention of one decode step reads at n_pos
        cached positions (all layers)."""
        return self.n_layer * n_pos * self.n_head_kv * self.head_dim * 4 * 2


# --- the benchmark spec's configurations ------------------------------------
TINY = ModelShape("tiny-q8_0", n_embd=288, n_layer=6, n_head=6, n_head_kv=6, n_ff=768,
                  n_vocab=32000, n_ctx=256, tied=True, t_embd=Q8_0, t_q=Q8_0, t_k=Q8_0,
                  t_v=Q8_0, t_o=Q8_0, t_gate=Q8_0, t_up=Q8_0, t_down=Q8_0, t_out=Q8_0)

LLAMA8B_Q4_0 = ModelShape("llama8b-q4_0", n_embd=4096, n_layer=32, n_head=32, n_head_kv=8,
                          n_ff=14336, n_vocab=128256, n_ctx=8192, rope_base=500000.0)

LLAMA8B_MIXED = ModelShape("llama8b-mixed", n_embd=4096, n_layer=32, n_head=32, n_head_kv=8,
                           n_ff=14336, n_vocab=128256, n_ctx=8192, rope_base=500000.0,
                           t_q=Q8_0, t_k=Q8_0, t_v=Q8_0, t_o=Q8_0, t_gate=Q5_0, t_up=Q5_0,
                           t_down=Q8_0, t_out=Q8_0)

LLAMA70B_Q4_0 = ModelShape("llama70b-q4_0", n_embd=8192, n_layer=80, n_head=64, n_head_kv=8,
                           n_ff=28672, n_vocab=128256, n_ctx=4096, rope_base=500000.0)

# --- small shapes for parity tests ----------------------------------------------
SMALL_Q4_0 = ModelShape("small-q4_0", n_embd=512, n_layer=2, n_head=4, n_head_kv=2, n_ff=1024,
                        n_vocab=2048, n_ctx=512, rope_base=500000.0)
SMALL_MIXED = replace(SMALL_Q4_0, name="small-mixed", t_q=Q8_0, t_k=Q8_0, t_v=Q8_0, t_o=Q8_0,
                      t_gate=Q5_0, t_up=Q5_0, t_down=Q8_0, t_out=Q8_0)
SMALL_TIED_Q8 = replace(TINY, name="small-tied-q8_0", n_layer=2, n_vocab=1000, n_ctx=128)
SMALL_NO_OUT_NORM = replace(SMALL_Q4_0, name="small-q4_0-no-out-norm", out_norm=False)
# the K-quant mix of a Q4_K_M file: Q4_K attention/gate/up, Q6_K down / v /
# head, Q4_K embedding; widths multiples of 256
SMALL_KQUANT = ModelShape("small-kquant", n_embd=512, n_layer=2, n_head=4, n_head_kv=2, n_ff=1536,
                          n_vocab=2048, n_ctx=512, rope_base=500000.0, t_embd=Q4_K, t_q=Q4_K, t_k=Q4_K,
                          t_v=Q6_K, t_o=Q4_K, t_gate=Q4_K, t_up=Q4_K, t_down=Q6_K, t_out=Q6_K)
SMALL_Q5_1 = replace(SMALL_Q4_0, name="small-q5_1", t_q=Q5_1, t_k=Q5_1, t_v=Q5_1, t_o=Q5_1, t_gate=Q5_1,
                     t_up=Q5_1, t_down=Q5_1, t_out=Q5_1, t_embd=Q5_1)
# splits over 2, 4 or 8 tensor-parallel ranks (8 KV heads, 256 FFN rows and
# 256 vocabulary rows per rank at 8 ranks)
SMALL_TP8 = ModelShape("small-tp8", n_embd=1024, n_layer=2, n_head=8, n_head_kv=8, n_ff=2048,
                       n_vocab=2048, n_ctx=512, rope_base=500000.0)

CONFIGS = {c.name: c for c in (TINY, LLAMA8B_Q4_0, LLAMA8B_MIXED, LLAMA70B_Q4_0, SMALL_TP8,
                               SMALL_Q4_0, SMALL_MIXED, SMALL_TIED_Q8, SMALL_NO_OUT_NORM, SMALL_KQUANT,
                               SMALL_Q5_1)}


def with_layers(cfg: ModelShape, n_layer: int) -> ModelShape:
    """cfg with only its first n_layer layers (same shapes per layer): a
    small case of the same kernels for profiler captures and parity slices."""
    if n_layer == cfg.n_layer:
        return cfg
    return replace(cfg, name=f"{cfg.name}-{n_layer}layer", n_layer=n_layer)
