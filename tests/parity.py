"""Parity helpers shared by the tests (tolerances of the acceptance spec).

Logits: per decode step max |a - b| <= 1e-2 and ||a - b||_2 / ||b||_2 <= 1e-3.
Dequantised weights: bit-exact.  Greedy tokens: identical.
"""
from __future__ import annotations

import numpy as np

LOGIT_ABS = 1e-2
LOGIT_REL = 1e-3


def logit_errors(got: np.ndarray, ref: np.ndarray) -> tuple[float, float]:
    d = got.astype(np.float64) - ref.astype(np.float64)
    rel = float(np.linalg.norm(d) / max(np.linalg.norm(ref.astype(np.float64)), 1e-30))
    return float(np.abs(d).max()), rel


def assert_logits_close(got: np.ndarray, ref: np.ndarray, where: str = "") -> tuple[float, float]:
    assert got.shape == ref.shape
    assert np.all(np.isfinite(got)), f"non-finite logits {where}"
    a, r = logit_errors(got, ref)
    assert a <= LOGIT_ABS and r <= LOGIT_REL, f"logits differ {where}: max-abs {a:.3g} rel {r:.3g}"
    return a, r


def top2_gap(x: np.ndarray) -> float:
    i = int(np.argmax(x))
    y = x.astype(np.float64).copy()
    y[i] = -np.inf
    return float(x[i] - y.max())


def greedy_compare(gpu_step, ref_step, first: int, pos0: int, n: int):
    """Teacher-forced greedy comparison.

    Both sides are fed the reference's own greedy token stream, so every step
    compares logits on identical inputs.  Returns (mismatches, worst_abs,
    worst_rel, min_gap) where mismatches lists (step, gpu_tok, ref_tok, gap).
    """
    tok = first
    mism = []
    worst_a = worst_r = 0.0
    min_gap = np.inf
    for i in range(n):
        g = gpu_step(tok, pos0 + i)
        r = ref_step(tok, pos0 + i)
        a, rr = logit_errors(g, r)
        worst_a, worst_r = max(worst_a, a), max(worst_r, rr)
        gap = top2_gap(r)
        min_gap = min(min_gap, gap)
        gt, rt = int(np.argmax(g)), int(np.argmax(r))
        if gt != rt:
            mism.append((i, gt, rt, gap))
        tok = rt
    return mism, worst_a, worst_r, min_gap
