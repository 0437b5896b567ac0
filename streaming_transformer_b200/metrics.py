"""Roofline arithmetic and latency statistics for the streaming step.

Algorithmic bytes of one stream-step: every weight byte once, plus the K and V
rows attention reads (2 L valid d elem), plus the K and V rows written
(2 L d elem). Activations (a few KB) are not counted. valid = min(t + 1, W)
for the step at position t, so a trace that starts from reset ramps from 1 to
W. FLOPs per stream-step: 2 * matrix parameters + 4 L valid d.
"""
from __future__ import annotations

import math

import numpy as np

from .model import ModelConfig

ELEM_BYTES = {"fp32": 4, "mixed": 2, "bf16": 2}


def weight_elements(c: ModelConfig) -> int:
    per_layer = 4 * c.width * c.width + 3 * c.width * c.ffn + 2 * c.width
    return c.width * c.features + c.layers * per_layer + 2 * c.width


def weight_bytes(c: ModelConfig, mode: str) -> int:
    return weight_elements(c) * ELEM_BYTES[mode]


def valid_lengths(c: ModelConfig, start: int, count: int) -> np.ndarray:
    t = np.arange(start, start + count, dtype=np.int64)
    return np.minimum(t + 1, c.window)


def step_bytes(c: ModelConfig, mode: str, valid: int | np.ndarray, streams: int = 1):
    """Algorithmic bytes for one step of ``streams`` streams (weights read once per step)."""
    e = ELEM_BYTES[mode]
    kv = 2 * c.layers * c.width * e * (np.asarray(valid) + 1) * streams
    return weight_bytes(c, mode) + kv


def trace_bytes(c: ModelConfig, mode: str, count: int, start: int = 0, streams: int = 1) -> int:
    """Total algorithmic bytes of ``count`` consecutive steps from position ``start``."""
    v = valid_lengths(c, start, count)
    return int(np.sum(step_bytes(c, mode, v, streams)))


def step_flops(c: ModelConfig, valid: int) -> int:
    return 2 * (weight_elements(c) - (2 * c.layers + 2) * c.width) + 4 * c.layers * valid * c.width


def nearest_rank(values, q: float) -> float:
    """reference bench/Main.cpp:50-56: sorted[ceil(q n) - 1]."""
    v = np.sort(np.asarray(values, dtype=np.float64))
    if v.size == 0:
        return float("nan")
    return float(v[max(0, math.ceil(q * v.size) - 1)])


def distribution(values_us) -> dict:
    return {"p50_us": nearest_rank(values_us, 0.5), "p95_us": nearest_rank(values_us, 0.95),
            "p99_us": nearest_rank(values_us, 0.99), "p999_us": nearest_rank(values_us, 0.999),
            "worst_us": float(np.max(values_us)) if len(values_us) else float("nan")}
