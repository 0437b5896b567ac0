"""Seeded synthetic models and event traces for the B200 benchmark configurations.

The benchmark configurations are quoted on seeded N(0, 0.02) weights with unit
norm gains, eps 1e-6 and N(0, 1) float32 input events, 32 features each. No
dataset or checkpoint is involved; these generators make the same shapes and
value distributions deterministically from a seed (numpy PCG64), so the GPU box
rebuilds bit-identical weights and traces without any file transfer.

``CONFIGS`` names the five configurations (C1..C5). The reference's own model
shapes (Small/Main/Large with randn/sqrt(cols) weights, reference
reference/model.py:27-47, configs/*.json) are loaded from checkpoints instead.
"""
from __future__ import annotations

import numpy as np

from .model import Model, ModelConfig, tensor_shapes

FEATURES = 32

# name -> (config, mode, window sweep / streams noted for the benchmark)
CONFIGS = {
    "c1-small-fp32": (ModelConfig(4, 256, 4, 1024, 64, FEATURES, 1e-6), "fp32"),
    "c2-main-fp32": (ModelConfig(8, 512, 8, 2048, 128, FEATURES, 1e-6), "fp32"),
    "c3-main-bf16": (ModelConfig(8, 512, 8, 2048, 128, FEATURES, 1e-6), "bf16"),
    "c4-large-bf16": (ModelConfig(12, 1024, 16, 4096, 256, FEATURES, 1e-6), "bf16"),
    "c5-large-fp32": (ModelConfig(12, 1024, 16, 4096, 512, FEATURES, 1e-6), "fp32"),
}


def config_with_window(config: ModelConfig, window: int) -> ModelConfig:
    return ModelConfig(config.layers, config.width, config.heads, config.ffn, window,
                       config.features, config.epsilon)


def make_tensors(config: ModelConfig, seed: int = 42, std: float = 0.02) -> dict[str, np.ndarray]:
    """N(0, std) float32 matrices, unit norm gains, drawn in manifest order."""
    rng = np.random.default_rng(seed)
    tensors = {}
    for name, shape in tensor_shapes(config).items():
        if len(shape) == 1:
            tensors[name] = np.ones(shape, dtype=np.float32)
        else:
            tensors[name] = (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)
    return tensors


def make_model(config: ModelConfig, mode: str, seed: int = 42) -> Model:
    """Synthetic model; matrices rounded to the storage type of ``mode``."""
    return Model.from_tensors(config, mode, make_tensors(config, seed))


def make_events(count: int, features: int = FEATURES, seed: int = 123) -> np.ndarray:
    """[count, features] N(0, 1) float32 events for one stream."""
    rng = np.random.default_rng(seed)
    return rng.standard_normal((count, features), dtype=np.float32)


def make_stream_events(streams: int, count: int, features: int = FEATURES,
                       base_seed: int = 1000) -> np.ndarray:
    """[count, streams, features]: stream s draws from seed base_seed + s."""
    out = np.empty((count, streams, features), dtype=np.float32)
    for s in range(streams):
        out[:, s, :] = make_events(count, features, base_seed + s)
    return out
