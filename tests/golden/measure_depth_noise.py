"""Print how far two correct CPU implementations of the step drift apart with
depth, at the Large shape (d1024, 12 layers): the reference's own
reference/model.py (bf16 storage: its fp16 cast points rounding to bf16) and
this repo's CPU restatement of its Cpu.cpp (oracle/). Both start from the same
random state past the window, as tests/test_gpu_batched_shapes.py loads it,
and take 3 steps; per layer it prints the relative L2 difference of the hidden
state and the largest coordinate difference relative to its vector's RMS.
These figures back the depth-scaled relative-L2 gate and the per-tensor
reading of the fp32 "1e-5 relative" bound in tests/policy.py.

    ST_REFERENCE=<reference checkout> python tests/golden/measure_depth_noise.py

Runs in the build container only (it imports the reference).
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))
if not os.environ.get("ST_REFERENCE"):
    raise SystemExit("set ST_REFERENCE to a checkout of the reference repository")
sys.path.insert(0, os.environ["ST_REFERENCE"])

from reference.model import Config, Streaming  # noqa: E402  (reference import, read only)

from oracle.oracle import Oracle  # noqa: E402
from streaming_transformer_b200 import synthetic  # noqa: E402
from test_gpu_batched_shapes import random_state  # noqa: E402


class StreamingBF16(Streaming):
    def cast(self, x):
        return x.bfloat16().to(self.dtype)


def score_drift(name, config, mode, model, c, weights) -> None:
    """The score sequences of the two implementations for the streams that
    tests/test_gpu_batched_shapes.py samples (its seeds and positions): the
    normalized RMSE RMS(diff) / max(1, RMS(ref)) that the score gate bounds."""
    for k, s in enumerate((0, 131, 255)):
        position = config.window + 37 * (k + 1)
        keys, values, hidden = random_state(config, mode, seed=900 + s)
        events = synthetic.make_events(3, config.features, seed=5000 + s)
        oracle = Oracle(model)
        oracle.load_state(position, keys, values, hidden)
        want = np.array([oracle.step(e) for e in events], dtype=np.float64)
        oracle.close()
        ref = (StreamingBF16 if mode == "bf16" else Streaming)(c, weights, "mixed" if mode == "bf16" else "fp32")
        ref.position = position
        ref.k = torch.from_numpy(keys.copy())
        ref.v = torch.from_numpy(values.copy())
        got = np.array([float(ref.step(torch.from_numpy(e))) for e in events], dtype=np.float64)
        nrmse = np.sqrt(np.mean((got - want) ** 2)) / max(1.0, np.sqrt(np.mean(want ** 2)))
        print(f"{name} stream {s} scores: normalized RMSE {nrmse:.3g}, max |diff| {np.max(np.abs(got - want)):.3g}")


def main() -> None:
    for name in ("c4-large-bf16", "c5-large-fp32"):
        config, mode = synthetic.CONFIGS[name]
        model = synthetic.make_model(config, mode, seed=31)
        position = config.window + 37
        keys, values, hidden = random_state(config, mode, seed=900)
        events = synthetic.make_events(3, config.features, seed=5000)
        oracle = Oracle(model)
        oracle.load_state(position, keys, values, hidden)
        for e in events:
            oracle.step(e)
        c = Config(layers=config.layers, width=config.width, heads=config.heads, ffn=config.ffn,
                   window=config.window, features=config.features, epsilon=config.epsilon)
        weights = {n: torch.from_numpy(np.ascontiguousarray(model.get(n))) for n in model.names()}
        ref = (StreamingBF16 if mode == "bf16" else Streaming)(c, weights, "mixed" if mode == "bf16" else "fp32")
        ref.position = position
        ref.k = torch.from_numpy(keys.copy())
        ref.v = torch.from_numpy(values.copy())
        for e in events:
            ref.step(torch.from_numpy(e))
        want = oracle.hidden()
        score_drift(name, config, mode, model, c, weights)
        for layer in range(config.layers):
            got = ref.intermediates[f"layers.{layer}.hidden"].float().numpy()
            diff = got - want[layer]
            rms = np.sqrt(np.mean(want[layer] ** 2))
            print(f"{name} layer {layer:2d}: relative L2 {np.linalg.norm(diff) / np.linalg.norm(want[layer]):.3g}, "
                  f"max |diff| / max(|r|, RMS) {np.max(np.abs(diff) / np.maximum(np.abs(want[layer]), rms)):.3g}")
        k_ref, k_or = ref.k.float().numpy(), oracle.keys()
        rms = np.sqrt(np.mean(k_or ** 2, axis=-1, keepdims=True))
        print(f"{name} keys: relative L2 {np.linalg.norm(k_ref - k_or) / np.linalg.norm(k_or):.3g}, "
              f"max |diff| / max(|r|, row RMS) {np.max(np.abs(k_ref - k_or) / np.maximum(np.abs(k_or), rms)):.3g}")
        oracle.close()


if __name__ == "__main__":
    main()
