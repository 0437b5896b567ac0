"""Generate the committed golden fixtures under tests/golden/ (run in the build container).

Needs a read-only checkout of the reference, named by $ST_REFERENCE; never
runs on the GPU box. Three families:

ref-small-{fp32,mixed}
    The reference's own committed checkpoint, trace and reset schedule
    (fixtures/small-*), plus a subset of its committed expected archive
    (fixtures/small-*/expected, written by reference/export.py:46-70 under
    torch 2.6): every score and hidden vector, K/V rings at sampled events.
ref-main-{fp32,mixed}
    The reference's committed Main checkpoint and trace (fixtures/main-*), with
    expected values computed here by importing reference/model.py
    (Streaming.step, reference/model.py:110-137): every score, sampled hidden
    vectors and K/V rings, reset before event 2W+3 as export.py does.
c1-small-{fp32,bf16}, c2-main-fp32
    B200 benchmark shapes (head_dim 64, eps 1e-6, seeded N(0, 0.02) weights from
    streaming_transformer_b200.synthetic). Weights are not stored: the tests
    regenerate them from the seed. Expected values again come from
    reference/model.py; bf16 replaces model.py's fp16 cast with a bf16 cast by
    subclassing Math.cast at run time (the reference file is not modified).

Output per directory: ``expected.npz`` + ``meta.json`` (and checkpoint files
for the ref-* families).
"""
from __future__ import annotations

import json
import os
import shutil
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
if not os.environ.get("ST_REFERENCE"):
    raise SystemExit("set ST_REFERENCE to a checkout of the reference repository")
REFERENCE = Path(os.environ["ST_REFERENCE"])
sys.path.insert(0, str(REFERENCE))

from reference.model import Config, Streaming  # noqa: E402  (reference import, read only)

from streaming_transformer_b200.model import Model  # noqa: E402
from streaming_transformer_b200 import synthetic  # noqa: E402

OUT = Path(__file__).resolve().parent


class StreamingBF16(Streaming):
    """reference Streaming with its fp16 cast points rounding to bf16 instead."""

    def cast(self, x):
        return x.bfloat16().to(self.dtype)


def load_expected(path: Path) -> dict[str, np.ndarray]:
    manifest = json.loads((path / "manifest.json").read_text())
    raw = (path / "tensors.bin").read_bytes()
    return {t["name"]: np.frombuffer(raw[t["offset"]:t["offset"] + t["nbytes"]], "<f4").reshape(t["shape"]).copy()
            for t in manifest["tensors"]}, manifest


def copy_checkpoint(src: Path, dst: Path) -> None:
    dst.mkdir(parents=True, exist_ok=True)
    for name in ("manifest.json", "tensors.bin", "trace.bin", "resets.json"):
        shutil.copyfile(src / name, dst / name)


def run_reference(config: dict, weights: dict, events: np.ndarray, resets: list[int], mode: str,
                  state_events: list[int], hidden_events: list[int] | None = None):
    """Drive reference Streaming over ``events``; collect scores, hidden, sampled K/V."""
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    c = Config(**config)
    cls = StreamingBF16 if mode == "bf16" else Streaming
    oracle = cls(c, weights, "mixed" if mode in ("mixed", "bf16") else "fp32")
    scores, hidden, keys, values = [], [], [], []
    for i, event in enumerate(events):
        if i in resets:
            oracle.reset()
        scores.append(float(oracle.step(torch.from_numpy(event))))
        if hidden_events is None or i in hidden_events:
            hidden.append(torch.stack([oracle.intermediates[f"layers.{l}.hidden"]
                                       for l in range(c.layers)]).float().numpy())
        if i in state_events:
            keys.append(oracle.k.float().numpy().copy())
            values.append(oracle.v.float().numpy().copy())
    return (np.array(scores, dtype=np.float32), np.array(hidden, dtype=np.float32),
            np.array(keys, dtype=np.float32), np.array(values, dtype=np.float32))


def write(dst: Path, meta: dict, **arrays) -> None:
    dst.mkdir(parents=True, exist_ok=True)
    np.savez(dst / "expected.npz", **arrays)
    meta = dict(meta, torch=torch.__version__, numpy=np.__version__,
                generator="tests/golden/make_golden.py")
    (dst / "meta.json").write_text(json.dumps(meta, indent=2) + "\n")
    print(dst.name, {k: v.shape for k, v in arrays.items()}, flush=True)


def ref_small(mode: str) -> None:
    src = REFERENCE / "fixtures" / f"small-{mode}"
    dst = OUT / f"ref-small-{mode}"
    copy_checkpoint(src, dst)
    tensors, manifest = load_expected(src / "expected")
    count = tensors["scores"].shape[0]
    window = manifest["config"]["window"]
    state_events = sorted({0, 1, window - 1, window, window + 1, 2 * window + 2,
                           2 * window + 3, 2 * window + 4, count - 1})
    write(dst, dict(source="reference fixtures/small-%s/expected (committed golden)" % mode,
                    mode=mode, events=count, resets=manifest["resets"], state_events=state_events,
                    hidden_events="all"),
          scores=tensors["scores"], hidden=tensors["hidden"],
          keys=tensors["keys"][state_events], values=tensors["values"][state_events],
          state_events=np.array(state_events))


def ref_main(mode: str) -> None:
    src = REFERENCE / "fixtures" / f"main-{mode}"
    dst = OUT / f"ref-main-{mode}"
    copy_checkpoint(src, dst)
    model = Model(dst)
    c = model.config
    events = np.fromfile(dst / "trace.bin", dtype="<f4").reshape(-1, c.features)
    resets = json.loads((dst / "resets.json").read_text())
    dtype = torch.float16 if mode == "mixed" else torch.float32
    weights = {n: torch.from_numpy(model.get(n)).to(dtype) for n in model.names()}
    count = events.shape[0]
    state_events = [2 * c.window + 2, count - 1]
    hidden_events = sorted({0, 1, c.window - 1, c.window, 2 * c.window + 2, 2 * c.window + 3, count - 1})
    scores, hidden, keys, values = run_reference(c.to_json(), weights, events, resets, mode,
                                                 state_events, hidden_events)
    write(dst, dict(source="reference/model.py Streaming on reference fixtures/main-%s" % mode,
                    mode=mode, events=count, resets=resets, state_events=state_events,
                    hidden_events=hidden_events),
          scores=scores, hidden=hidden, keys=keys, values=values,
          state_events=np.array(state_events), hidden_events=np.array(hidden_events))


def synthetic_golden(name: str, config_key: str, mode: str, count: int, seed: int = 42,
                     trace_seed: int = 123, state_layers: list[int] | None = None,
                     resets: list[int] | None = None, hidden_events: list[int] | None = None) -> None:
    """hidden_events None: every event's hidden vectors; resets None: one reset at W + 5."""
    config, _ = synthetic.CONFIGS[config_key]
    model = synthetic.make_model(config, mode, seed)
    events = synthetic.make_events(count, config.features, trace_seed)
    if mode == "bf16":
        weights = {n: torch.from_numpy(model.get(n)).bfloat16() for n in model.names()}
    else:
        weights = {n: torch.from_numpy(model.get(n)) for n in model.names()}
    if resets is None:
        resets = [config.window + 5] if count > config.window + 5 else []
    state_events = [count - 1]
    scores, hidden, keys, values = run_reference(config.to_json(), weights, events, resets, mode,
                                                 state_events, hidden_events)
    state_layers = state_layers or list(range(config.layers))
    keys, values = keys[:, state_layers], values[:, state_layers]
    write(OUT / name, dict(source="reference/model.py Streaming on synthetic weights",
                           config=config.to_json(), mode=mode, seed=seed, trace_seed=trace_seed,
                           events=count, resets=resets, state_events=state_events,
                           state_layers=state_layers,
                           hidden_events="all" if hidden_events is None else hidden_events),
          scores=scores, hidden=hidden, keys=keys, values=values, state_events=np.array(state_events))


def main() -> None:
    families = sys.argv[1:] or ["ref-small", "ref-main", "c1", "c2"]
    if "ref-small" in families:
        for mode in ("fp32", "mixed"):
            ref_small(mode)
    if "ref-main" in families:
        for mode in ("fp32", "mixed"):
            ref_main(mode)
    if "c1" in families:
        synthetic_golden("c1-small-fp32", "c1-small-fp32", "fp32", 80)
        synthetic_golden("c1-small-bf16", "c1-small-fp32", "bf16", 80)
    if "c2" in families:
        # the reference's fixture pattern (scripts/validate.py:40-52): 3W + 9
        # events with a reset before event 2W + 3, so the ring wraps twice
        w = synthetic.CONFIGS["c2-main-fp32"][0].window
        count = 3 * w + 9
        hidden_events = sorted({0, 1, w - 1, w, w + 1, 2 * w + 2, 2 * w + 3, 2 * w + 4, count - 1})
        synthetic_golden("c2-main-fp32", "c2-main-fp32", "fp32", count, state_layers=[0, 7],
                         resets=[2 * w + 3], hidden_events=hidden_events)


if __name__ == "__main__":
    main()
