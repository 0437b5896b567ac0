"""Load the committed golden fixtures (tests/golden/*) and the models they pin."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

from streaming_transformer_b200.model import Model, ModelConfig
from streaming_transformer_b200 import synthetic

GOLDEN = Path(__file__).resolve().parent / "golden"
REF_CASES = ["ref-small-fp32", "ref-small-mixed", "ref-main-fp32", "ref-main-mixed"]
SYNTHETIC_CASES = ["c1-small-fp32", "c1-small-bf16", "c2-main-fp32"]
ALL_CASES = REF_CASES + SYNTHETIC_CASES


class Golden:
    def __init__(self, name: str):
        self.name = name
        self.path = GOLDEN / name
        self.meta = json.loads((self.path / "meta.json").read_text())
        with np.load(self.path / "expected.npz") as data:
            self.expected = {k: data[k] for k in data.files}
        if name.startswith("ref-"):
            self.model = Model(self.path)
            c = self.model.config
            self.events = np.fromfile(self.path / "trace.bin", dtype="<f4").reshape(-1, c.features)
        else:
            config = ModelConfig.from_json(self.meta["config"])
            self.model = synthetic.make_model(config, self.meta["mode"], self.meta["seed"])
            self.events = synthetic.make_events(self.meta["events"], config.features, self.meta["trace_seed"])
        self.events = self.events[: self.meta["events"]]
        self.resets = list(self.meta["resets"])
        self.state_events = [int(i) for i in self.expected["state_events"]]
        hidden_events = self.meta.get("hidden_events", "all")
        self.hidden_events = (list(range(len(self.events))) if hidden_events == "all"
                              else [int(i) for i in hidden_events])
        self.state_layers = self.meta.get("state_layers", list(range(self.model.config.layers)))

    @property
    def mixed(self) -> bool:
        return self.model.mode != "fp32"
