"""Checkpoint format and model configuration (host side of the drop-in boundary).

Mirrors the reference's ``Stream::ModelConfig`` / ``Stream::Model``
(reference include/Model.hpp:12-39, src/runtime/Model.cpp:15-145):

* ``manifest.json`` + ``tensors.bin`` written by reference/export.py:31-43
  (version 1, little endian, ``out_in`` orientation, per-tensor and whole-file
  SHA-256, contiguous tensors in manifest order);
* the same config bounds (layers <= 16, width <= 1024, even head_dim,
  ffn <= 4096, window <= 4096, features <= 1024, finite positive epsilon);
* the same exact-shape checks for every tensor.

Modes: ``fp32`` and ``mixed`` (fp16 storage) as in the reference, plus ``bf16``
(bf16 storage, the numeric mode the B200 configs ask for; dtype ``bfloat16``
tensors are stored as the upper 16 bits of float32).
"""
from __future__ import annotations

import hashlib
import json
from dataclasses import dataclass, asdict
from pathlib import Path

import numpy as np

MODES = ("fp32", "mixed", "bf16")
MODE_CODES = {"fp32": 0, "mixed": 1, "bf16": 2}
LAYER_TENSORS = ("norm1", "norm2", "q", "k", "v", "out", "gate", "up", "down")


class CheckpointError(RuntimeError):
    """Raised for every format, hash, bound or shape violation (reference throws std::runtime_error)."""


@dataclass(frozen=True)
class ModelConfig:
    layers: int
    width: int
    heads: int
    ffn: int
    window: int
    features: int
    epsilon: float

    @staticmethod
    def from_json(j: dict) -> "ModelConfig":
        """reference src/runtime/Model.cpp:15-20 (fromJson validates)."""
        try:
            c = ModelConfig(int(j["layers"]), int(j["width"]), int(j["heads"]), int(j["ffn"]),
                            int(j["window"]), int(j["features"]), float(j["epsilon"]))
        except (KeyError, TypeError, ValueError) as error:
            raise CheckpointError(f"Invalid model configuration: {error}") from None
        c.validate()
        return c

    def validate(self) -> None:
        """reference src/runtime/Model.cpp:22-29."""
        ok = (1 <= self.layers <= 16 and 1 <= self.width <= 1024 and self.heads >= 1
              and self.width % self.heads == 0 and (self.width // self.heads) % 2 == 0
              and 1 <= self.ffn <= 4096 and 1 <= self.window <= 4096
              and 1 <= self.features <= 1024 and np.isfinite(self.epsilon) and self.epsilon > 0)
        if not ok:
            raise CheckpointError("Invalid or unsupported model dimensions")

    def cache_elements(self) -> int:
        """reference src/runtime/Model.cpp:31-33: layers * width * window per K (or V) ring."""
        return self.layers * self.width * self.window

    @property
    def head_dim(self) -> int:
        return self.width // self.heads

    def to_json(self) -> dict:
        return asdict(self)


def tensor_shapes(c: ModelConfig) -> dict[str, tuple[int, ...]]:
    """Exact shape contract in manifest order (reference src/runtime/Model.cpp:119-139,
    reference/model.py:35-46)."""
    shapes: dict[str, tuple[int, ...]] = {"input": (c.width, c.features)}
    for layer in range(c.layers):
        p = f"layers.{layer}."
        shapes[p + "norm1"] = (c.width,)
        shapes[p + "norm2"] = (c.width,)
        for name in ("q", "k", "v", "out"):
            shapes[p + name] = (c.width, c.width)
        shapes[p + "gate"] = (c.ffn, c.width)
        shapes[p + "up"] = (c.ffn, c.width)
        shapes[p + "down"] = (c.width, c.ffn)
    shapes["final_norm"] = (c.width,)
    shapes["score"] = (1, c.width)
    return shapes


def round_bf16(a: np.ndarray) -> np.ndarray:
    """float32 -> nearest-even bfloat16, returned as float32 (NaN kept)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32).copy()
    nan = np.isnan(a)
    out[nan] = a[nan]
    return out


def round_storage(a: np.ndarray, mode: str) -> np.ndarray:
    """Round float32 values to the storage type of ``mode`` (widened back to float32)."""
    a = np.asarray(a, dtype=np.float32)
    if mode == "mixed":
        return a.astype(np.float16).astype(np.float32)
    if mode == "bf16":
        return round_bf16(a)
    return a.copy()


def _sha256(raw: bytes) -> str:
    return hashlib.sha256(raw).hexdigest()


class Model:
    """Validated checkpoint (reference include/Model.hpp:25-35).

    ``get(name)`` returns the tensor widened to float32, as the reference widens
    fp16 storage to float (src/runtime/Model.cpp:100-109)."""

    def __init__(self, path: str | Path):
        path = Path(path)
        try:
            manifest = json.loads((path / "manifest.json").read_text())
        except (OSError, ValueError) as error:
            raise CheckpointError(f"Cannot read {path / 'manifest.json'}: {error}") from None
        self.manifest = manifest
        if (manifest.get("version") != 1 or manifest.get("byte_order") != "little"
                or manifest.get("orientation") != "out_in"):
            raise CheckpointError("Unsupported tensor format")
        self.config = ModelConfig.from_json(manifest.get("config", {}))
        mode = manifest.get("mode")
        if mode not in MODES:
            raise CheckpointError("Unknown numerical mode")
        self.mode = mode
        self.mixed = mode != "fp32"
        try:
            raw = (path / "tensors.bin").read_bytes()
        except OSError as error:
            raise CheckpointError(f"Cannot read {path / 'tensors.bin'}: {error}") from None
        if _sha256(raw) != manifest.get("sha256"):
            raise CheckpointError("Checkpoint hash mismatch")
        self._tensors: dict[str, np.ndarray] = {}
        end = 0
        for item in manifest.get("tensors", []):
            shape = tuple(int(d) for d in item["shape"])
            if any(d <= 0 for d in shape):
                raise CheckpointError("Invalid tensor dimensions")
            count = int(np.prod(shape))
            dtype = item["dtype"]
            size = {"float32": 4, "float16": 2, "bfloat16": 2}.get(dtype, 0)
            offset, nbytes = int(item["offset"]), int(item["nbytes"])
            if (not size or offset != end or nbytes != count * size or offset > len(raw)
                    or nbytes > len(raw) - offset):
                raise CheckpointError("Invalid tensor bounds")
            part = raw[offset:offset + nbytes]
            if _sha256(part) != item["sha256"]:
                raise CheckpointError("Tensor hash mismatch")
            if dtype == "float32":
                data = np.frombuffer(part, dtype="<f4").astype(np.float32)
            elif dtype == "float16":
                data = np.frombuffer(part, dtype="<f2").astype(np.float32)
            else:
                data = (np.frombuffer(part, dtype="<u2").astype(np.uint32) << 16).view(np.float32)
            name = item["name"]
            if name in self._tensors:
                raise CheckpointError("Duplicate tensor")
            self._tensors[name] = data.reshape(shape)
            end += nbytes
        if end != len(raw):
            raise CheckpointError("Trailing tensor bytes")
        for name, shape in tensor_shapes(self.config).items():
            if name not in self._tensors or self._tensors[name].shape != shape:
                raise CheckpointError("Shape mismatch: " + name)

    def get(self, name: str) -> np.ndarray:
        return self._tensors[name]

    def names(self) -> list[str]:
        return list(tensor_shapes(self.config))

    @staticmethod
    def from_tensors(config: ModelConfig, mode: str, tensors: dict[str, np.ndarray]) -> "Model":
        """In-memory model (no file), values rounded to the storage type of ``mode``."""
        if mode not in MODES:
            raise CheckpointError("Unknown numerical mode")
        config.validate()
        m = Model.__new__(Model)
        m.config, m.mode, m.mixed = config, mode, mode != "fp32"
        m.manifest = {"version": 1, "config": config.to_json(), "mode": mode}
        m._tensors = {}
        for name, shape in tensor_shapes(config).items():
            a = np.asarray(tensors[name], dtype=np.float32)
            if a.shape != shape:
                raise CheckpointError("Shape mismatch: " + name)
            m._tensors[name] = round_storage(a, mode).reshape(shape)
        return m


def write_checkpoint(path: str | Path, model: Model, extra: dict | None = None) -> None:
    """Write ``manifest.json`` + ``tensors.bin`` in the reference layout
    (reference/export.py:31-43). bf16 tensors use dtype ``bfloat16``."""
    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    data = bytearray()
    manifest = dict(version=1, byte_order="little", orientation="out_in",
                    config=model.config.to_json(), mode=model.mode, **(extra or {}), tensors=[])
    for name in model.names():
        a = model.get(name)
        if model.mode == "fp32":
            raw, dtype = a.astype("<f4").tobytes(), "float32"
        elif model.mode == "mixed":
            raw, dtype = a.astype("<f2").tobytes(), "float16"
        else:
            raw, dtype = (round_bf16(a).view(np.uint32) >> 16).astype("<u2").tobytes(), "bfloat16"
        manifest["tensors"].append(dict(name=name, shape=list(a.shape), dtype=dtype,
                                        offset=len(data), nbytes=len(raw), sha256=_sha256(raw)))
        data.extend(raw)
    manifest["sha256"] = _sha256(bytes(data))
    (path / "tensors.bin").write_bytes(bytes(data))
    (path / "manifest.json").write_text(json.dumps(manifest, indent=2) + "\n")
