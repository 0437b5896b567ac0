"""CPU-only checks of the boundary: the C ABI library loads and exports every
symbol include/streaming_b200.h declares; argument validation that happens
before any CUDA call; the checkpoint loader's format checks (reference
src/runtime/Model.cpp:15-145, tests/Native.cpp:10-17, tests/test_export.py:9-27)."""
import ctypes
import json
import re
import shutil
from pathlib import Path

import numpy as np
import pytest

from streaming_transformer_b200 import (Backend, CheckpointError, Model, ModelConfig, Runtime,
                                        RuntimeOptions, StreamError, library, write_checkpoint)
from streaming_transformer_b200 import runtime as rtmod
from streaming_transformer_b200 import synthetic
from streaming_transformer_b200.model import tensor_shapes

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "streaming_b200.h"


def declared_symbols():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(st_[a-z_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = library()
    names = declared_symbols()
    assert len(names) >= 19
    for name in names:
        assert hasattr(lib, name), name
    assert lib.st_abi_version() == 1


def test_default_options_match_reference():
    o = rtmod._Options()
    library().st_default_options(ctypes.byref(o))
    assert o.backend == Backend.GRAPH and o.blocks == 1 and o.idle_seconds == 30.0
    assert o.max_events == 0 and o.initial_sequence == 0 and not o.mapped
    d = RuntimeOptions()
    assert d.backend == Backend.GRAPH and d.blocks == 1 and d.idle_seconds == 30.0


def small_model(mode="fp32"):
    c = ModelConfig(1, 64, 4, 128, 64, 32, 1e-5)
    return synthetic.make_model(c, mode, 1)


@pytest.mark.parametrize("mutate,code", [
    (dict(heads=3), "INVALID"),      # width % heads
    (dict(window=4097), "INVALID"),
    (dict(layers=17), "INVALID"),
])
def test_create_rejects_invalid_dimensions_before_touching_a_gpu(mutate, code):
    m = small_model()
    c = m.config
    fields = dict(layers=c.layers, width=c.width, heads=c.heads, ffn=c.ffn, window=c.window,
                  features=c.features, epsilon=c.epsilon, mode=0, streams=1)
    fields.update(mutate)
    desc = rtmod._ModelDesc(**fields)
    opts = rtmod._Options()
    library().st_default_options(ctypes.byref(opts))
    h = ctypes.c_void_p()
    rc = library().st_create(ctypes.byref(desc), ctypes.byref(opts), ctypes.byref(h))
    assert rtmod.STATUS_NAMES[rc] == code
    assert b"Invalid or unsupported model dimensions" in library().st_last_error(None)
    assert not h.value


@pytest.mark.parametrize("options,code", [
    (RuntimeOptions(backend=Backend.CUBLAS), "UNSUPPORTED"),
    (RuntimeOptions(backend=Backend.CUBLAS_GRAPH), "UNSUPPORTED"),
    (RuntimeOptions(idle_seconds=0), "INVALID"),
    (RuntimeOptions(idle_seconds=3601), "INVALID"),
    (RuntimeOptions(blocks=-1), "INVALID"),
    (RuntimeOptions(initial_sequence=2 ** 64 - 1), "INVALID"),
])
def test_create_rejects_invalid_options(options, code):
    with pytest.raises(StreamError) as info:
        Runtime(small_model(), options)
    assert info.value.status == code


def test_config_validation_and_cache_elements():
    c = ModelConfig.from_json(dict(layers=1, width=64, heads=4, ffn=128, window=64, features=32, epsilon=1e-5))
    assert c.cache_elements() == 4096
    with pytest.raises(CheckpointError):
        ModelConfig.from_json(dict(layers=1, width=64, heads=3, ffn=128, window=64, features=32, epsilon=1e-5))
    with pytest.raises(CheckpointError):
        ModelConfig.from_json(dict(layers=1, width=64, heads=4, ffn=128, window=64, features=32, epsilon=0))


def test_golden_checkpoints_load(golden_dir):
    for name in ("ref-small-fp32", "ref-small-mixed", "ref-main-fp32", "ref-main-mixed"):
        m = Model(golden_dir / name)
        assert set(m.names()) == set(tensor_shapes(m.config))
        assert m.mixed == (m.mode != "fp32")


def test_checkpoint_corruption_and_shape_errors(tmp_path, golden_dir):
    src = golden_dir / "ref-small-fp32"
    dst = tmp_path / "ck"
    shutil.copytree(src, dst)
    raw = (dst / "tensors.bin").read_bytes()
    (dst / "tensors.bin").write_bytes(bytes([raw[0] ^ 1]) + raw[1:])
    with pytest.raises(CheckpointError, match="Checkpoint hash mismatch"):
        Model(dst)
    (dst / "tensors.bin").write_bytes(raw)
    manifest = json.loads((dst / "manifest.json").read_text())
    manifest["mode"] = "int8"
    (dst / "manifest.json").write_text(json.dumps(manifest))
    with pytest.raises(CheckpointError, match="Unknown numerical mode"):
        Model(dst)
    manifest["mode"] = "fp32"
    manifest["config"]["ffn"] = 64
    (dst / "manifest.json").write_text(json.dumps(manifest))
    with pytest.raises(CheckpointError):
        Model(dst)


@pytest.mark.parametrize("mode", ["fp32", "mixed", "bf16"])
def test_checkpoint_round_trip(tmp_path, mode):
    m = small_model(mode)
    write_checkpoint(tmp_path / mode, m)
    back = Model(tmp_path / mode)
    assert back.mode == mode
    for name in m.names():
        np.testing.assert_array_equal(back.get(name), m.get(name))
