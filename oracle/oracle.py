"""ctypes binding of the CPU oracle (TEST INFRASTRUCTURE ONLY).

The oracle restates the reference CPU step (reference src/cpu/Cpu.cpp:59-141) in C;
see st_oracle.c. Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline / reference legs may import this module, and only as the checker or
the timed CPU baseline. The product path never loads it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIBRARY = HERE / "_build" / "libst_oracle.so"
MODE_CODES = {"fp32": 0, "mixed": 1, "bf16": 2}


class _Config(ctypes.Structure):
    _fields_ = [("layers", ctypes.c_int), ("width", ctypes.c_int), ("heads", ctypes.c_int),
                ("ffn", ctypes.c_int), ("window", ctypes.c_int), ("features", ctypes.c_int),
                ("epsilon", ctypes.c_float), ("mode", ctypes.c_int)]


TRACE_FN = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_char_p,
                            ctypes.POINTER(ctypes.c_float), ctypes.c_int)

_lib = None


def build() -> Path:
    """Compile the oracle with its Makefile (no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIBRARY


def library() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            build()
        lib = ctypes.CDLL(str(LIBRARY))
        P = ctypes.c_void_p
        F = ctypes.POINTER(ctypes.c_float)
        lib.st_oracle_create.restype = P
        lib.st_oracle_create.argtypes = [ctypes.POINTER(_Config), ctypes.c_int]
        lib.st_oracle_destroy.argtypes = [P]
        lib.st_oracle_set_tensor.restype = ctypes.c_int
        lib.st_oracle_set_tensor.argtypes = [P, ctypes.c_char_p, F, ctypes.c_size_t]
        lib.st_oracle_ready.restype = ctypes.c_int
        lib.st_oracle_ready.argtypes = [P]
        lib.st_oracle_step.restype = ctypes.c_float
        lib.st_oracle_step.argtypes = [P, F]
        lib.st_oracle_step_traced.restype = ctypes.c_float
        lib.st_oracle_step_traced.argtypes = [P, F, TRACE_FN, P]
        lib.st_oracle_reset.argtypes = [P]
        lib.st_oracle_position.restype = ctypes.c_uint64
        lib.st_oracle_position.argtypes = [P]
        for name in ("st_oracle_keys", "st_oracle_values", "st_oracle_hidden"):
            getattr(lib, name).restype = F
            getattr(lib, name).argtypes = [P]
        lib.st_oracle_cache_elements.restype = ctypes.c_size_t
        lib.st_oracle_cache_elements.argtypes = [P]
        lib.st_oracle_load_state.argtypes = [P, ctypes.c_uint64, F, F, F]
        lib.st_oracle_round_half.restype = ctypes.c_float
        lib.st_oracle_round_half.argtypes = [ctypes.c_float]
        lib.st_oracle_round_bf16.restype = ctypes.c_float
        lib.st_oracle_round_bf16.argtypes = [ctypes.c_float]
        lib.st_oracle_run.argtypes = [P, F, ctypes.c_size_t, F]
        _lib = lib
    return _lib


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


class Oracle:
    """CPU twin of ``Stream::Cpu`` (reference include/Cpu.hpp:11-34) for one stream."""

    def __init__(self, model, threads: int = 1):
        self.lib = library()
        c = model.config
        self.config = c
        self.mode = model.mode
        cfg = _Config(c.layers, c.width, c.heads, c.ffn, c.window, c.features,
                      float(c.epsilon), MODE_CODES[model.mode])
        self.handle = self.lib.st_oracle_create(ctypes.byref(cfg), int(threads))
        if not self.handle:
            raise RuntimeError("Invalid or unsupported model dimensions")
        for name in model.names():
            data = np.ascontiguousarray(model.get(name), dtype=np.float32).ravel()
            if self.lib.st_oracle_set_tensor(self.handle, name.encode(), _fptr(data), data.size):
                raise RuntimeError("oracle rejected tensor " + name)
        assert self.lib.st_oracle_ready(self.handle)

    def close(self):
        if getattr(self, "handle", None):
            self.lib.st_oracle_destroy(self.handle)
            self.handle = None

    def __del__(self):
        self.close()

    def step(self, event: np.ndarray) -> float:
        event = np.ascontiguousarray(event, dtype=np.float32)
        return float(self.lib.st_oracle_step(self.handle, _fptr(event)))

    def step_traced(self, event: np.ndarray) -> tuple[float, dict[str, np.ndarray]]:
        trace: dict[str, np.ndarray] = {}

        def capture(_user, name, data, count):
            trace[name.decode()] = np.ctypeslib.as_array(data, shape=(count,)).copy()

        callback = TRACE_FN(capture)
        event = np.ascontiguousarray(event, dtype=np.float32)
        score = float(self.lib.st_oracle_step_traced(self.handle, _fptr(event), callback, None))
        return score, trace

    def run(self, events: np.ndarray) -> np.ndarray:
        events = np.ascontiguousarray(events, dtype=np.float32)
        scores = np.empty(events.shape[0], dtype=np.float32)
        self.lib.st_oracle_run(self.handle, _fptr(events), events.shape[0], _fptr(scores))
        return scores

    def reset(self):
        self.lib.st_oracle_reset(self.handle)

    @property
    def position(self) -> int:
        return int(self.lib.st_oracle_position(self.handle))

    def _view(self, fn, count) -> np.ndarray:
        return np.ctypeslib.as_array(fn(self.handle), shape=(count,)).copy()

    def keys(self) -> np.ndarray:
        c = self.config
        n = self.lib.st_oracle_cache_elements(self.handle)
        return self._view(self.lib.st_oracle_keys, n).reshape(c.layers, c.heads, c.window, c.head_dim)

    def values(self) -> np.ndarray:
        c = self.config
        n = self.lib.st_oracle_cache_elements(self.handle)
        return self._view(self.lib.st_oracle_values, n).reshape(c.layers, c.heads, c.window, c.head_dim)

    def hidden(self) -> np.ndarray:
        c = self.config
        return self._view(self.lib.st_oracle_hidden, c.layers * c.width).reshape(c.layers, c.width)

    def load_state(self, position: int, keys, values, hidden):
        k = np.ascontiguousarray(keys, dtype=np.float32).ravel()
        v = np.ascontiguousarray(values, dtype=np.float32).ravel()
        h = np.ascontiguousarray(hidden, dtype=np.float32).ravel()
        self.lib.st_oracle_load_state(self.handle, int(position), _fptr(k), _fptr(v), _fptr(h))


def round_half(x: float) -> float:
    return float(library().st_oracle_round_half(ctypes.c_float(x)))


def round_bf16(x: float) -> float:
    return float(library().st_oracle_round_bf16(ctypes.c_float(x)))


def cpu_count() -> int:
    return len(os.sched_getaffinity(0))
