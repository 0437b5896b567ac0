"""Python host binding of the C ABI (include/streaming_b200.h).

Mirrors the reference's ``Stream::Runtime`` interface (reference
include/Runtime.hpp:7-46): ``Backend``, ``RuntimeOptions``, ``Snapshot`` and
``Runtime.step / reset / stop / snapshot / info / device_trace``, plus
``probe()``. Errors surface as ``StreamError`` (a ``RuntimeError``, as the
reference throws ``std::runtime_error``) carrying the C status code.

The CUDA library is mandatory: importing works without a GPU, but creating a
Runtime loads ``lib/libstreaming_b200.so`` and fails loudly if it is missing or
no B200 is present. There is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import enum
import json
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from .model import MODE_CODES, Model

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libstreaming_b200.so"

ST_OK = 0
STATUS_NAMES = {
    -1: "INVALID", -2: "UNSUPPORTED", -3: "CUDA", -4: "STOPPED", -5: "EXHAUSTED",
    -6: "WORKER_EXITED", -7: "DEVICE_TIMEOUT", -8: "HOST_TIMEOUT", -9: "STATE",
}


class StreamError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{message} [{STATUS_NAMES.get(code, code)}]")
        self.code = code
        self.status = STATUS_NAMES.get(code, str(code))


class Backend(enum.IntEnum):
    """reference include/Runtime.hpp:7, same order."""
    CUDA = 0
    GRAPH = 1
    CUBLAS = 2
    CUBLAS_GRAPH = 3
    FUSED = 4
    PERSISTENT = 5


BACKEND_NAMES = {"cuda": Backend.CUDA, "graph": Backend.GRAPH, "cublas": Backend.CUBLAS,
                 "cublas-graph": Backend.CUBLAS_GRAPH, "fused": Backend.FUSED,
                 "persistent": Backend.PERSISTENT}


@dataclass
class RuntimeOptions:
    """reference include/Runtime.hpp:8-19 (defaults kept). ``blocks=0`` selects one CTA per SM."""
    backend: Backend = Backend.GRAPH
    blocks: int = 1
    backoff: bool = False
    mapped: bool = False
    vector_matvec: bool = False
    fused_attention: bool = False
    max_events: int = 0
    initial_sequence: int = 0
    idle_seconds: float = 30.0
    device: int = 0


@dataclass
class TensorParallel:
    """One stream split over ``size`` GPUs (st_create_tp): this process owns GPU
    ``rank`` of the stream. ``exchange(blob)`` must return every rank's blob in
    rank order (an all-gather among the stream's processes; see
    streaming_transformer_b200.tp.torch_exchange)."""
    rank: int
    size: int
    exchange: object


@dataclass
class Snapshot:
    """reference include/Runtime.hpp:20-23."""
    position: int
    keys: np.ndarray = field(repr=False)
    values: np.ndarray = field(repr=False)
    hidden: np.ndarray = field(repr=False)


class _ModelDesc(ctypes.Structure):
    _fields_ = [("layers", ctypes.c_int), ("width", ctypes.c_int), ("heads", ctypes.c_int),
                ("ffn", ctypes.c_int), ("window", ctypes.c_int), ("features", ctypes.c_int),
                ("epsilon", ctypes.c_float), ("mode", ctypes.c_int), ("streams", ctypes.c_int)]


class _Options(ctypes.Structure):
    _fields_ = [("backend", ctypes.c_int), ("blocks", ctypes.c_int), ("backoff", ctypes.c_int),
                ("mapped", ctypes.c_int), ("vector_matvec", ctypes.c_int), ("fused_attention", ctypes.c_int),
                ("max_events", ctypes.c_uint64), ("initial_sequence", ctypes.c_uint64),
                ("idle_seconds", ctypes.c_double), ("device", ctypes.c_int)]


_lib = None
F = ctypes.POINTER(ctypes.c_float)
TRACE_FN = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_float), ctypes.c_size_t)


def library() -> ctypes.CDLL:
    """Load the CUDA library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise StreamError(-3, f"CUDA library missing: {LIB_PATH} (run python -m streaming_transformer_b200.build)")
        lib = ctypes.CDLL(str(LIB_PATH))
        P, I, S = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
        U64 = ctypes.c_uint64
        sigs = {
            "st_create": (I, [ctypes.POINTER(_ModelDesc), ctypes.POINTER(_Options), ctypes.POINTER(P)]),
            "st_set_tensor": (I, [P, ctypes.c_char_p, F, S]),
            "st_start": (I, [P]),
            "st_step": (I, [P, F, F]),
            "st_step_batch": (I, [P, F, F]),
            "st_reset": (I, [P]),
            "st_reset_stream": (I, [P, I]),
            "st_stop": (I, [P]),
            "st_snapshot": (I, [P, I, ctypes.POINTER(U64), F, F, F]),
            "st_load_state": (I, [P, I, U64, F, F, F]),
            "st_trace_step": (I, [P, F, F, TRACE_FN, P]),
            "st_device_trace": (I, [P, F, S, F, ctypes.POINTER(ctypes.c_double)]),
            "st_device_timeline": (I, [P, F, S, ctypes.POINTER(ctypes.c_longlong), S, ctypes.POINTER(S)]),
            "st_device_timeline_cta": (I, [P, F, S, I, ctypes.POINTER(ctypes.c_longlong), S, ctypes.POINTER(S)]),
            "st_device_trace_resident": (I, [P, ctypes.c_void_p, S, ctypes.POINTER(ctypes.c_double),
                                             ctypes.POINTER(U64)]),
            "st_device_trace_continue": (I, [P, ctypes.c_void_p, S, ctypes.POINTER(ctypes.c_double),
                                             ctypes.POINTER(U64)]),
            "st_create_tp": (I, [ctypes.POINTER(_ModelDesc), ctypes.POINTER(_Options), I, I, ctypes.POINTER(P)]),
            "st_resume": (I, [P]),
            "st_tp_handle": (I, [P, ctypes.c_void_p, S, ctypes.POINTER(S)]),
            "st_tp_connect": (I, [P, ctypes.c_void_p, S]),
            "st_info": (I, [P, ctypes.c_char_p, S, ctypes.POINTER(S)]),
            "st_probe": (I, [I, ctypes.c_char_p, S, ctypes.POINTER(S)]),
            "st_kernel_launches": (U64, [P]),
            "st_last_error": (ctypes.c_char_p, [P]),
            "st_destroy": (None, [P]),
            "st_abi_version": (I, []),
            "st_default_options": (None, [ctypes.POINTER(_Options)]),
        }
        for name, (res, args) in sigs.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(F)


def _check(code: int, handle=None) -> None:
    if code != ST_OK:
        msg = library().st_last_error(handle)
        raise StreamError(code, msg.decode() if msg else "error")


def _json_call(fn, *args) -> dict:
    needed = ctypes.c_size_t(0)
    _check(fn(*args, None, 0, ctypes.byref(needed)))
    buf = ctypes.create_string_buffer(needed.value)
    _check(fn(*args, buf, needed.value, ctypes.byref(needed)))
    return json.loads(buf.value.decode())


def transport_bench(mode: str, count: int, backoff: bool = False, device: int = 0,
                    csv_path: str | None = None) -> dict:
    """reference transportBench (src/cuda/Runtime.cu:706-814) plus "grid-barrier"."""
    lib = library()
    fn = lib.st_transport_bench
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_char_p,
                   ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]
    lib.st_transport_error.restype = ctypes.c_char_p
    buf = ctypes.create_string_buffer(1 << 16)
    needed = ctypes.c_size_t(0)
    code = fn(int(device), mode.encode(), int(count), int(bool(backoff)),
              csv_path.encode() if csv_path else None, buf, len(buf), ctypes.byref(needed))
    if code != ST_OK:
        raise StreamError(code, lib.st_transport_error().decode())
    return json.loads(buf.value.decode())


class Schedule(ctypes.Structure):
    """st_schedule: arrivals per second, bursty (groups of 16), queue capacity,
    deadline (us) and the producer thread's CPU (-1: unpinned)."""
    _fields_ = [("rate", ctypes.c_double), ("bursty", ctypes.c_int), ("queue", ctypes.c_size_t),
                ("deadline_us", ctypes.c_double), ("producer_core", ctypes.c_int)]


STEP_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.POINTER(ctypes.c_float),
                           ctypes.POINTER(ctypes.c_float))


def _replay_call(call, inputs, rate, bursty, queue, deadline_us, producer_core):
    """Run call(inputs_ptr, count, schedule, samples, scores, json, capacity,
    needed) for one of the replay entry points; returns (report, samples, scores)."""
    lib = library()
    lib.st_replay_error.restype = ctypes.c_char_p
    x = np.ascontiguousarray(inputs, dtype=np.float32)
    count = x.shape[0]
    sc = Schedule(float(rate), int(bool(bursty)), int(queue), float(deadline_us), int(producer_core))
    samples = np.zeros((count, 4), dtype=np.float64)
    scores = np.full(count, np.nan, dtype=np.float32)
    buf = ctypes.create_string_buffer(1 << 14)
    need = ctypes.c_size_t(0)
    code = call(_fptr(x), count, ctypes.byref(sc), samples.ctypes.data_as(ctypes.POINTER(ctypes.c_double)),
                _fptr(scores), buf, len(buf), ctypes.byref(need))
    report = json.loads(buf.value.decode()) if buf.value else {}
    if code != ST_OK:
        raise StreamError(code, lib.st_replay_error().decode())
    return report, samples, scores


def replay_scheduled_with(step, inputs, rate: float, bursty: bool = False, queue: int = 4096,
                          deadline_us: float = 1000.0, producer_core: int = -1):
    """Scheduled-arrival replay through a Python step(event) -> score callable
    (st_replay_scheduled_with). Returns (report, samples [n][4] ns, scores)."""
    lib = library()
    fn = lib.st_replay_scheduled_with
    fn.restype = ctypes.c_int
    fn.argtypes = [STEP_FN, ctypes.c_void_p, F, ctypes.c_size_t, ctypes.c_size_t, ctypes.POINTER(Schedule),
                   ctypes.POINTER(ctypes.c_double), F, ctypes.c_char_p, ctypes.c_size_t,
                   ctypes.POINTER(ctypes.c_size_t)]
    features = np.asarray(inputs).shape[1]

    def trampoline(_user, inp, out):
        try:
            out[0] = float(step(np.ctypeslib.as_array(inp, shape=(features,)).copy()))
            return ST_OK
        except Exception:  # a failing step ends the replay with an error code
            return -1

    cb = STEP_FN(trampoline)
    return _replay_call(lambda x, n, *rest: fn(cb, None, x, n, features, *rest), inputs, rate, bursty, queue,
                        deadline_us, producer_core)


def probe(device: int = 0) -> dict:
    """reference probe() (src/cuda/Runtime.cu:134-161, 664)."""
    return _json_call(library().st_probe, device)


class Runtime:
    """One runtime per device: device state for ``streams`` independent streams.

    Owns every device and pinned buffer; ``close()`` (or garbage collection)
    stops the resident worker before freeing them (reference
    src/cuda/Runtime.cu:294-299).

    With the PERSISTENT backend a kernel stays resident on the device between
    steps. A device-wide synchronize (``cudaDeviceSynchronize``,
    ``torch.cuda.synchronize()``) issued meanwhile waits for that kernel, i.e.
    until ``stop()`` or the idle budget ends it; synchronize individual
    streams instead.
    """

    def __init__(self, model: Model, options: RuntimeOptions | None = None, streams: int = 1,
                 tp: "TensorParallel | None" = None):
        self.model = model
        self.options = options or RuntimeOptions()
        self.streams = int(streams)
        c = model.config
        self.config = c
        lib = library()
        desc = _ModelDesc(c.layers, c.width, c.heads, c.ffn, c.window, c.features,
                          float(c.epsilon), MODE_CODES[model.mode], self.streams)
        o = self.options
        opts = _Options(int(o.backend), int(o.blocks), int(bool(o.backoff)), int(bool(o.mapped)),
                        int(bool(o.vector_matvec)), int(bool(o.fused_attention)), int(o.max_events),
                        int(o.initial_sequence), float(o.idle_seconds), int(o.device))
        handle = ctypes.c_void_p()
        if tp is None:
            code = lib.st_create(ctypes.byref(desc), ctypes.byref(opts), ctypes.byref(handle))
        else:
            code = lib.st_create_tp(ctypes.byref(desc), ctypes.byref(opts), int(tp.rank), int(tp.size),
                                    ctypes.byref(handle))
        if code != ST_OK:
            raise StreamError(code, lib.st_last_error(None).decode())
        self._h = handle
        try:
            for name in model.names():
                data = np.ascontiguousarray(model.get(name), dtype=np.float32).ravel()
                _check(lib.st_set_tensor(self._h, name.encode(), _fptr(data), data.size), self._h)
            if tp is not None:
                # every GPU of the stream maps every other GPU's record buffers;
                # the exchange also lines the ranks up for st_start's collective
                # warm-up step
                need = ctypes.c_size_t(0)
                blob = ctypes.create_string_buffer(256)
                _check(lib.st_tp_handle(self._h, blob, 256, ctypes.byref(need)), self._h)
                blobs = tp.exchange(blob.raw[: need.value])
                joined = b"".join(blobs)
                _check(lib.st_tp_connect(self._h, ctypes.c_char_p(joined), len(blobs)), self._h)
            _check(lib.st_start(self._h), self._h)
        except Exception:
            self.close()
            raise
        self._in = np.zeros((self.streams, c.features), dtype=np.float32)
        self._out = np.zeros(self.streams, dtype=np.float32)
        # the per-step call reuses its pointers and bound entry point
        self._in0 = self._in[0]
        self._in_p = _fptr(self._in)
        self._out_p = _fptr(self._out)
        self._st_step = lib.st_step
        self._features = c.features

    # -- lifecycle
    def close(self) -> None:
        h = getattr(self, "_h", None)
        if h:
            library().st_destroy(h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # -- hot path
    def step(self, event) -> float:
        """reference Runtime::step: one event (features floats) -> one score."""
        self._in0[:] = np.asarray(event, dtype=np.float32).reshape(-1)[: self._features]
        code = self._st_step(self._h, self._in_p, self._out_p)
        if code != ST_OK:
            _check(code, self._h)
        return float(self._out[0])

    def step_batch(self, events) -> np.ndarray:
        """Advance every stream by one event: events [streams, features] -> scores [streams]."""
        e = np.ascontiguousarray(events, dtype=np.float32).reshape(self.streams, self.config.features)
        out = np.empty(self.streams, dtype=np.float32)
        _check(library().st_step_batch(self._h, _fptr(e), _fptr(out)), self._h)
        return out

    def reset(self) -> None:
        _check(library().st_reset(self._h), self._h)

    def reset_stream(self, stream: int) -> None:
        _check(library().st_reset_stream(self._h, int(stream)), self._h)

    def stop(self) -> None:
        _check(library().st_stop(self._h), self._h)

    def start_worker(self) -> None:
        """A new persistent worker after stop() (st_resume), e.g. after load_state."""
        _check(library().st_resume(self._h), self._h)

    def snapshot(self, stream: int = 0) -> Snapshot:
        c = self.config
        shape = (c.layers, c.heads, c.window, c.head_dim)
        keys = np.empty(shape, dtype=np.float32)
        values = np.empty(shape, dtype=np.float32)
        hidden = np.empty((c.layers, c.width), dtype=np.float32)
        pos = ctypes.c_uint64(0)
        _check(library().st_snapshot(self._h, int(stream), ctypes.byref(pos), _fptr(keys), _fptr(values),
                                     _fptr(hidden)), self._h)
        return Snapshot(int(pos.value), keys, values, hidden)

    def load_state(self, position: int, keys, values, hidden, stream: int = 0) -> None:
        k = np.ascontiguousarray(keys, dtype=np.float32)
        v = np.ascontiguousarray(values, dtype=np.float32)
        h = np.ascontiguousarray(hidden, dtype=np.float32)
        _check(library().st_load_state(self._h, int(stream), int(position), _fptr(k), _fptr(v), _fptr(h)), self._h)

    def trace_step(self, event) -> dict[str, np.ndarray]:
        """reference Runtime::traceStep: one step with per-op snapshots (CUDA backend)."""
        trace: dict[str, np.ndarray] = {}

        def capture(_user, name, data, count):
            trace[name.decode()] = np.ctypeslib.as_array(data, shape=(count,)).copy()

        cb = TRACE_FN(capture)
        self._in[0, :] = np.asarray(event, dtype=np.float32).reshape(-1)[: self.config.features]
        score = np.zeros(1, dtype=np.float32)
        _check(library().st_trace_step(self._h, _fptr(self._in), _fptr(score), cb, None), self._h)
        return trace

    def info(self) -> dict:
        return _json_call(library().st_info, self._h)

    def device_trace(self, events, return_scores: bool = False):
        """reference Runtime::deviceTrace: µs per step over a preloaded trace
        ([count, features] or [count, streams, features]); resets first."""
        e = np.ascontiguousarray(events, dtype=np.float32)
        count = e.shape[0]
        e = e.reshape(count, self.streams, self.config.features)
        us = ctypes.c_double(0)
        scores = np.empty((count, self.streams), dtype=np.float32) if return_scores else None
        _check(library().st_device_trace(self._h, _fptr(e), count, _fptr(scores) if scores is not None else None,
                                         ctypes.byref(us)), self._h)
        if return_scores:
            return us.value, (scores[:, 0] if self.streams == 1 else scores)
        return us.value

    def device_timeline(self, events, capacity: int = 1 << 18, cta: int = 0, warp: int | None = 0) -> np.ndarray:
        """Diagnostic: clock64() << 8 | tag at every phase boundary of a device-loop
        run over ``events``, recorded by every warp of one CTA (see
        st_device_timeline_cta). Returns warp ``warp``'s marks, or all warps'
        as a [16, capacity // 16] array (zero padded) when ``warp`` is None."""
        e = np.ascontiguousarray(events, dtype=np.float32)
        count = e.shape[0]
        marks = np.zeros(capacity, dtype=np.int64)
        used = ctypes.c_size_t(0)
        _check(library().st_device_timeline_cta(self._h, _fptr(e), count, int(cta),
                                                marks.ctypes.data_as(ctypes.POINTER(ctypes.c_longlong)),
                                                capacity, ctypes.byref(used)), self._h)
        per_warp = marks.reshape(16, capacity // 16)
        if warp is None:
            return per_warp
        row = per_warp[warp]
        return row[: int(np.count_nonzero(row))]

    def device_trace_resident(self, device_ptr: int, count: int) -> tuple[float, int]:
        """Device-only timing with the trace already in device memory (pointer from
        any allocator); returns (µs per step, kernels launched)."""
        us = ctypes.c_double(0)
        launches = ctypes.c_uint64(0)
        _check(library().st_device_trace_resident(self._h, ctypes.c_void_p(device_ptr), int(count),
                                                  ctypes.byref(us), ctypes.byref(launches)), self._h)
        return us.value, int(launches.value)

    def device_trace_continue(self, device_ptr: int, count: int) -> tuple[float, int]:
        """As device_trace_resident, but from the current state (no reset): positions
        continue, so a warm-up of at least a window gives steady-state steps."""
        us = ctypes.c_double(0)
        launches = ctypes.c_uint64(0)
        _check(library().st_device_trace_continue(self._h, ctypes.c_void_p(device_ptr), int(count),
                                                  ctypes.byref(us), ctypes.byref(launches)), self._h)
        return us.value, int(launches.value)

    def replay_scheduled(self, inputs, rate: float, bursty: bool = False, queue: int = 4096,
                         deadline_us: float = 1000.0, producer_core: int = -1):
        """Scheduled-arrival replay of a one-stream trace through st_step
        (st_replay_scheduled; reference bench/Main.cpp:282-343): events arrive
        at `rate` per second (bursty: groups of 16) into a queue of `queue`
        events, dropped when full, and are stepped in order by a native loop.
        Returns (report, samples [n][4] steady-clock ns: intended, enqueue,
        submit, complete; scores, NaN where dropped)."""
        lib = library()
        fn = lib.st_replay_scheduled
        fn.restype = ctypes.c_int
        fn.argtypes = [ctypes.c_void_p, F, ctypes.c_size_t, ctypes.POINTER(Schedule),
                       ctypes.POINTER(ctypes.c_double), F, ctypes.c_char_p, ctypes.c_size_t,
                       ctypes.POINTER(ctypes.c_size_t)]
        return _replay_call(lambda *args: fn(self._h, *args), inputs, rate, bursty, queue, deadline_us,
                            producer_core)

    @property
    def kernel_launches(self) -> int:
        return int(library().st_kernel_launches(self._h))
