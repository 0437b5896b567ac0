"""st_attention_static: the attention entry point that allocates nothing.

It serves callers that may not allocate device memory (stream host callbacks,
processes whose device memory pool belongs to another framework, real-time
loops that must not take allocator locks). Its output is checked against the
attention the existing st_trace_step entry point captures from a full step,
on consecutive calls that share (and overwrite) the library's fixed scratch
array. This file sorts last so that a run stopping at the first failure has
already run every other test; it also passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from policy import check_state
from streaming_transformer_b200 import Backend, ModelConfig, Runtime, RuntimeOptions, library
from streaming_transformer_b200 import synthetic
from streaming_transformer_b200.model import MODE_CODES

pytestmark = pytest.mark.gpu


def static_attention():
    lib = library()
    fn = lib.st_attention_static
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_uint64,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    lib.st_attention_static_error.restype = ctypes.c_char_p
    return fn, lib.st_attention_static_error


@pytest.mark.parametrize("mode", ["fp32", "mixed", "bf16"])
def test_static_attention_matches_step_attention_on_consecutive_calls(mode):
    import torch
    fn, _ = static_attention()
    dtype = {"fp32": torch.float32, "mixed": torch.float16, "bf16": torch.bfloat16}[mode]
    c = ModelConfig(2, 128, 2, 96, 40, 32, 1e-5)   # head_dim 64, two 32-slot chunks
    model = synthetic.make_model(c, mode, seed=11)
    events = synthetic.make_events(56, 32, seed=12)
    rt = Runtime(model, RuntimeOptions(backend=Backend.CUDA, blocks=0))
    try:
        for e in events[:50]:          # past one full ring revolution
            rt.step(e)
        stream = torch.cuda.current_stream()
        calls = 0
        for step in range(2):
            trace = rt.trace_step(events[50 + step])
            snap = rt.snapshot()
            position = snap.position - 1
            for layer in range(c.layers):
                q = torch.from_numpy(trace[f"layers.{layer}.q"]).cuda()
                keys = torch.from_numpy(snap.keys[layer]).to(dtype).contiguous().cuda()
                values = torch.from_numpy(snap.values[layer]).to(dtype).contiguous().cuda()
                out = torch.full((c.width,), float("nan"), dtype=torch.float32, device="cuda")
                rc = fn(0, MODE_CODES[mode], c.heads, c.head_dim, c.window, position, q.data_ptr(),
                        keys.data_ptr(), values.data_ptr(), out.data_ptr(), stream.cuda_stream)
                assert rc == 0
                stream.synchronize()
                calls += 1
                got = out.cpu().numpy()
                want = trace[f"layers.{layer}.attention"]
                assert np.all(np.isfinite(got))
                check_state(got[None, None, :], want[None, None, :], mode, f"static attention layer {layer}")
        assert calls == 4
    finally:
        rt.close()


def test_static_attention_rejects_sizes_beyond_its_array():
    fn, error = static_attention()
    dummy = ctypes.c_void_p(16)   # never dereferenced: validation fails first
    rc = fn(0, 0, 4, 64, 5000, 0, dummy, dummy, dummy, dummy, None)
    assert rc != 0 and b"attention dimensions" in error()
    rc = fn(0, 0, 32, 64, 64, 0, dummy, dummy, dummy, dummy, None)
    assert rc != 0 and b"attention dimensions" in error()
