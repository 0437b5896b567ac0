"""st_attention_static: the attention entry point that allocates nothing.

It serves callers that may not allocate device memory (stream host callbacks,
processes whose device memory pool belongs to another framework, real-time
loops that must not take allocator locks). On two consecutive calls per layer,
which share (and overwrite) the library's fixed scratch array, its output is
checked against the CPU oracle's attention for the same q and K/V ring (the
oracle's own step trace) and against the attention the existing st_trace_step
entry point captures from a full GPU step. This file sorts last so that a run
stopping at the first failure has already run every other test; it also
passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from oracle.oracle import Oracle
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


TORCH_DTYPE = {"fp32": "float32", "mixed": "float16", "bf16": "bfloat16"}


def call(fn, mode, heads, head_dim, window, position, q, keys, values):
    """One call through the C ABI on torch's current stream; returns the output."""
    import torch
    dtype = getattr(torch, TORCH_DTYPE[mode])
    qd = torch.from_numpy(np.ascontiguousarray(q, dtype=np.float32)).cuda()
    kd = torch.from_numpy(np.ascontiguousarray(keys, dtype=np.float32)).to(dtype).contiguous().cuda()
    vd = torch.from_numpy(np.ascontiguousarray(values, dtype=np.float32)).to(dtype).contiguous().cuda()
    out = torch.full((heads * head_dim,), float("nan"), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    rc = fn(0, MODE_CODES[mode], heads, head_dim, window, position, qd.data_ptr(), kd.data_ptr(), vd.data_ptr(),
            out.data_ptr(), stream.cuda_stream)
    assert rc == 0
    stream.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("mode", ["fp32", "mixed", "bf16"])
def test_static_attention_matches_oracle_and_step_attention_on_consecutive_calls(mode):
    fn, _ = static_attention()
    c = ModelConfig(2, 128, 2, 96, 40, 32, 1e-5)   # head_dim 64, two 32-slot chunks
    model = synthetic.make_model(c, mode, seed=11)
    events = synthetic.make_events(56, 32, seed=12)
    oracle = Oracle(model)
    rt = Runtime(model, RuntimeOptions(backend=Backend.CUDA, blocks=0))
    try:
        for e in events[:50]:          # past one full ring revolution
            rt.step(e)
            oracle.step(e)
        calls = 0
        for step in range(2):
            _, want = oracle.step_traced(events[50 + step])
            gpu = rt.trace_step(events[50 + step])
            position = oracle.position - 1
            keys, values = oracle.keys(), oracle.values()
            for layer in range(c.layers):
                got = call(fn, mode, c.heads, c.head_dim, c.window, position, want[f"layers.{layer}.q"],
                           keys[layer], values[layer])
                calls += 1
                assert np.all(np.isfinite(got))
                check_state(got[None, None, :], want[f"layers.{layer}.attention"][None, None, :], mode,
                            f"static attention vs oracle, layer {layer}")
                check_state(got[None, None, :], gpu[f"layers.{layer}.attention"][None, None, :], mode,
                            f"static attention vs st_trace_step, layer {layer}")
        assert calls == 4
    finally:
        rt.close()
        oracle.close()


def test_static_attention_serves_its_largest_admitted_shape():
    # 512 heads of head_dim 2 over a 4096-slot window need exactly the whole
    # array; the largest position must not wrap the retained-slot count.
    fn, error = static_attention()
    heads, head_dim, window = 512, 2, 4096
    rng = np.random.default_rng(3)
    q = rng.standard_normal(heads * head_dim).astype(np.float32)
    keys = rng.standard_normal((heads, window, head_dim)).astype(np.float32)
    values = rng.standard_normal((heads, window, head_dim)).astype(np.float32)
    got = call(fn, "fp32", heads, head_dim, window, 2 ** 64 - 1, q, keys, values)
    qh = q.reshape(heads, head_dim)
    logits = np.einsum("hd,hwd->hw", qh.astype(np.float64), keys) / np.sqrt(head_dim)
    p = np.exp(logits - logits.max(axis=1, keepdims=True))
    want = (np.einsum("hw,hwd->hd", p, values) / p.sum(axis=1, keepdims=True)).ravel()
    assert np.all(np.isfinite(got)), error()
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-5)


def test_static_attention_rejects_dimensions_beyond_its_limits():
    fn, error = static_attention()
    dummy = ctypes.c_void_p(16)   # never dereferenced: validation fails first
    rc = fn(0, 0, 4, 64, 5000, 0, dummy, dummy, dummy, dummy, None)
    assert rc != 0 and b"attention dimensions" in error()
    rc = fn(0, 0, 32, 64, 64, 0, dummy, dummy, dummy, dummy, None)
    assert rc != 0 and b"attention dimensions" in error()
