"""GPU parity of the batched multi-stream round at the benchmark's many-stream
configurations, which the small-shape stream tests do not reach:

* C4, Large bf16 (d1024 L12 H16 F4096 W256) with 256 streams: the GEMM phases
  run on the tensor cores with a 256-column TMEM accumulator and N = 256 MMAs.
* C5-A, Large fp32 (W512) with 256 streams on one GPU (2048 over 8 GPUs): the
  GEMM phases run on the tensor cores as three tf32 products per fp32 product
  (hi/lo split), and, with ST_TC=0, on the CUDA cores in fp32; both are held
  to the fp32 policy (1e-5 relative per tensor).

Stepping 256 Large streams past a ring revolution on the CPU would take hours,
so the sampled streams start from a seeded random state at a position past the
window, handed to the runtime and to the oracle alike (st_load_state, the
state hand-off that long-run validation uses; reference scripts/validate.py:55-75
replays the whole trace instead). Their attention therefore reads a full,
wrapped window from the first round. The first, a middle and the last stream
are then stepped for a few rounds together with all other streams and compared
with their own oracles: every score and the full K/V/hidden state. The
reference's own matvec tests sweep every model shape the same way
(reference tests/Primitives.cu:104-153).
"""
import numpy as np
import pytest

from oracle.oracle import Oracle
from policy import check_scores, check_state
from streaming_transformer_b200 import Backend, Runtime, RuntimeOptions, synthetic
from streaming_transformer_b200.model import round_storage

pytestmark = pytest.mark.gpu

STREAMS = 256
SAMPLED = (0, 131, STREAMS - 1)
ROUNDS = 3


def random_state(config, mode, seed):
    """K/V rows with the spread the projections give (N(0, 0.6)), rounded to storage."""
    rng = np.random.default_rng(seed)
    shape = (config.layers, config.heads, config.window, config.head_dim)
    keys = round_storage(rng.normal(0.0, 0.6, shape).astype(np.float32), mode)
    values = round_storage(rng.normal(0.0, 0.6, shape).astype(np.float32), mode)
    hidden = rng.normal(0.0, 1.0, (config.layers, config.width)).astype(np.float32)
    return keys, values, hidden


@pytest.mark.parametrize("name,engine", [("c4-large-bf16", "tensor"), ("c5-large-fp32", "tensor"),
                                         ("c5-large-fp32", "cuda-cores")])
def test_batched_round_at_benchmark_shape(name, engine, monkeypatch):
    if engine == "cuda-cores":
        monkeypatch.setenv("ST_TC", "0")
    config, mode = synthetic.CONFIGS[name]
    model = synthetic.make_model(config, mode, seed=31)
    events = np.stack([synthetic.make_events(ROUNDS, config.features, seed=5000 + s) for s in range(STREAMS)],
                      axis=1)  # [rounds, streams, features]
    rt = Runtime(model, RuntimeOptions(backend=Backend.FUSED, blocks=0), streams=STREAMS)
    states = {}
    try:
        info = rt.info()
        assert info["batched"], info
        if engine == "tensor":
            # fp32: a second 256-column accumulator takes the tf32 correction products
            assert info["batched_tensor_cores"] and info["tc_tmem_columns"] == (512 if mode == "fp32" else 256), info
        else:
            assert not info["batched_tensor_cores"], info
        for k, s in enumerate(SAMPLED):
            # positions past the window; slot = position % W differs per stream
            position = config.window + 37 * (k + 1)
            keys, values, hidden = random_state(config, mode, seed=900 + s)
            rt.load_state(position, keys, values, hidden, stream=s)
            states[s] = (position, keys, values, hidden)
        got = np.array([rt.step_batch(e) for e in events])  # [rounds, streams]
        snaps = {s: rt.snapshot(s) for s in SAMPLED}
        heads0 = rt.snapshot(1).position  # a stream that started from reset
    finally:
        rt.close()
    assert heads0 == ROUNDS
    o = Oracle(model)  # one oracle (a full weight copy), handed each sampled state in turn
    for s, state in states.items():
        o.load_state(*state)
        want = np.array([o.step(events[r, s]) for r in range(ROUNDS)], dtype=np.float32)
        check_scores(got[:, s], want, config.layers, mode, f"{name} stream {s}")
        snap = snaps[s]
        assert snap.position == o.position
        check_state(snap.keys, o.keys(), mode, f"{name} keys stream {s}")
        check_state(snap.values, o.values(), mode, f"{name} values stream {s}")
        check_state(snap.hidden[:, None, :], o.hidden()[:, None, :], mode, f"{name} hidden stream {s}")
    o.close()
