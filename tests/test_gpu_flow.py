"""GPU parity of the single-stream flow kernel (csrc/st_flow.cuh) at the shapes the
benchmark configurations use but the golden fixtures do not reach: the window
extremes of the C3 sweep (32 and 512 slots, i.e. 4 and 64 slots per cluster rank)
and the width-1024 instantiation with 4-CTA clusters (C4 bf16, C5 fp32). Each run is
compared step by step with the CPU oracle under the reference policy, state included.
"""
import pytest

from gpu_util import compare_to_oracle
from streaming_transformer_b200 import Backend, Runtime, RuntimeOptions
from streaming_transformer_b200 import synthetic

pytestmark = pytest.mark.gpu


def assert_flow(model, cluster=None):
    with Runtime(model, RuntimeOptions(backend=Backend.PERSISTENT, blocks=0)) as rt:
        info = rt.info()
    assert info["flow"] and info["resource_kernel"] == "k4_flow", info["resource_kernel"]
    if cluster is not None:
        assert info["cluster"] == cluster


@pytest.mark.parametrize("window", [32, 512])
def test_c3_window_extremes(window):
    # bf16 storage, d512 L8 H8; the run passes the ring wrap and a reset.
    config = synthetic.config_with_window(synthetic.CONFIGS["c3-main-bf16"][0], window)
    model = synthetic.make_model(config, "bf16", seed=window)
    assert_flow(model)
    events = synthetic.make_events(window + 28, 32, seed=window + 1)
    compare_to_oracle(model, events, RuntimeOptions(backend=Backend.PERSISTENT, blocks=0),
                      resets=(window + 20,), check_every=max(4, window // 4))


@pytest.mark.parametrize("name", ["c4-large-bf16", "c5-large-fp32"])
def test_large_shapes(name):
    # d1024 L12 H16 F4096: 16 heads need 4-CTA clusters (one head per cluster).
    config, mode = synthetic.CONFIGS[name]
    model = synthetic.make_model(config, mode, seed=11)
    assert_flow(model, cluster=4)
    events = synthetic.make_events(20, 32, seed=12)
    compare_to_oracle(model, events, RuntimeOptions(backend=Backend.PERSISTENT, blocks=0), resets=(14,),
                      check_every=6)
