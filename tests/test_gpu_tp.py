"""Tensor parallelism of one stream over two GPUs (st_create_tp), against the
CPU oracle: tests/tp_parity.py under torch.distributed.run, one rank per GPU.
Runs the benchmark's C5 Large fp32 shape (W512, 16 heads: 8 per GPU) and a
Main bf16 shape; needs two GPUs and is skipped on a single-GPU box."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
pytestmark = pytest.mark.gpu


def gpus() -> int:
    import torch
    return torch.cuda.device_count()


@pytest.mark.parametrize("config", ["c5-large-fp32", "c3-main-bf16"])
def test_tensor_parallel_stream_matches_oracle(config):
    if gpus() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29613", str(ROOT / "tests" / "tp_parity.py"),
           "--config", config, "--events", "5"]
    proc = subprocess.run(["timeout", "-k", "30", "600", *cmd], capture_output=True, text=True, env=env, cwd=ROOT)
    lines = [l for l in proc.stdout.splitlines() if l.startswith("{")]
    assert proc.returncode == 0 and lines, proc.stdout[-3000:] + proc.stderr[-3000:]
    report = json.loads(lines[-1])
    assert report["passed"] and report["tp"] == 2, report
    assert len(report["checks"]) == 4  # 2 ranks x FUSED, PERSISTENT
