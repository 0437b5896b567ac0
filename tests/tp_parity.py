"""Tensor-parallel parity run: one stream over every rank's GPU, checked
against the CPU oracle (launched by tests/test_gpu_tp.py under
torch.distributed.run, one rank per GPU; also usable by hand:

    python -m torch.distributed.run --standalone --nproc-per-node 2 tests/tp_parity.py --config c5-large-fp32

Every rank starts from the same seeded random state past the window (the
state hand-off of long-run validation), steps the same events on the
FUSED backend (one collective launch per event) and then on a PERSISTENT
worker, and rank 0 checks: every rank's scores against the oracle's, every
rank's own heads' K and V rows and the full hidden state. Prints one JSON line
on rank 0 and exits non-zero on a mismatch.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))


def main() -> int:
    import torch
    import torch.distributed as dist

    from oracle.oracle import Oracle
    from policy import score_errors, state_errors, fp32_relative_errors
    from streaming_transformer_b200 import Backend, Runtime, RuntimeOptions, synthetic
    from streaming_transformer_b200.model import round_storage
    from streaming_transformer_b200.tp import torch_tensor_parallel

    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="c5-large-fp32", choices=sorted(synthetic.CONFIGS))
    ap.add_argument("--events", type=int, default=6)
    a = ap.parse_args()

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=timedelta(seconds=120))
    rank, world = dist.get_rank(), dist.get_world_size()
    config, mode = synthetic.CONFIGS[a.config]
    model = synthetic.make_model(config, mode, seed=61)
    events = synthetic.make_events(2 * a.events, config.features, seed=62)
    rng = np.random.default_rng(63)
    shape = (config.layers, config.heads, config.window, config.head_dim)
    keys = round_storage(rng.normal(0.0, 0.6, shape).astype(np.float32), mode)
    values = round_storage(rng.normal(0.0, 0.6, shape).astype(np.float32), mode)
    hidden = np.zeros((config.layers, config.width), dtype=np.float32)
    position = config.window + 41

    tp = torch_tensor_parallel()
    got = {}
    snaps = {}
    for backend in (Backend.FUSED, Backend.PERSISTENT):
        rt = Runtime(model, RuntimeOptions(backend=backend, blocks=0, device=local), tp=tp)
        try:
            info = rt.info()
            if backend == Backend.PERSISTENT:
                rt.stop()  # state is loaded with the worker stopped, then a new one starts
            rt.load_state(position, keys, values, hidden)
            if backend == Backend.PERSISTENT:
                rt.start_worker()
            dist.barrier()
            got[backend.name] = np.array([rt.step(e) for e in events[: a.events]], dtype=np.float32)
            snaps[backend.name] = rt.snapshot()
            dist.barrier()
        finally:
            rt.close()
    # every rank's results to rank 0
    payload = {name: (got[name], snaps[name].keys, snaps[name].values, snaps[name].hidden, snaps[name].position)
               for name in got}
    gathered = [None] * world
    dist.all_gather_object(gathered, payload)
    ok = True
    report = {"config": a.config, "tp": world, "kernel": info.get("resource_kernel"),
              "cluster": info.get("cluster"), "clusters": info.get("clusters"), "checks": []}
    if rank == 0:
        o = Oracle(model)
        o.load_state(position, keys, values, hidden)
        want = np.array([o.step(e) for e in events[: a.events]], dtype=np.float32)
        wk, wv, wh = o.keys(), o.values(), o.hidden()
        hl = config.heads // world
        for r, result in enumerate(gathered):
            for name, (scores, k, v, h, pos) in result.items():
                sc = score_errors(scores, want, config.layers, mode)
                check = {"rank": r, "backend": name, "score_max_abs": sc["max_abs"], "position_ok": pos == o.position}
                passed = sc["passed"] and pos == o.position
                if mode == "fp32":
                    rel = fp32_relative_errors(scores, want)
                    check["score_relative_l2"] = rel["relative_l2"]
                    passed = passed and rel["passed"]
                own = slice(r * hl, (r + 1) * hl)
                for label, actual, ref in (("keys", k[:, own], wk[:, own]), ("values", v[:, own], wv[:, own]),
                                           ("hidden", h[:, None, :], wh[:, None, :])):
                    for layer in range(config.layers):
                        e = state_errors(actual[layer], ref[layer], layer, mode)
                        good = e["passed"]
                        if mode == "fp32":
                            good = good and fp32_relative_errors(actual[layer], ref[layer])["passed"]
                        if not good:
                            passed = False
                            check.setdefault("failed", []).append(f"{label} layer {layer}: {e}")
                check["passed"] = passed
                ok = ok and passed
                report["checks"].append(check)
        report["passed"] = ok
        print(json.dumps(report), flush=True)
    flag = torch.tensor([1 if ok else 0])
    dist.broadcast(flag, 0)
    dist.destroy_process_group()
    return 0 if int(flag.item()) == 1 else 2


if __name__ == "__main__":
    sys.exit(main())
