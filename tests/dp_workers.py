"""Child-process bodies of the data-parallel CPU tests (tests/test_dp_gloo.py):
gloo ranks on 127.0.0.1, started with the spawn method."""
from __future__ import annotations

import importlib.util
import os
import sys
import traceback
from datetime import timedelta
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent


def _package():
    name = "trba_b200"
    if name in sys.modules:
        return sys.modules[name]
    pkg = REPO / "trba-rust_b200"
    spec = importlib.util.spec_from_file_location(name, pkg / "__init__.py", submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def _init(rank, world, port, timeout_s=60):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))


class FakeModel:
    def __init__(self):
        self.calls = []

    def dp_init(self, id128, rank, world):
        self.calls.append((bytes(id128), rank, world))


def join_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        _package()
        from trba_b200 import dp
        import torch.distributed as dist
        m = FakeModel()
        r, w = dp.join(m, unique_id=lambda: os.urandom(128))
        mx = dp.max_over_ranks(10.0 * rank + 1.0)
        q.put(("ok", rank, r, w, m.calls, mx))
        dist.destroy_process_group()
    except Exception:
        q.put(("err", rank, traceback.format_exc()))


def oracle_dp_worker(rank, world, port, q, geom, shard_lines, seed):
    """One data-parallel step of the oracle on this rank's shard: gradients
    averaged over the gloo group (sum, then / world, in f32), then the
    optimiser step; returns the flat parameter vector."""
    try:
        _init(rank, world, port, timeout_s=300)
        import numpy as np
        import torch
        import torch.distributed as dist
        sys.path.insert(0, str(REPO / "oracle"))
        import step_oracle as so
        cfg = so.Config(**geom)
        names = [n for n, _, _ in so.manifest(cfg)]
        orc = so.OracleTrba(cfg, so.init_params(cfg, seed), so.CpuBackend(REPO / "oracle" / "liboracle.so"))
        img, ti, tg, ct = shard_lines[rank]
        res = orc.train_step(img, ti, tg, ct, optimize=False)
        flat = torch.from_numpy(np.concatenate([orc.g[n].ravel() for n in names]).astype(np.float32))
        dist.all_reduce(flat, op=dist.ReduceOp.SUM)
        flat = (flat / world).numpy()
        off = 0
        for n in names:
            k = orc.g[n].size
            orc.g[n] = flat[off:off + k].reshape(orc.g[n].shape).astype(np.float32)
            off += k
        orc.optimizer_step()
        params = np.concatenate([orc.p[n].ravel() for n in names]).astype(np.float32)
        q.put(("ok", rank, res["loss"], params))
        dist.destroy_process_group()
    except Exception:
        q.put(("err", rank, traceback.format_exc()))


def failing_peer_worker(rank, world, port, q):
    """Rank 1 leaves between steps without joining the next collective;
    rank 0's all-reduce must end with an error, not wait forever."""
    import time
    try:
        _init(rank, world, port, timeout_s=5)
        import torch
        import torch.distributed as dist
        t = torch.ones(4)
        dist.all_reduce(t)  # one good step on both ranks
        if rank == 1:
            q.put(("left", rank))
            q.close()
            q.join_thread()  # flush the message before leaving
            os._exit(0)  # leaves without destroy_process_group
        t0 = time.monotonic()
        try:
            dist.all_reduce(t)
            q.put(("no-error", rank, time.monotonic() - t0))
        except Exception as e:  # noqa: BLE001 - any error is the expected outcome
            q.put(("error", rank, time.monotonic() - t0, type(e).__name__))
    except Exception:
        q.put(("err", rank, traceback.format_exc()))
