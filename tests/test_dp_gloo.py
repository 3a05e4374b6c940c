"""Data-parallel host logic on CPU: world-size-2 gloo ranks on 127.0.0.1.

* the NCCL id of trba_b200.dp.join reaches every rank and every rank calls
  dp_init(id, rank, world); max_over_ranks returns the largest step time;
* one data-parallel oracle step (per-rank batch statistics and scales,
  gradients averaged, identical optimiser step) leaves identical parameters
  on both ranks, equal to one process averaging the two shards' gradients —
  the semantics the library's NCCL all-reduce (ncclAvg over the flat
  gradient buffer) implements on the GPU;
* a rank that leaves between steps makes the other rank's next collective
  end with an error within the process-group timeout instead of hanging."""
import multiprocessing as mp
import socket
import sys

import numpy as np
import pytest

from conftest import REPO
import dp_workers as W

sys.path.insert(0, str(REPO / "oracle"))
import step_oracle as so  # noqa: E402


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(target, world, *args, timeout=240):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=target, args=(r, world, port, q, *args)) for r in range(world)]
    for p in procs:
        p.start()
    out = []
    try:
        for _ in range(world):
            out.append(q.get(timeout=timeout))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
                p.join()
    errs = [o for o in out if o[0] == "err"]
    assert not errs, errs[0][2]
    return sorted(out, key=lambda o: o[1])


def test_shard_splits_evenly():
    import trba_b200.dp as dp
    for gb, world in [(512, 1), (512, 8), (10, 4), (3, 4)]:
        parts = [dp.shard(gb, world, r) for r in range(world)]
        assert parts[0][0] == 0 and parts[-1][1] == gb
        assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
        sizes = [b - a for a, b in parts]
        assert max(sizes) - min(sizes) <= 1
    assert dp.rank_seed(7, 0) != dp.rank_seed(7, 1)
    with pytest.raises(ValueError):
        dp.shard(8, 2, 2)


def test_join_broadcasts_one_nccl_id():
    out = _run(W.join_worker, 2)
    ids = set()
    for _, rank, r, w, calls, mx in out:
        assert (r, w) == (rank, 2)
        assert len(calls) == 1 and calls[0][1:] == (rank, 2)
        ids.add(calls[0][0])
        assert mx == 11.0
    assert len(ids) == 1 and len(next(iter(ids))) == 128


@pytest.mark.slow
def test_two_rank_oracle_step_equals_one_process_average():
    geom = dict(img_w=64, max_len=4)
    cfg = so.Config(**geom)
    seed, per_rank = 31, 2
    shards = [so.make_batch(cfg, per_rank, seed=500 + r) for r in range(2)]
    out = _run(W.oracle_dp_worker, 2, geom, shards, seed, timeout=600)
    p0, p1 = out[0][3], out[1][3]
    assert np.array_equal(p0, p1), "ranks diverged after one data-parallel step"

    names = [n for n, _, _ in so.manifest(cfg)]
    be = so.CpuBackend(REPO / "oracle" / "liboracle.so")
    grads = []
    for r in range(2):
        orc = so.OracleTrba(cfg, so.init_params(cfg, seed), be)
        orc.train_step(*shards[r], optimize=False)
        grads.append({n: orc.g[n].copy() for n in names})
    orc = so.OracleTrba(cfg, so.init_params(cfg, seed), be)
    orc.train_step(*shards[0], optimize=False)
    for n in names:
        orc.g[n] = ((grads[0][n] + grads[1][n]) / np.float32(2)).astype(np.float32)
    orc.optimizer_step()
    want = np.concatenate([orc.p[n].ravel() for n in names]).astype(np.float32)
    assert np.array_equal(p0, want)


def test_rank_leaving_between_steps_ends_the_peer_collective_with_an_error():
    out = _run(W.failing_peer_worker, 2, timeout=120)
    r0 = out[0]
    assert r0[0] == "error", f"rank 0 expected an error, got {r0}"
    assert r0[2] < 60.0
    assert out[1][0] == "left"


# ------------------------------------------------ NCCL failure detection --
def _watch(lib, done_after=None, error_after=None, timeout_ms=1e9):
    """Runs trba_dp_watch over fake probes: the 'stream' finishes at poll
    done_after, the 'communicator' reports an error at poll error_after."""
    import ctypes as C
    polls, aborts = [0], [0]
    probe = C.CFUNCTYPE(C.c_int, C.c_void_p)
    hook = C.CFUNCTYPE(None, C.c_void_p)

    def done(_):
        polls[0] += 1
        return 1 if done_after is not None and polls[0] >= done_after else 0

    def err(_):
        return 5 if error_after is not None and polls[0] >= error_after else 0

    def abort(_):
        aborts[0] += 1

    cbs = (probe(done), probe(err), hook(abort))  # kept alive for the call
    rc = lib.trba_dp_watch(*(C.cast(c, C.c_void_p) for c in cbs), None, float(timeout_ms), 50.0)
    return rc, polls[0], aborts[0]


def test_watchdog_returns_when_the_step_finishes(lib):
    rc, polls, aborts = _watch(lib, done_after=4)
    assert (rc, polls, aborts) == (0, 4, 0)


def test_watchdog_aborts_on_a_communicator_error(lib):
    """A peer's failure surfaces as ncclCommGetAsyncError != ncclSuccess: the
    communicator is aborted once and the wait returns 1."""
    rc, polls, aborts = _watch(lib, error_after=3)
    assert (rc, aborts) == (1, 1) and polls == 3


def test_watchdog_aborts_a_step_that_never_finishes(lib):
    """A rank that never joins leaves the all-reduce waiting: after the
    timeout the communicator is aborted once and the wait returns 2."""
    import time
    t0 = time.perf_counter()
    rc, polls, aborts = _watch(lib, timeout_ms=30.0)
    assert (rc, aborts) == (2, 1) and polls > 1
    assert time.perf_counter() - t0 < 5.0
