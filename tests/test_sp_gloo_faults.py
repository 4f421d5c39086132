"""Failures around the sequence-parallel exchange, injected on the host among CPU ranks (gloo):
a rank that leaves between steps, a rank that arrives late, and a corrupted shard state.  In each
case the other ranks must end with an error within the process group's timeout instead of waiting
for good.  The per-rank compute is the float64 oracle (tests/test_sp_gloo.py's stand-in), so no
GPU is touched."""
import datetime
import os
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from test_sp_gloo import OracleKernels, _case, _free_port

TIMEOUT_S = 4


def _step(sp, q, k, v, lam, lens, rank, validate=False):
    a = sum(lens[:rank])
    sl = slice(a, a + lens[rank])
    return sp.sequence_parallel_prefill(q[:, :, sl].contiguous(), k[:, :, sl].contiguous(), v[:, :, sl].contiguous(),
                                        lam, shard_lengths=lens, kernels=OracleKernels, validate=validate)


def _worker(rank, world, port, mode, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=TIMEOUT_S))
    from prime_moment_attention_b200 import sp
    lens = [16, 24]
    q, k, v, lam = _case(5, 1, 2, sum(lens), 8)
    result = {"steps": 0, "error": None, "seconds": None}
    try:
        _step(sp, q, k, v, lam, lens, rank)  # a good first step on every rank
        result["steps"] = 1
        if mode == "leave" and rank == 1:
            out[rank] = dict(result, left=True)
            os._exit(0)  # between steps, with nothing in flight
        if mode == "late" and rank == 1:
            time.sleep(TIMEOUT_S + 3)
        if mode == "corrupt" and rank == 1:
            q, k, v = q, k * float("nan"), v  # this rank's shard state becomes NaN
        t0 = time.monotonic()
        try:
            _step(sp, q, k, v, lam, lens, rank, validate=(mode == "corrupt"))
            result["steps"] = 2
        except Exception as e:  # the injected failure, as the surviving ranks see it
            result["error"] = type(e).__name__ + ": " + str(e)[:200]
        result["seconds"] = time.monotonic() - t0
        out[rank] = result
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(mode):
    out = mp.Manager().dict()
    t0 = time.monotonic()
    mp.start_processes(_worker, args=(2, _free_port(), mode, out), nprocs=2, start_method="spawn", join=True)
    return dict(out), time.monotonic() - t0


def test_rank_leaving_between_steps_fails_the_next_exchange():
    out, _ = _run("leave")
    assert out[1].get("left")
    r0 = out[0]
    assert r0["steps"] == 1 and r0["error"] is not None, r0
    assert r0["seconds"] < TIMEOUT_S + 10, r0


def test_late_rank_times_out_the_others():
    out, wall = _run("late")
    r0 = out[0]
    assert r0["steps"] == 1 and r0["error"] is not None, r0
    assert TIMEOUT_S - 1 < r0["seconds"] < TIMEOUT_S + 10, r0  # ended by the process group's timeout
    assert out[1]["error"] is not None  # the late rank finds its peer gone
    assert wall < 60


def test_corrupted_shard_state_is_refused_on_every_rank():
    out, _ = _run("corrupt")
    for r in (0, 1):
        assert out[r]["steps"] == 1 and out[r]["error"] is not None and "rank(s) [1]" in out[r]["error"], out[r]
