"""Failure detection between data-parallel ranks, on the host (CPU, gloo, world size 2).

A rank that stalls, raises or never publishes the NCCL id must make the healthy rank fail with
PeerFailure within a bounded time, before it would launch a collective that cannot complete.
The failures are made on the host: a rank that blocks, raises or exits.  No GPU is involved.
"""
import os
import socket
import sys
import time

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
PKG = os.path.join(ROOT, "audiocraft.cpp_b200")

TIMEOUT_S = 3.0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port, scenario, out, release):
    sys.path.insert(0, PKG)
    from datetime import timedelta

    import torch.distributed as dist

    import dp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    group = dp.host_group(TIMEOUT_S)
    t0 = time.monotonic()
    try:
        if scenario == "no_id" and rank == 0:
            os._exit(0)  # rank 0 leaves before publishing the NCCL id
        uid = dp.share_nccl_id(group, rank, lambda: b"\x07" * 128)
        assert uid == b"\x07" * 128
        if scenario == "stall" and rank == 1:
            release.wait(60)  # stalls between steps until the healthy rank has given up on it
            os._exit(0)
        if scenario == "raise" and rank == 1:
            raise RuntimeError("simulated failure of this rank's step")
        dp.check_peers(group, TIMEOUT_S, "step 1")
        out[rank] = ("ok", time.monotonic() - t0)
    except dp.PeerFailure as e:
        out[rank] = ("peer_failure", time.monotonic() - t0, str(e)[:200])
        release.set()
    except RuntimeError as e:
        out[rank] = ("raised", time.monotonic() - t0, str(e)[:200])
    os._exit(0)  # no process-group teardown with a missing peer


def _run(scenario):
    import multiprocessing as mproc
    ctx = mproc.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    release = ctx.Event()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, scenario, out, release)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, f"{scenario}: a rank did not finish"
    return dict(out)


def test_healthy_ranks_share_the_id_and_pass_the_check():
    out = _run("ok")
    assert out[0][0] == "ok" and out[1][0] == "ok", out


def test_stalled_rank_is_reported_within_the_timeout():
    out = _run("stall")
    assert out[0][0] == "peer_failure", out
    assert out[0][1] < TIMEOUT_S + 20, out
    assert "1" in out[0][2]  # the missing rank is named


def test_rank_that_raised_is_reported():
    out = _run("raise")
    assert out[1][0] == "raised", out
    assert out[0][0] == "peer_failure", out
    assert out[0][1] < TIMEOUT_S + 20, out


def test_missing_nccl_id_is_reported():
    out = _run("no_id")
    assert out[1][0] == "peer_failure", out
    assert out[1][1] < 60, out
