"""Replica coordination (breeze_b200.replicas) with real processes, on the CPU.

Two replica processes meet at a start line, work, and gather their results at
rank 0, as bench.py's multi-GPU run does. The failure cases take a replica
away between those steps -- it exits, or it hangs -- and check that the
surviving rank still finishes within its deadline and reports the missing
rank as failed. No GPU is involved: the failure is made on the host.
"""

import multiprocessing as mp
import os
import socket
import time

import pytest

from conftest import PKG_ROOT, ROOT


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _replica(rank, world, port, mode, out):
    import sys

    for p in (str(ROOT), str(PKG_ROOT)):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.pop("TORCHELASTIC_USE_AGENT_STORE", None)
    from breeze_b200.replicas import ReplicaGroup

    try:
        grp = ReplicaGroup(rank, world, "127.0.0.1", port, timeout_s=3.0, prefix=f"t{port}")
    except Exception as e:  # noqa: BLE001 - e.g. the port was taken between choosing and binding it
        if rank == 0:
            out.put({"store_error": repr(e)})
        return
    started = grp.meet("start", timeout_s=120.0)  # process start-up (imports) is not what is tested
    time.sleep(0.05)  # the replica's own work
    if rank == 1 and mode == "exit":
        os._exit(3)
    if rank == 1 and mode == "hang":
        time.sleep(60)
    t0 = time.monotonic()
    got = grp.gather("result", {"rank": rank, "value": 10.0 * (rank + 1)})
    waited = time.monotonic() - t0
    if rank == 0:
        out.put({"started": started, "got": got, "failed": sorted(grp.failed), "waited": waited})
    grp.close()  # rank 0 hosts the store: it stays until the others have left


def _run(mode, attempts=3):
    ctx = mp.get_context("spawn")
    for _ in range(attempts):
        out = ctx.Queue()
        port = _free_port()
        procs = [ctx.Process(target=_replica, args=(r, 2, port, mode, out)) for r in range(2)]
        for p in procs:
            p.start()
        res = out.get(timeout=120)
        procs[0].join(30)
        for p in procs:
            if p.is_alive():
                p.kill()
            p.join(10)
        if "store_error" not in res:  # a port taken by someone else: choose another
            return res, procs[0].exitcode, procs[1].exitcode
    raise AssertionError(f"no free port for the replica store: {res}")


def test_replicas_all_arrive():
    res, rc0, rc1 = _run("ok")
    assert res["started"] == [0, 1]
    assert res["got"] == {0: {"rank": 0, "value": 10.0}, 1: {"rank": 1, "value": 20.0}}
    assert res["failed"] == [] and rc0 == 0 and rc1 == 0


@pytest.mark.parametrize("mode", ["exit", "hang"])
def test_surviving_replica_finishes_and_reports_the_lost_one(mode):
    res, rc0, rc1 = _run(mode)
    assert res["started"] == [0, 1]
    assert list(res["got"]) == [0] and res["failed"] == [1]
    assert res["waited"] < 10.0  # the deadline, not the lost rank, ended the wait
    assert rc0 == 0
    assert rc1 == (3 if mode == "exit" else -9)
