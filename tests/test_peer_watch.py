"""Host-side failure detection for tensor parallelism (PeerWatch), on CPU:
two processes share a TCPStore on 127.0.0.1; rank 1 fails on the host in
one of three ways (it leaves between steps, it dies without a word, or it
never joins) while rank 0 keeps stepping. Rank 0 must learn of it before
its next launch and abort its engine (a stand-in object here that records
the call), and two healthy ranks must never see a false alarm."""
import multiprocessing as mp
import os
import socket
import time

import pytest

from conftest import PKG


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _FakeEngine:
    def __init__(self):
        self.aborted = 0

    def abort(self):
        self.aborted += 1


def _rank(rank, port, mode, out):
    import sys

    sys.path.insert(0, os.path.join(PKG, "python"))
    from torch.distributed import TCPStore

    import q4kb200 as q

    store = TCPStore("127.0.0.1", port, 2, rank == 0, timeout=__import__("datetime").timedelta(seconds=30))
    if rank == 1:
        if mode == "never":
            return  # connected to the store, never beats
        watch = q.PeerWatch(store, 1, 2, timeout_s=1.0)
        for _ in range(5):
            watch.beat()
            watch.check()
            time.sleep(0.05)
        if mode == "leave":
            watch.leave()
            return
        if mode == "die":
            os._exit(0)  # no goodbye
        # healthy: keep stepping until rank 0 says it is done
        while not store.check(["done"]):
            watch.beat()
            watch.check()
            time.sleep(0.05)
        return
    eng = _FakeEngine()
    watch = q.PeerWatch(store, 0, 2, timeout_s=1.0, engine=eng)
    t0 = time.monotonic()
    result = {"lost": None, "steps": 0, "aborted": 0}
    try:
        while time.monotonic() - t0 < (3.0 if mode == "healthy" else 10.0):
            watch.beat()
            watch.check()  # before the next launch
            result["steps"] += 1
            time.sleep(0.05)
    except q.PeerLost as e:
        result["lost"] = str(e)
        result["after_s"] = time.monotonic() - t0
    result["aborted"] = eng.aborted
    store.set("done", "1")
    out.put(result)


def _run(mode):
    ctx = mp.get_context("spawn")
    port = _free_port()
    out = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, port, mode, out)) for r in (0, 1)]
    for p in procs:
        p.start()
    res = out.get(timeout=60)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return res


@pytest.mark.parametrize("mode", ["leave", "die", "never"])
def test_lost_peer_is_detected_before_the_next_launch(mode):
    res = _run(mode)
    assert res["lost"] is not None, res
    assert res["aborted"] == 1, res
    if mode == "leave":
        assert "left" in res["lost"]
        assert res["after_s"] < 3.0, res
    else:
        # no word from the peer: found once its beat is older than the limit
        assert "has not beaten" in res["lost"]
        assert res["after_s"] < 6.0, res


def test_healthy_peers_raise_nothing():
    res = _run("healthy")
    assert res["lost"] is None, res
    assert res["aborted"] == 0
    assert res["steps"] > 20
