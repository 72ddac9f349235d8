"""Failure detection of the sequence-parallel group, on gloo ranks (CPU; no GPU is faulted or hung).

Failures are made on the host, between steps, as the copy-engine exchange requires (it has no time limit
of its own): a rank that reports an error, a rank that exits without a word, and a rank that never joins a
collective. The surviving rank must learn of it before its next step's launches (sp.Liveness, through the
store) or from the process group's timeout, raise, and tear down with sp.abort() instead of waiting."""
import os
import socket
import time
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIVE_S = 2.0     # Liveness deadline
PG_S = 3         # process-group (collective) timeout


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q, mode):
    import sys
    sys.path.insert(0, ROOT)
    import __graft_entry__
    __graft_entry__.load_package()
    import lbw_b200.sp as sp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=PG_S))
    sp.set_group(None)
    live = sp.Liveness(timeout_s=LIVE_S)
    rows = 4
    t1 = None  # start of step 1: detection times are measured from here, not from start-up (step 0 included)
    try:
        for step in range(3):
            if step == 1:
                t1 = time.monotonic()
            if step == 1 and rank == world - 1:        # the failing rank, between steps 0 and 1
                if mode == "error":
                    live.fail("injected: out of memory while preparing step 1")
                    q.put((rank, "reported"))
                    return
                if mode == "exit":
                    q.put((rank, "exited"))
                    q.close()
                    q.join_thread()
                    os._exit(3)
                if mode == "skip":                     # announces the step, then never joins its gather
                    live.beat(step)
                    time.sleep(PG_S + 3)
                    q.put((rank, "skipped"))
                    return
            live.beat(step)
            live.wait(step)
            dest = torch.zeros(world * rows, 3)
            dest[rank * rows:(rank + 1) * rows] = rank + 1 + 10 * step
            sp.gather_rows_inplace(dest, rows)
            expect = torch.arange(world).repeat_interleave(rows)[:, None].float() + 1 + 10 * step
            assert torch.equal(dest, expect.expand_as(dest))
        q.put((rank, "ok"))
        dist.destroy_process_group()
    except sp.PeerLost as e:
        sp.abort()
        q.put((rank, ("PeerLost", e.ranks, str(e), time.monotonic() - (t1 if t1 is not None else 0.0))))
    except RuntimeError as e:
        sp.abort()
        q.put((rank, ("RuntimeError", (), str(e), time.monotonic() - (t1 if t1 is not None else 0.0))))


def _run(mode, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res, [p.exitcode for p in procs]


def test_healthy_group_runs_every_step():
    res, codes = _run("none", 2)
    assert res == {0: "ok", 1: "ok"} and codes == [0, 0]


@pytest.mark.parametrize("mode,world", [("error", 2), ("exit", 3)])
def test_lost_rank_is_detected_before_the_next_step(mode, world):
    res, codes = _run(mode, world)
    last = world - 1
    assert res[last] == {"error": "reported", "exit": "exited"}[mode]
    for r in range(last):
        kind, ranks, msg, took = res[r]
        assert kind == "PeerLost" and ranks == (last,), res[r]
        assert "step 1" in msg
        if mode == "error":
            assert "injected: out of memory" in msg and took < LIVE_S   # reported: no deadline needed
        else:
            assert "did not reach it" in msg and LIVE_S <= took < LIVE_S + 5
        assert codes[r] == 0
    assert codes[last] == (3 if mode == "exit" else 0)


def test_rank_missing_a_collective_ends_it_by_timeout():
    res, codes = _run("skip", 2)
    assert res[1] == "skipped"
    kind, _, msg, took = res[0]
    assert kind == "RuntimeError" and "Timed out" in msg, res[0]
    assert PG_S <= took < PG_S + 5
    assert codes == [0, 0]
