"""Failure handling of the sequence-parallel K/V exchange on 2 GPUs (skipped with fewer), with no GPU faulted or
hung: the failures are made on the host, between steps.

* A rank leaves between steps (Liveness.leave): the survivor learns of it from the store before it launches the
  next exchange (PeerLost) and tears down with sp.abort().
* A rank stops taking part between steps without a word, so the survivor's next exchange waits on flags that
  rank never writes: the exchange's watchdog releases the waiting streams after its timeout, the survivor's
  device work finishes, check() raises PeerLost naming the rank, and sp.abort() tears down.
The silent rank stays alive (its buffers stay mapped) until the survivor has torn down. NVLS is off."""
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q, survivor_done):
    import sys
    from datetime import timedelta
    sys.path.insert(0, ROOT)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import __graft_entry__
    __graft_entry__.load_package()
    import torch.distributed as dist
    import lbw_b200.sp as sp
    try:
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        sp.set_group(None, enable=True)
        live = sp.Liveness(timeout_s=20.0)
        rows, cols = 256, 512
        k = torch.zeros(world * rows, cols, dtype=torch.bfloat16, device=dev)
        v = torch.zeros_like(k)
        pk = sp.PeerKV(rows, cols, dev, timeout_s=1.0)
        sp._PEERS[("test", rank)] = pk            # so that sp.abort() releases it
        # step 0: both ranks exchange
        live.beat(0)
        live.wait(0)
        k[rank * rows:(rank + 1) * rows] = rank + 1
        v[rank * rows:(rank + 1) * rows] = -(rank + 1)
        pk.gather(k, v)
        torch.cuda.synchronize()
        pk.check()
        ok0 = bool((k[:rows] == 1).all() and (k[rows:] == 2).all() and (v[rows:] == -2).all())
        if rank == 1:
            if mode == "leave":
                live.leave()                       # between steps, announced
            # "silent": no word, no exchange; stay alive until the survivor has torn down
            survivor_done.wait(timeout=120)
            sp.abort()
            q.put((rank, "ok" if ok0 else "bad step 0"))
            return
        # rank 0, step 1
        t0 = time.monotonic()
        if mode == "leave":
            live.beat(1)
            try:
                live.wait(1)
                q.put((rank, "PeerLost not raised"))
            except sp.PeerLost as e:
                sp.abort()
                q.put((rank, "ok" if ok0 and e.ranks == (1,) and time.monotonic() - t0 < 10 else f"late {e}"))
        else:
            pk.gather(k, v)                        # waits on rank 1's flags, which never come
            torch.cuda.synchronize()               # ends once the watchdog has released the exchange
            waited = time.monotonic() - t0
            try:
                pk.check()
                q.put((rank, "PeerLost not raised"))
            except sp.PeerLost as e:
                sp.abort()
                q.put((rank, "ok" if ok0 and e.ranks == (1,) and 0.5 < waited < 30 else f"{e} after {waited:.1f}s"))
        survivor_done.set()
    except Exception as e:  # noqa: BLE001
        survivor_done.set()
        q.put((rank, repr(e)))


@pytest.mark.parametrize("mode", ["leave", "silent"])
def test_rank_stops_between_steps(mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    done = ctx.Event()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q, done)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = dict(q.get(timeout=240) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert res == {0: "ok", 1: "ok"}, res
