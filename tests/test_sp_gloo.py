"""Sequence-parallel host logic on 2 gloo ranks (CPU): token shards, the in-place K/V gather into the
destination chunk, and the sharded RoPE token offsets."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, ROOT)
    import __graft_entry__
    __graft_entry__.load_package()
    import lbw_b200.sp as sp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sp.set_group(None)
        assert sp.active() and sp.world() == world and sp.rank() == rank
        full = torch.arange(24 * 6, dtype=torch.float32).view(24, 6)
        mine = sp.shard_tokens(full)
        assert torch.equal(mine, full[rank * 12:(rank + 1) * 12])
        assert torch.equal(sp.gather_tokens(mine.clone()), full)
        dest = torch.full((24, 6), float("nan"))
        dest[rank * 12:(rank + 1) * 12] = mine
        sp.gather_rows_inplace(dest, 12)
        assert torch.equal(dest, full)
        d4 = torch.zeros(1, 24, 2, 3)
        sp.write_and_gather(mine.view(12, 2, 3), d4)
        assert torch.equal(d4.view(24, 6), full)
        q.put((rank, "ok"))
    except Exception as e:  # report instead of hanging the other rank
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_sequence_parallel_gather_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}
