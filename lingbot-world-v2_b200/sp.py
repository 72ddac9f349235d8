"""Sequence (context) parallelism of the block: flat token shards + the K/V all-gather.

The reference's deployed CP mode (LINGBOT_CP_FLAT_SEQ=1, wan/modules/model_fast.py:1042-1079,
:2066-2108) gives rank r the contiguous run [r*L/P, (r+1)*L/P) of the chunk's frame-major tokens.
Every per-token op (norms, projections, FFN, cross-attention, FiLM) stays local; the one exchange is
the all-gather of the new chunk's K and V shards into every rank's destination chunk, in rank order,
so the cached chunks are replicated. Attention is not token-causal, so the local queries against the
full window are exact with no softmax reduction across ranks.

On CUDA the gather is PeerKV.gather: each rank stages its shard in a CUDA-IPC buffer and pulls the others'
with copy engines, synchronised by stream memory operations (liblbw's lbw_sp_kv_gather), so no SM is taken
from the attention it overlaps. gather_rows_inplace (one in-place all_gather_into_tensor per tensor) is the
same exchange through torch.distributed; the CPU (gloo) tests use it.

Failure detection is on the host: Liveness announces each rank's step in the process group's store so that a
rank learns of a failed, departed or stalled peer before it launches an exchange that would wait on it; an
exchange already waiting on a peer that stopped is released by PeerKV's watchdog after its timeout (PeerLost);
abort() tears the group down without the collective barrier. Collectives themselves end by the process group's
timeout.
"""
import ctypes

import torch
import torch.distributed as dist

_GROUP = None
_ACTIVE = False


def set_group(group=None, enable=True):
    """Shard the blocks' tokens over `group` (None = the default group) when enable is True."""
    global _GROUP, _ACTIVE
    _GROUP, _ACTIVE = group, bool(enable)


def active():
    return _ACTIVE and dist.is_available() and dist.is_initialized() and world() > 1


def world():
    return dist.get_world_size(_GROUP) if dist.is_initialized() else 1


def rank():
    return dist.get_rank(_GROUP) if dist.is_initialized() else 0


def shard_range(n_tokens, r=None, p=None):
    """[start, end) of rank r's contiguous token run; n_tokens must divide evenly."""
    p = world() if p is None else p
    r = rank() if r is None else r
    if n_tokens % p:
        raise ValueError(f"{n_tokens} tokens do not split evenly over {p} ranks")
    n = n_tokens // p
    return r * n, (r + 1) * n


def shard_tokens(x, dim=0):
    if not active():
        return x
    a, b = shard_range(x.shape[dim])
    return x.narrow(dim, a, b - a)


def gather_tokens(x, dim=0):
    """Inverse of shard_tokens: concatenate the ranks' runs along `dim`."""
    if not active():
        return x
    xs = x.movedim(dim, 0).contiguous()
    out = torch.empty((xs.shape[0] * world(),) + tuple(xs.shape[1:]), dtype=xs.dtype, device=xs.device)
    dist.all_gather_into_tensor(out, xs, group=_GROUP)
    return out.movedim(0, dim)


def gather_rows_inplace(dest2d, local_rows):
    """dest2d [P * local_rows, C]: rank r's rows [r*local_rows, (r+1)*local_rows) are filled; gather all."""
    if not active():
        return dest2d
    r = rank()
    if dest2d.shape[0] != local_rows * world():
        raise ValueError(f"destination chunk has {dest2d.shape[0]} rows, expected {local_rows} x {world()}")
    mine = dest2d[r * local_rows:(r + 1) * local_rows]
    if dist.get_backend(_GROUP) != "nccl":
        mine = mine.clone()
    dist.all_gather_into_tensor(dest2d, mine, group=_GROUP)
    return dest2d


def write_and_gather(shard, dest):
    """Write this rank's shard [L/P, n, d] into its rows of dest [1, L, n, d] and gather the rest."""
    d2 = dest.view(-1, dest.shape[-2] * dest.shape[-1])
    s2 = shard.reshape(-1, d2.shape[1])
    a = rank() * s2.shape[0] if active() else 0
    d2[a:a + s2.shape[0]].copy_(s2)
    gather_rows_inplace(d2, s2.shape[0])
    return dest


FLAG_BLOCK = 1024          # bytes of one rank's flag block (LBW_SP_FLAG_BLOCK in include/lbw.h)
_READY, _DONE, _GATHERED = 0, 64, 128   # word offsets inside a block


class PeerKV:
    """The copy-engine K/V exchange of one process group: this rank's IPC buffer plus the peers' buffers
    mapped into this process, and the group's flag blocks in a shared-memory segment of the node that every
    rank maps and registers with CUDA. Created collectively (every rank, same shapes); reused by every block.

    The streams of an exchange wait on flag words of this rank's own block (stream memory operations, which
    have no time limit of their own). A watchdog thread gives them one: when an exchange has been pending for
    timeout_s (LBW_SP_TIMEOUT_S, default 60) without any progress, it writes the awaited epochs into this rank's
    block, which lets the streams run on (the step's result is then invalid), and records PeerLost naming the
    ranks whose flags lagged; the next stage() / finish() / check() raises it, and abort() tears down."""

    def __init__(self, local_rows, cols, device, group=None, timeout_s=None):
        import mmap
        import os
        import threading
        from . import _lib
        self._lib = _lib
        lib = _lib.load()
        self.rows, self.cols, self.device, self.group = local_rows, cols, device, group
        self.rank, self.world = rank(), world()
        self.timeout_s = float(timeout_s if timeout_s is not None else os.environ.get("LBW_SP_TIMEOUT_S", "60"))
        nbytes = 4096 + 2 * local_rows * cols * 2
        own = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        with torch.cuda.device(device):
            _lib.check(lib.lbw_peer_buffer_create(nbytes, ctypes.byref(own), handle), "peer_buffer_create", 0)
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        ptrs = []
        with torch.cuda.device(device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    ptrs.append(own.value)
                    continue
                p = ctypes.c_void_p()
                _lib.check(lib.lbw_peer_buffer_open(ctypes.create_string_buffer(h, 64), ctypes.byref(p)),
                           f"peer_buffer_open(rank {r})", 0)
                ptrs.append(p.value)
        self._ptrs = (ctypes.c_void_p * self.world)(*ptrs)
        # flag blocks: a /dev/shm file made by the group's first rank, mapped by all, unlinked once all have it
        fbytes = max(4096, (self.world * FLAG_BLOCK + 4095) // 4096 * 4096)
        names = [None] * self.world
        name = f"/dev/shm/lbw_sp_{os.getpid()}_{id(self):x}" if self.rank == 0 else None
        if self.rank == 0:
            fd = os.open(name, os.O_CREAT | os.O_EXCL | os.O_RDWR, 0o600)
            os.ftruncate(fd, fbytes)
            os.close(fd)
        dist.all_gather_object(names, name, group=group)
        fd = os.open(names[0], os.O_RDWR)
        self._mm = mmap.mmap(fd, fbytes)
        os.close(fd)
        dist.barrier(group=group)
        if self.rank == 0:
            os.unlink(names[0])
        self._words = (ctypes.c_uint32 * (fbytes // 4)).from_buffer(self._mm)
        self._host = ctypes.addressof(self._words)
        dev_flags = ctypes.c_void_p()
        _lib.check(lib.lbw_host_flags_register(ctypes.c_void_p(self._host), fbytes, ctypes.byref(dev_flags)),
                   "host_flags_register", 0)
        self._flags = dev_flags
        self.epoch = 0
        self.failed = None
        self._stop = threading.Event()
        self._watchdog = threading.Thread(target=self._watch, name=f"lbw-sp-watchdog-{self.rank}", daemon=True)
        self._watchdog.start()

    def _word(self, owner, region, p):
        return owner * (FLAG_BLOCK // 4) + region + p

    def _release(self, epoch):
        """Write `epoch` into every ready/done word of this rank's block that is below it (host stores)."""
        for p in range(self.world):
            if p == self.rank:
                continue
            for region in (_READY, _DONE):
                i = self._word(self.rank, region, p)
                if self._words[i] < epoch:
                    self._words[i] = epoch

    def _watch(self):
        import time
        last, t_last = -1, time.monotonic()
        while not self._stop.wait(0.02):
            done = self._words[self._word(self.rank, _GATHERED, 0)]
            pending = self.epoch
            now = time.monotonic()
            if done != last or pending <= done:
                last, t_last = done, now
                continue
            if now - t_last > self.timeout_s and self.failed is None:
                lag = [p for p in range(self.world) if p != self.rank and
                       (self._words[self._word(self.rank, _READY, p)] < pending or
                        self._words[self._word(self.rank, _DONE, p)] < pending - 1)]
                self._release(pending)
                self.failed = PeerLost(f"K/V exchange {pending}: no progress for {self.timeout_s:.1f} s, waiting on "
                                       f"rank(s) {lag}; the pending exchanges were released (their results are "
                                       f"invalid)", lag)
            elif self.failed is not None:
                self._release(pending)   # exchanges enqueued after the failure must not wait either

    def check(self):
        """Raise the PeerLost the watchdog recorded, if any."""
        if self.failed is not None:
            raise self.failed

    def close(self, collective=True, timeout_s=30.0):
        """Release the exchange. collective=True: every rank's pulls have completed (device synchronisation +
        barrier) before the peers' mappings are closed and this rank's buffer is freed. collective=False (teardown
        after a lost peer, see abort()): no barrier; this rank's pending waits are released first and the device
        is waited for at most timeout_s; if it is still busy the buffers are left to the process's exit."""
        import threading
        if self._ptrs is None:
            return
        self._stop.set()
        self._watchdog.join(timeout=5)
        if collective:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
        else:
            self._release(max(self.epoch, 1))
            t = threading.Thread(target=torch.cuda.synchronize, args=(self.device,), daemon=True)
            t.start()
            t.join(timeout=timeout_s)
            if t.is_alive():
                self._ptrs = None
                return
        lib = self._lib.load()
        with torch.cuda.device(self.device):
            for r, p in enumerate(self._ptrs):
                self._lib.check(lib.lbw_peer_buffer_close(ctypes.c_void_p(p), int(r == self.rank)),
                                "peer_buffer_close", 0)
            self._lib.check(lib.lbw_host_flags_unregister(ctypes.c_void_p(self._host)), "host_flags_unregister", 0)
        self._ptrs = None
        del self._words
        self._mm.close()

    @property
    def gathered_flag(self):
        """Device address of this rank's 32-bit 'gathered' word: the epoch of the last completed exchange."""
        return self._ptrs[self.rank] + 512

    def fits(self, local_rows, cols, device):
        return (local_rows, cols, device) == (self.rows, self.cols, device)

    def _call(self, fn, k2d, v2d, stream):
        self._lib.check(getattr(self._lib.load(), fn)(
            self._ptrs, self._flags, self.rank, self.world, ctypes.c_uint(self.epoch),
            ctypes.c_void_p(k2d.data_ptr()), ctypes.c_void_p(v2d.data_ptr()), k2d.stride(0), self.rows, self.cols,
            ctypes.c_void_p(stream.cuda_stream)), fn, 0)

    def stage(self, k2d, v2d):
        """Start an exchange: this rank's rows of k2d, v2d ([world * local_rows, cols] bf16, row stride
        k2d.stride(0)) are copied to its buffer, in order on the current stream."""
        self.check()
        if k2d.shape != v2d.shape or k2d.shape[0] != self.rows * self.world or k2d.shape[1] != self.cols \
                or k2d.stride(0) != v2d.stride(0):
            raise ValueError(f"PeerKV: K/V {tuple(k2d.shape)} do not match {self.world} x {self.rows} rows")
        self.epoch += 1
        self._call("lbw_sp_kv_stage", k2d, v2d, torch.cuda.current_stream(self.device))

    def finish(self, k2d, v2d):
        """Complete the exchange begun by stage() on the current stream: the peers' rows land in k2d, v2d."""
        self.check()
        self._call("lbw_sp_kv_gather", k2d, v2d, torch.cuda.current_stream(self.device))

    def gather(self, k2d, v2d):
        """stage() + finish() on the current stream."""
        self.stage(k2d, v2d)
        self.finish(k2d, v2d)


_PEERS = {}


def peer_kv(k2d, local_rows):
    """The copy-engine exchange for destination chunks shaped like k2d (CUDA + NCCL group), else None. One per
    (group, device, shard shape), created collectively on first use."""
    if not (active() and k2d.is_cuda and dist.get_backend(_GROUP) == "nccl"):
        return None
    key = (id(_GROUP), world(), rank(), k2d.device, local_rows, k2d.shape[1])
    pk = _PEERS.get(key)
    if pk is None:
        pk = _PEERS[key] = PeerKV(local_rows, k2d.shape[1], k2d.device, _GROUP)
    return pk


def close_peers():
    """Collective: release every copy-engine exchange of this process (before destroying its process group)."""
    for key in list(_PEERS):
        _PEERS.pop(key).close()


def check_peers():
    """Raise PeerLost if the watchdog of an exchange of this process released a stalled exchange (its step's
    results are invalid); call after a step, before using its output."""
    for pk in _PEERS.values():
        pk.check()


class PeerLost(RuntimeError):
    """A rank of the group stopped taking part: it reported a failure, left, or missed a step's deadline."""

    def __init__(self, msg, ranks):
        super().__init__(msg)
        self.ranks = tuple(ranks)


class Liveness:
    """Between-step liveness of a group's ranks, kept in the process group's key-value store.

    A copy-engine exchange that a peer never joins is ended by PeerKV's watchdog (after its timeout, with an
    invalid step), but a rank should not launch the next step's exchange while a peer is known to be gone. Each
    rank calls beat(step) before a step's launches and wait(step) before its first exchange: wait returns once
    every rank has announced `step` (or a later one) and raises PeerLost, naming the ranks, when one has reported
    a failure (fail), left (leave) or not announced the step within `timeout_s`. Nothing here touches a GPU; only
    the store is used.
    """

    LEFT = -1

    def __init__(self, timeout_s=30.0, prefix="lbw/live", store=None, poll_s=0.005):
        import torch.distributed.distributed_c10d as c10d
        if not dist.is_initialized():
            raise RuntimeError("Liveness needs an initialised process group")
        if store is None:
            get = getattr(c10d, "_get_default_store", None)   # the store init_process_group created
            if get is None:
                raise RuntimeError("Liveness: this torch.distributed has no default store; pass store=")
            store = get()
        self.store = store
        self.timeout_s, self.poll_s, self.prefix = float(timeout_s), float(poll_s), prefix
        self.rank, self.world = rank(), world()
        self._ranks = (dist.get_process_group_ranks(_GROUP) if _GROUP is not None else list(range(self.world)))

    def _key(self, r, what="step"):
        return f"{self.prefix}/{what}/{self._ranks[r]}"

    def beat(self, step):
        """This rank starts `step` (a non-negative step counter that only grows)."""
        if step < 0:
            raise ValueError(f"step {step} < 0")
        self.store.set(self._key(self.rank), str(int(step)))

    def leave(self):
        """This rank leaves the group cleanly between steps; the others' next wait raises PeerLost."""
        self.store.set(self._key(self.rank), str(self.LEFT))

    def fail(self, reason):
        """Report this rank's failure (an exception between steps) to the others, then leave."""
        self.store.set(self._key(self.rank, "error"), str(reason)[:500])
        self.leave()

    def _peek(self, r):
        k = self._key(r)
        if not self.store.check([k]):
            return None
        return int(self.store.get(k))

    def wait(self, step):
        """Return when every rank has announced `step` or a later one; raise PeerLost otherwise (also when
        the store itself is gone, e.g. with the process that hosted it)."""
        try:
            return self._wait(step)
        except PeerLost:
            raise
        except (RuntimeError, OSError) as e:  # DistStoreError derives from RuntimeError
            raise PeerLost(f"step {step}: key-value store unreachable ({e})", ()) from e

    def _wait(self, step):
        import time
        deadline = time.monotonic() + self.timeout_s
        pending = [r for r in range(self.world) if r != self.rank]
        while True:
            lost, behind = [], []
            for r in pending:
                s = self._peek(r)
                if s == self.LEFT:
                    lost.append(r)
                elif s is None or s < step:
                    behind.append(r)
            if lost:
                why = []
                for r in lost:
                    ek = self._key(r, "error")
                    why.append(f"rank {r}: " + (self.store.get(ek).decode() if self.store.check([ek]) else "left"))
                raise PeerLost(f"step {step}: " + "; ".join(why), lost)
            if not behind:
                return
            if time.monotonic() > deadline:
                raise PeerLost(f"step {step}: rank(s) {behind} did not reach it within {self.timeout_s:.1f} s",
                               behind)
            pending = behind
            time.sleep(self.poll_s)


def abort(group=None):
    """Tear down after a PeerLost or a collective timeout: release the copy-engine exchanges without the
    collective barrier (the lost ranks would never reach it; exchanges still waiting on them are released and
    the device is waited for with a limit) and abort the process group, so no rank waits on a peer that is
    gone."""
    for key in list(_PEERS):
        _PEERS.pop(key).close(collective=False)
    if dist.is_initialized():
        import torch.distributed.distributed_c10d as c10d
        abort_pg = getattr(c10d, "_abort_process_group", None)
        if abort_pg is not None:
            abort_pg(group)          # ends the group's pending collectives without waiting for the lost ranks
        else:
            dist.destroy_process_group(group)


def gather_kv_inplace(k2d, v2d, local_rows):
    """All-gather the destination chunk's K and V rows (see gather_rows_inplace) on the current stream: over
    copy engines on CUDA with the NCCL backend, else through torch.distributed."""
    if not active():
        return
    pk = peer_kv(k2d, local_rows)
    if pk is not None:
        pk.gather(k2d, v2d)
        return
    gather_rows_inplace(k2d, local_rows)
    gather_rows_inplace(v2d, local_rows)
