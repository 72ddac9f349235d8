"""Discrete-event model of tcgen05 kernels' synchronisation, for checking a kernel's barrier protocol on the CPU.

The kernels of this library coordinate their warps (TMA producer, MMA issuer, softmax / epilogue warps) through
shared-memory mbarriers waited on by phase parity, and through tcgen05.commit, which arrives on an mbarrier once
every MMA issued before it by the thread has completed. A protocol written as programs over these primitives
(`wait`, `arrive`, `mma`, `commit`, `tma`, `work`; for streams `waitge` / `write` on 32-bit flags and `copy`) runs
here under random latencies. The model checks:
  * every parity wait returns exactly at the completion it intends (a wait that passes on an older or newer phase
    of the same parity is an aliasing bug that a GPU would turn into a rare data race);
  * no program is left waiting (deadlock);
  * the data hazards a program asserts (through `complete(tag)`) at the moment it acts.
MMAs execute in issue order (as one thread's tcgen05.mma do); commit arrivals may be delayed by a random jitter,
so that the protocol is also checked when the arrivals of two commits land in the opposite order.
compute-sanitizer is not available on the GPU pool this library is tested on; this model is the race check of the
protocols instead (test infrastructure only).
"""
import heapq
import itertools
import random


class Bar:
    """An mbarrier: `count` arrivals complete a phase; k = phases completed so far."""

    def __init__(self, name, count=1):
        self.name, self.count, self.pending, self.k, self.waiters = name, count, count, 0, []

    def passes(self, c):
        # a wait for the c-th completion (c >= 1) waits on parity (c - 1) & 1 and passes when k & 1 differs from
        # it; c == 0 is a producer's first-use wait (parity 1 on a fresh barrier, passes at k = 0)
        par = ((c - 1) & 1) if c >= 1 else 1
        return (self.k & 1) != par


class Flag:
    """A 32-bit word waited on with ">= value" (a CUDA stream memory-operation flag, or an event's record count)."""

    def __init__(self, name, value=0):
        self.name, self.value, self.waiters = name, value, []


class Model:
    def __init__(self, seed, commit_jitter=0.0, tma_latency=(200.0, 1500.0)):
        self.rng = random.Random(seed)
        self.t = 0.0
        self._q = []
        self._seq = itertools.count()
        self._pipe_free = 0.0
        self.ops = {}        # MMA tag -> completion time
        self.issued = []     # MMA tags in issue order
        self.loaded = {}     # TMA tag -> landing time
        self.jitter = commit_jitter
        self.tma_latency = tma_latency
        self._done = 0
        self._agents = 0

    def at(self, t, fn):
        heapq.heappush(self._q, (t, next(self._seq), fn))

    def _arrive(self, bar):
        bar.pending -= 1
        assert bar.pending >= 0, f"{bar.name}: more arrivals than its count"
        if bar.pending == 0:
            bar.k += 1
            bar.pending = bar.count
            waiters, bar.waiters = bar.waiters, []
            for w in waiters:
                self.at(self.t, w)

    def complete(self, tag):
        """True once the MMA `tag` has completed."""
        t = self.ops.get(tag)
        return t is not None and t <= self.t

    def spawn(self, gen, name):
        self._agents += 1

        def step(val=None):
            try:
                cmd = gen.send(val)
            except StopIteration:
                self._done += 1
                return
            kind = cmd[0]
            if kind == "wait":
                bar, c = cmd[1], cmd[2]

                def check():
                    if bar.passes(c):
                        assert bar.k == c, f"{name}: wait on {bar.name} for completion {c} passed at {bar.k}"
                        self.at(self.t, step)
                    else:
                        bar.waiters.append(check)
                check()
            elif kind == "arrive":
                self._arrive(cmd[1])
                self.at(self.t, step)
            elif kind == "work":
                self.at(self.t + cmd[1], step)
            elif kind == "mma":
                start = max(self.t, self._pipe_free)
                self._pipe_free = start + cmd[2]
                self.ops[cmd[1]] = self._pipe_free
                self.issued.append(cmd[1])
                self.at(self.t + 1, step)
            elif kind == "commit":
                bar = cmd[1]
                t_arr = self._pipe_free + (self.rng.uniform(0, self.jitter) if self.jitter else 0.0)
                self.at(max(t_arr, self.t), lambda: self._arrive(bar))
                self.at(self.t + 1, step)
            elif kind == "waitge":
                flag, v = cmd[1], cmd[2]

                def check_flag():
                    if flag.value >= v:
                        self.at(self.t, step)
                    else:
                        flag.waiters.append(check_flag)
                check_flag()
            elif kind == "write":
                flag, v = cmd[1], cmd[2]
                assert v >= flag.value, f"{name}: {flag.name} moved back from {flag.value} to {v}"
                flag.value = v
                waiters, flag.waiters = flag.waiters, []
                for w in waiters:
                    self.at(self.t, w)
                self.at(self.t, step)
            elif kind == "copy":
                # ("copy", on_start, on_end, duration): a copy-engine transfer in stream order; the callbacks
                # check and update the state of the buffers it reads and writes
                cmd[1]()
                end = cmd[2]

                def finish():
                    end()
                    step()
                self.at(self.t + cmd[3], finish)
            elif kind == "tma":
                bar, tag = cmd[1], cmd[2]

                def land():
                    self.loaded[tag] = self.t
                    self._arrive(bar)
                self.at(self.t + self.rng.uniform(*self.tma_latency), land)
                self.at(self.t + 1, step)
            else:
                raise ValueError(kind)
        self.at(self.t, step)

    def run(self):
        while self._q:
            t, _, fn = heapq.heappop(self._q)
            self.t = t
            fn()
        assert self._done == self._agents, f"deadlock: {self._done} of {self._agents} programs finished"
        return self.t
