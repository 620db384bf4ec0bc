"""One-to-many message channel for the step plans of tensor-parallel ranks on
one node, through POSIX shared memory.

Rank 0 pickles each batch of actions into a single shared slot and bumps a
sequence number; every follower spins (then naps) on the sequence number,
copies the payload out and acknowledges it. Rank 0 waits for every
acknowledgement of the previous message before it overwrites the slot, so
followers are never more than one message behind. A payload larger than the
slot travels through the fallback broadcast (the process group) instead, with
a marker in the slot. Every wait raises when the process it waits for has
exited (every rank records its pid in the header; the waiter checks it about
every 50 ms once it has started to nap). Waits on acknowledgements and votes
also end after ``timeout_s``; a follower's wait for the next plan has no time
limit by default (``recv_timeout_s``), since an idle server sends none.

This replaces a gloo/TCP ``broadcast_object_list`` per engine step (two
collectives, tens to hundreds of microseconds) with a memory copy; it plays
the role of the reference's shared-memory signals between processes on one box
(``deltaserve-plugin/deltaserve/coordinator.py:64-115``).
"""

from __future__ import annotations

import mmap
import os
import pickle
import platform
import time
import uuid

import numpy as np

_HDR = 8            # int64 words: [seq, length, via_fallback, ...], then per rank a message ack
_MAX_RANKS = 64     # word, a pid word and two vote words (one per parity)
_PID = _HDR + _MAX_RANKS
_VOTE = _HDR + 2 * _MAX_RANKS
_WORDS = _HDR + 4 * _MAX_RANKS
_DEFAULT = object()
_SHM_DIR = "/dev/shm" if os.path.isdir("/dev/shm") else "/tmp"


class ChannelUnavailable(RuntimeError):
    """Raised on every rank when any rank could not set up the segment."""


class ShmChannel:
    def __init__(self, comm, capacity: int = 8 << 20, timeout_s: float = 600.0, name: str | None = None,
                 recv_timeout_s: float | None = None):
        """Collective: every rank of ``comm`` constructs it (rank 0 creates the
        segment and shares its name through ``comm``). Raises
        ``ChannelUnavailable`` on every rank if any rank failed to map it."""
        self.comm = comm
        self.rank, self.size = comm.rank, comm.size
        if self.size > _MAX_RANKS:
            raise ValueError("too many ranks for the shared-memory channel")
        if platform.machine() not in ("x86_64", "AMD64"):
            # The payload-then-sequence publication relies on x86-64's total
            # store order; elsewhere the process group carries the plans (every
            # rank of one node takes this branch alike).
            raise ChannelUnavailable(f"shared-memory channel needs x86-64 store ordering, not {platform.machine()}")
        self.timeout_s = timeout_s
        # A follower waits for the next plan as long as rank 0 lives (an idle
        # server sends none); the pid check ends the wait if rank 0 exits.
        self.recv_timeout_s = recv_timeout_s
        self.header_bytes = _WORDS * 8
        size = self.header_bytes + capacity
        err = None
        self.buf = None
        if self.rank == 0:
            name = name or f"dsv_tp_{os.getpid()}_{uuid.uuid4().hex[:12]}"
            try:
                fd = os.open(os.path.join(_SHM_DIR, name), os.O_CREAT | os.O_EXCL | os.O_RDWR, 0o600)
                os.ftruncate(fd, size)
                self.buf = mmap.mmap(fd, size)
                os.close(fd)
            except OSError as e:
                err = e
        self.path = os.path.join(_SHM_DIR, comm.broadcast_object(name if self.rank == 0 else None))
        if self.rank != 0:
            try:
                fd = os.open(self.path, os.O_RDWR)
                self.buf = mmap.mmap(fd, size)
                os.close(fd)
            except OSError as e:
                err = e
        # every rank learns whether any rank failed, so all of them take the same path
        if comm.all_reduce_max_int(1 if err is not None else 0):
            if self.rank == 0:
                try:
                    os.unlink(self.path)
                except OSError:
                    pass
            if self.buf is not None:
                self.buf.close()
            raise ChannelUnavailable(f"shared-memory channel unavailable: {err!r}")
        self.name = name
        self.capacity = capacity
        self.words = np.ndarray((_WORDS,), dtype=np.int64, buffer=self.buf)
        if self.rank == 0:
            self.words[:] = 0
        comm.broadcast_object(None)      # header zeroed before anyone writes its pid
        self.words[_PID + self.rank] = os.getpid()
        self.seq = 0
        self.vseq = 0                    # votes taken
        comm.broadcast_object(None)      # every rank attached before the first message
        if self.rank == 0:
            # Every rank holds a mapping now: drop the name so nothing is left
            # behind in /dev/shm however the processes end.
            try:
                os.unlink(self.path)
            except OSError:
                pass

    def _gone(self, ranks) -> int | None:
        """The first of ``ranks`` whose process has exited, else None."""
        for r in ranks:
            pid = int(self.words[_PID + r])
            if pid <= 0:
                continue
            try:
                os.kill(pid, 0)
            except ProcessLookupError:
                return r
            except PermissionError:
                continue
            try:                     # an exited child that nobody has reaped yet
                with open(f"/proc/{pid}/stat", "rb") as f:
                    state = f.read().rsplit(b")", 1)[1].split()[0]
                if state in (b"Z", b"X"):
                    return r
            except (OSError, IndexError):
                pass
        return None

    def _wait(self, ready, ranks, spin: int, what: str, timeout_s=_DEFAULT) -> None:
        limit = self.timeout_s if timeout_s is _DEFAULT else timeout_s
        t0 = time.perf_counter()
        last_check = t0
        spins = 0
        while not ready():
            spins += 1
            if spins > spin:
                time.sleep(50e-6 if spins < 100 * spin else 1e-3)
                now = time.perf_counter()
                if now - last_check > 0.05:
                    last_check = now
                    dead = self._gone(ranks)
                    if dead is not None:
                        raise RuntimeError(f"shm channel: rank {dead} exited ({what})")
                    if limit is not None and now - t0 > limit:
                        raise TimeoutError(f"shm channel: timed out ({what})")

    # ------------------------------------------------------------ rank 0
    def send(self, obj) -> None:
        assert self.rank == 0
        w = self.words
        # the previous message has been read by every follower
        if self.seq > 0:
            seq, n = self.seq, self.size
            self._wait(lambda: int(w[_HDR + 1:_HDR + n].min()) >= seq, range(1, n), 200,
                       "a follower stopped reading step plans")
        data = pickle.dumps(obj, protocol=pickle.HIGHEST_PROTOCOL)
        if len(data) <= self.capacity:
            self.buf[self.header_bytes:self.header_bytes + len(data)] = data
            w[1] = len(data)
            w[2] = 0
            self.seq += 1
            w[0] = self.seq                  # published last
        else:
            w[1] = 0
            w[2] = 1
            self.seq += 1
            w[0] = self.seq
            self.comm.broadcast_object(obj)

    # ------------------------------------------------------------ followers
    def recv(self):
        assert self.rank != 0
        w = self.words
        want = self.seq + 1
        self._wait(lambda: int(w[0]) >= want, (0,), 2000, "waiting for a step plan from rank 0",
                   self.recv_timeout_s)
        self.seq = want
        if int(w[2]):
            w[_HDR + self.rank] = self.seq
            return self.comm.broadcast_object(None)
        n = int(w[1])
        data = bytes(self.buf[self.header_bytes:self.header_bytes + n])
        w[_HDR + self.rank] = self.seq       # acknowledged: rank 0 may overwrite the slot
        return pickle.loads(data)

    # ------------------------------------------------------------ host votes
    def all_max(self, flag: int) -> int:
        """Collective: the MAX of every rank's ``flag`` (0 or 1), the per-layer
        abort vote of an interruptible forward. Vote ``k`` of a rank is one
        store of ``2k + flag`` into its word of parity ``k & 1``; a rank reads
        the others' words of that parity once each shows vote ``k``. A rank
        can be at most one vote ahead of the slowest, so a word is never
        overwritten before every rank has read it."""
        w = self.words
        self.vseq += 1
        k = self.vseq
        base = _VOTE + (k & 1) * _MAX_RANKS
        w[base + self.rank] = 2 * k + (1 if flag else 0)
        n = self.size
        others = [r for r in range(n) if r != self.rank]
        self._wait(lambda: int((w[base:base + n] >> 1).min()) >= k, others, 2000,
                   "waiting for the other ranks' votes")
        return int((w[base:base + n] & 1).max())

    def close(self) -> None:
        try:
            self.words = None
            self.buf.close()
        except Exception:
            pass
