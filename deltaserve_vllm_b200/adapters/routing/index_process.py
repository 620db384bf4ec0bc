"""Encoders for indexing that run in processes of their own.

An indexing job encodes a few thousand dataset samples to build an adapter's
centroid. Done on a thread of the serving process it would hold that
process's interpreter lock between the engine's launches; here every chunk
goes to a spawned child process instead, which answers over a pipe, one chunk
at a time (:class:`EncoderProcess`):

* the **CPU process** holds its own copy of the encoder (read from disk, or
  the hashing encoder) and lowers its own scheduling class when it starts:
  ``SCHED_IDLE`` where the kernel allows it, else ``nice 19``. It then only
  gets the CPU time that the serving process leaves. Each chunk says how many
  intra-op threads to use (few while inference runs, more when idle).
* the **GPU process** runs the route encoder's own parameters: the serving
  process sends them as CUDA tensors over the spawn pipe (CUDA IPC: the child
  maps the same device memory; nothing is copied) and the child rebuilds the
  module around them (:meth:`SentenceEncoder.from_shared`). It may compute
  only while the engine holds no inference request. :class:`IndexGrant` --
  one byte of shared memory that the serving process writes and the child
  reads -- is checked before every encoder layer; a cleared grant abandons
  the chunk at that layer and the reply is ``preempted`` (the samples are
  then encoded again on the CPU). A process and not a thread also keeps a
  failure there (an out-of-memory in a large chunk) out of the serving
  process, and its activations out of the serving process's allocator.

:class:`InlineExecutor` has the same interface and encodes in the caller's
thread (``adapter_routing.indexing_process: false``).

Reference behaviour: ``deltaserve-plugin/deltaserve/adapter_routing/index_process.py:1-90``
(the grant, the shared encoder, layer-granular preemption); the transport
here is a spawn pipe owned by the engine rather than a unix socket, because
the engine and the encoder's owner are the same process.
"""

from __future__ import annotations

import ctypes
import os
import time

import numpy as np

from ... import dprint


class Preempted(Exception):
    """The grant was cleared while the chunk was being encoded."""


class IndexGrant:
    """May the GPU indexing process compute? One byte of shared memory
    (an anonymous shared mapping handed to the child when it is spawned): the
    serving process writes it, the child reads it before every layer."""

    def __init__(self, ctx=None):
        import multiprocessing as mp
        self._v = (ctx or mp.get_context("spawn")).RawValue(ctypes.c_ubyte, 0)

    def set(self, granted: bool) -> None:
        self._v.value = 1 if granted else 0

    @property
    def granted(self) -> bool:
        return bool(self._v.value)


def lower_priority() -> str:
    """Put the calling process in the idle scheduling class (it runs only on
    otherwise idle CPUs), or at nice 19 where that is not permitted."""
    try:
        os.sched_setscheduler(0, os.SCHED_IDLE, os.sched_param(0))
        return "SCHED_IDLE"
    except (AttributeError, OSError):
        pass
    try:
        os.nice(19 - os.nice(0))
        return "nice 19"
    except OSError:
        return "unchanged"


def parse_cpus(spec) -> list[int] | None:
    """``"0-3,8,10-11"`` (or a list of ints) -> the CPU numbers; None for all."""
    if spec is None or spec == "":
        return None
    if isinstance(spec, (list, tuple)):
        return sorted({int(c) for c in spec})
    out: set[int] = set()
    for part in str(spec).split(","):
        part = part.strip()
        if not part:
            continue
        lo, _, hi = part.partition("-")
        a, b = int(lo), int(hi or lo)
        if b < a:
            raise ValueError(f"bad CPU range '{part}'")
        out.update(range(a, b + 1))
    return sorted(out)


def _install_grant_checks(encoder, grant: IndexGrant) -> int:
    """A pre-forward hook on every encoder layer that abandons the forward
    (raises :class:`Preempted`) once the grant is cleared."""
    layers = encoder.layers() if hasattr(encoder, "layers") else []

    def check(_mod, _args):
        if not grant.granted:
            raise Preempted()

    for layer in layers:
        layer.register_forward_pre_hook(check)
    return len(layers)


def _child_main(conn, encoder, device: str, shared: bool, grant, cpus, low_priority: bool) -> None:
    """The indexing process: build the encoder (with ``shared``, around the
    tensors that arrive as the pipe's first message), then answer
    ``("encode", seq, texts, threads)`` with ``("ok", seq, embeddings)``,
    ``("preempted", seq)`` or ``("error", seq, message)`` until ``("stop",)``
    or until the serving process goes away (the pipe closes)."""
    try:
        prio = lower_priority() if low_priority else "unchanged"
        if cpus:
            os.sched_setaffinity(0, cpus)
        if shared:
            from .encoder import SentenceEncoder
            _, config, state = conn.recv()
            encoder = SentenceEncoder.from_shared(encoder.path, encoder.prefix, encoder.max_tokens,
                                                  device, config, state)
            del state
        else:
            if hasattr(encoder, "device"):
                encoder.device = device
            if hasattr(encoder, "load"):
                encoder.load()
        checked = _install_grant_checks(encoder, grant) if grant is not None else 0
    except Exception as e:  # noqa: BLE001 -- reported to the parent, which raises
        conn.send(("error", 0, f"{type(e).__name__}: {e}"))
        return
    conn.send(("ready", os.getpid(), {"priority": prio, "layers_checked": checked, "device": device}))
    try:
        _serve(conn, encoder, grant)
    finally:
        # Drop every reference to tensors received from the parent before the
        # process ends (they live only in this frame and the encoder), so the
        # parent's CUDA IPC bookkeeping sees them released.
        encoder = None
        import gc
        gc.collect()
        if shared and str(device).startswith("cuda"):
            import torch
            torch.cuda.synchronize()


def _serve(conn, encoder, grant) -> None:
    threads_now = 0
    while True:
        try:
            msg = conn.recv()
        except (EOFError, OSError):
            return
        if msg[0] == "stop":
            return
        if msg[0] != "encode":
            continue
        _, seq, texts, threads = msg
        try:
            if grant is not None and not grant.granted:
                raise Preempted()
            if threads and threads != threads_now:
                import torch
                torch.set_num_threads(int(threads))
                threads_now = threads
            emb = np.asarray(encoder.encode(list(texts)), np.float32)
            reply = ("ok", seq, emb)
        except Preempted:
            reply = ("preempted", seq)
        except Exception as e:  # noqa: BLE001 -- the parent decides what a failed chunk means
            reply = ("error", seq, f"{type(e).__name__}: {e}")
        try:
            conn.send(reply)
        except (BrokenPipeError, OSError):
            return


class EncoderProcess:
    """Parent side of one indexing process: one chunk in flight at a time.

    ``encoder`` is an unloaded encoder object (it is pickled into the child,
    which loads it). ``shared`` = ``(config, state)`` from
    :meth:`SentenceEncoder.shared_state` makes the child run on those tensors
    instead (the GPU process). ``grant`` gates every layer of the child's
    forward."""

    def __init__(self, encoder, device: str = "cpu", shared=None, grant: IndexGrant | None = None,
                 cpus=None, low_priority: bool = True, name: str = "cpu",
                 start_timeout_s: float = 300.0, chunk_timeout_s: float = 600.0):
        self.encoder, self.device, self.shared, self.grant = encoder, device, shared, grant
        self.cpus, self.low_priority, self.name = parse_cpus(cpus), bool(low_priority), name
        self.start_timeout_s, self.chunk_timeout_s = float(start_timeout_s), float(chunk_timeout_s)
        self._proc = self._conn = None
        self._seq = 0
        self._inflight: int | None = None
        self._t_submit = 0.0
        self.info: dict = {}

    @property
    def ready(self) -> bool:
        return self._proc is not None and self._proc.is_alive()

    @property
    def pid(self) -> int | None:
        return self._proc.pid if self._proc is not None else None

    def start(self) -> "EncoderProcess":
        # torch's spawn context pickles tensors by sharing them (CUDA IPC
        # handles, shared-memory CPU storage), which the GPU process needs.
        import torch.multiprocessing as tmp
        ctx = tmp.get_context("spawn")
        parent, child = ctx.Pipe()
        self._proc = ctx.Process(target=_child_main, name=f"dsv-indexer-{self.name}", daemon=True,
                                 args=(child, self.encoder, self.device, self.shared is not None, self.grant,
                                       self.cpus, self.low_priority))
        self._proc.start()
        child.close()
        self._conn = parent
        if self.shared is not None:
            parent.send(("state", *self.shared))
        if not parent.poll(self.start_timeout_s):
            self.stop()
            raise RuntimeError(f"the {self.name} indexing process did not come up")
        try:
            msg = parent.recv()
        except EOFError:
            msg = ("error", 0, "the process exited while starting")
        if msg[0] != "ready":
            self.stop()
            raise RuntimeError(f"{self.name} indexing process: {msg[2]}")
        self.info = dict(msg[2], pid=msg[1])
        dprint(f"[indexing] {self.name} process pid={msg[1]} on {self.device} "
               f"({self.info['priority']}, {self.info['layers_checked']} layers gated)")
        return self

    def submit(self, texts: list[str], threads: int = 0) -> None:
        if self._inflight is not None:
            raise RuntimeError("a chunk is already in flight")
        if not self.ready:
            raise RuntimeError(f"the {self.name} indexing process is not running")
        self._seq += 1
        self._conn.send(("encode", self._seq, list(texts), int(threads)))
        self._inflight, self._t_submit = self._seq, time.monotonic()

    def poll(self, timeout: float = 0.0):
        """The chunk's embeddings once they are back, else None. Raises
        :class:`Preempted`, or RuntimeError when the chunk failed, the process
        exited, or it has not answered within ``chunk_timeout_s``."""
        if self._inflight is None:
            return None
        while True:
            if not self._conn.poll(timeout):
                if not self._proc.is_alive():
                    self._inflight = None
                    raise RuntimeError(f"the {self.name} indexing process exited "
                                       f"(code {self._proc.exitcode})")
                if time.monotonic() - self._t_submit > self.chunk_timeout_s:
                    self._inflight = None
                    raise RuntimeError(f"the {self.name} indexing process did not answer")
                return None
            try:
                reply = self._conn.recv()
            except (EOFError, OSError):
                self._inflight = None
                raise RuntimeError(f"the {self.name} indexing process exited") from None
            if reply[1] != self._inflight:
                timeout = 0.0               # the late answer of a cancelled chunk
                continue
            self._inflight = None
            if reply[0] == "ok":
                return reply[2]
            if reply[0] == "preempted":
                raise Preempted()
            raise RuntimeError(reply[2])

    def encode(self, texts: list[str], threads: int = 0):
        """Synchronous round trip (tests, warm-up)."""
        self.submit(texts, threads)
        while True:
            out = self.poll(0.05)
            if out is not None:
                return out

    def cancel(self) -> None:
        """Stop waiting for the chunk in flight (its answer is dropped when it comes)."""
        self._inflight = None

    def stop(self) -> None:
        proc, conn = self._proc, self._conn
        self._proc = self._conn = None
        self._inflight = None
        if conn is not None:
            try:
                conn.send(("stop",))
            except (BrokenPipeError, OSError):
                pass
        if proc is not None:
            proc.join(timeout=5.0)
            if proc.is_alive():
                proc.terminate()
                proc.join(timeout=3.0)
            if proc.is_alive():
                proc.kill()
                proc.join(timeout=3.0)
        if conn is not None:
            conn.close()
        if proc is not None and str(self.device).startswith("cuda"):
            import torch
            torch.cuda.ipc_collect()       # release the tensors the child held

    def describe(self) -> dict:
        return {"name": self.name, "device": self.device, "running": self.ready, **self.info}


class InlineExecutor:
    """The executor interface over an encoder in the calling thread."""

    device = "cpu"

    def __init__(self, encoder, name: str = "cpu"):
        self.encoder, self.name = encoder, name
        self._out = None
        self._err: Exception | None = None
        self._busy = False

    ready = True
    info: dict = {}

    def submit(self, texts: list[str], threads: int = 0) -> None:
        self._busy = True
        try:
            self._out, self._err = np.asarray(self.encoder.encode(list(texts)), np.float32), None
        except Exception as e:  # noqa: BLE001 -- raised by poll
            self._out, self._err = None, e

    def poll(self, timeout: float = 0.0):
        if not self._busy:
            return None
        self._busy = False
        if self._err is not None:
            raise RuntimeError(f"{type(self._err).__name__}: {self._err}")
        return self._out

    def encode(self, texts: list[str], threads: int = 0):
        self.submit(texts, threads)
        return self.poll()

    def cancel(self) -> None:
        self._busy = False

    def stop(self) -> None:
        pass

    def describe(self) -> dict:
        return {"name": self.name, "device": "cpu", "running": True, "inline": True}
