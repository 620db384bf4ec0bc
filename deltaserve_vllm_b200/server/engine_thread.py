"""The engine loop on its own thread, driven by HTTP handlers.

Every engine mutation (adding/aborting requests, finetuning control, saves,
adapter operations) is a command executed by the engine thread between steps,
so the engine itself stays single-threaded. Handlers get the command's result
as an ``asyncio`` future. Request completion (and, for streaming, each new
token) is delivered to the handler's event loop thread-safely.

A request's arrival is also flagged immediately (before its ``add`` command
runs) so the step in flight can stop feeding the backward at its next layer
boundary: the in-process equivalent of the reference's shared-memory arrival
counter (``deltaserve-plugin/deltaserve/coordinator.py:64-115``).
"""

from __future__ import annotations

import asyncio
import concurrent.futures as cf
import queue
import threading
import time
import traceback
from dataclasses import dataclass

from .. import dprint


@dataclass
class _Waiter:
    loop: asyncio.AbstractEventLoop
    done: asyncio.Future
    tokens: asyncio.Queue | None = None  # streaming


class EngineThread:
    def __init__(self, engine, idle_sleep_s: float = 0.0005):
        self.engine = engine
        self.idle_sleep_s = idle_sleep_s
        self._cmds: queue.Queue = queue.Queue()
        self._waiters: dict[str, _Waiter] = {}
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, name="dsv-engine", daemon=True)
        self.error: str | None = None
        self.steps = 0
        engine.request_listeners.append(self._on_request_event)
        self._streamed: dict[str, int] = {}
        self._last_idle_tick = 0.0

    # ------------------------------------------------------------ lifecycle
    def start(self) -> None:
        self._thread.start()

    def stop(self, timeout: float = 30.0) -> None:
        self._stop.set()
        self._thread.join(timeout)

    @property
    def alive(self) -> bool:
        return self._thread.is_alive()

    # ------------------------------------------------------------ commands
    def submit(self, fn) -> cf.Future:
        """Run ``fn(engine)`` on the engine thread; returns a concurrent future."""
        fut: cf.Future = cf.Future()
        self._cmds.put((fn, fut))
        return fut

    async def call(self, fn):
        return await asyncio.wrap_future(self.submit(fn))

    def notify_arrival(self) -> None:
        self.engine.arrival_flag = True

    def register(self, request_id: str, stream: bool) -> _Waiter:
        loop = asyncio.get_running_loop()
        w = _Waiter(loop, loop.create_future(), asyncio.Queue() if stream else None)
        self._waiters[request_id] = w
        return w

    def unregister(self, request_id: str) -> None:
        self._waiters.pop(request_id, None)
        self._streamed.pop(request_id, None)

    # ------------------------------------------------------------ engine side
    def _on_request_event(self, kind: str, req) -> None:
        w = self._waiters.get(req.request_id)
        if w is None:
            return
        if kind == "finish":
            if w.tokens is not None:
                self._push_tokens(req, w)
                w.loop.call_soon_threadsafe(w.tokens.put_nowait, None)
            w.loop.call_soon_threadsafe(_set_result, w.done, req)

    def _push_tokens(self, req, w: _Waiter) -> None:
        sent = self._streamed.get(req.request_id, 0)
        new = req.output_ids[sent:]
        if new:
            self._streamed[req.request_id] = sent + len(new)
            w.loop.call_soon_threadsafe(w.tokens.put_nowait, list(new))

    def _stream_progress(self) -> None:
        for rid, w in list(self._waiters.items()):
            if w.tokens is None:
                continue
            req = self.engine.requests.get(rid)
            if req is not None:
                self._push_tokens(req, w)

    def _run(self) -> None:
        eng = self.engine
        while not self._stop.is_set():
            try:
                while True:
                    fn, fut = self._cmds.get_nowait()
                    if fut.set_running_or_notify_cancel():
                        try:
                            fut.set_result(fn(eng))
                        except BaseException as e:  # report to the caller
                            fut.set_exception(e)
            except queue.Empty:
                pass
            try:
                if eng.has_unfinished() or eng.has_ft_work():
                    eng.step()
                    self.steps += 1
                    if any(w.tokens is not None for w in self._waiters.values()):
                        self._stream_progress()
                else:
                    now = time.monotonic()
                    if now - self._last_idle_tick >= 0.01:
                        self._last_idle_tick = now
                        eng.idle_tick()
                    time.sleep(self.idle_sleep_s)
            except BaseException:
                self.error = traceback.format_exc()
                dprint("[engine-thread] step failed:\n" + self.error)
                time.sleep(0.05)


def _set_result(fut: asyncio.Future, value) -> None:
    if not fut.done():
        fut.set_result(value)
