"""Drives one LLMEngine from a background thread so HTTP handlers (or any other
caller) can submit requests concurrently; continuous batching happens inside the
engine's step loop."""
from __future__ import annotations

import concurrent.futures as cf
import logging
import queue
import threading
from typing import List, Optional, Sequence

from ..engine import LLMEngine, Request, SamplingParams

log = logging.getLogger(__name__)


class EngineService:
    def __init__(self, engine: LLMEngine):
        self.engine = engine
        self._q: "queue.Queue[tuple]" = queue.Queue()
        self._pending = {}
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._loop, name="axr-engine", daemon=True)
        self._thread.start()

    def submit(self, prompt: Sequence[int], params: Optional[SamplingParams] = None,
               amf_prefix_len: Optional[int] = None) -> "cf.Future[Request]":
        fut: "cf.Future[Request]" = cf.Future()
        self._q.put((list(prompt), params or SamplingParams(), amf_prefix_len, fut))
        return fut

    def run_in_engine(self, fn, *args, **kwargs) -> "cf.Future":
        """Run ``fn(engine, *args, **kwargs)`` on the engine thread between steps (the way
        worker-API calls such as amf_save_kv reach the KV cache safely)."""
        fut: cf.Future = cf.Future()
        self._q.put(("__call__", (fn, args, kwargs), None, fut))
        return fut

    def _loop(self) -> None:
        eng = self.engine
        while not self._stop.is_set():
            try:
                block = not eng.has_unfinished()
                while True:
                    item = self._q.get(timeout=0.05 if block else 0.0) if block else self._q.get_nowait()
                    block = False
                    prompt, params, pre, fut = item
                    if isinstance(prompt, str) and prompt == "__call__":
                        fn, args, kwargs = params
                        try:
                            fut.set_result(fn(eng, *args, **kwargs))
                        except Exception as exc:
                            fut.set_exception(exc)
                        continue
                    try:
                        r = eng.add_request(prompt, params, amf_prefix_len=pre)
                        self._pending[r.req_id] = fut
                    except Exception as exc:
                        fut.set_exception(exc)
            except queue.Empty:
                pass
            if not eng.has_unfinished():
                continue
            try:
                done: List[Request] = eng.step()
            except Exception as exc:  # fail every in-flight request, keep serving
                log.exception("engine step failed")
                for fut in self._pending.values():
                    if not fut.done():
                        fut.set_exception(exc)
                self._pending.clear()
                eng.waiting.clear()
                for r in list(eng.running):
                    eng.bm.release(r.blocks)
                    eng.free_rows.append(r.row)
                eng.running.clear()
                continue
            for r in done:
                fut = self._pending.pop(r.req_id, None)
                if fut is not None and not fut.done():
                    fut.set_result(r)

    def close(self) -> None:
        self._stop.set()
        self._thread.join(timeout=5)
        self.engine.close()
