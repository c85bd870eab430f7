"""One-item lookahead between a prefill worker and the decode loop.

Same contract as `ordered_prefetch_map` of the reference engine (prefilling_dllm_engine/prefilling_dllm/pd_pipeline.py:22-63,
exercised by its tests/test_pd_pipeline.py): item 0 is prepared first; while item i is being consumed, item i + 1 is
prepared on a worker thread named `pd-prefetch*`; results come back in input order; if consuming fails (or the
generator is closed), a prefetched item that was or is being prepared is handed to `release_prepared` so its KV pages
go back to the allocator, and one that has not started is dropped.

The worker is a plain thread fed through a queue, one per call, so a prefill that raised does not poison a pool.
"""

from __future__ import annotations

import queue
import threading
from typing import Callable, Iterable, Iterator, Optional, TypeVar

ItemT = TypeVar("ItemT")
PreparedT = TypeVar("PreparedT")
ResultT = TypeVar("ResultT")

_worker_serial = 0
_serial_lock = threading.Lock()


class _Job:
    """One background preparation: not started → running → done (value or error), or cancelled before it started."""

    def __init__(self, fn: Callable, item) -> None:
        self._fn, self._item = fn, item
        self._lock = threading.Lock()
        self._done = threading.Event()
        self._started = False
        self._cancelled = False
        self._value = None
        self._error: Optional[BaseException] = None

    def run(self) -> None:
        with self._lock:
            if self._cancelled:
                return
            self._started = True
        try:
            self._value = self._fn(self._item)
        except BaseException as exc:  # handed to whoever waits for the result
            self._error = exc
        finally:
            self._done.set()

    def cancel(self) -> bool:
        """True if the job will never run."""
        with self._lock:
            if self._started:
                return False
            self._cancelled = True
            self._done.set()
            return True

    def result(self):
        self._done.wait()
        if self._error is not None:
            raise self._error
        return self._value


def _worker_loop(jobs: "queue.Queue[Optional[_Job]]") -> None:
    while True:
        job = jobs.get()
        if job is None:
            return
        job.run()


def ordered_prefetch_map(items: Iterable[ItemT], *, prepare: Callable[[ItemT], PreparedT],
                         consume: Callable[[ItemT, PreparedT], ResultT],
                         release_prepared: Optional[Callable[[PreparedT], None]] = None) -> Iterator[ResultT]:
    """Yield `consume(item, prepare(item))` in input order, preparing the next item while the current one is consumed."""
    iterator = iter(items)
    try:
        current_item = next(iterator)
    except StopIteration:
        return
    global _worker_serial
    with _serial_lock:
        serial = _worker_serial
        _worker_serial += 1
    jobs: "queue.Queue[Optional[_Job]]" = queue.Queue()
    worker = threading.Thread(target=_worker_loop, args=(jobs,), name=f"pd-prefetch_{serial}", daemon=True)
    worker.start()
    try:
        current = _Job(prepare, current_item)
        jobs.put(current)
        while True:
            prepared = current.result()
            upcoming: Optional[_Job] = None
            try:
                next_item = next(iterator)
            except StopIteration:
                pass
            else:
                upcoming = _Job(prepare, next_item)
                jobs.put(upcoming)
            try:
                yield consume(current_item, prepared)
            except BaseException:
                if upcoming is not None and release_prepared is not None and not upcoming.cancel():
                    release_prepared(upcoming.result())
                elif upcoming is not None:
                    upcoming.cancel()
                raise
            if upcoming is None:
                return
            current_item, current = next_item, upcoming
    finally:
        jobs.put(None)
        worker.join()
