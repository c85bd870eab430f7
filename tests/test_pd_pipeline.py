"""Host-side PD plumbing: the lookahead pipeline and the per-thread context (CPU only).

Same scenarios as the reference engine's tests/test_pd_pipeline.py: the next item is prepared while the current one is
consumed, a prefetched record is released when decoding fails, and forward contexts do not leak between threads.
"""

import queue
import threading

import pytest

from prefilling_dllm_b200.context import get_context_diffusion_lm, reset_context_diffusion_lm, set_context_diffusion_lm
from prefilling_dllm_b200.pd_pipeline import ordered_prefetch_map


def test_next_item_is_prepared_while_current_is_consumed():
    events = queue.Queue()
    second_prepared = threading.Event()
    names = []
    released = []

    def prepare(item):
        names.append(threading.current_thread().name)
        events.put(("prepare_start", item))
        if item == 2:
            second_prepared.set()
        return f"record-{item}"

    def consume(item, record):
        if item == 1:
            assert second_prepared.wait(timeout=2.0), "item 2 must be prepared while item 1 is still being consumed"
        return f"{item}:{record}"

    results = list(ordered_prefetch_map([1, 2], prepare=prepare, consume=consume, release_prepared=released.append))
    assert results == ["1:record-1", "2:record-2"]
    assert released == []
    assert [events.get_nowait() for _ in range(2)] == [("prepare_start", 1), ("prepare_start", 2)]
    assert all(name.startswith("pd-prefetch") for name in names)


def test_prefetched_item_is_released_when_consume_fails():
    second_prepared = threading.Event()
    released = []

    def prepare(item):
        if item == 2:
            second_prepared.set()
        return f"record-{item}"

    def consume(item, record):
        if item == 1:
            assert second_prepared.wait(timeout=2.0)
            raise RuntimeError("decode failed")
        return record

    with pytest.raises(RuntimeError, match="decode failed"):
        list(ordered_prefetch_map([1, 2, 3], prepare=prepare, consume=consume, release_prepared=released.append))
    assert released == ["record-2"]


def test_closing_the_generator_releases_the_lookahead_and_order_is_kept():
    released = []
    gen = ordered_prefetch_map(range(5), prepare=lambda i: i * 10, consume=lambda i, r: (i, r), release_prepared=released.append)
    assert next(gen) == (0, 0)
    assert next(gen) == (1, 10)
    gen.close()
    assert released in ([20], [])      # item 2 was in flight (released) or had not started (dropped)
    assert list(ordered_prefetch_map([], prepare=lambda i: i, consume=lambda i, r: r)) == []
    assert list(ordered_prefetch_map(range(4), prepare=lambda i: i + 1, consume=lambda i, r: i * r)) == [0, 2, 6, 12]


def test_prepare_error_surfaces_at_its_own_item():
    def prepare(item):
        if item == 1:
            raise ValueError("prefill failed")
        return item

    seen = []
    with pytest.raises(ValueError, match="prefill failed"):
        for out in ordered_prefetch_map([0, 1, 2], prepare=prepare, consume=lambda i, r: r):
            seen.append(out)
    assert seen == [0]


def test_forward_context_is_per_thread():
    reset_context_diffusion_lm()
    set_context_diffusion_lm(True, max_seqlen_q=11)
    seen = {}
    ready, done = threading.Event(), threading.Event()

    def worker():
        reset_context_diffusion_lm()
        set_context_diffusion_lm(False, max_seqlen_q=22)
        seen["worker"] = get_context_diffusion_lm().max_seqlen_q
        ready.set()
        done.wait(timeout=2.0)

    thread = threading.Thread(target=worker)
    thread.start()
    assert ready.wait(timeout=2.0)
    assert get_context_diffusion_lm().max_seqlen_q == 11 and get_context_diffusion_lm().is_prefill
    done.set()
    thread.join()
    assert seen["worker"] == 22
    reset_context_diffusion_lm()
    assert get_context_diffusion_lm().max_seqlen_q == 0
