"""Host-side pieces that need no GPU: the page allocator with its whole-prompt prefix cache (reference
_PrefixPageAllocator, prefilling_dllm_engine/prefilling_dllm/fastdllm_engine.py:88-167) and chunk splitting
(prefilling_dllm_eval/fastdllm_parallelcomp.py:158-180), checked against the oracle's restatement."""

import os
import sys
import threading

import pytest
import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from oracle import hotpath as O  # noqa: E402
from prefilling_dllm_b200.model import DreamArch, PageAllocator, slots_for  # noqa: E402
from prefilling_dllm_b200.parallelcomp import split_token_chunks  # noqa: E402


def test_allocator_fifo_refcounts_and_exhaustion():
    alloc = PageAllocator(num_pages=6, page_size=256)
    a = alloc.allocate_pages(2)
    b = alloc.allocate_pages(3)
    assert a == [0, 1] and b == [2, 3, 4] and alloc.num_free_pages == 1
    with pytest.raises(RuntimeError, match="Cannot allocate 2 pages, only 1 free"):
        alloc.allocate_pages(2)
    alloc.ref_pages(a)                 # a second owner
    alloc.release_pages(a)
    assert alloc.num_free_pages == 1   # still referenced
    alloc.release_pages(a)
    assert alloc.num_free_pages == 3
    assert alloc.allocate_pages(3) == [5, 0, 1]      # freed pages go to the back of the queue


def test_prefix_cache_lookup_eviction_and_ensure_free():
    alloc = PageAllocator(num_pages=4, page_size=256)
    prompt_a, prompt_b = [1, 5, 9], [1, 5, 10]
    pages_a = alloc.allocate_pages(2)
    entry = alloc.register_prefix(prompt_a, pages_a, prompt_len=3, last_context_logit=torch.zeros(8))
    assert entry.ref_count == 0 and alloc.lookup_prefix(prompt_a) is entry and alloc.lookup_prefix(prompt_b) is None
    assert alloc.compute_prompt_hash(prompt_a) == alloc.compute_prompt_hash(list(prompt_a)) != alloc.compute_prompt_hash(prompt_b)
    entry.ref_count += 1               # a record is using it
    assert not alloc.evict_one() and alloc.num_free_pages == 2
    alloc.release_prefix(prompt_a)     # the record is done
    alloc.ensure_free(3)               # needs the cached prefix to go
    assert alloc.num_free_pages == 4 and alloc.lookup_prefix(prompt_a) is None
    alloc.ensure_free(9)               # nothing left to evict: returns, the allocation itself will raise
    with pytest.raises(RuntimeError):
        alloc.allocate_pages(9)


def test_allocator_is_thread_safe():
    alloc = PageAllocator(num_pages=64, page_size=256)
    seen, errors = [], []

    def worker():
        try:
            for _ in range(200):
                pages = alloc.allocate_pages(2)
                seen.append(tuple(pages))
                alloc.release_pages(pages)
        except Exception as exc:  # pragma: no cover
            errors.append(exc)

    threads = [threading.Thread(target=worker) for _ in range(8)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors and alloc.num_free_pages == 64 and all(r == 0 for r in alloc.page_ref_count)
    assert all(p[0] != p[1] for p in seen)


def test_slots_for_walks_pages_in_list_order():
    assert slots_for([7, 2], 254, 4, 256) == [7 * 256 + 254, 7 * 256 + 255, 2 * 256, 2 * 256 + 1]
    assert slots_for([3], 0, 0, 256) == []


@pytest.mark.parametrize("n,size,tail", [(0, 4, False), (3, 4, False), (8, 4, False), (10, 4, False), (10, 4, True), (9, 1, True), (5, 0, False)])
def test_split_token_chunks_matches_the_oracle(n, size, tail):
    ids = list(range(100, 100 + n))
    assert split_token_chunks(ids, size, split_from_tail=tail) == O.split_token_chunks(ids, size, split_from_tail=tail)
    chunks = split_token_chunks(ids, size, split_from_tail=tail)
    assert [t for c in chunks for t in c] == ids
    if size > 0 and n > 0:
        assert all(len(c) <= size for c in chunks)
        short = [i for i, c in enumerate(chunks) if len(c) < size]
        assert short in ([], [0] if tail else [len(chunks) - 1])     # the remainder leads when splitting from the tail


def test_dataclasses_match_the_reference_field_for_field():
    """tests/golden/config_defaults.json holds the reference's dataclass fields and defaults (made by
    tests/golden/make_config_defaults.py from the unmodified reference module)."""
    import dataclasses
    import json

    from prefilling_dllm_b200 import parallelcomp as pc

    with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "config_defaults.json")) as handle:
        ref = json.load(handle)
    ours_only = {"FastDLLMParallelCompConfig": {"num_kv_pages", "decode_cuda_graph"}}
    methods = ref.pop("FastDLLMParallelComp.methods")
    functions = ref.pop("module_functions")
    import inspect

    for name, params in methods.items():      # public methods: same parameter names, kinds and defaults
        fn = getattr(pc.FastDLLMParallelComp, name)
        mine = [[p.name, p.kind == p.KEYWORD_ONLY, "<required>" if p.default is inspect.Parameter.empty else p.default]
                for p in list(inspect.signature(fn).parameters.values())[1:]]
        assert mine == params, name
    for name, params in functions.items():
        assert [p.name for p in inspect.signature(getattr(pc, name)).parameters.values()] == params, name
    for name, fields in ref.items():
        mine = {}
        for f in dataclasses.fields(getattr(pc, name)):
            if f.default is not dataclasses.MISSING:
                mine[f.name] = f.default
            elif f.default_factory is not dataclasses.MISSING:
                mine[f.name] = f.default_factory()
            else:
                mine[f.name] = "<required>"
        assert [k for k in mine if k not in ours_only.get(name, set())] == [k for k in mine if k in fields], name
        assert set(fields) <= set(mine), (name, set(fields) - set(mine))
        assert {k: mine[k] for k in fields} == fields, name
    arch = DreamArch.dream_7b()
    assert arch.head_dim == 128 and arch.num_attention_heads // arch.num_key_value_heads == 7 and arch.logit_shift
    assert not DreamArch.llada_8b().logit_shift and not DreamArch.llada_8b().attention_bias


def test_engine_facade_has_the_reference_api():
    """tests/golden/engine_api.json: dataclass fields and method signatures of the reference engine, extracted from its
    source by tests/golden/make_engine_api.py. Records must match field for field (name, order, default); every
    reference parameter must be accepted under the same name with the same default."""
    import dataclasses
    import inspect
    import json

    from prefilling_dllm_b200 import engine as E

    with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "engine_api.json")) as handle:
        api = json.load(handle)
    for name, fields in api["dataclasses"].items():
        mine = [[f.name, f.default if f.default is not dataclasses.MISSING else "<required>"] for f in dataclasses.fields(getattr(E, name))]
        assert mine == fields, name
    for name, sig in api["methods"].items():
        fn = getattr(E.FastDLLMDreamEngine, name)
        params = list(inspect.signature(fn).parameters.values())[1:]
        by_name = {p.name: p for p in params}
        forwards = any(p.kind == p.VAR_KEYWORD for p in params)
        n_req = len(sig["positional"]) - len(sig["positional_defaults"])
        ref = [(n, "<required>" if i < n_req else sig["positional_defaults"][i - n_req], False) for i, n in enumerate(sig["positional"])]
        ref += [(n, d, True) for n, d in sig["keyword_only"]]
        for pname, default, kw_only in ref:
            if pname not in by_name:
                assert forwards, f"{name}: parameter {pname} is missing"
                continue
            p = by_name[pname]
            assert (p.kind == p.KEYWORD_ONLY) == kw_only, f"{name}.{pname}: positional / keyword-only differs"
            if default == "<required>":
                assert p.default is inspect.Parameter.empty, f"{name}.{pname} must be required"
            elif isinstance(default, (int, float, str, bool)) or default is None:
                assert p.default == default, f"{name}.{pname}: default {p.default!r} != {default!r}"


def test_delta_windows_and_mode_checks_of_the_engine_facade():
    """Host side of the sparse prefill / decode delta paths: which rows an anchor's correction reaches (reference
    attention_v4.py:145-158) equals the oracle's windows, and the argument checks raise what the reference raises
    (fastdllm_engine.py:1924-1935, :2012-2017, :2079-2080)."""
    from oracle import engine_flow as E
    from prefilling_dllm_b200.engine import FastDLLMDreamEngine as Engine

    for direction, left, right in (("left", 3, 0), ("right", 0, 2), ("both", 1, 2), ("left", 0, 0)):
        anchors = list(range(0 if direction == "right" else 3, 19, 4))
        rows, which = Engine._spread_rows(anchors, 19, left=left, right=right, direction=direction)
        mine = torch.zeros(1, 19, 1)
        for r, w in zip(rows, which):
            mine[0, r, 0] += float(w + 1)
        dense = torch.zeros(1, len(anchors), 1) + torch.arange(1, len(anchors) + 1).view(1, -1, 1)
        theirs = E._spread_delta(torch.zeros(1, 19, 1), dense, anchors, left=left, right=right, direction=direction, scale=1.0)
        assert torch.equal(mine, theirs), direction

    ok = dict(prefill_sparse_mode="none", prefill_delta_mode="none", prefill_delta_selection_mode="none", prefill_delta_direction="left",
              decode_delta_mode="none", has_keep=True)
    Engine._check_modes(**ok)
    Engine._check_modes(**dict(ok, prefill_sparse_mode="eviction_mask", prefill_delta_mode="s4_left3", prefill_delta_direction="both"))
    Engine._check_modes(**dict(ok, decode_delta_mode="s4_left3"))
    for bad, error in ((dict(prefill_sparse_mode="other"), ValueError), (dict(prefill_sparse_mode="eviction_mask", has_keep=False), ValueError),
                       (dict(prefill_sparse_mode="eviction_mask", prefill_delta_mode="s8"), ValueError),
                       (dict(prefill_sparse_mode="eviction_mask", prefill_delta_direction="up"), ValueError),
                       (dict(decode_delta_mode="s8"), ValueError),
                       (dict(prefill_sparse_mode="eviction_mask", prefill_delta_selection_mode="selection_dense_add"), NotImplementedError)):
        with pytest.raises(error):
            Engine._check_modes(**dict(ok, **bad))
