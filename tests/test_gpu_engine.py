"""GPU parity of the PD engine facade (prefilling_dllm_b200.engine) with the reference engine.

The reference engine cannot run without CUDA + NCCL: tests/golden/engine_reference.json holds what it produced, unmodified, on
a B200 (tests/golden/make_engine_golden.py), and its flow is restated on the CPU contract model (oracle/engine_flow.py, pinned
on that fixture by tests/test_engine_golden.py) for the cases the fixture does not hold. The toy checkpoint is the one the
goldens were made with. fp32, SIMT attention kernel.
Gates: first token, number of denoise steps and token ids equal; chunk scores within 1e-4; selected chunks and keep
lists bit-exact (up to exact ties at the cut); KV payloads bit-exact across snapshot / load / engine-to-engine copy.
"""

import json
import os
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
sys.path.insert(0, os.path.dirname(HERE))

BOS, MASK, BLOCK = 1, 1023, 32


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    import make_golden

    path = str(tmp_path_factory.mktemp("ckpt_engine"))
    make_golden.write_toy_checkpoint(path)
    return path


@pytest.fixture(scope="module")
def cpu_model(ckpt):
    from oracle.contract_model.model.modeling_dream import DreamModel

    return DreamModel.from_pretrained(ckpt).eval()


def _engine(ckpt, pages=24, **kw):
    from prefilling_dllm_b200.engine import FastDLLMDreamEngine

    return FastDLLMDreamEngine(ckpt, max_model_len=8192, block_length=BLOCK, mask_token_id=MASK, threshold=0.9, dtype=torch.float32, enforce_eager=kw.pop("enforce_eager", False),
                               num_kv_pages=pages, **kw)


@pytest.fixture(scope="module")
def engine(ckpt):
    return _engine(ckpt)


def _prompt(n=600, seed=3):
    g = torch.Generator().manual_seed(seed)
    return [BOS] + torch.randint(3, 1023, (n - 1,), generator=g).tolist()


def _rotate(k, positions, theta=1e6):
    """[S, Hkv, D] un-rotated keys → rotated at `positions` (what the engine keeps in its pages)."""
    d = k.shape[-1]
    inv = 1.0 / (theta ** (torch.arange(0, d, 2).float() / d))
    f = torch.tensor(positions).float().unsqueeze(-1) * inv
    emb = torch.cat((f, f), dim=-1)
    cos, sin = emb.cos().unsqueeze(1), emb.sin().unsqueeze(1)
    return k * cos + torch.cat((-k[..., d // 2:], k[..., : d // 2]), dim=-1) * sin


def test_pd_split_matches_the_restated_engine(engine, cpu_model):
    from oracle import engine_flow as E

    prompt = _prompt()
    want = E.prefill_and_decode(cpu_model, prompt, block_length=BLOCK, mask_id=MASK, threshold=0.9)
    free0 = engine._prefix_cache.num_free_pages
    rec = engine.prefill_to_pd_record(prompt, max_new_tokens=BLOCK)
    assert (rec.prompt_len, rec.full_prompt_len, rec.decode_len, rec.kv_mode) == (600, 600, BLOCK, "full_dense")
    assert rec.suffix_positions == list(range(600, 600 + BLOCK)) and rec.prompt_positions == list(range(600))
    assert len(rec.prompt_page_ids) == 3 and len(rec.block_page_ids) == 1 and not rec.owns_prompt_pages
    assert rec.first_token_id == want["first_token"]
    assert torch.allclose(rec.last_context_logit.cpu(), want["last_context_logit"], atol=2e-4)
    snap = engine.snapshot_pd_record_kv(rec)
    assert snap.prompt_len == 600 and snap.page_size == 256 and snap.kv_mode == "full_dense" and len(snap.k_by_layer) == 2
    for layer, (k_ref, v_ref) in enumerate(want["past"]):
        assert snap.k_by_layer[layer].device.type == "cpu" and tuple(snap.k_by_layer[layer].shape) == (600, 2, 64)
        assert torch.allclose(snap.v_by_layer[layer], v_ref[0].view(600, 2, 64), atol=1e-5)
        assert torch.allclose(snap.k_by_layer[layer], _rotate(k_ref[0].view(600, 2, 64), list(range(600))), atol=1e-4)
    out = engine.decode_from_pd_record(rec, max_new_tokens=BLOCK)
    assert out.token_ids == want["token_ids"] and out.n_diff_steps == want["n_diff_steps"]
    # the record is consumed: block pages are back, the prompt pages stay with the prefix cache
    assert engine._prefix_cache.num_free_pages == free0 - 3
    again = engine.prefill_to_pd_record(prompt, max_new_tokens=BLOCK)
    assert again.cached_prefix is not None and again.prompt_page_ids == rec.prompt_page_ids and again.first_token_id == rec.first_token_id
    stop = want["token_ids"][3]
    short = engine.decode_from_pd_record(again, max_new_tokens=5, stop_token_ids=[stop])
    assert short.token_ids == want["token_ids"][:want["token_ids"].index(stop)]      # cut at the first stop token
    assert engine._prefix_cache.evict_one() and engine._prefix_cache.num_free_pages == free0


def test_engine_facade_matches_the_reference_engine(engine):
    """The same calls that tests/golden/make_engine_golden.py made on the UNMODIFIED reference `FastDLLMDreamEngine` (run on a
    B200, float64 model, its sdpa backend), made on this library's engine in float32: the prefill/decode split (first token,
    last-context logit, ids, step counts, KV checksums — both keep rotated keys in their pages), post-hoc eviction, the engine's
    draft, chunk scores and selection, per-head keep lists (up to swaps between tied scores at the cut), the chunk-local KV
    generate, the sparse prefill over an eviction mask and the decode-time delta correction."""
    import make_engine_golden as G

    with open(os.path.join(HERE, "golden", "engine_reference.json")) as handle:
        ref = json.load(handle)
    if "unavailable" in ref:
        pytest.skip("the reference engine could not be run where the fixture was made: " + ref["unavailable"])
    free0 = engine._prefix_cache.num_free_pages
    got = G.record(engine)
    for mine, theirs in zip(got["pd_split"], ref["pd_split"]):
        for key in ("first_token_id", "prompt_len_record", "suffix_positions", "token_ids", "n_diff_steps", "fused_token_ids", "k_shape"):
            assert mine[key] == theirs[key], key
        assert torch.allclose(torch.tensor(mine["last_context_logit"]), torch.tensor(theirs["last_context_logit"]), atol=2e-4)
        for key in ("k_abs_sum", "v_abs_sum"):
            assert all(abs(a - b) < 1e-4 * b for a, b in zip(mine[key], theirs[key])), key
    for key in ("kv_mode", "prompt_len_record", "full_prompt_len", "first_token_id", "suffix_positions", "token_ids", "n_diff_steps"):
        assert got["posthoc_eviction"][key] == ref["posthoc_eviction"][key], key
    mine, theirs = got["selection"], ref["selection"]
    for key in ("draft_ids", "draft_mask", "selected", "selection_query_ids", "score_token_mask"):
        assert mine[key] == theirs[key], key
    assert max(abs(mine["scores"][k] - v) for k, v in theirs["scores"].items()) < 1e-4
    assert abs(mine["chunk2_causal"] - theirs["chunk2_causal"]) < 1e-4
    assert abs(mine["chunk2_query_to_chunk"] - theirs["chunk2_query_to_chunk"]) < 1e-4
    mine, theirs = got["per_head_keep"], ref["per_head_keep"]
    assert mine["full_prompt_len"] == theirs["full_prompt_len"]
    assert [(m["start"], m["end"], m["kept_tokens"]) for m in mine["meta"]] == [(m["start"], m["end"], m["kept_tokens"]) for m in theirs["meta"]]
    swaps = 0
    for layer_m, layer_t in zip(mine["keep"], theirs["keep"]):
        for head_m, head_t in zip(layer_m, layer_t):
            assert len(head_m) == len(head_t)
            swaps += len(set(head_m) ^ set(head_t)) // 2
    print(f"per-head keep lists: {swaps} positions differ from the reference engine's (exact ties at the cut)")
    assert swaps <= 8         # oracle-side test (tests/test_engine_golden.py) checks that every such swap is between exactly tied scores
    assert got["chunk_local"] == ref["chunk_local"]
    # sparse prefill over the eviction mask (plain and with the strided delta correction, three directions) and the decode-time
    # delta correction against the full-KV reservoir
    for name, theirs in ref["sparse_and_delta"]["cases"].items():
        mine = got["sparse_and_delta"]["cases"][name]
        assert "error" not in mine and "error" not in theirs, (name, mine.get("error"), theirs.get("error"))
        for key in ("kv_mode", "prompt_len_record", "full_prompt_len", "first_token_id", "suffix_positions", "n_prompt_pages", "token_ids", "n_diff_steps"):
            assert mine[key] == theirs[key], (name, key)
        assert torch.allclose(torch.tensor(mine["last_context_logit"]), torch.tensor(theirs["last_context_logit"]), atol=2e-4), name
    # keep lists off the defaults: pooling, reduce, keep-low, the chunk->query and bidirectional directions, a window of last layers
    swaps = 0
    for name, theirs in ref["per_head_keep_variants"]["cases"].items():
        mine = got["per_head_keep_variants"]["cases"][name]
        assert "error" not in mine and "error" not in theirs, (name, mine.get("error"), theirs.get("error"))
        assert mine["kept"] == theirs["kept"], name
        for layer_m, layer_t in zip(mine["keep"], theirs["keep"]):
            for head_m, head_t in zip(layer_m, layer_t):
                assert len(head_m) == len(head_t), name
                swaps += len(set(head_m) ^ set(head_t)) // 2
        print(f"keep variant {name}: {swaps} positions differ so far")
    assert swaps <= 24        # exact ties at the cut only (the oracle-side check of the default variant shows what these are)
    # the sampler settings: filters at temperature 0 (several slots per step), and a positive temperature from a seeded generator
    for name, theirs in ref["sampling"]["cases"].items():
        mine = got["sampling"]["cases"][name]
        assert "error" not in mine and "error" not in theirs, (name, mine.get("error"), theirs.get("error"))
        for key in ("first_token_id", "token_ids", "n_diff_steps"):
            assert mine[key] == theirs[key], (name, key)
    while engine._prefix_cache.evict_one():
        pass
    assert engine._prefix_cache.num_free_pages == free0


def test_pd_split_with_unshifted_logits(ckpt, cpu_model):
    """An architecture that reads token p from logits[p] (LLaDA's read-out; same toy weights): the first block token comes
    from the first MASK slot's own row of the joint prefill, the steps use the un-shifted unmask rule, a prefix-cache hit
    gives the same record, and the Dream-only selection twins refuse."""
    import dataclasses

    from oracle import engine_flow as E

    eng = _engine(ckpt, pages=12)
    eng.model.arch = dataclasses.replace(eng.model.arch, logit_shift=False)
    prompt = _prompt(500, seed=9)
    want = E.prefill_and_decode(cpu_model, prompt, block_length=BLOCK, mask_id=MASK, threshold=0.9, shift=False)
    shifted = E.prefill_and_decode(cpu_model, prompt, block_length=BLOCK, mask_id=MASK, threshold=0.9)
    assert want["token_ids"] != shifted["token_ids"]          # the two read-outs really differ on this input
    rec = eng.prefill_to_pd_record(prompt, max_new_tokens=BLOCK)
    assert rec.first_token_id == want["first_token"]
    assert torch.allclose(rec.last_context_logit.cpu(), want["last_context_logit"], atol=2e-4)
    out = eng.decode_from_pd_record(rec, max_new_tokens=BLOCK)
    assert out.token_ids == want["token_ids"] and out.n_diff_steps == want["n_diff_steps"]
    again = eng.prefill_to_pd_record(prompt, max_new_tokens=BLOCK)
    assert again.cached_prefix is not None and again.first_token_id == want["first_token"]
    both = eng.decode_from_pd_records([again], max_new_tokens=BLOCK)
    assert both[0].token_ids == want["token_ids"]
    with pytest.raises(NotImplementedError, match="shifted logits"):
        eng.generate_partial_draft_rounds_for_selection(prompt, max_new_tokens=4, partial_rounds=1)


def test_several_blocks_with_unshifted_logits(ckpt, cpu_model):
    """Records of three blocks (80 tokens) on the un-shifted read-out: every block's first token comes from the first MASK
    slot's own row of the suffix initialisation. One by one and in shared steps, against the restated block loop."""
    import dataclasses

    from oracle import engine_flow as E

    eng = _engine(ckpt, pages=24)
    eng.model.arch = dataclasses.replace(eng.model.arch, logit_shift=False)
    prompts = [_prompt(500, seed=51), _prompt(333, seed=52)]
    wants = [E.decode_blocks(cpu_model, p, max_new=80, block_length=BLOCK, mask_id=MASK, threshold=0.9, shift=False) for p in prompts]
    free0 = eng._prefix_cache.num_free_pages
    for p, want in zip(prompts, wants):
        out = eng.decode_from_pd_record(eng.prefill_to_pd_record(p, max_new_tokens=80), max_new_tokens=80)
        assert out.token_ids == want["token_ids"] and out.n_diff_steps == want["n_diff_steps"]
    shared = eng.decode_from_pd_records([eng.prefill_to_pd_record(p, max_new_tokens=80) for p in prompts], max_new_tokens=80)
    for out, want in zip(shared, wants):
        assert out.token_ids == want["token_ids"] and out.n_diff_steps == want["n_diff_steps"]
    from prefilling_dllm_b200 import ops

    ops.check_status(eng.device)
    while eng._prefix_cache.evict_one():
        pass
    assert eng._prefix_cache.num_free_pages == free0


def test_snapshot_load_and_engine_to_engine_copy(engine, ckpt):
    other = _engine(ckpt, pages=16)
    prompt = _prompt(700, seed=5)
    rec = engine.prefill_to_pd_record(prompt, max_new_tokens=BLOCK)
    snap_cpu = engine.snapshot_pd_record_kv(rec)
    snap_gpu = engine.snapshot_pd_record_kv(rec, device="cuda")
    assert snap_gpu.k_by_layer[0].is_cuda and torch.equal(snap_gpu.k_by_layer[1].cpu(), snap_cpu.k_by_layer[1])
    loaded = other.make_pd_record_from_kv_snapshot(rec, snap_cpu)
    copied = other.make_pd_record_from_remote_engine(engine, rec)
    assert loaded.owns_prompt_pages and copied.owns_prompt_pages and loaded.cached_prefix is None
    assert set(loaded.prompt_page_ids).isdisjoint(copied.prompt_page_ids)
    for rec_b in (loaded, copied):
        snap_b = other.snapshot_pd_record_kv(rec_b)
        for layer in range(2):
            assert torch.equal(snap_b.k_by_layer[layer], snap_cpu.k_by_layer[layer])
            assert torch.equal(snap_b.v_by_layer[layer], snap_cpu.v_by_layer[layer])
    ids = engine.decode_from_pd_record(rec, max_new_tokens=BLOCK).token_ids
    assert other.decode_from_pd_record(loaded, max_new_tokens=BLOCK).token_ids == ids
    assert other.decode_from_pd_record(copied, max_new_tokens=BLOCK).token_ids == ids
    assert other._prefix_cache.num_free_pages == 16
    # validation at the boundary (reference :734-745, :683-690)
    rec2 = engine.prefill_to_pd_record(prompt, max_new_tokens=BLOCK)
    try:
        from dataclasses import replace

        with pytest.raises(ValueError, match="page_size mismatch"):
            other.make_pd_record_from_kv_snapshot(rec2, replace(snap_cpu, page_size=128))
        with pytest.raises(ValueError, match="prompt_len mismatch"):
            other.make_pd_record_from_kv_snapshot(rec2, replace(snap_cpu, prompt_len=699))
        with pytest.raises(ValueError, match="mode mismatch"):
            other.make_pd_record_from_kv_snapshot(rec2, replace(snap_cpu, kv_mode="compacted_posthoc_eviction"))
        with pytest.raises(ValueError, match="shape mismatch"):
            other.make_pd_record_from_kv_snapshot(rec2, replace(snap_cpu, k_by_layer=[t[:-1] for t in snap_cpu.k_by_layer]))
        with pytest.raises(ValueError, match="layer count mismatch"):
            other.make_pd_record_from_kv_snapshot(rec2, replace(snap_cpu, k_by_layer=snap_cpu.k_by_layer[:1]))
        assert other._prefix_cache.num_free_pages == 16, "a rejected snapshot must not leak pages"
    finally:
        engine.release_pd_record(rec2)
    engine._prefix_cache.evict_one()


def test_posthoc_eviction_with_head_independent_keep(engine, cpu_model):
    from oracle import engine_flow as E

    prompt = _prompt(600, seed=7)
    keep = [0] + list(range(1, 600, 3))                      # 201 tokens: fits one page, two tail pages are released
    want = E.prefill_and_decode(cpu_model, prompt, block_length=BLOCK, mask_id=MASK, threshold=0.9, keep=keep)
    nested = [[keep, keep] for _ in range(2)]
    free0 = engine._prefix_cache.num_free_pages
    rec = engine.prefill_to_pd_record(prompt, max_new_tokens=BLOCK, prompt_keep_indices_per_layer_per_head=nested,
                                      active_prompt_positions=keep)
    assert rec.kv_mode == "compacted_posthoc_eviction" and rec.owns_prompt_pages and rec.cached_prefix is None
    assert (rec.prompt_len, rec.full_prompt_len, len(rec.prompt_page_ids)) == (len(keep), 600, 1)
    assert rec.suffix_positions[0] == max(keep) + 1 and rec.first_token_id == want["first_token"]
    out = engine.decode_from_pd_record(rec, max_new_tokens=BLOCK)
    assert out.token_ids == want["token_ids"] and out.n_diff_steps == want["n_diff_steps"]
    assert engine._prefix_cache.num_free_pages == free0
    with pytest.raises(ValueError, match="active_prompt_positions is required"):
        engine.prefill_to_pd_record(prompt, max_new_tokens=BLOCK, prompt_keep_indices_per_layer_per_head=nested)
    with pytest.raises(ValueError, match="layer count mismatch"):
        engine.prefill_to_pd_record(prompt, max_new_tokens=BLOCK, prompt_keep_indices_per_layer_per_head=nested[:1], active_prompt_positions=keep)
    with pytest.raises(ValueError, match="outside full prompt length"):
        engine.prefill_to_pd_record(prompt, max_new_tokens=BLOCK, prompt_keep_indices_per_layer_per_head=[[[0, 600]] * 2] * 2,
                                    active_prompt_positions=[0, 1])
    assert engine._prefix_cache.num_free_pages == free0


def test_rejections(engine):
    prompt = _prompt(64)
    with pytest.raises(ValueError):
        engine.prefill_to_pd_record(prompt, max_new_tokens=0)
    with pytest.raises(NotImplementedError, match="one generation block"):       # the chunk-local path keeps the reference's limit
        engine.generate_token_ids_from_chunk_local_kv(prefix_ids=[BOS], prefix_positions=[0], chunk_ids_list=[], chunk_positions_list=[],
                                                      chunk_keep_indices_per_layer_per_head=[], query_ids=prompt, query_positions=list(range(1, 65)),
                                                      local_query_ids=prompt[-8:], max_new_tokens=BLOCK + 1)
    with pytest.raises(ValueError, match="Unsupported prefill_sparse_mode"):
        engine.prefill_to_pd_record(prompt, max_new_tokens=8, prefill_sparse_mode="banded")
    with pytest.raises(ValueError, match="requires prompt_keep_indices"):
        engine.prefill_to_pd_record(prompt, max_new_tokens=8, prefill_sparse_mode="eviction_mask")
    with pytest.raises(ValueError, match="length mismatch"):
        engine.prefill_to_pd_record(prompt, max_new_tokens=8, prompt_positions=[0, 1])
    with pytest.raises(ValueError, match="requires prompt_keep_indices"):
        engine.prefill_to_pd_record(prompt, max_new_tokens=8, active_prompt_positions=[0])
    rec = engine.prefill_to_pd_record(prompt, max_new_tokens=8)
    with pytest.raises(ValueError, match="exceeds record decode_len"):
        engine.decode_from_pd_record(rec, max_new_tokens=BLOCK + 1)
    assert engine.decode_from_pd_record(rec, max_new_tokens=0).token_ids == []
    engine.release_pd_record(rec)
    engine._prefix_cache.evict_one()
    assert engine._prefix_cache.num_free_pages == engine._prefix_cache.num_pages
    with pytest.raises(RuntimeError, match="Cannot allocate"):
        engine.prefill_to_pd_record(_prompt(7000), max_new_tokens=8)
    assert engine._prefix_cache.num_free_pages == engine._prefix_cache.num_pages


def test_selection_twins(engine, cpu_model):
    import make_golden
    from oracle import engine_flow as E
    from oracle import hotpath as O

    context, query = make_golden.toy_inputs()
    chunks = [O.maybe_prepend_bos_to_chunk(c, [BOS], 512) for c in O.split_token_chunks(context, 512)]
    draft = E.engine_draft(cpu_model, [BOS] + query, draft_len=4, partial_rounds=1, mask_id=MASK)
    assert engine.generate_partial_draft_rounds_for_selection([BOS] + query, max_new_tokens=4, partial_rounds=1) == draft
    selection, label_mask = query + draft[0], [True] * len(query) + draft[1]
    want_scores = [E.score_chunk(cpu_model, [BOS], c, selection, label_mask) for c in chunks]
    selected, scores, sel_ids, mask = engine.select_chunks_by_engine([BOS], chunks, query, topk_chunks=4)
    assert sel_ids == selection and mask == label_mask
    assert max(abs(scores[i] - want_scores[i]) for i in range(len(chunks))) < 1e-4
    assert selected == O.rank_chunks(want_scores, 4)
    one = engine.score_chunk_self_information_engine([BOS], chunks[2], selection, score_token_mask=label_mask)
    assert abs(one - want_scores[2]) < 1e-4
    q2c = engine.score_chunk_self_information_engine([BOS], chunks[2], selection, score_token_mask=label_mask, score_attention_mask="query_to_chunk")
    assert abs(q2c - E.score_chunk(cpu_model, [BOS], chunks[2], selection, label_mask, "query_to_chunk")) < 1e-4
    # per-head keep indices over a prompt of [BOS ‖ chunk a ‖ chunk b ‖ query]
    a, b = chunks[selected[0]], chunks[selected[1]]
    spans = [dict(chunk_ids=a, start=1, end=1 + len(a)), dict(chunk_ids=b, start=1 + len(a), end=1 + len(a) + len(b))]
    full_len = 1 + len(a) + len(b) + len(query)
    keep, meta = engine.compute_prompt_keep_indices_per_layer_per_head(full_prompt_len=full_len, prefix_ids=[BOS], chunk_spans=spans,
                                                                      query_ids=query, token_capacity=128)
    assert len(keep) == 2 and len(keep[0]) == 2 and len(keep[0][0]) == 1 + 128 + 128 + len(query)
    assert [m["kept_tokens"] for m in meta] == [128, 128] and all(m["union_kept_tokens"] >= 128 for m in meta)
    for span, chunk in zip(spans, (a, b)):
        ref_keep, pooled = E.per_head_keep(cpu_model, [BOS], chunk, query[-8:], capacity=128, num_kv_heads=2, layers=[0])
        for layer in range(2):           # token_score_layers=1: layer 0's indices serve every layer
            for h in range(2):
                mine = [i - span["start"] for i in keep[layer][h] if span["start"] <= i < span["end"]]
                theirs = ref_keep[0][h].tolist()
                diff = set(mine) ^ set(theirs)
                cut = min(float(pooled[0][h][i].detach()) for i in theirs[1:])
                assert len(mine) == 128 and all(abs(float(pooled[0][h][i]) - cut) <= 1e-6 * abs(cut) for i in diff)
        assert keep[0][0][0] == 0 and keep[0][0][-len(query):] == list(range(full_len - len(query), full_len))


def test_chunk_local_kv_generate(engine, cpu_model):
    import make_golden
    from oracle import engine_flow as E
    from oracle import hotpath as O

    context, query = make_golden.toy_inputs()
    chunks = [O.maybe_prepend_bos_to_chunk(c, [BOS], 512) for c in O.split_token_chunks(context, 512)][:2]
    keeps = [[0] + list(range(5, 512, 4)), [0] + list(range(2, 512, 4))]
    chunk_pos = [list(range(1, 513)), list(range(1, 513))]                 # "reuse" positions: every chunk at 1..512
    q_pos = list(range(513, 513 + len(query)))
    kw = dict(prefix_ids=[BOS], prefix_positions=[0], chunk_ids_list=chunks, chunk_positions_list=chunk_pos, query_ids=query,
              query_positions=q_pos, local_query_ids=query[-8:])
    want = E.chunk_local_generate(cpu_model, keep_list=keeps, block_length=BLOCK, mask_id=MASK, threshold=0.9, **kw)
    nested = [[[k, k] for _ in range(2)] for k in keeps]
    free0 = engine._prefix_cache.num_free_pages
    out = engine.generate_token_ids_from_chunk_local_kv(chunk_keep_indices_per_layer_per_head=nested, max_new_tokens=BLOCK, **kw)
    assert out.token_ids == want["token_ids"] and out.n_diff_steps == want["n_diff_steps"]
    assert engine._prefix_cache.num_free_pages == free0
    with pytest.raises(ValueError, match="keep-indices list length mismatch"):
        engine.generate_token_ids_from_chunk_local_kv(chunk_keep_indices_per_layer_per_head=nested[:1], max_new_tokens=BLOCK, **kw)


def test_two_blocks_on_the_engine_reproduce_the_reference_eval_golden(engine, ckpt):
    """max_new_tokens = 2 x block_length on the PD engine (the reference engine stops at one block; the block loop follows its
    eval class). The eval class's golden run `two_blocks` is exactly this flow on [BOS ‖ selected chunks ‖ query] — a joint
    prefill with all 64 MASK slots, then the dual-cache loop — and in float32 the engine's fp32 softmax is the eval class's:
    the ids must come out the same. Checked through the explicit boundary, through a KV snapshot loaded into a second
    engine, and on a prefix-cache hit (where the partially filled last prompt page is copied before the suffix is appended)."""
    import json
    import os

    import make_golden
    from oracle import hotpath as O

    with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "toy_reference.json")) as handle:
        ref = json.load(handle)["runs"]["two_blocks"]
    context, query = make_golden.toy_inputs()
    size = ref["flags"]["chunk_size"]
    chunks = [O.maybe_prepend_bos_to_chunk(c, [BOS], size) for c in O.split_token_chunks(context, size)]
    prompt = [BOS] + [t for ci in ref["selected_chunk_indices"] for t in chunks[ci]] + query
    while engine._prefix_cache.evict_one():
        pass
    free0 = engine._prefix_cache.num_free_pages
    rec = engine.prefill_to_pd_record(prompt, max_new_tokens=64)
    assert rec.decode_len == 64 and rec.prompt_len == len(prompt) and rec.suffix_positions == list(range(len(prompt), len(prompt) + 64))
    snap = engine.snapshot_pd_record_kv(rec)
    out = engine.decode_from_pd_record(rec, max_new_tokens=64)
    match = sum(int(a == b) for a, b in zip(out.token_ids, ref["sequences"])) / 64
    print(f"engine, two blocks: greedy token match with the reference eval class {match:.3f}, {out.n_diff_steps} denoise forwards")
    assert len(out.token_ids) == 64 and match >= 0.99
    # a second engine gets only the prompt KV (snapshot) and recomputes the MASK slots itself
    other = _engine(ckpt, pages=16)
    moved = other.make_pd_record_from_kv_snapshot(rec, snap)
    assert other.decode_from_pd_record(moved, max_new_tokens=64).token_ids == out.token_ids
    assert other._prefix_cache.num_free_pages == 16
    # prefix-cache hit: the shared prompt pages end mid-page, the suffix goes behind a private copy of that page
    again = engine.prefill_to_pd_record(prompt, max_new_tokens=64)
    assert again.cached_prefix is not None and not again.owns_prompt_pages and len(prompt) % 256 != 0
    assert engine.decode_from_pd_record(again, max_new_tokens=64).token_ids == out.token_ids
    one_block = engine.prefill_to_pd_record(prompt, max_new_tokens=BLOCK)       # another entry: the prompt KV saw 32 MASK slots
    assert one_block.cached_prefix is None
    engine.release_pd_record(one_block)
    from prefilling_dllm_b200 import ops

    ops.check_status(engine.device)
    while engine._prefix_cache.evict_one():
        pass
    assert engine._prefix_cache.num_free_pages == free0


@pytest.mark.parametrize("layers_per_message", [1, 4])
def test_kv_streamed_during_the_prefill(engine, ckpt, layers_per_message):
    """The prompt KV leaves the prefill engine as wire messages while the prefill runs (a group of layers per message,
    gathered on a side stream after that group's page writes) and lands in a second engine's pages group by group: same KV
    bits and same ids as decoding where the prefill ran; a prefix-cache hit streams the cached pages; a serialised
    whole snapshot carries the same payload."""
    from prefilling_dllm_b200 import ops, pd_wire

    other = _engine(ckpt, pages=16)
    prompt = _prompt(700, seed=41)
    while engine._prefix_cache.evict_one():
        pass
    for attempt in ("computed", "prefix-cache hit"):
        messages = []
        writer = pd_wire.KVStreamWriter(engine, messages.append, layers_per_message=layers_per_message)
        rec = engine.prefill_to_pd_record(prompt, max_new_tokens=BLOCK, kv_stream=writer)
        assert (rec.cached_prefix is not None) == (attempt == "prefix-cache hit")
        kinds = [pd_wire.unpack_message(m)[0] for m in messages]
        n_groups = -(-2 // layers_per_message)
        assert kinds == [pd_wire.TYPE_HEADER] + [pd_wire.TYPE_LAYERS] * n_groups + [pd_wire.TYPE_TRAILER], attempt
        assert writer.bytes_sent == sum(len(m) for m in messages) > 2 * 2 * 700 * 2 * 64 * 4
        reader = pd_wire.KVStreamReader(other)
        for m in messages:
            reader.feed(m)
        moved = reader.record
        assert moved is not None and moved.owns_prompt_pages and moved.prompt_len == 700 and moved.first_token_id == rec.first_token_id
        a, b = engine.snapshot_pd_record_kv(rec), other.snapshot_pd_record_kv(moved)
        for layer in range(2):
            assert torch.equal(a.k_by_layer[layer], b.k_by_layer[layer]) and torch.equal(a.v_by_layer[layer], b.v_by_layer[layer]), attempt
        assert torch.equal(moved.last_context_logit.cpu(), rec.last_context_logit.cpu())
        whole = pd_wire.snapshot_from_bytes(pd_wire.snapshot_to_bytes(a))
        assert torch.equal(whole.k_by_layer[1], b.k_by_layer[1]) and whole.prompt_len == 700
        ids = engine.decode_from_pd_record(rec, max_new_tokens=BLOCK).token_ids
        assert other.decode_from_pd_record(moved, max_new_tokens=BLOCK).token_ids == ids
        assert other._prefix_cache.num_free_pages == 16
    # a stream that skips a group is refused and the pages it held are returned
    reader = pd_wire.KVStreamReader(other)
    reader.feed(messages[0])
    with pytest.raises(ValueError, match="PD KV stream"):
        reader.feed(pd_wire.pack_message(pd_wire.TYPE_LAYERS, dict(first_layer=1, count=1), b""))
    assert other._prefix_cache.num_free_pages == 16
    ops.check_status(engine.device)
    ops.check_status(other.device)
    while engine._prefix_cache.evict_one():
        pass


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_engine_to_engine_copy_across_gpus(engine, ckpt):
    """Prefill on GPU 0, hand the prompt KV to an engine on GPU 1 with ONE kernel that reads GPU 0's pages through peer
    access, decode there: same KV bits, same ids as decoding where the prefill ran."""
    other = _engine(ckpt, pages=16, device_start=1)
    prompt = _prompt(700, seed=11)
    rec = engine.prefill_to_pd_record(prompt, max_new_tokens=BLOCK)
    remote = other.make_pd_record_from_remote_engine(engine, rec)
    assert remote.last_context_logit.device == torch.device("cuda", 1) and remote.owns_prompt_pages
    a, b = engine.snapshot_pd_record_kv(rec), other.snapshot_pd_record_kv(remote)
    for layer in range(2):
        assert torch.equal(a.k_by_layer[layer], b.k_by_layer[layer]) and torch.equal(a.v_by_layer[layer], b.v_by_layer[layer])
    ids = engine.decode_from_pd_record(rec, max_new_tokens=BLOCK).token_ids
    assert other.decode_from_pd_record(remote, max_new_tokens=BLOCK).token_ids == ids
    from prefilling_dllm_b200 import ops

    ops.check_status(torch.device("cuda", 1))
    assert other._prefix_cache.num_free_pages == 16
    engine._prefix_cache.evict_one()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_engine_to_engine_copy_survives_reuse_of_the_source_pages(engine, ckpt):
    """The copy kernel runs on the destination GPU's stream and returns at once. Releasing the source record and
    overwriting its pages straight afterwards must not change what the destination received: work enqueued later on the
    source's stream is ordered after the copy."""
    other = _engine(ckpt, pages=16, device_start=1)
    prompt = _prompt(700, seed=31)
    while engine._prefix_cache.evict_one():
        pass
    rec = engine.prefill_to_pd_record(prompt, max_new_tokens=BLOCK)
    want = engine.snapshot_pd_record_kv(rec)
    pages = list(rec.prompt_page_ids)
    remote = other.make_pd_record_from_remote_engine(engine, rec)
    engine.release_pd_record(rec)
    while engine._prefix_cache.evict_one():
        pass
    with torch.cuda.device(engine.device):
        engine.model.kv_cache[:, :, pages] = 7.0          # what a new prefill into the recycled pages would do
    got = other.snapshot_pd_record_kv(remote)
    for layer in range(2):
        assert torch.equal(want.k_by_layer[layer].cpu(), got.k_by_layer[layer].cpu())
        assert torch.equal(want.v_by_layer[layer].cpu(), got.v_by_layer[layer].cpu())
    other.release_pd_record(remote)
    assert other._prefix_cache.num_free_pages == 16


def test_batched_decode_of_several_blocks_equals_one_by_one(engine):
    """Records of three blocks (80 new tokens: 32 + 32 + 16) with different prompt lengths, one of them a prefix-cache hit whose
    last prompt page is shared: decoded in shared steps they give the ids and forward counts of decoding each on its own."""
    prompts = [_prompt(600, seed=41), _prompt(300, seed=42), _prompt(512, seed=43)]
    free0 = engine._prefix_cache.num_free_pages
    single = [engine.decode_from_pd_record(engine.prefill_to_pd_record(p, max_new_tokens=80), max_new_tokens=80) for p in prompts]
    records = [engine.prefill_to_pd_record(p, max_new_tokens=80) for p in prompts]
    assert all(r.cached_prefix is not None for r in records)
    batched = engine.decode_from_pd_records(records, max_new_tokens=80)
    for one, many in zip(single, batched):
        assert len(many.token_ids) == len(one.token_ids)
        assert many.token_ids == one.token_ids and many.n_diff_steps == one.n_diff_steps
    from prefilling_dllm_b200 import ops

    ops.check_status(engine.device)
    while engine._prefix_cache.evict_one():
        pass
    assert engine._prefix_cache.num_free_pages == free0


def test_batched_decode_equals_one_by_one(engine):
    """Three requests with different prompt lengths denoised in shared steps: same ids and step counts as decoding each
    record on its own; every page comes back."""
    prompts = [_prompt(600, seed=21), _prompt(300, seed=22), _prompt(777, seed=23)]
    free0 = engine._prefix_cache.num_free_pages
    single = [engine.decode_from_pd_record(engine.prefill_to_pd_record(p, max_new_tokens=BLOCK), max_new_tokens=BLOCK) for p in prompts]
    records = [engine.prefill_to_pd_record(p, max_new_tokens=BLOCK) for p in prompts]      # prefix-cache hits
    assert all(r.cached_prefix is not None for r in records)
    batched = engine.decode_from_pd_records(records, max_new_tokens=BLOCK)
    for one, many in zip(single, batched):
        assert many.token_ids == one.token_ids and many.n_diff_steps == one.n_diff_steps
    assert engine.decode_from_pd_records([], max_new_tokens=BLOCK) == []
    while engine._prefix_cache.evict_one():
        pass
    assert engine._prefix_cache.num_free_pages == free0


def test_decode_delta_state_travels_with_the_record(ckpt):
    """A record with a decode-delta reservoir handed to another engine (snapshot path and direct page copy) decodes to the
    same ids there; batched decode falls back to one record after the other for such records."""
    import make_engine_golden as G

    a, b = _engine(ckpt, pages=16), _engine(ckpt, pages=16)
    ids, nested = G.prompt(600, 13), G.per_head_keep_lists()
    kwargs = dict(max_new_tokens=BLOCK, prompt_keep_indices_per_layer_per_head=nested, active_prompt_positions=nested[0][0],
                  decode_delta_mode="s4_left3")
    want = a.decode_from_pd_record(a.prefill_to_pd_record(ids, **kwargs), max_new_tokens=BLOCK)
    free_a, free_b = a._prefix_cache.num_free_pages, b._prefix_cache.num_free_pages
    src = a.prefill_to_pd_record(ids, **kwargs)
    assert src.decode_delta_state["full_k"][0].shape[0] == 600 and src.prompt_len == 200
    moved = b.make_pd_record_from_remote_engine(a, src)
    loaded = b.make_pd_record_from_kv_snapshot(src, a.snapshot_pd_record_kv(src))
    a.release_pd_record(src)
    outs = b.decode_from_pd_records([moved, loaded], max_new_tokens=BLOCK)
    assert [o.token_ids for o in outs] == [want.token_ids, want.token_ids] and outs[0].n_diff_steps == want.n_diff_steps
    assert a._prefix_cache.num_free_pages == free_a and b._prefix_cache.num_free_pages == free_b
