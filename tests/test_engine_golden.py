"""The CPU restatement of the ENGINE's PD flow (oracle/engine_flow.py) against golden vectors of the reference engine itself.

tests/golden/engine_reference.json holds what the UNMODIFIED reference `FastDLLMDreamEngine` produced on a B200 for the seeded
toy checkpoint in float64 with its sdpa attention backend (tests/golden/make_engine_golden.py drives the staged copy; the engine cannot run on a CPU box).
These tests pin the restatement that the GPU engine tests use as their checker; tests/test_gpu_engine.py holds the library's
engine facade to the same file directly.
"""

import json
import os
import sys

import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
sys.path.insert(0, os.path.dirname(HERE))

BOS, MASK, BLOCK = 1, 1023, 32


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(HERE, "golden", "engine_reference.json")) as handle:
        data = json.load(handle)
    if "unavailable" in data:
        pytest.skip("the reference engine could not be run where the fixture was made: " + data["unavailable"])
    return data


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    import make_golden
    from oracle.contract_model.model.modeling_dream import DreamModel

    path = str(tmp_path_factory.mktemp("ckpt_engine_golden"))
    make_golden.write_toy_checkpoint(path)
    return DreamModel.from_pretrained(path).eval()


def test_prefill_decode_split(golden, model):
    import make_engine_golden as G
    from oracle import engine_flow as E

    for ref in golden["pd_split"]:
        prompt = G.prompt(ref["prompt_len"], ref["seed"])
        got = E.prefill_and_decode(model, prompt, block_length=BLOCK, mask_id=MASK, threshold=golden["threshold"])
        assert got["first_token"] == ref["first_token_id"]
        assert torch.allclose(got["last_context_logit"], torch.tensor(ref["last_context_logit"]), atol=2e-4)
        assert got["token_ids"] == ref["token_ids"] == ref["fused_token_ids"]
        assert got["n_diff_steps"] == ref["n_diff_steps"]
        # the pages hold rotated keys and plain values: compare the value checksums (layout-free)
        for layer, (_, v) in enumerate(got["past"]):
            assert abs(float(v.float().abs().sum()) - ref["v_abs_sum"][layer]) < 1e-3 * ref["v_abs_sum"][layer]


def test_posthoc_eviction(golden, model):
    import make_engine_golden as G
    from oracle import engine_flow as E

    ref = golden["posthoc_eviction"]
    prompt = G.prompt(ref["prompt_len"], ref["seed"])
    got = E.prefill_and_decode(model, prompt, block_length=BLOCK, mask_id=MASK, threshold=golden["threshold"], keep=ref["keep"])
    assert got["first_token"] == ref["first_token_id"]
    assert got["token_ids"] == ref["token_ids"] and got["n_diff_steps"] == ref["n_diff_steps"]
    assert ref["suffix_positions"][0] == max(ref["keep"]) + 1 and ref["prompt_len_record"] == len(ref["keep"])


def _chunks():
    import make_golden
    from oracle import hotpath as O

    context, query = make_golden.toy_inputs()
    return [O.maybe_prepend_bos_to_chunk(c, [BOS], 512) for c in O.split_token_chunks(context, 512)], query


def test_selection_twins(golden, model):
    from oracle import engine_flow as E
    from oracle import hotpath as O

    ref = golden["selection"]
    chunks, query = _chunks()
    draft = E.engine_draft(model, [BOS] + query, draft_len=4, partial_rounds=1, mask_id=MASK)
    assert list(draft[0]) == ref["draft_ids"] and list(draft[1]) == ref["draft_mask"]
    selection, label_mask = query + list(draft[0]), [True] * len(query) + list(draft[1])
    assert selection == ref["selection_query_ids"] and label_mask == ref["score_token_mask"]
    scores = [E.score_chunk(model, [BOS], c, selection, label_mask) for c in chunks]
    assert max(abs(scores[i] - ref["scores"][str(i)]) for i in range(len(chunks))) < 1e-4
    assert O.rank_chunks(scores, 4) == ref["selected"]
    assert abs(scores[2] - ref["chunk2_causal"]) < 1e-4
    assert abs(E.score_chunk(model, [BOS], chunks[2], selection, label_mask, "query_to_chunk") - ref["chunk2_query_to_chunk"]) < 1e-4


def test_per_head_keep(golden, model):
    from oracle import engine_flow as E

    ref = golden["per_head_keep"]
    sel = golden["selection"]["selected"]
    chunks, query = _chunks()
    swaps = 0
    for span_meta, ci in zip(ref["meta"], sel[:2]):
        mine, pooled = E.per_head_keep(model, [BOS], chunks[ci], query[-8:], capacity=128, num_kv_heads=2, layers=[0])
        for layer in range(2):            # token_score_layers=1: layer 0's indices serve every layer
            for h in range(2):
                theirs = [i - span_meta["start"] for i in ref["keep"][layer][h] if span_meta["start"] <= i < span_meta["end"]]
                ours = mine[0][h].tolist()
                diff = set(ours) ^ set(theirs)
                cut = min(float(pooled[0][h][i].detach()) for i in ours[1:])
                # exact ties at the cut: torch.topk's pick is unspecified (CPU and CUDA differ)
                assert len(theirs) == 128 and all(abs(float(pooled[0][h][i]) - cut) <= 1e-6 * abs(cut) for i in diff), (ci, layer, h, sorted(diff))
                swaps += len(diff) // 2
        assert span_meta["kept_tokens"] == 128
    full = ref["full_prompt_len"]
    assert ref["keep"][0][0][0] == 0 and ref["keep"][0][0][-len(query):] == list(range(full - len(query), full))
    assert swaps < 16


def test_chunk_local_generate(golden, model):
    from oracle import engine_flow as E

    ref = golden["chunk_local"]
    chunks, query = _chunks()
    chunk_pos = [list(range(1, 513)), list(range(1, 513))]
    q_pos = list(range(513, 513 + len(query)))
    got = E.chunk_local_generate(model, keep_list=ref["keeps"], block_length=BLOCK, mask_id=MASK, threshold=golden["threshold"],
                                 prefix_ids=[BOS], prefix_positions=[0], chunk_ids_list=chunks[:2], chunk_positions_list=chunk_pos,
                                 query_ids=query, query_positions=q_pos, local_query_ids=query[-8:])
    assert got["token_ids"] == ref["token_ids"] and got["n_diff_steps"] == ref["n_diff_steps"]


def test_sparse_prefill_and_decode_delta(golden, model):
    """Sparse prefill over the eviction mask (plain, and with the strided delta correction in its three directions) and the
    decode-time delta correction against the full-KV reservoir: every case the reference engine recorded."""
    import make_engine_golden as G
    from oracle import engine_flow as E

    ref = golden["sparse_and_delta"]
    prompt = G.prompt(ref["prompt_len"], ref["seed"])
    nested = G.per_head_keep_lists()
    model = model.double()
    try:
        for name, kwargs in G.SPARSE_DELTA_CASES.items():
            case = ref["cases"][name]
            assert "error" not in case, (name, case)
            if "prefill_sparse_mode" in kwargs:
                got = E.sparse_prefill_and_decode(
                    model, prompt, nested, block_length=BLOCK, mask_id=MASK, threshold=golden["threshold"],
                    delta=kwargs.get("prefill_delta_mode", "none") != "none", stride=kwargs.get("prefill_delta_stride", 8),
                    left=kwargs.get("prefill_delta_left", 7), right=kwargs.get("prefill_delta_right", 0),
                    direction=kwargs.get("prefill_delta_direction", "left"), scale=kwargs.get("prefill_delta_scale", 1.0))
                assert case["kv_mode"] == "full_prefill_sparse_delta" and case["prompt_len_record"] == case["full_prompt_len"] == len(prompt)
            else:
                got = E.posthoc_eviction_with_decode_delta(
                    model, prompt, nested, nested[0][0], block_length=BLOCK, mask_id=MASK, threshold=golden["threshold"],
                    stride=kwargs.get("decode_delta_stride", 4), left=kwargs.get("decode_delta_left", 3), scale=kwargs.get("decode_delta_scale", 1.0))
                assert case["kv_mode"] == "compacted_posthoc_eviction" and case["prompt_len_record"] == len(nested[0][0])
                assert case["suffix_positions"][0] == max(nested[0][0]) + 1
            assert got["first_token"] == case["first_token_id"], name
            assert torch.allclose(got["last_context_logit"], torch.tensor(case["last_context_logit"], dtype=torch.float64), atol=2e-4), name
            assert got["token_ids"] == case["token_ids"], name
            assert got["n_diff_steps"] == case["n_diff_steps"], name
    finally:
        model.float()


def test_sampler_settings_at_temperature_zero(golden, model):
    """top-k / top-p at temperature 0 leave the arg-max alone but change the confidences the threshold rule sees: the whole block in
    one step at top_k = 1, several slots per step otherwise. (The positive-temperature case of the fixture draws from the CUDA
    generator and is held to the engine on the GPU only.)"""
    import make_engine_golden as G
    from oracle import engine_flow as E

    ref = golden["sampling"]
    prompt = G.prompt(ref["prompt_len"], ref["seed"])
    model = model.double()
    try:
        for name, kwargs in G.SAMPLING_CASES.items():
            case = ref["cases"][name]
            assert "error" not in case, (name, case)
            if kwargs.get("temperature", 0.0) > 0:
                continue
            got = E.prefill_and_decode(model, prompt, block_length=BLOCK, mask_id=MASK, threshold=golden["threshold"], sampler=dict(kwargs))
            assert got["first_token"] == case["first_token_id"], name
            assert got["token_ids"] == case["token_ids"], name
            assert got["n_diff_steps"] == case["n_diff_steps"], name
        assert ref["cases"]["top_k_1"]["n_diff_steps"] == 1
    finally:
        model.float()


def test_per_head_keep_variants(golden, model):
    """Keep lists off the defaults (average pooling, no pooling + mean reduce, keep-low, chunk->query and bidirectional directions, a
    window of last layers): every list of the reference engine, up to swaps between scores tied at the cut."""
    import make_engine_golden as G
    from oracle import engine_flow as E

    ref = golden["per_head_keep_variants"]
    sel = golden["selection"]["selected"]
    chunks, query = _chunks()
    spans = golden["per_head_keep"]["meta"]
    swaps = 0
    for name, kwargs in G.KEEP_VARIANTS.items():
        case = ref["cases"][name]
        assert "error" not in case, (name, case)
        n_layers = int(kwargs.get("token_score_layers", 1))
        layers = [0] if kwargs.get("token_score_layer_mode", "first") == "first" else list(range(2 - n_layers, 2))
        for span_meta, ci in zip(spans, sel[:2]):
            mine, pooled = E.per_head_keep(
                model, [BOS], chunks[ci], query[-8:], capacity=128, num_kv_heads=2, layers=layers,
                attention_mask=kwargs.get("token_attention_mask", "causal"), pool_kernel=int(kwargs.get("token_score_pool_kernel", 7)),
                pooling=kwargs.get("token_score_pooling", "maxpool"), reduce_mode=kwargs.get("token_score_reduce", "sum"),
                direction=kwargs.get("token_score_direction", "query_to_chunk"), keep_high=kwargs.get("token_score_keep", "high") == "high")
            for layer in range(2):            # layers beyond the scored window reuse the last scored layer's lists
                scored = min(layer, len(layers) - 1)
                for h in range(2):
                    theirs = [i - span_meta["start"] for i in case["keep"][layer][h] if span_meta["start"] <= i < span_meta["end"]]
                    ours = mine[scored][h].tolist()
                    diff = set(ours) ^ set(theirs)
                    values = pooled[scored][h].detach()
                    cut = (min if kwargs.get("token_score_keep", "high") == "high" else max)(float(values[i]) for i in ours[1:])
                    assert len(theirs) == 128 and all(abs(float(values[i]) - cut) <= 1e-5 * max(abs(cut), 1e-12) for i in diff), (name, ci, layer, h, sorted(diff))
                    swaps += len(diff) // 2
    assert swaps < 64
