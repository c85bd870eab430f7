"""CPU pin of the oracle (oracle/hotpath.py) against the reference's own outputs.

tests/golden/toy_reference.json was produced by the UNMODIFIED reference class (tests/golden/make_golden.py). Here the
same stages are chained from the oracle's restated functions over the CPU contract model, and every intermediate the
golden file holds must come out again: chunking and chunk BOS, the partial draft, the self-information chunk scores
and the selected indices, the pooled query→chunk token scores and keep lists, and the confidence-threshold block loop.
No GPU and no reference checkout are needed.
"""

import json
import os
import sys

import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
sys.path.insert(0, os.path.dirname(HERE))

from oracle import hotpath as O  # noqa: E402

BOS, MASK = 1, 1023


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(HERE, "golden", "toy_reference.json")) as handle:
        return json.load(handle)


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    import make_golden
    from oracle.contract_model.model.modeling_dream import DreamModel

    path = str(tmp_path_factory.mktemp("ckpt_toy_cpu"))
    make_golden.write_toy_checkpoint(path)
    return DreamModel.from_pretrained(path).eval()


@pytest.fixture(scope="module")
def inputs():
    import make_golden

    return make_golden.toy_inputs()


def _causal_mask(length):
    mask = torch.full((1, 1, length, length), float("-inf"))
    return torch.triu(mask, diagonal=1)


def _positions(values):
    return torch.tensor([list(values)], dtype=torch.long)


@pytest.fixture(scope="module")
def chunks(golden, inputs):
    flags = golden["flags"]
    context, _ = inputs
    return [O.maybe_prepend_bos_to_chunk(c, [BOS], flags["chunk_size"]) for c in O.split_token_chunks(context, flags["chunk_size"])]


@pytest.fixture(scope="module")
def draft(golden, model, inputs):
    """Partial draft (reference :2595-2676): slot 0 from the last context logit, then rounds that confirm one slot each."""
    flags = golden["flags"]
    _, query = inputs
    ctx = [BOS] + query
    n_draft = flags["score_draft_tokens"]
    with torch.no_grad():
        out = model(torch.tensor([ctx]), attention_mask=None, position_ids=_positions(range(len(ctx))), use_cache=True)
        last_logit = out.logits[0, -1]
        block = torch.full((n_draft,), MASK, dtype=torch.long)
        block[0] = int(torch.argmax(last_logit))
        confirmed = [True] + [False] * (n_draft - 1)
        for _ in range(flags["score_draft_partial_rounds"]):
            step = model(block.unsqueeze(0), attention_mask=None, position_ids=_positions(range(len(ctx) + n_draft)),
                         past_key_values=out.past_key_values, use_cache=False)
            new_block, _, _ = O.unmask_step(step.logits[0], block, mask_token_id=MASK, threshold=2.0, last_logit=last_logit)
            confirmed = [c or bool(a != b) for c, a, b in zip(confirmed, new_block.tolist(), block.tolist())]
            block = new_block
    return block.tolist(), confirmed


def test_chunking_and_chunk_bos(golden, chunks):
    ref = golden["runs"]["readme_full_prompt_mask"]
    assert len(chunks) == ref["candidate_chunks"]
    assert all(c[0] == BOS and len(c) <= golden["flags"]["chunk_size"] for c in chunks)
    for meta in ref["chunk_meta"]:
        assert len(chunks[meta["chunk_index"]]) == meta["original_tokens"]


def test_partial_draft(golden, draft, inputs):
    _, query = inputs
    for name, ref in golden["runs"].items():
        if "draft_ids" in ref:          # variants that draft with score_draft_partial_rounds
            assert draft[0] == ref["draft_ids"]
            assert draft[1] == ref["draft_confirmed"]
    # score_draft_partial_steps=2 stops after the same two slots (reference :2512-2593)
    steps = golden["runs"]["draft_partial_steps"]
    assert steps["selection_query_ids"] == query + draft[0] and steps["score_token_mask"] == [True] * len(query) + draft[1]


def _draft_block(model, query, n_draft, fill):
    """Draft of n_draft slots behind [BOS ‖ query] with no context; `fill(logits, block, last_logit)` is the transfer rule."""
    ctx = [BOS] + query
    with torch.no_grad():
        out = model(torch.tensor([ctx]), attention_mask=None, position_ids=_positions(range(len(ctx))), use_cache=True)
        last_logit = out.logits[0, -1]
        block = torch.full((n_draft,), MASK, dtype=torch.long)
        block[0] = int(torch.argmax(last_logit))
        guard = 0
        while bool((block == MASK).any()) and guard < n_draft + 8:
            guard += 1
            step = model(block.unsqueeze(0), attention_mask=None, position_ids=_positions(range(len(ctx) + n_draft)),
                         past_key_values=out.past_key_values, use_cache=False)
            block = fill(step.logits[0], block, last_logit)
    return block.tolist()


def test_draft_paths_of_the_config_defaults(golden, model, inputs):
    """score_draft_partial_rounds unset (the dataclass default): a complete confidence-threshold draft (reference
    :1828-1837 → generate_from_cache), or with score_draft_fixed_steps the fixed-step diffusion sampler (:2443-2510)."""
    _, query = inputs
    ref = golden["runs"]["draft_dataclass_defaults"]
    n = ref["flags"]["score_draft_tokens"]
    ids = _draft_block(model, query, n, lambda lg, blk, last: O.unmask_step(lg, blk, mask_token_id=MASK, threshold=ref["flags"]["threshold"],
                                                                            last_logit=last)[0])
    assert ref["selection_query_ids"] == query + ids and ref["score_token_mask"] is None
    ref = golden["runs"]["draft_fixed_steps"]
    n, steps = ref["flags"]["score_draft_tokens"], ref["flags"]["score_draft_steps"]
    counts = iter(c for c in O.fixed_step_transfer_counts(n - 1, steps) if c > 0)
    ids = _draft_block(model, query, n, lambda lg, blk, last: O.transfer_most_confident(lg, blk, mask_token_id=MASK, count=next(counts),
                                                                                        last_logit=last))
    assert ref["selection_query_ids"] == query + ids and ref["score_token_mask"] is None


@pytest.fixture(scope="module")
def chunk_scores(golden, model, inputs, chunks, draft):
    """draft-self-information score of every chunk (reference :1314-1423)."""
    _, query = inputs
    selection = query + draft[0]
    label_mask = [True] * len(query) + draft[1]
    scores = []
    with torch.no_grad():
        for chunk in chunks:
            row = [BOS] + chunk + selection
            label_pos, labels = O.score_labels(1, len(chunk), selection, label_mask)
            out = model(torch.tensor([row]), attention_mask=_causal_mask(len(row)), position_ids=_positions(range(len(row))))
            rows = out.logits[0, [p - 1 for p in label_pos]]
            score, _ = O.self_information_scores(rows.unsqueeze(0), torch.tensor(labels))
            scores.append(float(score[0]))
    return scores


def test_chunk_scores_and_selection(golden, chunk_scores):
    for name, ref in golden["runs"].items():
        if name in ("draft_dataclass_defaults", "draft_fixed_steps"):   # other draft, other labels, other scores
            continue
        want = [ref["chunk_scores"][str(i)] for i in range(len(chunk_scores))]
        assert max(abs(a - b) for a, b in zip(chunk_scores, want)) < 1e-5, name
        assert O.rank_chunks(chunk_scores, ref["flags"]["topk_chunks"]) == ref["selected_chunk_indices"], name


def _head_scores(model, chunk, window):
    """Per layer fp32 [Hq, C]: attention mass the query window puts on each chunk token (reference :1639-1667), from
    the eager probabilities of a causal forward over [prefix ‖ chunk ‖ window]."""
    joint = [BOS] + chunk + window
    length = len(joint)
    with torch.no_grad():
        out = model(torch.tensor([joint]), attention_mask=_causal_mask(length), position_ids=_positions(range(length)),
                    output_attentions=True)
    rows = slice(1 + len(chunk), length)
    return [attn[0][:, rows, 1:1 + len(chunk)].float().sum(dim=1) for attn in out.attentions]


def test_token_scores_and_global_keep(golden, model, inputs, chunks, draft):
    ref = golden["runs"]["evict_global_cap128"]
    _, query = inputs
    window = query[-8:]  # token_score_use_generated is off: the eviction query is the plain query (reference :1955-1995)
    cap = ref["flags"]["token_capacity"]
    for order, ci in enumerate(ref["selected_chunk_indices"]):
        chunk = chunks[ci]
        scores = O.global_token_scores(_head_scores(model, chunk, window))
        want = torch.tensor(ref["token_scores"][order])
        assert torch.allclose(scores, want, rtol=1e-5, atol=1e-7)
        keep = O.select_positions_from_token_scores(scores, capacity=cap, chunk_len=len(chunk)).tolist()
        assert keep == ref["keep_positions"][order]
    assert sum(m["kept_tokens"] for m in ref["chunk_meta"]) + 1 == ref["cache_tokens"]


def test_per_head_keep_up_to_exact_ties(golden, model, inputs, chunks):
    """torch.topk's pick among EXACTLY equal scores at the cut is unspecified (max-pool plateaus make such ties
    common); the restatement keeps the lower position. Everything strictly above the cut must match."""
    ref = golden["runs"]["evict_per_head_cap128_chunk_query"]
    _, query = inputs
    window = query[-8:]
    cap, hkv = ref["flags"]["token_capacity"], 2
    swaps = 0
    for order, ci in enumerate(ref["selected_chunk_indices"]):
        chunk = chunks[ci]
        for layer, hs in enumerate(_head_scores(model, chunk, window)):
            pooled = O.per_head_token_scores(hs, hkv)
            for h in range(hkv):
                mine = O.select_positions_from_token_scores(pooled[h], capacity=cap, chunk_len=len(chunk)).tolist()
                theirs = ref["keep_positions_per_head"][order][layer][h]
                assert len(mine) == len(theirs) == cap
                diff = set(mine) ^ set(theirs)
                if diff:
                    cut = min(float(pooled[h][i]) for i in mine[1:])
                    assert all(float(pooled[h][i]) == cut for i in diff)
                    swaps += len(diff) // 2
    assert swaps < 32  # a handful of tie swaps among 4 chunks x 2 layers x 2 heads x 128 kept


@pytest.mark.parametrize("variant", ["readme_full_prompt_mask", "two_blocks"])
def test_block_denoising(golden, model, inputs, chunks, variant):
    """Joint prefill over [prefix ‖ selected chunks ‖ query ‖ MASKs] and the dual-cache confidence-threshold loop
    (reference :2776-3024, :2399-2441): block states before every forward and the final ids."""
    ref = golden["runs"][variant]
    flags = ref["flags"]
    _, query = inputs
    prompt = [BOS] + [t for ci in ref["selected_chunk_indices"] for t in chunks[ci]] + query
    max_new, blen = flags["max_new_tokens"], flags["block_length"]
    full = prompt + [MASK] * max_new
    n0 = len(prompt)
    positions = _positions(range(len(full)))
    states, generated = [], []
    with torch.no_grad():
        out = model(torch.tensor([full]), attention_mask=None, position_ids=positions, use_cache=True)
        cache = out.past_key_values
        last_logit = out.logits[0, n0 - 1]
        for b in range(max_new // blen):
            lo = n0 + b * blen
            if b > 0:
                # suffix initialisation (reference :2368-2397): all remaining MASKs against prompt + finished blocks
                done = [(k[:, :lo], v[:, :lo]) for k, v in cache]
                suffix = torch.full((1, len(full) - lo), MASK, dtype=torch.long)
                cache = model(suffix, attention_mask=None, position_ids=positions, past_key_values=done, use_cache=True).past_key_values
            block = torch.full((blen,), MASK, dtype=torch.long)
            block[0] = int(torch.argmax(last_logit))
            replace = torch.zeros((1, len(full)), dtype=torch.bool)
            replace[0, lo:lo + blen] = True
            while bool((block == MASK).any()):
                states.append(block.tolist())
                step = model(block.unsqueeze(0), attention_mask=None, position_ids=positions, past_key_values=cache,
                             use_cache=False, dual_cache=True, replace_position=replace)
                block, _, _ = O.unmask_step(step.logits[0], block, mask_token_id=MASK, threshold=flags["threshold"], last_logit=last_logit)
            generated.extend(block.tolist())
            states.append(block.tolist())  # the commit forward of the finished block
            commit = model(block.unsqueeze(0), attention_mask=None, position_ids=positions, past_key_values=cache,
                           use_cache=True, dual_cache=True, replace_position=replace)
            cache, last_logit = commit.past_key_values, commit.logits[0, -1]
    assert generated == ref["sequences"]
    # the golden list also holds the 4-slot draft round, which goes through the same forward helper
    assert states == [s for s in ref["block_states_before_each_forward"] if len(s) == blen]


def test_engine_flow_block_loop_reproduces_the_two_block_golden(golden, model, inputs, chunks):
    """`oracle.engine_flow.decode_blocks` (the checker of the engine's records of several blocks) on the prompt of the reference
    class's `two_blocks` run: its ids. That run keeps the prefill's MASK-slot K/V for the first block where this function
    recomputes them from the prompt K/V, which gives the same values."""
    from oracle import engine_flow as E

    ref = golden["runs"]["two_blocks"]
    _, query = inputs
    prompt = [BOS] + [t for ci in ref["selected_chunk_indices"] for t in chunks[ci]] + query
    out = E.decode_blocks(model, prompt, max_new=64, block_length=32, mask_id=MASK, threshold=ref["flags"]["threshold"], shift=True,
                          softmax_dtype=None)
    assert out["token_ids"] == ref["sequences"]
    unshifted = E.decode_blocks(model, prompt, max_new=40, block_length=32, mask_id=MASK, threshold=ref["flags"]["threshold"], shift=False)
    assert len(unshifted["token_ids"]) == 40 and MASK not in unshifted["token_ids"] and unshifted["token_ids"] != ref["sequences"][:40]


def test_whole_request_port_and_staged_reference_class(golden, model, inputs, tmp_path):
    """The chained CPU restatement of a whole README-flags request reproduces the golden ids and selection; when the
    reference's own class is staged under oracle/_ref it is run as well (it is what produced the golden)."""
    from oracle import build_ref, toy_request

    context, query = inputs
    ref = golden["runs"]["readme_full_prompt_mask"]
    got = toy_request.run_port(model, context, query, ref["flags"], bos=BOS, mask_id=MASK)
    assert got["sequences"] == ref["sequences"] and got["selected"] == ref["selected_chunk_indices"]
    assert max(abs(a - ref["chunk_scores"][str(i)]) for i, a in enumerate(got["scores"])) < 1e-5
    if not build_ref.staged():
        pytest.skip("oracle/_ref not staged on this machine (oracle/build_ref.py)")
    import make_golden

    ckpt = str(tmp_path / "ckpt")
    make_golden.write_toy_checkpoint(ckpt)
    theirs = toy_request.run_reference_class(ckpt, context, query, ref["flags"])
    assert theirs["sequences"] == ref["sequences"] and theirs["selected"] == ref["selected_chunk_indices"]
