"""The GPU runtime at the head shape and dtype the tensor-core attention kernel serves, against the reference class.

tests/golden/toy128_reference.json holds what the UNMODIFIED reference `FastDLLMParallelComp` produced on CPU for a
Dream-architecture toy with head_dim 128 (2 layers, hidden 512, 4 query / 2 KV heads, vocabulary 4096), in float32 and in
bfloat16 (tests/golden/make_golden.py). Two runs of the GPU runtime are held to it:

  * float32 — the SIMT attention kernel; the same exact gates as the head_dim-64 toy;
  * bfloat16 — every attention call must have run on the tcgen05 kernel. A random-init model decides between nearly
    equal probabilities (about 1 / vocabulary each), so two bf16 implementations that round in a different order flip
    near-ties, and one flipped token changes everything after it. The run is therefore compared STAGE BY STAGE with the
    reference's own upstream results substituted before the next stage (draft -> scores and selection -> keep lists ->
    every denoise step given the reference's block state before it), and a disagreement only passes when it is a
    near-tie under the GPU's own numbers: pooled eviction scores within 1e-2 relative of the cut; for a denoise step, the
    log-probabilities of the reference's transfer and of ours closer than the bf16 noise of that step. The noise is
    MEASURED: the same forced trajectory is run in float32 on the SIMT path (which the float32 test holds exactly to the
    reference), and the step's bf16 logits must (a) agree with the float32 logits to bf16 accuracy (relative error below
    3e-2 over the block's rows, which a wrong mask, page or tile would miss by orders of magnitude); (b) wherever the
    float32 run's own decision has a margin above the noise bound, the bf16 run must take the same (slot, token); and (c) any
    transfer that differs from the bf16 reference's must have a log-probability gap below twice that bound. The bound: 10 x
    the RMS difference between the two precisions plus three bf16 ulps of the deciding logit. Why 10: the gap compares two logits in each of two bf16 implementations
    (ours and the reference's CPU run), four noise terms of that RMS, so its standard deviation is 2 RMS, and with some
    ten near-top candidates on each of a hundred-odd steps a 4-sigma excursion is expected somewhere; 10 RMS is 5 sigma.
    The ulps: each implementation rounds its LM-head output to bf16 and the reference rounds the probability itself to
    bf16 before ranking the slots. All MASK rows of a random-init model carry almost
    the same distribution, so WHICH slot is filled first is decided inside that noise on most steps; the raw
    (slot, token) agreement is printed and has a low floor of its own.
"""

import json
import math
import os
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
NEAR_TIE = 1e-2


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(HERE, "golden", "toy128_reference.json")) as handle:
        return json.load(handle)


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    import make_golden

    path = str(tmp_path_factory.mktemp("ckpt_toy128"))
    make_golden.write_toy_checkpoint(path, config=make_golden.TOY128)
    return path


def _run(ckpt, ref, dtype, *, force):
    """generate() with every stage recorded; with `force`, the reference's result of a stage replaces ours before the next."""
    import make_golden
    import prefilling_dllm_b200.ops as ops
    from prefilling_dllm_b200.parallelcomp import load_fastdllm_parallelcomp

    flags = dict(ref["flags"])
    rt = load_fastdllm_parallelcomp(pretrained=ckpt, device="cuda", dtype=dtype, decode_cuda_graph=not force, **flags)
    mask_id = rt._mask_token_id()
    blen = flags["block_length"]
    cap = {"kernels": [], "steps": [], "keep": [], "pooled": [], "logits": [], "slots": [], "after": []}

    orig_attn, orig_unmask, orig_select = ops.paged_attention, ops.unmask_step_batched, ops.evict_select
    orig_selection = rt._selection_query_ids_with_score_target
    orig_keep = rt._keep_positions_for_chunk
    orig_keep_ph = rt._keep_positions_per_layer_per_head_for_chunk
    # block states before every forward of the block loop; a state without MASK is a block's commit forward (no transfer
    # follows it), every other state is followed by the state its denoise step produced
    states = [s for s in ref["block_states_before_each_forward"] if len(s) == blen]
    pairs = [(states[i], states[i + 1]) for i in range(len(states) - 1) if mask_id in states[i]]
    cursor = {"i": 0}

    def attn(*a, **kw):
        used = orig_attn(*a, **kw)
        cap["kernels"].append(used)
        return used

    def selection(prefix_ids, scoring_query_ids):
        ids, count, mask = orig_selection(prefix_ids, scoring_query_ids)
        cap["selection_query_ids"], cap["score_token_mask"] = list(ids), None if mask is None else [bool(x) for x in mask]
        if force:
            ids, mask = list(ref["selection_query_ids"]), ref["score_token_mask"]
        return ids, count, mask

    def select_and_record(head_scores, **kw):
        keep_idx, pooled = orig_select(head_scores, **dict(kw, return_pooled=True))
        cap["pooled"].append(pooled.float().cpu())
        return keep_idx

    def keep(*a):
        out = orig_keep(*a)
        cap["keep"].append(list(out))
        if force and "keep_positions" in ref:
            out = list(ref["keep_positions"][len(cap["keep"]) - 1])
        return out

    def keep_ph(*a):
        out = orig_keep_ph(*a)
        cap["keep"].append([t.tolist() for t in out])
        if force and "keep_positions_per_head" in ref:
            theirs = ref["keep_positions_per_head"][len(cap["keep"]) - 1]
            out = [torch.tensor(layer, dtype=t.dtype, device=t.device) for layer, t in zip(theirs, out)]
        return out

    def unmask(logits, block_ids, **kw):
        before = block_ids.clone()
        counts = orig_unmask(logits, block_ids, **kw)
        i = cursor["i"]
        cursor["i"] += 1
        if not force or i >= len(pairs):
            return counts
        want_before = torch.tensor(pairs[i][0], device=block_ids.device).view_as(block_ids)
        want_after = torch.tensor(pairs[i][1], device=block_ids.device).view_as(block_ids)
        rec = {"step": i, "same_input": bool(torch.equal(before, want_before)), "same": bool(torch.equal(block_ids, want_after))}
        last = kw.get("last_logit")
        rows = logits[0].float()
        shifted = torch.cat([last[0:1].float(), rows[:-1]], dim=0) if kw.get("shift", True) else rows
        masked_rows = (before[0] == mask_id).nonzero().flatten().cpu()
        cap["logits"].append(shifted.cpu()[masked_rows])      # the rows the step decides on, fp32 copies
        cap["slots"].append(masked_rows.tolist())
        cap["after"].append(block_ids[0].tolist())            # this run's own state after the step (before forcing)
        if rec["same_input"] and not rec["same"]:
            # near-tie? compare, under THIS run's probabilities, the reference's transfers with ours
            logp = torch.log_softmax(shifted, dim=-1)
            mine = [(s, int(block_ids[0, s])) for s in range(blen) if int(before[0, s]) == mask_id and int(block_ids[0, s]) != mask_id]
            theirs = [(s, int(want_after[0, s])) for s in range(blen) if int(want_before[0, s]) == mask_id and int(want_after[0, s]) != mask_id]
            lp_mine = min(float(logp[s, t]) for s, t in mine)
            lp_theirs = min(float(logp[s, t]) for s, t in theirs)
            top = max(abs(float(shifted[s, t])) for s, t in mine + theirs)
            ulp = 2.0 ** (math.floor(math.log2(max(top, 1e-30))) - 7)      # bf16: 8 significant bits
            rec.update(mine=mine, theirs=theirs, gap=abs(lp_mine - lp_theirs), tol=3 * ulp)
        cap["steps"].append(rec)
        block_ids.copy_(want_after)
        counts[:, 2] = (want_after == mask_id).sum()
        return counts

    ops.paged_attention, ops.unmask_step_batched, ops.evict_select = attn, unmask, select_and_record
    rt._selection_query_ids_with_score_target = selection
    rt._keep_positions_for_chunk, rt._keep_positions_per_layer_per_head_for_chunk = keep, keep_ph
    context, query = make_golden.toy_inputs(vocab=make_golden.TOY128["vocab_size"])
    try:
        result = rt.generate(prefix_ids=rt.bos_ids(), context_ids=context, query_ids=query)
    finally:
        ops.paged_attention, ops.unmask_step_batched, ops.evict_select = orig_attn, orig_unmask, orig_select
    ops.check_status(rt.device)
    assert rt.model.allocator.num_free_pages == rt.model.num_pages, "pages leaked"
    return result, cap


VARIANTS = ["readme_full_prompt_mask", "chunk_query_evict_global_cap128_two_blocks", "evict_per_head_cap128_full_prompt"]


def _check_bookkeeping(result, ref):
    assert result.cache_tokens == ref["cache_tokens"] and result.removed_tokens == ref["removed_tokens"]
    for mine, theirs in zip(result.chunk_meta, ref["chunk_meta"]):
        for key in ("chunk_index", "original_tokens", "kept_tokens", "cache_start", "cache_end", "rope_start", "rope_end"):
            assert getattr(mine, key) == theirs[key], key


def _keep_lists_equal_up_to_ties(cap, ref, rel_tol):
    """Global lists: [chunk][positions]; per-head: [chunk][layer][head][positions]. Returns the number of swapped picks."""
    swaps = 0
    theirs_all = ref.get("keep_positions") or ref.get("keep_positions_per_head") or []
    assert len(cap["keep"]) == len(theirs_all)
    for ci, (mine_c, ref_c) in enumerate(zip(cap["keep"], theirs_all)):
        if mine_c == ref_c:
            continue
        pooled = cap["pooled"][ci]          # one evict_select call per chunk whenever eviction is on
        rows = [(mine_c, ref_c, pooled.reshape(-1, pooled.shape[-1])[0])] if "keep_positions" in ref else [
            (mine_c[layer][h], ref_c[layer][h], pooled[layer, h]) for layer in range(len(ref_c)) for h in range(len(ref_c[layer]))]
        for mine, theirs, scores in rows:
            assert len(mine) == len(theirs) and mine[0] == 0 and theirs[0] == 0
            diff = set(mine) ^ set(theirs)
            if diff:
                cut = min(float(scores[i]) for i in mine[1:])
                assert all(abs(float(scores[i]) - cut) <= rel_tol * abs(cut) for i in diff), (ci, sorted(diff))
                swaps += len(diff) // 2
    return swaps


@pytest.mark.parametrize("variant", VARIANTS)
def test_float32_run_is_exact(golden, ckpt, variant):
    ref = golden["runs"][f"{variant}/float32"]
    result, cap = _run(ckpt, ref, "float32", force=False)
    assert set(cap["kernels"]) == {"simt"}
    assert cap["selection_query_ids"] == ref["selection_query_ids"] and cap["score_token_mask"] == ref["score_token_mask"]
    scores = [result.chunk_scores[i] for i in range(len(ref["chunk_scores"]))]
    assert max(abs(a - ref["chunk_scores"][str(i)]) for i, a in enumerate(scores)) < 1e-4
    assert result.selected_chunk_indices == ref["selected_chunk_indices"]
    _check_bookkeeping(result, ref)
    swaps = _keep_lists_equal_up_to_ties(cap, ref, 0.0)
    if swaps:   # exact ties at a cut picked differently: hold the rest of the path to the gate with the reference's picks
        result, _ = _run(ckpt, dict(ref, block_states_before_each_forward=[]), "float32", force=True)
    match = sum(int(a == b) for a, b in zip(result.sequences, ref["sequences"])) / len(ref["sequences"])
    print(f"{variant}/float32: {swaps} exact-tie swaps in keep lists, greedy token match {match:.3f}")
    assert match >= 0.99


@pytest.mark.parametrize("variant", VARIANTS)
def test_bfloat16_run_on_the_tensor_core_kernel(golden, ckpt, variant):
    ref = golden["runs"][f"{variant}/bfloat16"]
    ref32 = golden["runs"][f"{variant}/float32"]
    _, cap32 = _run(ckpt, ref, "float32", force=True)       # the same forced trajectory in float32: the yardstick for bf16 noise
    result, cap = _run(ckpt, ref, "bfloat16", force=True)
    assert set(cap["kernels"]) == {"tc"}, f"attention kernels used: {set(cap['kernels'])}"
    # draft
    assert cap["selection_query_ids"] == ref["selection_query_ids"], "draft differs from the reference's bf16 draft"
    assert cap["score_token_mask"] == ref["score_token_mask"]
    # chunk scores and the bit-exact selection, with the gap at the cut
    n = len(ref["chunk_scores"])
    scores = [result.chunk_scores[i] for i in range(n)]
    d16 = max(abs(scores[i] - ref["chunk_scores"][str(i)]) for i in range(n))
    d32 = max(abs(scores[i] - ref32["chunk_scores"][str(i)]) for i in range(n))
    ordered = sorted((ref["chunk_scores"][str(i)] for i in range(n)), reverse=True)
    k = len(ref["selected_chunk_indices"])
    print(f"{variant}/bfloat16: max |score - reference bf16| = {d16:.2e}, vs reference fp32 = {d32:.2e}, "
          f"gap at the top-{k} cut = {ordered[k - 1] - ordered[k]:.2e}")
    assert d16 < 2e-3 and d32 < 3e-3
    assert result.selected_chunk_indices == ref["selected_chunk_indices"] == ref32["selected_chunk_indices"]
    _check_bookkeeping(result, ref)
    # eviction keep lists: equal up to near-ties of the pooled scores at the cut
    swaps = _keep_lists_equal_up_to_ties(cap, ref, NEAR_TIE)
    # every denoise step, given the reference's block state before it
    steps = cap["steps"]
    assert len(steps) >= ref["flags"]["max_new_tokens"] // 2
    assert all(s["same_input"] for s in steps), "a block's first token differs from the reference's"
    same = sum(int(s["same"]) for s in steps)
    # (a) the bf16 logits of every step against the float32 run of the same trajectory
    assert len(cap["logits"]) == len(cap32["logits"]) == len(steps)
    rel, rms = [], []
    for l16, l32 in zip(cap["logits"], cap32["logits"]):
        rel.append(float((l16 - l32).norm() / l32.norm()))
        rms.append(float((l16 - l32).pow(2).mean().sqrt()))
    print(f"{variant}/bfloat16: logits vs the float32 run of the same trajectory: relative error max {max(rel):.2e} / median "
          f"{sorted(rel)[len(rel) // 2]:.2e}; RMS difference per logit max {max(rms):.2e}")
    assert max(rel) < 3e-2
    # (b) wherever exact arithmetic decides clearly, bf16 decides the same. The float32 run's own decision at a step and its
    # margin — the log-probability gap between its transfer and the best other candidate (another slot's arg-max, or the
    # runner-up token of the same slot) — come from its logits; a margin above the noise bound must be reproduced.
    decided, agreed = 0, 0
    for i, (l32, slots, after32, after16) in enumerate(zip(cap32["logits"], cap32["slots"], cap32["after"], cap["after"])):
        logp = torch.log_softmax(l32, dim=-1)
        top2 = logp.topk(2, dim=-1).values                     # per candidate slot: best and runner-up token
        order = top2[:, 0].argsort(descending=True)
        best = float(top2[order[0], 0])
        other = max(float(top2[order[0], 1]), float(top2[order[1], 0]) if len(order) > 1 else float("-inf"))
        bound = 10 * rms[i] + 3 * 2.0 ** (math.floor(math.log2(max(float(l32.abs().max()), 1e-30))) - 7)
        if best - other > bound:
            decided += 1
            agreed += int(after16 == after32)
    print(f"{variant}/bfloat16: {decided}/{len(steps)} steps have a float32 decision margin above the noise bound; bf16 reproduces {agreed} of them")
    assert agreed == decided
    # (c) transfers that differ from the bf16 reference's: every one within twice the bound (the two bf16 implementations each
    # carry that noise), and the size of the worst is printed
    flips = [dict(s, tol=s["tol"] + 10 * rms[i]) for i, s in enumerate(steps) if not s["same"]]
    worst = max((s["gap"] / s["tol"] for s in flips), default=0.0)
    print(f"{variant}/bfloat16: {swaps} near-tie swaps in keep lists; {same}/{len(steps)} denoise steps transfer the reference's "
          f"(slot, token); the other {len(flips)} differ by at most {worst:.2f} x (10 RMS of the step's bf16 noise + 3 bf16 ulps)")
    assert all(s["gap"] <= 2 * s["tol"] for s in flips), [(s["step"], s["mine"], s["theirs"], s["gap"], s["tol"]) for s in flips if s["gap"] > 2 * s["tol"]]
    assert same / len(steps) >= 0.25
