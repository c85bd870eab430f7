"""One whole request of the README flow on the CPU toy, two ways. TEST INFRASTRUCTURE ONLY (tests/ and bench.py's CPU arm).

  * run_reference_class: the reference's own `FastDLLMParallelComp` (staged copy under oracle/_ref, see build_ref.py) over
    oracle/contract_model, on the host cores — the CPU baseline `kind: "reference"`;
  * run_port: the same flow chained from the restatements in oracle/hotpath.py (draft, scoring, ranking, joint prefill,
    dual-cache block denoising; E:fastdllm_parallelcomp.py:1800-1953, 2776-3024) — the fallback `kind: "port"` when nothing is
    staged, and a whole-flow check of the restatements against the goldens (tests/test_oracle_golden.py).

Both return {"sequences", "selected", "seconds": {phase: s}, "decode_tok_per_s"}; flags follow the reference's config.
"""

from __future__ import annotations

import os
import time
from typing import Dict, List, Sequence

import torch

from . import hotpath as O

HERE = os.path.dirname(os.path.abspath(__file__))


def _positions(values) -> torch.Tensor:
    return torch.tensor([list(values)], dtype=torch.long)


def _causal_mask(length: int) -> torch.Tensor:
    mask = torch.full((1, 1, length, length), float("-inf"))
    return torch.triu(mask, diagonal=1)


def run_port(model, context: Sequence[int], query: Sequence[int], flags: Dict, *, bos: int = 1, mask_id: int = 1023,
             backend: str = "dream") -> Dict:
    """README flow (full_prompt_mask, partial draft rounds, single-chunk causal scoring, no eviction) from oracle/hotpath.py.
    backend "llada": the reference's un-shifted read-out on the same weights (E:fastdllm_parallelcomp.py:1017-1024) — a block's
    first token comes from the first MASK slot's own row (:2390-2397, :2915-2922), every step reads slot p from logits[p], and
    chunks are scored leave-one-out (:1166-1201): one forward per label with that label masked, its log-probability read at
    its own row. PARITY UNPINNED for this backend: the reference needs the Fast-dLLM v1 LLaDA plug-in to run it."""
    shift = backend != "llada"
    if flags.get("cache_build_mode") != "full_prompt_mask" or int(flags.get("token_capacity") or 0) != 0 or flags.get("score_draft_partial_rounds") is None:
        raise ValueError("run_port covers the README flags only")
    query = list(query)
    secs: Dict[str, float] = {}
    t0 = time.perf_counter()
    chunks = [O.maybe_prepend_bos_to_chunk(c, [bos], flags["chunk_size"]) for c in O.split_token_chunks(context, flags["chunk_size"])]
    n_draft = int(flags["score_draft_tokens"])
    with torch.no_grad():
        # draft: slot 0 from the last context logit, then rounds that confirm the single most confident slot
        ctx = [bos] + query
        out = model(torch.tensor([ctx]), attention_mask=None, position_ids=_positions(range(len(ctx))), use_cache=True)
        last_logit = out.logits[0, -1]
        block = torch.full((n_draft,), mask_id, dtype=torch.long)
        if shift:
            block[0] = int(torch.argmax(last_logit))
        else:
            init = model(block.unsqueeze(0), attention_mask=None, position_ids=_positions(range(len(ctx) + n_draft)),
                         past_key_values=out.past_key_values, use_cache=False)
            block[0] = int(torch.argmax(init.logits[0, 0]))
        confirmed = [True] + [False] * (n_draft - 1)
        for _ in range(int(flags["score_draft_partial_rounds"])):
            step = model(block.unsqueeze(0), attention_mask=None, position_ids=_positions(range(len(ctx) + n_draft)),
                         past_key_values=out.past_key_values, use_cache=False)
            new_block, _, _ = O.unmask_step(step.logits[0], block, mask_token_id=mask_id, threshold=2.0,
                                            last_logit=last_logit if shift else None, shift=shift)
            confirmed = [c or bool(a != b) for c, a, b in zip(confirmed, new_block.tolist(), block.tolist())]
            block = new_block
        secs["draft"] = time.perf_counter() - t0
        # scoring: causal forward of [BOS | chunk | query | draft], mean log-probability of the labelled positions
        t1 = time.perf_counter()
        selection = query + block.tolist()
        label_mask = [True] * len(query) + confirmed
        scores: List[float] = []
        for chunk in chunks:
            row = [bos] + chunk + selection
            label_pos, labels = O.score_labels(1, len(chunk), selection, label_mask)
            if shift:
                res = model(torch.tensor([row]), attention_mask=_causal_mask(len(row)), position_ids=_positions(range(len(row))))
                rows = res.logits[0, [p - 1 for p in label_pos]]
            else:
                picked = []
                for p in label_pos:
                    hidden_label = list(row)
                    hidden_label[p] = mask_id
                    res = model(torch.tensor([hidden_label]), attention_mask=_causal_mask(len(row)), position_ids=_positions(range(len(row))))
                    picked.append(res.logits[0, p])
                rows = torch.stack(picked, dim=0)
            score, _ = O.self_information_scores(rows.unsqueeze(0), torch.tensor(labels))
            scores.append(float(score[0]))
        selected = O.rank_chunks(scores, int(flags["topk_chunks"]))
        secs["scoring"] = time.perf_counter() - t1
        # joint prefill + dual-cache block denoising
        t2 = time.perf_counter()
        prompt = [bos] + [t for ci in selected for t in chunks[ci]] + query
        max_new, blen = int(flags["max_new_tokens"]), int(flags["block_length"])
        full = prompt + [mask_id] * max_new
        n0 = len(prompt)
        positions = _positions(range(len(full)))
        res = model(torch.tensor([full]), attention_mask=None, position_ids=positions, use_cache=True)
        cache, last_logit = res.past_key_values, res.logits[0, n0 - 1]
        first_logit = last_logit if shift else res.logits[0, n0]
        secs["prefill"] = time.perf_counter() - t2
        t3 = time.perf_counter()
        generated: List[int] = []
        for b in range(max_new // blen):
            lo = n0 + b * blen
            if b > 0:
                done = [(k[:, :lo], v[:, :lo]) for k, v in cache]
                suffix = torch.full((1, len(full) - lo), mask_id, dtype=torch.long)
                init = model(suffix, attention_mask=None, position_ids=positions, past_key_values=done, use_cache=True)
                cache = init.past_key_values
                first_logit = last_logit if shift else init.logits[0, 0]
            block = torch.full((blen,), mask_id, dtype=torch.long)
            block[0] = int(torch.argmax(first_logit))
            replace = torch.zeros((1, len(full)), dtype=torch.bool)
            replace[0, lo:lo + blen] = True
            while bool((block == mask_id).any()):
                step = model(block.unsqueeze(0), attention_mask=None, position_ids=positions, past_key_values=cache, use_cache=False,
                             dual_cache=True, replace_position=replace)
                block, _, _ = O.unmask_step(step.logits[0], block, mask_token_id=mask_id, threshold=float(flags["threshold"]),
                                            last_logit=last_logit if shift else None, shift=shift)
            generated.extend(block.tolist())
            commit = model(block.unsqueeze(0), attention_mask=None, position_ids=positions, past_key_values=cache, use_cache=True,
                           dual_cache=True, replace_position=replace)
            cache, last_logit = commit.past_key_values, commit.logits[0, -1]
        secs["decode"] = time.perf_counter() - t3
    secs["total"] = time.perf_counter() - t0
    return {"sequences": generated, "selected": selected, "scores": scores, "seconds": secs,
            "decode_tok_per_s": len(generated) / secs["decode"]}


def run_reference_class(ckpt: str, context: Sequence[int], query: Sequence[int], flags: Dict, *, dtype: str = "float32", repeats: int = 1) -> Dict:
    """The staged, unmodified reference class on CPU; phases timed by wrapping its bound methods. Raises
    build_ref.RefUnavailable when oracle/_ref is empty."""
    from . import build_ref

    ref = build_ref.load_eval_module()
    runtime = ref.load_fastdllm_parallelcomp(pretrained=ckpt, fastdllm_dream_dir=os.path.join(HERE, "contract_model"), device="cpu",
                                             dtype=dtype, trust_remote_code=False, **flags)
    secs = {"draft": 0.0, "scoring": 0.0, "decode": 0.0}

    def timed(name, fn):
        def wrapper(*a, **k):
            t = time.perf_counter()
            try:
                return fn(*a, **k)
            finally:
                secs[name] += time.perf_counter() - t
        return wrapper

    runtime._selection_query_ids_with_score_target = timed("draft", runtime._selection_query_ids_with_score_target)
    runtime.score_chunks_self_information_batched = timed("scoring", runtime.score_chunks_self_information_batched)
    runtime._denoise_block_confidence_threshold = timed("decode", runtime._denoise_block_confidence_threshold)
    result = None
    t0 = time.perf_counter()
    for _ in range(max(1, repeats)):
        result = runtime.generate(prefix_ids=runtime.bos_ids(), context_ids=list(context), query_ids=list(query))
    total = (time.perf_counter() - t0) / max(1, repeats)
    secs = {k: v / max(1, repeats) for k, v in secs.items()}
    secs["total"] = total
    secs["prefill"] = max(0.0, total - secs["draft"] - secs["scoring"] - secs["decode"])
    n_new = len(result.sequences)
    return {"sequences": list(result.sequences), "selected": list(result.selected_chunk_indices), "seconds": secs,
            "decode_tok_per_s": n_new / secs["decode"] if secs["decode"] > 0 else None}
