"""CPU restatement of the reference ENGINE's prefill/decode flow. Test infrastructure: not imported by the product.

Follows prefilling_dllm_engine/prefilling_dllm/fastdllm_engine.py on the CPU contract model
(oracle/contract_model): joint `[prompt ‖ MASK block]` prefill (:2004-2040, :2084-2088), block denoising against the
prompt KV with an fp32 softmax (:2111-2157, :1658-1681), the engine's own draft for chunk selection, which re-forwards
the whole prompt every round (:1014-1060), chunk scoring (:1097-1152) and the chunk-local KV generate (:1683-1876).

Parity pinned: tests/golden/engine_reference.json holds what the UNMODIFIED reference engine produced on a B200 in
float64 with its sdpa attention backend (tests/golden/make_engine_golden.py drives a staged copy; the engine cannot be
imported without a GPU, its model runner initialises CUDA and NCCL at construction). tests/test_engine_golden.py holds
every function below to that file; the arithmetic shared with the eval class (model, unmask rule, score tail) is also
pinned by tests/golden/toy_reference.json.

The contract model caches un-rotated keys and takes the position of every key on each call, which expresses the
engine's post-RoPE pages exactly as long as all KV heads keep the same tokens (one position list per key).
"""

from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch

from . import hotpath as O


def _positions(values: Sequence[int]) -> torch.Tensor:
    return torch.tensor([list(values)], dtype=torch.long)


def _additive(mask_bool: torch.Tensor) -> torch.Tensor:
    out = torch.zeros(mask_bool.shape, dtype=torch.float32)
    out[~mask_bool] = float("-inf")
    return out.view(1, 1, *mask_bool.shape)


def selection_mask(mode: str, seq_len: int, prefix_len: int, chunk_len: int) -> Optional[torch.Tensor]:
    """fastdllm_engine.py:930-953 as an additive mask (None = full)."""
    mode = (mode or "full").lower()
    if mode in {"full", "none"}:
        return None
    if mode == "causal":
        return _additive(torch.tril(torch.ones(seq_len, seq_len, dtype=torch.bool)))
    if mode == "query_to_chunk":
        mask = torch.ones(seq_len, seq_len, dtype=torch.bool)
        mask[prefix_len:prefix_len + chunk_len, prefix_len + chunk_len:] = False
        return _additive(mask)
    raise ValueError(mode)


def sample_tokens(logits: torch.Tensor, *, temperature: float = 0.0, top_k: Optional[int] = None, top_p: Optional[float] = None):
    """The engine's sampler (fastdllm_engine.py:1658-1681): fp32, temperature, top-k BEFORE top-p (the eval class filters the
    other way round), softmax; (max probability, arg-max) at temperature 0, else a categorical draw and its probability."""
    work = logits.float()
    if temperature > 0:
        work = work / temperature
    floor = torch.finfo(work.dtype).min
    if top_k is not None:
        kth = torch.topk(work, min(int(top_k), work.shape[-1]), dim=-1).values[..., -1, None]
        work = work.masked_fill(work < kth, floor)
    if top_p is not None and top_p < 1:
        ordered, order = torch.sort(work, descending=True, dim=-1)
        gone = torch.cumsum(torch.softmax(ordered, dim=-1), dim=-1) > float(top_p)
        gone = torch.cat([torch.zeros_like(gone[..., :1]), gone[..., :-1]], dim=-1)
        work = work.masked_fill(torch.zeros_like(gone).scatter(-1, order, gone), floor)
    probs = torch.softmax(work, dim=-1)
    if temperature > 0:
        token = torch.distributions.Categorical(probs=probs).sample()
        return torch.gather(probs, -1, token.unsqueeze(-1)).squeeze(-1), token
    return probs.max(dim=-1)


def sampled_unmask(logits: torch.Tensor, block: torch.Tensor, last_logit: Optional[torch.Tensor], *, mask_id: int, threshold: float,
                   sampler: dict, shift: bool = True) -> torch.Tensor:
    """fastdllm_engine.py:2143-2157 — the masked slots are sampled; the most confident is accepted, and every other one whose
    confidence reaches the threshold. Returns the new block."""
    shifted = logits
    if shift:
        shifted = torch.cat([(logits[:1] if last_logit is None else last_logit.reshape(1, -1).to(logits.dtype)), logits[:-1]], dim=0)
    masked = block == mask_id
    confidence, sampled = sample_tokens(shifted[masked], **sampler)
    order = torch.argsort(confidence, descending=True, stable=True)
    slots = masked.nonzero(as_tuple=True)[0]
    out = block.clone()
    for rank, j in enumerate(order.tolist()):
        if rank == 0 or float(confidence[j]) >= threshold:
            out[slots[j]] = sampled[j]
    return out


def denoise_block(model, past, key_positions: Sequence[int], block_positions: Sequence[int], first_token: int,
                  last_context_logit: torch.Tensor, *, mask_id: int, threshold: float, shift: bool = True,
                  sampler: Optional[dict] = None) -> Tuple[List[int], int]:
    """:2133-2157 — every step forwards the whole block against `past` (concatenated, not stored). `shift=False`: the
    un-shifted read-out of the eval class's LLaDA backend (fastdllm_parallelcomp.py:1017-1024); the reference engine has
    no such model."""
    block = torch.full((len(block_positions),), mask_id, dtype=torch.long)
    block[0] = first_token
    steps = 0
    pos = _positions(list(key_positions) + list(block_positions))
    with torch.no_grad():
        while bool((block == mask_id).any()):
            steps += 1
            out = model(block.unsqueeze(0), attention_mask=None, position_ids=pos, past_key_values=past, use_cache=False)
            if sampler:
                block = sampled_unmask(out.logits[0], block, last_context_logit if shift else None, mask_id=mask_id, threshold=threshold,
                                       sampler=sampler, shift=shift)
                continue
            block, _, _ = O.unmask_step(out.logits[0], block, mask_token_id=mask_id, threshold=threshold,
                                        last_logit=last_context_logit if shift else None, shift=shift, softmax_dtype=torch.float32)
    return block.tolist(), steps


def prefill_and_decode(model, prompt_ids: Sequence[int], *, block_length: int, mask_id: int, threshold: float,
                       prompt_positions: Optional[Sequence[int]] = None, keep: Optional[Sequence[int]] = None, shift: bool = True,
                       sampler: Optional[dict] = None):
    """prefill_to_pd_record + decode_from_pd_record. `keep`: ONE ascending index list applied to every layer and KV
    head (post-hoc eviction with head-independent indices); keys keep the rotation of their original position and
    the block moves to max(kept positions) + 1 (:1953-1958).
    Returns dict(first_token, last_context_logit, token_ids, n_diff_steps, k_by_layer, v_by_layer)."""
    prompt_ids = list(prompt_ids)
    n = len(prompt_ids)
    prompt_positions = list(range(n)) if prompt_positions is None else list(prompt_positions)
    suffix_start = max(prompt_positions) + 1
    full_pos = prompt_positions + list(range(suffix_start, suffix_start + block_length))
    with torch.no_grad():
        out = model(torch.tensor([prompt_ids + [mask_id] * block_length]), attention_mask=None, position_ids=_positions(full_pos),
                    use_cache=True)
    last = out.logits[0, n - 1] if shift else out.logits[0, n]   # un-shifted: the first MASK slot's own row
    first = int(sample_tokens(last.reshape(1, -1), **sampler)[1][0]) if sampler and sampler.get("temperature", 0.0) > 0 else int(torch.argmax(last))
    idx = torch.arange(n) if keep is None else torch.tensor(list(keep), dtype=torch.long)
    past = [(k[:, idx], v[:, idx]) for k, v in out.past_key_values]
    key_positions = [prompt_positions[i] for i in idx.tolist()]
    block_start = max(key_positions) + 1
    ids, steps = denoise_block(model, past, key_positions, list(range(block_start, block_start + block_length)), first, last,
                               mask_id=mask_id, threshold=threshold, shift=shift, sampler=sampler)
    return dict(first_token=first, last_context_logit=last, token_ids=ids, n_diff_steps=steps, past=past, key_positions=key_positions)


def decode_blocks(model, prompt_ids: Sequence[int], *, max_new: int, block_length: int, mask_id: int, threshold: float,
                  shift: bool = True, softmax_dtype: Optional[torch.dtype] = torch.float32):
    """A record of several generation blocks: joint prefill of [prompt ‖ max_new MASK slots] (only the prompt's K/V and the
    last-context logit are kept), then the eval class's dual-cache block loop (fastdllm_parallelcomp.py:2678-2774, :2368-2441):
    every block forwards all remaining MASK slots against [prompt ‖ finished blocks] (suffix initialisation), the active
    block's rows replace their slots at every step, a commit forward stores the finished block. `shift=False`: the first
    token of a block is the arg-max of the first MASK slot's OWN row of the suffix forward and the steps read slot p from
    logits[p] (:1017-1024). The reference engine stops at one block (fastdllm_engine.py:1911-1915); parity of this function
    with the reference is pinned for shift=True through the eval goldens (tests/test_oracle_golden.py).
    Returns dict(token_ids, n_diff_steps)."""
    prompt_ids = list(prompt_ids)
    n0 = len(prompt_ids)
    total = n0 + max_new
    positions = _positions(range(total))
    generated: List[int] = []
    steps = 0
    with torch.no_grad():
        out = model(torch.tensor([prompt_ids + [mask_id] * max_new]), attention_mask=None, position_ids=positions, use_cache=True)
        cache = [(k[:, :n0], v[:, :n0]) for k, v in out.past_key_values]
        last_logit = out.logits[0, n0 - 1]
        for start in range(0, max_new, block_length):
            blen = min(block_length, max_new - start)
            lo = n0 + start
            done = [(k[:, :lo], v[:, :lo]) for k, v in cache]
            suffix = torch.full((1, total - lo), mask_id, dtype=torch.long)
            init = model(suffix, attention_mask=None, position_ids=positions, past_key_values=done, use_cache=True)
            cache = init.past_key_values
            block = torch.full((blen,), mask_id, dtype=torch.long)
            block[0] = int(torch.argmax(last_logit if shift else init.logits[0, 0]))
            replace = torch.zeros((1, total), dtype=torch.bool)
            replace[0, lo:lo + blen] = True
            while bool((block == mask_id).any()):
                steps += 1
                step = model(block.unsqueeze(0), attention_mask=None, position_ids=positions, past_key_values=cache, use_cache=False,
                             dual_cache=True, replace_position=replace)
                block, _, _ = O.unmask_step(step.logits[0], block, mask_token_id=mask_id, threshold=threshold,
                                            last_logit=last_logit if shift else None, shift=shift, softmax_dtype=softmax_dtype)
            generated.extend(block.tolist())
            commit = model(block.unsqueeze(0), attention_mask=None, position_ids=positions, past_key_values=cache, use_cache=True,
                           dual_cache=True, replace_position=replace)
            cache, last_logit = commit.past_key_values, commit.logits[0, -1]
    return dict(token_ids=generated, n_diff_steps=steps)


def engine_draft(model, prompt_ids: Sequence[int], *, draft_len: int, partial_rounds: int, mask_id: int) -> Tuple[List[int], List[bool]]:
    """generate_partial_draft_rounds_for_selection :1014-1060 — nothing cached, one full bidirectional forward per round."""
    prompt_ids = list(prompt_ids)
    p = len(prompt_ids)
    block = [mask_id] * draft_len
    confirmed = [False] * draft_len
    pos = _positions(range(p + draft_len))

    def shifted_block_logits():
        with torch.no_grad():
            logits = model(torch.tensor([prompt_ids + block]), attention_mask=None, position_ids=pos).logits[0]
        return logits[p - 1:p + draft_len - 1]       # slot j reads row p + j - 1

    block[0] = int(torch.argmax(shifted_block_logits()[0]))
    confirmed[0] = True
    for _ in range(max(0, partial_rounds)):
        masked = [i for i, t in enumerate(block) if t == mask_id]
        if not masked:
            break
        conf, x0 = O.sample_tokens_greedy(shifted_block_logits()[masked], torch.float32)
        best = int(torch.argmax(conf))
        block[masked[best]] = int(x0[best])
        confirmed[masked[best]] = True
    return block, confirmed


def score_chunk(model, prefix_ids, chunk_ids, query_ids, label_mask, attention_mask: str = "causal") -> float:
    """score_chunk_self_information_engine :1097-1152."""
    joint = list(prefix_ids) + list(chunk_ids) + list(query_ids)
    positions, labels = O.score_labels(len(prefix_ids), len(chunk_ids), query_ids, label_mask)
    mask = selection_mask(attention_mask, len(joint), len(prefix_ids), len(chunk_ids))
    with torch.no_grad():
        logits = model(torch.tensor([joint]), attention_mask=mask, position_ids=_positions(range(len(joint)))).logits[0]
    score, _ = O.self_information_scores(logits[[p - 1 for p in positions]].unsqueeze(0), torch.tensor(labels))
    return float(score[0])


def per_head_keep(model, prefix_ids, chunk_ids, window_ids, *, capacity: int, num_kv_heads: int, layers: Sequence[int],
                  attention_mask: str = "causal", pool_kernel: int = 7, pooling: str = "maxpool", reduce_mode: str = "sum",
                  direction: str = "query_to_chunk", keep_high: bool = True) -> Tuple[List[torch.Tensor], List[torch.Tensor]]:
    """compute_prompt_keep_indices_per_layer_per_head :1365-1470 for one chunk: the hidden states run under FULL attention
    and only the score softmax applies `attention_mask`. `direction` (:1296-1323): the mass the query window's rows put on each
    chunk token, the mass each chunk row puts on the window's keys (zero unless the mask is "full": chunk rows do not see the
    window under the other two), or their sum. Returns (keep [Hkv, capacity] per selected layer, pooled scores)."""
    joint = list(prefix_ids) + list(chunk_ids) + list(window_ids)
    length, p, c, w = len(joint), len(prefix_ids), len(chunk_ids), len(window_ids)
    captured = {}
    hooks = []
    for li in layers:
        attn = model.model.layers[li].self_attn
        hooks.append(attn.register_forward_pre_hook(
            lambda mod, args, kwargs, li=li: captured.__setitem__(li, (args[0] if args else kwargs["hidden_states"]).detach()), with_kwargs=True))
    try:
        with torch.no_grad():
            model(torch.tensor([joint]), attention_mask=None, position_ids=_positions(range(length)))
    finally:
        for h in hooks:
            h.remove()
    keeps, pooled_all = [], []
    cos, sin = model.model.rotary_emb(torch.zeros(1, length, 1), _positions(range(length)))
    for li in layers:
        attn = model.model.layers[li].self_attn
        hidden = captured[li]
        q = attn.q_proj(hidden).view(length, attn.num_heads, attn.head_dim)
        k = attn.k_proj(hidden).view(length, attn.num_key_value_heads, attn.head_dim)

        def rot(x):
            half = x.shape[-1] // 2
            return x * cos[0].unsqueeze(1) + torch.cat((-x[..., half:], x[..., :half]), dim=-1) * sin[0].unsqueeze(1)

        qr, kr, scale = rot(q), rot(k), attn.head_dim ** -0.5
        parts = []
        if direction in ("query_to_chunk", "bidirectional"):
            parts.append(O.query_to_chunk_scores(qr, kr, prefix_len=p, chunk_len=c, query_len=w, scale=scale, reduce_mode=reduce_mode,
                                                 causal=(attention_mask == "causal")))
        if direction in ("chunk_to_query", "bidirectional"):
            if attention_mask in ("full", "none"):
                group = qr.shape[1] // kr.shape[1]
                logits = torch.einsum("chd,lhd->hcl", qr.float()[p:p + c], kr.float().repeat_interleave(group, dim=1)) * scale
                mass = torch.softmax(logits, dim=-1)[:, :, p + c:p + c + w]
                parts.append(mass.mean(dim=2) if reduce_mode == "mean" else mass.sum(dim=2))
            else:
                parts.append(torch.zeros(qr.shape[1], c))
        scores = parts[0] if len(parts) == 1 else parts[0] + parts[1]
        pooled = O.per_head_token_scores(scores, num_kv_heads, pooling, pool_kernel)
        keeps.append(torch.stack([O.select_positions_from_token_scores(pooled[h], capacity=capacity, chunk_len=c, keep_high=keep_high)
                                  for h in range(num_kv_heads)]))
        pooled_all.append(pooled)
    return keeps, pooled_all


def chunk_local_generate(model, *, prefix_ids, prefix_positions, chunk_ids_list, chunk_positions_list, keep_list, query_ids,
                         query_positions, local_query_ids, block_length: int, mask_id: int, threshold: float,
                         local_attention_mask: str = "causal"):
    """generate_token_ids_from_chunk_local_kv :1683-1876 with ONE keep list per chunk (the same for all layers / heads)."""
    prefix_ids, prefix_positions = list(prefix_ids), list(prefix_positions)
    p = len(prefix_ids)
    with torch.no_grad():
        parts = []
        key_positions: List[int] = []
        if prefix_ids:
            out = model(torch.tensor([prefix_ids]), attention_mask=None, position_ids=_positions(prefix_positions), use_cache=True)
            parts.append(out.past_key_values)
            key_positions += prefix_positions
        for chunk_ids, chunk_pos, keep in zip(chunk_ids_list, chunk_positions_list, keep_list):
            chunk_ids, chunk_pos = list(chunk_ids), list(chunk_pos)
            lq_start = max(chunk_pos) + 1
            local = prefix_ids + chunk_ids + list(local_query_ids)
            local_pos = prefix_positions + chunk_pos + list(range(lq_start, lq_start + len(local_query_ids)))
            mask = selection_mask(local_attention_mask, len(local), p, len(chunk_ids))
            out = model(torch.tensor([local]), attention_mask=mask, position_ids=_positions(local_pos), use_cache=True)
            idx = torch.tensor([p + i for i in keep], dtype=torch.long)
            parts.append([(k[:, idx], v[:, idx]) for k, v in out.past_key_values])
            key_positions += [chunk_pos[i] for i in keep]
        layers = len(parts[0])
        past = [(torch.cat([part[l][0] for part in parts], dim=1), torch.cat([part[l][1] for part in parts], dim=1)) for l in range(layers)]
        suffix_start = max(query_positions) + 1
        block_positions = list(range(suffix_start, suffix_start + block_length))
        suffix = list(query_ids) + [mask_id] * block_length
        out = model(torch.tensor([suffix]), attention_mask=None, position_ids=_positions(key_positions + list(query_positions) + block_positions),
                    past_key_values=past, use_cache=True)
        q = len(query_ids)
        last = out.logits[0, q - 1]
        first = int(torch.argmax(last))
        base = len(key_positions)
        past_q = [(k[:, :base + q], v[:, :base + q]) for k, v in out.past_key_values]
    ids, steps = denoise_block(model, past_q, key_positions + list(query_positions), block_positions, first, last, mask_id=mask_id,
                               threshold=threshold)
    return dict(first_token=first, token_ids=ids, n_diff_steps=steps)


# --------------------------------------------------------------------------------------------------------------------
# Sparse prefill over an eviction mask and the decode-time delta correction (layers/attention/attention_v4.py:86-289).
# These change what an attention layer computes, so the layers are walked explicitly here instead of through the contract
# model's forward: per layer, rotated q/k and v per head, one `attention(layer, q, k, v)` call, the residual and the MLP.
# --------------------------------------------------------------------------------------------------------------------
def _walk_layers(model, ids: Sequence[int], positions: Sequence[int], attention):
    """`attention(layer, q [H, n, D], k [Hkv, n, D], v [Hkv, n, D]) -> [H, n, D]` with q and k already rotated to `positions`.
    Returns the logits [n, vocab]."""
    from .contract_model.model.modeling_dream import rotate_half

    base = model.model
    h = base.embed_tokens(torch.tensor([list(ids)], dtype=torch.long))
    cos, sin = base.rotary_emb(h, _positions(positions))
    n = h.shape[1]
    for li, layer in enumerate(base.layers):
        a = layer.self_attn
        x = layer.input_layernorm(h)
        q = a.q_proj(x).view(n, a.num_heads, a.head_dim).transpose(0, 1)
        k = a.k_proj(x).view(n, a.num_key_value_heads, a.head_dim).transpose(0, 1)
        v = a.v_proj(x).view(n, a.num_key_value_heads, a.head_dim).transpose(0, 1)
        q = q * cos + rotate_half(q) * sin
        k = k * cos + rotate_half(k) * sin
        o = attention(li, q, k, v)
        h = h + a.o_proj(o.transpose(0, 1).reshape(1, n, a.num_heads * a.head_dim))
        h = h + layer.mlp(layer.post_attention_layernorm(h))
    return model.lm_head(base.norm(h))[0]


def _attend(q, k, v, allowed: Optional[torch.Tensor] = None):
    """softmax(q k^T / sqrt(d)) v per query head, KV heads repeated; `allowed` [rows, keys] bool or None."""
    group = q.shape[0] // k.shape[0]
    k, v = k.repeat_interleave(group, dim=0), v.repeat_interleave(group, dim=0)
    scores = torch.matmul(q, k.transpose(1, 2)) / (q.shape[-1] ** 0.5)
    if allowed is not None:
        scores = scores.masked_fill(~allowed, float("-inf"))
    return torch.matmul(torch.softmax(scores, dim=-1), v)


def _spread_delta(out, dense_at_anchors, anchors: Sequence[int], *, left: int, right: int, direction: str, scale: float):
    """attention_v4.py:145-158, :274-288 — out + the delta of every anchor row added to the rows of its window."""
    n = out.shape[1]
    delta = (dense_at_anchors - out[:, list(anchors)]) * scale
    fixed = out.clone()
    for idx, a in enumerate(anchors):
        lo = a if direction == "right" else max(0, a - left)
        hi = a if direction == "left" else min(n - 1, a + right)
        fixed[:, lo:hi + 1] += delta[:, idx:idx + 1]
    return fixed


def sparse_prefill_and_decode(model, prompt_ids: Sequence[int], keep_nested, *, block_length: int, mask_id: int, threshold: float,
                              delta: bool = False, stride: int = 8, left: int = 7, right: int = 0, direction: str = "left",
                              scale: float = 1.0):
    """prefill_sparse_mode="eviction_mask" (fastdllm_engine.py:2010-2040, attention_v4.py:164-289): in layer l every row of
    the joint prefill attends only the union over KV heads of `keep_nested[l]` plus the MASK slots; with `delta` the dense
    attention is evaluated at every stride-th row (from stride-1, or from 0 for direction "right") and the difference is
    spread over that anchor's window. The prompt KV is NOT compacted: the block decodes against all of it, densely.
    Returns dict(first_token, last_context_logit, token_ids, n_diff_steps)."""
    prompt_ids = list(prompt_ids)
    n0, n = len(prompt_ids), len(prompt_ids) + block_length
    offset = 0 if direction == "right" else stride - 1
    anchors = list(range(offset, n, stride))
    kept_kv = []

    def attention(layer, q, k, v):
        kept_kv.append((k[:, :n0], v[:, :n0]))
        key_ok = torch.zeros(n, dtype=torch.bool)
        key_ok[torch.tensor(sorted({int(i) for head in keep_nested[layer] for i in head if 0 <= int(i) < n}), dtype=torch.long)] = True
        key_ok[n0:] = True
        out = _attend(q, k, v, key_ok.unsqueeze(0).expand(n, n))
        if delta and anchors:
            out = _spread_delta(out, _attend(q[:, anchors], k, v), anchors, left=left, right=right, direction=direction, scale=scale)
        return out

    with torch.no_grad():
        logits = _walk_layers(model, prompt_ids + [mask_id] * block_length, range(n), attention)
        last = logits[n0 - 1]
        first = int(torch.argmax(last))
        block = torch.full((block_length,), mask_id, dtype=torch.long)
        block[0] = first
        steps = 0
        while bool((block == mask_id).any()):
            steps += 1
            step = _walk_layers(model, block.tolist(), range(n0, n),
                                lambda layer, q, k, v: _attend(q, torch.cat([kept_kv[layer][0], k], dim=1), torch.cat([kept_kv[layer][1], v], dim=1)))
            block, _, _ = O.unmask_step(step, block, mask_token_id=mask_id, threshold=threshold, last_logit=last, shift=True,
                                        softmax_dtype=torch.float32)
    return dict(first_token=first, last_context_logit=last, token_ids=block.tolist(), n_diff_steps=steps)


def posthoc_eviction_with_decode_delta(model, prompt_ids: Sequence[int], keep_nested, active_positions: Sequence[int], *, block_length: int,
                                       mask_id: int, threshold: float, stride: int = 4, left: int = 3, scale: float = 1.0):
    """Per-layer, per-KV-head post-hoc eviction with decode_delta_mode="s4_left3" (fastdllm_engine.py:2061-2082,
    attention_v4.py:86-162): after a dense joint prefill, head h of layer l keeps the rotated K/V rows `keep_nested[l][h]`;
    the block is denoised at positions max(active_positions)+1.. against them, and in every layer of every step the rows
    stride-1, 2*stride-1, ... are also evaluated against the FULL prompt KV (kept aside before the eviction); that
    difference, times `scale`, is added to the anchor row and the `left` rows before it.
    Returns dict(first_token, last_context_logit, token_ids, n_diff_steps)."""
    prompt_ids = list(prompt_ids)
    n0, n = len(prompt_ids), len(prompt_ids) + block_length
    full_kv = []

    def dense(layer, q, k, v):
        full_kv.append((k[:, :n0], v[:, :n0]))
        return _attend(q, k, v)

    anchors = list(range(stride - 1, block_length, stride))
    start = max(int(p) for p in active_positions) + 1

    def corrected(layer, q, k, v):
        fk, fv = full_kv[layer]
        idx = [torch.tensor([int(i) for i in head], dtype=torch.long) for head in keep_nested[layer]]
        kk = torch.stack([fk[h, idx[h]] for h in range(fk.shape[0])])
        kv = torch.stack([fv[h, idx[h]] for h in range(fv.shape[0])])
        out = _attend(q, torch.cat([kk, k], dim=1), torch.cat([kv, v], dim=1))
        if not anchors:
            return out
        exact = _attend(q[:, anchors], torch.cat([fk, k], dim=1), torch.cat([fv, v], dim=1))
        return _spread_delta(out, exact, anchors, left=left, right=0, direction="left", scale=scale)

    with torch.no_grad():
        logits = _walk_layers(model, prompt_ids + [mask_id] * block_length, range(n), dense)
        last = logits[n0 - 1]
        first = int(torch.argmax(last))
        block = torch.full((block_length,), mask_id, dtype=torch.long)
        block[0] = first
        steps = 0
        while bool((block == mask_id).any()):
            steps += 1
            step = _walk_layers(model, block.tolist(), range(start, start + block_length), corrected)
            block, _, _ = O.unmask_step(step, block, mask_token_id=mask_id, threshold=threshold, last_logit=last, shift=True,
                                        softmax_dtype=torch.float32)
    return dict(first_token=first, last_context_logit=last, token_ids=block.tolist(), n_diff_steps=steps)
