"""CPU restatement of the Prefilling-dLLM long-context hot path. TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm may import this file; the
product package never does. Every function restates one piece of the reference's algorithm in plain
torch-on-CPU (fp32 unless the reference computes in another type) and cites the reference file:line it
follows. Paths are relative to the reference project root; E: = prefilling_dllm_eval/,
G: = prefilling_dllm_engine/prefilling_dllm/.

Pinning: the host-logic functions (chunking, BOS truncation, draft, scoring tail, ranking, eviction keep
lists, positions, accept rule) are pinned by tests/golden/toy_reference.json, produced by running the
UNMODIFIED reference class E:fastdllm_parallelcomp.py on CPU (tests/golden/make_golden.py). The model the
reference drives (Fast-dLLM v1 `model/modeling_dream.py`, NVlabs/Fast-dLLM, un-vendored and unpinned by the
reference) is absent, so its arithmetic is restated in oracle/contract_model from the Dream files the
reference does vendor (E:model_cache/dream/model_dream.py) and cross-checked against that vendored model:
parity of the model arithmetic itself is therefore "unpinned" against Fast-dLLM v1 proper.
"""

from __future__ import annotations

import math
from typing import List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

# --------------------------------------------------------------------------------------------------
# rows 1-2, 9: chunking, chunk BOS, positions
# --------------------------------------------------------------------------------------------------


def split_token_chunks(token_ids: Sequence[int], chunk_size: int, split_from_tail: bool = False) -> List[List[int]]:
    """E:fastdllm_parallelcomp.py:158-180."""
    ids = list(token_ids)
    if not ids:
        return []
    if chunk_size <= 0 or len(ids) <= chunk_size:
        return [ids]
    chunks: List[List[int]] = []
    cursor = 0
    if split_from_tail:
        rem = len(ids) % chunk_size
        if rem > 0:
            chunks.append(ids[:rem])
            cursor = rem
    while cursor < len(ids):
        chunks.append(ids[cursor:cursor + chunk_size])
        cursor += chunk_size
    return chunks


def maybe_prepend_bos_to_chunk(chunk_ids: Sequence[int], bos_ids: Sequence[int], chunk_size: int, chunk_bos: bool = True) -> List[int]:
    """E:fastdllm_parallelcomp.py:897-908 — [BOS]+chunk cut back to chunk_size (a full chunk loses its last token)."""
    ids = list(chunk_ids)
    bos = list(bos_ids)
    if not chunk_bos or not bos or ids[:len(bos)] == bos:
        return ids
    out = bos + ids
    if chunk_size > 0 and len(out) > chunk_size:
        out = out[:chunk_size]
    return out


def chunk_rope_start(mode: str, prefix_len: int, chunk_order: int, chunk_index: int, chunk_size: int) -> int:
    """E:fastdllm_parallelcomp.py:922-930."""
    if mode == "reuse":
        return prefix_len
    if mode == "continuous":
        return prefix_len + chunk_order * max(1, chunk_size)
    if mode == "absolute":
        return prefix_len + chunk_index * max(1, chunk_size)
    raise ValueError(f"Unsupported chunk_position_mode: {mode}")


def final_query_rope_start(mode: str, prefix_len: int, cache_positions: Sequence[int], selected_count: int, chunk_size: int) -> int:
    """E:fastdllm_parallelcomp.py:940-948."""
    if mode == "after_reused_window":
        return prefix_len + max(1, chunk_size)
    if mode == "after_selected_chunks":
        return prefix_len + selected_count * max(1, chunk_size)
    if mode == "after_cache":
        return (max(cache_positions) + 1) if cache_positions else prefix_len
    raise ValueError(f"Unsupported query_position_mode: {mode}")


# --------------------------------------------------------------------------------------------------
# row 17 / kernel (5): KV page writes and the gather
# --------------------------------------------------------------------------------------------------


def store_kvcache_unified(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                          slot_mapping: torch.Tensor) -> None:
    """G:layers/attention/ops/kv_cache_kernels.py:34-55 — row `slot` of the flattened pool := token row; slot<0 skips."""
    flat_k = k_cache.view(-1, k_cache.shape[-2] * k_cache.shape[-1])
    flat_v = v_cache.view(-1, v_cache.shape[-2] * v_cache.shape[-1])
    for tok, slot in enumerate(slot_mapping.tolist()):
        if slot < 0:
            continue
        flat_k[slot] = key[tok].reshape(-1)
        flat_v[slot] = value[tok].reshape(-1)


def store_kvcache_distinct(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                           slot_mapping: torch.Tensor) -> None:
    """G:layers/attention/ops/kv_cache_kernels.py:58-106 — K [pages,H,D/x,page,x], V [pages,H,D,page]."""
    _, h, dx, page_size, x = k_cache.shape
    for tok, slot in enumerate(slot_mapping.tolist()):
        if slot < 0:
            continue
        page, off = divmod(slot, page_size)
        k_cache[page, :, :, off, :] = key[tok].view(h, dx, x)
        v_cache[page, :, :, off] = value[tok]


def load_kvcache(k_cache: torch.Tensor, v_cache: torch.Tensor, block_tables: torch.Tensor, context_lens: Sequence[int],
                 cu_seqlens_q: Sequence[int], k_new: torch.Tensor, v_new: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """G:layers/attention/ops/kv_cache_kernels.py:175-327 (checked upstream by CHECK_LOADING :364-394)."""
    page_size = k_cache.shape[1]
    ks, vs = [], []
    for s, ctx in enumerate(context_lens):
        remaining = int(ctx)
        for page in block_tables[s].tolist():
            if remaining <= 0:
                break
            if page < 0:
                continue
            take = min(page_size, remaining)
            ks.append(k_cache[page, :take])
            vs.append(v_cache[page, :take])
            remaining -= take
        ks.append(k_new[cu_seqlens_q[s]:cu_seqlens_q[s + 1]])
        vs.append(v_new[cu_seqlens_q[s]:cu_seqlens_q[s + 1]])
    return torch.cat(ks, dim=0), torch.cat(vs, dim=0)


def distinct_to_unified(k_cache: torch.Tensor, v_cache: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """G:layers/attention/ops/triton_decode_attn_dlm.py:32-35 (the rearranges inside CHECK_ATTENTION)."""
    pages, h, dx, page_size, x = k_cache.shape
    k_u = k_cache.permute(0, 3, 1, 2, 4).reshape(pages, page_size, h, dx * x).contiguous()
    v_u = v_cache.permute(0, 3, 1, 2).contiguous()
    return k_u, v_u


# --------------------------------------------------------------------------------------------------
# row 17 / kernels (3)+(1): attention of new rows over [selected pages ‖ new rows]
# --------------------------------------------------------------------------------------------------


def new_key_visibility(q_len: int, *, mask: Optional[torch.Tensor], bidirectional: bool, diffusion_blk: int, causal: bool) -> torch.Tensor:
    """Visibility [q_len, q_len] of new keys for new rows.

    d2f rule, G:layers/attention/ops/prefix_prefill.py:169-204: the key loop of row block start_m covers
    n < (start_m+1)*BLOCK_M with BLOCK_M = 2*diffusion_blk unless BIDIRECTIONAL (then all n < q_len), and the
    dense mask is read with sequence-LOCAL indices. causal: E:fastdllm_parallelcomp.py:950-961.
    """
    m = torch.arange(q_len).view(-1, 1)
    n = torch.arange(q_len).view(1, -1)
    if causal:
        return n <= m
    vis = torch.ones(q_len, q_len, dtype=torch.bool)
    if not bidirectional:
        block_m = 2 * diffusion_blk
        vis &= n < (m // block_m + 1) * block_m
    if mask is not None:
        vis &= mask[:q_len, :q_len].bool()
    return vis


def paged_attention(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, *, cu_seqlens_q: Sequence[int],
                    k_cache: Optional[torch.Tensor] = None, v_cache: Optional[torch.Tensor] = None,
                    block_table: Optional[torch.Tensor] = None, seq_lens: Optional[Sequence[int]] = None,
                    sm_scale: Optional[float] = None, mask: Optional[torch.Tensor] = None, bidirectional: bool = True,
                    diffusion_blk: int = 32, causal: bool = False) -> torch.Tensor:
    """fp32 softmax(QK^T*scale + mask)V with GQA over the gathered keys.

    The math of CHECK_ATTENTION (G:layers/attention/ops/triton_decode_attn_dlm.py:18-45): gather the selected
    pages in block-table order, append the new K/V, SDPA (MATH) with a dense bool mask and enable_gqa.
    Inputs of any float dtype are promoted to fp32; the result is fp32 [T, Hq, D].
    A row that sees no key yields zeros (the d2f kernel's l_i starts at 1, prefix_prefill.py:94, 224).
    """
    t, hq, d = q.shape
    hkv = k_new.shape[1]
    group = hq // hkv
    scale = sm_scale if sm_scale is not None else 1.0 / math.sqrt(d)
    out = torch.zeros(t, hq, d, dtype=torch.float32)
    for s in range(len(cu_seqlens_q) - 1):
        b, e = int(cu_seqlens_q[s]), int(cu_seqlens_q[s + 1])
        q_len = e - b
        if q_len <= 0:
            continue
        ctx = 0
        ks, vs = [], []
        if k_cache is not None and seq_lens is not None:
            ctx = max(0, int(seq_lens[s]) - q_len)
            page_size = k_cache.shape[1]
            remaining = ctx
            for page in block_table[s].tolist():
                if remaining <= 0:
                    break
                take = min(page_size, remaining)
                ks.append(k_cache[page, :take].float())
                vs.append(v_cache[page, :take].float())
                remaining -= take
        ks.append(k_new[b:e].float())
        vs.append(v_new[b:e].float())
        kk = torch.cat(ks, dim=0)  # [ctx + q_len, Hkv, D]
        vv = torch.cat(vs, dim=0)
        vis_new = new_key_visibility(q_len, mask=mask, bidirectional=bidirectional, diffusion_blk=diffusion_blk, causal=causal)
        vis = torch.cat([torch.ones(q_len, ctx, dtype=torch.bool), vis_new], dim=1)  # context is always visible
        qs = q[b:e].float().permute(1, 0, 2)                                   # [Hq, q_len, D]
        kk = kk.permute(1, 0, 2).repeat_interleave(group, dim=0)               # [Hq, S, D]
        vv = vv.permute(1, 0, 2).repeat_interleave(group, dim=0)
        logits = torch.matmul(qs, kk.transpose(1, 2)) * scale
        logits = logits.masked_fill(~vis.unsqueeze(0), float("-inf"))
        probs = torch.softmax(logits, dim=-1)
        probs = torch.nan_to_num(probs, nan=0.0)  # fully masked row → zeros
        out[b:e] = torch.matmul(probs, vv).permute(1, 0, 2)
    return out


# --------------------------------------------------------------------------------------------------
# rows 12, 18 / kernel (4): shifted logits, greedy sampling, accept rule
# --------------------------------------------------------------------------------------------------


def shift_logits(logits: torch.Tensor, last_logit: Optional[torch.Tensor] = None) -> torch.Tensor:
    """[rows, V] variant of E:fastdllm_parallelcomp.py:1007-1015 and G:fastdllm_engine.py:1648-1656."""
    shifted = torch.empty_like(logits)
    shifted[0] = logits[0] if last_logit is None else last_logit.reshape(-1)
    if logits.shape[0] > 1:
        shifted[1:] = logits[:-1]
    return shifted


def sample_tokens_greedy(logits: torch.Tensor, softmax_dtype: Optional[torch.dtype]) -> Tuple[torch.Tensor, torch.Tensor]:
    """Greedy branch of sample_tokens: E:fastdllm_parallelcomp.py:216, 223-225 (softmax in the logits dtype)
    or of _sample_tokens: G:fastdllm_engine.py:1659, 1675, 1680 (logits.float() first)."""
    work = logits if softmax_dtype is None else logits.to(softmax_dtype)
    probs = torch.softmax(work, dim=-1)
    confidence, x0 = probs.max(dim=-1)
    return confidence, x0


def unmask_step(logits: torch.Tensor, block_ids: torch.Tensor, *, mask_token_id: int, threshold: float,
                last_logit: Optional[torch.Tensor] = None, shift: bool = True,
                softmax_dtype: Optional[torch.dtype] = None) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """One iteration of the confidence-threshold loop.

    E:fastdllm_parallelcomp.py:2414-2440 / G:fastdllm_engine.py:2135-2157: every masked slot gets
    (confidence, arg-max); the slots are ranked by confidence, rank 0 is always transferred and rank i >= 1 iff
    confidence_i >= threshold (compared in the confidence dtype). Returns (new block_ids, confidence over all
    slots with -inf on unmasked ones, arg-max per slot). torch.topk's order among equal confidences is
    unspecified; this restatement gives rank 0 to the lowest slot.
    """
    ids = block_ids.clone()
    mask_index = ids == mask_token_id
    work = shift_logits(logits, last_logit) if shift else logits
    conf_dtype = work.dtype if softmax_dtype is None else softmax_dtype
    full_conf = torch.full((ids.numel(),), float("-inf"), dtype=conf_dtype)
    x0_full = ids.clone()
    if not bool(mask_index.any()):
        return ids, full_conf, x0_full
    confidence, x0 = sample_tokens_greedy(work[mask_index], softmax_dtype)
    full_conf[mask_index] = confidence.to(conf_dtype)
    x0_full[mask_index] = x0
    best = int(torch.argmax(full_conf.float()).item())  # first maximal element
    transfer = torch.zeros_like(mask_index)
    transfer[best] = True
    transfer |= mask_index & (full_conf >= threshold)
    ids[transfer] = x0_full[transfer]
    return ids, full_conf, x0_full


def fixed_step_transfer_counts(masked: int, steps_per_block: int) -> List[int]:
    """How many slots each step of the fixed-step diffusion sampler transfers (E:fastdllm_parallelcomp.py:2455, 2492-2496):
    t = linspace(1, 1e-3, steps + 1) in fp32; step i moves int(masks_left * (1 - t[i+1] / t[i])) slots, the last step all
    that is left; a step that would move none runs no transfer."""
    timesteps = torch.linspace(1, 1e-3, steps_per_block + 1)
    out, left = [], int(masked)
    for step in range(steps_per_block):
        if left <= 0:
            break
        count = int(left * (1 - timesteps[step + 1] / timesteps[step])) if step < steps_per_block - 1 else left
        out.append(max(0, count))
        left -= max(0, count)
    return out


def transfer_most_confident(logits: torch.Tensor, block_ids: torch.Tensor, *, mask_token_id: int, count: int,
                            last_logit: Optional[torch.Tensor] = None, shift: bool = True) -> torch.Tensor:
    """Fill the `count` most confident masked slots with their arg-max (E:fastdllm_parallelcomp.py:2497-2504 with alg_temp 0,
    :2548-2552 of the partial draft): confidence = max softmax probability in the logits dtype."""
    ids = block_ids.clone()
    _, full_conf, x0_full = unmask_step(logits, ids, mask_token_id=mask_token_id, threshold=2.0, last_logit=last_logit, shift=shift)
    count = min(int(count), int((ids == mask_token_id).sum()))
    if count > 0:
        idx = torch.topk(full_conf.float(), count).indices
        ids[idx] = x0_full[idx]
    return ids


# --------------------------------------------------------------------------------------------------
# rows 5-6 / kernels (2a)(2b): self-information score tail and chunk ranking
# --------------------------------------------------------------------------------------------------


def self_information_scores(label_rows: torch.Tensor, labels: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """E:fastdllm_parallelcomp.py:1415-1422 on rows already gathered at label_pos-1.

    label_rows [n_chunks, n_labels, V] any float dtype; labels [n_labels]. Returns (scores [n_chunks] fp32 with
    non-finite → -inf, nll [n_chunks, n_labels])."""
    log_probs = F.log_softmax(label_rows.float(), dim=-1)
    index = labels.view(1, -1, 1).expand(log_probs.shape[0], -1, 1)
    nll = -log_probs.gather(dim=-1, index=index).squeeze(-1)
    scores = -nll.mean(dim=-1)
    scores = torch.where(torch.isfinite(scores), scores, torch.full_like(scores, float("-inf")))
    return scores, nll


def rank_chunks(scores: Sequence[float], topk_chunks: int, keep_first_chunk: bool = False) -> List[int]:
    """E:fastdllm_parallelcomp.py:1949-1953 — Python's stable sort, descending, then ascending indices."""
    n = len(scores)
    clean = [s if math.isfinite(s) else float("-inf") for s in scores]
    forced = [0] if keep_first_chunk and n > 0 else []
    remaining = [i for i in range(n) if i not in forced]
    ranked = sorted(remaining, key=lambda i: clean[i], reverse=True)
    topk = len(ranked) if topk_chunks <= 0 else min(topk_chunks, len(ranked))
    return sorted(set(forced + ranked[:topk]))


def score_labels(prefix_len: int, chunk_len: int, query_ids: Sequence[int], score_token_mask: Optional[Sequence[bool]]) -> Tuple[List[int], List[int]]:
    """Label positions and ids for one scoring row, E:fastdllm_parallelcomp.py:1365-1382 (mask / full-query cases)."""
    query_ids = list(query_ids)
    if score_token_mask is not None:
        local = [i for i, keep in enumerate(score_token_mask) if keep]
        return [prefix_len + chunk_len + i for i in local], [query_ids[i] for i in local]
    start = prefix_len + chunk_len
    return list(range(start, start + len(query_ids))), query_ids


# --------------------------------------------------------------------------------------------------
# rows 7-8 / kernel (2c): query→chunk attention mass, pooling, keep positions
# --------------------------------------------------------------------------------------------------


def query_to_chunk_scores(q: torch.Tensor, k: torch.Tensor, *, prefix_len: int, chunk_len: int, query_len: int,
                          scale: float, reduce_mode: str = "sum", causal: bool = True) -> torch.Tensor:
    """fp32 [Hq, chunk_len]: sum over the query-window rows of softmax(q·k*scale)[chunk columns].

    G:layers/attention/ops/triton_eviction_scorer.py:6-111 (two Triton passes) — the same quantity as
    _chunk_attention_head_scores over eager attention probabilities, E:fastdllm_parallelcomp.py:1639-1667, and as
    the torch branch G:fastdllm_engine.py:1279-1323. q [L, Hq, D], k [L, Hkv, D], already rotated."""
    length, hq, _ = q.shape
    hkv = k.shape[1]
    group = hq // hkv
    rows = torch.arange(prefix_len + chunk_len, prefix_len + chunk_len + query_len)
    qf = q.float()[rows]                                        # [w, Hq, D]
    kf = k.float().repeat_interleave(group, dim=1)              # [L, Hq, D]
    logits = torch.einsum("whd,lhd->hwl", qf, kf) * scale
    if causal:
        keys = torch.arange(length).view(1, 1, -1)
        logits = logits.masked_fill(keys > rows.view(1, -1, 1), float("-inf"))
    probs = torch.softmax(logits, dim=-1)[:, :, prefix_len:prefix_len + chunk_len]
    return probs.mean(dim=1) if reduce_mode == "mean" else probs.sum(dim=1)


def pool_scores(head_scores: torch.Tensor, pooling: str, pool_kernel: int) -> torch.Tensor:
    """E:fastdllm_parallelcomp.py:1607-1617 on [H, C]."""
    pooling = (pooling or "none").lower()
    chunk_len = head_scores.shape[-1]
    if pooling == "none" or chunk_len == 0:
        return head_scores
    kernel = max(1, min(int(pool_kernel), chunk_len))
    padding = kernel // 2
    x = head_scores.unsqueeze(1)
    if pooling == "avgpool":
        x = F.avg_pool1d(x, kernel_size=kernel, padding=padding, stride=1)
    elif pooling == "maxpool":
        x = F.max_pool1d(x, kernel_size=kernel, padding=padding, stride=1)
    else:
        raise ValueError(f"Unsupported token_score_pooling: {pooling}")
    return x.squeeze(1)[..., :chunk_len]


def global_token_scores(head_scores_by_layer: Sequence[torch.Tensor], pooling: str = "maxpool", pool_kernel: int = 7,
                        head_reduce: str = "sum", layer_reduce: str = "mean") -> torch.Tensor:
    """E:fastdllm_parallelcomp.py:1593-1637: pool → reduce heads → reduce layers → [C]."""
    layers = []
    for hs in head_scores_by_layer:
        pooled = pool_scores(hs, pooling, pool_kernel)
        layers.append({"mean": pooled.mean(dim=0), "sum": pooled.sum(dim=0), "max": pooled.max(dim=0).values}[head_reduce])
    stacked = torch.stack(layers, dim=0)
    return {"mean": stacked.mean(dim=0), "sum": stacked.sum(dim=0), "max": stacked.max(dim=0).values}[layer_reduce]


def per_head_token_scores(head_scores: torch.Tensor, num_kv_heads: int, pooling: str = "maxpool", pool_kernel: int = 7) -> torch.Tensor:
    """E:fastdllm_parallelcomp.py:1742-1760 / G:fastdllm_engine.py:1396-1432: pool, then mean of each KV group → [Hkv, C]."""
    pooled = pool_scores(head_scores, pooling, pool_kernel)
    return torch.stack([g.mean(dim=0) for g in torch.tensor_split(pooled, num_kv_heads, dim=0)], dim=0)


def select_positions_from_token_scores(token_scores: torch.Tensor, *, capacity: int, chunk_len: int, keep_high: bool = True,
                                       force_keep_first: bool = True) -> torch.Tensor:
    """E:fastdllm_parallelcomp.py:1997-2023 / G:fastdllm_engine.py:904-927.

    torch.topk's choice among equal scores at the cut is unspecified; this restatement keeps the lower position
    (a stable sort), which is also what the CUDA kernel does."""
    keep_count = min(max(1, int(capacity)), chunk_len)
    if token_scores.numel() != chunk_len:
        head = keep_count // 2
        tail = keep_count - head
        keep = sorted(set(list(range(head)) + list(range(chunk_len - tail, chunk_len))))
        return torch.tensor(keep[:keep_count], dtype=torch.long)

    def stable_topk(values: torch.Tensor, k: int) -> torch.Tensor:
        order = torch.sort(values, descending=keep_high, stable=True).indices
        return order[:k]

    if force_keep_first and chunk_len > 0:
        if keep_count == 1:
            return torch.zeros(1, dtype=torch.long)
        candidates = torch.arange(1, chunk_len)
        if candidates.numel() <= keep_count - 1:
            selected = candidates
        else:
            selected = candidates[stable_topk(token_scores[1:], keep_count - 1)]
        return torch.sort(torch.cat([torch.zeros(1, dtype=torch.long), selected])).values
    return torch.sort(stable_topk(token_scores, keep_count)).values


def compact_per_head(cache_rows: torch.Tensor, keep: torch.Tensor) -> torch.Tensor:
    """G:fastdllm_engine.py:607-638 on dense rows: out[j, h] = rows[keep[h, j], h]. rows [S, Hkv, D], keep [Hkv, n]."""
    hkv = cache_rows.shape[1]
    return torch.stack([cache_rows[keep[h], h] for h in range(hkv)], dim=1)
