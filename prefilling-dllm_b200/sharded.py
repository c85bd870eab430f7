"""Chunk-sharded prefill across the GPUs of one box: one process per GPU, `torch.distributed` for the two exchanges.

The independent-chunk cache modes (`chunk_query` / `chunk_only`, reference prefilling_dllm_eval/fastdllm_parallelcomp.py:2201-2328)
make every chunk's work depend only on `[prefix ‖ chunk ‖ query ‖ draft]`, so chunks shard:

  1. every rank drafts the score target itself (same weights, same inputs: no exchange);
  2. rank r scores the chunks it owns — `[r·N/W, (r+1)·N/W)` with the remainder on the first ranks;
  3. ONE all-gather of the fp32 scores; every rank then ranks all N scores with the same stable rule and holds the
     same selection (no second collective);
  4. the selected chunks are dealt round-robin over the ranks, starting at the decode rank (a chunk's prefill needs only its
     token ids and the selection, not its scoring pass, and selected chunks cluster where the relevant text is: no rank
     prefills more than ceil(K / W) of them); each rank evicts and prefills its share locally;
  5. those ranks send the kept KV rows of all layers (one contiguous `[kept, layers, 2, Hkv, D]` payload per chunk — ONE gather
     launch over the pool seen as `2 * layers * pages` pages — plus the kept RoPE positions) to the decode rank with grouped
     point-to-point operations. The decode rank receives every payload straight into its slice of one buffer and writes
     all layers of all chunks into its own page pool with ONE page-write launch (a slot mapping over every layer), in
     selected-index order behind its prefix KV; then it prefills the query and denoises.

Decode itself is data-parallel over requests (different requests use different decode ranks); there is no tensor
parallelism. The planning and exchange helpers work on CPU tensors over `gloo` as well, which is how the host logic is
tested without GPUs; everything that computes goes through the CUDA runtime and has no CPU path.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class ChunkShardPlan:
    """Which rank owns which candidate chunk: contiguous blocks, the first `N mod W` ranks hold one more."""

    num_chunks: int
    world_size: int

    def bounds(self, rank: int) -> Tuple[int, int]:
        base, extra = divmod(self.num_chunks, self.world_size)
        start = rank * base + min(rank, extra)
        return start, start + base + (1 if rank < extra else 0)

    def chunks_of(self, rank: int) -> List[int]:
        lo, hi = self.bounds(rank)
        return list(range(lo, hi))

    def owner(self, chunk_index: int) -> int:
        if not 0 <= chunk_index < self.num_chunks:
            raise IndexError(chunk_index)
        for rank in range(self.world_size):
            lo, hi = self.bounds(rank)
            if lo <= chunk_index < hi:
                return rank
        raise AssertionError("unreachable")

    @property
    def max_per_rank(self) -> int:
        return math.ceil(self.num_chunks / self.world_size) if self.world_size else 0


def all_gather_chunk_scores(local_scores: torch.Tensor, plan: ChunkShardPlan, rank: int, group=None) -> torch.Tensor:
    """fp32 scores of the chunks this rank owns → fp32 scores of all N chunks, identical on every rank.

    Ranks may own different numbers of chunks, so each contribution is padded to `plan.max_per_rank` with -inf for the
    fixed-size all-gather and trimmed again by the plan."""
    lo, hi = plan.bounds(rank)
    if local_scores.numel() != hi - lo:
        raise ValueError(f"rank {rank} owns {hi - lo} chunks but has {local_scores.numel()} scores")
    width = plan.max_per_rank
    padded = torch.full((width,), float("-inf"), dtype=torch.float32, device=local_scores.device)
    padded[: hi - lo] = local_scores.to(torch.float32)
    gathered = torch.empty((plan.world_size * width,), dtype=torch.float32, device=local_scores.device)
    dist.all_gather_into_tensor(gathered, padded, group=group)
    rows = gathered.view(plan.world_size, width)
    return torch.cat([rows[r, : plan.bounds(r)[1] - plan.bounds(r)[0]] for r in range(plan.world_size)])


def rank_chunks(scores: Sequence[float], topk_chunks: int, keep_first_chunk: bool = False) -> List[int]:
    """The reference's ranking (fastdllm_parallelcomp.py:1949-1953): stable descending sort, so equal scores keep the
    lower index first; top-K; optional forced chunk 0; ascending indices. Host code on N <= a few dozen floats, run
    identically by every rank on the all-gathered scores."""
    n = len(scores)
    clean = [s if math.isfinite(s) else float("-inf") for s in scores]
    forced = [0] if keep_first_chunk and n > 0 else []
    ranked = sorted((i for i in range(n) if i not in forced), key=lambda i: clean[i], reverse=True)
    topk = len(ranked) if topk_chunks <= 0 else min(int(topk_chunks), len(ranked))
    return sorted(set(forced + ranked[:topk]))


@dataclass(frozen=True)
class KVTransfer:
    chunk_index: int
    order: int          # rank of the chunk among the selected ones (its place in the decode cache)
    src_rank: int
    kept_tokens: int


def prefill_ranks(selected: Sequence[int], world_size: int, decode_rank: int = 0) -> Dict[int, int]:
    """Which rank prefills which SELECTED chunk. Scoring is sharded by contiguous ownership (`ChunkShardPlan`), but the
    selected chunks cluster wherever the relevant text is, and a chunk's prefill needs nothing of its scoring pass — every rank
    holds the token ids and, after the all-gather, the selection. So the selected chunks are dealt round-robin, starting
    at the decode rank (whose share then needs no transfer): no rank prefills more than ceil(K / W) chunks."""
    return {ci: (decode_rank + order) % world_size for order, ci in enumerate(selected)}


def plan_kv_transfers(selected: Sequence[int], kept_tokens: Dict[int, int], plan: ChunkShardPlan,
                      src_ranks: Optional[Dict[int, int]] = None) -> List[KVTransfer]:
    """One transfer per selected chunk, in selected-index order (the order of the decode cache). `src_ranks[ci]`: the rank that
    holds chunk ci's prefilled KV (default: the chunk's scoring owner)."""
    return [KVTransfer(chunk_index=ci, order=order, src_rank=plan.owner(ci) if src_ranks is None else int(src_ranks[ci]),
                       kept_tokens=int(kept_tokens[ci]))
            for order, ci in enumerate(selected)]


def exchange_chunk_kv(transfers: Sequence[KVTransfer], *, rank: int, decode_rank: int, payloads: Dict[int, torch.Tensor],
                      positions: Dict[int, torch.Tensor], payload_shape: Callable[[int], Tuple[int, ...]], dtype: torch.dtype,
                      device, group=None, recv_into: Optional[Dict[int, torch.Tensor]] = None
                      ) -> Tuple[Dict[int, torch.Tensor], Dict[int, torch.Tensor]]:
    """Move every selected chunk's kept KV and kept RoPE positions from its owner to `decode_rank`.

    payloads[ci]: contiguous KV of chunk ci on its owner, shape `payload_shape(kept)`; positions[ci]: int64 [kept].
    All sends and receives of one request are posted as ONE grouped batch (NCCL: a single ncclGroup of send/recv pairs
    over NVLink). Returns, on the decode rank, (payload by chunk, positions by chunk) for every selected chunk — its own
    chunks are passed through without a copy — and empty dicts elsewhere. `recv_into[ci]` (decode rank, optional): a contiguous
    tensor of the payload's shape that chunk ci is received into (a slice of the caller's buffer) instead of a fresh one; the
    decode rank's own chunks are copied into theirs."""
    ops: List[dist.P2POp] = []
    got_kv: Dict[int, torch.Tensor] = {}
    got_pos: Dict[int, torch.Tensor] = {}
    for t in transfers:
        if t.src_rank == decode_rank:
            if rank == decode_rank:
                kv = payloads[t.chunk_index]
                if recv_into is not None and t.chunk_index in recv_into:
                    recv_into[t.chunk_index].copy_(kv)
                    kv = recv_into[t.chunk_index]
                got_kv[t.chunk_index], got_pos[t.chunk_index] = kv, positions[t.chunk_index]
            continue
        if rank == t.src_rank:
            kv, pos = payloads[t.chunk_index].contiguous(), positions[t.chunk_index].to(torch.int64).contiguous()
            if tuple(kv.shape) != tuple(payload_shape(t.kept_tokens)) or pos.numel() != t.kept_tokens:
                raise ValueError(f"chunk {t.chunk_index}: payload {tuple(kv.shape)} / {pos.numel()} positions do not match the plan")
            ops.append(dist.P2POp(dist.isend, kv, decode_rank, group=group))
            ops.append(dist.P2POp(dist.isend, pos, decode_rank, group=group))
        elif rank == decode_rank:
            kv = recv_into[t.chunk_index] if recv_into is not None and t.chunk_index in recv_into else torch.empty(payload_shape(t.kept_tokens), dtype=dtype, device=device)
            if tuple(kv.shape) != tuple(payload_shape(t.kept_tokens)) or not kv.is_contiguous():
                raise ValueError(f"chunk {t.chunk_index}: receive buffer {tuple(kv.shape)} does not match the plan")
            pos = torch.empty((t.kept_tokens,), dtype=torch.int64, device=device)
            got_kv[t.chunk_index], got_pos[t.chunk_index] = kv, pos
            ops.append(dist.P2POp(dist.irecv, kv, t.src_rank, group=group))
            ops.append(dist.P2POp(dist.irecv, pos, t.src_rank, group=group))
    if ops:
        for work in dist.batch_isend_irecv(ops):
            work.wait()
    return got_kv, got_pos


class ShardedChunkPrefill:
    """Runs one request's chunk scoring and chunk prefill sharded over the ranks of `group`, then decodes on one rank.

    `runtime`: this rank's `FastDLLMParallelComp` (same checkpoint and flags on every rank, one GPU each) in an
    independent-chunk cache mode."""

    def __init__(self, runtime, group=None):
        if runtime.config.cache_build_mode not in {"chunk_query", "chunk_only"}:
            raise ValueError("sharding needs an independent-chunk cache mode (chunk_query / chunk_only): in the full-prompt modes "
                             "the selected chunks attend each other in the joint prefill")
        self.rt = runtime
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def _payload_shape(self, kept: int) -> Tuple[int, ...]:
        a = self.rt.arch
        return (int(kept), a.num_hidden_layers, 2, a.num_key_value_heads, a.head_dim)

    def _gather_rows(self, cache, start: int, n: int) -> torch.Tensor:
        """[n, layers, 2 (K, V), Hkv, D] copy of cache tokens [start, start + n) of every layer: one gather launch over the
        pages that hold them in all (K|V, layer) planes, one strided copy into the payload layout."""
        from . import ops

        m = self.rt.model
        if n <= 0:
            return torch.empty(self._payload_shape(0), dtype=m.dtype, device=m.device)
        page, layers, pages = m.page_size, m.arch.num_hidden_layers, m.num_pages
        p0, p1 = start // page, (start + n - 1) // page
        base = torch.tensor(cache.page_ids[p0:p1 + 1], dtype=torch.int32, device=m.device)
        planes = torch.arange(2 * layers, dtype=torch.int32, device=m.device) * pages
        ids = (planes.view(-1, 1) + base.view(1, -1)).reshape(-1).contiguous()
        kv = m.kv_cache
        pool = kv.view(2 * layers * pages, kv.shape[3], kv.shape[4], kv.shape[5])
        dense = ops.gather_pages(pool, ids, int(ids.numel()) * page).view(2, layers, (p1 - p0 + 1) * page, kv.shape[4], kv.shape[5])
        off = start - p0 * page
        return dense[:, :, off:off + n].permute(2, 1, 0, 3, 4).contiguous()

    @torch.inference_mode()
    def generate(self, *, prefix_ids, context_ids, query_ids, scoring_query_ids=None, decode_rank: int = 0):
        """Returns the FastDLLMParallelCompResult on `decode_rank`, None on the other ranks."""
        from . import ops
        from .parallelcomp import FastDLLMChunkMeta, PagedCache, split_token_chunks

        rt, cfg = self.rt, self.rt.config
        prefix_ids, context_ids, query_ids = list(prefix_ids), list(context_ids), list(query_ids)
        scoring_query_ids = list(scoring_query_ids if scoring_query_ids is not None else query_ids)
        chunks = [rt._maybe_prepend_bos_to_chunk(c) for c in split_token_chunks(context_ids, cfg.chunk_size, split_from_tail=cfg.split_from_tail)]
        plan = ChunkShardPlan(len(chunks), self.world)
        # 1-2: draft (redundant on every rank), local scores
        selection_q, count, mask = rt._selection_query_ids_with_score_target(prefix_ids, scoring_query_ids)
        mine = plan.chunks_of(self.rank)
        local = rt.score_chunks_self_information_batched(prefix_ids, [chunks[i] for i in mine], selection_q, score_token_count=count,
                                                         score_token_mask=mask) if mine else {}
        local_t = torch.tensor([local[j] for j in range(len(mine))], dtype=torch.float32, device=rt.device)
        # 3: the one collective of the data path
        all_scores = all_gather_chunk_scores(local_t, plan, self.rank, self.group).tolist()
        selected = rank_chunks(all_scores, int(cfg.topk_chunks), bool(cfg.keep_first_chunk))
        scores = {i: (s if math.isfinite(s) else float("-inf")) for i, s in enumerate(all_scores)}
        # 4: the selected chunks, dealt evenly over the ranks, are evicted + prefilled into a scratch cache [prefix ‖ chunk rows]
        prefill_on = prefill_ranks(selected, self.world, decode_rank)
        evict_q = rt._token_eviction_query_ids(scoring_query_ids, selection_q, mask)
        window_q = rt._window_query(selection_q, cfg.token_score_query_window)
        p_len = len(prefix_ids)
        capacity = int(cfg.token_capacity or 0)
        kept_tokens = {ci: (min(capacity, len(chunks[ci])) if capacity > 0 else len(chunks[ci])) for ci in selected}
        payloads: Dict[int, torch.Tensor] = {}
        positions: Dict[int, torch.Tensor] = {}
        unions: Dict[int, List[int]] = {}
        mine_items = [(order, ci, list(chunks[ci])) for order, ci in enumerate(selected) if prefill_on[ci] == self.rank]
        done_packed = False
        if len(mine_items) >= 2:
            # this rank's share in packed forwards (one pass over the weights for all of it), into one scratch cache
            scratch = PagedCache(rt, p_len + sum(2 * len(c) for _, _, c in mine_items) + rt.model.page_size)
            try:
                if prefix_ids:
                    rt._forward_packed([prefix_ids], [rt._range_positions(0, p_len)], causal=False, store_slots=scratch.slots(0, p_len),
                                       want_logits=False)
                    scratch.length = p_len
                packed = rt._prefill_chunks_packed(scratch, p_len, prefix_ids, mine_items, evict_q, window_q)
                if packed is not None:
                    at = p_len
                    for (order, ci, chunk), (kept, kept_pos, union, _) in zip(mine_items, packed):
                        if kept != kept_tokens[ci]:
                            raise RuntimeError(f"chunk {ci}: kept {kept} tokens, the plan expected {kept_tokens[ci]}")
                        payloads[ci] = self._gather_rows(scratch, at, kept)
                        positions[ci] = torch.tensor(kept_pos, dtype=torch.int64, device=rt.device)
                        unions[ci] = list(union)
                        at += kept
                    done_packed = True
            finally:
                scratch.release()
        for order, ci in enumerate(selected):
            if prefill_on[ci] != self.rank or done_packed:
                continue
            chunk = list(chunks[ci])
            scratch = PagedCache(rt, p_len + 2 * len(chunk) + rt.model.page_size)
            try:
                if prefix_ids:
                    rt._forward_packed([prefix_ids], [rt._range_positions(0, p_len)], causal=False, store_slots=scratch.slots(0, p_len),
                                       want_logits=False)
                    scratch.length = p_len
                kept, kept_pos, union, _ = rt._prefill_one_chunk(scratch, p_len, prefix_ids, chunk, order, ci, evict_q, window_q)
                if kept != kept_tokens[ci]:
                    raise RuntimeError(f"chunk {ci}: kept {kept} tokens, the plan expected {kept_tokens[ci]}")
                payloads[ci] = self._gather_rows(scratch, p_len, kept)
                positions[ci] = torch.tensor(kept_pos, dtype=torch.int64, device=rt.device)
                unions[ci] = list(union)
            finally:
                scratch.release()
        # 5: hand-off to the decode rank
        transfers = plan_kv_transfers(selected, kept_tokens, plan, prefill_on)
        recv_into = None
        if self.rank == decode_rank and selected:
            # every chunk's payload lands in its slice of one [sum kept, layers, 2, Hkv, D] buffer, in selected order
            landing = torch.empty(self._payload_shape(sum(kept_tokens[ci] for ci in selected)), dtype=rt.model.dtype, device=rt.device)
            recv_into, off = {}, 0
            for ci in selected:
                recv_into[ci] = landing[off:off + kept_tokens[ci]]
                off += kept_tokens[ci]
        got_kv, got_pos = exchange_chunk_kv(transfers, rank=self.rank, decode_rank=decode_rank, payloads=payloads, positions=positions,
                                            payload_shape=self._payload_shape, dtype=rt.model.dtype, device=rt.device, group=self.group,
                                            recv_into=recv_into)
        ops.check_status(rt.device)
        if self.rank != decode_rank:
            return None
        total = p_len + sum(kept_tokens.values())
        cache = PagedCache(rt, total + len(query_ids) + rt.max_new_tokens + 2 * rt.model.page_size)
        try:
            cache_positions: List[int] = []
            if prefix_ids:
                rt._forward_packed([prefix_ids], [rt._range_positions(0, p_len)], causal=False, store_slots=cache.slots(0, p_len), want_logits=False)
                cache.length = p_len
                cache_positions.extend(rt._range_positions(0, p_len))
            meta = []
            if selected:
                # ONE page write for every layer of every chunk: rows (token, layer) of the landing buffer, K and V side by
                # side, go to the slots of that token in that layer's planes of the pool
                a = rt.arch
                rows = landing.view(landing.shape[0] * a.num_hidden_layers, 2, a.num_key_value_heads, a.head_dim)
                k_pool, v_pool = rt.model.plane_pools()
                cache.slots(p_len, landing.shape[0])                                   # capacity check
                ops.store_kvcache_unified_layout(rows[:, 0], rows[:, 1], k_pool, v_pool,
                                                 rt.model.all_layer_slots(cache.page_ids, p_len, landing.shape[0]), "diffusion_lm")
            for order, ci in enumerate(selected):
                kept, dst = kept_tokens[ci], cache.length
                c_start = rt._chunk_rope_start(p_len, order, ci)
                cache.length = dst + kept
                cache_positions.extend(got_pos[ci].tolist())
                meta.append(FastDLLMChunkMeta(chunk_index=ci, original_tokens=len(chunks[ci]), kept_tokens=kept,
                                              removed_tokens=len(chunks[ci]) - kept, cache_start=dst, cache_end=dst + kept, rope_start=c_start,
                                              rope_end=c_start + len(chunks[ci]), score=scores.get(ci),
                                              kept_positions=unions.get(ci) or [p - c_start for p in got_pos[ci].tolist()]))
            q_start = rt._final_query_rope_start(p_len, cache_positions, selected_count=len(selected))
            generated = rt.generate_from_cache(past_key_values=cache, cache_positions=cache_positions, query_ids=query_ids,
                                               query_rope_start=q_start)
        finally:
            cache.release()
        removed = sum(len(chunks[ci]) - kept_tokens[ci] for ci in selected)
        return rt._result(generated, selected, scores, cfg.cache_build_mode, p_len, len(query_ids), len(context_ids), len(chunks), total,
                          removed, meta)
